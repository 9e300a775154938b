// Status strings and build identification for the C ABI.
#include "common.cuh"

extern "C" const char* moe_status_string(int status) {
  switch (status) {
    case MOE_OK: return "ok";
    case MOE_ERR_INVALID_ARG: return "invalid argument";
    case MOE_ERR_UNSUPPORTED: return "unsupported shape or configuration";
    case MOE_ERR_CUDA: return "CUDA launch or runtime error";
    case MOE_ERR_WORKSPACE: return "workspace missing or too small";
    case MOE_ERR_ALIGNMENT: return "pointer not 16-byte aligned";
    case MOE_ERR_TIMEOUT: return "device wait timed out";
    default: return "unknown status";
  }
}

extern "C" const char* moe_version(void) { return "moe_b200 sm_100a 0.1"; }
