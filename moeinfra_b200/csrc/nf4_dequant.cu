// NF4 blockwise dequant (bit-exact bf16) and nested-absmax rebuild.
//
// Reference semantics: bitsandbytes 0.50.2 dequantize_4bit as reached from
// transfer/nf4_reconstruct.py:45-54 (blocksize 64 at :9, dtype bf16 at :12)
// and the nested QuantState of :17-38 (blocksize 256 at :13).
//
// HBM-bound: per 16 packed bytes (32 elements) a thread reads 16 B + 4 B of
// absmax and writes 64 B of bf16.  Grid-stride over 16-byte chunks with
// 128-bit loads/stores; the 16-entry codebook sits in shared memory.
#include "common.cuh"

namespace moe {
namespace {

__global__ void __launch_bounds__(256) k_nf4_dequant_vec(const uint4* __restrict__ q,
                                                         const float* __restrict__ absmax,
                                                         const float* __restrict__ code,
                                                         int64_t nchunks, int block_shift,
                                                         uint4* __restrict__ out) {
  __shared__ float s_code[16];
  if (threadIdx.x < 16) s_code[threadIdx.x] = code[threadIdx.x];
  __syncthreads();
  for (int64_t c = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; c < nchunks;
       c += (int64_t)gridDim.x * blockDim.x) {
    uint4 v = q[c];
    // 32 elements per chunk; blocksize >= 32 so the chunk lies in one block.
    float a = absmax[(c * 32) >> block_shift];
    uint32_t w[4] = {v.x, v.y, v.z, v.w};
    uint32_t o[16];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
#pragma unroll
      for (int b = 0; b < 4; ++b) {
        uint32_t byte = (w[i] >> (8 * b)) & 0xFFu;
        float p0 = __fmul_rn(s_code[byte >> 4], a);
        float p1 = __fmul_rn(s_code[byte & 15u], a);
        __nv_bfloat162 r = __floats2bfloat162_rn(p0, p1);
        o[i * 4 + b] = *reinterpret_cast<uint32_t*>(&r);
      }
    }
    uint4* dst = out + c * 4;
    dst[0] = make_uint4(o[0], o[1], o[2], o[3]);
    dst[1] = make_uint4(o[4], o[5], o[6], o[7]);
    dst[2] = make_uint4(o[8], o[9], o[10], o[11]);
    dst[3] = make_uint4(o[12], o[13], o[14], o[15]);
  }
}

// Scalar path: unaligned pointers or a tail shorter than one chunk.
__global__ void k_nf4_dequant_scalar(const uint8_t* __restrict__ q, const float* __restrict__ absmax,
                                     const float* __restrict__ code, int64_t begin, int64_t numel,
                                     int block_shift, uint16_t* __restrict__ out) {
  for (int64_t i = begin + blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < numel;
       i += (int64_t)gridDim.x * blockDim.x) {
    uint32_t byte = q[i >> 1];
    uint32_t nib = (i & 1) ? (byte & 15u) : (byte >> 4);
    float p = __fmul_rn(code[nib], absmax[i >> block_shift]);
    out[i] = __bfloat16_as_ushort(__float2bfloat16_rn(p));
  }
}

__global__ void k_nested_absmax(const uint8_t* __restrict__ qabs, const float* __restrict__ absmax2,
                                const float* __restrict__ code2, float offset, int64_t n, int bs2,
                                float* __restrict__ out) {
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x) {
    out[i] = __fadd_rn(__fmul_rn(code2[qabs[i]], absmax2[i / bs2]), offset);
  }
}

int log2_exact(int v) {
  if (v <= 0 || (v & (v - 1))) return -1;
  int s = 0;
  while ((1 << s) < v) ++s;
  return s;
}

}  // namespace
}  // namespace moe

extern "C" int moe_nf4_dequant(const uint8_t* q, const float* absmax, const float* code,
                               int64_t numel, int blocksize, uint16_t* out_bf16, void* stream) {
  using namespace moe;
  if (numel < 0 || (numel & 1)) return MOE_ERR_INVALID_ARG;
  if (numel == 0) return MOE_OK;
  if (!q || !absmax || !code || !out_bf16) return MOE_ERR_INVALID_ARG;
  int shift = log2_exact(blocksize);
  if (shift < 5) return MOE_ERR_INVALID_ARG;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  int64_t begin = 0;
  if (aligned16(q) && aligned16(out_bf16)) {
    int64_t nchunks = numel / 32;
    if (nchunks > 0) {
      int64_t blocks = ceil_div(nchunks, 256);
      int grid = static_cast<int>(blocks < sm_count() * 8 ? blocks : sm_count() * 8);
      k_nf4_dequant_vec<<<grid, 256, 0, s>>>(reinterpret_cast<const uint4*>(q), absmax, code,
                                             nchunks, shift, reinterpret_cast<uint4*>(out_bf16));
      MOE_CHECK_LAUNCH();
    }
    begin = nchunks * 32;
  }
  if (begin < numel) {
    int64_t rem = numel - begin;
    int64_t blocks = ceil_div(rem, 256);
    int grid = static_cast<int>(blocks < sm_count() * 8 ? blocks : sm_count() * 8);
    k_nf4_dequant_scalar<<<grid, 256, 0, s>>>(q, absmax, code, begin, numel, shift, out_bf16);
    MOE_CHECK_LAUNCH();
  }
  return MOE_OK;
}

extern "C" int moe_nf4_nested_absmax(const uint8_t* qabs, const float* absmax2, const float* code2,
                                     float offset, int64_t nblocks, int blocksize2,
                                     float* out_absmax, void* stream) {
  using namespace moe;
  if (nblocks < 0 || blocksize2 <= 0) return MOE_ERR_INVALID_ARG;
  if (nblocks == 0) return MOE_OK;
  if (!qabs || !absmax2 || !code2 || !out_absmax) return MOE_ERR_INVALID_ARG;
  int64_t blocks = ceil_div(nblocks, 256);
  int grid = static_cast<int>(blocks < sm_count() * 8 ? blocks : sm_count() * 8);
  k_nested_absmax<<<grid, 256, 0, static_cast<cudaStream_t>(stream)>>>(
      qabs, absmax2, code2, offset, nblocks, blocksize2, out_absmax);
  MOE_CHECK_LAUNCH();
  return MOE_OK;
}
