// Device layout of resident NF4 matrices ("tile16") and its bit-exact dequant.
//
// The reference store keeps each projection row-major over [rows, cols]
// (packed codes, 2 per byte, element 2j in the high nibble of byte j; one fp32
// absmax per 64 consecutive elements of a row).  Once a matrix is resident,
// the kernels read it in tiles of 16 rows x one 64-element block: the 16 rows'
// 32-byte block segments are stored together, so a warp's MMA-fragment load
// (rows g and g+8, bytes 8t..8t+7) is 256 contiguous bytes.
//
//   packed: byte offset ((rb * (cols/64) + kb) * 16 + r) * 32 + j
//           holds store bytes of row 16*rb + r, block kb, byte j (0..31)
//   absmax: index (rb * (cols/64) + kb) * 16 + r
//
// rows % 16 == 0 and cols % 64 == 0.  The permutation is exact (bytes and fp32
// words are moved, never recomputed).
#include "common.cuh"

namespace moe {
namespace {

// One thread moves one 32-byte block segment (2 x 16 B) and its absmax word.
__global__ void k_tile16(const uint4* __restrict__ q, const float* __restrict__ absmax, int64_t rows,
                         int64_t nblk, uint4* __restrict__ q_out, float* __restrict__ absmax_out) {
  const int64_t total = rows * nblk;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total;
       i += (int64_t)gridDim.x * blockDim.x) {
    // i enumerates the destination: ((rb * nblk + kb) * 16 + r)
    const int64_t r = i & 15, tile = i >> 4;
    const int64_t rb = tile / nblk, kb = tile - rb * nblk;
    const int64_t src_row = rb * 16 + r;
    const int64_t src = src_row * nblk + kb;  // block index in store order
    q_out[2 * i] = q[2 * src];
    q_out[2 * i + 1] = q[2 * src + 1];
    absmax_out[i] = absmax[src];
  }
}

// bf16(code * absmax) for a tile16 matrix, written row-major [rows, cols].
__global__ void k_dequant_tile16(const uint4* __restrict__ q, const float* __restrict__ absmax,
                                 const float* __restrict__ code, int64_t rows, int64_t nblk,
                                 uint4* __restrict__ out) {
  __shared__ float s_code[16];
  if (threadIdx.x < 16) s_code[threadIdx.x] = code[threadIdx.x];
  __syncthreads();
  const int64_t total = rows * nblk * 2;  // 16-byte halves of block segments
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t seg = i >> 1, half = i & 1;
    const int64_t r = seg & 15, tile = seg >> 4;
    const int64_t rb = tile / nblk, kb = tile - rb * nblk;
    const float a = absmax[seg];
    const uint4 v = q[i];
    const uint32_t w[4] = {v.x, v.y, v.z, v.w};
    uint32_t o[16];
#pragma unroll
    for (int k = 0; k < 4; ++k) {
#pragma unroll
      for (int b = 0; b < 4; ++b) {
        const uint32_t byte = (w[k] >> (8 * b)) & 0xFFu;
        __nv_bfloat162 p = __floats2bfloat162_rn(__fmul_rn(s_code[byte >> 4], a),
                                                 __fmul_rn(s_code[byte & 15u], a));
        o[k * 4 + b] = *reinterpret_cast<uint32_t*>(&p);
      }
    }
    // 32 elements: row rb*16+r, columns kb*64 + half*32 .. +32
    uint4* dst = out + ((rb * 16 + r) * nblk * 64 + kb * 64 + half * 32) / 8;
    dst[0] = make_uint4(o[0], o[1], o[2], o[3]);
    dst[1] = make_uint4(o[4], o[5], o[6], o[7]);
    dst[2] = make_uint4(o[8], o[9], o[10], o[11]);
    dst[3] = make_uint4(o[12], o[13], o[14], o[15]);
  }
}

int grid_for(int64_t work) {
  const int64_t b = ceil_div(work, 256);
  const int64_t cap = (int64_t)sm_count() * 8;
  return static_cast<int>(b < 1 ? 1 : (b < cap ? b : cap));
}

}  // namespace
}  // namespace moe

extern "C" int moe_nf4_tile16(const uint8_t* q, const float* absmax, int64_t rows, int64_t cols,
                              uint8_t* q_out, float* absmax_out, void* stream) {
  using namespace moe;
  if (rows < 0 || cols < 0 || rows % 16 || cols % 64) return MOE_ERR_INVALID_ARG;
  if (rows == 0 || cols == 0) return MOE_OK;
  if (!q || !absmax || !q_out || !absmax_out) return MOE_ERR_INVALID_ARG;
  if (!aligned16(q) || !aligned16(q_out)) return MOE_ERR_ALIGNMENT;
  const int64_t nblk = cols / 64;
  k_tile16<<<grid_for(rows * nblk), 256, 0, static_cast<cudaStream_t>(stream)>>>(
      reinterpret_cast<const uint4*>(q), absmax, rows, nblk, reinterpret_cast<uint4*>(q_out),
      absmax_out);
  MOE_CHECK_LAUNCH();
  return MOE_OK;
}

extern "C" int moe_nf4_dequant_tile16(const uint8_t* q, const float* absmax, const float* code,
                                      int64_t rows, int64_t cols, uint16_t* out_bf16,
                                      void* stream) {
  using namespace moe;
  if (rows < 0 || cols < 0 || rows % 16 || cols % 64) return MOE_ERR_INVALID_ARG;
  if (rows == 0 || cols == 0) return MOE_OK;
  if (!q || !absmax || !code || !out_bf16) return MOE_ERR_INVALID_ARG;
  if (!aligned16(q) || !aligned16(out_bf16)) return MOE_ERR_ALIGNMENT;
  const int64_t nblk = cols / 64;
  k_dequant_tile16<<<grid_for(rows * nblk * 2), 256, 0, static_cast<cudaStream_t>(stream)>>>(
      reinterpret_cast<const uint4*>(q), absmax, code, rows, nblk, reinterpret_cast<uint4*>(out_bf16));
  MOE_CHECK_LAUNCH();
  return MOE_OK;
}
