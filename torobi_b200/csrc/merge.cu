// Merging a LoRA pair into its quantized base for export:
//   out[r, c] = deq(r, c) + scale * sum_i b[r, i] * a[i, c]
// deq is the stored weight as the GEMM sees it (RNE_bf16(scale_g * q +
// bias_g), the exact dequantization); the low-rank sum is taken in f32 in
// increasing i with every product and sum rounded on its own (no fused
// multiply-add), then scaled and added, so the CPU oracle reproduces it bit
// for bit.  Without a pair it is the dequantization in f32.
//
// The reference refuses to export an adapted model until this exists
// (lib/torobi/export.rb:118-140: "W + scale * BA, and the adapter dropped");
// the export writes fp32 (engine/src/export.rs:1-9).
//
// HBM-bound: reads bits/8 + 4/g bytes per weight, writes 4 (f32) or 2 (bf16).
// One thread = 8 consecutive columns of kRows consecutive rows, so each
// 8-column slice of A is loaded once for kRows rows.
#include <cuda_bf16.h>

#include "tq_ptx.cuh"
#include "tq_runtime.h"

namespace tq {
namespace {

constexpr int kRows = 4;

template <int BITS, bool F32_OUT>
__global__ void __launch_bounds__(256) merge_kernel(const uint32_t* __restrict__ codes,
                                                    const uint16_t* __restrict__ scales,
                                                    const uint16_t* __restrict__ biases,
                                                    int rows, int cols, int group_shift,
                                                    const float* __restrict__ a,
                                                    const float* __restrict__ b, int rank,
                                                    float scale, void* __restrict__ out) {
  const int c8 = cols / 8;
  const int row_blocks = (rows + kRows - 1) / kRows;
  const int64_t items = static_cast<int64_t>(row_blocks) * c8;
  const int gpr = cols >> group_shift;
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  for (int64_t it = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; it < items;
       it += stride) {
    const int cb = static_cast<int>(it % c8);
    const int r0 = static_cast<int>(it / c8) * kRows;
    const int c0 = cb * 8;
    float acc[kRows][8];
#pragma unroll
    for (int rr = 0; rr < kRows; ++rr)
#pragma unroll
      for (int j = 0; j < 8; ++j) acc[rr][j] = 0.0f;
    for (int i = 0; i < rank; ++i) {
      const float4* ap = reinterpret_cast<const float4*>(a + static_cast<size_t>(i) * cols + c0);
      const float4 lo = __ldg(ap), hi = __ldg(ap + 1);
      const float av[8] = {lo.x, lo.y, lo.z, lo.w, hi.x, hi.y, hi.z, hi.w};
#pragma unroll
      for (int rr = 0; rr < kRows; ++rr) {
        const int r = r0 + rr < rows ? r0 + rr : rows - 1;
        const float bv = __ldg(b + static_cast<size_t>(r) * rank + i);
#pragma unroll
        for (int j = 0; j < 8; ++j) acc[rr][j] = __fadd_rn(acc[rr][j], __fmul_rn(bv, av[j]));
      }
    }
#pragma unroll
    for (int rr = 0; rr < kRows; ++rr) {
      const int r = r0 + rr;
      if (r >= rows) break;
      const size_t g = static_cast<size_t>(r) * gpr + (c0 >> group_shift);
      const uint32_t s2 = bf16_dup(__ldg(reinterpret_cast<const unsigned short*>(scales) + g));
      const uint32_t b2 = bf16_dup(__ldg(reinterpret_cast<const unsigned short*>(biases) + g));
      uint32_t d[4];
      if constexpr (BITS == 4) {
        dequant_u4x8(__ldg(codes + static_cast<size_t>(r) * (cols / 8) + cb), s2, b2, d);
      } else {
        const uint2 w = __ldg(reinterpret_cast<const uint2*>(codes) +
                              static_cast<size_t>(r) * (cols / 8) + cb);
        uint32_t lo[2], hi[2];
        dequant_u8x4(w.x, s2, b2, lo);
        dequant_u8x4(w.y, s2, b2, hi);
        d[0] = lo[0];
        d[1] = lo[1];
        d[2] = hi[0];
        d[3] = hi[1];
      }
      float v[8];
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        v[2 * k] = __fadd_rn(__uint_as_float(d[k] << 16), __fmul_rn(scale, acc[rr][2 * k]));
        v[2 * k + 1] =
            __fadd_rn(__uint_as_float(d[k] & 0xFFFF0000u), __fmul_rn(scale, acc[rr][2 * k + 1]));
      }
      const size_t o = static_cast<size_t>(r) * cols + c0;
      if constexpr (F32_OUT) {
        float4* op = reinterpret_cast<float4*>(static_cast<float*>(out) + o);
        op[0] = make_float4(v[0], v[1], v[2], v[3]);
        op[1] = make_float4(v[4], v[5], v[6], v[7]);
      } else {
        *reinterpret_cast<uint4*>(static_cast<uint16_t*>(out) + o) =
            make_uint4(pack_bf16x2_f32(v[0], v[1]), pack_bf16x2_f32(v[2], v[3]),
                       pack_bf16x2_f32(v[4], v[5]), pack_bf16x2_f32(v[6], v[7]));
      }
    }
  }
}

template <int BITS>
void launch_merge(bool f32_out, int grid, cudaStream_t s, const uint32_t* c, const uint16_t* sc,
                  const uint16_t* bi, int rows, int cols, int shift, const float* a,
                  const float* b, int rank, float scale, void* out) {
  if (f32_out)
    merge_kernel<BITS, true><<<grid, 256, 0, s>>>(c, sc, bi, rows, cols, shift, a, b, rank, scale,
                                                  out);
  else
    merge_kernel<BITS, false><<<grid, 256, 0, s>>>(c, sc, bi, rows, cols, shift, a, b, rank,
                                                   scale, out);
}

}  // namespace
}  // namespace tq

extern "C" int tq_lora_merge(const void* codes, const void* scales, const void* biases,
                             int64_t rows, int64_t cols, int group_size, int bits,
                             const float* lora_a, const float* lora_b, int64_t rank, float scale,
                             void* out, int out_dtype, void* stream) {
  using namespace tq;
  if (bits != 4 && bits != 8) return fail(TQ_ERR_UNSUPPORTED, "lora_merge: bits must be 4 or 8");
  if (group_size != 32 && group_size != 64 && group_size != 128)
    return fail(TQ_ERR_UNSUPPORTED, "lora_merge: group_size must be 32, 64 or 128");
  if (rows < 0 || cols < 0 || cols % group_size != 0)
    return fail(TQ_ERR_INVALID, "lora_merge: bad shape [%lld, %lld] for group %d",
                (long long)rows, (long long)cols, group_size);
  if (rows > (1ll << 31) - 1 || cols > (1ll << 31) - 1)
    return fail(TQ_ERR_INVALID, "lora_merge: dimensions must fit in 31 bits");
  if (rank < 0 || rank > 256 || ((rank > 0) != (lora_a != nullptr && lora_b != nullptr)))
    return fail(TQ_ERR_INVALID, "lora_merge: rank %lld needs both factors (or rank 0 and none)",
                (long long)rank);
  if (out_dtype != TQ_DTYPE_F32 && out_dtype != TQ_DTYPE_BF16)
    return fail(TQ_ERR_UNSUPPORTED, "lora_merge: out_dtype must be TQ_DTYPE_F32 or TQ_DTYPE_BF16");
  if (rows == 0 || cols == 0) return TQ_OK;
  if (!codes || !scales || !biases || !out) return fail(TQ_ERR_INVALID, "lora_merge: null pointer");
  if (!aligned(codes, 8) || !aligned(out, 16) || (rank && (!aligned(lora_a, 16) || !aligned(lora_b, 4))))
    return fail(TQ_ERR_MISALIGNED, "lora_merge: codes 8-, out and lora_a 16-, lora_b 4-byte aligned");
  const int shift = group_size == 32 ? 5 : (group_size == 64 ? 6 : 7);
  const int64_t items = ((rows + kRows - 1) / kRows) * (cols / 8);
  int64_t want = (items + 255) / 256;
  const int64_t cap = static_cast<int64_t>(sm_count()) * 8;
  const int grid = static_cast<int>(want < 1 ? 1 : (want > cap ? cap : want));
  cudaStream_t s = as_stream(stream);
  const bool f32_out = out_dtype == TQ_DTYPE_F32;
  const int r = static_cast<int>(rows), c = static_cast<int>(cols), k = static_cast<int>(rank);
  const uint32_t* cp = static_cast<const uint32_t*>(codes);
  const uint16_t* sp = static_cast<const uint16_t*>(scales);
  const uint16_t* bp = static_cast<const uint16_t*>(biases);
  if (bits == 4)
    launch_merge<4>(f32_out, grid, s, cp, sp, bp, r, c, shift, lora_a, lora_b, k, scale, out);
  else
    launch_merge<8>(f32_out, grid, s, cp, sp, bp, r, c, shift, lora_a, lora_b, k, scale, out);
  return check_cuda(cudaGetLastError(), "lora_merge launch");
}
