// The update side of the step: the global gradient norm, a fused AdamW over
// the flattened LoRA parameters, and the bf16 copies of the adapter the
// GEMM kernels read.  All element-wise and HBM-bound; every element is touched
// once with 16-byte accesses where the layout allows.
#include <cuda_bf16.h>

#include "tq_ptx.cuh"
#include "tq_runtime.h"

namespace tq {
namespace {

__global__ void __launch_bounds__(256) sumsq_kernel(const float* __restrict__ x, int64_t n,
                                                    float* __restrict__ out) {
  griddep_wait();
  griddep_launch_dependents();
  float acc = 0.0f;
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  const int64_t n4 = n / 4;
  const float4* x4 = reinterpret_cast<const float4*>(x);
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n4; i += stride) {
    const float4 v = __ldg(x4 + i);
    acc += v.x * v.x + v.y * v.y + v.z * v.z + v.w * v.w;
  }
  for (int64_t i = n4 * 4 + static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n;
       i += stride) {
    const float v = __ldg(x + i);
    acc += v * v;
  }
  for (int off = 16; off > 0; off >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, off);
  __shared__ float warp_sums[8];
  if ((threadIdx.x & 31) == 0) warp_sums[threadIdx.x >> 5] = acc;
  __syncthreads();
  if (threadIdx.x < 32) {
    float v = threadIdx.x < (blockDim.x >> 5) ? warp_sums[threadIdx.x] : 0.0f;
    for (int off = 16; off > 0; off >>= 1) v += __shfl_xor_sync(0xffffffffu, v, off);
    if (threadIdx.x == 0) atomicAdd(out, v);
  }
}

struct AdamArgs {
  float lr, beta1, beta2, eps, wd, grad_scale, bias1, bias2, clip;
};

__device__ __forceinline__ float adam_one(float p, float g, float& m, float& v, const AdamArgs& a) {
  m = __fadd_rn(__fmul_rn(m, a.beta1), __fmul_rn(g, __fsub_rn(1.0f, a.beta1)));
  v = __fadd_rn(__fmul_rn(v, a.beta2), __fmul_rn(__fmul_rn(g, g), __fsub_rn(1.0f, a.beta2)));
  const float m_hat = __fdiv_rn(m, a.bias1);
  const float v_hat = __fdiv_rn(v, a.bias2);
  const float denom = __fadd_rn(__fsqrt_rn(v_hat), a.eps);
  float next = __fsub_rn(p, __fmul_rn(__fdiv_rn(m_hat, denom), a.lr));
  if (a.wd != 0.0f) next = __fsub_rn(next, __fmul_rn(p, __fmul_rn(a.lr, a.wd)));
  return next;
}

__global__ void __launch_bounds__(256) adamw_kernel(float* __restrict__ params,
                                                    const float* __restrict__ grads,
                                                    float* __restrict__ m, float* __restrict__ v,
                                                    int64_t n, AdamArgs a,
                                                    const float* __restrict__ norm_sq,
                                                    uint16_t* __restrict__ params_bf16) {
  griddep_wait();
  griddep_launch_dependents();
  float gscale = a.grad_scale;
  if (norm_sq) {
    const float ns = *norm_sq;
    if (!isfinite(ns)) return;  // skipped step: nothing moves
    if (a.clip > 0.0f) {
      const float norm = __fmul_rn(sqrtf(ns), fabsf(a.grad_scale));
      if (norm > a.clip) gscale = __fmul_rn(gscale, __fdiv_rn(a.clip, norm));
    }
  }
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  const int64_t n4 = n / 4;
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n4; i += stride) {
    float4 p4 = reinterpret_cast<float4*>(params)[i];
    const float4 g4 = __ldg(reinterpret_cast<const float4*>(grads) + i);
    float4 m4 = reinterpret_cast<float4*>(m)[i];
    float4 v4 = reinterpret_cast<float4*>(v)[i];
    p4.x = adam_one(p4.x, __fmul_rn(g4.x, gscale), m4.x, v4.x, a);
    p4.y = adam_one(p4.y, __fmul_rn(g4.y, gscale), m4.y, v4.y, a);
    p4.z = adam_one(p4.z, __fmul_rn(g4.z, gscale), m4.z, v4.z, a);
    p4.w = adam_one(p4.w, __fmul_rn(g4.w, gscale), m4.w, v4.w, a);
    reinterpret_cast<float4*>(params)[i] = p4;
    reinterpret_cast<float4*>(m)[i] = m4;
    reinterpret_cast<float4*>(v)[i] = v4;
    if (params_bf16) {
      const uint32_t lo = __bfloat16_as_ushort(__float2bfloat16_rn(p4.x)) |
                          (uint32_t(__bfloat16_as_ushort(__float2bfloat16_rn(p4.y))) << 16);
      const uint32_t hi = __bfloat16_as_ushort(__float2bfloat16_rn(p4.z)) |
                          (uint32_t(__bfloat16_as_ushort(__float2bfloat16_rn(p4.w))) << 16);
      reinterpret_cast<uint2*>(params_bf16)[i] = make_uint2(lo, hi);
    }
  }
  for (int64_t i = n4 * 4 + static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n;
       i += stride) {
    float mm = m[i], vv = v[i];
    const float p = adam_one(params[i], __fmul_rn(grads[i], gscale), mm, vv, a);
    params[i] = p;
    m[i] = mm;
    v[i] = vv;
    if (params_bf16) params_bf16[i] = __bfloat16_as_ushort(__float2bfloat16_rn(p));
  }
}

// dst[c, r] = bf16(src[r, c]) through a 32x33 shared tile.
__global__ void transpose_bf16_kernel(const float* __restrict__ src, int64_t rows, int64_t cols,
                                      uint16_t* __restrict__ dst) {
  griddep_wait();
  griddep_launch_dependents();
  __shared__ float tile[32][33];
  const int64_t r0 = static_cast<int64_t>(blockIdx.y) * 32;
  const int64_t c0 = static_cast<int64_t>(blockIdx.x) * 32;
  for (int i = threadIdx.y; i < 32; i += blockDim.y) {
    const int64_t r = r0 + i, c = c0 + threadIdx.x;
    if (r < rows && c < cols) tile[i][threadIdx.x] = src[r * cols + c];
  }
  __syncthreads();
  for (int i = threadIdx.y; i < 32; i += blockDim.y) {
    const int64_t c = c0 + i, r = r0 + threadIdx.x;
    if (r < rows && c < cols)
      dst[c * rows + r] = __bfloat16_as_ushort(__float2bfloat16_rn(tile[threadIdx.x][i]));
  }
}

int grid_for(int64_t items, int block) {
  const int64_t want = (items + block - 1) / block;
  const int64_t cap = static_cast<int64_t>(sm_count()) * 8;
  return static_cast<int>(want < 1 ? 1 : (want > cap ? cap : want));
}

}  // namespace
}  // namespace tq

extern "C" int tq_sumsq(const float* x, int64_t n, float* out, int accumulate, void* stream) {
  using namespace tq;
  if (n < 0) return fail(TQ_ERR_INVALID, "negative length");
  if (!out) return fail(TQ_ERR_INVALID, "null output");
  cudaStream_t s = as_stream(stream);
  int rc = TQ_OK;
  if (!accumulate) {
    rc = check_cuda(cudaMemsetAsync(out, 0, sizeof(float), s), "memset");
    if (rc) return rc;
  }
  if (n == 0) return TQ_OK;
  if (!x || !aligned(x, 16)) return fail(TQ_ERR_MISALIGNED, "x must be non-null and 16-byte aligned");
  return launch_kernel(sumsq_kernel, dim3(grid_for(n / 4 + 1, 256)), dim3(256), 0, s, 1,
                       "sumsq launch", x, n, out);
}

extern "C" int tq_adamw(float* params, const float* grads, float* m, float* v, int64_t n, int64_t t,
                        float lr, float beta1, float beta2, float eps, float weight_decay,
                        float grad_scale, const float* norm_sq, float clip, void* params_bf16,
                        void* stream) {
  using namespace tq;
  if (n < 0) return fail(TQ_ERR_INVALID, "negative length");
  if (t < 1) return fail(TQ_ERR_INVALID, "the step count t starts at 1, got %lld", (long long)t);
  if (n == 0) return TQ_OK;
  if (!params || !grads || !m || !v) return fail(TQ_ERR_INVALID, "null pointer");
  if (!aligned(params, 16) || !aligned(grads, 16) || !aligned(m, 16) || !aligned(v, 16) ||
      (params_bf16 && !aligned(params_bf16, 8)))
    return fail(TQ_ERR_MISALIGNED, "params, grads and moments must be 16-byte aligned");
  AdamArgs a;
  a.lr = lr;
  a.beta1 = beta1;
  a.beta2 = beta2;
  a.eps = eps;
  a.wd = weight_decay;
  a.grad_scale = grad_scale;
  // Bias corrections as the reference computes them: 1 - beta^t in f32.
  a.bias1 = 1.0f - powf(beta1, static_cast<float>(t));
  a.bias2 = 1.0f - powf(beta2, static_cast<float>(t));
  a.clip = clip;
  return launch_kernel(adamw_kernel, dim3(grid_for(n / 4 + 1, 256)), dim3(256), 0,
                       as_stream(stream), 1, "adamw launch", params, grads, m, v, n, a, norm_sq,
                       static_cast<uint16_t*>(params_bf16));
}

extern "C" int tq_transpose_to_bf16(const float* src, int64_t rows, int64_t cols, void* dst,
                                    void* stream) {
  using namespace tq;
  if (rows < 0 || cols < 0) return fail(TQ_ERR_INVALID, "negative shape");
  if (rows == 0 || cols == 0) return TQ_OK;
  if (!src || !dst) return fail(TQ_ERR_INVALID, "null pointer");
  const dim3 block(32, 8);
  const dim3 grid(static_cast<unsigned>((cols + 31) / 32), static_cast<unsigned>((rows + 31) / 32));
  return launch_kernel(transpose_bf16_kernel, grid, block, 0, as_stream(stream), 1,
                       "transpose launch", src, rows, cols, static_cast<uint16_t*>(dst));
}
