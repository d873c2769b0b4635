// Cross-entropy of bf16 logits, in f32, forward and backward.
//
// The reference's loss node answers logsumexp(logits) - logits[target] per
// position and reduces nothing (engine/src/interp.rs:434-444, the
// cross_entropy op of config/ops.yml:212-220); its VJP, as MLX derives it, is
// dloss * (softmax(logits) - onehot(target)).  One CTA per row: the forward
// reads the row once (a running max and sum of exponentials per thread,
// combined across the block) and writes lse and the loss; the backward reads
// the row again and writes the bf16 gradient, which may overwrite the
// logits themselves, so no second [rows, vocab] buffer is needed (the
// ops.yml note asks exactly that of the backward).  HBM-bound: 2 bytes per
// logit forward, 4 backward.
#include <cuda_bf16.h>

#include "tq_ptx.cuh"
#include "tq_runtime.h"

namespace tq {
namespace {

constexpr int kCeThreads = 512;

struct MaxSum {
  float m;  // running maximum
  float s;  // sum of exp(z - m)
};

__device__ __forceinline__ MaxSum ms_merge(MaxSum a, MaxSum b) {
  const float m = fmaxf(a.m, b.m);
  if (m == -INFINITY) return {m, 0.0f};
  return {m, a.s * __expf(a.m - m) + b.s * __expf(b.m - m)};
}

__device__ __forceinline__ float bf16_lo(uint32_t w) { return __uint_as_float(w << 16); }
__device__ __forceinline__ float bf16_hi(uint32_t w) { return __uint_as_float(w & 0xFFFF0000u); }

__device__ __forceinline__ float ldg_bf16(const uint16_t* p) {
  return __uint_as_float(static_cast<uint32_t>(__ldg(reinterpret_cast<const unsigned short*>(p)))
                         << 16);
}

// Folds eight logits into the running (max, sum).
__device__ __forceinline__ void ms_add8(MaxSum& acc, const float (&z)[8]) {
  float mx = z[0];
#pragma unroll
  for (int i = 1; i < 8; ++i) mx = fmaxf(mx, z[i]);
  float s = 0.0f;
#pragma unroll
  for (int i = 0; i < 8; ++i) s += __expf(z[i] - mx);
  acc = ms_merge(acc, MaxSum{mx, s});
}

__device__ __forceinline__ void unpack8(uint4 v, float (&z)[8]) {
  const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    z[2 * i] = bf16_lo(w[i]);
    z[2 * i + 1] = bf16_hi(w[i]);
  }
}

// Block-wide merge; every thread gets the row's (max, sum).
__device__ __forceinline__ MaxSum block_merge(MaxSum v, MaxSum* sh) {
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) {
    MaxSum o{__shfl_xor_sync(0xffffffffu, v.m, off), __shfl_xor_sync(0xffffffffu, v.s, off)};
    v = ms_merge(v, o);
  }
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (lane == 0) sh[warp] = v;
  __syncthreads();
  if (warp == 0) {
    v = lane < kCeThreads / 32 ? sh[lane] : MaxSum{-INFINITY, 0.0f};
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) {
      MaxSum o{__shfl_xor_sync(0xffffffffu, v.m, off), __shfl_xor_sync(0xffffffffu, v.s, off)};
      v = ms_merge(v, o);
    }
    if (lane == 0) sh[0] = v;
  }
  __syncthreads();
  return sh[0];
}

// VEC: rows start on 16-byte boundaries and vocab % 8 == 0 (8 logits a load).
// A target outside [0, vocab) contributes lse (no logit is picked).
template <bool VEC>
__global__ void __launch_bounds__(kCeThreads) ce_fwd_kernel(const uint16_t* __restrict__ z,
                                                            const int64_t* __restrict__ tgt,
                                                            int vocab, int64_t ld,
                                                            float* __restrict__ lse,
                                                            float* __restrict__ loss) {
  griddep_wait();
  griddep_launch_dependents();
  __shared__ MaxSum sh[kCeThreads / 32];
  const int64_t r = blockIdx.x;
  const uint16_t* row = z + r * ld;
  MaxSum acc{-INFINITY, 0.0f};
  if constexpr (VEC) {
    const uint4* rv = reinterpret_cast<const uint4*>(row);
    const int nv = vocab / 8;
    for (int i = threadIdx.x; i < nv; i += kCeThreads) {
      float f[8];
      unpack8(__ldg(rv + i), f);
      ms_add8(acc, f);
    }
  } else {
    for (int i = threadIdx.x; i < vocab; i += kCeThreads)
      acc = ms_merge(acc, MaxSum{ldg_bf16(row + i), 1.0f});
  }
  const MaxSum tot = block_merge(acc, sh);
  if (threadIdx.x == 0) {
    const float l = tot.m + __logf(tot.s);
    const int64_t t = tgt[r];
    const float picked = (t >= 0 && t < vocab) ? ldg_bf16(row + t) : 0.0f;
    lse[r] = l;
    loss[r] = l - picked;
  }
}

template <bool VEC>
__global__ void __launch_bounds__(kCeThreads) ce_bwd_kernel(const uint16_t* z,
                                                            const int64_t* __restrict__ tgt,
                                                            const float* __restrict__ lse,
                                                            int vocab, int64_t ld,
                                                            const float* __restrict__ dloss,
                                                            float scale, uint16_t* dz) {
  griddep_wait();
  griddep_launch_dependents();
  const int64_t r = blockIdx.x;
  const uint16_t* row = z + r * ld;
  uint16_t* out = dz + r * ld;
  const float l = lse[r];
  const float g = scale * (dloss ? dloss[r] : 1.0f);
  const int64_t t = tgt[r];
  if constexpr (VEC) {
    const uint4* rv = reinterpret_cast<const uint4*>(row);
    uint4* ov = reinterpret_cast<uint4*>(out);
    const int nv = vocab / 8;
    for (int i = threadIdx.x; i < nv; i += kCeThreads) {
      float f[8];
      unpack8(rv[i], f);  // plain load: the output may overwrite this row
      uint32_t w[4];
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        float a = __expf(f[2 * k] - l);
        float b = __expf(f[2 * k + 1] - l);
        const int64_t j = static_cast<int64_t>(i) * 8 + 2 * k;
        if (j == t) a -= 1.0f;
        if (j + 1 == t) b -= 1.0f;
        w[k] = pack_bf16x2_f32(g * a, g * b);
      }
      ov[i] = make_uint4(w[0], w[1], w[2], w[3]);
    }
  } else {
    for (int i = threadIdx.x; i < vocab; i += kCeThreads) {
      float p = __expf(__uint_as_float(static_cast<uint32_t>(row[i]) << 16) - l);
      if (i == t) p -= 1.0f;
      out[i] = __bfloat16_as_ushort(__float2bfloat16_rn(g * p));
    }
  }
}

int ce_check(const void* logits, const int64_t* targets, int64_t rows, int64_t vocab, int64_t ld,
             const char* who) {
  if (rows < 0 || vocab <= 0 || ld < vocab)
    return fail(TQ_ERR_INVALID, "%s: need rows >= 0, vocab > 0 and ld >= vocab (got %lld, %lld, %lld)",
                who, (long long)rows, (long long)vocab, (long long)ld);
  if (vocab > (1ll << 31) - 1 || rows > (1ll << 31) - 1)
    return fail(TQ_ERR_INVALID, "%s: rows and vocab must fit in 31 bits", who);
  if (rows > 0 && (!logits || !targets)) return fail(TQ_ERR_INVALID, "%s: null pointer", who);
  if (!aligned(logits, 2) || !aligned(targets, 8))
    return fail(TQ_ERR_MISALIGNED, "%s: logits must be 2-byte and targets 8-byte aligned", who);
  return TQ_OK;
}

bool ce_vec(const void* a, const void* b, int64_t vocab, int64_t ld) {
  return vocab % 8 == 0 && ld % 8 == 0 && aligned(a, 16) && aligned(b, 16);
}

}  // namespace
}  // namespace tq

extern "C" int tq_cross_entropy_fwd(const void* logits, const int64_t* targets, int64_t rows,
                                    int64_t vocab, int64_t ld, float* lse, float* loss,
                                    void* stream) {
  using namespace tq;
  int rc = ce_check(logits, targets, rows, vocab, ld, "cross_entropy_fwd");
  if (rc) return rc;
  if (rows == 0) return TQ_OK;
  if (!lse || !loss) return fail(TQ_ERR_INVALID, "cross_entropy_fwd: null output");
  if (!aligned(lse, 4) || !aligned(loss, 4))
    return fail(TQ_ERR_MISALIGNED, "cross_entropy_fwd: lse and loss must be 4-byte aligned");
  const uint16_t* z = static_cast<const uint16_t*>(logits);
  const int v = static_cast<int>(vocab);
  const unsigned grid = static_cast<unsigned>(rows);
  auto kernel = ce_vec(logits, logits, vocab, ld) ? ce_fwd_kernel<true> : ce_fwd_kernel<false>;
  return launch_kernel(kernel, dim3(grid), dim3(kCeThreads), 0, as_stream(stream), 1,
                       "cross_entropy_fwd launch", z, targets, v, ld, lse, loss);
}

extern "C" int tq_cross_entropy_bwd(const void* logits, const int64_t* targets, const float* lse,
                                    int64_t rows, int64_t vocab, int64_t ld, const float* dloss,
                                    float scale, void* dlogits, void* stream) {
  using namespace tq;
  int rc = ce_check(logits, targets, rows, vocab, ld, "cross_entropy_bwd");
  if (rc) return rc;
  if (rows == 0) return TQ_OK;
  if (!lse || !dlogits) return fail(TQ_ERR_INVALID, "cross_entropy_bwd: null pointer");
  if (!aligned(dlogits, 2) || !aligned(lse, 4) || (dloss && !aligned(dloss, 4)))
    return fail(TQ_ERR_MISALIGNED, "cross_entropy_bwd: misaligned lse, dloss or dlogits");
  const uint16_t* z = static_cast<const uint16_t*>(logits);
  uint16_t* dz = static_cast<uint16_t*>(dlogits);
  const int v = static_cast<int>(vocab);
  const unsigned grid = static_cast<unsigned>(rows);
  auto kernel = ce_vec(logits, dlogits, vocab, ld) ? ce_bwd_kernel<true> : ce_bwd_kernel<false>;
  return launch_kernel(kernel, dim3(grid), dim3(kCeThreads), 0, as_stream(stream), 1,
                       "cross_entropy_bwd launch", z, targets, lse, v, ld, dloss, scale, dz);
}
