// The decoder glue around the quantized linears, fused: RMSNorm, rotary
// embedding and SwiGLU, forward and backward.  Each reads and writes bf16
// once with 16-byte accesses and does its arithmetic in f32.
//
//   RMSNorm  y = x * rsqrt(mean(x^2) + eps) * w        (engine/src/interp.rs:312-319)
//   RoPE     [a, b] -> [a cos - b sin, b cos + a sin]  on the two halves of each
//            head, angle p / theta^(2i/d)               (engine/src/interp.rs:350-388)
//   SwiGLU   a = (g * sigmoid(g)) * u                   (lib/torobi/models/llama.rb:320-327)
//
// The norm gains are frozen in QLoRA (only adapters train), so the norm's
// backward produces dx only.
#include <cuda_bf16.h>

#include "tq_ptx.cuh"
#include "tq_runtime.h"

namespace tq {
namespace {

__device__ __forceinline__ void bf8_to_f32(const uint4& v, float (&f)[8]) {
  const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    f[2 * i] = __uint_as_float(w[i] << 16);
    f[2 * i + 1] = __uint_as_float(w[i] & 0xFFFF0000u);
  }
}

__device__ __forceinline__ uint4 f32_to_bf8(const float (&f)[8]) {
  uint32_t w[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) w[i] = pack_bf16x2_f32(f[2 * i], f[2 * i + 1]);
  return make_uint4(w[0], w[1], w[2], w[3]);
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) v += __shfl_xor_sync(0xffffffffu, v, off);
  return v;
}

// One warp per row; H % 8 == 0.
// ADD: the row is s = RNE_bf16(x + res), written to s_out, and the norm is
// taken of that stored s (the residual add and the norm that follows it in
// the pre-norm block, in one pass).
// VPL > 0: the row fits in VPL 16-byte vectors a lane (H <= 256 VPL), which
// stay in registers between the sum of squares and the scaling, so the row
// is read from memory once; all VPL loads of a lane are in flight together.
// VPL == 0: any H, the second pass reading the row again (recomputing s from
// x and res rather than reading back its own stores).  Both give the same
// bits: the same operations in the same order.
template <bool ADD, int VPL>
__global__ void __launch_bounds__(256) rmsnorm_fwd_kernel(const uint4* __restrict__ x,
                                                          const uint4* __restrict__ res,
                                                          const uint4* __restrict__ w, int64_t rows,
                                                          int hv, float eps,
                                                          uint4* __restrict__ s_out,
                                                          uint4* __restrict__ y,
                                                          float* __restrict__ rstd) {
  griddep_wait();
  griddep_launch_dependents();
  const int lane = threadIdx.x & 31;
  const int64_t row = static_cast<int64_t>(blockIdx.x) * (blockDim.x >> 5) + (threadIdx.x >> 5);
  if (row >= rows) return;
  const uint4* xr = x + row * hv;
  const uint4* rr = ADD ? res + row * hv : nullptr;
  auto load_row = [&](int i, float (&f)[8]) {
    if constexpr (ADD) {
      float e[8];
      bf8_to_f32(__ldg(xr + i), f);
      bf8_to_f32(__ldg(rr + i), e);
#pragma unroll
      for (int j = 0; j < 8; ++j) f[j] += e[j];
      const uint4 sv = f32_to_bf8(f);  // the stored residual stream
      bf8_to_f32(sv, f);
      return sv;
    } else {
      const uint4 sv = __ldg(xr + i);
      bf8_to_f32(sv, f);
      return sv;
    }
  };
  float ss = 0.0f;
  uint4* yr = y + row * hv;
  if constexpr (VPL > 0) {
    uint4 sv[VPL];
#pragma unroll
    for (int v = 0; v < VPL; ++v) {
      const int i = lane + 32 * v;
      if (i < hv) {
        if constexpr (ADD) {
          sv[v] = __ldg(xr + i);
          const uint4 e = __ldg(rr + i);
          float f[8], g[8];
          bf8_to_f32(sv[v], f);
          bf8_to_f32(e, g);
#pragma unroll
          for (int j = 0; j < 8; ++j) f[j] += g[j];
          sv[v] = f32_to_bf8(f);
        } else {
          sv[v] = __ldg(xr + i);
        }
      }
    }
#pragma unroll
    for (int v = 0; v < VPL; ++v) {
      const int i = lane + 32 * v;
      if (i < hv) {
        if constexpr (ADD) s_out[row * hv + i] = sv[v];
        float f[8];
        bf8_to_f32(sv[v], f);
#pragma unroll
        for (int j = 0; j < 8; ++j) ss = fmaf(f[j], f[j], ss);
      }
    }
    ss = warp_sum(ss);
    const float r = rsqrtf(ss / static_cast<float>(hv * 8) + eps);
    if (rstd && lane == 0) rstd[row] = r;
#pragma unroll
    for (int v = 0; v < VPL; ++v) {
      const int i = lane + 32 * v;
      if (i < hv) {
        float f[8], g[8];
        bf8_to_f32(sv[v], f);
        bf8_to_f32(__ldg(w + i), g);
#pragma unroll
        for (int j = 0; j < 8; ++j) f[j] = f[j] * r * g[j];
        yr[i] = f32_to_bf8(f);
      }
    }
  } else {
    for (int i = lane; i < hv; i += 32) {
      float f[8];
      const uint4 sv = load_row(i, f);
      if constexpr (ADD) s_out[row * hv + i] = sv;
#pragma unroll
      for (int j = 0; j < 8; ++j) ss = fmaf(f[j], f[j], ss);
    }
    ss = warp_sum(ss);
    const float r = rsqrtf(ss / static_cast<float>(hv * 8) + eps);
    if (rstd && lane == 0) rstd[row] = r;
    for (int i = lane; i < hv; i += 32) {
      float f[8], g[8];
      load_row(i, f);
      bf8_to_f32(__ldg(w + i), g);
#pragma unroll
      for (int j = 0; j < 8; ++j) f[j] = f[j] * r * g[j];
      yr[i] = f32_to_bf8(f);
    }
  }
}

// dx = r * (dy*w) - x * r^3 * mean(dy*w*x)   (+ dres when given)
__global__ void __launch_bounds__(256) rmsnorm_bwd_kernel(const uint4* __restrict__ x,
                                                          const uint4* __restrict__ w,
                                                          const float* __restrict__ rstd,
                                                          const uint4* __restrict__ dy,
                                                          const uint4* __restrict__ dres,
                                                          int64_t rows, int hv,
                                                          uint4* __restrict__ dx) {
  griddep_wait();
  griddep_launch_dependents();
  const int lane = threadIdx.x & 31;
  const int64_t row = static_cast<int64_t>(blockIdx.x) * (blockDim.x >> 5) + (threadIdx.x >> 5);
  if (row >= rows) return;
  const uint4* xr = x + row * hv;
  const uint4* dyr = dy + row * hv;
  float dot = 0.0f;
  for (int i = lane; i < hv; i += 32) {
    float f[8], g[8], d[8];
    bf8_to_f32(__ldg(xr + i), f);
    bf8_to_f32(__ldg(w + i), g);
    bf8_to_f32(__ldg(dyr + i), d);
#pragma unroll
    for (int j = 0; j < 8; ++j) dot = fmaf(d[j] * g[j], f[j], dot);
  }
  dot = warp_sum(dot);
  const float r = rstd[row];
  const float c = r * r * r * dot / static_cast<float>(hv * 8);
  uint4* dxr = dx + row * hv;
  const uint4* drr = dres ? dres + row * hv : nullptr;
  for (int i = lane; i < hv; i += 32) {
    float f[8], g[8], d[8];
    bf8_to_f32(__ldg(xr + i), f);
    bf8_to_f32(__ldg(w + i), g);
    bf8_to_f32(__ldg(dyr + i), d);
    float o[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) o[j] = r * d[j] * g[j] - f[j] * c;
    if (drr) {
      float e[8];
      bf8_to_f32(__ldg(drr + i), e);
#pragma unroll
      for (int j = 0; j < 8; ++j) o[j] += e[j];
    }
    dxr[i] = f32_to_bf8(o);
  }
}

// x [tokens, heads, dim] bf16 with tokens = batch * seq (position = token %
// seq); cos/sin [seq, dim/2] f32.  One thread per 8 pairs.  sign = -1 applies
// the inverse rotation (the backward).
// I: the index type, 32-bit whenever the launch's items fit (the per-item
// divisions by heads and seq are then 32-bit; 64-bit ones cost several
// times more and bounded this kernel).
template <typename I>
__global__ void __launch_bounds__(256) rope_kernel(const uint4* __restrict__ x, int64_t tokens,
                                                   int heads, int dim, int seq,
                                                   const float* __restrict__ cosv,
                                                   const float* __restrict__ sinv, float sign,
                                                   uint4* __restrict__ y) {
  griddep_wait();
  griddep_launch_dependents();
  const int half = dim / 2;
  const I per_head = static_cast<I>(half / 8);  // threads per head
  const I n = static_cast<I>(tokens) * static_cast<I>(heads) * per_head;
  const I stride = static_cast<I>(gridDim.x) * blockDim.x;
  for (I idx = static_cast<I>(blockIdx.x) * blockDim.x + threadIdx.x; idx < n; idx += stride) {
    const int c = static_cast<int>(idx % per_head);
    const I th = idx / per_head;                  // token * heads + head
    const I token = th / static_cast<I>(heads);
    const int pos = static_cast<int>(token % static_cast<I>(seq));
    const int64_t base = static_cast<int64_t>(th) * (dim / 8);  // in 16-byte vectors
    float a[8], b[8];
    bf8_to_f32(__ldg(x + base + c), a);
    bf8_to_f32(__ldg(x + base + per_head + c), b);
    const float4* cp = reinterpret_cast<const float4*>(cosv + static_cast<int64_t>(pos) * half + c * 8);
    const float4* sp = reinterpret_cast<const float4*>(sinv + static_cast<int64_t>(pos) * half + c * 8);
    const float4 c0 = __ldg(cp), c1 = __ldg(cp + 1), s0 = __ldg(sp), s1 = __ldg(sp + 1);
    const float cs[8] = {c0.x, c0.y, c0.z, c0.w, c1.x, c1.y, c1.z, c1.w};
    const float sn[8] = {s0.x, s0.y, s0.z, s0.w, s1.x, s1.y, s1.z, s1.w};
    float oa[8], ob[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const float s = sign * sn[j];
      oa[j] = a[j] * cs[j] - b[j] * s;
      ob[j] = b[j] * cs[j] + a[j] * s;
    }
    y[base + c] = f32_to_bf8(oa);
    y[base + per_head + c] = f32_to_bf8(ob);
  }
}

__device__ __forceinline__ float sigmoidf_(float v) { return 1.0f / (1.0f + __expf(-v)); }

__global__ void __launch_bounds__(256) swiglu_fwd_kernel(const uint4* __restrict__ g,
                                                         const uint4* __restrict__ u, int64_t nv,
                                                         uint4* __restrict__ a) {
  griddep_wait();
  griddep_launch_dependents();
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < nv; i += stride) {
    float fg[8], fu[8], o[8];
    bf8_to_f32(__ldg(g + i), fg);
    bf8_to_f32(__ldg(u + i), fu);
#pragma unroll
    for (int j = 0; j < 8; ++j) o[j] = fg[j] * sigmoidf_(fg[j]) * fu[j];
    a[i] = f32_to_bf8(o);
  }
}

__global__ void __launch_bounds__(256) swiglu_bwd_kernel(const uint4* __restrict__ g,
                                                         const uint4* __restrict__ u,
                                                         const uint4* __restrict__ da, int64_t nv,
                                                         uint4* __restrict__ dg,
                                                         uint4* __restrict__ du) {
  griddep_wait();
  griddep_launch_dependents();
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < nv; i += stride) {
    float fg[8], fu[8], fd[8], og[8], ou[8];
    bf8_to_f32(__ldg(g + i), fg);
    bf8_to_f32(__ldg(u + i), fu);
    bf8_to_f32(__ldg(da + i), fd);
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const float s = sigmoidf_(fg[j]);
      const float silu = fg[j] * s;
      ou[j] = fd[j] * silu;
      og[j] = fd[j] * fu[j] * s * (1.0f + fg[j] * (1.0f - s));
    }
    dg[i] = f32_to_bf8(og);
    du[i] = f32_to_bf8(ou);
  }
}

int grid_for(int64_t items, int block, int per_sm = 8) {
  const int64_t want = (items + block - 1) / block;
  const int64_t cap = static_cast<int64_t>(sm_count()) * per_sm;
  return static_cast<int>(want < 1 ? 1 : (want > cap ? cap : want));
}

bool a16(const void* p) { return p == nullptr || aligned(p, 16); }

// Vectors a lane holds when a row of hv 16-byte vectors stays in registers
// (0: the row is too long; the kernel then reads it twice).  The backward
// keeps its two reads: holding x and dy of a 4096-wide row (169 registers)
// left one block per SM and ran 8192 x 4096 in 102 us against 74.
int row_vpl(int64_t hv) { return hv <= 128 ? 4 : (hv <= 256 ? 8 : (hv <= 512 ? 16 : 0)); }

template <bool ADD>
using FwdKernel = void (*)(const uint4*, const uint4*, const uint4*, int64_t, int, float, uint4*,
                           uint4*, float*);

template <bool ADD>
FwdKernel<ADD> fwd_kernel_for(int64_t hv) {
  switch (row_vpl(hv)) {
    case 4: return rmsnorm_fwd_kernel<ADD, 4>;
    case 8: return rmsnorm_fwd_kernel<ADD, 8>;
    case 16: return rmsnorm_fwd_kernel<ADD, 16>;
    default: return rmsnorm_fwd_kernel<ADD, 0>;
  }
}


// Whether the byte ranges [a, a + n) and [b, b + n) share a byte.
bool overlap(const void* a, const void* b, size_t n) {
  const uintptr_t x = reinterpret_cast<uintptr_t>(a), y = reinterpret_cast<uintptr_t>(b);
  return x < y + n && y < x + n;
}

}  // namespace
}  // namespace tq

extern "C" int tq_rmsnorm_fwd(const void* x, const void* w, int64_t rows, int64_t hidden,
                              float eps, void* y, float* rstd, void* stream) {
  using namespace tq;
  if (rows < 0 || hidden <= 0 || hidden % 8 != 0)
    return fail(TQ_ERR_INVALID, "rmsnorm: hidden (%lld) must be a positive multiple of 8",
                (long long)hidden);
  if (rows == 0) return TQ_OK;
  if (!x || !w || !y) return fail(TQ_ERR_INVALID, "rmsnorm: null pointer");
  if (!a16(x) || !a16(w) || !a16(y) || (rstd && !aligned(rstd, 4)))
    return fail(TQ_ERR_MISALIGNED, "rmsnorm: x, w and y must be 16-byte aligned");
  const int warps = 8;
  const unsigned grid = static_cast<unsigned>((rows + warps - 1) / warps);
  return launch_kernel(fwd_kernel_for<false>(hidden / 8), dim3(grid), dim3(warps * 32), 0,
                       as_stream(stream), 1, "rmsnorm_fwd launch", static_cast<const uint4*>(x),
                       nullptr, static_cast<const uint4*>(w), rows, static_cast<int>(hidden / 8),
                       eps, nullptr, static_cast<uint4*>(y), rstd);
}

extern "C" int tq_add_rmsnorm_fwd(const void* x, const void* res, const void* w, int64_t rows,
                                  int64_t hidden, float eps, void* s, void* y, float* rstd,
                                  void* stream) {
  using namespace tq;
  if (rows < 0 || hidden <= 0 || hidden % 8 != 0)
    return fail(TQ_ERR_INVALID, "add_rmsnorm: hidden (%lld) must be a positive multiple of 8",
                (long long)hidden);
  if (rows == 0) return TQ_OK;
  if (!x || !res || !w || !s || !y) return fail(TQ_ERR_INVALID, "add_rmsnorm: null pointer");
  if (!a16(x) || !a16(res) || !a16(w) || !a16(s) || !a16(y) || (rstd && !aligned(rstd, 4)))
    return fail(TQ_ERR_MISALIGNED, "add_rmsnorm: x, res, w, s and y must be 16-byte aligned");
  // The kernel forms s = x + res, then reads x and res again for the norm of
  // s: an s or y written over either input would be summed twice.
  const size_t bytes = static_cast<size_t>(rows) * static_cast<size_t>(hidden) * 2;
  if (overlap(s, x, bytes) || overlap(s, res, bytes) || overlap(y, x, bytes) ||
      overlap(y, res, bytes) || overlap(y, s, bytes))
    return fail(TQ_ERR_INVALID,
                "add_rmsnorm: s and y must not overlap x, res or each other (no in-place form)");
  const int warps = 8;
  const unsigned grid = static_cast<unsigned>((rows + warps - 1) / warps);
  return launch_kernel(fwd_kernel_for<true>(hidden / 8), dim3(grid), dim3(warps * 32), 0,
                       as_stream(stream), 1, "add_rmsnorm_fwd launch",
                       static_cast<const uint4*>(x), static_cast<const uint4*>(res),
                       static_cast<const uint4*>(w), rows, static_cast<int>(hidden / 8), eps,
                       static_cast<uint4*>(s), static_cast<uint4*>(y), rstd);
}

extern "C" int tq_rmsnorm_bwd(const void* x, const void* w, const float* rstd, const void* dy,
                              const void* dres, int64_t rows, int64_t hidden, void* dx,
                              void* stream) {
  using namespace tq;
  if (rows < 0 || hidden <= 0 || hidden % 8 != 0)
    return fail(TQ_ERR_INVALID, "rmsnorm: hidden (%lld) must be a positive multiple of 8",
                (long long)hidden);
  if (rows == 0) return TQ_OK;
  if (!x || !w || !rstd || !dy || !dx) return fail(TQ_ERR_INVALID, "rmsnorm: null pointer");
  if (!a16(x) || !a16(w) || !a16(dy) || !a16(dres) || !a16(dx))
    return fail(TQ_ERR_MISALIGNED, "rmsnorm: tensors must be 16-byte aligned");
  const int warps = 8;
  const unsigned grid = static_cast<unsigned>((rows + warps - 1) / warps);
  return launch_kernel(rmsnorm_bwd_kernel, dim3(grid), dim3(warps * 32), 0, as_stream(stream), 1,
                       "rmsnorm_bwd launch", static_cast<const uint4*>(x),
                       static_cast<const uint4*>(w), rstd, static_cast<const uint4*>(dy),
                       static_cast<const uint4*>(dres), rows, static_cast<int>(hidden / 8),
                       static_cast<uint4*>(dx));
}

extern "C" int tq_rope(const void* x, int64_t tokens, int64_t heads, int64_t dim, int64_t seq,
                       const float* cosv, const float* sinv, int inverse, void* y, void* stream) {
  using namespace tq;
  if (tokens < 0 || heads <= 0 || dim <= 0 || dim % 16 != 0 || seq <= 0)
    return fail(TQ_ERR_INVALID, "rope: dim (%lld) must be a positive multiple of 16",
                (long long)dim);
  if (tokens % seq != 0)
    return fail(TQ_ERR_INVALID, "rope: %lld tokens are not whole sequences of %lld",
                (long long)tokens, (long long)seq);
  if (tokens == 0) return TQ_OK;
  if (!x || !cosv || !sinv || !y) return fail(TQ_ERR_INVALID, "rope: null pointer");
  if (!a16(x) || !a16(y) || !a16(cosv) || !a16(sinv))
    return fail(TQ_ERR_MISALIGNED, "rope: tensors must be 16-byte aligned");
  const int64_t n = tokens * heads * (dim / 16);
  const int grid = grid_for(n, 256);
  // 32-bit indices while every index the grid-stride loop forms fits.
  auto kernel = n + static_cast<int64_t>(grid) * 256 < (1ll << 32) ? rope_kernel<uint32_t>
                                                                    : rope_kernel<int64_t>;
  return launch_kernel(kernel, dim3(grid), dim3(256), 0, as_stream(stream), 1, "rope launch",
                       static_cast<const uint4*>(x), tokens, static_cast<int>(heads),
                       static_cast<int>(dim), static_cast<int>(seq), cosv, sinv,
                       inverse ? -1.0f : 1.0f, static_cast<uint4*>(y));
}

extern "C" int tq_swiglu_fwd(const void* g, const void* u, int64_t n, void* a, void* stream) {
  using namespace tq;
  if (n < 0 || n % 8 != 0) return fail(TQ_ERR_INVALID, "swiglu: n (%lld) must be a multiple of 8",
                                       (long long)n);
  if (n == 0) return TQ_OK;
  if (!g || !u || !a) return fail(TQ_ERR_INVALID, "swiglu: null pointer");
  if (!a16(g) || !a16(u) || !a16(a)) return fail(TQ_ERR_MISALIGNED, "swiglu: 16-byte alignment");
  return launch_kernel(swiglu_fwd_kernel, dim3(grid_for(n / 8, 256)), dim3(256), 0,
                       as_stream(stream), 1, "swiglu_fwd launch", static_cast<const uint4*>(g),
                       static_cast<const uint4*>(u), n / 8, static_cast<uint4*>(a));
}

extern "C" int tq_swiglu_bwd(const void* g, const void* u, const void* da, int64_t n, void* dg,
                             void* du, void* stream) {
  using namespace tq;
  if (n < 0 || n % 8 != 0) return fail(TQ_ERR_INVALID, "swiglu: n (%lld) must be a multiple of 8",
                                       (long long)n);
  if (n == 0) return TQ_OK;
  if (!g || !u || !da || !dg || !du) return fail(TQ_ERR_INVALID, "swiglu: null pointer");
  if (!a16(g) || !a16(u) || !a16(da) || !a16(dg) || !a16(du))
    return fail(TQ_ERR_MISALIGNED, "swiglu: 16-byte alignment");
  return launch_kernel(swiglu_bwd_kernel, dim3(grid_for(n / 8, 256)), dim3(256), 0,
                       as_stream(stream), 1, "swiglu_bwd launch", static_cast<const uint4*>(g),
                       static_cast<const uint4*>(u), static_cast<const uint4*>(da), n / 8,
                       static_cast<uint4*>(dg), static_cast<uint4*>(du));
}
