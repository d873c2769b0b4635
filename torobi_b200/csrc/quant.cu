// Affine quantize / dequantize kernels (MLX layout) and their C entry points.
//
// Both are HBM-bound streams: quantize reads 2 bytes per element and writes
// bits/8 + 4/group_size; dequantize the reverse.  Each thread owns whole
// 16-byte vectors so every global access is a 128-bit transaction, and a
// group's min/max is reduced across the group_size/32 lanes that hold it with
// warp shuffles (groups never straddle a warp: 32 lanes x 32 elements covers
// a whole number of groups for group_size in {32, 64, 128}).
#include <cuda_bf16.h>

#include <cstdio>

#include "tq_ptx.cuh"
#include "tq_runtime.h"

namespace tq {
namespace {

__device__ __forceinline__ float mlx_max(float a, float b) { return a < b ? b : a; }
__device__ __forceinline__ float mlx_min(float a, float b) { return b < a ? b : a; }

__device__ __forceinline__ float bf16_bits_to_f32(uint32_t h) { return __uint_as_float(h << 16); }

// Lane-wise max / min of two bf16 pairs; a NaN lane yields the other operand.
__device__ __forceinline__ uint32_t bf16x2_max(uint32_t a, uint32_t b) {
  uint32_t d;
  asm("max.bf16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
  return d;
}
__device__ __forceinline__ uint32_t bf16x2_min(uint32_t a, uint32_t b) {
  uint32_t d;
  asm("min.bf16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
  return d;
}

// f32 -> bf16 bits, round to nearest even (NaN -> canonical quiet NaN 0x7FC0).
__device__ __forceinline__ uint16_t f32_to_bf16_bits(float f) {
  if (f != f) return 0x7FC0;
  const uint32_t u = __float_as_uint(f);
  return static_cast<uint16_t>((u + 0x7FFFu + ((u >> 16) & 1u)) >> 16);
}

// Quantizes 32 consecutive elements (four 16-byte vectors r[0..3]) held by
// lane `lane` of a warp whose 32 lanes hold 32 consecutive such runs (pi is
// this run's index).  LANES = lanes per group = group_size / 32 (1, 2 or 4);
// a group's min/max is reduced across its lanes with shuffles, so every lane
// of the warp must call this.  Thirty-two elements a thread spread the
// group's three divisions, which every lane of the group computes, over four
// times the elements of one vector a thread.
template <int BITS, int LANES>
__device__ __forceinline__ void quantize_run(const uint4 (&r)[4], bool live, int64_t pi,
                                             const uint16_t* __restrict__ src,
                                             int lane, uint32_t* __restrict__ codes,
                                             uint16_t* __restrict__ scales,
                                             uint16_t* __restrict__ biases) {
  constexpr int kE = 32;
  constexpr float n_bins = static_cast<float>((1 << BITS) - 1);
  constexpr float eps = 1e-7f;
  uint32_t words[16];
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    words[4 * k] = r[k].x;
    words[4 * k + 1] = r[k].y;
    words[4 * k + 2] = r[k].z;
    words[4 * k + 3] = r[k].w;
  }
  // Group max/min on bf16 pairs: exact (the result is one of the inputs), a
  // NaN element is passed over as the f32 comparisons of the oracle do, and
  // the sign of a zero extreme cannot change the scale or bias below.
  uint32_t mx2 = 0xFF80FF80u, mn2 = 0x7F807F80u;  // (-inf, -inf), (+inf, +inf)
  if (live) {
#pragma unroll
    for (int j = 0; j < 16; ++j) {
      mx2 = bf16x2_max(mx2, words[j]);
      mn2 = bf16x2_min(mn2, words[j]);
    }
  }
  float w_max = fmaxf(bf16_bits_to_f32(mx2 & 0xFFFFu), bf16_bits_to_f32(mx2 >> 16));
  float w_min = fminf(bf16_bits_to_f32(mn2 & 0xFFFFu), bf16_bits_to_f32(mn2 >> 16));
#pragma unroll
  for (int off = 1; off < LANES; off <<= 1) {
    w_max = mlx_max(w_max, __shfl_xor_sync(0xffffffffu, w_max, off));
    w_min = mlx_min(w_min, __shfl_xor_sync(0xffffffffu, w_min, off));
  }
  const bool side = fabsf(w_min) > fabsf(w_max);
  float scale = mlx_max(__fdiv_rn(__fsub_rn(w_max, w_min), n_bins), eps);
  scale = side ? scale : -scale;
  const float edge = side ? w_min : w_max;
  const float q0 = rintf(__fdiv_rn(edge, scale));
  float bias = 0.0f;
  if (q0 != 0.0f) {
    scale = __fdiv_rn(edge, q0);
    bias = edge;
  }
  // q = rint(fl((v - bias) / scale)) without a division per element.  With
  // rs = fl(1 / scale) and y = fl(d * rs), |y - fl(d / scale)| is at most
  // 1.5 * 2^-23 * |d / scale|: below 2^-14 * 0.75 while |y| < 512, and the
  // codes of a group keep |y| near [0, 2^bits - 1].  So rint(y) is the
  // answer unless y lies within 2^-12 of a half-integer (where the rounding
  // of the quotient itself decides), is not finite, or is that large.  Of
  // those, an exact quotient (d - y * scale == 0 by one fma, d normal) is y
  // itself; the rest, about 0.05-0.2 % of elements, take the IEEE division.
  //
  // |y| < 512 holds for every element of the group when it holds for the
  // largest |d| (rounding is monotone, so no element's y exceeds
  // fl(max|d| * |rs|)); one test a group replaces one an element.  Groups
  // with an infinite or NaN extreme, or a huge q0, fail it and take the
  // exact path throughout.
  constexpr float kRound = 12582912.0f;  // 1.5 * 2^23
  constexpr int kMaxCode = (1 << BITS) - 1;
  const float rs = __frcp_rn(scale);
  const float d_top = fmaxf(fabsf(__fsub_rn(w_max, bias)), fabsf(__fsub_rn(w_min, bias)));
  const bool in_range = __fmul_rn(d_top, fabsf(rs)) < 512.0f;
  uint32_t packed[BITS] = {};  // 32 codes: 4 words at 4 bits, 8 at 8
  if constexpr (BITS == 4) {
    // Without a branch or a conversion instruction: t = y + 1.5 * 2^23
    // rounds y to an integer (ties to even, |y| < 2^22), so t - 1.5 * 2^23
    // is rint(y) and t's low mantissa bits are that integer; the code is it
    // clamped to [0, 15].  Elements needing more are marked in `fix` and
    // redone after the loop from their bf16 value (an L1 hit).
    uint32_t fix = 0;
#pragma unroll
    for (int j = 0; j < kE; ++j) {
      const uint32_t h = words[j >> 1];
      const float vj = (j & 1) ? __uint_as_float(h & 0xFFFF0000u) : __uint_as_float(h << 16);
      const float d = __fsub_rn(vj, bias);
      const float y = __fmul_rn(d, rs);
      const float t = __fadd_rn(y, kRound);
      const float q = __fsub_rn(t, kRound);
      if (!(fabsf(__fsub_rn(y, q)) < 0.5f - 0x1p-12f)) fix |= 1u << j;
      const int qi = static_cast<int>(__float_as_uint(t) - __float_as_uint(kRound));
      packed[j >> 3] += static_cast<uint32_t>(__vimin_s32_relu(qi, kMaxCode)) << (4 * (j & 7));
    }
    if (!in_range) fix = 0xFFFFFFFFu;
    if (!live) fix = 0;  // src is only valid for a live run
    while (fix) {
      const int j = __ffs(fix) - 1;
      fix &= fix - 1;
      const float vj = bf16_bits_to_f32(__ldg(src + j));
      const float d = __fsub_rn(vj, bias);
      const float y = __fmul_rn(d, rs);
      const bool exact =
          fabsf(y) < 512.0f && fabsf(d) > 0x1p-100f && __fmaf_rn(-y, scale, d) == 0.0f;
      const float yq = exact ? y : __fdiv_rn(d, scale);
      const uint32_t code = min(__float2uint_rn(yq), static_cast<uint32_t>(kMaxCode));
      const int sh = 4 * (j & 7);
#pragma unroll
      for (int k = 0; k < 4; ++k)
        if (k == (j >> 3)) packed[k] = (packed[k] & ~(15u << sh)) | (code << sh);
    }
  } else {
    // At 8 bits the bf16 grid often puts quotients exactly on half-integers
    // (about one code per representable value), so the exceptions are
    // handled in line: a deferred pass over them ran 13-19 % slower here.
    // The code is the quotient converted with round-to-nearest-even and
    // saturation (negatives and NaN give 0), capped at 255.
#pragma unroll
    for (int j = 0; j < kE; ++j) {
      const uint32_t h = words[j >> 1];
      const float vj = (j & 1) ? __uint_as_float(h & 0xFFFF0000u) : __uint_as_float(h << 16);
      const float d = __fsub_rn(vj, bias);
      const float y = __fmul_rn(d, rs);
      float yq = y;
      if (!(fabsf(__fsub_rn(y, rintf(y))) < 0.5f - 0x1p-12f) || !in_range) {
        const bool exact = fabsf(y) < 512.0f && fabsf(d) > 0x1p-100f &&
                           __fmaf_rn(-y, scale, d) == 0.0f;
        if (!exact) yq = __fdiv_rn(d, scale);
      }
      const uint32_t code = min(__float2uint_rn(yq), static_cast<uint32_t>(kMaxCode));
      packed[j >> 2] += code << (8 * (j & 3));
    }
  }
  if (live) {
    uint4* out = reinterpret_cast<uint4*>(codes) + pi * (BITS / 4);
    out[0] = make_uint4(packed[0], packed[1], packed[2], packed[3]);
    if constexpr (BITS == 8) out[1] = make_uint4(packed[4], packed[5], packed[6], packed[7]);
    if ((lane & (LANES - 1)) == 0) {
      const int64_t gi = pi / LANES;
      scales[gi] = f32_to_bf16_bits(scale);
      biases[gi] = f32_to_bf16_bits(bias);
    }
  }
}

// Each warp takes 32 consecutive runs of 32 elements per iteration; the four
// loads of a thread's run are in flight before it works on any.
template <int BITS, int LANES>
__global__ void __launch_bounds__(256) quantize_kernel(const uint4* __restrict__ w,
                                                       int64_t n_runs, uint32_t* __restrict__ codes,
                                                       uint16_t* __restrict__ scales,
                                                       uint16_t* __restrict__ biases) {
  const int lane = threadIdx.x & 31;
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  for (int64_t base = static_cast<int64_t>(blockIdx.x) * blockDim.x + (threadIdx.x & ~31);
       base < n_runs; base += stride) {
    const int64_t pi = base + lane;
    const bool live = pi < n_runs;
    uint4 r[4];
#pragma unroll
    for (int k = 0; k < 4; ++k) r[k] = live ? __ldg(w + 4 * pi + k) : make_uint4(0, 0, 0, 0);
    quantize_run<BITS, LANES>(r, live, pi, reinterpret_cast<const uint16_t*>(w + 4 * pi), lane,
                              codes, scales, biases);
  }
}

// One code word a lane per step (8 elements at 4 bits, 4 at 8), so a warp
// reads 128 contiguous bytes and writes 512 (256) contiguous bytes per
// instruction; each thread takes kWords words, 32 apart, all loaded (with
// their groups' scale and bias) before any is dequantized.
constexpr int kWords = 8;

// One warp-span of kWords * 32 words starting at `base`: lane `lane` takes
// words base + 32k + lane, all loaded (with their groups' scale and bias)
// before any is dequantized.
template <int BITS>
__device__ __forceinline__ void dequantize_span(const uint32_t* __restrict__ codes,
                                                int64_t n_words, int64_t base, int lane,
                                                int group_shift,
                                                const uint16_t* __restrict__ scales,
                                                const uint16_t* __restrict__ biases,
                                                uint16_t* __restrict__ out) {
  constexpr int kElems = 32 / BITS;  // elements per word
  uint32_t c[kWords], s2[kWords], b2[kWords];
#pragma unroll
  for (int k = 0; k < kWords; ++k) {
    const int64_t wi = base + 32 * k + lane;
    const bool live = wi < n_words;
    c[k] = live ? __ldg(codes + wi) : 0u;
    const int64_t gi = live ? (wi * kElems) >> group_shift : 0;  // a group never straddles a word
    s2[k] = bf16_dup(__ldg(scales + gi));
    b2[k] = bf16_dup(__ldg(biases + gi));
  }
#pragma unroll
  for (int k = 0; k < kWords; ++k) {
    const int64_t wi = base + 32 * k + lane;
    if (wi >= n_words) break;
    if constexpr (BITS == 4) {
      uint32_t o[4];
      dequant_u4x8(c[k], s2[k], b2[k], o);
      reinterpret_cast<uint4*>(out)[wi] = make_uint4(o[0], o[1], o[2], o[3]);
    } else {
      uint32_t o[2];
      dequant_u8x4(c[k], s2[k], b2[k], o);
      reinterpret_cast<uint2*>(out)[wi] = make_uint2(o[0], o[1]);
    }
  }
}

template <int BITS>
__global__ void __launch_bounds__(256) dequantize_kernel(const uint32_t* __restrict__ codes,
                                                         int64_t n_words, int group_shift,
                                                         const uint16_t* __restrict__ scales,
                                                         const uint16_t* __restrict__ biases,
                                                         uint16_t* __restrict__ out) {
  const int lane = threadIdx.x & 31;
  const int64_t span = 32 * kWords;  // words a warp covers per iteration
  const int64_t warps = static_cast<int64_t>(gridDim.x) * (blockDim.x >> 5);
  for (int64_t base = (static_cast<int64_t>(blockIdx.x) * (blockDim.x >> 5) + (threadIdx.x >> 5)) *
                      span;
       base < n_words; base += warps * span)
    dequantize_span<BITS>(codes, n_words, base, lane, group_shift, scales, biases, out);
}

// ------------------------------------------------------------- batches ----
//
// Many matrices in one launch (every linear of a model at load time).  Each
// job's work is laid out in a virtual index space padded to whole warp
// iterations (32 runs for quantize, one span of words for dequantize), so a
// warp finds its job once per iteration by a binary search over the starts
// and never straddles two; the tables travel as a kernel parameter.
constexpr int kBatchMax = 256;  // tables of about 12 KB, within the 32 KB of kernel parameters

struct QuantizeBatch {
  int n;
  int64_t start[kBatchMax + 1];  // virtual run index of each job's first run; start[n] = end
  int64_t runs[kBatchMax];
  const uint4* w[kBatchMax];
  uint32_t* codes[kBatchMax];
  uint16_t* scales[kBatchMax];
  uint16_t* biases[kBatchMax];
};

struct DequantizeBatch {
  int n;
  int64_t start[kBatchMax + 1];  // virtual word index of each job's first word
  int64_t words[kBatchMax];
  const uint32_t* codes[kBatchMax];
  const uint16_t* scales[kBatchMax];
  const uint16_t* biases[kBatchMax];
  uint16_t* out[kBatchMax];
};

// The last job whose start is <= v (starts ascending, start[0] = 0).
__device__ __forceinline__ int find_job(const int64_t* start, int n, int64_t v) {
  int lo = 0, hi = n - 1;
  while (lo < hi) {
    const int mid = (lo + hi + 1) >> 1;
    if (start[mid] <= v) lo = mid;
    else hi = mid - 1;
  }
  return lo;
}

template <int BITS, int LANES>
__global__ void __launch_bounds__(256) quantize_batch_kernel(const __grid_constant__ QuantizeBatch b) {
  const int lane = threadIdx.x & 31;
  const int64_t end = b.start[b.n];
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  for (int64_t base = static_cast<int64_t>(blockIdx.x) * blockDim.x + (threadIdx.x & ~31);
       base < end; base += stride) {
    const int j = find_job(b.start, b.n, base);
    const int64_t pi = base - b.start[j] + lane;
    const bool live = pi < b.runs[j];
    const uint4* w = b.w[j];
    uint4 r[4];
#pragma unroll
    for (int k = 0; k < 4; ++k) r[k] = live ? __ldg(w + 4 * pi + k) : make_uint4(0, 0, 0, 0);
    quantize_run<BITS, LANES>(r, live, pi, reinterpret_cast<const uint16_t*>(w + 4 * pi), lane,
                              b.codes[j], b.scales[j], b.biases[j]);
  }
}

template <int BITS>
__global__ void __launch_bounds__(256) dequantize_batch_kernel(const __grid_constant__ DequantizeBatch b,
                                                               int group_shift) {
  const int lane = threadIdx.x & 31;
  const int64_t span = 32 * kWords;
  const int64_t end = b.start[b.n];
  const int64_t warps = static_cast<int64_t>(gridDim.x) * (blockDim.x >> 5);
  for (int64_t base = (static_cast<int64_t>(blockIdx.x) * (blockDim.x >> 5) + (threadIdx.x >> 5)) *
                      span;
       base < end; base += warps * span) {
    const int j = find_job(b.start, b.n, base);
    dequantize_span<BITS>(b.codes[j], b.words[j], base - b.start[j], lane, group_shift,
                          b.scales[j], b.biases[j], b.out[j]);
  }
}

int check_qargs(int64_t rows, int64_t cols, int group_size, int bits) {
  if (bits != 4 && bits != 8) return fail(TQ_ERR_UNSUPPORTED, "bits must be 4 or 8, got %d", bits);
  if (group_size != 32 && group_size != 64 && group_size != 128)
    return fail(TQ_ERR_UNSUPPORTED, "group_size must be 32, 64 or 128, got %d", group_size);
  if (rows < 0 || cols < 0) return fail(TQ_ERR_INVALID, "negative shape [%lld, %lld]",
                                        (long long)rows, (long long)cols);
  if (cols % group_size != 0)
    return fail(TQ_ERR_INVALID,
                "the last dimension (%lld) must be divisible by the quantization group size (%d)",
                (long long)cols, group_size);
  return TQ_OK;
}

int grid_for(int64_t work_items, int block) {
  const int64_t want = (work_items + block - 1) / block;
  const int64_t cap = static_cast<int64_t>(sm_count()) * 16;
  return static_cast<int>(want < 1 ? 1 : (want > cap ? cap : want));
}

}  // namespace
}  // namespace tq

extern "C" int tq_quantize(const void* w, int64_t rows, int64_t cols, int group_size, int bits,
                           void* codes, void* scales, void* biases, void* stream) {
  using namespace tq;
  int rc = check_qargs(rows, cols, group_size, bits);
  if (rc) return rc;
  if (rows == 0 || cols == 0) return TQ_OK;
  if (!w || !codes || !scales || !biases) return fail(TQ_ERR_INVALID, "null pointer");
  if (!aligned(w, 16) || !aligned(codes, 16))
    return fail(TQ_ERR_MISALIGNED, "w and codes must be 16-byte aligned");
  if (!aligned(scales, 2) || !aligned(biases, 2))
    return fail(TQ_ERR_MISALIGNED, "scales and biases must be 2-byte aligned");
  const int64_t n_runs = rows * cols / 32;  // cols % 32 == 0
  const int block = 256;
  const int grid = grid_for(n_runs, block);
  cudaStream_t s = as_stream(stream);
  const uint4* wv = static_cast<const uint4*>(w);
  uint32_t* c = static_cast<uint32_t*>(codes);
  uint16_t* sc = static_cast<uint16_t*>(scales);
  uint16_t* bi = static_cast<uint16_t*>(biases);
  const int lanes = group_size / 32;
  if (bits == 4) {
    if (lanes == 1) quantize_kernel<4, 1><<<grid, block, 0, s>>>(wv, n_runs, c, sc, bi);
    else if (lanes == 2) quantize_kernel<4, 2><<<grid, block, 0, s>>>(wv, n_runs, c, sc, bi);
    else quantize_kernel<4, 4><<<grid, block, 0, s>>>(wv, n_runs, c, sc, bi);
  } else {
    if (lanes == 1) quantize_kernel<8, 1><<<grid, block, 0, s>>>(wv, n_runs, c, sc, bi);
    else if (lanes == 2) quantize_kernel<8, 2><<<grid, block, 0, s>>>(wv, n_runs, c, sc, bi);
    else quantize_kernel<8, 4><<<grid, block, 0, s>>>(wv, n_runs, c, sc, bi);
  }
  return check_cuda(cudaGetLastError(), "quantize launch");
}

extern "C" int tq_dequantize(const void* codes, const void* scales, const void* biases,
                             int64_t rows, int64_t cols, int group_size, int bits, void* w,
                             void* stream) {
  using namespace tq;
  int rc = check_qargs(rows, cols, group_size, bits);
  if (rc) return rc;
  if (rows == 0 || cols == 0) return TQ_OK;
  if (!w || !codes || !scales || !biases) return fail(TQ_ERR_INVALID, "null pointer");
  if (!aligned(w, 16) || !aligned(codes, 16))
    return fail(TQ_ERR_MISALIGNED, "w and codes must be 16-byte aligned");
  const int64_t n_words = rows * cols * bits / 32;
  const int block = 256;
  const int grid = grid_for((n_words + kWords - 1) / kWords, block);
  const int shift = group_size == 32 ? 5 : (group_size == 64 ? 6 : 7);
  cudaStream_t s = as_stream(stream);
  const uint32_t* cw = static_cast<const uint32_t*>(codes);
  const uint16_t* sp = static_cast<const uint16_t*>(scales);
  const uint16_t* bp = static_cast<const uint16_t*>(biases);
  uint16_t* op = static_cast<uint16_t*>(w);
  if (bits == 4)
    dequantize_kernel<4><<<grid, block, 0, s>>>(cw, n_words, shift, sp, bp, op);
  else
    dequantize_kernel<8><<<grid, block, 0, s>>>(cw, n_words, shift, sp, bp, op);
  return check_cuda(cudaGetLastError(), "dequantize launch");
}

namespace {

// The per-matrix checks of tq_quantize / tq_dequantize, for job `i`.
int check_job(int64_t i, const void* in, int64_t rows, int64_t cols, const void* codes,
              const void* scales, const void* biases, int group_size, int bits, bool quantize) {
  using namespace tq;
  int rc = check_qargs(rows, cols, group_size, bits);
  if (rc) {
    char msg[256];
    snprintf(msg, sizeof msg, "%s", tq_last_error());  // fail() rewrites that buffer
    return fail(rc, "job %lld: %s", static_cast<long long>(i), msg);
  }
  if (rows == 0 || cols == 0) return TQ_OK;
  if (!in || !codes || !scales || !biases)
    return fail(TQ_ERR_INVALID, "job %lld: null pointer", static_cast<long long>(i));
  if (!aligned(in, 16) || !aligned(codes, 16))
    return fail(TQ_ERR_MISALIGNED, "job %lld: %s and codes must be 16-byte aligned",
                static_cast<long long>(i), quantize ? "w" : "out");
  if (!aligned(scales, 2) || !aligned(biases, 2))
    return fail(TQ_ERR_MISALIGNED, "job %lld: scales and biases must be 2-byte aligned",
                static_cast<long long>(i));
  return TQ_OK;
}

}  // namespace

extern "C" int tq_quantize_batch(const TqQuantizeJob* jobs, int n_jobs, int group_size, int bits,
                                 void* stream) {
  using namespace tq;
  if (n_jobs < 0 || (n_jobs > 0 && !jobs)) return fail(TQ_ERR_INVALID, "quantize_batch: bad job list");
  int rc = check_qargs(0, group_size, group_size, bits);
  if (rc) return rc;
  for (int i = 0; i < n_jobs; ++i) {
    const TqQuantizeJob& j = jobs[i];
    rc = check_job(i, j.w, j.rows, j.cols, j.codes, j.scales, j.biases, group_size, bits, true);
    if (rc) return rc;
  }
  cudaStream_t s = as_stream(stream);
  const int lanes = group_size / 32;
  QuantizeBatch b;
  int i = 0;
  while (i < n_jobs) {
    b.n = 0;
    int64_t v = 0;
    for (; i < n_jobs && b.n < kBatchMax; ++i) {
      const TqQuantizeJob& j = jobs[i];
      const int64_t runs = j.rows * j.cols / 32;
      if (runs == 0) continue;
      b.start[b.n] = v;
      b.runs[b.n] = runs;
      b.w[b.n] = static_cast<const uint4*>(j.w);
      b.codes[b.n] = static_cast<uint32_t*>(j.codes);
      b.scales[b.n] = static_cast<uint16_t*>(j.scales);
      b.biases[b.n] = static_cast<uint16_t*>(j.biases);
      v += (runs + 31) / 32 * 32;  // whole warp iterations
      ++b.n;
    }
    if (b.n == 0) break;
    b.start[b.n] = v;
    const int grid = grid_for(v, 256);
    if (bits == 4) {
      if (lanes == 1) quantize_batch_kernel<4, 1><<<grid, 256, 0, s>>>(b);
      else if (lanes == 2) quantize_batch_kernel<4, 2><<<grid, 256, 0, s>>>(b);
      else quantize_batch_kernel<4, 4><<<grid, 256, 0, s>>>(b);
    } else {
      if (lanes == 1) quantize_batch_kernel<8, 1><<<grid, 256, 0, s>>>(b);
      else if (lanes == 2) quantize_batch_kernel<8, 2><<<grid, 256, 0, s>>>(b);
      else quantize_batch_kernel<8, 4><<<grid, 256, 0, s>>>(b);
    }
    rc = check_cuda(cudaGetLastError(), "quantize_batch launch");
    if (rc) return rc;
  }
  return TQ_OK;
}

extern "C" int tq_dequantize_batch(const TqDequantizeJob* jobs, int n_jobs, int group_size,
                                   int bits, void* stream) {
  using namespace tq;
  if (n_jobs < 0 || (n_jobs > 0 && !jobs))
    return fail(TQ_ERR_INVALID, "dequantize_batch: bad job list");
  int rc = check_qargs(0, group_size, group_size, bits);
  if (rc) return rc;
  for (int i = 0; i < n_jobs; ++i) {
    const TqDequantizeJob& j = jobs[i];
    rc = check_job(i, j.w, j.rows, j.cols, j.codes, j.scales, j.biases, group_size, bits, false);
    if (rc) return rc;
  }
  cudaStream_t s = as_stream(stream);
  const int shift = group_size == 32 ? 5 : (group_size == 64 ? 6 : 7);
  constexpr int64_t kSpan = 32 * kWords;
  DequantizeBatch b;
  int i = 0;
  while (i < n_jobs) {
    b.n = 0;
    int64_t v = 0;
    for (; i < n_jobs && b.n < kBatchMax; ++i) {
      const TqDequantizeJob& j = jobs[i];
      const int64_t words = j.rows * j.cols * bits / 32;
      if (words == 0) continue;
      b.start[b.n] = v;
      b.words[b.n] = words;
      b.codes[b.n] = static_cast<const uint32_t*>(j.codes);
      b.scales[b.n] = static_cast<const uint16_t*>(j.scales);
      b.biases[b.n] = static_cast<const uint16_t*>(j.biases);
      b.out[b.n] = static_cast<uint16_t*>(j.w);
      v += (words + kSpan - 1) / kSpan * kSpan;  // whole warp spans
      ++b.n;
    }
    if (b.n == 0) break;
    b.start[b.n] = v;
    const int grid = grid_for(v / kWords, 256);
    if (bits == 4)
      dequantize_batch_kernel<4><<<grid, 256, 0, s>>>(b, shift);
    else
      dequantize_batch_kernel<8><<<grid, 256, 0, s>>>(b, shift);
    rc = check_cuda(cudaGetLastError(), "dequantize_batch launch");
    if (rc) return rc;
  }
  return TQ_OK;
}
