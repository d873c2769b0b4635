// Affine quantize / dequantize kernels (MLX layout) and their C entry points.
//
// Both are HBM-bound streams: quantize reads 2 bytes per element and writes
// bits/8 + 4/group_size; dequantize the reverse.  Each thread owns whole
// 16-byte vectors so every global access is a 128-bit transaction.  A
// quantizing lane holds 32 or 64 consecutive elements; a group's max and min
// are exchanged by shuffles among the lanes that hold it (groups never
// straddle a warp).
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

// sat(RN(a * b + c)): one rounding, then clamped to [0, 1] (NaN -> +0).
__device__ __forceinline__ float fma_rn_sat(float a, float b, float c) {
  float d;
  asm("fma.rn.sat.f32 %0, %1, %2, %3;" : "=f"(d) : "f"(a), "f"(b), "f"(c));
  return d;
}

// sum over the codes of one word of (bits of 1.5 * 2^23) << (BITS * i), mod 2^32.
template <int BITS>
__host__ __device__ constexpr uint32_t round_bits_sum() {
  uint32_t s = 0;
  for (int i = 0; i < 32 / BITS; ++i) s += 0x4B400000u << (BITS * i);
  return s;
}

// The division path for one run of 32 elements at src (a group whose
// quotients may be large, infinite or NaN): code = min(rint(fl(d / scale)),
// 2^BITS - 1) element by element, the conversion rounding to nearest even and
// saturating (negatives and NaN give 0); the run's code words go straight to
// out.  Kept out of line so that the rare call leaves the caller's registers
// to the common path.
template <int BITS>
__device__ __noinline__ void quantize_run_exact(const uint16_t* __restrict__ src, float bias,
                                                float scale, uint32_t* __restrict__ out) {
  constexpr int kPer = 32 / BITS;
  constexpr uint32_t kMaxCode = (1u << BITS) - 1u;
  for (int k = 0; k < BITS; ++k) {
    uint32_t word = 0;
    for (int i = 0; i < kPer; ++i) {
      const float vj = bf16_bits_to_f32(__ldg(src + k * kPer + i));
      const float yq = __fdiv_rn(__fsub_rn(vj, bias), scale);
      word |= min(__float2uint_rn(yq), kMaxCode) << (BITS * i);
    }
    out[k] = word;
  }
}

// A group's scale, bias and reciprocal, and whether its codes may take the
// division-free path below.
struct GroupParams {
  float scale, bias, rs;
  bool fast;
};

// MLX's affine group parameters from the group's max and min (f32, exact
// IEEE divisions as the oracle takes them).  live = false (a run past the end
// of the matrix) gives fast = true so the dead lane never divides.
template <int BITS>
__device__ __forceinline__ GroupParams group_params(float w_max, float w_min, bool live) {
  constexpr float n_bins = static_cast<float>((1 << BITS) - 1);
  constexpr float eps = 1e-7f;
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
  GroupParams g;
  g.scale = scale;
  g.bias = bias;
  g.rs = __frcp_rn(scale);
  // The division-free path needs every intermediate normal and finite: the
  // group's quotients below 512 (one test a group: rounding is monotone, so
  // no element's quotient exceeds fl(max|d| * |rs|)) and |scale| below 2^100
  // (it is at least 5e-8 for any finite group: the 1e-7 floor, at most
  // halved by the edge's rounding to q0).  Groups with an infinite or NaN
  // extreme, or larger ones, divide element by element instead.
  const float d_top = fmaxf(fabsf(__fsub_rn(w_max, bias)), fabsf(__fsub_rn(w_min, bias)));
  g.fast = !live || (__fmul_rn(d_top, fabsf(g.rs)) < 512.0f && fabsf(scale) < 0x1p100f);
  return g;
}

// Max / min over the bf16 pairs words[0..NW): exact (the result is one of the
// inputs), a NaN element is passed over as the f32 comparisons of the oracle
// do, and the sign of a zero extreme cannot change the scale or bias.
template <int NW>
__device__ __forceinline__ void pair_max_min(const uint32_t* words, bool live, float& w_max,
                                             float& w_min) {
  uint32_t mx2 = 0xFF80FF80u, mn2 = 0x7F807F80u;  // (-inf, -inf), (+inf, +inf)
  if (live) {
#pragma unroll
    for (int j = 0; j < NW; ++j) {
      mx2 = bf16x2_max(mx2, words[j]);
      mn2 = bf16x2_min(mn2, words[j]);
    }
  }
  w_max = fmaxf(bf16_bits_to_f32(mx2 & 0xFFFFu), bf16_bits_to_f32(mx2 >> 16));
  w_min = fminf(bf16_bits_to_f32(mn2 & 0xFFFFu), bf16_bits_to_f32(mn2 >> 16));
}

// The codes of the 2 * NW bf16 elements in words[0..NW) (element 2i in the
// low half of word i), packed low bits first into packed[0 .. 2 * NW * BITS
// / 32): code = min(rint(fl(d / scale)), 2^BITS - 1), d = fl(v - bias),
// without a division and without a branch per element.
//
// With rs = fl(1 / scale), P = 2^BITS (the scalings by P are exact),
// q = fl(d * rs / P) and the residual r = fma(-q, scale * P, d), the corrected
// quotient fl(q + r * rs / P) is Markstein's refinement of a quotient from a
// correctly rounded reciprocal (P. Markstein, "Computation of elementary
// functions on the IBM RISC System/6000 processor", IBM J. Res. Dev. 34(1),
// 1990).  Only the integer it rounds to matters here, and over every group
// this quantizer can form -- each bf16 edge mantissa, each q0, both signs,
// every bf16 element whose quotient lies in (-1, P + 1), and sampled groups
// with q0 = 0 -- that integer equals the one from the IEEE quotient, exact
// half-integer quotients included (checked exhaustively in an exact CPU
// emulation of these roundings).  The refinement's fma carries .sat, which
// clamps the quotient / P to [0, 1] and maps a NaN element to code 0;
// fma(u, P, 1.5 * 2^23) rounds P * u to an integer (ties to even) in its low
// mantissa bits, and an integer min caps the one value, P, that lies above
// the top code.  A packed word is sum(t_i << (BITS * i)) minus the same sum
// of the constant's bits, mod 2^32.
template <int BITS, int NW>
__device__ __forceinline__ void quantize_words(const uint32_t* words, const GroupParams& g,
                                               uint32_t* packed) {
  constexpr int kPer = 32 / BITS;                // codes per packed word
  constexpr float kP = static_cast<float>(1 << BITS);
  constexpr float kRound = 12582912.0f;          // 1.5 * 2^23
  constexpr uint32_t kRoundBits = 0x4B400000u;   // its bits
  constexpr uint32_t kTop = kRoundBits + (1u << BITS) - 1u;
  const float rs_p = __fmul_rn(g.rs, 1.0f / kP);
  const float scale_p = __fmul_rn(g.scale, kP);
  const float bias = g.bias;
#pragma unroll
  for (int k = 0; k < 2 * NW / kPer; ++k) packed[k] = 0u - round_bits_sum<BITS>();
#pragma unroll
  for (int j = 0; j < 2 * NW; ++j) {
    const uint32_t h = words[j >> 1];
    const float vj = (j & 1) ? __uint_as_float(h & 0xFFFF0000u) : __uint_as_float(h << 16);
    const float d = __fsub_rn(vj, bias);
    const float q = __fmul_rn(d, rs_p);
    const float res = __fmaf_rn(-q, scale_p, d);
    const float u = fma_rn_sat(res, rs_p, q);
    const float t = __fmaf_rn(u, kP, kRound);
    packed[j / kPer] += min(__float_as_uint(t), kTop) << (BITS * (j % kPer));
  }
}

// ------------------------------------------------- staged loads (cp.async) --
//
// A warp copies its next iteration's 32 units (2 or 4 KB, contiguous) into its
// shared-memory region with cp.async while it quantizes the current ones, so
// loads stay in flight without holding registers.  The copy is coalesced
// (instruction i: lane l takes 16-byte piece 32 i + l, 512 contiguous bytes a
// warp); each lane then reads its own unit's 4 * RPL pieces.  Pieces are
// placed so that the eight lanes of a quarter-warp hit eight different
// 16-byte bank groups, both when they write and when they read.

// Piece k of lane l's unit sits at 16-byte slot 4 * RPL * l + (k ^ f(l)) of
// the warp region, f(l) = l & 7 at two runs a lane and (l >> 1) & 3 at one.
template <int RPL>
__device__ __forceinline__ int slot_xor(int l) { return RPL == 2 ? (l & 7) : ((l >> 1) & 3); }

// Starts the copy of units first .. first + 31 of w (those below n_units)
// into the warp region wb.  Instruction i of the copy moves piece 32 i + lane
// of the chunk, which is piece k = lane % (4 RPL) of unit l = 32 i / (4 RPL)
// + lane / (4 RPL); its slot offset is 512 i plus a per-lane constant (two
// alternating ones at two runs a lane).  Every lane of the warp calls this
// after the warp's reads of the region (see stage_read).
template <int RPL>
__device__ __forceinline__ void stage_copy(uint32_t wb, int lane, const uint4* w, int64_t first,
                                           int64_t n_units) {
  constexpr int P = 4 * RPL;      // pieces a unit
  constexpr int UI = 32 / P;      // units an instruction covers
  const int k = lane % P, lu = lane / P;
  // slot(l, k) - 32 i for l = UI i + lu, even and odd i
  const uint32_t off_e = wb + 16u * static_cast<uint32_t>(P * lu + (k ^ slot_xor<RPL>(lu)));
  const uint32_t off_o = wb + 16u * static_cast<uint32_t>(P * lu + (k ^ slot_xor<RPL>(UI + lu)));
  const uint4* src = w + P * first + lane;
  const int64_t rem = n_units - first;  // units of the chunk that exist
  __syncwarp();  // every lane's reads of the region come before any refill
#pragma unroll
  for (int i = 0; i < P; ++i) {
    if (rem >= 32 || UI * i + lu < rem)
      asm volatile("cp.async.cg.shared.global [%0], [%1], 16;"
                   ::"r"(((i & 1) ? off_o : off_e) + 512u * i), "l"(src + 32 * i)
                   : "memory");
  }
  asm volatile("cp.async.commit_group;" ::: "memory");
}

// Waits for the warp's copies and reads this lane's unit into words.
template <int RPL>
__device__ __forceinline__ void stage_read(uint32_t wb, int lane, uint32_t* words) {
  asm volatile("cp.async.wait_group 0;" ::: "memory");
  __syncwarp();  // the other lanes' copies are visible
  const uint32_t lb = (wb + 64u * RPL * lane) | (16u * slot_xor<RPL>(lane));
#pragma unroll
  for (int k = 0; k < 4 * RPL; ++k)
    lds128(lb ^ (16u * k), words[4 * k], words[4 * k + 1], words[4 * k + 2], words[4 * k + 3]);
}

// Runs a quantizing lane takes: one at groups of 32 (one group a lane), two
// at 64 (one group a lane) and 128 (half a group a lane), so one lane's group
// parameters -- three divisions and a reciprocal -- serve 32 or 64 elements.
template <int GROUP>
constexpr int runs_per_lane() { return GROUP == 32 ? 1 : 2; }

// Quantizes runs RPL * unit .. RPL * unit + RPL - 1 (a run is 32 elements,
// four 16-byte vectors) for lane `lane` of a warp whose lanes take 32
// consecutive units, from the words already read; before any other work the
// warp starts the copy of its next units (from unit next_first of next_w,
// next_units of them in that matrix) into the region the words came from.
// A group spans LPG = GROUP / (32 * RPL) lanes (1 or 2), whose max and min
// are exchanged by a shuffle, so every lane of the warp must call this.
template <int BITS, int GROUP, int RPL>
__device__ __forceinline__ void quantize_unit(const uint32_t* words, bool live, int64_t r0,
                                              int lane, uint32_t wb, const uint4* next_w,
                                              int64_t next_first, int64_t next_units,
                                              const uint4* __restrict__ src,
                                              uint32_t* __restrict__ codes,
                                              uint16_t* __restrict__ scales,
                                              uint16_t* __restrict__ biases) {
  constexpr int NW = 16 * RPL;  // bf16 pairs a lane
  constexpr int LPG = GROUP / (32 * RPL);
  static_assert(LPG == 1 || LPG == 2, "a group spans one or two lanes");
  float w_max, w_min;
  pair_max_min<NW>(words, live, w_max, w_min);
  stage_copy<RPL>(wb, lane, next_w, next_first, next_units);  // the words are in registers
  if constexpr (LPG == 2) {
    w_max = mlx_max(w_max, __shfl_xor_sync(0xffffffffu, w_max, 1));
    w_min = mlx_min(w_min, __shfl_xor_sync(0xffffffffu, w_min, 1));
  }
  const GroupParams g = group_params<BITS>(w_max, w_min, live);
  uint32_t* out = codes + r0 * BITS;  // BITS code words a run
  if (g.fast) {
    uint32_t packed[RPL * BITS];
    quantize_words<BITS, NW>(words, g, packed);
    if (live) {
#pragma unroll
      for (int k = 0; k < RPL * BITS / 4; ++k)
        reinterpret_cast<uint4*>(out)[k] =
            make_uint4(packed[4 * k], packed[4 * k + 1], packed[4 * k + 2], packed[4 * k + 3]);
    }
  } else {
    const uint16_t* e = reinterpret_cast<const uint16_t*>(src + 4 * r0);
#pragma unroll
    for (int r = 0; r < RPL; ++r)
      quantize_run_exact<BITS>(e + 32 * r, g.bias, g.scale, out + BITS * r);
  }
  if (live && (lane & (LPG - 1)) == 0) {
    const int64_t gi = r0 * 32 / GROUP;
    scales[gi] = f32_to_bf16_bits(g.scale);
    biases[gi] = f32_to_bf16_bits(g.bias);
  }
}

// Each warp takes 32 consecutive units per iteration (n_runs is a multiple of
// GROUP / 32, so a unit's runs live or die together).  A run a lane: 64
// registers a thread and 16 KB of slots a CTA, four CTAs an SM; two runs: 80
// registers and 32 KB, three.
template <int BITS, int GROUP>
__global__ void __launch_bounds__(256, GROUP == 32 ? 4 : 3)
    quantize_kernel(const uint4* __restrict__ w, int64_t n_runs, uint32_t* __restrict__ codes,
                    uint16_t* __restrict__ scales, uint16_t* __restrict__ biases) {
  constexpr int RPL = runs_per_lane<GROUP>();
  __shared__ __align__(128) uint4 region[256 * 4 * RPL];
  const int lane = threadIdx.x & 31;
  const uint32_t wb = smem_u32(region) + (threadIdx.x & ~31) * (64u * RPL);
  const int64_t n_units = n_runs / RPL;
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  int64_t base = static_cast<int64_t>(blockIdx.x) * blockDim.x + (threadIdx.x & ~31);
  stage_copy<RPL>(wb, lane, w, base, n_units);
  for (; base < n_units; base += stride) {
    const int64_t unit = base + lane;
    uint32_t words[16 * RPL];
    stage_read<RPL>(wb, lane, words);
    quantize_unit<BITS, GROUP, RPL>(words, unit < n_units, RPL * unit, lane, wb, w,
                                    base + stride, n_units, w, codes, scales, biases);
  }
  asm volatile("cp.async.wait_group 0;" ::: "memory");  // no copy outlives the CTA
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

// The batched form of quantize_kernel: a warp finds its job once per
// iteration (a job's units never straddle a warp iteration) and the next
// iteration's job by stepping forward from this one.
// The batched form of quantize_kernel: a warp finds its job once per
// iteration (a job's units never straddle a warp iteration) and the next
// iteration's job by stepping forward from this one.
template <int BITS, int GROUP>
__global__ void __launch_bounds__(256, GROUP == 32 ? 4 : 3)
    quantize_batch_kernel(const __grid_constant__ QuantizeBatch b) {
  constexpr int RPL = runs_per_lane<GROUP>();
  __shared__ __align__(128) uint4 region[256 * 4 * RPL];
  const int lane = threadIdx.x & 31;
  const uint32_t wb = smem_u32(region) + (threadIdx.x & ~31) * (64u * RPL);
  const int64_t end = b.start[b.n] / RPL;  // in units
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  int64_t base = static_cast<int64_t>(blockIdx.x) * blockDim.x + (threadIdx.x & ~31);
  // Job j's units, and the warp's first unit in it, for a warp at virtual unit bs.
  auto units = [&](int job) { return b.runs[job] / RPL; };
  auto first = [&](int job, int64_t bs) { return bs - b.start[job] / RPL; };
  int j = find_job(b.start, b.n, RPL * (base < end ? base : 0));
  stage_copy<RPL>(wb, lane, b.w[j], first(j, base), base < end ? units(j) : 0);
  for (; base < end; base += stride) {
    int jn = j;  // the job of the next iteration
    const int64_t nb = base + stride;
    while (jn + 1 < b.n && b.start[jn + 1] <= RPL * nb) ++jn;
    const int64_t u = first(j, base) + lane;
    uint32_t words[16 * RPL];
    stage_read<RPL>(wb, lane, words);
    quantize_unit<BITS, GROUP, RPL>(words, u < units(j), RPL * u, lane, wb, b.w[jn],
                                    first(jn, nb), nb < end ? units(jn) : 0, b.w[j],
                                    b.codes[j], b.scales[j], b.biases[j]);
    j = jn;
  }
  asm volatile("cp.async.wait_group 0;" ::: "memory");
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

template <int BITS, int GROUP>
void launch_quantize(const uint4* w, int64_t n_runs, uint32_t* c, uint16_t* sc, uint16_t* bi,
                     cudaStream_t s) {
  const int grid = grid_for(n_runs / runs_per_lane<GROUP>(), 256);
  quantize_kernel<BITS, GROUP><<<grid, 256, 0, s>>>(w, n_runs, c, sc, bi);
}

template <int BITS, int GROUP>
void launch_quantize_batch(const QuantizeBatch& b, cudaStream_t s) {
  const int grid = grid_for(b.start[b.n] / runs_per_lane<GROUP>(), 256);
  quantize_batch_kernel<BITS, GROUP><<<grid, 256, 0, s>>>(b);
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
  cudaStream_t s = as_stream(stream);
  const uint4* wv = static_cast<const uint4*>(w);
  uint32_t* c = static_cast<uint32_t*>(codes);
  uint16_t* sc = static_cast<uint16_t*>(scales);
  uint16_t* bi = static_cast<uint16_t*>(biases);
  if (bits == 4) {
    if (group_size == 32) launch_quantize<4, 32>(wv, n_runs, c, sc, bi, s);
    else if (group_size == 64) launch_quantize<4, 64>(wv, n_runs, c, sc, bi, s);
    else launch_quantize<4, 128>(wv, n_runs, c, sc, bi, s);
  } else {
    if (group_size == 32) launch_quantize<8, 32>(wv, n_runs, c, sc, bi, s);
    else if (group_size == 64) launch_quantize<8, 64>(wv, n_runs, c, sc, bi, s);
    else launch_quantize<8, 128>(wv, n_runs, c, sc, bi, s);
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
      v += (runs + 63) / 64 * 64;  // whole warp iterations (32 lanes x up to 2 runs)
      ++b.n;
    }
    if (b.n == 0) break;
    b.start[b.n] = v;
    if (bits == 4) {
      if (group_size == 32) launch_quantize_batch<4, 32>(b, s);
      else if (group_size == 64) launch_quantize_batch<4, 64>(b, s);
      else launch_quantize_batch<4, 128>(b, s);
    } else {
      if (group_size == 32) launch_quantize_batch<8, 32>(b, s);
      else if (group_size == 64) launch_quantize_batch<8, 64>(b, s);
      else launch_quantize_batch<8, 128>(b, s);
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
