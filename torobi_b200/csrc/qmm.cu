// quantized_matmul on the 5th-generation tensor cores (tcgen05 / TMEM), with
// the LoRA up-projection and the linear's bias fused into the accumulator.
//
// Each CTA (one per SM, persistent) computes 128 x BN tiles of the output
// TRANSPOSED in tensor memory:
// the UMMA's M side (128 TMEM lanes) is the weight's output features and its
// N side (BN columns) is the tokens.  Putting the quantized weight on the M
// side halves the dequantization work per MMA flop against the other
// orientation (a 128-row weight tile feeds a 128 x BN MMA instead of a BN-row
// tile feeding a BN x 128 one).
//
//   warp 0      TMA producer: activation tile (bf16, 128B swizzle), the raw
//               packed-code tile and the group scale/bias tiles of each stage;
//               the LoRA tiles once per output tile.
//   warp 1      TMEM allocator and the single UMMA-issuing thread.
//   warps 2-9   dequantizers (two per scheduler): packed codes (shared) -> bf16
//               weight tile in the UMMA canonical 128B-swizzled layout,
//               w = RNE(scale*q + bias); each thread owns 32 codes of a row.
//   warps 10-13 epilogue: TMEM -> registers -> (+ bias) -> bf16 -> global,
//               overlapped with the next tile (two TMEM accumulators).
//
// transpose (linear forward, y = x . W^T): the reduction runs along W's packed
// axis, so the dequantized tile is K-major.  Backward wrt x (y = dy . W): the
// reduction runs along W's rows and the output along its packed axis, so the
// same tile is written MN-major -- the same kernel with the roles swapped.
//
// The LoRA branch: lora_down (the [m, rank] scaled down-projection) and
// lora_up (B [n, rank] forward, A [rank, k] backward) are loaded once and one
// extra K=16 UMMA adds lora_up . lora_down^T into the same accumulator before
// the main loop, so base + adapter leave TMEM with one rounding to bf16.
#include <cuda_bf16.h>

#include <cstdlib>
#include <mutex>

#include "tq_ptx.cuh"
#include "tq_runtime.h"

namespace tq {
namespace {

constexpr int kBM = 128;        // weight-side rows per tile (UMMA M)
constexpr int kBK = 64;         // reduction elements per pipeline stage
constexpr int kThreads = 448;   // 14 warps
constexpr int kDqWarps = 8;     // dequantizing warps (two per scheduler)
constexpr int kSmemLimit = 232448;
constexpr int kRing = 4;        // fallback path: scale/bias register ring (k-steps)

// Shared-memory plan.  Two rings:
//   stage ring (S deep, filled by TMA): activation tile, packed codes and --
//     when the scale rows are 16-byte aligned (STMA) -- the group scale and
//     bias tiles the step needs;
//   dequantized-weight ring (A deep, written by the dequantizing warps).
// Splitting them lets the TMA run S stages ahead while only A bf16 weight
// tiles are held.
template <int BITS, bool TRANS, int BN, bool STMA>
struct Cfg {
  static constexpr int X_BYTES = BN * kBK * 2;
  static constexpr int A_BYTES = kBM * kBK * 2;
  static constexpr int C_BYTES = kBM * kBK * BITS / 8;
  // Scale (and bias) tile: 8 groups (16 bytes, the TMA minimum) x the rows
  // the step touches: 128 output features forward, 64 weight rows backward.
  static constexpr int SC_ROWS = TRANS ? kBM : kBK;
  static constexpr int SC_BYTES = STMA ? SC_ROWS * 16 : 0;
  static constexpr int STAGE_BYTES = X_BYTES + C_BYTES + 2 * SC_BYTES;
  static constexpr int LUP_BYTES = kBM * 16 * 2;            // [128 x 16] bf16
  static constexpr int LDN_BYTES = BN * 16 * 2;             // [BN x 16] bf16
  static constexpr int LORA_BYTES = ((LUP_BYTES + LDN_BYTES + 1023) / 1024) * 1024;
  static constexpr int BAR_BYTES = 512;
  // Epilogue staging: per epilogue warp two [32 tokens x 32 features] bf16
  // buffers, written from TMEM and stored to y by TMA.
  static constexpr int EPI_CHUNK = 32 * 32 * 2;
  static constexpr int EPI_BYTES = 4 * 2 * EPI_CHUNK;
  static constexpr int FIXED = 1024 + LORA_BYTES + EPI_BYTES + BAR_BYTES;
  // Dequantizing groups on alternate k-steps: with scale tiles, two for the
  // large token tiles (the MMA is long) and four for the small ones (the
  // MMA is short and the dequantization's latency is the whole step); one
  // dequantized-tile buffer more than groups.
  static constexpr int DQ_GROUPS = !STMA ? 1 : (BN <= 64 ? 4 : 2);
  static constexpr int A_WANT = DQ_GROUPS == 4 ? 5 : 3;
  static constexpr int stages_with(int a) { return (kSmemLimit - FIXED - a * A_BYTES) / STAGE_BYTES; }
  static constexpr int A_BUFS = stages_with(A_WANT) >= 4 ? A_WANT : (stages_with(3) >= 4 ? 3 : 2);
  static constexpr int STAGES_RAW = (kSmemLimit - FIXED - A_BUFS * A_BYTES) / STAGE_BYTES;
  static constexpr int STAGES = STAGES_RAW > 8 ? 8 : STAGES_RAW;
  static constexpr int SMEM = FIXED + A_BUFS * A_BYTES + STAGES * STAGE_BYTES;
  static constexpr int ACC_COLS = BN < 32 ? 32 : BN;        // one accumulator
  static constexpr int TMEM_COLS = 2 * ACC_COLS;            // double-buffered
  static_assert(STAGES >= 2, "shared memory too small for two stages");
  static_assert(SMEM <= kSmemLimit, "shared memory budget");
  static_assert(8 * (2 * STAGES + 2 * A_BUFS + 6) + 8 <= BAR_BYTES, "barrier area");
  static_assert(STAGE_BYTES % 1024 == 0, "stage tiles stay 1024-byte aligned");
};

struct Params {
  const uint16_t* scales;
  const uint16_t* biases;
  const uint16_t* bias_vec;  // [n_out] bf16 or null
  uint16_t* y;               // [m, n_out] bf16
  int m;
  int n_out;                 // output features of this GEMM
  int k_red;                 // reduction length
  int w_rows;                // rows of the stored weight
  int groups_per_row;        // w_cols / group_size
  int group_shift;
  int lora_rank;             // 0, 8 or 16
  int tiles_n;               // output tiles along n_out
  int tiles_total;           // tiles_n * tiles along m
  int splits;                // k-splits per tile (split-K); 1 = none
  int k_steps_per_split;     // k-steps of every split but maybe the last
  float* ws;                 // splits > 1: f32 partials [splits, m, n_out]
  int tma_y;                 // the bf16 output goes out through TMA stores (tm_y)
  int acc;                   // add into y: y = RNE(RNE(result) + y)
  int keep_weights;          // weight loads marked L2 evict_last (else evict_normal)
  int* status;
};

__device__ __forceinline__ uint16_t ldg_u16(const uint16_t* p) {
  return __ldg(reinterpret_cast<const unsigned short*>(p));
}

__device__ __forceinline__ uint32_t lds_u16(uint32_t addr) {
  uint16_t v;
  asm volatile("ld.shared.u16 %0, [%1];" : "=h"(v) : "r"(addr) : "memory");
  return v;
}

// Groups of one k-step for dequantizing thread t (0..127): first and second
// (group 32 splits a 64-wide step in two), and the weight row they sit on.
// The group one dequantizing thread t (0..255) needs for one k-step, and the
// weight row it sits on.  Forward: t covers row t % 128, k half t / 128 (32
// codes, one group for every group size).  Backward: t covers weight row
// k0 + t % 64 and output quarter t / 64 (32 outputs, one group).
struct GroupCoord {
  int row;       // weight row
  uint32_t g;    // group along the weight row
  bool rv;       // row inside the weight
};

template <bool TRANS>
__device__ __forceinline__ GroupCoord group_coord(const Params& p, int t, int out0, int k0) {
  GroupCoord c;
  if constexpr (TRANS) {
    c.row = out0 + (t & 127);  // weight row = output feature
    c.g = static_cast<uint32_t>(k0 + 32 * (t >> 7)) >> p.group_shift;
    c.rv = c.row < p.n_out;
  } else {
    c.row = k0 + (t & 63);  // weight row = reduction index
    c.g = static_cast<uint32_t>(out0 + 32 * (t >> 6)) >> p.group_shift;
    c.rv = c.row < p.w_rows;
  }
  return c;
}

// First group of the 8-group window a step's TMA scale tile covers (x of the
// box, a multiple of 8 so the copy starts on a 16-byte boundary).
template <bool TRANS>
__device__ __forceinline__ int scale_window(const Params& p, int out0, int k0) {
  return static_cast<int>((static_cast<uint32_t>(TRANS ? k0 : out0) >> p.group_shift) & ~7u);
}

// Fallback path (scale rows not 16-byte aligned): raw bits loaded by the
// dequantizing thread kRing-1 steps ahead; bit 16 flags out-of-range.
struct GroupRaw {
  uint32_t s, b;
};

template <bool TRANS>
__device__ __forceinline__ GroupRaw load_groups(const Params& p, int t, int out0, int k0) {
  const GroupCoord c = group_coord<TRANS>(p, t, out0, k0);
  const uint32_t gpr = static_cast<uint32_t>(p.groups_per_row);
  const bool v = c.rv && c.g < gpr;
  const size_t i = v ? static_cast<size_t>(c.row) * gpr + c.g : 0;
  GroupRaw g;
  g.s = ldg_u16(p.scales + i) | (v ? 0u : 0x10000u);
  g.b = ldg_u16(p.biases + i);
  return g;
}

__device__ __forceinline__ uint32_t widen(uint32_t raw, uint32_t flag_from) {
  return (flag_from & 0x10000u) ? 0u : bf16_dup(static_cast<uint16_t>(raw));
}

// Packed codes (shared, as TMA left them) -> bf16 weight tile in the UMMA's
// 128B-swizzled canonical layout.  Virtual dequantizing thread v (0..255) owns
// 32 codes of one weight row: load_run fetches them (4 words at 4 bits, 8 at
// 8), store_run dequantizes them with the group's bf16 scale/bias pair s2/b2
// and writes them.  Split so that a thread can issue the loads of two runs
// before the stores of either (the shared-memory accesses are ordered asm).
template <int BITS, bool TRANS>
__device__ __forceinline__ void load_run(uint32_t cb, int v, uint32_t (&w)[BITS]) {
  if constexpr (TRANS) {
    // K-major: row r = output feature, k half hh.
    const int r = v & 127;
    const int hh = v >> 7;
    if constexpr (BITS == 4) {
      lds128(cb + swz<32>(r * 32 + hh * 16), w[0], w[1], w[2], w[3]);
    } else {
#pragma unroll
      for (int c = 0; c < 2; ++c)
        lds128(cb + swz<64>(r * 64 + (2 * hh + c) * 16), w[4 * c], w[4 * c + 1], w[4 * c + 2],
               w[4 * c + 3]);
    }
  } else {
    // MN-major: kr = reduction row (0..63), qq = output quarter (32 outputs).
    const int kr = v & 63;
    const int qq = v >> 6;
    if constexpr (BITS == 4) {
      lds128(cb + swz<64>(kr * 64 + qq * 16), w[0], w[1], w[2], w[3]);
    } else {
#pragma unroll
      for (int c = 0; c < 2; ++c)
        lds128(cb + swz<128>(kr * 128 + (2 * qq + c) * 16), w[4 * c], w[4 * c + 1],
               w[4 * c + 2], w[4 * c + 3]);
    }
  }
}

template <int BITS, bool TRANS>
__device__ __forceinline__ void store_run(uint32_t ab, int v, const uint32_t (&w)[BITS],
                                          uint32_t s2, uint32_t b2) {
  uint32_t base;
  int j0, sw;
  if constexpr (TRANS) {
    // Chunks 4hh..4hh+3 of row r's eight 16-byte chunks.
    const int r = v & 127;
    base = ab + r * 128;
    j0 = 4 * (v >> 7);
    sw = r & 7;
  } else {
    // Atoms of 64 outputs x 8 reduction rows, 8 K-groups per 64-output block.
    const int kr = v & 63;
    const int qq = v >> 6;
    base = ab + (qq >> 1) * 8192 + (kr >> 3) * 1024 + (kr & 7) * 128;
    j0 = (qq & 1) * 4;
    sw = kr & 7;
  }
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    uint32_t o[4];
    if constexpr (BITS == 4) {
      dequant_u4x8(w[j], s2, b2, o);
    } else {
      uint32_t lo[2], hi[2];
      dequant_u8x4(w[2 * j], s2, b2, lo);
      dequant_u8x4(w[2 * j + 1], s2, b2, hi);
      o[0] = lo[0];
      o[1] = lo[1];
      o[2] = hi[0];
      o[3] = hi[1];
    }
    sts128(base + (((j0 + j) ^ sw) << 4), o[0], o[1], o[2], o[3]);
  }
}

template <int BITS, bool TRANS>
__device__ __forceinline__ void dequant_tile(uint32_t cb, uint32_t ab, int t, uint32_t s2,
                                             uint32_t b2) {
  uint32_t w[BITS];
  load_run<BITS, TRANS>(cb, t, w);
  store_run<BITS, TRANS>(ab, t, w, s2, b2);
}

// Byte offset of virtual thread v's group scale (and bias) in the stage's
// 8-group scale tile.
template <bool TRANS>
__device__ __forceinline__ uint32_t scale_off(const Params& p, int v, int out0, int k0) {
  const GroupCoord gc = group_coord<TRANS>(p, v, out0, k0);
  const uint32_t gx = static_cast<uint32_t>(scale_window<TRANS>(p, out0, k0));
  const uint32_t row = TRANS ? static_cast<uint32_t>(v & 127) : static_cast<uint32_t>(v & 63);
  return row * 16 + (gc.g - gx) * 2;
}

// Scale-tile path: one thread of a group of 256/G dequantizes virtual
// threads tt + i * 256/G (i < G) of a k-step, every load issued before the
// first store.
template <int BITS, bool TRANS, int G>
__device__ __forceinline__ void dequant_runs(const Params& p, uint32_t sc, uint32_t bi,
                                             uint32_t cb, uint32_t ab, int tt, int out0, int k0) {
  constexpr int kStride = 256 / G;
  uint32_t off[G], w[G][BITS], sv[G], bv[G];
#pragma unroll
  for (int i = 0; i < G; ++i) off[i] = scale_off<TRANS>(p, tt + i * kStride, out0, k0);
#pragma unroll
  for (int i = 0; i < G; ++i) load_run<BITS, TRANS>(cb, tt + i * kStride, w[i]);
#pragma unroll
  for (int i = 0; i < G; ++i) {
    sv[i] = lds_u16(sc + off[i]);
    bv[i] = lds_u16(bi + off[i]);
  }
#pragma unroll
  for (int i = 0; i < G; ++i)
    store_run<BITS, TRANS>(ab, tt + i * kStride, w[i], bf16_dup(static_cast<uint16_t>(sv[i])),
                           bf16_dup(static_cast<uint16_t>(bv[i])));
}


// Persistent: CTA b takes tiles b, b + grid, ...; tile t covers output
// features (t % tiles_n) * 128 and tokens (t / tiles_n) * BN.
template <int BITS, bool TRANS, int BN, bool STMA>
__global__ void __launch_bounds__(kThreads, 1)
    qmm_kernel(const __grid_constant__ CUtensorMap tm_x, const __grid_constant__ CUtensorMap tm_c,
               const __grid_constant__ CUtensorMap tm_lup, const __grid_constant__ CUtensorMap tm_ldn,
               const __grid_constant__ CUtensorMap tm_sc, const __grid_constant__ CUtensorMap tm_bi,
               const __grid_constant__ CUtensorMap tm_y, const Params p) {
  using C = Cfg<BITS, TRANS, BN, STMA>;
  constexpr int S = C::STAGES;
  constexpr int A = C::A_BUFS;
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw = smem_u32(smem_raw);
  const uint32_t base = (raw + 1023u) & ~1023u;
  uint8_t* const gbase = smem_raw + (base - raw);

  const uint32_t lup = base;                                  // LoRA up tile
  const uint32_t ldn = base + C::LUP_BYTES;                   // LoRA down tile
  const uint32_t epi = base + C::LORA_BYTES;                  // epilogue staging
  const uint32_t abufs = epi + C::EPI_BYTES;                  // dequantized-weight ring
  const uint32_t stages = abufs + A * C::A_BYTES;             // TMA stage ring
  auto a_s = [&](int a) { return abufs + a * C::A_BYTES; };
  auto x_s = [&](int s) { return stages + s * C::STAGE_BYTES; };
  auto c_s = [&](int s) { return stages + s * C::STAGE_BYTES + C::X_BYTES; };
  auto sc_s = [&](int s) { return stages + s * C::STAGE_BYTES + C::X_BYTES + C::C_BYTES; };
  auto bi_s = [&](int s) { return sc_s(s) + C::SC_BYTES; };
  const uint32_t bars = stages + S * C::STAGE_BYTES;
  auto full_b = [&](int s) { return bars + 8u * s; };
  auto empty_b = [&](int s) { return bars + 8u * (S + s); };
  auto aready_b = [&](int a) { return bars + 8u * (2 * S + a); };
  auto aempty_b = [&](int a) { return bars + 8u * (2 * S + A + a); };
  const uint32_t lora_full = bars + 8u * (2 * S + 2 * A);
  const uint32_t lora_empty = lora_full + 8u;
  auto acc_full = [&](int b) { return lora_full + 16u + 8u * b; };
  auto acc_empty = [&](int b) { return lora_full + 32u + 8u * b; };
  const uint32_t tmem_slot = lora_full + 48u;
  volatile uint32_t* tmem_slot_ptr =
      reinterpret_cast<volatile uint32_t*>(gbase + (tmem_slot - base));

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int num_k = (p.k_red + kBK - 1) / kBK;
  const bool has_lora = p.lora_rank > 0;
  const int lora_chunks = p.lora_rank / 8;
  // Work units: (tile, k-split) pairs, unit u = tile * splits + split, so a
  // tile's splits run side by side.  CTA b takes units b, b + grid, ...
  const int units_total = p.tiles_total * p.splits;
  const int my_tiles = static_cast<int>(blockIdx.x) < units_total
                           ? (units_total - 1 - static_cast<int>(blockIdx.x)) / gridDim.x + 1
                           : 0;
  auto unit_tile = [&](int lt) {
    return static_cast<int>((blockIdx.x + lt * gridDim.x) / p.splits);
  };
  auto unit_split = [&](int lt) {
    return static_cast<int>((blockIdx.x + lt * gridDim.x) % p.splits);
  };
  auto tile_out0 = [&](int lt) { return (unit_tile(lt) % p.tiles_n) * kBM; };
  auto tile_m0 = [&](int lt) { return (unit_tile(lt) / p.tiles_n) * BN; };
  auto k_first = [&](int lt) { return unit_split(lt) * p.k_steps_per_split; };
  auto k_count = [&](int lt) {
    const int b = k_first(lt);
    const int e = b + p.k_steps_per_split < num_k ? b + p.k_steps_per_split : num_k;
    return e - b;
  };
  // Only split 0 of a tile adds the LoRA branch.
  auto unit_lora = [&](int lt) { return has_lora && unit_split(lt) == 0; };

  // Zero the LoRA tiles once: with rank 8 the second K-chunk stays zero.
  if (has_lora) {
    for (int i = threadIdx.x; i < C::LORA_BYTES / 16; i += kThreads)
      sts128(base + 16u * i, 0u, 0u, 0u, 0u);
    fence_proxy_async_smem();
  }
  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(full_b(s), 1);
      mbar_init(empty_b(s), 1);
    }
    for (int a = 0; a < A; ++a) {
      mbar_init(aready_b(a), kDqWarps / C::DQ_GROUPS);
      mbar_init(aempty_b(a), 1);
    }
    mbar_init(lora_full, 1);
    mbar_init(lora_empty, 1);
    for (int b = 0; b < 2; ++b) {
      mbar_init(acc_full(b), 1);
      mbar_init(acc_empty(b), 4);
    }
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, C::TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot_ptr;
  // Signalled only once this CTA holds its tensor memory: a dependent
  // kernel's CTA placed on this SM may then wait for it, never hold it.
  griddep_launch_dependents();
  griddep_wait();

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (elect_one_sync()) {
      tma_prefetch_desc(&tm_x);
      // codes and scales: reused by every token tile
      const uint64_t keep = p.keep_weights ? l2_evict_last() : l2_evict_normal();
      tma_prefetch_desc(&tm_c);
      if constexpr (STMA) {
        tma_prefetch_desc(&tm_sc);
        tma_prefetch_desc(&tm_bi);
      }
      if (has_lora) {
        tma_prefetch_desc(&tm_lup);
        tma_prefetch_desc(&tm_ldn);
      }
      bool ok = true;
      int it = 0;
      int lora_loads = 0;
      for (int lt = 0; lt < my_tiles && ok; ++lt) {
        const int out0 = tile_out0(lt), m0 = tile_m0(lt);
        if (unit_lora(lt)) {
          ok = mbar_wait(lora_empty, (lora_loads & 1) ^ 1, p.status);
          if (!ok) break;
          mbar_arrive_expect_tx(lora_full, lora_chunks * (kBM * 16 + BN * 16));
          for (int ch = 0; ch < lora_chunks; ++ch) {
            if constexpr (TRANS) {
              // B [n_out, rank]: K-major, no swizzle; chunk = 8 rank columns.
              tma_load_2d(lup + ch * kBM * 16, &tm_lup, lora_full, ch * 8, out0);
            } else {
              // A [rank, k]: MN-major 128B-swizzled atoms (64 k x 8 rank).
              tma_load_2d(lup + ch * 1024, &tm_lup, lora_full, out0, ch * 8);
              tma_load_2d(lup + 2048 + ch * 1024, &tm_lup, lora_full, out0 + 64, ch * 8);
            }
            tma_load_2d(ldn + ch * BN * 16, &tm_ldn, lora_full, ch * 8, m0);
          }
          ++lora_loads;
        }
        const int kb = k_first(lt), ke = kb + k_count(lt);
        for (int kk = kb; kk < ke; ++kk, ++it) {
          const int s = it % S;
          const uint32_t ph = (it / S) & 1;
          ok = mbar_wait(empty_b(s), ph ^ 1, p.status);
          if (!ok) break;
          const int k0 = kk * kBK;
          mbar_arrive_expect_tx(full_b(s), C::X_BYTES + C::C_BYTES + 2 * C::SC_BYTES);
          tma_load_2d(x_s(s), &tm_x, full_b(s), k0, m0);
          if constexpr (TRANS)
            tma_load_2d_hint(c_s(s), &tm_c, full_b(s), k0 * BITS / 32, out0, keep);
          else
            tma_load_2d_hint(c_s(s), &tm_c, full_b(s), out0 * BITS / 32, k0, keep);
          if constexpr (STMA) {
            const int gx = scale_window<TRANS>(p, out0, k0);
            const int gy = TRANS ? out0 : k0;
            tma_load_2d_hint(sc_s(s), &tm_sc, full_b(s), gx, gy, keep);
            tma_load_2d_hint(bi_s(s), &tm_bi, full_b(s), gx, gy, keep);
          }
        }
      }
      // Never leave a copy in flight: wait for the last phase of every stage.
      for (int i = it - S < 0 ? 0 : it - S; i < it; ++i)
        mbar_wait(full_b(i % S), (i / S) & 1, p.status);
      if (lora_loads > 0) mbar_wait(lora_full, (lora_loads - 1) & 1, p.status);
    }
  } else if (warp == 1) {
    // ---------------------------------------------------------- MMA issuer
    if (elect_one_sync()) {
      constexpr uint32_t idesc = make_idesc_bf16(kBM, BN, !TRANS, false);
      bool ok = true;
      int it = 0;
      int lora_uses = 0;
      for (int lt = 0; lt < my_tiles && ok; ++lt) {
        const int buf = lt & 1;
        ok = mbar_wait(acc_empty(buf), ((lt >> 1) & 1) ^ 1, p.status);
        if (!ok) break;
        tc_fence_after();
        const uint32_t d = tmem + buf * C::ACC_COLS;
        uint32_t acc = 0;
        if (unit_lora(lt)) {
          ok = mbar_wait(lora_full, lora_uses & 1, p.status);
          ++lora_uses;
          if (!ok) break;
          tc_fence_after();
          uint64_t adesc;
          if constexpr (TRANS)
            adesc = make_sdesc(lup, kBM * 16, 128, kSwNone);  // LBO: K chunk, SBO: 8-row group
          else
            adesc = make_sdesc(lup, 2048, 1024, kSw128);     // LBO: MN atom, SBO: K group
          const uint64_t bdesc = make_sdesc(ldn, BN * 16, 128, kSwNone);
          umma_bf16(d, adesc, bdesc, idesc, 0);
          umma_commit(lora_empty);
          acc = 1;
        }
        const int kc = k_count(lt);
        for (int kk = 0; kk < kc; ++kk, ++it) {
          const int s = it % S;
          const int a = it % A;
          ok = mbar_wait(full_b(s), (it / S) & 1, p.status) &&
               mbar_wait(aready_b(a), (it / A) & 1, p.status);
          if (!ok) break;
          tc_fence_after();
#pragma unroll
          for (int k4 = 0; k4 < kBK / 16; ++k4) {
            uint64_t adesc;
            if constexpr (TRANS)
              adesc = make_sdesc(a_s(a) + k4 * 32, 16, 1024, kSw128);
            else
              adesc = make_sdesc(a_s(a) + k4 * 2048, 8192, 1024, kSw128);
            const uint64_t bdesc = make_sdesc(x_s(s) + k4 * 32, 16, 1024, kSw128);
            umma_bf16(d, adesc, bdesc, idesc, acc);
            acc = 1;
          }
          umma_commit(empty_b(s));
          umma_commit(aempty_b(a));
        }
        umma_commit(acc_full(buf));
      }
      // Nothing may outlive the CTA's TMEM: the last commit covers every UMMA.
      if (my_tiles > 0)
        mbar_wait(acc_full((my_tiles - 1) & 1), ((my_tiles - 1) >> 1) & 1, p.status);
    }
  } else if (warp < 2 + kDqWarps) {
    // ---------------------------------------------------- dequant warps
    const int t = threadIdx.x - 64;  // 0..255
    // Split-K is only used with STMA, so on the fallback path every unit has
    // num_k steps and a flat step index maps back to (unit, k-step).
    const int total = my_tiles * num_k;
    auto coords = [&](int j, int& out0, int& k0) {
      const int lt = j / num_k;
      out0 = tile_out0(lt);
      k0 = (j - lt * num_k) * kBK;
    };
    auto step = [&](int j, int out0, int k0, uint32_t s2, uint32_t b2) -> bool {
      const int s = j % S;
      const int a = j % A;
      if (!mbar_wait(full_b(s), (j / S) & 1, p.status)) return false;
      if (!mbar_wait(aempty_b(a), ((j / A) & 1) ^ 1, p.status)) return false;
      dequant_tile<BITS, TRANS>(c_s(s), a_s(a), t, s2, b2);
      fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) mbar_arrive(aready_b(a));
      return true;
    };
    if constexpr (STMA) {
      constexpr int G = C::DQ_GROUPS;
      const int grp = t / (256 / G);
      const int tt = t % (256 / G);
      int j = 0;
      bool ok = true;
      for (int lt = 0; lt < my_tiles && ok; ++lt) {
        const int out0 = tile_out0(lt), kb = k_first(lt), kc = k_count(lt);
        for (int kk = 0; kk < kc && ok; ++kk, ++j) {
          if ((j % G) != grp) continue;
          const int s = j % S;
          const int a = j % A;
          const int k0 = (kb + kk) * kBK;
          ok = mbar_wait(full_b(s), (j / S) & 1, p.status) &&
               mbar_wait(aempty_b(a), ((j / A) & 1) ^ 1, p.status);
          if (!ok) break;
          dequant_runs<BITS, TRANS, G>(p, sc_s(s), bi_s(s), c_s(s), a_s(a), tt, out0, k0);
          fence_proxy_async_smem();
          __syncwarp();
          if (lane == 0) mbar_arrive(aready_b(a));
        }
      }
    } else {
      GroupRaw ring[kRing];
#pragma unroll
      for (int u = 0; u < kRing - 1; ++u) {
        if (u < total) {
          int out0, k0;
          coords(u, out0, k0);
          ring[u] = load_groups<TRANS>(p, t, out0, k0);
        }
      }
      bool ok = true;
      for (int j0 = 0; j0 < total && ok; j0 += kRing) {
#pragma unroll
        for (int u = 0; u < kRing; ++u) {
          const int j = j0 + u;
          if (j < total && ok) {
            if (j + kRing - 1 < total) {
              int out0, k0;
              coords(j + kRing - 1, out0, k0);
              ring[(u + kRing - 1) % kRing] = load_groups<TRANS>(p, t, out0, k0);
            }
            const GroupRaw& g = ring[u];
            int out0, k0;
            coords(j, out0, k0);
            ok = step(j, out0, k0, widen(g.s, g.s), widen(g.b, g.s));
          }
        }
      }
    }
  } else {
    // ------------------------------------------------------------ epilogue
    const int q = warp & 3;              // TMEM lane quadrant this warp may read
    const int r = q * 32 + lane;         // output feature within the tile
    // With tma_y, each 32-token chunk of this warp's 32 features goes through
    // one of its two staging buffers ([token][feature] bf16) and out by a TMA
    // store, clipped at y's edges; one bulk group per chunk (empty when the
    // box lies wholly past y) keeps "all but the newest group have read"
    // covering the buffer about to be reused.
    const uint32_t stage_w = epi + static_cast<uint32_t>(q) * 2 * C::EPI_CHUNK;
    if (p.tma_y && lane == 0) tma_prefetch_desc(&tm_y);
    int chunk = 0;
    bool ok = true;
    for (int lt = 0; lt < my_tiles && ok; ++lt) {
      const int buf = lt & 1;
      ok = mbar_wait(acc_full(buf), (lt >> 1) & 1, p.status);
      tc_fence_after();
      const int out0 = tile_out0(lt), m0 = tile_m0(lt);
      const int og = out0 + r;
      float bias = 0.0f;
      if (p.bias_vec && og < p.n_out)
        bias = __uint_as_float(uint32_t(ldg_u16(p.bias_vec + og)) << 16);
      const uint32_t d = tmem + buf * C::ACC_COLS + (static_cast<uint32_t>(q * 32) << 16);
#pragma unroll 1
      for (int c0 = 0; c0 < BN; c0 += 32) {
        uint32_t v[32];
        tmem_ld_32x32b_x32(d + c0, v);
        tmem_ld_wait();
        if (ok && p.tma_y) {
          const uint32_t sb = stage_w + static_cast<uint32_t>(chunk & 1) * C::EPI_CHUNK;
          ++chunk;
          if (lane == 0) tma_store_wait_read1();
          __syncwarp();
#pragma unroll
          for (int j = 0; j < 32; ++j)
            sts16(sb + j * 64 + lane * 2,
                  __bfloat16_as_ushort(__float2bfloat16_rn(__uint_as_float(v[j]) + bias)));
          fence_proxy_async_smem();
          __syncwarp();
          if (lane == 0) {
            const int og0 = out0 + q * 32;
            if (og0 < p.n_out && m0 + c0 < p.m) {
              if (p.acc)
                tma_reduce_add_2d(&tm_y, sb, og0, m0 + c0);
              else
                tma_store_2d(&tm_y, sb, og0, m0 + c0);
            }
            tma_store_commit();
          }
        } else if (ok && og < p.n_out) {
          const int mlim = p.m - (m0 + c0);
          if (p.splits > 1) {
            // f32 partial of this split; the reduce kernel adds bias and rounds.
            float* wp = p.ws + (static_cast<size_t>(unit_split(lt)) * p.m + m0 + c0) * p.n_out + og;
#pragma unroll
            for (int j = 0; j < 32; ++j)
              if (j < mlim) wp[static_cast<size_t>(j) * p.n_out] = __uint_as_float(v[j]);
          } else {
            uint16_t* yp = p.y + static_cast<size_t>(m0 + c0) * p.n_out + og;
#pragma unroll
            for (int j = 0; j < 32; ++j) {
              if (j < mlim) {
                uint16_t* e = yp + static_cast<size_t>(j) * p.n_out;
                __nv_bfloat16 r = __float2bfloat16_rn(__uint_as_float(v[j]) + bias);
                if (p.acc)
                  r = __float2bfloat16_rn(__bfloat162float(r) +
                                          __uint_as_float(uint32_t(*e) << 16));
                *e = __bfloat16_as_ushort(r);
              }
            }
          }
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(acc_empty(buf));
    }
    // The staging buffers stay valid until every store has read them.
    if (p.tma_y && lane == 0) tma_store_wait_all();
    __syncwarp();
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc(tmem, C::TMEM_COLS);
  }
}

}  // namespace
}  // namespace tq

#include "qmm_pair.cuh"
#include "qmm_pair_ts.cuh"
#include "qmm_small.cuh"

namespace tq {
namespace {

struct Args {
  const void* x;
  const void* codes;
  const void* scales;
  const void* biases;
  const void* bias;
  const void* lora_up;
  const void* lora_down;
  int64_t m, w_rows, w_cols;
  int transpose, group_size, bits;
  int rank;
  void* y;
  void* ws = nullptr;        // split-K workspace (f32), or null: no split
  size_t ws_bytes = 0;
  int64_t ld_down = 0;       // row pitch of lora_down in elements (0: rank)
  int acc = 0;               // add the result into y instead of storing it
};

// How a call is run: the token tile, whether the scale tiles ride in the TMA
// stages, and the k-split.  The workspace query and the launch share it.
struct Plan {
  int bn = 32;
  bool stma = false;
  bool pair = false;  // two CTAs per 256-row tile (cta_group::2)
  bool ts = false;    // pair forward with the weight tile in tensor memory
  int splits = 1;
  int k_steps_per_split = 1;
  size_t ws_bytes = 0;
  bool small = false;  // register-dequant kernel for a handful of tokens
  int small_cs = 1;    // its CTAs per 128-row block (cluster splitting k)
};

// TQ_QMM_BN pins the token tile (256, 128, 64 or 32) for tuning runs.
int forced_bn() {
  static const int forced = [] {
    const char* e = getenv("TQ_QMM_BN");
    return e ? atoi(e) : 0;
  }();
  return forced;
}

int pick_bn(int64_t m, int64_t n_out) {
  const int64_t tiles_n = (n_out + kBM - 1) / kBM;
  const int sms = sm_count();
  const int forced = forced_bn();
  if (forced == 256 || forced == 128 || forced == 64 || forced == 32) return forced;
  // Largest token tile that still gives every SM a tile (M-side padding is
  // zero-filled by TMA and never stored).
  for (int cand : {256, 128, 64}) {
    if (m >= cand / 2 && ((m + cand - 1) / cand) * tiles_n >= sms) return cand;
  }
  if (m > 128) return 128;
  if (m > 32) return 64;
  return 32;
}

// The small-token forward (qmm_small.cuh): 4-bit codes, no LoRA, k a
// multiple of 128, rows of 16.  TQ_QMM_SMALL=0 keeps such calls on the
// tensor-memory kernel, for comparison.
bool small_ok(const Args& a) {
  static const bool off = [] {
    const char* e = getenv("TQ_QMM_SMALL");
    return e && e[0] == '0';
  }();
  return !off && !a.acc && a.transpose && a.bits == 4 && a.m >= 1 && a.m <= kSmallMaxM && a.rank == 0 &&
         a.w_cols % kSmallChunk == 0 && a.w_rows % 16 == 0 && aligned(a.x, 16) &&
         aligned(a.y, 16);
}

// Smallest cluster (1, 2, 4, 8) whose CTAs give every SM two, keeping at
// least two k-chunks per CTA; at most 4 with 32 tokens (shared memory).
int small_cluster(const Args& a) {
  const int64_t blocks = (a.w_rows + kSmallRows - 1) / kSmallRows;
  const int64_t chunks = a.w_cols / kSmallChunk;
  const int cap = a.m > 24 ? 4 : kSmallMaxCluster;
  int cs = 1;
  while (cs < cap && blocks * cs < 2 * sm_count() && chunks / (2 * cs) >= 2) cs *= 2;
  return cs;
}

Plan make_plan(const Args& a, bool allow_split) {
  Plan pl;
  if (small_ok(a)) {
    pl.small = true;
    pl.small_cs = small_cluster(a);
    return pl;
  }
  const int64_t n_out = a.transpose ? a.w_rows : a.w_cols;
  const int64_t k_red = a.transpose ? a.w_cols : a.w_rows;
  pl.bn = pick_bn(a.m, n_out);
  const int64_t gpr = a.w_cols / a.group_size;
  pl.stma = gpr % 8 == 0 && aligned(a.scales, 16) && aligned(a.biases, 16);
  const int num_k = static_cast<int>((k_red + kBK - 1) / kBK);
  pl.k_steps_per_split = num_k;
  if (allow_split && pl.stma) {
    const int64_t tiles = ((n_out + kBM - 1) / kBM) * ((a.m + pl.bn - 1) / pl.bn);
    const int sms = sm_count();
    if (tiles < sms && num_k >= 8) {
      // As many splits as keep every unit in one wave over the SMs.
      int splits = static_cast<int>(sms / tiles);
      const int max_splits = num_k / 4 < 16 ? num_k / 4 : 16;  // >= 4 k-steps per split
      if (splits > max_splits) splits = max_splits;
      if (splits > 1) {
        const int per = (num_k + splits - 1) / splits;
        pl.splits = (num_k + per - 1) / per;
        pl.k_steps_per_split = per;
        pl.ws_bytes = static_cast<size_t>(pl.splits) * a.m * n_out * sizeof(float);
      }
    }
  }
  // Large problems run on CTA pairs when there are enough 256-row tiles to
  // give every pair one (TQ_QMM_PAIR=0 keeps single CTAs, for comparison).
  static const bool pair_off = [] {
    const char* e = getenv("TQ_QMM_PAIR");
    return e && e[0] == '0';
  }();
  // TQ_QMM_TS=1 runs the forward pairs with the dequantized weight tile in
  // tensor memory (token tiles of 192 or 128).  Off by default: exact, and
  // it takes the weight tile's store and operand read out of shared memory,
  // but at 16384 x 4096 x 4096 it ran 1334 TFLOP/s against 1409 for the
  // shared-memory pairs (the tensor pipe was no busier: 71 % against 74 % of
  // active cycles), so shared-memory traffic is not what bounds the pairs.
  static const bool ts_off = [] {
    const char* e = getenv("TQ_QMM_TS");
    return !(e && e[0] == '1');
  }();
  if (!pair_off && pl.stma && pl.splits == 1 && n_out > kBM && aligned(a.y, 16)) {
    const int64_t pair_tiles_n = (n_out + 2 * kBM - 1) / (2 * kBM);
    const int pairs = sm_count() / 2;
    const int forced = forced_bn();
    const bool ts = a.transpose && !ts_off;
    const int top = ts ? 192 : 256;
    const int cands[2] = {top, 128};
    // Among the token tiles that keep at least three quarters of the pairs
    // busy, the one with the least estimated time: waves x tile cost, a
    // 128-token tile costing 1/0.7 of its tokens' share of a 256-token one
    // (its weight tile is dequantized for half as many tokens).  At 1024
    // tokens x 4096 outputs this picks one wave of 256-token tiles (64 of
    // 74 pairs) over two waves of 128-token ones.
    double best = 0.0;
    for (int cand : cands) {
      if ((forced == 256 || forced == 192 || forced == 128) &&
          (forced == 128) != (cand == 128))
        continue;
      const int64_t tiles = ((a.m + cand - 1) / cand) * pair_tiles_n;
      if (a.m < cand / 2 || 4 * tiles < 3 * pairs) continue;
      const int64_t waves = (tiles + pairs - 1) / pairs;
      const double cost = static_cast<double>(waves) * cand / (cand == 128 ? 0.7 : 1.0);
      if (!pl.pair || cost < best) {
        pl.pair = true;
        pl.ts = ts;
        pl.bn = cand;
        best = cost;
      }
    }
  }
  return pl;
}

// y[m, n] = bf16(sum over splits of ws[s, m, n] + bias[n]); 8 outputs a
// thread.  acc: that value is then added to y's and rounded again.
__global__ void __launch_bounds__(256) splitk_reduce_kernel(const float* __restrict__ ws,
                                                            int splits, int64_t m, int n,
                                                            const uint16_t* __restrict__ bias,
                                                            int acc_y, uint16_t* __restrict__ y) {
  griddep_wait();
  griddep_launch_dependents();
  const int64_t nv = m * n / 8;
  const int64_t plane = m * n;
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  for (int64_t v = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; v < nv; v += stride) {
    const int64_t e = v * 8;
    float acc[8];
    const float4* p0 = reinterpret_cast<const float4*>(ws + e);
    float4 a0 = __ldg(p0), a1 = __ldg(p0 + 1);
    acc[0] = a0.x; acc[1] = a0.y; acc[2] = a0.z; acc[3] = a0.w;
    acc[4] = a1.x; acc[5] = a1.y; acc[6] = a1.z; acc[7] = a1.w;
    for (int sp = 1; sp < splits; ++sp) {
      const float4* ps = reinterpret_cast<const float4*>(ws + sp * plane + e);
      a0 = __ldg(ps);
      a1 = __ldg(ps + 1);
      acc[0] += a0.x; acc[1] += a0.y; acc[2] += a0.z; acc[3] += a0.w;
      acc[4] += a1.x; acc[5] += a1.y; acc[6] += a1.z; acc[7] += a1.w;
    }
    if (bias) {
      const int col = static_cast<int>(e % n);
#pragma unroll
      for (int j = 0; j < 8; ++j) acc[j] += __uint_as_float(uint32_t(__ldg(bias + col + j)) << 16);
    }
    if (acc_y) {
      const uint4 old = reinterpret_cast<const uint4*>(y)[v];
      const uint32_t w[4] = {old.x, old.y, old.z, old.w};
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        acc[2 * j] = __bfloat162float(__float2bfloat16_rn(acc[2 * j])) + __uint_as_float(w[j] << 16);
        acc[2 * j + 1] = __bfloat162float(__float2bfloat16_rn(acc[2 * j + 1])) +
                         __uint_as_float(w[j] & 0xFFFF0000u);
      }
    }
    uint4 o;
    o.x = pack_bf16x2_f32(acc[0], acc[1]);
    o.y = pack_bf16x2_f32(acc[2], acc[3]);
    o.z = pack_bf16x2_f32(acc[4], acc[5]);
    o.w = pack_bf16x2_f32(acc[6], acc[7]);
    reinterpret_cast<uint4*>(y)[v] = o;
  }
}

// The six tensor maps of one call.  x_rows: token rows per box (the token
// tile, or its half for a CTA of a pair); sc_rows: weight rows per scale box.
struct Maps {
  CUtensorMap x, c, lup, ldn, sc, bi;
};

template <int BITS, bool TRANS>
int make_maps(const Args& a, int x_rows, int sc_rows, bool stma, Maps& mp) {
  const int64_t k_red = TRANS ? a.w_cols : a.w_rows;
  CUtensorMap &tm_x = mp.x, &tm_c = mp.c, &tm_lup = mp.lup, &tm_ldn = mp.ldn, &tm_sc = mp.sc,
              &tm_bi = mp.bi;
  const int BN = x_rows;
  int rc;
  {
    const uint64_t dims[2] = {static_cast<uint64_t>(k_red), static_cast<uint64_t>(a.m)};
    const uint64_t strides[1] = {static_cast<uint64_t>(k_red) * 2};
    const uint32_t box[2] = {kBK, static_cast<uint32_t>(BN)};
    rc = encode_tmap(&tm_x, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, a.x, dims, strides, box,
                     CU_TENSOR_MAP_SWIZZLE_128B);
    if (rc) return rc;
  }
  {
    const uint64_t words = static_cast<uint64_t>(a.w_cols) * BITS / 32;
    const uint64_t dims[2] = {words, static_cast<uint64_t>(a.w_rows)};
    const uint64_t strides[1] = {words * 4};
    uint32_t box[2];
    CUtensorMapSwizzle sw;
    if constexpr (TRANS) {
      box[0] = kBK * BITS / 32;
      box[1] = kBM;
      sw = BITS == 4 ? CU_TENSOR_MAP_SWIZZLE_32B : CU_TENSOR_MAP_SWIZZLE_64B;
    } else {
      box[0] = kBM * BITS / 32;
      box[1] = kBK;
      sw = BITS == 4 ? CU_TENSOR_MAP_SWIZZLE_64B : CU_TENSOR_MAP_SWIZZLE_128B;
    }
    rc = encode_tmap(&tm_c, CU_TENSOR_MAP_DATA_TYPE_UINT32, 2, a.codes, dims, strides, box, sw);
    if (rc) return rc;
  }
  if (stma) {
    const uint64_t gpr = static_cast<uint64_t>(a.w_cols / a.group_size);
    const uint64_t dims[2] = {gpr, static_cast<uint64_t>(a.w_rows)};
    const uint64_t strides[1] = {gpr * 2};
    const uint32_t box[2] = {8, static_cast<uint32_t>(sc_rows)};
    rc = encode_tmap(&tm_sc, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, a.scales, dims, strides, box,
                     CU_TENSOR_MAP_SWIZZLE_NONE);
    if (rc) return rc;
    rc = encode_tmap(&tm_bi, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, a.biases, dims, strides, box,
                     CU_TENSOR_MAP_SWIZZLE_NONE);
    if (rc) return rc;
  } else {
    tm_sc = tm_x;
    tm_bi = tm_x;
  }
  if (a.rank > 0) {
    if constexpr (TRANS) {
      const uint64_t dims[2] = {static_cast<uint64_t>(a.rank), static_cast<uint64_t>(a.w_rows)};
      const uint64_t strides[1] = {static_cast<uint64_t>(a.rank) * 2};
      const uint32_t box[2] = {8, kBM};
      rc = encode_tmap(&tm_lup, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, a.lora_up, dims, strides, box,
                       CU_TENSOR_MAP_SWIZZLE_NONE);
    } else {
      const uint64_t dims[2] = {static_cast<uint64_t>(a.w_cols), static_cast<uint64_t>(a.rank)};
      const uint64_t strides[1] = {static_cast<uint64_t>(a.w_cols) * 2};
      const uint32_t box[2] = {64, 8};
      rc = encode_tmap(&tm_lup, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, a.lora_up, dims, strides, box,
                       CU_TENSOR_MAP_SWIZZLE_128B);
    }
    if (rc) return rc;
    const uint64_t ld = static_cast<uint64_t>(a.ld_down ? a.ld_down : a.rank);
    const uint64_t dims[2] = {static_cast<uint64_t>(a.rank), static_cast<uint64_t>(a.m)};
    const uint64_t strides[1] = {ld * 2};
    const uint32_t box[2] = {8, static_cast<uint32_t>(BN)};
    rc = encode_tmap(&tm_ldn, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, a.lora_down, dims, strides, box,
                     CU_TENSOR_MAP_SWIZZLE_NONE);
    if (rc) return rc;
  } else {
    tm_lup = tm_x;
    tm_ldn = tm_x;
  }
  return TQ_OK;
}

// The packed weight and its scales are loaded with an L2 evict_last policy
// (every token tile reads them again); TQ_QMM_KEEP=0 loads them at normal
// priority, for comparison runs.
int keep_weights() {
  static const int keep = [] {
    const char* e = getenv("TQ_QMM_KEEP");
    return e && e[0] == '0' ? 0 : 1;
  }();
  return keep;
}

Params make_params(const Args& a, const Plan& pl, int tile_rows, int bn, int* status) {
  const int64_t k_red = a.transpose ? a.w_cols : a.w_rows;
  const int64_t n_out = a.transpose ? a.w_rows : a.w_cols;
  Params p;
  p.scales = static_cast<const uint16_t*>(a.scales);
  p.biases = static_cast<const uint16_t*>(a.biases);
  p.bias_vec = static_cast<const uint16_t*>(a.bias);
  p.y = static_cast<uint16_t*>(a.y);
  p.m = static_cast<int>(a.m);
  p.n_out = static_cast<int>(n_out);
  p.k_red = static_cast<int>(k_red);
  p.w_rows = static_cast<int>(a.w_rows);
  p.groups_per_row = static_cast<int>(a.w_cols / a.group_size);
  p.group_shift = a.group_size == 32 ? 5 : (a.group_size == 64 ? 6 : 7);
  p.lora_rank = a.rank;
  p.tiles_n = static_cast<int>((n_out + tile_rows - 1) / tile_rows);
  const int64_t tiles_m = (a.m + bn - 1) / bn;
  p.tiles_total = static_cast<int>(p.tiles_n * tiles_m);
  p.splits = pl.splits;
  p.k_steps_per_split = pl.k_steps_per_split;
  p.ws = static_cast<float*>(a.ws);
  p.tma_y = 0;
  p.acc = a.acc;
  p.keep_weights = keep_weights();
  p.status = status;
  return p;
}

template <int BITS, bool TRANS, int BN, bool STMA>
int launch(const Args& a, const Plan& pl, cudaStream_t stream, int* status) {
  using C = Cfg<BITS, TRANS, BN, STMA>;
  const int64_t n_out = TRANS ? a.w_rows : a.w_cols;
  Maps mp;
  int rc = make_maps<BITS, TRANS>(a, BN, C::SC_ROWS, STMA, mp);
  if (rc) return rc;
  Params p = make_params(a, pl, kBM, BN, status);
  // Without a split the bf16 output goes out by TMA stores when y allows it
  // (16-byte aligned; the row pitch is n_out * 2 bytes, a multiple of 16).
  CUtensorMap tm_y = mp.x;
  p.tma_y = 0;
  if (pl.splits == 1 && aligned(a.y, 16)) {
    const uint64_t dims[2] = {static_cast<uint64_t>(n_out), static_cast<uint64_t>(a.m)};
    const uint64_t strides[1] = {static_cast<uint64_t>(n_out) * 2};
    const uint32_t box[2] = {32, 32};
    rc = encode_tmap(&tm_y, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, a.y, dims, strides, box,
                     CU_TENSOR_MAP_SWIZZLE_NONE);
    if (rc) return rc;
    p.tma_y = 1;
  }
  auto kernel = qmm_kernel<BITS, TRANS, BN, STMA>;
  rc = set_max_smem_once(reinterpret_cast<const void*>(kernel), C::SMEM,
                         "cudaFuncSetAttribute(qmm smem)");
  if (rc) return rc;
  const int units = p.tiles_total * p.splits;
  const int grid = units < sm_count() ? units : sm_count();
  rc = launch_kernel(kernel, dim3(grid), dim3(kThreads), C::SMEM, stream, 1, "qmm launch", mp.x,
                     mp.c, mp.lup, mp.ldn, mp.sc, mp.bi, tm_y, p);
  if (rc || pl.splits == 1) return rc;
  const int64_t nv = a.m * n_out / 8;
  int rgrid = static_cast<int>((nv + 255) / 256);
  if (rgrid > sm_count() * 8) rgrid = sm_count() * 8;
  return launch_kernel(splitk_reduce_kernel, dim3(rgrid), dim3(256), 0, stream, 1,
                       "split-K reduce launch", static_cast<const float*>(a.ws), pl.splits, a.m,
                       static_cast<int>(n_out), static_cast<const uint16_t*>(a.bias), a.acc,
                       static_cast<uint16_t*>(a.y));
}

template <int BITS, bool TRANS, int BN>
int launch_scales(const Args& a, const Plan& pl, cudaStream_t stream, int* status) {
  // The scale/bias tiles ride in the TMA stages when their rows start on
  // 16-byte boundaries (groups per row a multiple of 8, 16-byte aligned
  // base); otherwise each dequantizing thread loads its own.
  return pl.stma ? launch<BITS, TRANS, BN, true>(a, pl, stream, status)
                 : launch<BITS, TRANS, BN, false>(a, pl, stream, status);
}

// Pairs of CTAs the GPU holds at once for a pair kernel (cluster of 2, one
// CTA per SM), per device; sm_count / 2 if the query fails.
template <class K>
int resident_pairs(K kernel, int smem) {
  constexpr int kMaxDev = 64;
  static int cache[kMaxDev] = {};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDev) return sm_count() / 2;
  if (cache[dev] > 0) return cache[dev];
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(2, 1, 1);
  cfg.blockDim = dim3(kThreads, 1, 1);
  cfg.dynamicSmemBytes = static_cast<size_t>(smem);
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  int n = 0;
  if (cudaOccupancyMaxActiveClusters(&n, reinterpret_cast<const void*>(kernel), &cfg) !=
          cudaSuccess ||
      n <= 0) {
    cudaGetLastError();
    n = sm_count() / 2;
  }
  cache[dev] = n;
  return n;
}

template <int BITS, bool TRANS, int BN, int G>
int launch_pair(const Args& a, const Plan& pl, cudaStream_t stream, int* status) {
  using C = PairCfg<BITS, TRANS, BN, G>;
  Maps mp;
  int rc = make_maps<BITS, TRANS>(a, BN / 2, C::SC_ROWS, true, mp);
  if (rc) return rc;
  const Params p = make_params(a, pl, kPairRows, BN, status);
  // y as the epilogue's TMA store target: boxes of 32 features x 32 tokens.
  CUtensorMap tm_y;
  {
    const int64_t n_out = TRANS ? a.w_rows : a.w_cols;
    const uint64_t dims[2] = {static_cast<uint64_t>(n_out), static_cast<uint64_t>(a.m)};
    const uint64_t strides[1] = {static_cast<uint64_t>(n_out) * 2};
    const uint32_t box[2] = {32, 32};
    rc = encode_tmap(&tm_y, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, a.y, dims, strides, box,
                     CU_TENSOR_MAP_SWIZZLE_NONE);
    if (rc) return rc;
  }
  auto kernel = qmm_pair_kernel<BITS, TRANS, BN, G>;
  rc = set_max_smem_once(reinterpret_cast<const void*>(kernel), C::SMEM,
                         "cudaFuncSetAttribute(qmm pair smem)");
  if (rc) return rc;
  const int pairs = resident_pairs(kernel, C::SMEM);
  const int grid_pairs = p.tiles_total < pairs ? p.tiles_total : pairs;
  return launch_kernel(kernel, dim3(2 * grid_pairs), dim3(kThreads), C::SMEM, stream, dim3(2),
                       "qmm pair launch", mp.x, mp.c, mp.lup, mp.ldn, mp.sc, mp.bi, tm_y, p);
}

template <int BITS, int BN>
int launch_pair_ts(const Args& a, const Plan& pl, cudaStream_t stream, int* status) {
  using C = PairTsCfg<BITS, BN>;
  Maps mp;
  int rc = make_maps<BITS, true>(a, BN / 2, C::SC_ROWS, true, mp);
  if (rc) return rc;
  const Params p = make_params(a, pl, kPairRows, BN, status);
  CUtensorMap tm_y;
  {
    const uint64_t dims[2] = {static_cast<uint64_t>(a.w_rows), static_cast<uint64_t>(a.m)};
    const uint64_t strides[1] = {static_cast<uint64_t>(a.w_rows) * 2};
    const uint32_t box[2] = {32, 32};
    rc = encode_tmap(&tm_y, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, a.y, dims, strides, box,
                     CU_TENSOR_MAP_SWIZZLE_NONE);
    if (rc) return rc;
  }
  auto kernel = qmm_pair_ts_kernel<BITS, BN>;
  rc = set_max_smem_once(reinterpret_cast<const void*>(kernel), C::SMEM,
                         "cudaFuncSetAttribute(qmm pair ts smem)");
  if (rc) return rc;
  const int pairs = resident_pairs(kernel, C::SMEM);
  const int grid_pairs = p.tiles_total < pairs ? p.tiles_total : pairs;
  return launch_kernel(kernel, dim3(2 * grid_pairs), dim3(kThreads), C::SMEM, stream, dim3(2),
                       "qmm pair ts launch", mp.x, mp.c, mp.lup, mp.ldn, mp.sc, mp.bi, tm_y, p);
}

template <int BITS, bool TRANS>
int launch_bn(const Args& a, const Plan& pl, cudaStream_t stream, int* status) {
  if constexpr (TRANS) {
    if (pl.ts)
      return pl.bn == 192 ? launch_pair_ts<BITS, 192>(a, pl, stream, status)
                          : launch_pair_ts<BITS, 128>(a, pl, stream, status);
  }
  if (pl.pair) {
    // Dequantizing groups: two forward (deeper TMA ring), four for dX
    // (measured 0.5-2 % and 3.6-4.8 % better respectively at M >= 8192).
    constexpr int G = TRANS ? 2 : 4;
    return pl.bn == 256 ? launch_pair<BITS, TRANS, 256, G>(a, pl, stream, status)
                        : launch_pair<BITS, TRANS, 128, G>(a, pl, stream, status);
  }
  switch (pl.bn) {
    case 256: return launch_scales<BITS, TRANS, 256>(a, pl, stream, status);
    case 128: return launch_scales<BITS, TRANS, 128>(a, pl, stream, status);
    case 64: return launch_scales<BITS, TRANS, 64>(a, pl, stream, status);
    default: return launch_scales<BITS, TRANS, 32>(a, pl, stream, status);
  }
}

template <int MT>
int launch_small_mt(const Args& a, const Plan& pl, cudaStream_t stream, int* status) {
  using C = SmallCfg<MT>;
  int rc = set_max_smem_once(reinterpret_cast<const void*>(qmm_small_kernel<MT>),
                             C::smem(kSmallMaxCluster), "cudaFuncSetAttribute(qmm_small)");
  if (rc) return rc;
  // Two CTAs share an SM when their shared memory fits: ask for the largest
  // shared-memory carveout (the default may leave room for one).
  static const bool carveout_set = [] {
    return cudaFuncSetAttribute(reinterpret_cast<const void*>(qmm_small_kernel<MT>),
                                cudaFuncAttributePreferredSharedMemoryCarveout,
                                cudaSharedmemCarveoutMaxShared) == cudaSuccess;
  }();
  (void)carveout_set;
  CUtensorMap tm_x, tm_c;
  {
    const uint64_t dims[2] = {static_cast<uint64_t>(a.w_cols), static_cast<uint64_t>(a.m)};
    const uint64_t strides[1] = {static_cast<uint64_t>(a.w_cols) * 2};
    const uint32_t box[2] = {64, static_cast<uint32_t>(C::MPAD)};
    rc = encode_tmap(&tm_x, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, a.x, dims, strides, box,
                     CU_TENSOR_MAP_SWIZZLE_128B);
    if (rc) return rc;
  }
  {
    // Codes as u32 [w_rows, w_cols / 8]: 16 words (one 128-k chunk) x 128 rows.
    const uint64_t dims[2] = {static_cast<uint64_t>(a.w_cols / 8), static_cast<uint64_t>(a.w_rows)};
    const uint64_t strides[1] = {static_cast<uint64_t>(a.w_cols / 2)};
    const uint32_t box[2] = {kSmallChunk / 8, static_cast<uint32_t>(kSmallRows)};
    rc = encode_tmap(&tm_c, CU_TENSOR_MAP_DATA_TYPE_UINT32, 2, a.codes, dims, strides, box,
                     CU_TENSOR_MAP_SWIZZLE_64B);
    if (rc) return rc;
  }
  SmallParams p{};
  p.codes = static_cast<const uint32_t*>(a.codes);
  p.scales = static_cast<const uint16_t*>(a.scales);
  p.biases = static_cast<const uint16_t*>(a.biases);
  p.bias = static_cast<const uint16_t*>(a.bias);
  p.y = static_cast<uint16_t*>(a.y);
  p.m = static_cast<int>(a.m);
  p.n = static_cast<int>(a.w_rows);
  p.k = static_cast<int>(a.w_cols);
  p.group = a.group_size;
  p.cs = pl.small_cs;
  p.status = status;
  const int64_t blocks = (a.w_rows + kSmallRows - 1) / kSmallRows;
  return launch_kernel(qmm_small_kernel<MT>, dim3(static_cast<unsigned>(blocks * pl.small_cs)),
                       dim3(kSmallThreads), static_cast<size_t>(C::smem(pl.small_cs)), stream,
                       dim3(static_cast<unsigned>(pl.small_cs)), "quantized_matmul (small) launch",
                       tm_x, tm_c, p);
}

int launch_small(const Args& a, const Plan& pl, cudaStream_t stream, int* status) {
  switch ((a.m + 7) / 8) {
    case 1: return launch_small_mt<1>(a, pl, stream, status);
    case 2: return launch_small_mt<2>(a, pl, stream, status);
    case 3: return launch_small_mt<3>(a, pl, stream, status);
    default: return launch_small_mt<4>(a, pl, stream, status);
  }
}

int validate(const Args& a) {
  if (a.bits != 4 && a.bits != 8) return fail(TQ_ERR_UNSUPPORTED, "bits must be 4 or 8, got %d", a.bits);
  if (a.group_size != 32 && a.group_size != 64 && a.group_size != 128)
    return fail(TQ_ERR_UNSUPPORTED, "group_size must be 32, 64 or 128, got %d", a.group_size);
  if (a.m < 0 || a.w_rows < 0 || a.w_cols < 0) return fail(TQ_ERR_INVALID, "negative shape");
  if (a.w_cols % a.group_size != 0)
    return fail(TQ_ERR_INVALID, "w_cols (%lld) must be divisible by group_size (%d)",
                (long long)a.w_cols, a.group_size);
  if (a.w_rows % 8 != 0)
    return fail(TQ_ERR_INVALID, "w_rows (%lld) must be a multiple of 8", (long long)a.w_rows);
  if (a.m > (1ll << 31) - 1 || a.w_rows > (1ll << 31) - 1 || a.w_cols > (1ll << 31) - 1)
    return fail(TQ_ERR_INVALID, "dimensions must fit in 31 bits");
  if (a.rank != 0 && a.rank != 8 && a.rank != 16)
    return fail(TQ_ERR_UNSUPPORTED, "LoRA rank must be 8 or 16 (or 0 for none), got %d", a.rank);
  if (a.rank && (!a.lora_up || !a.lora_down))
    return fail(TQ_ERR_INVALID, "rank %d needs both lora_up and lora_down", a.rank);
  if (a.rank && a.ld_down != 0 && (a.ld_down < a.rank || a.ld_down % 8 != 0))
    return fail(TQ_ERR_INVALID, "ld_down (%lld) must be 0 or a multiple of 8 >= rank (%d)",
                (long long)a.ld_down, a.rank);
  if (!a.transpose && a.bias) return fail(TQ_ERR_INVALID, "bias is only defined for transpose != 0");
  return TQ_OK;
}

int validate_ptrs(const Args& a) {
  if (a.m == 0 || a.w_rows == 0 || a.w_cols == 0) return TQ_OK;  // nothing is touched
  if (!a.x || !a.codes || !a.scales || !a.biases || !a.y) return fail(TQ_ERR_INVALID, "null pointer");
  if (!aligned(a.x, 16) || !aligned(a.codes, 16) || (a.rank && (!aligned(a.lora_up, 16) ||
                                                                 !aligned(a.lora_down, 16))))
    return fail(TQ_ERR_MISALIGNED, "x, codes, lora_up and lora_down must be 16-byte aligned");
  if (!aligned(a.y, 2) || !aligned(a.scales, 2) || !aligned(a.biases, 2))
    return fail(TQ_ERR_MISALIGNED, "y, scales and biases must be 2-byte aligned");
  return TQ_OK;
}

int run(const Args& a, void* stream) {
  int rc = validate(a);
  if (rc) return rc;
  rc = validate_ptrs(a);
  if (rc) return rc;
  if (a.m == 0 || a.w_rows == 0 || a.w_cols == 0) return TQ_OK;
  // A workspace turns on split-K when the tiles alone cannot fill the GPU.
  const Plan pl = make_plan(a, a.ws != nullptr);
  if (pl.splits > 1) {
    if (a.ws_bytes < pl.ws_bytes)
      return fail(TQ_ERR_INVALID, "workspace of %zu bytes is smaller than the %zu this call needs",
                  a.ws_bytes, pl.ws_bytes);
    if (!aligned(a.ws, 16)) return fail(TQ_ERR_MISALIGNED, "workspace must be 16-byte aligned");
    if (((a.transpose ? a.w_rows : a.w_cols) % 8) != 0)
      return fail(TQ_ERR_INVALID, "split-K needs an output width that is a multiple of 8");
  }
  int* status = device_status_ptr(&rc);
  if (!status) return rc;
  cudaStream_t s = as_stream(stream);
  if (pl.small) return launch_small(a, pl, s, status);
  if (a.bits == 4)
    return a.transpose ? launch_bn<4, true>(a, pl, s, status) : launch_bn<4, false>(a, pl, s, status);
  return a.transpose ? launch_bn<8, true>(a, pl, s, status) : launch_bn<8, false>(a, pl, s, status);
}

}  // namespace
}  // namespace tq

extern "C" int tq_quantized_matmul(const void* x, const void* codes, const void* scales,
                                   const void* biases, int64_t m, int64_t w_rows, int64_t w_cols,
                                   int transpose, int group_size, int bits, void* y, void* stream) {
  tq::Args a{x, codes, scales, biases, nullptr, nullptr, nullptr, m, w_rows, w_cols,
             transpose, group_size, bits, 0, y};
  return tq::run(a, stream);
}

extern "C" int tq_qlora_matmul(const void* x, const void* codes, const void* scales,
                               const void* biases, int64_t m, int64_t w_rows, int64_t w_cols,
                               int transpose, int group_size, int bits, const void* bias,
                               const void* lora_up, const void* lora_down, int64_t ld_down,
                               int64_t rank, void* y, void* stream) {
  if (rank < 0 || rank > 16) return tq::fail(TQ_ERR_UNSUPPORTED, "LoRA rank must be 8 or 16");
  tq::Args a{x, codes, scales, biases, bias, lora_up, lora_down, m, w_rows, w_cols,
             transpose, group_size, bits, static_cast<int>(rank), y};
  a.ld_down = ld_down;
  return tq::run(a, stream);
}

extern "C" int tq_qmm_workspace_bytes(int64_t m, int64_t w_rows, int64_t w_cols, int transpose,
                                      int group_size, int bits, size_t* bytes) {
  if (!bytes) return tq::fail(TQ_ERR_INVALID, "null output");
  tq::Args a{nullptr, nullptr, nullptr, nullptr, nullptr, nullptr, nullptr, m, w_rows, w_cols,
             transpose, group_size, bits, 0, nullptr};
  // Scales are taken as 16-byte aligned here (the caller's allocator's rule);
  // a call whose scales are not falls back to no split and needs nothing.
  a.scales = a.biases = reinterpret_cast<const void*>(static_cast<uintptr_t>(256));
  int rc = tq::validate(a);
  if (rc) return rc;
  *bytes = (m == 0 || w_rows == 0 || w_cols == 0) ? 0 : tq::make_plan(a, true).ws_bytes;
  return TQ_OK;
}

extern "C" int tq_quantized_matmul_ws(const void* x, const void* codes, const void* scales,
                                      const void* biases, int64_t m, int64_t w_rows,
                                      int64_t w_cols, int transpose, int group_size, int bits,
                                      void* y, void* workspace, size_t workspace_bytes,
                                      void* stream) {
  tq::Args a{x, codes, scales, biases, nullptr, nullptr, nullptr, m, w_rows, w_cols,
             transpose, group_size, bits, 0, y, workspace, workspace_bytes};
  return tq::run(a, stream);
}

extern "C" int tq_qlora_matmul_ws(const void* x, const void* codes, const void* scales,
                                  const void* biases, int64_t m, int64_t w_rows, int64_t w_cols,
                                  int transpose, int group_size, int bits, const void* bias,
                                  const void* lora_up, const void* lora_down, int64_t ld_down,
                                  int64_t rank, void* y, void* workspace,
                                  size_t workspace_bytes, void* stream) {
  if (rank < 0 || rank > 16) return tq::fail(TQ_ERR_UNSUPPORTED, "LoRA rank must be 8 or 16");
  tq::Args a{x, codes, scales, biases, bias, lora_up, lora_down, m, w_rows, w_cols,
             transpose, group_size, bits, static_cast<int>(rank), y, workspace, workspace_bytes};
  a.ld_down = ld_down;
  return tq::run(a, stream);
}

extern "C" int tq_qlora_matmul_accumulate(const void* x, const void* codes, const void* scales,
                                          const void* biases, int64_t m, int64_t w_rows,
                                          int64_t w_cols, int transpose, int group_size,
                                          int bits, const void* bias, const void* lora_up,
                                          const void* lora_down, int64_t ld_down, int64_t rank,
                                          void* y, void* workspace, size_t workspace_bytes,
                                          void* stream) {
  if (rank < 0 || rank > 16) return tq::fail(TQ_ERR_UNSUPPORTED, "LoRA rank must be 8 or 16");
  tq::Args a{x, codes, scales, biases, bias, lora_up, lora_down, m, w_rows, w_cols,
             transpose, group_size, bits, static_cast<int>(rank), y, workspace, workspace_bytes};
  a.ld_down = ld_down;
  a.acc = 1;
  return tq::run(a, stream);
}

// ------------------------------------------------- fixed-scratch variant ---
//
// tq_quantized_matmul_noalloc: the split-K GEMM with its f32 partials in a
// file-scope device array instead of a caller workspace, for callers that
// cannot allocate device memory at call time (an allocator-free runtime, a
// host that has handed its whole memory budget to a pool it does not own).
// The array is part of this module's image: every GPU that loads the library
// holds its 8 MiB until the process exits.

namespace tq {
namespace {

constexpr size_t kNoAllocScratchBytes = TQ_NOALLOC_SCRATCH_BYTES;

// Split-K partials of tq_quantized_matmul_noalloc, shared by all its calls on
// a device.  Host code must not pass this name to a kernel: on the host it is
// only a stand-in; the device address comes from cudaGetSymbolAddress.
static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocScratchBytes];

constexpr int kScratchMaxDevices = 64;
void* g_scratch_ptr[kScratchMaxDevices] = {};
std::mutex g_scratch_mu;

// The device address of the scratch array on the current device, resolved
// once per device with that device current.
int noalloc_scratch(void** out) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kScratchMaxDevices)
    return fail(TQ_ERR_CUDA, "no current CUDA device");
  std::lock_guard<std::mutex> lock(g_scratch_mu);
  if (!g_scratch_ptr[dev]) {
    void* p = nullptr;
    const int rc = check_cuda(cudaGetSymbolAddress(&p, g_noalloc_scratch),
                              "cudaGetSymbolAddress(split-K scratch)");
    if (rc) return rc;
    g_scratch_ptr[dev] = p;
  }
  *out = g_scratch_ptr[dev];
  return TQ_OK;
}

}  // namespace
}  // namespace tq

extern "C" int tq_quantized_matmul_noalloc(const void* x, const void* codes, const void* scales,
                                           const void* biases, int64_t m, int64_t w_rows,
                                           int64_t w_cols, int transpose, int group_size,
                                           int bits, void* y, void* stream) {
  using namespace tq;
  Args a{x, codes, scales, biases, nullptr, nullptr, nullptr, m, w_rows, w_cols,
         transpose, group_size, bits, 0, y};
  int rc = validate(a);
  if (rc) return rc;
  rc = validate_ptrs(a);
  if (rc) return rc;
  if (m == 0 || w_rows == 0 || w_cols == 0) return TQ_OK;
  const Plan pl = make_plan(a, true);
  if (pl.ws_bytes > kNoAllocScratchBytes)
    return fail(TQ_ERR_INVALID,
                "tq_quantized_matmul_noalloc: this shape needs %zu bytes of split-K scratch, "
                "more than the fixed %zu-byte array (use tq_quantized_matmul_ws)",
                pl.ws_bytes, kNoAllocScratchBytes);
  // Every partial the reduce reads is written by the GEMM of the same call
  // first, so the array needs no clearing between calls.
  rc = noalloc_scratch(&a.ws);
  if (rc) return rc;
  a.ws_bytes = kNoAllocScratchBytes;
  return run(a, stream);
}
