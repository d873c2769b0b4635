// Grouped-query scaled dot-product attention on the tensor cores: the
// decoder's attention node (causal, no mask tensor; engine/src/interp.rs:405-432,
// lib/torobi/models/llama.rb:297-316), forward and backward.
//
// Layout: q [batch, seq, heads, dim], k and v [batch, seq, kv_heads, dim],
// bf16, contiguous -- the projections' output as it stands, so no transpose
// copy sits on either side.  Query head h reads key/value head
// h / (heads / kv_heads).  o has q's layout; lse [batch, heads, seq] f32 is
// the natural-log log-sum-exp of each query row's scaled scores, kept for the
// backward.  dim is 64 or 128.
//
// The forward and the backward kernels are described where they start below.
#include <cuda_bf16.h>

#include <cmath>
#include <cstdlib>
#include <type_traits>

#include "tq_ptx.cuh"
#include "tq_runtime.h"

namespace tq {
namespace {

constexpr int kTile = 128;  // query rows and key rows per tile
constexpr float kLog2e = 1.4426950408889634f;
constexpr float kLn2 = 0.6931471805599453f;
constexpr float kRescaleLog2 = 8.0f;  // move m only when the row max grows by > 2^8

// 2^x on the FMA pipe, for a share of the softmax's exponentials (the MUFU
// unit alone would take as long as the tile's MMAs).  Range reduction by the
// round-to-nearest of x + 1.5 * 2^23 (n = nearest integer, f = x - n in
// [-0.5, 0.5]), 2^f by a cubic least-squares fit in relative error (fitted for
// this kernel; max relative error 7.5e-5 in f32, below bf16's 2^-9), and n
// added to the exponent field.  x is clamped at -125 so that the result stays
// a normal number.
__device__ __forceinline__ float exp2_poly(float x) {
  x = fmaxf(x, -125.0f);
  const float t = __fadd_rn(x, 12582912.0f);
  const float f = __fsub_rn(x, __fsub_rn(t, 12582912.0f));
  float p = fmaf(0.055174145847558975f, f, 0.24261757731437683f);
  p = fmaf(p, f, 0.6932610869407654f);
  p = fmaf(p, f, 0.9999275803565979f);
  return __uint_as_float(__float_as_uint(p) + (__float_as_uint(t) << 23));
}

struct AttnShape {
  int batch, seq, heads, kv_heads, group, n_tiles;
  int causal;
  float scale_log2;  // softmax scale * log2(e)
};

// ------------------------------------------------------------------ forward --
//
// One CTA per pair of adjacent 128-query tiles (2p, 2p + 1) of one head and
// sequence, heaviest causal pairs first; both tiles share every key/value
// tile the pair needs (tile 2p stops one key tile earlier under the mask).
//   warp 0       TMA: both query tiles once, key and value tiles through a ring
//   warp 1       one thread issues every tcgen05 MMA
//   warp 2       allocates / frees the 512 TMEM columns
//   warps 4-7    softmax of query tile 0 (thread i owns row i, TMEM lane i)
//   warps 8-11   softmax of query tile 1
// TMEM: S_0 | S_1 (128 f32 columns each) | O_0 | O_1 (dim columns each).  The
// softmax writes P_w (bf16 pairs, 64 columns) over the first half of S_w,
// chunk by chunk after reading it.  MMA issue order per key tile j:
//   PV_0(j) = O_0 += P_0(j) V_j,  S_0(j+1) = Q_0 K_{j+1}^T,
//   PV_1(j),                      S_1(j+1)
// so one tile's next scores are computed while the other tile's softmax
// runs.  S_w(j+1) overwrites P_w(j) right after PV_w(j) reads it: tcgen05.mma
// operations issued by one thread execute in issue order.
// The softmax reads each row twice from TMEM in 32-column chunks (maximum,
// then exponentials), which keeps the two softmax warpgroups within the
// 168 registers a 384-thread CTA has per thread.

template <int D>
struct FwdCfg {
  static_assert(D == 64 || D == 128, "head dim");
  static constexpr int SLABS = D / 64;            // 128-byte swizzle atoms along dim
  static constexpr int SLAB_BYTES = kTile * 128;  // 128 rows x 64 bf16
  static constexpr int TILE_BYTES = SLABS * SLAB_BYTES;
  // Key tiles are needed a step before value tiles, so their ring is deeper.
  static constexpr int KST = D == 128 ? 3 : 4;
  static constexpr int VST = D == 128 ? 2 : 4;
  static constexpr int Q_OFF = 0;  // two query tiles
  static constexpr int K_OFF = 2 * TILE_BYTES;
  static constexpr int V_OFF = K_OFF + KST * TILE_BYTES;
  static constexpr int BAR_OFF = V_OFF + VST * TILE_BYTES;
  // q_full, k_full[KST], k_empty[KST], v_full[VST], v_empty[VST], s_full[2],
  // p_ready[2], o_done[2]; then the TMEM slot
  static constexpr int NBAR = 1 + 2 * KST + 2 * VST + 6;
  static constexpr int SMEM = 1024 + BAR_OFF + 8 * (NBAR + 1);
  static constexpr int S_COL = 0;    // S_w (and P_w) at 128 w
  static constexpr int O_COL = 256;  // O_w at 256 + D w
  static constexpr int TMEM_COLS = 512;
  static_assert(O_COL + 2 * D <= TMEM_COLS, "tensor memory map");
  static_assert(SMEM <= 232448, "shared memory per CTA");
};

struct FwdParams {
  AttnShape sh;
  int n_pairs;
  uint16_t* out;
  float* lse;
  int* status;
};

template <int D>
__global__ void __launch_bounds__(384, 1)
    attn_fwd_kernel(const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_k,
                    const __grid_constant__ CUtensorMap tm_v, const FwdParams p) {
  using C = FwdCfg<D>;
  constexpr int KST = C::KST;
  constexpr int VST = C::VST;
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw = smem_u32(smem_raw);
  const uint32_t base = (raw + 1023u) & ~1023u;
  uint8_t* const gbase = smem_raw + (base - raw);
  auto q_s = [&](int w) { return base + C::Q_OFF + w * C::TILE_BYTES; };
  auto k_s = [&](int s) { return base + C::K_OFF + s * C::TILE_BYTES; };
  auto v_s = [&](int s) { return base + C::V_OFF + s * C::TILE_BYTES; };
  const uint32_t bars = base + C::BAR_OFF;
  const uint32_t q_full = bars;
  auto k_full = [&](int s) { return bars + 8u * (1 + s); };
  auto k_empty = [&](int s) { return bars + 8u * (1 + KST + s); };
  auto v_full = [&](int s) { return bars + 8u * (1 + 2 * KST + s); };
  auto v_empty = [&](int s) { return bars + 8u * (1 + 2 * KST + VST + s); };
  constexpr int X = 1 + 2 * KST + 2 * VST;
  // Per query tile w, each completing once per key tile j (phase j):
  // s_full (S_w(j) landed), p_ready (P_w(j) written, O_w rescaled), o_done
  // (PV_w(j) finished).  S_w(j+1) is only issued after p_ready's phase j, so
  // no waiter is ever two phases behind.
  auto s_full = [&](int w) { return bars + 8u * (X + w); };
  auto p_ready = [&](int w) { return bars + 8u * (X + 2 + w); };
  auto o_done = [&](int w) { return bars + 8u * (X + 4 + w); };
  const uint32_t tmem_slot = bars + 8u * C::NBAR;
  volatile uint32_t* tmem_slot_ptr =
      reinterpret_cast<volatile uint32_t*>(gbase + (tmem_slot - base));

  const AttnShape& sh = p.sh;
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int bh_count = sh.batch * sh.heads;
  const int bh = blockIdx.x % bh_count;
  const int pair = p.n_pairs - 1 - static_cast<int>(blockIdx.x / bh_count);
  const int b = bh / sh.heads;
  const int h = bh % sh.heads;
  const int hk = h / sh.group;
  const int t0 = 2 * pair;                             // first query tile
  const bool has1 = t0 + 1 < sh.n_tiles;               // second query tile exists
  const int n_kv0 = sh.causal ? t0 + 1 : sh.n_tiles;  // key tiles of query tile 0
  const int n_kv1 = has1 ? (sh.causal ? t0 + 2 : sh.n_tiles) : 0;
  const int n_kv = n_kv0 > n_kv1 ? n_kv0 : n_kv1;
  auto nkv_of = [&](int w) { return w == 0 ? n_kv0 : n_kv1; };

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    for (int s = 0; s < KST; ++s) {
      mbar_init(k_full(s), 1);
      mbar_init(k_empty(s), 1);
    }
    for (int s = 0; s < VST; ++s) {
      mbar_init(v_full(s), 1);
      mbar_init(v_empty(s), 1);
    }
    for (int w = 0; w < 2; ++w) {
      mbar_init(s_full(w), 1);
      mbar_init(p_ready(w), 4);
      mbar_init(o_done(w), 1);
    }
    fence_mbar_init();
  }
  if (warp == 2) {
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
    // ------------------------------------------------------------- TMA
    if (elect_one_sync()) {
      tma_prefetch_desc(&tm_q);
      tma_prefetch_desc(&tm_k);
      tma_prefetch_desc(&tm_v);
      mbar_arrive_expect_tx(q_full, (has1 ? 2 : 1) * C::TILE_BYTES);
      for (int w = 0; w < (has1 ? 2 : 1); ++w)
        for (int sl = 0; sl < C::SLABS; ++sl)
          tma_load_4d(q_s(w) + sl * C::SLAB_BYTES, &tm_q, q_full, sl * 64, h, (t0 + w) * kTile, b);
      int nk = 0, nv = 0;  // tiles issued
      // Key tile j + 1 is issued ahead of value tile j (the MMA wants K_{j+1}
      // for the next scores before it wants V_j).
      auto load_k = [&](int j) -> bool {
        const int s = j % KST;
        if (!mbar_wait(k_empty(s), ((j / KST) & 1) ^ 1, p.status)) return false;
        mbar_arrive_expect_tx(k_full(s), C::TILE_BYTES);
        for (int sl = 0; sl < C::SLABS; ++sl)
          tma_load_4d(k_s(s) + sl * C::SLAB_BYTES, &tm_k, k_full(s), sl * 64, hk, j * kTile, b);
        ++nk;
        return true;
      };
      bool ok = n_kv > 0 ? load_k(0) : true;
      for (int j = 0; j < n_kv && ok; ++j) {
        if (j + 1 < n_kv && !load_k(j + 1)) break;
        const int s = j % VST;
        if (!mbar_wait(v_empty(s), ((j / VST) & 1) ^ 1, p.status)) break;
        mbar_arrive_expect_tx(v_full(s), C::TILE_BYTES);
        for (int sl = 0; sl < C::SLABS; ++sl)
          tma_load_4d(v_s(s) + sl * C::SLAB_BYTES, &tm_v, v_full(s), sl * 64, hk, j * kTile, b);
        ++nv;
      }
      // Never leave a copy in flight.
      mbar_wait(q_full, 0, p.status);
      for (int j = nk - KST < 0 ? 0 : nk - KST; j < nk; ++j)
        mbar_wait(k_full(j % KST), (j / KST) & 1, p.status);
      for (int j = nv - VST < 0 ? 0 : nv - VST; j < nv; ++j)
        mbar_wait(v_full(j % VST), (j / VST) & 1, p.status);
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------- MMA
    if (elect_one_sync()) {
      constexpr uint32_t idesc_s = make_idesc_bf16(kTile, kTile, false, false);
      constexpr uint32_t idesc_o = make_idesc_bf16(kTile, D, false, true);
      bool ok = mbar_wait(q_full, 0, p.status);
      // S_w(j) = Q_w K_j^T into S_w.
      auto issue_s = [&](int w, int j) {
        const int s = j % KST;
        const uint32_t d = tmem + C::S_COL + w * kTile;
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk) {
          const uint32_t off = (kk >> 2) * C::SLAB_BYTES + (kk & 3) * 32;
          umma_bf16(d, make_sdesc(q_s(w) + off, 16, 1024, kSw128),
                    make_sdesc(k_s(s) + off, 16, 1024, kSw128), idesc_s, kk > 0);
        }
        umma_commit(s_full(w));
      };
      // O_w += P_w(j) V_j, P_w from the first 64 columns of S_w.
      auto issue_pv = [&](int w, int j) {
        const int s = j % VST;
#pragma unroll
        for (int kk = 0; kk < kTile / 16; ++kk)
          umma_bf16_ts(tmem + C::O_COL + w * D, tmem + C::S_COL + w * kTile + kk * 8,
                       make_sdesc(v_s(s) + kk * 2048, C::SLAB_BYTES, 1024, kSw128), idesc_o,
                       (j > 0 || kk > 0) ? 1u : 0u);
        umma_commit(o_done(w));
      };
      // Key tile 0: both tiles' scores.
      if (ok) ok = mbar_wait(k_full(0), 0, p.status);
      if (ok) {
        tc_fence_after();
        issue_s(0, 0);
        if (n_kv1 > 0) issue_s(1, 0);
        umma_commit(k_empty(0));
      }
      for (int j = 0; j < n_kv && ok; ++j) {
        const int s = j % VST;
        const bool next = j + 1 < n_kv;
        if (next) {
          ok = mbar_wait(k_full((j + 1) % KST), ((j + 1) / KST) & 1, p.status);
          if (!ok) break;
        }
        ok = mbar_wait(v_full(s), (j / VST) & 1, p.status);
        if (!ok) break;
        for (int w = 0; w < 2 && ok; ++w) {
          if (j >= nkv_of(w)) continue;
          ok = mbar_wait(p_ready(w), j & 1, p.status);
          if (!ok) break;
          tc_fence_after();
          issue_pv(w, j);
          if (j + 1 < nkv_of(w)) issue_s(w, j + 1);
        }
        if (!ok) break;
        umma_commit(v_empty(s));
        if (next) umma_commit(k_empty((j + 1) % KST));
      }
      // Nothing may outlive the CTA's TMEM: wait for each tile's last PV.
      for (int w = 0; w < 2; ++w)
        if (nkv_of(w) > 0) mbar_wait(o_done(w), (nkv_of(w) - 1) & 1, p.status);
    }
  } else if (warp >= 4) {
    // --------------------------------------------------------- softmax
    const int w = (warp - 4) >> 2;  // query tile of this warpgroup
    const int quad = warp & 3;
    const int row = quad * 32 + lane;
    const int qw0 = (t0 + w) * kTile;
    const int qpos = qw0 + row;
    const int nk = nkv_of(w);
    const uint32_t lrow = tmem + (static_cast<uint32_t>(quad * 32) << 16);
    const uint32_t scol = lrow + C::S_COL + w * kTile;
    const uint32_t ocol = lrow + C::O_COL + w * D;
    const float c = sh.scale_log2;
    float m = -INFINITY;
    float l = 0.0f;
    bool ok = true;
    for (int j = 0; j < nk; ++j) {
      ok = mbar_wait(s_full(w), j & 1, p.status);
      if (!ok) break;
      tc_fence_after();
      const int kv0 = j * kTile;
      int lim = kTile - 1;  // last column of this key tile that counts for the row
      if ((sh.causal && kv0 + kTile - 1 > qw0) || kv0 + kTile > sh.seq) {
        lim = sh.seq - 1 - kv0;
        if (sh.causal && qpos - kv0 < lim) lim = qpos - kv0;
      }
      // Only the diagonal key tile (causal) and the one past seq need a mask:
      // both passes come in a masked and an unmasked form.
      const bool masked = lim < kTile - 1 || (sh.causal && kv0 + kTile - 1 > qw0);
      // Pass 1: the row maximum (eight interleaved chains, then a tree).
      float m8[8];
#pragma unroll
      for (int e = 0; e < 8; ++e) m8[e] = -INFINITY;
      auto pass1 = [&](auto mask_tag) {
        constexpr bool M = decltype(mask_tag)::value;
#pragma unroll
        for (int c4 = 0; c4 < kTile / 32; ++c4) {
          uint32_t r[32];
          tmem_ld_32x32b_x32(scol + c4 * 32, r);
          tmem_ld_wait();
#pragma unroll
          for (int i = 0; i < 32; ++i)
            if (!M || c4 * 32 + i <= lim) m8[i & 7] = fmaxf(m8[i & 7], __uint_as_float(r[i]));
        }
      };
      if (masked)
        pass1(std::true_type{});
      else
        pass1(std::false_type{});
      const float mx = fmaxf(fmaxf(fmaxf(m8[0], m8[1]), fmaxf(m8[2], m8[3])),
                             fmaxf(fmaxf(m8[4], m8[5]), fmaxf(m8[6], m8[7])));
      const float m_new = fmaxf(m, mx * c);
      if (j == 0) {
        m = m_new;
      } else if (__any_sync(0xffffffffu, m_new > m + kRescaleLog2)) {
        // Move m and rescale this row of O_w.  PV_w(j-1) has finished: S_w(j)
        // was issued after it.
        const float f = m == -INFINITY ? 0.0f : ex2_approx(m - m_new);
        ok = mbar_wait(o_done(w), (j - 1) & 1, p.status);
        if (!ok) break;
        tc_fence_after();
#pragma unroll 1
        for (int c4 = 0; c4 < D / 16; ++c4) {
          uint32_t o[16];
          tmem_ld_32x32b_x16(ocol + c4 * 16, o);
          tmem_ld_wait();
#pragma unroll
          for (int i = 0; i < 16; ++i) o[i] = __float_as_uint(__uint_as_float(o[i]) * f);
          tmem_st_32x32b_x16(ocol + c4 * 16, o);
        }
        tmem_st_wait();
        l *= f;
        m = m_new;
      }
      const float mref = m == -INFINITY ? 0.0f : m;
      // Pass 2: P = exp2(S c - m), three of four exponentials on the MUFU
      // unit and one on the FMA pipe, written as bf16 pairs over the first
      // half of S_w (chunk k's 16 columns lie in chunks already read); the
      // next chunk's load is in flight while one is computed.
      float a4[4] = {0.0f, 0.0f, 0.0f, 0.0f};
      auto pass2 = [&](auto mask_tag) {
        constexpr bool M = decltype(mask_tag)::value;
        uint32_t rb[2][32];
        tmem_ld_32x32b_x32(scol, rb[0]);
        tmem_ld_wait();
#pragma unroll
        for (int c4 = 0; c4 < kTile / 32; ++c4) {
          if (c4 + 1 < kTile / 32) tmem_ld_32x32b_x32(scol + (c4 + 1) * 32, rb[(c4 + 1) & 1]);
          const uint32_t(&r)[32] = rb[c4 & 1];
          uint32_t pk[16];
#pragma unroll
          for (int i = 0; i < 32; i += 4) {
            const int col = c4 * 32 + i;
            float p0 = ex2_approx(fmaf(__uint_as_float(r[i]), c, -mref));
            float p1 = ex2_approx(fmaf(__uint_as_float(r[i + 1]), c, -mref));
            float p2 = ex2_approx(fmaf(__uint_as_float(r[i + 2]), c, -mref));
            float p3 = exp2_poly(fmaf(__uint_as_float(r[i + 3]), c, -mref));
            if (M) {
              if (col > lim) p0 = 0.0f;
              if (col + 1 > lim) p1 = 0.0f;
              if (col + 2 > lim) p2 = 0.0f;
              if (col + 3 > lim) p3 = 0.0f;
            }
            a4[0] += p0;
            a4[1] += p1;
            a4[2] += p2;
            a4[3] += p3;
            pk[i / 2] = pack_bf16x2_f32(p0, p1);
            pk[i / 2 + 1] = pack_bf16x2_f32(p2, p3);
          }
          tmem_st_32x32b_x16(scol + c4 * 16, pk);
          if (c4 + 1 < kTile / 32) tmem_ld_wait();
        }
      };
      if (masked)
        pass2(std::true_type{});
      else
        pass2(std::false_type{});
      l += (a4[0] + a4[1]) + (a4[2] + a4[3]);
      tmem_st_wait();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(p_ready(w));
    }
    if (ok && nk > 0) ok = mbar_wait(o_done(w), (nk - 1) & 1, p.status);
    tc_fence_after();
    if (ok && nk > 0) {
      const float inv = l > 0.0f ? 1.0f / l : 0.0f;
      const bool valid = qpos < sh.seq;
      uint16_t* orow = p.out + ((static_cast<size_t>(b) * sh.seq + qpos) * sh.heads + h) * D;
#pragma unroll
      for (int c4 = 0; c4 < D / 32; ++c4) {
        uint32_t o[32];
        tmem_ld_32x32b_x32(ocol + c4 * 32, o);
        tmem_ld_wait();
        uint32_t wd[16];
#pragma unroll
        for (int i = 0; i < 16; ++i)
          wd[i] = pack_bf16x2_f32(__uint_as_float(o[2 * i]) * inv,
                                  __uint_as_float(o[2 * i + 1]) * inv);
        if (valid) {
          uint4* dst = reinterpret_cast<uint4*>(orow + c4 * 32);
#pragma unroll
          for (int i = 0; i < 4; ++i)
            dst[i] = make_uint4(wd[4 * i], wd[4 * i + 1], wd[4 * i + 2], wd[4 * i + 3]);
        }
      }
      if (valid)
        p.lse[(static_cast<size_t>(b) * sh.heads + h) * sh.seq + qpos] =
            l > 0.0f ? (m + log2f(l)) * kLn2 : -INFINITY;
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 2) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc(tmem, C::TMEM_COLS);
  }
}

// ----------------------------------------------------------------- backward --
//
// Three launches, no atomics (the gradients are deterministic):
//   prep   per query row: lse2 = lse * log2(e) and delta = sum_d dO * O (f32),
//          each (sequence, head)'s rows padded to whole 128-row tiles (padding
//          rows: lse2 = +inf, so their probabilities are 0, and delta = 0);
//   dq     one CTA per (128-query tile, head, sequence), key tiles of 64
//          (two compute warpgroups, each half of every tile's columns):
//            S = Q K_j^T, dP = dO V_j^T (tensor memory, double-buffered),
//            dS = P * (dP - delta) with P = exp2(S c - lse2)  (compute warps),
//            dQ += dS K_j  (dS written back to tensor memory, A from TMEM);
//   dkv    one CTA per (128-key tile, key/value head, sequence), looping over
//          the query heads that share the key/value head and their 64-row
//          query tiles (two compute warpgroups, each half of every tile's
//          columns):
//            S^T = K Q_i^T, dP^T = V dO_i^T, P^T and dS^T (compute warps, into
//            shared memory as K-major operands), dV += P^T dO_i, dK += dS^T Q_i.
// dQ and dK are scaled by the softmax scale once at the end.  As in the
// forward, every barrier used per tile t comes in two (t's parity) and a
// parity wait is never more than one phase behind.

constexpr int kHalf = 64;  // the streamed tile of the backward kernels

struct PrepParams {
  const uint16_t* out;
  const uint16_t* dout;
  const float* lse;
  float* lse2;
  float* delta;
  int batch, seq, heads, seq_pad, dim;
};

// Eight lanes per row, dim / 8 elements each.
__global__ void __launch_bounds__(256) attn_bwd_prep_kernel(const PrepParams p) {
  griddep_wait();
  griddep_launch_dependents();
  const long long gid = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x;
  const long long row = gid >> 3;
  const int sub = threadIdx.x & 7;
  const long long rows = static_cast<long long>(p.batch) * p.heads * p.seq_pad;
  const bool in = row < rows;
  const int bh = in ? static_cast<int>(row / p.seq_pad) : 0;
  const int s = in ? static_cast<int>(row % p.seq_pad) : 0;
  const bool real = in && s < p.seq;
  float acc = 0.0f;
  if (real) {
    const int b = bh / p.heads, h = bh % p.heads;
    const int per = p.dim / 8;
    const size_t off = ((static_cast<size_t>(b) * p.seq + s) * p.heads + h) * p.dim + sub * per;
    for (int c = 0; c < per; c += 8) {
      const uint4 o = *reinterpret_cast<const uint4*>(p.out + off + c);
      const uint4 d = *reinterpret_cast<const uint4*>(p.dout + off + c);
      const uint32_t ow[4] = {o.x, o.y, o.z, o.w};
      const uint32_t dw[4] = {d.x, d.y, d.z, d.w};
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        acc = fmaf(__uint_as_float(ow[i] << 16), __uint_as_float(dw[i] << 16), acc);
        acc = fmaf(__uint_as_float(ow[i] & 0xFFFF0000u), __uint_as_float(dw[i] & 0xFFFF0000u),
                   acc);
      }
    }
  }
  acc += __shfl_xor_sync(0xffffffffu, acc, 1);
  acc += __shfl_xor_sync(0xffffffffu, acc, 2);
  acc += __shfl_xor_sync(0xffffffffu, acc, 4);
  if (in && sub == 0) {
    float l2 = INFINITY;
    if (real) {
      const float l = p.lse[static_cast<size_t>(bh) * p.seq + s];
      l2 = l == -INFINITY ? INFINITY : l * kLog2e;
    }
    p.lse2[row] = l2;
    p.delta[row] = real ? acc : 0.0f;
  }
}

struct BwdParams {
  AttnShape sh;
  int seq_pad;
  float scale;
  const float* lse2;
  const float* delta;
  uint16_t* dq;
  uint16_t* dk;
  uint16_t* dv;
  int* status;
};

template <int D>
struct DqCfg {
  static constexpr int SLABS = D / 64;
  static constexpr int QSLAB = kTile * 128;  // 128 rows x 64 bf16
  static constexpr int QTILE = SLABS * QSLAB;
  static constexpr int KSLAB = kHalf * 128;  // 64 rows x 64 bf16
  static constexpr int KTILE = SLABS * KSLAB;
  static constexpr int KST = D == 128 ? 5 : 8;
  static constexpr int VST = KST;
  static constexpr int Q_OFF = 0;
  static constexpr int DO_OFF = QTILE;
  static constexpr int K_OFF = 2 * QTILE;
  static constexpr int V_OFF = K_OFF + KST * KTILE;
  static constexpr int BAR_OFF = V_OFF + VST * KTILE;
  // q_full, k_full[KST], k_empty[KST], v_full[VST], v_empty[VST], s_full[2],
  // s_free[2], ds_ready[2], dq_full; then the TMEM slot
  static constexpr int NBAR = 1 + 2 * KST + 2 * VST + 7;
  static constexpr int SMEM_USED = 1024 + BAR_OFF + 8 * (NBAR + 1);
  // At least ~116 KB, so that one CTA (and its 512 TMEM columns) fits an SM.
  static constexpr int SMEM = SMEM_USED > 118784 ? SMEM_USED : 118784;
  static constexpr int S_COL = 0;     // S_b at 64 b
  static constexpr int DP_COL = 128;  // dP_b at 128 + 64 b
  static constexpr int DQ_COL = 256;
  static constexpr int DS_COL = 256 + D;  // dS_b (bf16 pairs) at DS_COL + 32 b
  static constexpr int TMEM_COLS = 512;
  static_assert(DS_COL + 64 <= TMEM_COLS, "tensor memory map");
  static_assert(SMEM <= 232448, "shared memory per CTA");
};

template <int D>
__global__ void __launch_bounds__(384, 1)
    attn_bwd_dq_kernel(const __grid_constant__ CUtensorMap tm_q,
                       const __grid_constant__ CUtensorMap tm_do,
                       const __grid_constant__ CUtensorMap tm_k,
                       const __grid_constant__ CUtensorMap tm_v, const BwdParams p) {
  using C = DqCfg<D>;
  constexpr int KST = C::KST;
  constexpr int VST = C::VST;
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw = smem_u32(smem_raw);
  const uint32_t base = (raw + 1023u) & ~1023u;
  uint8_t* const gbase = smem_raw + (base - raw);
  const uint32_t q_s = base + C::Q_OFF;
  const uint32_t do_s = base + C::DO_OFF;
  auto k_s = [&](int s) { return base + C::K_OFF + s * C::KTILE; };
  auto v_s = [&](int s) { return base + C::V_OFF + s * C::KTILE; };
  const uint32_t bars = base + C::BAR_OFF;
  const uint32_t q_full = bars;
  auto k_full = [&](int s) { return bars + 8u * (1 + s); };
  auto k_empty = [&](int s) { return bars + 8u * (1 + KST + s); };
  auto v_full = [&](int s) { return bars + 8u * (1 + 2 * KST + s); };
  auto v_empty = [&](int s) { return bars + 8u * (1 + 2 * KST + VST + s); };
  constexpr int X = 1 + 2 * KST + 2 * VST;
  auto s_full = [&](int b) { return bars + 8u * (X + b); };
  auto s_free = [&](int b) { return bars + 8u * (X + 2 + b); };
  auto ds_ready = [&](int b) { return bars + 8u * (X + 4 + b); };
  const uint32_t dq_full = bars + 8u * (X + 6);
  const uint32_t tmem_slot = bars + 8u * C::NBAR;
  volatile uint32_t* tmem_slot_ptr =
      reinterpret_cast<volatile uint32_t*>(gbase + (tmem_slot - base));

  const AttnShape& sh = p.sh;
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int bh_count = sh.batch * sh.heads;
  const int bh = blockIdx.x % bh_count;
  const int qt = sh.n_tiles - 1 - static_cast<int>(blockIdx.x / bh_count);
  const int b = bh / sh.heads;
  const int h = bh % sh.heads;
  const int hk = h / sh.group;
  const int q0 = qt * kTile;
  const int n_half = (sh.seq + kHalf - 1) / kHalf;
  int n_kv = n_half;
  if (sh.causal && (q0 + kTile - 1) / kHalf + 1 < n_kv) n_kv = (q0 + kTile - 1) / kHalf + 1;

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    for (int s = 0; s < KST; ++s) {
      mbar_init(k_full(s), 1);
      mbar_init(k_empty(s), 1);
    }
    for (int s = 0; s < VST; ++s) {
      mbar_init(v_full(s), 1);
      mbar_init(v_empty(s), 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(s_full(i), 1);
      mbar_init(s_free(i), 8);
      mbar_init(ds_ready(i), 8);
    }
    mbar_init(dq_full, 1);
    fence_mbar_init();
  }
  if (warp == 2) {
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
    // ------------------------------------------------------------- TMA
    if (elect_one_sync()) {
      tma_prefetch_desc(&tm_q);
      tma_prefetch_desc(&tm_do);
      tma_prefetch_desc(&tm_k);
      tma_prefetch_desc(&tm_v);
      mbar_arrive_expect_tx(q_full, 2 * C::QTILE);
      for (int sl = 0; sl < C::SLABS; ++sl) {
        tma_load_4d(q_s + sl * C::QSLAB, &tm_q, q_full, sl * 64, h, q0, b);
        tma_load_4d(do_s + sl * C::QSLAB, &tm_do, q_full, sl * 64, h, q0, b);
      }
      int nk = 0, nv = 0;
      for (int j = 0; j < n_kv; ++j) {
        const int ks = j % KST, vs = j % VST;
        if (!mbar_wait(k_empty(ks), ((j / KST) & 1) ^ 1, p.status)) break;
        mbar_arrive_expect_tx(k_full(ks), C::KTILE);
        for (int sl = 0; sl < C::SLABS; ++sl)
          tma_load_4d(k_s(ks) + sl * C::KSLAB, &tm_k, k_full(ks), sl * 64, hk, j * kHalf, b);
        ++nk;
        if (!mbar_wait(v_empty(vs), ((j / VST) & 1) ^ 1, p.status)) break;
        mbar_arrive_expect_tx(v_full(vs), C::KTILE);
        for (int sl = 0; sl < C::SLABS; ++sl)
          tma_load_4d(v_s(vs) + sl * C::KSLAB, &tm_v, v_full(vs), sl * 64, hk, j * kHalf, b);
        ++nv;
      }
      mbar_wait(q_full, 0, p.status);
      for (int j = nk - KST < 0 ? 0 : nk - KST; j < nk; ++j)
        mbar_wait(k_full(j % KST), (j / KST) & 1, p.status);
      for (int j = nv - VST < 0 ? 0 : nv - VST; j < nv; ++j)
        mbar_wait(v_full(j % VST), (j / VST) & 1, p.status);
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------- MMA
    if (elect_one_sync()) {
      constexpr uint32_t idesc_s = make_idesc_bf16(kTile, kHalf, false, false);
      constexpr uint32_t idesc_dq = make_idesc_bf16(kTile, D, false, true);
      bool ok = mbar_wait(q_full, 0, p.status);
      // dQ += dS_j K_j: A = dS_j from tensor memory, B = K_j MN-major (N = dim).
      auto issue_dq = [&](int j) -> bool {
        if (!mbar_wait(ds_ready(j & 1), (j >> 1) & 1, p.status)) return false;
        tc_fence_after();
        const int ks = j % KST;
#pragma unroll
        for (int kk = 0; kk < kHalf / 16; ++kk)
          umma_bf16_ts(tmem + C::DQ_COL, tmem + C::DS_COL + (j & 1) * 32 + kk * 8,
                       make_sdesc(k_s(ks) + kk * 2048, C::KSLAB, 1024, kSw128), idesc_dq,
                       (j > 0 || kk > 0) ? 1u : 0u);
        umma_commit(k_empty(ks));
        return true;
      };
      int done_dq = 0;
      for (int j = 0; j < n_kv && ok; ++j) {
        const int ks = j % KST, vs = j % VST;
        ok = mbar_wait(k_full(ks), (j / KST) & 1, p.status) &&
             mbar_wait(v_full(vs), (j / VST) & 1, p.status) &&
             (j < 2 || mbar_wait(s_free(j & 1), ((j - 2) >> 1) & 1, p.status));
        if (!ok) break;
        tc_fence_after();
        const uint32_t sd = tmem + C::S_COL + (j & 1) * kHalf;
        const uint32_t pd = tmem + C::DP_COL + (j & 1) * kHalf;
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk) {
          const uint32_t qoff = (kk >> 2) * C::QSLAB + (kk & 3) * 32;
          const uint32_t koff = (kk >> 2) * C::KSLAB + (kk & 3) * 32;
          umma_bf16(sd, make_sdesc(q_s + qoff, 16, 1024, kSw128),
                    make_sdesc(k_s(ks) + koff, 16, 1024, kSw128), idesc_s, kk > 0);
        }
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk) {
          const uint32_t qoff = (kk >> 2) * C::QSLAB + (kk & 3) * 32;
          const uint32_t koff = (kk >> 2) * C::KSLAB + (kk & 3) * 32;
          umma_bf16(pd, make_sdesc(do_s + qoff, 16, 1024, kSw128),
                    make_sdesc(v_s(vs) + koff, 16, 1024, kSw128), idesc_s, kk > 0);
        }
        umma_commit(s_full(j & 1));
        umma_commit(v_empty(vs));
        if (j >= 1) {
          ok = issue_dq(j - 1);
          if (ok) done_dq = j;
        }
      }
      if (ok && n_kv > 0 && issue_dq(n_kv - 1)) done_dq = n_kv;
      umma_commit(dq_full);
      // Nothing may outlive the CTA's TMEM: the last commit covers every MMA.
      mbar_wait(dq_full, 0, p.status);
      (void)done_dq;
    }
  } else if (warp >= 4) {
    // ------------------------------------------------------ compute warps
    // Two warpgroups on the same 128 rows: warps 4-7 take key columns 0-31
    // of each 64-key tile, warps 8-11 columns 32-63 (the gradient is
    // elementwise given the row's lse and delta); likewise halves of dQ.
    const int half = (warp - 4) >> 2;
    const int quad = warp & 3;
    const int row = quad * 32 + lane;
    const int qpos = q0 + row;
    const uint32_t lrow = tmem + (static_cast<uint32_t>(quad * 32) << 16);
    const size_t srow = static_cast<size_t>(bh) * p.seq_pad + qpos;
    const float lse2 = p.lse2[srow];
    const float dl = p.delta[srow];
    const float c = sh.scale_log2;
    bool ok = true;
    for (int j = 0; j < n_kv; ++j) {
      ok = mbar_wait(s_full(j & 1), (j >> 1) & 1, p.status);
      if (!ok) break;
      tc_fence_after();
      uint32_t sv[32], dv[32];
      tmem_ld_32x32b_x32(lrow + C::S_COL + (j & 1) * kHalf + half * 32, sv);
      tmem_ld_32x32b_x32(lrow + C::DP_COL + (j & 1) * kHalf + half * 32, dv);
      tmem_ld_wait();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(s_free(j & 1));
      const int kv0 = j * kHalf + half * 32;
      int lim = 31;  // last column of this half tile that counts
      if ((sh.causal && kv0 + 31 > q0) || kv0 + 32 > sh.seq) {
        lim = sh.seq - 1 - kv0;
        if (sh.causal && qpos - kv0 < lim) lim = qpos - kv0;
      }
      uint32_t pk[16];
#pragma unroll
      for (int i = 0; i < 32; i += 2) {
        float p0 = ex2_approx(fmaf(__uint_as_float(sv[i]), c, -lse2));
        float p1 = (i & 2) ? exp2_poly(fmaf(__uint_as_float(sv[i + 1]), c, -lse2))
                           : ex2_approx(fmaf(__uint_as_float(sv[i + 1]), c, -lse2));
        if (i > lim) p0 = 0.0f;
        if (i + 1 > lim) p1 = 0.0f;
        pk[i / 2] = pack_bf16x2_f32(p0 * (__uint_as_float(dv[i]) - dl),
                                    p1 * (__uint_as_float(dv[i + 1]) - dl));
      }
      tmem_st_32x32b_x16(lrow + C::DS_COL + (j & 1) * 32 + half * 16, pk);
      tmem_st_wait();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(ds_ready(j & 1));
    }
    if (ok) ok = mbar_wait(dq_full, 0, p.status);
    tc_fence_after();
    if (ok) {
      const bool valid = qpos < sh.seq;
      uint16_t* orow = p.dq + ((static_cast<size_t>(b) * sh.seq + qpos) * sh.heads + h) * D;
#pragma unroll
      for (int c4 = half * (D / 64); c4 < (half + 1) * (D / 64); ++c4) {
        uint32_t o[32];
        tmem_ld_32x32b_x32(lrow + C::DQ_COL + c4 * 32, o);
        tmem_ld_wait();
        uint32_t w[16];
#pragma unroll
        for (int i = 0; i < 16; ++i)
          w[i] = pack_bf16x2_f32(__uint_as_float(o[2 * i]) * p.scale,
                                 __uint_as_float(o[2 * i + 1]) * p.scale);
        if (valid) {
          uint4* dst = reinterpret_cast<uint4*>(orow + c4 * 32);
#pragma unroll
          for (int i = 0; i < 4; ++i)
            dst[i] = make_uint4(w[4 * i], w[4 * i + 1], w[4 * i + 2], w[4 * i + 3]);
        }
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 2) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc(tmem, C::TMEM_COLS);
  }
}

template <int D>
struct DkvCfg {
  static constexpr int SLABS = D / 64;
  static constexpr int KSLAB = kTile * 128;  // K_j, V_j: 128 rows x 64 bf16
  static constexpr int KTILE = SLABS * KSLAB;
  static constexpr int QSLAB = kHalf * 128;  // Q_i, dO_i: 64 rows x 64 bf16
  static constexpr int QTILE = SLABS * QSLAB;
  static constexpr int PTILE = kTile * 128;  // P^T or dS^T: 128 key rows x 64 queries bf16
  static constexpr int QST = D == 128 ? 3 : 6;
  static constexpr int STAT_BYTES = 2 * kHalf * 4;  // lse2 and delta of one query tile
  static constexpr int K_OFF = 0;
  static constexpr int V_OFF = KTILE;
  static constexpr int Q_OFF = 2 * KTILE;
  static constexpr int DO_OFF = Q_OFF + QST * QTILE;
  static constexpr int P_OFF = DO_OFF + QST * QTILE;
  static constexpr int DS_OFF = P_OFF + 2 * PTILE;
  static constexpr int STAT_OFF = DS_OFF + 2 * PTILE;
  static constexpr int BAR_OFF = STAT_OFF + QST * STAT_BYTES;
  // kv_full, q_full[QST], q_empty[QST], s_full[2], s_free[2], pds_ready[2],
  // acc_full; then the TMEM slot
  static constexpr int NBAR = 1 + 2 * QST + 7;
  static constexpr int SMEM = 1024 + BAR_OFF + 8 * (NBAR + 1);
  static constexpr int S_COL = 0;     // S^T_b at 64 b
  static constexpr int DP_COL = 128;  // dP^T_b at 128 + 64 b
  static constexpr int DV_COL = 256;
  static constexpr int DK_COL = 256 + D;
  static constexpr int TMEM_COLS = 512;
  static_assert(DK_COL + D <= TMEM_COLS, "tensor memory map");
  static_assert(SMEM <= 232448, "shared memory per CTA");
  static_assert(SMEM > 118784, "one CTA per SM");
};

template <int D>
__global__ void __launch_bounds__(384, 1)
    attn_bwd_dkv_kernel(const __grid_constant__ CUtensorMap tm_q,
                        const __grid_constant__ CUtensorMap tm_do,
                        const __grid_constant__ CUtensorMap tm_k,
                        const __grid_constant__ CUtensorMap tm_v, const BwdParams p) {
  using C = DkvCfg<D>;
  constexpr int QST = C::QST;
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw = smem_u32(smem_raw);
  const uint32_t base = (raw + 1023u) & ~1023u;
  uint8_t* const gbase = smem_raw + (base - raw);
  const uint32_t k_s = base + C::K_OFF;
  const uint32_t v_s = base + C::V_OFF;
  auto q_s = [&](int s) { return base + C::Q_OFF + s * C::QTILE; };
  auto do_s = [&](int s) { return base + C::DO_OFF + s * C::QTILE; };
  auto p_s = [&](int b) { return base + C::P_OFF + b * C::PTILE; };
  auto ds_s = [&](int b) { return base + C::DS_OFF + b * C::PTILE; };
  auto stat_s = [&](int s) { return base + C::STAT_OFF + s * C::STAT_BYTES; };
  const uint32_t bars = base + C::BAR_OFF;
  const uint32_t kv_full = bars;
  auto q_full = [&](int s) { return bars + 8u * (1 + s); };
  auto q_empty = [&](int s) { return bars + 8u * (1 + QST + s); };
  constexpr int X = 1 + 2 * QST;
  auto s_full = [&](int b) { return bars + 8u * (X + b); };
  auto s_free = [&](int b) { return bars + 8u * (X + 2 + b); };
  auto pds_ready = [&](int b) { return bars + 8u * (X + 4 + b); };
  const uint32_t acc_full = bars + 8u * (X + 6);
  const uint32_t tmem_slot = bars + 8u * C::NBAR;
  volatile uint32_t* tmem_slot_ptr =
      reinterpret_cast<volatile uint32_t*>(gbase + (tmem_slot - base));

  const AttnShape& sh = p.sh;
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int bk_count = sh.batch * sh.kv_heads;
  const int bk = blockIdx.x % bk_count;
  const int jt = static_cast<int>(blockIdx.x / bk_count);  // causal: key tile 0 has most work
  const int b = bk / sh.kv_heads;
  const int hk = bk % sh.kv_heads;
  const int kv0 = jt * kTile;
  const int n_half = (sh.seq + kHalf - 1) / kHalf;
  const int i0 = sh.causal ? kv0 / kHalf : 0;  // first query tile that sees this key tile
  const int nq = n_half - i0;
  const int T = sh.group * nq;

  if (threadIdx.x == 0) {
    mbar_init(kv_full, 1);
    for (int s = 0; s < QST; ++s) {
      mbar_init(q_full(s), 1);
      mbar_init(q_empty(s), 1 + 8);  // the MMAs' commit and the compute warps' stat reads
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(s_full(i), 1);
      mbar_init(s_free(i), 8);
      mbar_init(pds_ready(i), 8);
    }
    mbar_init(acc_full, 1);
    fence_mbar_init();
  }
  if (warp == 2) {
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
    // ------------------------------------------------------------- TMA
    if (elect_one_sync()) {
      tma_prefetch_desc(&tm_q);
      tma_prefetch_desc(&tm_do);
      tma_prefetch_desc(&tm_k);
      tma_prefetch_desc(&tm_v);
      mbar_arrive_expect_tx(kv_full, 2 * C::KTILE);
      for (int sl = 0; sl < C::SLABS; ++sl) {
        tma_load_4d(k_s + sl * C::KSLAB, &tm_k, kv_full, sl * 64, hk, kv0, b);
        tma_load_4d(v_s + sl * C::KSLAB, &tm_v, kv_full, sl * 64, hk, kv0, b);
      }
      int issued = 0;
      for (int t = 0; t < T; ++t) {
        const int s = t % QST;
        if (!mbar_wait(q_empty(s), ((t / QST) & 1) ^ 1, p.status)) break;
        const int h = hk * sh.group + t / nq;
        const int qq0 = (i0 + t % nq) * kHalf;
        const size_t srow = static_cast<size_t>(b * sh.heads + h) * p.seq_pad + qq0;
        mbar_arrive_expect_tx(q_full(s), 2 * C::QTILE + C::STAT_BYTES);
        for (int sl = 0; sl < C::SLABS; ++sl) {
          tma_load_4d(q_s(s) + sl * C::QSLAB, &tm_q, q_full(s), sl * 64, h, qq0, b);
          tma_load_4d(do_s(s) + sl * C::QSLAB, &tm_do, q_full(s), sl * 64, h, qq0, b);
        }
        bulk_load(stat_s(s), p.lse2 + srow, kHalf * 4, q_full(s));
        bulk_load(stat_s(s) + kHalf * 4, p.delta + srow, kHalf * 4, q_full(s));
        ++issued;
      }
      mbar_wait(kv_full, 0, p.status);
      for (int t = issued - QST < 0 ? 0 : issued - QST; t < issued; ++t)
        mbar_wait(q_full(t % QST), (t / QST) & 1, p.status);
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------- MMA
    if (elect_one_sync()) {
      constexpr uint32_t idesc_s = make_idesc_bf16(kTile, kHalf, false, false);
      constexpr uint32_t idesc_acc = make_idesc_bf16(kTile, D, false, true);
      bool ok = mbar_wait(kv_full, 0, p.status);
      // dV += P^T_t dO_t and dK += dS^T_t Q_t: A K-major from shared memory,
      // B MN-major (N = dim, K = the tile's 64 queries).
      auto issue_acc = [&](int t) -> bool {
        if (!mbar_wait(pds_ready(t & 1), (t >> 1) & 1, p.status)) return false;
        tc_fence_after();
        const int s = t % QST;
#pragma unroll
        for (int kk = 0; kk < kHalf / 16; ++kk)
          umma_bf16(tmem + C::DV_COL, make_sdesc(p_s(t & 1) + kk * 32, 16, 1024, kSw128),
                    make_sdesc(do_s(s) + kk * 2048, C::QSLAB, 1024, kSw128), idesc_acc,
                    (t > 0 || kk > 0) ? 1u : 0u);
#pragma unroll
        for (int kk = 0; kk < kHalf / 16; ++kk)
          umma_bf16(tmem + C::DK_COL, make_sdesc(ds_s(t & 1) + kk * 32, 16, 1024, kSw128),
                    make_sdesc(q_s(s) + kk * 2048, C::QSLAB, 1024, kSw128), idesc_acc,
                    (t > 0 || kk > 0) ? 1u : 0u);
        umma_commit(q_empty(s));
        return true;
      };
      for (int t = 0; t < T && ok; ++t) {
        const int s = t % QST;
        ok = mbar_wait(q_full(s), (t / QST) & 1, p.status) &&
             (t < 2 || mbar_wait(s_free(t & 1), ((t - 2) >> 1) & 1, p.status));
        if (!ok) break;
        tc_fence_after();
        const uint32_t sd = tmem + C::S_COL + (t & 1) * kHalf;
        const uint32_t pd = tmem + C::DP_COL + (t & 1) * kHalf;
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk) {
          const uint32_t koff = (kk >> 2) * C::KSLAB + (kk & 3) * 32;
          const uint32_t qoff = (kk >> 2) * C::QSLAB + (kk & 3) * 32;
          umma_bf16(sd, make_sdesc(k_s + koff, 16, 1024, kSw128),
                    make_sdesc(q_s(s) + qoff, 16, 1024, kSw128), idesc_s, kk > 0);
        }
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk) {
          const uint32_t koff = (kk >> 2) * C::KSLAB + (kk & 3) * 32;
          const uint32_t qoff = (kk >> 2) * C::QSLAB + (kk & 3) * 32;
          umma_bf16(pd, make_sdesc(v_s + koff, 16, 1024, kSw128),
                    make_sdesc(do_s(s) + qoff, 16, 1024, kSw128), idesc_s, kk > 0);
        }
        umma_commit(s_full(t & 1));
        if (t >= 1) ok = issue_acc(t - 1);
      }
      if (ok && T > 0) issue_acc(T - 1);
      umma_commit(acc_full);
      mbar_wait(acc_full, 0, p.status);
    }
  } else if (warp >= 4) {
    // ------------------------------------------------------ compute warps
    // Two warpgroups on the same 128 key rows: warps 4-7 take query columns
    // 0-31 of each 64-query tile, warps 8-11 columns 32-63; likewise halves
    // of the dV and dK rows at the end.
    const int half = (warp - 4) >> 2;
    const int quad = warp & 3;
    const int row = quad * 32 + lane;
    const int kvpos = kv0 + row;
    const uint32_t lrow = tmem + (static_cast<uint32_t>(quad * 32) << 16);
    const float c = sh.scale_log2;
    bool ok = true;
    for (int t = 0; t < T; ++t) {
      const int s = t % QST;
      const int qq0 = (i0 + t % nq) * kHalf + half * 32;
      ok = mbar_wait(s_full(t & 1), (t >> 1) & 1, p.status);
      if (!ok) break;
      tc_fence_after();
      uint32_t sv[32], dv[32];
      tmem_ld_32x32b_x32(lrow + C::S_COL + (t & 1) * kHalf + half * 32, sv);
      tmem_ld_32x32b_x32(lrow + C::DP_COL + (t & 1) * kHalf + half * 32, dv);
      tmem_ld_wait();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(s_free(t & 1));
      // The query tile's lse2 and delta (landed with its Q and dO).
      ok = mbar_wait(q_full(s), (t / QST) & 1, p.status);
      if (!ok) break;
      const float* st = reinterpret_cast<const float*>(gbase + (stat_s(s) - base)) + half * 32;
      // A key row sees query q only if q >= kvpos (causal); rows past seq
      // carry lse2 = +inf, so their probabilities are 0 already.
      int first = 0;
      if (sh.causal && qq0 < kvpos) first = kvpos - qq0;
      uint32_t pk[16], dk[16];
#pragma unroll
      for (int i = 0; i < 32; i += 4) {
        const float4 l4 = *reinterpret_cast<const float4*>(st + i);
        const float4 d4 = *reinterpret_cast<const float4*>(st + kHalf + i);
        const float la[4] = {l4.x, l4.y, l4.z, l4.w};
        const float da[4] = {d4.x, d4.y, d4.z, d4.w};
        float pv[4], dsv[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const float x = fmaf(__uint_as_float(sv[i + e]), c, -la[e]);
          float pe = e == 3 ? exp2_poly(x) : ex2_approx(x);
          if (i + e < first) pe = 0.0f;
          pv[e] = pe;
          dsv[e] = pe * (__uint_as_float(dv[i + e]) - da[e]);
        }
        pk[i / 2] = pack_bf16x2_f32(pv[0], pv[1]);
        pk[i / 2 + 1] = pack_bf16x2_f32(pv[2], pv[3]);
        dk[i / 2] = pack_bf16x2_f32(dsv[0], dsv[1]);
        dk[i / 2 + 1] = pack_bf16x2_f32(dsv[2], dsv[3]);
      }
      // The stat reads above are ordered before the copies that refill the
      // stage (generic-proxy reads, async-proxy writes).
      fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) mbar_arrive(q_empty(s));
      // Row `row` of the K-major operand: 64 bf16 = eight 16-byte chunks,
      // chunk ch stored at ch ^ (row & 7) (the 128-byte swizzle); this half
      // writes chunks 4 half .. 4 half + 3.
      const uint32_t prow = p_s(t & 1) + row * 128;
      const uint32_t drow = ds_s(t & 1) + row * 128;
#pragma unroll
      for (int q4 = 0; q4 < 4; ++q4) {
        const uint32_t off = static_cast<uint32_t>(((4 * half + q4) ^ (row & 7)) * 16);
        sts128(prow + off, pk[4 * q4], pk[4 * q4 + 1], pk[4 * q4 + 2], pk[4 * q4 + 3]);
        sts128(drow + off, dk[4 * q4], dk[4 * q4 + 1], dk[4 * q4 + 2], dk[4 * q4 + 3]);
      }
      fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) mbar_arrive(pds_ready(t & 1));
    }
    if (ok) ok = mbar_wait(acc_full, 0, p.status);
    tc_fence_after();
    if (ok) {
      const bool valid = kvpos < sh.seq;
      const size_t roff = ((static_cast<size_t>(b) * sh.seq + kvpos) * sh.kv_heads + hk) * D;
#pragma unroll
      for (int which = 0; which < 2; ++which) {
        const uint32_t col = which == 0 ? C::DV_COL : C::DK_COL;
        const float f = which == 0 ? 1.0f : p.scale;
        uint16_t* orow = (which == 0 ? p.dv : p.dk) + roff;
#pragma unroll
        for (int c4 = half * (D / 64); c4 < (half + 1) * (D / 64); ++c4) {
          uint32_t o[32];
          tmem_ld_32x32b_x32(lrow + col + c4 * 32, o);
          tmem_ld_wait();
          uint32_t w[16];
#pragma unroll
          for (int i = 0; i < 16; ++i)
            w[i] = pack_bf16x2_f32(__uint_as_float(o[2 * i]) * f, __uint_as_float(o[2 * i + 1]) * f);
          if (valid) {
            uint4* dst = reinterpret_cast<uint4*>(orow + c4 * 32);
#pragma unroll
            for (int i = 0; i < 4; ++i)
              dst[i] = make_uint4(w[4 * i], w[4 * i + 1], w[4 * i + 2], w[4 * i + 3]);
          }
        }
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 2) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc(tmem, C::TMEM_COLS);
  }
}


// [batch, seq, heads, dim] bf16 as a 4D tensor map, one 64-wide dim slab x
// `rows` rows of one head per box (128-byte swizzle).
int map_bshd(CUtensorMap* map, const void* ptr, int64_t batch, int64_t seq, int64_t heads,
             int64_t dim, uint32_t rows = kTile) {
  const uint64_t dims[4] = {static_cast<uint64_t>(dim), static_cast<uint64_t>(heads),
                            static_cast<uint64_t>(seq), static_cast<uint64_t>(batch)};
  const uint64_t strides[3] = {static_cast<uint64_t>(dim) * 2,
                               static_cast<uint64_t>(heads * dim) * 2,
                               static_cast<uint64_t>(seq * heads * dim) * 2};
  const uint32_t box[4] = {64, 1, rows, 1};
  return encode_tmap(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 4, ptr, dims, strides, box,
                     CU_TENSOR_MAP_SWIZZLE_128B);
}

int check_shape(int64_t batch, int64_t seq, int64_t heads, int64_t kv_heads, int64_t dim) {
  if (batch < 0 || seq < 0 || heads <= 0 || kv_heads <= 0)
    return fail(TQ_ERR_INVALID, "attention: batch and seq must be >= 0, heads and kv_heads > 0");
  if (heads % kv_heads != 0)
    return fail(TQ_ERR_INVALID, "attention: heads (%lld) must be a multiple of kv_heads (%lld)",
                (long long)heads, (long long)kv_heads);
  if (dim != 64 && dim != 128)
    return fail(TQ_ERR_UNSUPPORTED, "attention: head dim must be 64 or 128, got %lld",
                (long long)dim);
  const int64_t tiles = (seq + kTile - 1) / kTile;
  if (seq > (1ll << 30) || batch * heads * tiles > (1ll << 31) - 1 ||
      batch * seq * heads * dim > (1ll << 40))
    return fail(TQ_ERR_INVALID, "attention: shape too large");
  return TQ_OK;
}

AttnShape make_shape(int64_t batch, int64_t seq, int64_t heads, int64_t kv_heads, float scale,
                     int causal) {
  AttnShape s{};
  s.batch = static_cast<int>(batch);
  s.seq = static_cast<int>(seq);
  s.heads = static_cast<int>(heads);
  s.kv_heads = static_cast<int>(kv_heads);
  s.group = static_cast<int>(heads / kv_heads);
  s.n_tiles = static_cast<int>((seq + kTile - 1) / kTile);
  s.causal = causal ? 1 : 0;
  s.scale_log2 = scale * kLog2e;
  return s;
}

template <int D>
int launch_fwd(const void* q, const void* k, const void* v, const AttnShape& sh, void* out,
               float* lse, int* status, cudaStream_t stream) {
  using C = FwdCfg<D>;
  int rc = set_max_smem_once(reinterpret_cast<const void*>(attn_fwd_kernel<D>), C::SMEM,
                             "cudaFuncSetAttribute(attn_fwd)");
  if (rc) return rc;
  CUtensorMap tq_, tk, tv;
  if ((rc = map_bshd(&tq_, q, sh.batch, sh.seq, sh.heads, D))) return rc;
  if ((rc = map_bshd(&tk, k, sh.batch, sh.seq, sh.kv_heads, D))) return rc;
  if ((rc = map_bshd(&tv, v, sh.batch, sh.seq, sh.kv_heads, D))) return rc;
  FwdParams p{};
  p.sh = sh;
  p.n_pairs = (sh.n_tiles + 1) / 2;
  p.out = static_cast<uint16_t*>(out);
  p.lse = lse;
  p.status = status;
  const unsigned grid = static_cast<unsigned>(sh.batch) * sh.heads * p.n_pairs;
  return launch_kernel(attn_fwd_kernel<D>, dim3(grid), dim3(384), C::SMEM, stream, 1,
                       "attention forward launch", tq_, tk, tv, p);
}

template <int D>
int launch_bwd(const void* q, const void* k, const void* v, const void* out, const void* dout,
               const float* lse, const AttnShape& sh, float scale, void* dq, void* dk, void* dv,
               float* lse2, float* delta, int seq_pad, int* status, cudaStream_t stream) {
  using Q = DqCfg<D>;
  using KV = DkvCfg<D>;
  int rc = set_max_smem_once(reinterpret_cast<const void*>(attn_bwd_dq_kernel<D>), Q::SMEM,
                             "cudaFuncSetAttribute(attn_bwd_dq)");
  if (rc) return rc;
  rc = set_max_smem_once(reinterpret_cast<const void*>(attn_bwd_dkv_kernel<D>), KV::SMEM,
                         "cudaFuncSetAttribute(attn_bwd_dkv)");
  if (rc) return rc;
  PrepParams pp{};
  pp.out = static_cast<const uint16_t*>(out);
  pp.dout = static_cast<const uint16_t*>(dout);
  pp.lse = lse;
  pp.lse2 = lse2;
  pp.delta = delta;
  pp.batch = sh.batch;
  pp.seq = sh.seq;
  pp.heads = sh.heads;
  pp.seq_pad = seq_pad;
  pp.dim = D;
  const long long rows = static_cast<long long>(sh.batch) * sh.heads * seq_pad;
  rc = launch_kernel(attn_bwd_prep_kernel, dim3(static_cast<unsigned>((rows * 8 + 255) / 256)),
                     dim3(256), 0, stream, 1, "attention backward prep launch", pp);
  if (rc) return rc;
  // Query-side maps (128-row boxes for dq, 64-row boxes for dkv) and the
  // key/value maps the other way round.
  CUtensorMap q128, do128, k64, v64, q64, do64, k128, v128;
  if ((rc = map_bshd(&q128, q, sh.batch, sh.seq, sh.heads, D, kTile))) return rc;
  if ((rc = map_bshd(&do128, dout, sh.batch, sh.seq, sh.heads, D, kTile))) return rc;
  if ((rc = map_bshd(&k64, k, sh.batch, sh.seq, sh.kv_heads, D, kHalf))) return rc;
  if ((rc = map_bshd(&v64, v, sh.batch, sh.seq, sh.kv_heads, D, kHalf))) return rc;
  if ((rc = map_bshd(&q64, q, sh.batch, sh.seq, sh.heads, D, kHalf))) return rc;
  if ((rc = map_bshd(&do64, dout, sh.batch, sh.seq, sh.heads, D, kHalf))) return rc;
  if ((rc = map_bshd(&k128, k, sh.batch, sh.seq, sh.kv_heads, D, kTile))) return rc;
  if ((rc = map_bshd(&v128, v, sh.batch, sh.seq, sh.kv_heads, D, kTile))) return rc;
  BwdParams p{};
  p.sh = sh;
  p.seq_pad = seq_pad;
  p.scale = scale;
  p.lse2 = lse2;
  p.delta = delta;
  p.dq = static_cast<uint16_t*>(dq);
  p.dk = static_cast<uint16_t*>(dk);
  p.dv = static_cast<uint16_t*>(dv);
  p.status = status;
  const unsigned grid_q = static_cast<unsigned>(sh.batch) * sh.heads * sh.n_tiles;
  rc = launch_kernel(attn_bwd_dq_kernel<D>, dim3(grid_q), dim3(384), Q::SMEM, stream, 1,
                     "attention backward dq launch", q128, do128, k64, v64, p);
  if (rc) return rc;
  const unsigned grid_kv = static_cast<unsigned>(sh.batch) * sh.kv_heads * sh.n_tiles;
  return launch_kernel(attn_bwd_dkv_kernel<D>, dim3(grid_kv), dim3(384), KV::SMEM, stream, 1,
                       "attention backward dkv launch", q64, do64, k128, v128, p);
}

}  // namespace
}  // namespace tq

extern "C" int tq_attention_fwd(const void* q, const void* k, const void* v, int64_t batch,
                                int64_t seq, int64_t heads, int64_t kv_heads, int64_t head_dim,
                                float scale, int causal, void* out, float* lse, void* stream) {
  using namespace tq;
  int rc = check_shape(batch, seq, heads, kv_heads, head_dim);
  if (rc) return rc;
  if (!(scale > 0.0f) || !std::isfinite(scale))
    return fail(TQ_ERR_INVALID, "attention: scale must be positive and finite");
  if (batch == 0 || seq == 0) return TQ_OK;
  if (!q || !k || !v || !out || !lse) return fail(TQ_ERR_INVALID, "attention: null pointer");
  if (!aligned(q, 16) || !aligned(k, 16) || !aligned(v, 16) || !aligned(out, 16) ||
      !aligned(lse, 4))
    return fail(TQ_ERR_MISALIGNED, "attention: q, k, v and out must be 16-byte aligned");
  int* status = device_status_ptr(&rc);
  if (!status) return rc;
  const AttnShape sh = make_shape(batch, seq, heads, kv_heads, scale, causal);
  if (head_dim == 64) return launch_fwd<64>(q, k, v, sh, out, lse, status, as_stream(stream));
  return launch_fwd<128>(q, k, v, sh, out, lse, status, as_stream(stream));
}

extern "C" int tq_attention_bwd_workspace_bytes(int64_t batch, int64_t seq, int64_t heads,
                                                size_t* bytes) {
  using namespace tq;
  if (!bytes) return fail(TQ_ERR_INVALID, "attention: null bytes pointer");
  if (batch < 0 || seq < 0 || heads <= 0)
    return fail(TQ_ERR_INVALID, "attention: batch and seq must be >= 0, heads > 0");
  const int64_t seq_pad = (seq + kTile - 1) / kTile * kTile;
  *bytes = static_cast<size_t>(2 * batch * heads * seq_pad) * sizeof(float);
  return TQ_OK;
}

extern "C" int tq_attention_bwd(const void* q, const void* k, const void* v, const void* out,
                                const void* dout, const float* lse, int64_t batch, int64_t seq,
                                int64_t heads, int64_t kv_heads, int64_t head_dim, float scale,
                                int causal, void* dq, void* dk, void* dv, void* workspace,
                                size_t workspace_bytes, void* stream) {
  using namespace tq;
  int rc = check_shape(batch, seq, heads, kv_heads, head_dim);
  if (rc) return rc;
  if (!(scale > 0.0f) || !std::isfinite(scale))
    return fail(TQ_ERR_INVALID, "attention: scale must be positive and finite");
  if (batch == 0 || seq == 0) return TQ_OK;
  size_t need = 0;
  rc = tq_attention_bwd_workspace_bytes(batch, seq, heads, &need);
  if (rc) return rc;
  if (workspace_bytes < need)
    return fail(TQ_ERR_INVALID, "attention: workspace of %zu bytes, %zu needed", workspace_bytes,
                need);
  if (!q || !k || !v || !out || !dout || !lse || !dq || !dk || !dv || !workspace)
    return fail(TQ_ERR_INVALID, "attention: null pointer");
  if (!aligned(q, 16) || !aligned(k, 16) || !aligned(v, 16) || !aligned(out, 16) ||
      !aligned(dout, 16) || !aligned(dq, 16) || !aligned(dk, 16) || !aligned(dv, 16) ||
      !aligned(workspace, 256) || !aligned(lse, 4))
    return fail(TQ_ERR_MISALIGNED,
                "attention: tensors must be 16-byte aligned and the workspace 256-byte aligned");
  int* status = device_status_ptr(&rc);
  if (!status) return rc;
  const AttnShape sh = make_shape(batch, seq, heads, kv_heads, scale, causal);
  const int seq_pad = sh.n_tiles * kTile;
  float* lse2 = static_cast<float*>(workspace);
  float* delta = lse2 + static_cast<size_t>(batch * heads) * seq_pad;
  if (head_dim == 64)
    return launch_bwd<64>(q, k, v, out, dout, lse, sh, scale, dq, dk, dv, lse2, delta, seq_pad,
                          status, as_stream(stream));
  return launch_bwd<128>(q, k, v, out, dout, lse, sh, scale, dq, dk, dv, lse2, delta, seq_pad,
                         status, as_stream(stream));
}
