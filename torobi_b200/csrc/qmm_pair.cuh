// Pair form of the quantized GEMM: the two CTAs of a cluster share one tile
// of 256 weight-side rows x BN tokens and one tcgen05.mma.cta_group::2 per
// K=16 slice.  Included by qmm.cu after the single-CTA kernel, whose
// dequantization, group lookup and parameters it reuses.
//
// Why: with one CTA per 128-row tile, every SM's shared memory carries the
// whole token tile twice per k-step (TMA write + UMMA read) next to the
// dequantized weight tile; that traffic, not the tensor pipe, bounds the
// single-CTA kernel.  In a pair each CTA holds half of the token tile while
// the MMA still spans all BN tokens, so the token traffic per SM halves.
//
// Roles (448 threads, as the single-CTA kernel):
//   warp 0      TMA: this CTA's codes and scale tiles (own barrier), its half
//               of the token tile and its LoRA tiles (the even CTA's barrier)
//   warp 1      TMEM allocation in both CTAs; in the even CTA the thread that
//               issues the pair UMMAs and commits to both CTAs' barriers
//   warps 2-9   dequantize this CTA's 128 weight rows (G groups on
//               alternate k-steps: 2 forward, 4 for dX), then arrive on the
//               even CTA's "weight tile ready" barrier
//   warps 10-13 epilogue: this CTA's 128 rows of the accumulator (its TMEM)
// Barriers only the even CTA waits on (token tile full, weight tile ready,
// LoRA full, accumulator drained) count both CTAs' arrivals; barriers each
// CTA waits on for its own buffers (stage free, weight buffer free,
// accumulator full) get one commit from the even CTA's MMA thread each.
#pragma once

namespace tq {
namespace {

constexpr int kPairRows = 2 * kBM;  // weight-side rows of a pair tile

template <int BITS, bool TRANS, int BN, int G>
struct PairCfg {
  static constexpr int XH_ROWS = BN / 2;                    // this CTA's tokens
  static constexpr int XH_BYTES = XH_ROWS * kBK * 2;
  static constexpr int A_BYTES = kBM * kBK * 2;
  static constexpr int C_BYTES = kBM * kBK * BITS / 8;
  static constexpr int SC_ROWS = TRANS ? kBM : kBK;
  static constexpr int SC_BYTES = SC_ROWS * 16;
  static constexpr int STAGE_BYTES = XH_BYTES + C_BYTES + 2 * SC_BYTES;
  static constexpr int LUP_BYTES = kBM * 16 * 2;            // [128 x 16] bf16
  static constexpr int LDN_BYTES = XH_ROWS * 16 * 2;        // [BN/2 x 16] bf16
  static constexpr int LORA_BYTES = ((LUP_BYTES + LDN_BYTES + 1023) / 1024) * 1024;
  static constexpr int BAR_BYTES = 512;
  // Epilogue staging: per epilogue warp two [32 tokens x 32 features] bf16
  // buffers, written from TMEM and stored to y by TMA.
  static constexpr int EPI_CHUNK = 32 * 32 * 2;
  static constexpr int EPI_BYTES = 4 * 2 * EPI_CHUNK;
  static constexpr int FIXED = 1024 + LORA_BYTES + EPI_BYTES + BAR_BYTES;
  // G dequantizing groups on alternate k-steps, one weight-tile buffer more.
  static constexpr int DQ_GROUPS = G;
  static constexpr int stages_with(int a) { return (kSmemLimit - FIXED - a * A_BYTES) / STAGE_BYTES; }
  // A buffer per group and one for the MMA, unless that leaves fewer than
  // six TMA stages and one buffer fewer does not.
  static constexpr int A_BUFS =
      stages_with(G + 1) >= 6 ? G + 1
      : stages_with(G) >= 6   ? G
      : stages_with(G + 1) >= 4 ? G + 1
                                : (stages_with(3) >= 4 ? 3 : 2);
  static constexpr int STAGES_RAW = (kSmemLimit - FIXED - A_BUFS * A_BYTES) / STAGE_BYTES;
  static constexpr int STAGES = STAGES_RAW > 8 ? 8 : STAGES_RAW;
  static constexpr int SMEM = FIXED + A_BUFS * A_BYTES + STAGES * STAGE_BYTES;
  static constexpr int ACC_COLS = BN;
  static constexpr int TMEM_COLS = 2 * ACC_COLS;
  static_assert(BN == 128 || BN == 256, "pair tiles span 128 or 256 tokens");
  static_assert(STAGES >= 2, "shared memory too small for two stages");
  static_assert(SMEM <= kSmemLimit, "shared memory budget");
  // Barrier area: stage (full, xfull, empty), weight ring (ready, empty),
  // LoRA (full, empty), accumulators (full x2, empty x2), then the TMEM
  // address word.
  static constexpr int OFF_LORA = 8 * (3 * STAGES + 2 * A_BUFS);
  static constexpr int OFF_TMEM = OFF_LORA + 48;
  static_assert(OFF_TMEM + 4 <= BAR_BYTES, "barrier area");
  static_assert(STAGE_BYTES % 1024 == 0, "stage tiles stay 1024-byte aligned");
};

// Persistent over pairs: pair q (CTAs 2q, 2q+1) takes tiles q, q + pairs, ...;
// tile t covers weight-side rows (t % tiles_n) * 256 (CTA rank r owns the
// 128 rows from + 128 r) and tokens (t / tiles_n) * BN (CTA r loads the half
// from + r * BN / 2).  p.tiles_n counts 256-row tiles; no split-K.
template <int BITS, bool TRANS, int BN, int G>
__global__ void __launch_bounds__(kThreads, 1)
    qmm_pair_kernel(const __grid_constant__ CUtensorMap tm_x,
                    const __grid_constant__ CUtensorMap tm_c,
                    const __grid_constant__ CUtensorMap tm_lup,
                    const __grid_constant__ CUtensorMap tm_ldn,
                    const __grid_constant__ CUtensorMap tm_sc,
                    const __grid_constant__ CUtensorMap tm_bi,
                    const __grid_constant__ CUtensorMap tm_y, const Params p) {
  using C = PairCfg<BITS, TRANS, BN, G>;
  constexpr int S = C::STAGES;
  constexpr int A = C::A_BUFS;
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw = smem_u32(smem_raw);
  const uint32_t base = (raw + 1023u) & ~1023u;
  uint8_t* const gbase = smem_raw + (base - raw);

  // Same offsets in both CTAs (the pair UMMA reads the peer at the leader's).
  const uint32_t lup = base;
  const uint32_t ldn = base + C::LUP_BYTES;
  const uint32_t epi = base + C::LORA_BYTES;                       // epilogue staging
  const uint32_t abufs = epi + C::EPI_BYTES;
  const uint32_t stages = abufs + A * C::A_BYTES;
  auto a_s = [&](int a) { return abufs + a * C::A_BYTES; };
  auto x_s = [&](int s) { return stages + s * C::STAGE_BYTES; };
  auto c_s = [&](int s) { return stages + s * C::STAGE_BYTES + C::XH_BYTES; };
  auto sc_s = [&](int s) { return c_s(s) + C::C_BYTES; };
  auto bi_s = [&](int s) { return sc_s(s) + C::SC_BYTES; };
  const uint32_t bars = stages + S * C::STAGE_BYTES;
  auto full_b = [&](int s) { return bars + 8u * s; };              // own codes + scales
  auto xfull_b = [&](int s) { return bars + 8u * (S + s); };       // even CTA: both token halves
  auto empty_b = [&](int s) { return bars + 8u * (2 * S + s); };   // own stage free
  auto aready_b = [&](int a) { return bars + 8u * (3 * S + a); };  // even CTA: both weight halves
  auto aempty_b = [&](int a) { return bars + 8u * (3 * S + A + a); };
  const uint32_t lora_full = bars + C::OFF_LORA;                   // even CTA: both CTAs' tiles
  const uint32_t lora_empty = lora_full + 8u;
  auto acc_full = [&](int b) { return lora_full + 16u + 8u * b; };
  auto acc_empty = [&](int b) { return lora_full + 32u + 8u * b; };  // even CTA: both epilogues
  const uint32_t tmem_slot = bars + C::OFF_TMEM;
  volatile uint32_t* tmem_slot_ptr =
      reinterpret_cast<volatile uint32_t*>(gbase + (tmem_slot - base));

  const uint32_t rank = cluster_ctarank();
  const bool leader = rank == 0;
  auto lead = [&](uint32_t bar) { return mapa_shared(bar, 0); };
  auto peer = [&](uint32_t bar) { return mapa_shared(bar, 1); };

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int num_k = (p.k_red + kBK - 1) / kBK;
  const bool has_lora = p.lora_rank > 0;
  const int lora_chunks = p.lora_rank / 8;
  const int pair = static_cast<int>(blockIdx.x >> 1);
  const int pairs = static_cast<int>(gridDim.x >> 1);
  const int my_tiles = pair < p.tiles_total ? (p.tiles_total - 1 - pair) / pairs + 1 : 0;
  auto tile_of = [&](int lt) { return pair + lt * pairs; };
  // This CTA's first weight-side row, and the pair's first token.
  auto tile_out0 = [&](int lt) {
    return (tile_of(lt) % p.tiles_n) * kPairRows + static_cast<int>(rank) * kBM;
  };
  auto tile_m0 = [&](int lt) { return (tile_of(lt) / p.tiles_n) * BN; };

  if (has_lora) {
    for (int i = threadIdx.x; i < C::LORA_BYTES / 16; i += kThreads)
      sts128(base + 16u * i, 0u, 0u, 0u, 0u);
    fence_proxy_async_smem();
  }
  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(full_b(s), 1);
      mbar_init(xfull_b(s), 1);
      mbar_init(empty_b(s), 1);
    }
    for (int a = 0; a < A; ++a) {
      mbar_init(aready_b(a), 2 * (kDqWarps / G));
      mbar_init(aempty_b(a), 1);
    }
    mbar_init(lora_full, 1);
    mbar_init(lora_empty, 1);
    for (int b = 0; b < 2; ++b) {
      mbar_init(acc_full(b), 1);
      mbar_init(acc_empty(b), 8);
    }
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc_pair(tmem_slot, C::TMEM_COLS);
    tmem_relinquish_pair();
  }
  // Barriers initialised and TMEM allocated in both CTAs before either
  // signals the other.
  __syncwarp();
  tc_fence_before();
  cluster_sync();
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
      tma_prefetch_desc(&tm_sc);
      tma_prefetch_desc(&tm_bi);
      if (has_lora) {
        tma_prefetch_desc(&tm_lup);
        tma_prefetch_desc(&tm_ldn);
      }
      const uint32_t lora_full_l = lead(lora_full);
      bool ok = true;
      int it = 0;
      int lora_loads = 0;
      for (int lt = 0; lt < my_tiles && ok; ++lt) {
        const int out0 = tile_out0(lt);
        const int mh = tile_m0(lt) + static_cast<int>(rank) * C::XH_ROWS;
        if (has_lora) {
          ok = mbar_wait(lora_empty, (lora_loads & 1) ^ 1, p.status);
          if (!ok) break;
          if (leader)
            mbar_arrive_expect_tx(lora_full, 2 * lora_chunks * (kBM * 16 + C::XH_ROWS * 16));
          for (int ch = 0; ch < lora_chunks; ++ch) {
            if constexpr (TRANS) {
              tma_load_2d_pair(lup + ch * kBM * 16, &tm_lup, lora_full_l, ch * 8, out0);
            } else {
              tma_load_2d_pair(lup + ch * 1024, &tm_lup, lora_full_l, out0, ch * 8);
              tma_load_2d_pair(lup + 2048 + ch * 1024, &tm_lup, lora_full_l, out0 + 64, ch * 8);
            }
            tma_load_2d_pair(ldn + ch * C::XH_ROWS * 16, &tm_ldn, lora_full_l, ch * 8, mh);
          }
          ++lora_loads;
        }
        for (int kk = 0; kk < num_k; ++kk, ++it) {
          const int s = it % S;
          const uint32_t ph = (it / S) & 1;
          ok = mbar_wait(empty_b(s), ph ^ 1, p.status);
          if (!ok) break;
          const int k0 = kk * kBK;
          if (leader) mbar_arrive_expect_tx(xfull_b(s), 2 * C::XH_BYTES);
          tma_load_2d_pair(x_s(s), &tm_x, lead(xfull_b(s)), k0, mh);
          mbar_arrive_expect_tx(full_b(s), C::C_BYTES + 2 * C::SC_BYTES);
          if constexpr (TRANS)
            tma_load_2d_hint(c_s(s), &tm_c, full_b(s), k0 * BITS / 32, out0, keep);
          else
            tma_load_2d_hint(c_s(s), &tm_c, full_b(s), out0 * BITS / 32, k0, keep);
          const int gx = scale_window<TRANS>(p, out0, k0);
          const int gy = TRANS ? out0 : k0;
          tma_load_2d_hint(sc_s(s), &tm_sc, full_b(s), gx, gy, keep);
          tma_load_2d_hint(bi_s(s), &tm_bi, full_b(s), gx, gy, keep);
        }
      }
      // Never leave a copy in flight.  Own codes and scales land on own
      // barriers; both CTAs' token halves and LoRA tiles on the even CTA's,
      // whose producer waits for them (the peer stays resident until the
      // closing cluster barrier).
      for (int i = it - S < 0 ? 0 : it - S; i < it; ++i) {
        mbar_wait(full_b(i % S), (i / S) & 1, p.status);
        if (leader) mbar_wait(xfull_b(i % S), (i / S) & 1, p.status);
      }
      if (leader && lora_loads > 0)
        mbar_wait(lora_full, (lora_loads - 1) & 1, p.status);
    }
  } else if (warp == 1) {
    // ---------------------------------------------------------- MMA issuer
    if (leader && elect_one_sync()) {
      constexpr uint32_t idesc = make_idesc_bf16(kPairRows, BN, !TRANS, false);
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
        if (has_lora) {
          ok = mbar_wait(lora_full, lora_uses & 1, p.status);
          ++lora_uses;
          if (!ok) break;
          tc_fence_after();
          uint64_t adesc;
          if constexpr (TRANS)
            adesc = make_sdesc(lup, kBM * 16, 128, kSwNone);
          else
            adesc = make_sdesc(lup, 2048, 1024, kSw128);
          const uint64_t bdesc = make_sdesc(ldn, C::XH_ROWS * 16, 128, kSwNone);
          umma_bf16_pair(d, adesc, bdesc, idesc, 0);
          umma_commit_pair(lead(lora_empty));
          umma_commit_pair(peer(lora_empty));
          acc = 1;
        }
        for (int kk = 0; kk < num_k; ++kk, ++it) {
          const int s = it % S;
          const int a = it % A;
          ok = mbar_wait(xfull_b(s), (it / S) & 1, p.status) &&
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
            umma_bf16_pair(d, adesc, bdesc, idesc, acc);
            acc = 1;
          }
          umma_commit_pair(lead(empty_b(s)));
          umma_commit_pair(peer(empty_b(s)));
          umma_commit_pair(lead(aempty_b(a)));
          umma_commit_pair(peer(aempty_b(a)));
        }
        umma_commit_pair(lead(acc_full(buf)));
        umma_commit_pair(peer(acc_full(buf)));
      }
      // Every UMMA done before the pair frees TMEM.
      if (my_tiles > 0)
        mbar_wait(acc_full((my_tiles - 1) & 1), ((my_tiles - 1) >> 1) & 1, p.status);
    }
  } else if (warp < 2 + kDqWarps) {
    // ---------------------------------------------------- dequant warps
    // G groups of 8/G warps on alternate k-steps, as the single-CTA kernel.
    const int t = threadIdx.x - 64;  // 0..255
    const int grp = t / (256 / G);
    const int tt = t % (256 / G);
    int j = 0;
    bool ok = true;
    for (int lt = 0; lt < my_tiles && ok; ++lt) {
      const int out0 = tile_out0(lt);
      for (int kk = 0; kk < num_k && ok; ++kk, ++j) {
        if ((j % G) != grp) continue;
        const int s = j % S;
        const int a = j % A;
        const int k0 = kk * kBK;
        ok = mbar_wait(full_b(s), (j / S) & 1, p.status) &&
             mbar_wait(aempty_b(a), ((j / A) & 1) ^ 1, p.status);
        if (!ok) break;
        dequant_runs<BITS, TRANS, G>(p, sc_s(s), bi_s(s), c_s(s), a_s(a), tt, out0, k0);
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) mbar_arrive_cluster(lead(aready_b(a)));
      }
    }
  } else {
    // ------------------------------------------------------------ epilogue
    // Each 32-token chunk of this warp's 32 features goes through one of its
    // two staging buffers ([token][feature] bf16) and out by a TMA store,
    // which clips tokens past m and features past n_out.
    const int q = warp & 3;
    const uint32_t stage_w = epi + static_cast<uint32_t>(q) * 2 * C::EPI_CHUNK;
    if (lane == 0) tma_prefetch_desc(&tm_y);
    bool ok = true;
    int chunk = 0;
    for (int lt = 0; lt < my_tiles && ok; ++lt) {
      const int buf = lt & 1;
      ok = mbar_wait(acc_full(buf), (lt >> 1) & 1, p.status);
      tc_fence_after();
      const int og0 = tile_out0(lt) + q * 32;
      const int og = og0 + lane;
      const int m0 = tile_m0(lt);
      float bias = 0.0f;
      if (p.bias_vec && og < p.n_out)
        bias = __uint_as_float(uint32_t(ldg_u16(p.bias_vec + og)) << 16);
      const uint32_t d = tmem + buf * C::ACC_COLS + (static_cast<uint32_t>(q * 32) << 16);
#pragma unroll 1
      for (int c0 = 0; c0 < BN; c0 += 32, ++chunk) {
        uint32_t v[32];
        tmem_ld_32x32b_x32(d + c0, v);
        tmem_ld_wait();
        if (!ok) continue;
        const uint32_t sb = stage_w + static_cast<uint32_t>(chunk & 1) * C::EPI_CHUNK;
        // The store issued from this buffer two chunks ago has read it.
        if (lane == 0) tma_store_wait_read1();
        __syncwarp();
#pragma unroll
        for (int jj = 0; jj < 32; ++jj)
          sts16(sb + jj * 64 + lane * 2,
                __bfloat16_as_ushort(__float2bfloat16_rn(__uint_as_float(v[jj]) + bias)));
        fence_proxy_async_smem();
        __syncwarp();
        // One group per chunk (empty when the box lies wholly past y), so
        // "all but the newest group have read" always covers this buffer's
        // previous store.
        if (lane == 0) {
          if (og0 < p.n_out && m0 + c0 < p.m) {
            if (p.acc)
              tma_reduce_add_2d(&tm_y, sb, og0, m0 + c0);
            else
              tma_store_2d(&tm_y, sb, og0, m0 + c0);
          }
          tma_store_commit();
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive_cluster(lead(acc_empty(buf)));
    }
    // The staging buffers stay valid until every store has read them.
    if (lane == 0) tma_store_wait_all();
    __syncwarp();
  }
  // Both CTAs done with every barrier, copy and accumulator before TMEM is
  // freed and either CTA exits.
  __syncwarp();
  tc_fence_before();
  cluster_sync();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc_pair(tmem, C::TMEM_COLS);
  }
}

}  // namespace
}  // namespace tq
