// Forward pair kernel with the dequantized weight tile in tensor memory.
// Included by qmm.cu after the pair kernel, whose tile order, producer,
// barriers and epilogue it follows.
//
// Why: in the pair kernel every k-step moves through each SM's shared memory
// the TMA's token half, codes and scale tiles, the dequantizing warps' bf16
// weight tile (stored, then read again by the MMA) and the MMA's own operand
// reads -- more bytes per k-step than the shared memory moves in the MMA's
// time, which is what held the tensor pipe near two thirds busy.  Here the
// dequantizing warps write the bf16 weight tile straight into tensor memory
// (tcgen05.st, one lane per weight row) and the MMA reads A from there
// (tcgen05.mma ... [a_tmem]): the weight tile's store and its operand read
// leave shared memory altogether.
//
// Tensor memory (512 columns): two accumulators of BN columns, then A_BUFS
// weight buffers of 32 columns (a 128-row x 64-wide bf16 k-step, two values
// per 32-bit column).  BN = 192 keeps four weight buffers beside the double
// accumulator (2 x 192 + 4 x 32 = 512).
//
// Dequantizing warps 2-9 in two groups of four on alternate k-steps; the
// warps of a group cover the four TMEM lane quadrants (warp id % 4), each
// thread one weight row and the whole 64-wide k-step (two runs of 32 codes),
// stored as one 32-column tcgen05.st.
#pragma once

namespace tq {
namespace {

template <int BITS, int BN>
struct PairTsCfg {
  static constexpr int XH_ROWS = BN / 2;
  static constexpr int XH_BYTES = XH_ROWS * kBK * 2;
  static constexpr int C_BYTES = kBM * kBK * BITS / 8;
  static constexpr int SC_ROWS = kBM;
  static constexpr int SC_BYTES = SC_ROWS * 16;
  static constexpr int STAGE_BYTES = XH_BYTES + C_BYTES + 2 * SC_BYTES;
  static constexpr int LUP_BYTES = kBM * 16 * 2;
  static constexpr int LDN_BYTES = XH_ROWS * 16 * 2;
  static constexpr int LORA_BYTES = ((LUP_BYTES + LDN_BYTES + 1023) / 1024) * 1024;
  static constexpr int BAR_BYTES = 512;
  static constexpr int EPI_CHUNK = 32 * 32 * 2;
  static constexpr int EPI_BYTES = 4 * 2 * EPI_CHUNK;
  static constexpr int FIXED = 1024 + LORA_BYTES + EPI_BYTES + BAR_BYTES;
  static constexpr int STAGES_RAW = (kSmemLimit - FIXED) / STAGE_BYTES;
  static constexpr int STAGES = STAGES_RAW > 8 ? 8 : STAGES_RAW;
  static constexpr int SMEM = FIXED + STAGES * STAGE_BYTES;
  static constexpr int ACC_COLS = BN;
  static constexpr int A_COL0 = 2 * BN;                     // first weight-buffer column
  static constexpr int A_COLS = kBK / 2;                    // 32 columns per k-step
  static constexpr int A_BUFS_RAW = (512 - A_COL0) / A_COLS;
  static constexpr int A_BUFS = A_BUFS_RAW > 4 ? 4 : A_BUFS_RAW;
  static constexpr int TMEM_COLS = 512;
  static constexpr int DQ_GROUPS = 2;
  static_assert(BN % 32 == 0 && BN >= 64 && BN <= 192, "token tile of the TS pair kernel");
  static_assert(A_BUFS >= 2, "tensor memory for two weight buffers");
  static_assert(STAGES >= 4, "shared memory for four stages");
  static_assert(SMEM <= kSmemLimit, "shared memory budget");
  static constexpr int OFF_LORA = 8 * (3 * STAGES + 2 * A_BUFS);
  static constexpr int OFF_TMEM = OFF_LORA + 48;
  static_assert(OFF_TMEM + 4 <= BAR_BYTES, "barrier area");
  static_assert(STAGE_BYTES % 1024 == 0, "stage tiles stay 1024-byte aligned");
};

// 32 codes of one weight row (a run, as load_run fetched them) -> 16 bf16x2
// words in k order, w = RNE(scale * q + bias): the tensor-memory image of
// the run (column j holds k = 2j, 2j + 1).
template <int BITS, int OFF>
__device__ __forceinline__ void dequant_run_regs(const uint32_t (&w)[BITS], uint32_t s2,
                                                 uint32_t b2, uint32_t (&o)[32]) {
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    if constexpr (BITS == 4) {
      uint32_t q[4];
      dequant_u4x8(w[j], s2, b2, q);
#pragma unroll
      for (int i = 0; i < 4; ++i) o[OFF + 4 * j + i] = q[i];
    } else {
      uint32_t lo[2], hi[2];
      dequant_u8x4(w[2 * j], s2, b2, lo);
      dequant_u8x4(w[2 * j + 1], s2, b2, hi);
      o[OFF + 4 * j] = lo[0];
      o[OFF + 4 * j + 1] = lo[1];
      o[OFF + 4 * j + 2] = hi[0];
      o[OFF + 4 * j + 3] = hi[1];
    }
  }
}

template <int BITS, int BN>
__global__ void __launch_bounds__(kThreads, 1)
    qmm_pair_ts_kernel(const __grid_constant__ CUtensorMap tm_x,
                       const __grid_constant__ CUtensorMap tm_c,
                       const __grid_constant__ CUtensorMap tm_lup,
                       const __grid_constant__ CUtensorMap tm_ldn,
                       const __grid_constant__ CUtensorMap tm_sc,
                       const __grid_constant__ CUtensorMap tm_bi,
                       const __grid_constant__ CUtensorMap tm_y, const Params p) {
  using C = PairTsCfg<BITS, BN>;
  constexpr int S = C::STAGES;
  constexpr int A = C::A_BUFS;
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw = smem_u32(smem_raw);
  const uint32_t base = (raw + 1023u) & ~1023u;
  uint8_t* const gbase = smem_raw + (base - raw);

  const uint32_t lup = base;
  const uint32_t ldn = base + C::LUP_BYTES;
  const uint32_t epi = base + C::LORA_BYTES;
  const uint32_t stages = epi + C::EPI_BYTES;
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
  const uint32_t lora_full = bars + C::OFF_LORA;
  const uint32_t lora_empty = lora_full + 8u;
  auto acc_full = [&](int b) { return lora_full + 16u + 8u * b; };
  auto acc_empty = [&](int b) { return lora_full + 32u + 8u * b; };
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
      mbar_init(aready_b(a), 2 * (kDqWarps / C::DQ_GROUPS));
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
            tma_load_2d_pair(lup + ch * kBM * 16, &tm_lup, lora_full_l, ch * 8, out0);
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
          tma_load_2d_hint(c_s(s), &tm_c, full_b(s), k0 * BITS / 32, out0, keep);
          const int gx = scale_window<true>(p, out0, k0);
          tma_load_2d_hint(sc_s(s), &tm_sc, full_b(s), gx, out0, keep);
          tma_load_2d_hint(bi_s(s), &tm_bi, full_b(s), gx, out0, keep);
        }
      }
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
      constexpr uint32_t idesc = make_idesc_bf16(kPairRows, BN, false, false);
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
          const uint64_t adesc = make_sdesc(lup, kBM * 16, 128, kSwNone);
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
          const uint32_t at = tmem + C::A_COL0 + a * C::A_COLS;
#pragma unroll
          for (int k4 = 0; k4 < kBK / 16; ++k4) {
            const uint64_t bdesc = make_sdesc(x_s(s) + k4 * 32, 16, 1024, kSw128);
            umma_bf16_pair_ts(d, at + k4 * 8, bdesc, idesc, acc);
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
      if (my_tiles > 0)
        mbar_wait(acc_full((my_tiles - 1) & 1), ((my_tiles - 1) >> 1) & 1, p.status);
    }
  } else if (warp < 2 + kDqWarps) {
    // ---------------------------------------------------- dequant warps
    // Thread: weight row q4 * 32 + lane of this CTA's 128 (its TMEM lane),
    // both 32-code runs of the k-steps of its group (k-step parity).
    const int q4 = warp & 3;
    const int grp = (warp - 2) >> 2;
    const int row = q4 * 32 + lane;
    const uint32_t lane_base = static_cast<uint32_t>(q4 * 32) << 16;
    int j = 0;
    bool ok = true;
    for (int lt = 0; lt < my_tiles && ok; ++lt) {
      const int out0 = tile_out0(lt);
      for (int kk = 0; kk < num_k && ok; ++kk, ++j) {
        if ((j & 1) != grp) continue;
        const int s = j % S;
        const int a = j % A;
        const int k0 = kk * kBK;
        ok = mbar_wait(full_b(s), (j / S) & 1, p.status) &&
             mbar_wait(aempty_b(a), ((j / A) & 1) ^ 1, p.status);
        if (!ok) break;
        uint32_t w0[BITS], w1[BITS];
        load_run<BITS, true>(c_s(s), row, w0);
        load_run<BITS, true>(c_s(s), row + 128, w1);
        const uint32_t o0 = scale_off<true>(p, row, out0, k0);
        const uint32_t o1 = scale_off<true>(p, row + 128, out0, k0);
        const uint32_t s0 = lds_u16(sc_s(s) + o0), b0 = lds_u16(bi_s(s) + o0);
        const uint32_t s1 = lds_u16(sc_s(s) + o1), b1 = lds_u16(bi_s(s) + o1);
        uint32_t v[32];
        dequant_run_regs<BITS, 0>(w0, bf16_dup(static_cast<uint16_t>(s0)),
                                  bf16_dup(static_cast<uint16_t>(b0)), v);
        dequant_run_regs<BITS, 16>(w1, bf16_dup(static_cast<uint16_t>(s1)),
                                   bf16_dup(static_cast<uint16_t>(b1)), v);
        tmem_st_32x32b_x32(tmem + lane_base + C::A_COL0 + a * C::A_COLS, v);
        tmem_st_wait();
        tc_fence_before();
        // The code and scale reads of the stage are ordered before the TMA
        // that refills it once the MMA has committed.
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) mbar_arrive_cluster(lead(aready_b(a)));
      }
    }
  } else {
    // ------------------------------------------------------------ epilogue
    const int q = warp & 3;
    const int r = q * 32 + lane;
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
      (void)r;
#pragma unroll 1
      for (int c0 = 0; c0 < BN; c0 += 32, ++chunk) {
        uint32_t v[32];
        tmem_ld_32x32b_x32(d + c0, v);
        tmem_ld_wait();
        if (!ok) continue;
        const uint32_t sb = stage_w + static_cast<uint32_t>(chunk & 1) * C::EPI_CHUNK;
        if (lane == 0) tma_store_wait_read1();
        __syncwarp();
#pragma unroll
        for (int jj = 0; jj < 32; ++jj)
          sts16(sb + jj * 64 + lane * 2,
                __bfloat16_as_ushort(__float2bfloat16_rn(__uint_as_float(v[jj]) + bias)));
        fence_proxy_async_smem();
        __syncwarp();
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
    if (lane == 0) tma_store_wait_all();
    __syncwarp();
  }
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
