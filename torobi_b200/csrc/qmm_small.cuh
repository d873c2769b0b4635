// quantized_matmul forward for a handful of tokens (M <= 32, 4-bit codes):
// y[m, n] = sum_k x[m, k] * deq(W)[n, k] (+ bias[n]).
//
// At such token counts the GEMM streams the packed weight (0.5625 bytes per
// weight at group 64) against a tiny x: it is HBM-bound, and what limits the
// tensor-memory kernel there is the per-k-step hand-off of each dequantized
// weight tile through shared memory.  Here the weight never leaves
// registers past a TMA ring: each lane reads its packed words from the
// staged weight tile (16 bytes per row per 128-k chunk, four lanes covering a
// row's 64 bytes), dequantizes them exactly as the other kernels do
// (dequant_u4x8: RNE(scale * q + bias) from the exact value), and feeds them
// to warp-level m16n8k16 MMAs with M = 16 weight rows, N = 8 tokens.  The
// ring (not registers) holds the bytes in flight that HBM latency asks for:
// with the words loaded into registers, eight warps per SM kept 24 KB in
// flight and the kernel moved under 1 TB/s.
//
// The MLX layout (eight codes per word along k) is kept by permuting k the
// same way on both operands: lane 4g + t holds words 4i.. of rows g and
// g + 8, and word i, half h (codes 4h..4h+3) supplies the MMA's A registers
// {(q4h, q4h+1) row g, row g+8, (q4h+2, q4h+3) row g, row g+8} -- columns
// 2t, 2t+1 and 2t+8, 2t+9 of the MMA's k = 16 -- so physical k
// 32t + 8i + 4h + {0, 1, 2, 3} plays the MMA's k 2t, 2t+1, 2t+8, 2t+9.  The
// matching B registers are x[token][32t + 8i + 4h .. + 3], four consecutive
// bf16 of the staged x chunk.
//
// CTA: eight compute warps, one 16-row slab of a 128-row block each, all on
// the same k range, and one TMA warp that streams, per 128-k chunk, the
// block's packed codes (128 rows x 64 bytes, 64-byte swizzle) and x [tokens,
// chunk] (two 128-byte-swizzled boxes) through a ring.
// When the row blocks alone cannot fill the GPU, a cluster of up to eight
// CTAs splits k; the others add their f32 partials into the leader's shared
// memory, which sums them in rank order (deterministic), adds the bias and
// rounds once.  No workspace.
#pragma once

#include "tq_ptx.cuh"

namespace tq {
namespace {

constexpr int kSmallMaxM = 32;
constexpr int kSmallChunk = 128;                // k per chunk
constexpr int kSmallWarps = 8;                  // compute warps, a 16-row slab each
constexpr int kSmallRows = 16 * kSmallWarps;    // weight rows per CTA
constexpr int kSmallThreads = 32 * (kSmallWarps + 1);
constexpr int kSmallXStages = 6;
constexpr int kSmallMaxCluster = 8;
constexpr int kSmallDepth = 2;                  // scale chunks in flight per warp

struct SmallParams {
  const uint32_t* codes;   // [n, k / 8]
  const uint16_t* scales;  // [n, k / group]
  const uint16_t* biases;
  const uint16_t* bias;    // the linear's bias [n], or null
  uint16_t* y;             // [m, n]
  int m, n, k, group;
  int cs;                  // CTAs per row block (the cluster), splitting k
  int* status;
};

template <int MT>  // token tiles of 8
struct SmallCfg {
  static constexpr int MPAD = 8 * MT;
  static constexpr int W_BYTES = kSmallRows * 64;   // 128 rows x 128 codes
  static constexpr int BOX_BYTES = MPAD * 128;      // MPAD tokens x 64 k (bf16)
  static constexpr int STAGE_BYTES = W_BYTES + 2 * BOX_BYTES;
  static constexpr int BAR_OFF = kSmallXStages * STAGE_BYTES;
  static constexpr int PART_OFF = BAR_OFF + 256;
  static constexpr int PART_BYTES = kSmallRows * MPAD * 4;  // f32 [MPAD][128 rows]
  static constexpr int RECV_OFF = PART_OFF + PART_BYTES;    // leader: ranks 1..cs-1
  static int smem(int cs) { return 1024 + RECV_OFF + (cs - 1) * PART_BYTES; }
  static_assert(8 * 2 * kSmallXStages <= 256, "barrier area");
};

template <int MT>
__global__ void __launch_bounds__(kSmallThreads, 1)
    qmm_small_kernel(const __grid_constant__ CUtensorMap tm_x,
                     const __grid_constant__ CUtensorMap tm_c, const SmallParams p) {
  griddep_wait();
  griddep_launch_dependents();
  using C = SmallCfg<MT>;
  constexpr int XS = kSmallXStages;
  constexpr int D = kSmallDepth;
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw = smem_u32(smem_raw);
  const uint32_t base = (raw + 1023u) & ~1023u;
  uint8_t* const gbase = smem_raw + (base - raw);
  auto x_s = [&](int s) { return base + s * C::STAGE_BYTES; };
  const uint32_t bars = base + C::BAR_OFF;
  auto x_full = [&](int s) { return bars + 8u * s; };
  auto x_empty = [&](int s) { return bars + 8u * (XS + s); };
  float* const part = reinterpret_cast<float*>(gbase + C::PART_OFF);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int cs = p.cs;
  const int crank = cs > 1 ? static_cast<int>(cluster_ctarank()) : 0;
  const int row0 = static_cast<int>(blockIdx.x / cs) * kSmallRows;
  const int chunks = p.k / kSmallChunk;
  const int c_begin = static_cast<int>(static_cast<int64_t>(crank) * chunks / cs);
  const int nc = static_cast<int>(static_cast<int64_t>(crank + 1) * chunks / cs) - c_begin;
  if (cs > 1) cluster_arrive_relaxed();  // paired with the wait before the partials move

  if (threadIdx.x == 0) {
    for (int s = 0; s < XS; ++s) {
      mbar_init(x_full(s), 1);
      mbar_init(x_empty(s), kSmallWarps);
    }
    fence_mbar_init();
  }
  __syncthreads();

  if (warp == kSmallWarps) {
    // ------------------------------------------------------------- TMA
    if (elect_one_sync()) {
      tma_prefetch_desc(&tm_x);
      tma_prefetch_desc(&tm_c);
      int issued = 0;
      for (int c = 0; c < nc; ++c) {
        const int s = c % XS;
        if (!mbar_wait(x_empty(s), ((c / XS) & 1) ^ 1, p.status)) break;
        mbar_arrive_expect_tx(x_full(s), C::STAGE_BYTES);
        const int k0 = (c_begin + c) * kSmallChunk;
        tma_load_2d(x_s(s), &tm_c, x_full(s), k0 / 8, row0);
        tma_load_2d(x_s(s) + C::W_BYTES, &tm_x, x_full(s), k0, 0);
        tma_load_2d(x_s(s) + C::W_BYTES + C::BOX_BYTES, &tm_x, x_full(s), k0 + 64, 0);
        ++issued;
      }
      // Never leave a copy in flight.
      for (int c = issued - XS < 0 ? 0 : issued - XS; c < issued; ++c)
        mbar_wait(x_full(c % XS), (c / XS) & 1, p.status);
    }
  } else {
    // ---------------------------------------------------- compute warps
    const int g = lane >> 2;
    const int t = lane & 3;
    const int slab0 = row0 + 16 * warp;
    const bool act = slab0 < p.n;  // n is a multiple of 16
    const int r0 = act ? slab0 + g : 0;
    const int r1 = r0 + 8;
    const int gpr = p.k / p.group;
    const uint16_t* s0p = p.scales + static_cast<size_t>(r0) * gpr;
    const uint16_t* s1p = p.scales + static_cast<size_t>(act ? r1 : 0) * gpr;
    const uint16_t* b0p = p.biases + static_cast<size_t>(r0) * gpr;
    const uint16_t* b1p = p.biases + static_cast<size_t>(act ? r1 : 0) * gpr;
    // Rows g and g + 8 of this warp's slab in the staged codes: row r's 16
    // bytes for lane t sit at chunk t ^ ((r >> 1) & 3) of its 64 (the TMA's
    // 64-byte swizzle: 16-byte chunk bits [4, 6) XOR address bits [7, 9)).
    const int ra = 16 * warp + g, rb = ra + 8;
    const uint32_t wa_off = ra * 64 + ((t ^ ((ra >> 1) & 3)) << 4);
    const uint32_t wb_off = rb * 64 + ((t ^ ((rb >> 1) & 3)) << 4);

    float acc[MT][4];
#pragma unroll
    for (int nt = 0; nt < MT; ++nt)
#pragma unroll
      for (int e = 0; e < 4; ++e) acc[nt][e] = 0.0f;
    uint16_t sc0[D], sc1[D], bi0[D], bi1[D];
    // Chunk c's group scale and bias for this lane's 32 k (from 32t).
    auto load = [&](int slot, int c) {
      const int gi = ((c_begin + c) * kSmallChunk + 32 * t) / p.group;
      if (act) {
        sc0[slot] = __ldg(s0p + gi);
        sc1[slot] = __ldg(s1p + gi);
        bi0[slot] = __ldg(b0p + gi);
        bi1[slot] = __ldg(b1p + gi);
      } else {
        sc0[slot] = sc1[slot] = bi0[slot] = bi1[slot] = 0;
      }
    };
#pragma unroll
    for (int d = 0; d < D; ++d)
      if (d < nc) load(d, d);
    bool ok = true;
    for (int c0 = 0; c0 < nc && ok; c0 += D) {
#pragma unroll
      for (int d = 0; d < D; ++d) {
        const int c = c0 + d;
        if (c < nc && ok) {
          const int s = c % XS;
          ok = mbar_wait(x_full(s), (c / XS) & 1, p.status);
          if (ok) {
            const uint32_t xb = x_s(s) + C::W_BYTES + (t >> 1) * C::BOX_BYTES;
            const uint32_t sa = bf16_dup(sc0[d]), ba = bf16_dup(bi0[d]);
            const uint32_t sb = bf16_dup(sc1[d]), bb = bf16_dup(bi1[d]);
            uint32_t wa[4], wb[4];
            lds128(x_s(s) + wa_off, wa[0], wa[1], wa[2], wa[3]);
            lds128(x_s(s) + wb_off, wb[0], wb[1], wb[2], wb[3]);
#pragma unroll
            for (int i = 0; i < 4; ++i) {
              uint32_t oa[4], ob[4];
              dequant_u4x8(wa[i], sa, ba, oa);
              dequant_u4x8(wb[i], sb, bb, ob);
#pragma unroll
              for (int nt = 0; nt < MT; ++nt) {
                const int n = 8 * nt + g;
                uint32_t x0, x1, x2, x3;
                lds128(xb + n * 128 + ((((t & 1) * 4 + i) ^ (n & 7)) << 4), x0, x1, x2, x3);
                mma_16816_bf16(acc[nt], oa[0], ob[0], oa[1], ob[1], x0, x1);
                mma_16816_bf16(acc[nt], oa[2], ob[2], oa[3], ob[3], x2, x3);
              }
            }
            // This warp's reads of the stage are ordered before the TMA
            // that refills it (generic-proxy reads, async-proxy writes):
            // without the fence a refill was seen to land under reads still
            // pending when two CTAs shared an SM.
            fence_proxy_async_smem();
            __syncwarp();
            if (lane == 0) mbar_arrive(x_empty(s));
            if (c + D < nc) load(d, c + D);
          }
        }
      }
    }
    // This warp's 16 rows x MPAD tokens into the CTA's partial [token][row].
    const int rl = 16 * warp + g;
#pragma unroll
    for (int nt = 0; nt < MT; ++nt) {
      const float* v = acc[nt];
      const int tok = 8 * nt + 2 * t;
      part[tok * kSmallRows + rl] = v[0];
      part[(tok + 1) * kSmallRows + rl] = v[1];
      part[tok * kSmallRows + rl + 8] = v[2];
      part[(tok + 1) * kSmallRows + rl + 8] = v[3];
    }
  }
  __syncthreads();
  if (cs > 1) {
    // Every CTA of the cluster has started: ranks 1.. store their partials
    // into the leader's shared memory.
    cluster_wait();
    if (crank != 0) {
      const uint32_t dst = mapa_shared(base + C::RECV_OFF + (crank - 1) * C::PART_BYTES, 0);
      for (int i = threadIdx.x; i < C::PART_BYTES / 16; i += kSmallThreads) {
        const uint4 v = reinterpret_cast<const uint4*>(part)[i];
        st_cluster_v4(dst + 16u * i, v.x, v.y, v.z, v.w);
      }
    }
    cluster_sync();
    if (crank != 0) return;
  }
  // y[token, row0 .. row0 + 127], eight rows (16 bytes) per item.
  const float* recv = reinterpret_cast<const float*>(gbase + C::RECV_OFF);
  for (int it = threadIdx.x; it < p.m * (kSmallRows / 8); it += kSmallThreads) {
    const int tok = it / (kSmallRows / 8);
    const int rr = (it % (kSmallRows / 8)) * 8;
    if (row0 + rr >= p.n) continue;
    float v[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) v[j] = part[tok * kSmallRows + rr + j];
    for (int q = 1; q < cs; ++q)
#pragma unroll
      for (int j = 0; j < 8; ++j)
        v[j] += recv[(q - 1) * (C::PART_BYTES / 4) + tok * kSmallRows + rr + j];
    if (p.bias) {
#pragma unroll
      for (int j = 0; j < 8; ++j) v[j] += __uint_as_float(uint32_t(__ldg(p.bias + row0 + rr + j)) << 16);
    }
    uint4 o;
    o.x = pack_bf16x2_f32(v[0], v[1]);
    o.y = pack_bf16x2_f32(v[2], v[3]);
    o.z = pack_bf16x2_f32(v[4], v[5]);
    o.w = pack_bf16x2_f32(v[6], v[7]);
    *reinterpret_cast<uint4*>(p.y + static_cast<size_t>(tok) * p.n + row0 + rr) = o;
  }
}

}  // namespace
}  // namespace tq
