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
// Forward, one CTA per (128-query tile, head, sequence), heaviest causal tiles
// first:
//   warp 0     TMA: the query tile once, key and value tiles through a ring
//   warp 1     one thread issues every tcgen05 MMA
//   warp 2     allocates / frees the 512 TMEM columns
//   warps 4-7  softmax: thread i owns query row i (TMEM lane i)
// TMEM: two score buffers S (128 f32 columns each), the output accumulator O
// (dim columns), two probability buffers P (bf16 pairs, 64 columns each).
//   S_j = Q K_j^T            (A and B from shared memory, K-major)
//   P_j = exp2(S_j * c - m)  (softmax warps, written back into TMEM)
//   O  += P_j V_j            (A = P_j from TMEM, B = V_j MN-major)
// The MMA issues S_{j+1} before waiting for P_j, so the next scores are ready
// when the softmax warps finish a tile.  The running maximum m is only moved
// (and O rescaled in TMEM) when a row's maximum grows by more than 2^8: P
// then stays below 256, exact in f32 and in range for bf16, and the final
// 1/l uses the same stale m as every P, so the result is unchanged.
#include <cuda_bf16.h>

#include <cmath>
#include <cstdlib>

#include "tq_ptx.cuh"
#include "tq_runtime.h"

namespace tq {
namespace {

constexpr int kTile = 128;  // query rows and key rows per tile
constexpr float kLog2e = 1.4426950408889634f;
constexpr float kLn2 = 0.6931471805599453f;
constexpr float kRescaleLog2 = 8.0f;  // move m only when the row max grows by > 2^8

struct AttnShape {
  int batch, seq, heads, kv_heads, group, n_tiles;
  int causal;
  float scale_log2;  // softmax scale * log2(e)
};

// ------------------------------------------------------------------ forward --

template <int D>
struct FwdCfg {
  static_assert(D == 64 || D == 128, "head dim");
  static constexpr int SLABS = D / 64;            // 128-byte swizzle atoms along dim
  static constexpr int SLAB_BYTES = kTile * 128;  // 128 rows x 64 bf16
  static constexpr int TILE_BYTES = SLABS * SLAB_BYTES;
  static constexpr int STAGES = D == 128 ? 2 : 4;
  static constexpr int Q_OFF = 0;
  static constexpr int K_OFF = TILE_BYTES;
  static constexpr int V_OFF = K_OFF + STAGES * TILE_BYTES;
  static constexpr int BAR_OFF = V_OFF + STAGES * TILE_BYTES;
  // q_full, k_full[S], k_empty[S], v_full[S], v_empty[S], s_full[2], p_ready[2], o_done[2], slot
  static constexpr int NBAR = 1 + 4 * STAGES + 2 + 2 + 2;
  static constexpr int SMEM = 1024 + BAR_OFF + 8 * (NBAR + 1);
  static constexpr int S_COL = 0;          // S_b at S_COL + 128 b
  static constexpr int O_COL = 256;
  static constexpr int P_COL = 256 + D;    // P_b at P_COL + 64 b
  static constexpr int TMEM_COLS = 512;
  static_assert(P_COL + 128 <= TMEM_COLS, "tensor memory map");
  static_assert(SMEM <= 232448, "shared memory per CTA");
};

struct FwdParams {
  AttnShape sh;
  uint16_t* out;
  float* lse;
  int* status;
};

template <int D>
__global__ void __launch_bounds__(256, 1)
    attn_fwd_kernel(const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_k,
                    const __grid_constant__ CUtensorMap tm_v, const FwdParams p) {
  using C = FwdCfg<D>;
  constexpr int ST = C::STAGES;
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw = smem_u32(smem_raw);
  const uint32_t base = (raw + 1023u) & ~1023u;
  uint8_t* const gbase = smem_raw + (base - raw);
  const uint32_t q_s = base + C::Q_OFF;
  auto k_s = [&](int s) { return base + C::K_OFF + s * C::TILE_BYTES; };
  auto v_s = [&](int s) { return base + C::V_OFF + s * C::TILE_BYTES; };
  const uint32_t bars = base + C::BAR_OFF;
  const uint32_t q_full = bars;
  auto k_full = [&](int s) { return bars + 8u * (1 + s); };
  auto k_empty = [&](int s) { return bars + 8u * (1 + ST + s); };
  auto v_full = [&](int s) { return bars + 8u * (1 + 2 * ST + s); };
  auto v_empty = [&](int s) { return bars + 8u * (1 + 3 * ST + s); };
  auto s_full = [&](int b) { return bars + 8u * (1 + 4 * ST + b); };
  auto p_ready = [&](int b) { return bars + 8u * (3 + 4 * ST + b); };
  // O += P_j V_j completes on o_done(j & 1).  Every barrier used per tile j
  // comes in two, indexed by j's parity, and phase j >> 1 of one is only
  // waited on once tile j - 2's has completed: a parity wait is never more
  // than one phase behind.
  auto o_done = [&](int b) { return bars + 8u * (5 + 4 * ST + b); };
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
  const int n_kv = sh.causal ? qt + 1 : sh.n_tiles;

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    for (int s = 0; s < ST; ++s) {
      mbar_init(k_full(s), 1);
      mbar_init(k_empty(s), 1);
      mbar_init(v_full(s), 1);
      mbar_init(v_empty(s), 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(s_full(i), 1);
      mbar_init(p_ready(i), 4);
      mbar_init(o_done(i), 1);
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

  if (warp == 0) {
    // ------------------------------------------------------------- TMA
    if (elect_one_sync()) {
      tma_prefetch_desc(&tm_q);
      tma_prefetch_desc(&tm_k);
      tma_prefetch_desc(&tm_v);
      mbar_arrive_expect_tx(q_full, C::TILE_BYTES);
      for (int sl = 0; sl < C::SLABS; ++sl)
        tma_load_4d(q_s + sl * C::SLAB_BYTES, &tm_q, q_full, sl * 64, h, q0, b);
      int nk = 0, nv = 0;  // tiles issued
      for (int j = 0; j < n_kv; ++j) {
        const int s = j % ST;
        const uint32_t ph = (j / ST) & 1;
        if (!mbar_wait(k_empty(s), ph ^ 1, p.status)) break;
        mbar_arrive_expect_tx(k_full(s), C::TILE_BYTES);
        for (int sl = 0; sl < C::SLABS; ++sl)
          tma_load_4d(k_s(s) + sl * C::SLAB_BYTES, &tm_k, k_full(s), sl * 64, hk, j * kTile, b);
        ++nk;
        if (!mbar_wait(v_empty(s), ph ^ 1, p.status)) break;
        mbar_arrive_expect_tx(v_full(s), C::TILE_BYTES);
        for (int sl = 0; sl < C::SLABS; ++sl)
          tma_load_4d(v_s(s) + sl * C::SLAB_BYTES, &tm_v, v_full(s), sl * 64, hk, j * kTile, b);
        ++nv;
      }
      // Never leave a copy in flight.
      mbar_wait(q_full, 0, p.status);
      for (int j = nk - ST < 0 ? 0 : nk - ST; j < nk; ++j)
        mbar_wait(k_full(j % ST), (j / ST) & 1, p.status);
      for (int j = nv - ST < 0 ? 0 : nv - ST; j < nv; ++j)
        mbar_wait(v_full(j % ST), (j / ST) & 1, p.status);
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------- MMA
    if (elect_one_sync()) {
      constexpr uint32_t idesc_s = make_idesc_bf16(kTile, kTile, false, false);
      constexpr uint32_t idesc_o = make_idesc_bf16(kTile, D, false, true);
      bool ok = mbar_wait(q_full, 0, p.status);
      auto issue_s = [&](int j) -> bool {
        const int s = j % ST;
        if (!mbar_wait(k_full(s), (j / ST) & 1, p.status)) return false;
        tc_fence_after();
        const uint32_t d = tmem + C::S_COL + (j & 1) * kTile;
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk) {
          const uint32_t off = (kk >> 2) * C::SLAB_BYTES + (kk & 3) * 32;
          umma_bf16(d, make_sdesc(q_s + off, 16, 1024, kSw128),
                    make_sdesc(k_s(s) + off, 16, 1024, kSw128), idesc_s, kk > 0);
        }
        umma_commit(s_full(j & 1));
        umma_commit(k_empty(s));
        return true;
      };
      if (ok) ok = issue_s(0);
      int issued_pv = 0;
      for (int j = 0; j < n_kv && ok; ++j) {
        if (j + 1 < n_kv && !issue_s(j + 1)) break;
        const int s = j % ST;
        ok = mbar_wait(p_ready(j & 1), (j >> 1) & 1, p.status) &&
             mbar_wait(v_full(s), (j / ST) & 1, p.status);
        if (!ok) break;
        tc_fence_after();
        const uint32_t pa = tmem + C::P_COL + (j & 1) * 64;
#pragma unroll
        for (int kk = 0; kk < kTile / 16; ++kk)
          umma_bf16_ts(tmem + C::O_COL, pa + kk * 8,
                       make_sdesc(v_s(s) + kk * 2048, C::SLAB_BYTES, 1024, kSw128), idesc_o,
                       (j > 0 || kk > 0) ? 1u : 0u);
        umma_commit(v_empty(s));
        umma_commit(o_done(j & 1));
        ++issued_pv;
      }
      // Nothing may outlive the CTA's TMEM: the last commit covers every MMA.
      if (issued_pv > 0) {
        const int t = issued_pv - 1;
        mbar_wait(o_done(t & 1), (t >> 1) & 1, p.status);
      }
    }
  } else if (warp >= 4) {
    // --------------------------------------------------------- softmax
    const int quad = warp & 3;
    const int row = quad * 32 + lane;
    const int qpos = q0 + row;
    const uint32_t lrow = tmem + (static_cast<uint32_t>(quad * 32) << 16);
    const float c = sh.scale_log2;
    float m = -INFINITY;
    float l = 0.0f;
    bool ok = true;
    int j = 0;
    for (; j < n_kv; ++j) {
      ok = mbar_wait(s_full(j & 1), (j >> 1) & 1, p.status);
      if (!ok) break;
      tc_fence_after();
      float sv[kTile];
      {
        uint32_t (&r)[kTile] = *reinterpret_cast<uint32_t(*)[kTile]>(sv);
#pragma unroll
        for (int q4 = 0; q4 < kTile / 32; ++q4)
          tmem_ld_32x32b_x32(lrow + C::S_COL + (j & 1) * kTile + q4 * 32,
                             *reinterpret_cast<uint32_t(*)[32]>(r + q4 * 32));
        tmem_ld_wait();
      }
      const int kv0 = j * kTile;
      if ((sh.causal && kv0 + kTile - 1 > q0) || kv0 + kTile > sh.seq) {
        int lim = sh.seq - 1 - kv0;  // last valid column of this tile
        if (sh.causal && qpos - kv0 < lim) lim = qpos - kv0;
#pragma unroll
        for (int i = 0; i < kTile; ++i)
          if (i > lim) sv[i] = -INFINITY;
      }
      float mx = sv[0];
#pragma unroll
      for (int i = 1; i < kTile; ++i) mx = fmaxf(mx, sv[i]);
      const float m_tile = mx * c;
      const float m_new = fmaxf(m, m_tile);
      if (j == 0) {
        m = m_new;
      } else if (__any_sync(0xffffffffu, m_new > m + kRescaleLog2)) {
        // Move m and rescale this row's O (after the previous P V landed).
        const float f = m == -INFINITY ? 0.0f : ex2_approx(m - m_new);
        ok = mbar_wait(o_done((j - 1) & 1), ((j - 1) >> 1) & 1, p.status);
        if (!ok) break;
        tc_fence_after();
#pragma unroll
        for (int c4 = 0; c4 < D / 32; ++c4) {
          uint32_t o[32];
          tmem_ld_32x32b_x32(lrow + C::O_COL + c4 * 32, o);
          tmem_ld_wait();
#pragma unroll
          for (int i = 0; i < 32; ++i) o[i] = __float_as_uint(__uint_as_float(o[i]) * f);
          tmem_st_32x32b_x32(lrow + C::O_COL + c4 * 32, o);
        }
        tmem_st_wait();
        l *= f;
        m = m_new;
      }
      const float mref = m == -INFINITY ? 0.0f : m;
      float rs = 0.0f;
      uint32_t pk[kTile / 2];
#pragma unroll
      for (int i = 0; i < kTile; i += 2) {
        const float p0 = ex2_approx(fmaf(sv[i], c, -mref));
        const float p1 = ex2_approx(fmaf(sv[i + 1], c, -mref));
        rs += p0 + p1;
        pk[i / 2] = pack_bf16x2_f32(p0, p1);
      }
      l += rs;
      const uint32_t pcol = lrow + C::P_COL + (j & 1) * 64;
      tmem_st_32x32b_x32(pcol, *reinterpret_cast<uint32_t(*)[32]>(pk));
      tmem_st_32x32b_x32(pcol + 32, *reinterpret_cast<uint32_t(*)[32]>(pk + 32));
      tmem_st_wait();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(p_ready(j & 1));
    }
    if (ok && n_kv > 0) ok = mbar_wait(o_done((n_kv - 1) & 1), ((n_kv - 1) >> 1) & 1, p.status);
    tc_fence_after();
    if (ok) {
      const float inv = l > 0.0f ? 1.0f / l : 0.0f;
      const bool valid = qpos < sh.seq;
      uint16_t* orow = p.out + ((static_cast<size_t>(b) * sh.seq + qpos) * sh.heads + h) * D;
#pragma unroll
      for (int c4 = 0; c4 < D / 32; ++c4) {
        uint32_t o[32];
        tmem_ld_32x32b_x32(lrow + C::O_COL + c4 * 32, o);
        tmem_ld_wait();
        uint32_t w[16];
#pragma unroll
        for (int i = 0; i < 16; ++i)
          w[i] = pack_bf16x2_f32(__uint_as_float(o[2 * i]) * inv,
                                 __uint_as_float(o[2 * i + 1]) * inv);
        if (valid) {
          uint4* dst = reinterpret_cast<uint4*>(orow + c4 * 32);
#pragma unroll
          for (int i = 0; i < 4; ++i)
            dst[i] = make_uint4(w[4 * i], w[4 * i + 1], w[4 * i + 2], w[4 * i + 3]);
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

// [batch, seq, heads, dim] bf16 as a 4D tensor map, one 64-wide dim slab x
// 128 rows of one head per box (128-byte swizzle).
int map_bshd(CUtensorMap* map, const void* ptr, int64_t batch, int64_t seq, int64_t heads,
             int64_t dim) {
  const uint64_t dims[4] = {static_cast<uint64_t>(dim), static_cast<uint64_t>(heads),
                            static_cast<uint64_t>(seq), static_cast<uint64_t>(batch)};
  const uint64_t strides[3] = {static_cast<uint64_t>(dim) * 2,
                               static_cast<uint64_t>(heads * dim) * 2,
                               static_cast<uint64_t>(seq * heads * dim) * 2};
  const uint32_t box[4] = {64, 1, kTile, 1};
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
  p.out = static_cast<uint16_t*>(out);
  p.lse = lse;
  p.status = status;
  const unsigned grid = static_cast<unsigned>(sh.batch) * sh.heads * sh.n_tiles;
  attn_fwd_kernel<D><<<grid, 256, C::SMEM, stream>>>(tq_, tk, tv, p);
  return check_cuda(cudaGetLastError(), "attention forward launch");
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
