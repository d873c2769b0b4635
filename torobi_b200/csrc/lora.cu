// The LoRA side branch's skinny products on the tensor cores.
//
// Both are GEMMs with a 16-wide side (rank 8 or 16; rank 8 zero-padded by the
// TMA out-of-bounds fill), so they are HBM-bound on streaming the big operand
// once.  One kernel serves both: a 128-row tile of the big operand on the
// UMMA's M side (TMEM lanes), the rank on its N side (16 columns).
//
//   down  (A K-major):  D[i, j] = sum_k x[i, k] * a[j, k]           i over rows of x
//   grad  (A MN-major): D[c, j] = sum_m x[m, c] * p_t[j, m]         c over columns of x
//
// down writes RNE(scale * D) as bf16 in [m, rank] and, optionally, [rank, m];
// grad reduces a slice of m per CTA and adds its partial into f32 g with
// atomics (g [c, rank] or [rank, c]).
#include <cuda_bf16.h>

#include "tq_ptx.cuh"
#include "tq_runtime.h"

namespace tq {
namespace {

constexpr int kBM = 128;
constexpr int kBK = 64;
constexpr int kThreads = 192;
constexpr int kStages = 8;
constexpr int kABytes = kBM * kBK * 2;  // 16 KB
constexpr int kBBytes = 16 * kBK * 2;   // 2 KB
constexpr int kStageBytes = kABytes + kBBytes;
constexpr int kSmem = 1024 + kStages * kStageBytes + 256;

struct SkinnyParams {
  int rows;        // down: m (rows of x); grad: c (columns of x)
  int red;         // reduction length (down: k; grad: m)
  int steps_per_cta;
  int rank;
  float scale;
  uint16_t* out;   // down
  uint16_t* out_t; // down (optional)
  float* g;        // grad
  int g_layout;    // grad: 0 -> [c, rank], 1 -> [rank, c]
  int ld_t;        // down: row pitch of out_t
  int* status;
};

template <bool GRAD>
__global__ void __launch_bounds__(kThreads, 1)
    skinny_kernel(const __grid_constant__ CUtensorMap tm_a, const __grid_constant__ CUtensorMap tm_b,
                  const SkinnyParams p) {
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw = smem_u32(smem_raw);
  const uint32_t base = (raw + 1023u) & ~1023u;
  uint8_t* const gbase = smem_raw + (base - raw);
  auto a_s = [&](int s) { return base + s * kStageBytes; };
  auto b_s = [&](int s) { return base + s * kStageBytes + kABytes; };
  const uint32_t bars = base + kStages * kStageBytes;
  auto full_b = [&](int s) { return bars + 8u * s; };
  auto empty_b = [&](int s) { return bars + 8u * (kStages + s); };
  const uint32_t acc_b = bars + 8u * (2 * kStages);
  const uint32_t tmem_slot = bars + 8u * (2 * kStages + 1);
  volatile uint32_t* tmem_slot_ptr =
      reinterpret_cast<volatile uint32_t*>(gbase + (tmem_slot - base));

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int row0 = blockIdx.x * kBM;
  const int total_steps = (p.red + kBK - 1) / kBK;
  const int step0 = blockIdx.y * p.steps_per_cta;
  int step1 = step0 + p.steps_per_cta;
  if (step1 > total_steps) step1 = total_steps;
  const int nsteps = step1 > step0 ? step1 - step0 : 0;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(full_b(s), 1);
      mbar_init(empty_b(s), 1);
    }
    mbar_init(acc_b, 1);
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, 32);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot_ptr;

  if (warp == 0) {
    if (elect_one_sync()) {
      tma_prefetch_desc(&tm_a);
      tma_prefetch_desc(&tm_b);
      bool ok = true;
      int issued = 0;
      for (int i = 0; i < nsteps && ok; ++i) {
        const int s = i % kStages;
        const uint32_t ph = (i / kStages) & 1;
        ok = mbar_wait(empty_b(s), ph ^ 1, p.status);
        if (!ok) break;
        const int r0 = (step0 + i) * kBK;
        mbar_arrive_expect_tx(full_b(s), kABytes + kBBytes);
        if constexpr (GRAD) {
          tma_load_2d(a_s(s), &tm_a, full_b(s), row0, r0);
          tma_load_2d(a_s(s) + 8192, &tm_a, full_b(s), row0 + 64, r0);
        } else {
          tma_load_2d(a_s(s), &tm_a, full_b(s), r0, row0);
        }
        tma_load_2d(b_s(s), &tm_b, full_b(s), r0, 0);
        ++issued;
      }
      for (int i = issued - kStages < 0 ? 0 : issued - kStages; i < issued; ++i)
        mbar_wait(full_b(i % kStages), (i / kStages) & 1, p.status);
    }
  } else if (warp == 1) {
    if (elect_one_sync()) {
      constexpr uint32_t idesc = make_idesc_bf16(kBM, 16, GRAD, false);
      uint32_t acc = 0;
      bool ok = true;
      for (int i = 0; i < nsteps && ok; ++i) {
        const int s = i % kStages;
        ok = mbar_wait(full_b(s), (i / kStages) & 1, p.status);
        if (!ok) break;
        tc_fence_after();
#pragma unroll
        for (int kk = 0; kk < kBK / 16; ++kk) {
          uint64_t adesc;
          if constexpr (GRAD)
            adesc = make_sdesc(a_s(s) + kk * 2048, 8192, 1024, kSw128);
          else
            adesc = make_sdesc(a_s(s) + kk * 32, 16, 1024, kSw128);
          const uint64_t bdesc = make_sdesc(b_s(s) + kk * 32, 16, 1024, kSw128);
          umma_bf16(tmem, adesc, bdesc, idesc, acc);
          acc = 1;
        }
        umma_commit(empty_b(s));
      }
      umma_commit(acc_b);
      mbar_wait(acc_b, 0, p.status);
    }
  } else {
    const bool ok = mbar_wait(acc_b, 0, p.status);
    tc_fence_after();
    const int q = warp & 3;
    const int r = row0 + q * 32 + lane;
    uint32_t v[16];
    tmem_ld_32x32b_x16(tmem + (static_cast<uint32_t>(q * 32) << 16), v);
    tmem_ld_wait();
    if (ok && nsteps > 0 && r < p.rows) {
      if constexpr (GRAD) {
        for (int j = 0; j < p.rank; ++j) {
          float* dst = p.g_layout == 0 ? p.g + static_cast<size_t>(r) * p.rank + j
                                       : p.g + static_cast<size_t>(j) * p.rows + r;
          atomicAdd(dst, __uint_as_float(v[j]));
        }
      } else {
        uint16_t h[16];
#pragma unroll
        for (int j = 0; j < 16; ++j)
          h[j] = __bfloat16_as_ushort(__float2bfloat16_rn(__uint_as_float(v[j]) * p.scale));
        uint4* dst = reinterpret_cast<uint4*>(p.out + static_cast<size_t>(r) * p.rank);
        dst[0] = make_uint4(h[0] | (uint32_t(h[1]) << 16), h[2] | (uint32_t(h[3]) << 16),
                            h[4] | (uint32_t(h[5]) << 16), h[6] | (uint32_t(h[7]) << 16));
        if (p.rank == 16)
          dst[1] = make_uint4(h[8] | (uint32_t(h[9]) << 16), h[10] | (uint32_t(h[11]) << 16),
                              h[12] | (uint32_t(h[13]) << 16), h[14] | (uint32_t(h[15]) << 16));
        if (p.out_t) {
          for (int j = 0; j < p.rank; ++j) p.out_t[static_cast<size_t>(j) * p.ld_t + r] = h[j];
        }
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc(tmem, 32);
  }
}

// Opt in to the large dynamic shared memory (once per device).
int set_smem_once() {
  int rc = set_max_smem_once(reinterpret_cast<const void*>(skinny_kernel<false>), kSmem,
                             "cudaFuncSetAttribute(skinny)");
  if (rc) return rc;
  return set_max_smem_once(reinterpret_cast<const void*>(skinny_kernel<true>), kSmem,
                           "cudaFuncSetAttribute(skinny)");
}

}  // namespace
}  // namespace tq

extern "C" int tq_lora_down(const void* x, const void* a, int64_t m, int64_t k, int64_t rank,
                            float scale, void* out, void* out_t, int64_t ld_t, void* stream) {
  using namespace tq;
  if (rank != 8 && rank != 16) return fail(TQ_ERR_UNSUPPORTED, "LoRA rank must be 8 or 16, got %lld", (long long)rank);
  if (m < 0 || k < 0) return fail(TQ_ERR_INVALID, "negative shape");
  if (k % 8 != 0) return fail(TQ_ERR_INVALID, "k (%lld) must be a multiple of 8", (long long)k);
  if (m > (1ll << 31) - 1 || k > (1ll << 31) - 1) return fail(TQ_ERR_INVALID, "dimensions must fit in 31 bits");
  if (out_t && (ld_t < m || ld_t % 8 != 0))
    return fail(TQ_ERR_INVALID, "ld_t (%lld) must be >= m (%lld) and a multiple of 8",
                (long long)ld_t, (long long)m);
  if (m == 0) return TQ_OK;
  if (!x || !a || !out) return fail(TQ_ERR_INVALID, "null pointer");
  if (!aligned(x, 16) || !aligned(a, 16) || !aligned(out, 16) || (out_t && !aligned(out_t, 2)))
    return fail(TQ_ERR_MISALIGNED, "x, a and out must be 16-byte aligned");
  int rc = set_smem_once();
  if (rc) return rc;
  int* status = device_status_ptr(&rc);
  if (!status) return rc;
  if (k == 0) {
    rc = check_cuda(cudaMemsetAsync(out, 0, m * rank * 2, as_stream(stream)), "memset");
    if (rc || !out_t) return rc;
    return check_cuda(cudaMemsetAsync(out_t, 0, ld_t * rank * 2, as_stream(stream)), "memset");
  }
  CUtensorMap tm_a, tm_b;
  {
    const uint64_t dims[2] = {static_cast<uint64_t>(k), static_cast<uint64_t>(m)};
    const uint64_t strides[1] = {static_cast<uint64_t>(k) * 2};
    const uint32_t box[2] = {kBK, kBM};
    rc = encode_tmap(&tm_a, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, x, dims, strides, box,
                     CU_TENSOR_MAP_SWIZZLE_128B);
    if (rc) return rc;
  }
  {
    const uint64_t dims[2] = {static_cast<uint64_t>(k), static_cast<uint64_t>(rank)};
    const uint64_t strides[1] = {static_cast<uint64_t>(k) * 2};
    const uint32_t box[2] = {kBK, 16};
    rc = encode_tmap(&tm_b, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, a, dims, strides, box,
                     CU_TENSOR_MAP_SWIZZLE_128B);
    if (rc) return rc;
  }
  SkinnyParams p{};
  p.rows = static_cast<int>(m);
  p.red = static_cast<int>(k);
  p.steps_per_cta = static_cast<int>((k + kBK - 1) / kBK);
  p.rank = static_cast<int>(rank);
  p.scale = scale;
  p.out = static_cast<uint16_t*>(out);
  p.out_t = static_cast<uint16_t*>(out_t);
  p.ld_t = static_cast<int>(ld_t);
  p.status = status;
  const dim3 grid(static_cast<unsigned>((m + kBM - 1) / kBM), 1);
  skinny_kernel<false><<<grid, kThreads, kSmem, as_stream(stream)>>>(tm_a, tm_b, p);
  return check_cuda(cudaGetLastError(), "lora_down launch");
}

extern "C" int tq_lora_grad(const void* x, const void* p_t, int64_t ld_p, int64_t m, int64_t c,
                            int64_t rank, int out_layout, int accumulate, void* g, void* stream) {
  using namespace tq;
  if (rank != 8 && rank != 16) return fail(TQ_ERR_UNSUPPORTED, "LoRA rank must be 8 or 16, got %lld", (long long)rank);
  if (m < 0 || c < 0) return fail(TQ_ERR_INVALID, "negative shape");
  if (c % 8 != 0) return fail(TQ_ERR_INVALID, "c (%lld) must be a multiple of 8", (long long)c);
  if (ld_p < m || ld_p % 8 != 0)
    return fail(TQ_ERR_INVALID, "ld_p (%lld) must be >= m (%lld) and a multiple of 8",
                (long long)ld_p, (long long)m);
  if (m > (1ll << 31) - 1 || c > (1ll << 31) - 1) return fail(TQ_ERR_INVALID, "dimensions must fit in 31 bits");
  if (out_layout != 0 && out_layout != 1) return fail(TQ_ERR_INVALID, "out_layout must be 0 or 1");
  if (c == 0) return TQ_OK;
  if (!x || !p_t || !g) return fail(TQ_ERR_INVALID, "null pointer");
  if (!aligned(x, 16) || !aligned(p_t, 16) || !aligned(g, 4))
    return fail(TQ_ERR_MISALIGNED, "x and p_t must be 16-byte aligned");
  cudaStream_t s = as_stream(stream);
  int rc = TQ_OK;
  if (!accumulate) {
    rc = check_cuda(cudaMemsetAsync(g, 0, c * rank * sizeof(float), s), "memset");
    if (rc) return rc;
  }
  if (m == 0) return TQ_OK;
  rc = set_smem_once();
  if (rc) return rc;
  int* status = device_status_ptr(&rc);
  if (!status) return rc;
  CUtensorMap tm_a, tm_b;
  {
    const uint64_t dims[2] = {static_cast<uint64_t>(c), static_cast<uint64_t>(m)};
    const uint64_t strides[1] = {static_cast<uint64_t>(c) * 2};
    const uint32_t box[2] = {64, kBK};
    rc = encode_tmap(&tm_a, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, x, dims, strides, box,
                     CU_TENSOR_MAP_SWIZZLE_128B);
    if (rc) return rc;
  }
  {
    const uint64_t dims[2] = {static_cast<uint64_t>(m), static_cast<uint64_t>(rank)};
    const uint64_t strides[1] = {static_cast<uint64_t>(ld_p) * 2};
    const uint32_t box[2] = {kBK, 16};
    rc = encode_tmap(&tm_b, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, p_t, dims, strides, box,
                     CU_TENSOR_MAP_SWIZZLE_128B);
    if (rc) return rc;
  }
  const int64_t tiles = (c + kBM - 1) / kBM;
  const int64_t steps = (m + kBK - 1) / kBK;
  // Enough CTAs to cover the SMs twice over, each reducing a contiguous slice.
  int64_t splits = (2 * sm_count() + tiles - 1) / tiles;
  if (splits > steps) splits = steps;
  if (splits < 1) splits = 1;
  const int64_t per = (steps + splits - 1) / splits;
  splits = (steps + per - 1) / per;
  SkinnyParams p{};
  p.rows = static_cast<int>(c);
  p.red = static_cast<int>(m);
  p.steps_per_cta = static_cast<int>(per);
  p.rank = static_cast<int>(rank);
  p.scale = 1.0f;
  p.g = static_cast<float*>(g);
  p.g_layout = out_layout;
  p.status = status;
  const dim3 grid(static_cast<unsigned>(tiles), static_cast<unsigned>(splits));
  skinny_kernel<true><<<grid, kThreads, kSmem, s>>>(tm_a, tm_b, p);
  return check_cuda(cudaGetLastError(), "lora_grad launch");
}
