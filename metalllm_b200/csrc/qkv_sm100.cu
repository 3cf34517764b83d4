// qkv_sm100.cu -- computeQKV (attention.metal:19-53) on sm_100a:
//   Q = X Wq, K = X Wk, V = X Wv     X [rows][N], W [N][N] (row = input
//                                    feature), outputs [rows][N], bf16
// One CTA per (128-row, BN-column) output tile computes all three products
// from one shared X tile, as the reference's threadgroups do
// (attention.metal:43-52): per 64-wide K step, TMA brings X (K-major) and the
// three W tiles (MN-major: output columns contiguous) into a 3-stage ring, one
// thread issues 3 x 4 tcgen05.mma into three TMEM accumulators (fp32), and
// four epilogue warps convert them to bf16 and store them with TMA.
//
// Roles (192 threads): warp 0 TMA producer, warp 1 TMEM owner + UMMA issuer,
// warps 2-5 epilogue (thread = output row = TMEM lane).  All mbarrier waits
// are bounded; on time-out the CTA winds down and sets STATUS_QKV_TIMEOUT.
#include "common.cuh"
#include "sm100.cuh"
#include "tmap.h"

namespace ma {
namespace {

using namespace sm100;

constexpr int BM = 128;   // output rows per CTA
constexpr int BK = 64;    // K per stage (one 128-byte swizzle row of bf16)
constexpr int STAGES = 3;
constexpr int NUM_THREADS = 192;

template <int BN>
struct QkvCfg {
  static constexpr uint32_t X_BYTES = BM * BK * 2;   // 16 KB
  static constexpr uint32_t W_BYTES = BK * BN * 2;   // 8 / 16 KB per weight
  static constexpr uint32_t STAGE_BYTES = X_BYTES + 3 * W_BYTES;
  static constexpr uint32_t OFF_STAGE = 0;
  static constexpr uint32_t OFF_BAR = STAGES * STAGE_BYTES;
  // full[STAGES], empty[STAGES], done
  static constexpr uint32_t OFF_TSLOT = OFF_BAR + (2 * STAGES + 1) * 8;
  static constexpr uint32_t SMEM_BYTES = OFF_TSLOT + 16 + 1024;
  static constexpr uint32_t TMEM_COLS = 3 * BN <= 256 ? 256 : 512;
  // epilogue staging (after the main loop): one output tile, BN/64 blocks of
  // [128 rows][128 B], placed at the start of the stage ring
  static constexpr uint32_t OUT_BYTES = BM * BN * 2;
  static_assert(OUT_BYTES <= STAGES * STAGE_BYTES, "staging must fit in the ring");
};

template <int BN>
__global__ void __launch_bounds__(NUM_THREADS, 1)
    qkv_kernel(const __grid_constant__ CUtensorMap tmX, const __grid_constant__ CUtensorMap tmWq,
               const __grid_constant__ CUtensorMap tmWk, const __grid_constant__ CUtensorMap tmWv,
               const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
               const __grid_constant__ CUtensorMap tmV, int N, uint32_t* status) {
  pdl_wait_and_release();
  using C = QkvCfg<BN>;
  extern __shared__ uint8_t smem_raw[];
  __shared__ int abort_flag;
  const uint32_t raw = smem_u32(smem_raw);
  const uint32_t sbase = (raw + 1023u) & ~1023u;
  uint8_t* gbase = smem_raw + (sbase - raw);
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const int row0 = blockIdx.x * BM, col0 = blockIdx.y * BN;
  const int nk = N / BK;

  const uint32_t bar0 = sbase + C::OFF_BAR;
  auto BAR_F = [&](int s) { return bar0 + 8u * s; };
  auto BAR_E = [&](int s) { return bar0 + 8u * (STAGES + s); };
  const uint32_t BAR_DONE = bar0 + 8u * (2 * STAGES);
  const uint32_t tslot = sbase + C::OFF_TSLOT;
  if (threadIdx.x == 0) {
    abort_flag = 0;
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(BAR_F(s), 1);
      mbar_init(BAR_E(s), 1);
    }
    mbar_init(BAR_DONE, 1);
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc(tslot, C::TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *reinterpret_cast<volatile uint32_t*>(gbase + C::OFF_TSLOT);
  volatile int* abort_p = &abort_flag;

  if (warp == 0) {
    if (lane == 0) {
      const CUtensorMap* wmap[3] = {&tmWq, &tmWk, &tmWv};
      for (int k = 0; k < nk; ++k) {
        const int st = k % STAGES;
        if (k >= STAGES && !mbar_wait(BAR_E(st), ((k / STAGES) - 1) & 1, abort_p)) break;
        const uint32_t sx = sbase + C::OFF_STAGE + st * C::STAGE_BYTES;
        mbar_arrive_expect_tx(BAR_F(st), C::STAGE_BYTES);
        tma_load_2d(sx, &tmX, BAR_F(st), k * BK, row0);
        for (int w = 0; w < 3; ++w)
          for (int nb = 0; nb < BN / 64; ++nb)
            tma_load_2d(sx + C::X_BYTES + w * C::W_BYTES + nb * (BK * 128), wmap[w], BAR_F(st),
                        col0 + nb * 64, k * BK);
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      constexpr uint32_t IDESC = idesc_bf16_f32(BM, BN, 0, 1);
      for (int k = 0; k < nk; ++k) {
        const int st = k % STAGES;
        if (!mbar_wait(BAR_F(st), (k / STAGES) & 1, abort_p)) break;
        tc_fence_after();
        const uint32_t sx = sbase + C::OFF_STAGE + st * C::STAGE_BYTES;
#pragma unroll
        for (int w = 0; w < 3; ++w) {
          const uint32_t sw = sx + C::X_BYTES + w * C::W_BYTES;
#pragma unroll
          for (int kk = 0; kk < BK / 16; ++kk) {
            const uint64_t ad = smem_desc_sw128(sx + kk * 32, 16, 1024);
            const uint64_t bd = smem_desc_sw128(sw + kk * 2048, BK * 128, 1024);
            umma_bf16_ss(tmem + w * BN, ad, bd, IDESC, (k > 0 || kk > 0) ? 1u : 0u);
          }
        }
        umma_commit(BAR_E(st));
        if (k + 1 == nk) umma_commit(BAR_DONE);
      }
    }
  } else {
    // ----------------------------------------------------------- epilogue
    const int quarter = warp & 3;
    const int row = quarter * 32 + lane;
    const uint32_t trow = tmem + ((uint32_t)(quarter * 32) << 16);
    const bool leader = (warp == 2 && lane == 0);
    const CUtensorMap* omap[3] = {&tmQ, &tmK, &tmV};
    bool ok = mbar_wait_warp(BAR_DONE, 0, abort_p);
    for (int w = 0; w < 3; ++w) {
      // the previous output's store must have read the staging buffer
      if (w > 0 && leader) bulk_wait_read<0>();
      ok = bar_red_and(1, 128, ok);
      if (ok) {
        tc_fence_after();
        uint8_t* stage = gbase + C::OFF_STAGE;
#pragma unroll
        for (int cc = 0; cc < BN; cc += 16) {
          uint32_t r[16];
          tmem_ld16(trow + w * BN + cc, r);
          tmem_wait_ld_dep(r);
          uint4 v0, v1;
          v0.x = pack_bf16(__uint_as_float(r[0]), __uint_as_float(r[1]));
          v0.y = pack_bf16(__uint_as_float(r[2]), __uint_as_float(r[3]));
          v0.z = pack_bf16(__uint_as_float(r[4]), __uint_as_float(r[5]));
          v0.w = pack_bf16(__uint_as_float(r[6]), __uint_as_float(r[7]));
          v1.x = pack_bf16(__uint_as_float(r[8]), __uint_as_float(r[9]));
          v1.y = pack_bf16(__uint_as_float(r[10]), __uint_as_float(r[11]));
          v1.z = pack_bf16(__uint_as_float(r[12]), __uint_as_float(r[13]));
          v1.w = pack_bf16(__uint_as_float(r[14]), __uint_as_float(r[15]));
          const int kb = cc / 64, ch = (cc % 64) / 8;
          uint8_t* rowp = stage + kb * (BM * 128) + row * 128;
          *reinterpret_cast<uint4*>(rowp + ((ch ^ (row & 7)) * 16)) = v0;
          *reinterpret_cast<uint4*>(rowp + (((ch + 1) ^ (row & 7)) * 16)) = v1;
        }
        fence_proxy_async_smem();
      }
      ok = bar_red_and(1, 128, ok);
      if (ok && leader) {
        for (int kb = 0; kb < BN / 64; ++kb)
          tma_store_2d(omap[w], sbase + C::OFF_STAGE + kb * (BM * 128), col0 + kb * 64, row0);
        bulk_commit();
      }
    }
    if (leader) bulk_wait<0>();
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, C::TMEM_COLS);
  }
  if (threadIdx.x == 0 && abort_flag) atomicOr(status, STATUS_QKV_TIMEOUT);
}

template <int BN>
cudaError_t launch(const __nv_bfloat16* X, __nv_bfloat16* q, __nv_bfloat16* k, __nv_bfloat16* v,
                   const __nv_bfloat16* qw, const __nv_bfloat16* kw, const __nv_bfloat16* vw,
                   int rows, int N, uint32_t* status, cudaStream_t st) {
  using C = QkvCfg<BN>;
  CUtensorMap tx, twq, twk, twv, tq, tk, tv;
  const CUtensorMapDataType bf = CU_TENSOR_MAP_DATA_TYPE_BFLOAT16;
  const CUtensorMapSwizzle sw = CU_TENSOR_MAP_SWIZZLE_128B;
  if (!make_tmap_2d(&tx, X, bf, 2, N, rows, 64, BM, sw) ||
      !make_tmap_2d(&twq, qw, bf, 2, N, N, 64, BK, sw) ||
      !make_tmap_2d(&twk, kw, bf, 2, N, N, 64, BK, sw) ||
      !make_tmap_2d(&twv, vw, bf, 2, N, N, 64, BK, sw) ||
      !make_tmap_2d(&tq, q, bf, 2, N, rows, 64, BM, sw) ||
      !make_tmap_2d(&tk, k, bf, 2, N, rows, 64, BM, sw) ||
      !make_tmap_2d(&tv, v, bf, 2, N, rows, 64, BM, sw))
    return cudaErrorInvalidValue;
  cudaError_t e = cudaFuncSetAttribute(qkv_kernel<BN>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       C::SMEM_BYTES);
  if (e != cudaSuccess) return e;
  const dim3 grid((rows + BM - 1) / BM, N / BN);
  launch_pdl(qkv_kernel<BN>, grid, NUM_THREADS, C::SMEM_BYTES, st, tx, twq, twk, twv, tq, tk, tv, N, status);
  count_launches(1);
  return cudaGetLastError();
}

}  // namespace

cudaError_t launch_qkv(const __nv_bfloat16* X, __nv_bfloat16* q, __nv_bfloat16* k,
                       __nv_bfloat16* v, const __nv_bfloat16* qw, const __nv_bfloat16* kw,
                       const __nv_bfloat16* vw, int rows, int N, uint32_t* status,
                       cudaStream_t st) {
  return N % 128 == 0 ? launch<128>(X, q, k, v, qw, kw, vw, rows, N, status, st)
                      : launch<64>(X, q, k, v, qw, kw, vw, rows, N, status, st);
}

}  // namespace ma
