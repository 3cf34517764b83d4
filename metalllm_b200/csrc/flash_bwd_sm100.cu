// flash_bwd_sm100.cu -- flashAttentionBackward (attention.metal:198-299) on
// sm_100a with tcgen05 UMMA, TMEM accumulators and TMA.
//
// Work unit, as in the reference (attention.metal:219-223): one CTA owns one
// 128-key tile of one (batch, head) and walks the query tiles i from the
// diagonal to the end (causal: earlier queries never see these keys).  Per
// query tile (128 queries):
//   S^T  = K Q_i^T                 UMMA 128x128xD  -> TMEM
//   dP^T = V dO_i^T                UMMA 128x128xD  -> TMEM
//   P^T  = exp2(S^T c - l_i log2e), 0 where key > query   (compute warps)
//   dS^T = P^T (dP^T - D_i) / sqrt(D)                       (compute warps)
//   dV  += P^T dO_i                UMMA 128xDx128  (TMEM-resident)
//   dK  += dS^T Q_i                UMMA 128xDx128  (TMEM-resident)
//   dQ_i = dS K                    UMMA 128xDx128  -> TMEM -> smem -> TMA
//                                  bulk reduce-add into fp32 dQ in global
// dS^T is written once to shared memory (bf16, K-major 128-byte swizzle); the
// dQ UMMA reads the same buffer as an MN-major operand.  At D=64, P^T goes to
// TMEM (bf16 pairs) and dV's UMMA takes it from there; at D=128 TMEM is full
// and P^T goes to shared memory like dS^T.  dK/dV are owned by the CTA and
// stored once (bf16); dQ is accumulated in fp32 by the bulk reductions of
// every key tile, so the launcher zeroes it first (the reference's host zeroes
// it, model.h:549).  The CTAs of one (batch, head) are launched next to each
// other, so its Q/dO tiles are re-read from L2 rather than HBM.
//
// Roles (384 threads, three warpgroups):
//   warpgroup 0 (120 registers per thread after setmaxnreg):
//     warp 0   TMA producer: K/V once, Q_i/dO_i into a STAGES-deep ring
//     warp 1   TMEM owner; lane 0 issues every UMMA and commit
//     warp 2   statistics: stages -l_i*log2(e) and -D_i/sqrt(D) per query
//              (strided in global memory) 8 tiles ahead
//     warp 3   lane 0 issues the dQ bulk reductions
//   warpgroups 1, 2 (192 registers): compute, thread = key row = TMEM lane;
//              warpgroup 1 takes query columns 0-63, warpgroup 2 columns
//              64-127; dQ drain into the staging buffer and dK/dV epilogue.
// D=64 schedule ("early S"): S^T/dP^T of tile i+1 are issued as soon as the
// compute warps have read tile i's, so they run on the tensor core while the
// compute warps form P^T_i/dS^T_i; dV_i, dK_i and dQ_i follow.  dQ_{i-1} is
// drained after tile i is handed over.  D=128 has no TMEM room for that (S^T,
// dP^T, dV, dK fill all 512 columns; dQ reuses the S^T columns) and runs the
// steps in order, draining dQ_i before S^T_{i+1}.
//
// Conventions as the reference: P = exp(S/sqrt(D) - l) with l read as stored,
// D read as stored (bf16), dS includes 1/sqrt(D).  The reference rounds S,
// dP, P, dS and the dQ tile to bf16 and accumulates dK/dV in bf16 memory;
// here S, dP, dQ and dK/dV stay fp32 until their single store, and P, dS are
// bf16 (the UMMA operand type).
//
// All mbarrier waits are bounded (about 2 s); on time-out the CTA winds down,
// frees its TMEM and sets STATUS_BWD_TIMEOUT.  The compute warps meet only at
// mbarriers inside the loop and at one named barrier (same count on every
// path) for the epilogue.
#include "common.cuh"
#include "sm100.cuh"
#include "tmap.h"

namespace ma {
namespace {

using namespace sm100;

constexpr int BK = 128;  // keys per CTA
constexpr int BQ = 128;  // queries per step
constexpr int NUM_THREADS = 384;
constexpr int NCOMP = 256;  // compute threads (warpgroups 1 and 2)
constexpr int LAUNCH_REGS = 168;    // 65536 / 384, rounded down to a multiple of 8
constexpr int REGS_PRODUCER = 120;  // warpgroup 0 after setmaxnreg.dec
constexpr int REGS_COMPUTE = 192;   // warpgroups 1, 2 after setmaxnreg.inc
static_assert(128 * REGS_PRODUCER + 256 * REGS_COMPUTE == NUM_THREADS * LAUNCH_REGS,
              "register split must equal the launch allocation");
constexpr int SSTAGES = 8;  // statistics stages
constexpr float LOG2E = 1.4426950408889634f;

template <int HD>
struct BwdCfg {
  static constexpr int KB = HD / 64;
  static constexpr bool D64 = HD == 64;
  static constexpr int STAGES = D64 ? 3 : 1;     // Q_i/dO_i stages
  static constexpr bool P_IN_TMEM = D64;         // P^T in TMEM (else smem)
  static constexpr bool EARLY_S = D64;           // S_{i+1} before dV_i/dK_i/dQ_i
  static constexpr bool DQ_ALIAS = !D64;         // dQ accumulator reuses the S^T columns
  static constexpr bool DQS_ALIAS = !D64;        // dQ staging reuses the P^T/dS^T smem
  static constexpr uint32_t KV_BYTES = BK * HD * 2;
  static constexpr uint32_t QD_BYTES = BQ * HD * 2;
  static constexpr uint32_t PT_BYTES = BK * BQ * 2;
  static constexpr uint32_t DQS_BYTES = BQ * HD * 4;
  static constexpr uint32_t STAT_BYTES = 2 * BQ * 4;  // -l*log2e[128], -D/sqrt(D)[128]
  static constexpr uint32_t OFF_K = 0;
  static constexpr uint32_t OFF_V = OFF_K + KV_BYTES;
  static constexpr uint32_t OFF_Q = OFF_V + KV_BYTES;                // [STAGES]
  static constexpr uint32_t OFF_DO = OFF_Q + STAGES * QD_BYTES;      // [STAGES]
  static constexpr uint32_t OFF_PT = OFF_DO + STAGES * QD_BYTES;     // only without P_IN_TMEM
  static constexpr uint32_t OFF_DST = OFF_PT + (P_IN_TMEM ? 0 : PT_BYTES);
  static constexpr uint32_t OFF_DQS = DQS_ALIAS ? OFF_PT : OFF_DST + PT_BYTES;
  static constexpr uint32_t OFF_STAT = DQS_ALIAS ? OFF_DST + PT_BYTES : OFF_DQS + DQS_BYTES;
  static constexpr uint32_t OFF_BAR = OFF_STAT + SSTAGES * STAT_BYTES;
  // epilogue staging of dV and dK (bf16): the P^T/dS^T region (D=128) or the
  // dS^T region (D=64, 16 KB each)
  static constexpr uint32_t OFF_EPI_V = P_IN_TMEM ? OFF_DST : OFF_PT;
  static constexpr uint32_t OFF_EPI_K = P_IN_TMEM ? OFF_DST + BK * HD * 2 : OFF_DST;
  // kv_full, qd_full[S], qd_empty[S], st_full[8], st_empty[8], s_full, s_free,
  // p_ready, p_free, dq_full, dq_free, dqs_full, dqs_free, done
  static constexpr int NBAR = 1 + 2 * STAGES + 2 * SSTAGES + 9;
  static constexpr uint32_t OFF_TSLOT = OFF_BAR + NBAR * 8;
  static constexpr uint32_t SMEM_BYTES = OFF_TSLOT + 16 + 1024;
  static constexpr uint32_t TCOL_S = 0;
  static constexpr uint32_t TCOL_DP = 128;
  static constexpr uint32_t TCOL_DV = 256;
  static constexpr uint32_t TCOL_DK = 256 + HD;
  static constexpr uint32_t TCOL_DQ = DQ_ALIAS ? 0 : 256 + 2 * HD;
  static constexpr uint32_t TCOL_PT = 256 + 3 * HD;  // D=64 only: 64 columns of bf16 pairs
};

struct BwdParams {
  int T, N, NH, bh_begin, nbh, nkt;
  float scale, scale_log2;
  const float* lse;
  const __nv_bfloat16* Dv;
  uint32_t* status;
};

// P^T and dS^T for 64 query columns of one key row.  s[] holds S^T on entry
// and P^T on exit; dp[] holds dP^T on entry and dS^T on exit.  nl = -l*log2e
// and nd = -D/sqrt(D) per query column (shared memory, broadcast reads).
template <bool DIAG>
__device__ __forceinline__ void p_ds_row(float (&s)[64], float (&dp)[64], const float* nl,
                                         const float* nd, float c, float sc, int krow, int qcol0) {
  const float2 c2 = make_float2(c, c), sc2 = make_float2(sc, sc);
#pragma unroll
  for (int j = 0; j < 64; j += 4) {
    const float4 L = *reinterpret_cast<const float4*>(nl + j);
    const float4 Dn = *reinterpret_cast<const float4*>(nd + j);
    const float2 t0 = __ffma2_rn(make_float2(s[j], s[j + 1]), c2, make_float2(L.x, L.y));
    const float2 t1 = __ffma2_rn(make_float2(s[j + 2], s[j + 3]), c2, make_float2(L.z, L.w));
    float p0 = ex2(t0.x), p1 = ex2(t0.y), p2 = ex2(t1.x), p3 = ex2(t1.y);
    if (DIAG) {  // key after query: P = 0 (attention.metal:282)
      const int q = qcol0 + j;
      if (krow > q) p0 = 0.0f;
      if (krow > q + 1) p1 = 0.0f;
      if (krow > q + 2) p2 = 0.0f;
      if (krow > q + 3) p3 = 0.0f;
    }
    const float2 d0 = __ffma2_rn(make_float2(dp[j], dp[j + 1]), sc2, make_float2(Dn.x, Dn.y));
    const float2 d1 = __ffma2_rn(make_float2(dp[j + 2], dp[j + 3]), sc2, make_float2(Dn.z, Dn.w));
    const float2 r0 = __fmul2_rn(make_float2(p0, p1), d0);
    const float2 r1 = __fmul2_rn(make_float2(p2, p3), d1);
    s[j] = p0;
    s[j + 1] = p1;
    s[j + 2] = p2;
    s[j + 3] = p3;
    dp[j] = r0.x;
    dp[j + 1] = r0.y;
    dp[j + 2] = r1.x;
    dp[j + 3] = r1.y;
  }
}

// 64 bf16 values of one row as 8 swizzled 16-byte chunks of a K-major SW128
// row (row base `rowp`, swizzle phase `row & 7`).
__device__ __forceinline__ void store_row_sw128(uint8_t* rowp, int row, const float (&v)[64]) {
#pragma unroll
  for (int ch = 0; ch < 8; ++ch) {
    const int c0 = ch * 8;
    uint4 w;
    w.x = pack_bf16(v[c0 + 0], v[c0 + 1]);
    w.y = pack_bf16(v[c0 + 2], v[c0 + 3]);
    w.z = pack_bf16(v[c0 + 4], v[c0 + 5]);
    w.w = pack_bf16(v[c0 + 6], v[c0 + 7]);
    *reinterpret_cast<uint4*>(rowp + ((ch ^ (row & 7)) * 16)) = w;
  }
}

template <int HD>
__global__ void __launch_bounds__(NUM_THREADS, 1)
    flash_bwd_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                     const __grid_constant__ CUtensorMap tmV, const __grid_constant__ CUtensorMap tmdO,
                     const __grid_constant__ CUtensorMap tmdQ, const __grid_constant__ CUtensorMap tmdK,
                     const __grid_constant__ CUtensorMap tmdV, const BwdParams prm) {
  using C = BwdCfg<HD>;
  extern __shared__ uint8_t smem_raw[];
  __shared__ int abort_flag;
  const uint32_t raw = smem_u32(smem_raw);
  const uint32_t sbase = (raw + 1023u) & ~1023u;
  uint8_t* gbase = smem_raw + (sbase - raw);

  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  // the key tiles of one (batch, head) are adjacent in launch order (heaviest
  // first within the group), so they share Q/dO through L2
  const int idx = blockIdx.x;
  const int bh = prm.bh_begin + idx / prm.nkt;
  const int kt = idx % prm.nkt;
  const int b = bh / prm.NH, h = bh % prm.NH;
  const int nq = prm.nkt - kt;  // query tiles kt .. nkt-1
  const int col0 = h * HD;

  const uint32_t bar0 = sbase + C::OFF_BAR;
  const uint32_t BAR_KV = bar0;
  auto BAR_QF = [&](int s) { return bar0 + 8u * (1 + s); };
  auto BAR_QE = [&](int s) { return bar0 + 8u * (1 + C::STAGES + s); };
  auto BAR_TF = [&](int s) { return bar0 + 8u * (1 + 2 * C::STAGES + s); };
  auto BAR_TE = [&](int s) { return bar0 + 8u * (1 + 2 * C::STAGES + SSTAGES + s); };
  const uint32_t BAR_SF = bar0 + 8u * (1 + 2 * C::STAGES + 2 * SSTAGES);
  const uint32_t BAR_SE = BAR_SF + 8;
  const uint32_t BAR_PR = BAR_SF + 16;
  const uint32_t BAR_PE = BAR_SF + 24;
  const uint32_t BAR_DQF = BAR_SF + 32;
  const uint32_t BAR_DQE = BAR_SF + 40;
  const uint32_t BAR_DSF = BAR_SF + 48;  // dQ staging written
  const uint32_t BAR_DSE = BAR_SF + 56;  // dQ staging read by the reduction
  const uint32_t BAR_DONE = BAR_SF + 64;
  const uint32_t tslot = sbase + C::OFF_TSLOT;
  float* stat_base = reinterpret_cast<float*>(gbase + C::OFF_STAT);

  if (threadIdx.x == 0) {
    abort_flag = 0;
    mbar_init(BAR_KV, 1);
    for (int s = 0; s < C::STAGES; ++s) {
      mbar_init(BAR_QF(s), 1);
      mbar_init(BAR_QE(s), 1);
    }
    for (int s = 0; s < SSTAGES; ++s) {
      mbar_init(BAR_TF(s), 32);
      mbar_init(BAR_TE(s), NCOMP);
    }
    mbar_init(BAR_SF, 1);
    mbar_init(BAR_SE, NCOMP);
    mbar_init(BAR_PR, NCOMP);
    mbar_init(BAR_PE, 1);
    mbar_init(BAR_DQF, 1);
    mbar_init(BAR_DQE, NCOMP);
    mbar_init(BAR_DSF, NCOMP);
    mbar_init(BAR_DSE, 1);
    mbar_init(BAR_DONE, 1);
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc(tslot, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *reinterpret_cast<volatile uint32_t*>(gbase + C::OFF_TSLOT);
  volatile int* abort_p = &abort_flag;

  if (warp < 4) {
    reg_dealloc<REGS_PRODUCER>();
    if (warp == 0) {
      // --------------------------------------------------------- producer
      if (lane == 0) {
        tma_prefetch_desc(&tmQ);
        tma_prefetch_desc(&tmdO);
        mbar_arrive_expect_tx(BAR_KV, 2 * C::KV_BYTES);
        for (int kb = 0; kb < C::KB; ++kb) {
          tma_load_3d(sbase + C::OFF_K + kb * BK * 128, &tmK, BAR_KV, col0 + kb * 64, kt * BK, b);
          tma_load_3d(sbase + C::OFF_V + kb * BK * 128, &tmV, BAR_KV, col0 + kb * 64, kt * BK, b);
        }
        for (int i = 0; i < nq; ++i) {
          const int st = i % C::STAGES;
          if (i >= C::STAGES && !mbar_wait(BAR_QE(st), ((i - C::STAGES) / C::STAGES) & 1, abort_p))
            break;
          const int qt = kt + i;
          mbar_arrive_expect_tx(BAR_QF(st), 2 * C::QD_BYTES);
          for (int kb = 0; kb < C::KB; ++kb) {
            tma_load_3d(sbase + C::OFF_Q + st * C::QD_BYTES + kb * BQ * 128, &tmQ, BAR_QF(st),
                        col0 + kb * 64, qt * BQ, b);
            tma_load_3d(sbase + C::OFF_DO + st * C::QD_BYTES + kb * BQ * 128, &tmdO, BAR_QF(st),
                        col0 + kb * 64, qt * BQ, b);
          }
        }
      }
    } else if (warp == 1) {
      // -------------------------------------------------------------- MMA
      if (lane == 0) {
        constexpr uint32_t IDESC_S = idesc_bf16_f32(BK, BQ, 0, 0);   // S^T, dP^T
        constexpr uint32_t IDESC_KV = idesc_bf16_f32(BK, HD, 0, 1);  // dV, dK
        constexpr uint32_t IDESC_Q = idesc_bf16_f32(BQ, HD, 1, 1);   // dQ
        const uint32_t sk = sbase + C::OFF_K, sv = sbase + C::OFF_V;
        const uint32_t spt = sbase + C::OFF_PT, sdst = sbase + C::OFF_DST;
        bool ok = mbar_wait(BAR_KV, 0, abort_p);
        // S^T_i and dP^T_i into their TMEM columns
        auto issue_s = [&](int i) -> bool {
          const int st = i % C::STAGES;
          if (!mbar_wait(BAR_QF(st), (i / C::STAGES) & 1, abort_p)) return false;
          if (i >= 1 && !mbar_wait(BAR_SE, (i - 1) & 1, abort_p)) return false;
          if (C::DQ_ALIAS && i >= 1 && !mbar_wait(BAR_DQE, (i - 1) & 1, abort_p)) return false;
          tc_fence_after();
          const uint32_t sq = sbase + C::OFF_Q + st * C::QD_BYTES;
          const uint32_t sdo = sbase + C::OFF_DO + st * C::QD_BYTES;
#pragma unroll
          for (int kk = 0; kk < HD / 16; ++kk) {
            const uint32_t off = (kk >> 2) * (BK * 128) + (kk & 3) * 32;
            umma_bf16_ss(tmem + C::TCOL_S, smem_desc_sw128(sk + off, 16, 1024),
                         smem_desc_sw128(sq + off, 16, 1024), IDESC_S, kk > 0 ? 1u : 0u);
          }
#pragma unroll
          for (int kk = 0; kk < HD / 16; ++kk) {
            const uint32_t off = (kk >> 2) * (BK * 128) + (kk & 3) * 32;
            umma_bf16_ss(tmem + C::TCOL_DP, smem_desc_sw128(sv + off, 16, 1024),
                         smem_desc_sw128(sdo + off, 16, 1024), IDESC_S, kk > 0 ? 1u : 0u);
          }
          umma_commit(BAR_SF);
          return true;
        };
        if (ok) ok = issue_s(0);
        for (int i = 0; ok && i < nq; ++i) {
          if (C::EARLY_S && i + 1 < nq && !issue_s(i + 1)) break;
          const int st = i % C::STAGES;
          const uint32_t sq = sbase + C::OFF_Q + st * C::QD_BYTES;
          const uint32_t sdo = sbase + C::OFF_DO + st * C::QD_BYTES;
          if (!mbar_wait(BAR_PR, i & 1, abort_p)) break;
          tc_fence_after();
#pragma unroll
          for (int kk = 0; kk < BQ / 16; ++kk) {  // dV += P^T dO_i
            const uint64_t bd = smem_desc_sw128(sdo + kk * 2048, BQ * 128, 1024);
            if (C::P_IN_TMEM) {
              umma_bf16_ts(tmem + C::TCOL_DV, tmem + C::TCOL_PT + kk * 8, bd, IDESC_KV,
                           (i > 0 || kk > 0) ? 1u : 0u);
            } else {
              const uint64_t ad = smem_desc_sw128(spt + (kk >> 2) * (BK * 128) + (kk & 3) * 32, 16, 1024);
              umma_bf16_ss(tmem + C::TCOL_DV, ad, bd, IDESC_KV, (i > 0 || kk > 0) ? 1u : 0u);
            }
          }
#pragma unroll
          for (int kk = 0; kk < BQ / 16; ++kk) {  // dK += dS^T Q_i
            const uint64_t ad = smem_desc_sw128(sdst + (kk >> 2) * (BK * 128) + (kk & 3) * 32, 16, 1024);
            const uint64_t bd = smem_desc_sw128(sq + kk * 2048, BQ * 128, 1024);
            umma_bf16_ss(tmem + C::TCOL_DK, ad, bd, IDESC_KV, (i > 0 || kk > 0) ? 1u : 0u);
          }
          umma_commit(BAR_QE(st));
          // the dQ columns must have been drained (dQ_{i-1})
          if (i >= 1 && !mbar_wait(BAR_DQE, (i - 1) & 1, abort_p)) break;
          tc_fence_after();
#pragma unroll
          for (int kk = 0; kk < BK / 16; ++kk) {  // dQ_i = dS K (A = dS^T as MN-major)
            const uint64_t ad = smem_desc_sw128(sdst + kk * 2048, BK * 128, 1024);
            const uint64_t bd = smem_desc_sw128(sk + kk * 2048, BK * 128, 1024);
            umma_bf16_ss(tmem + C::TCOL_DQ, ad, bd, IDESC_Q, kk > 0 ? 1u : 0u);
          }
          umma_commit(BAR_DQF);
          umma_commit(BAR_PE);
          if (!C::EARLY_S && i + 1 < nq && !issue_s(i + 1)) break;
          if (i + 1 == nq) umma_commit(BAR_DONE);
        }
      }
    } else if (warp == 2) {
      // ------------------------------------------------------- statistics
      const long long rbase = (long long)b * prm.T;
      for (int i = 0; i < nq; ++i) {
        const int st = i % SSTAGES;
        if (i >= SSTAGES && !mbar_wait_warp(BAR_TE(st), ((i / SSTAGES) - 1) & 1, abort_p)) break;
        const int qt = kt + i;
        float* stt = stat_base + st * (2 * BQ);
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          const int qi = lane * 4 + u;
          const int q = qt * BQ + qi;
          float nl = 0.0f, nd = 0.0f;
          if (q < prm.T) {
            const long long si = (rbase + q) * prm.NH + h;
            nl = -__ldg(prm.lse + si) * LOG2E;
            nd = -__bfloat162float(prm.Dv[si]) * prm.scale;
          }
          stt[qi] = nl;
          stt[BQ + qi] = nd;
        }
        mbar_arrive(BAR_TF(st));
      }
    } else {
      // ------------------------------------------------- dQ reduce issuer
      if (lane == 0) {
        for (int j = 0; j < nq; ++j) {
          if (!mbar_wait(BAR_DSF, j & 1, abort_p)) break;
          for (int box = 0; box < HD / 32; ++box)
            tma_reduce_add_3d(&tmdQ, sbase + C::OFF_DQS + box * (BQ * 128), col0 + box * 32,
                              (kt + j) * BQ, b);
          bulk_commit();
          bulk_wait_read<0>();  // the staging buffer may be rewritten
          mbar_arrive(BAR_DSE);
        }
        bulk_wait<0>();
      }
    }
  } else {
    reg_alloc<REGS_COMPUTE>();
    // ------------------------------------------------------------ compute
    const int cw = warp - 4;                   // 0..7
    const int quarter = warp & 3;              // TMEM lane quarter
    const int krow = quarter * 32 + lane;      // key row (and dQ query row) within the tile
    const int half = cw >> 2;                  // query columns half*64 .. +63
    const uint32_t tl = tmem + ((uint32_t)(quarter * 32) << 16);
    const float c = prm.scale_log2, sc = prm.scale;
    bool ok = true;

    // dQ_j: TMEM -> fp32 staging (128-byte swizzle, 32-column boxes); the
    // reduce issuer (warp 3) sends it to global memory
    auto drain_dq = [&](int j) {
      if (ok) ok = mbar_wait_warp(BAR_DQF, j & 1, abort_p);
      if (ok && j >= 1) ok = mbar_wait_warp(BAR_DSE, (j - 1) & 1, abort_p);
      if (!ok) return;
      tc_fence_after();
      constexpr int CPH = HD / 2;  // columns per half
      uint8_t* dqs = gbase + C::OFF_DQS;
#pragma unroll
      for (int cc = 0; cc < CPH; cc += 32) {
        uint32_t r[32];
        tmem_ld32(tl + C::TCOL_DQ + half * CPH + cc, r);
        tmem_wait_ld_dep(r);
        const int box = (half * CPH + cc) / 32;
        uint8_t* rowp = dqs + box * (BQ * 128) + krow * 128;
#pragma unroll
        for (int ch = 0; ch < 8; ++ch) {
          uint4 v = make_uint4(r[ch * 4 + 0], r[ch * 4 + 1], r[ch * 4 + 2], r[ch * 4 + 3]);
          *reinterpret_cast<uint4*>(rowp + ((ch ^ (krow & 7)) * 16)) = v;
        }
      }
      tc_fence_before();
      mbar_arrive(BAR_DQE);
      fence_proxy_async_smem();
      mbar_arrive(BAR_DSF);
    };

    for (int i = 0; ok && i < nq; ++i) {
      const int ss = i % SSTAGES;
      ok = mbar_wait_warp(BAR_SF, i & 1, abort_p);
      if (!ok) break;
      tc_fence_after();
      float s[64], dp[64];
      {
        uint32_t ra[32], rb[32];
        tmem_ld32(tl + C::TCOL_S + half * 64, ra);
        tmem_ld32(tl + C::TCOL_S + half * 64 + 32, rb);
        tmem_wait_ld_dep(ra, rb);
#pragma unroll
        for (int j = 0; j < 32; ++j) {
          s[j] = __uint_as_float(ra[j]);
          s[32 + j] = __uint_as_float(rb[j]);
        }
        tmem_ld32(tl + C::TCOL_DP + half * 64, ra);
        tmem_ld32(tl + C::TCOL_DP + half * 64 + 32, rb);
        tmem_wait_ld_dep(ra, rb);
#pragma unroll
        for (int j = 0; j < 32; ++j) {
          dp[j] = __uint_as_float(ra[j]);
          dp[32 + j] = __uint_as_float(rb[j]);
        }
      }
      tc_fence_before();
      mbar_arrive(BAR_SE);
      ok = mbar_wait_warp(BAR_TF(ss), (i / SSTAGES) & 1, abort_p);
      if (!ok) break;
      const float* stt = stat_base + ss * (2 * BQ) + half * 64;
      if (i == 0) p_ds_row<true>(s, dp, stt, stt + BQ, c, sc, krow, half * 64);
      else p_ds_row<false>(s, dp, stt, stt + BQ, c, sc, krow, half * 64);
      mbar_arrive(BAR_TE(ss));
      // the previous tile's UMMAs must be done with P^T/dS^T (and, when the
      // dQ staging shares their smem, its reduction must have read it)
      if (i >= 1) ok = mbar_wait_warp(BAR_PE, (i - 1) & 1, abort_p);
      if (ok && C::DQS_ALIAS && i >= 1) ok = mbar_wait_warp(BAR_DSE, (i - 1) & 1, abort_p);
      if (!ok) break;
      if (C::P_IN_TMEM) {
        uint32_t pk[32];
#pragma unroll
        for (int j = 0; j < 32; ++j) pk[j] = pack_bf16(s[2 * j], s[2 * j + 1]);
        tmem_st32(tl + C::TCOL_PT + half * 32, pk);
        tmem_wait_st();
      } else {
        store_row_sw128(gbase + C::OFF_PT + half * (BK * 128) + krow * 128, krow, s);
      }
      store_row_sw128(gbase + C::OFF_DST + half * (BK * 128) + krow * 128, krow, dp);
      fence_proxy_async_smem();
      tc_fence_before();
      mbar_arrive(BAR_PR);
      if (C::EARLY_S) {
        if (i >= 1) drain_dq(i - 1);
      } else {
        drain_dq(i);
      }
    }
    if (C::EARLY_S && ok && nq >= 1) drain_dq(nq - 1);

    // --------------------------------------------------- dK / dV epilogue
    bool epi = ok && mbar_wait_warp(BAR_DONE, 0, abort_p);
    // D=128: the last dQ staging (in the P^T/dS^T smem) must have been read
    if (epi && C::DQS_ALIAS) epi = mbar_wait_warp(BAR_DSE, (nq - 1) & 1, abort_p);
    if (epi) {
      tc_fence_after();
      constexpr int CPH = HD / 2;
#pragma unroll
      for (int which = 0; which < 2; ++which) {
        const uint32_t tcol = which == 0 ? C::TCOL_DV : C::TCOL_DK;
        uint8_t* stage = gbase + (which == 0 ? C::OFF_EPI_V : C::OFF_EPI_K);
#pragma unroll
        for (int cc = 0; cc < CPH; cc += 16) {
          uint32_t r[16];
          tmem_ld16(tl + tcol + half * CPH + cc, r);
          tmem_wait_ld_dep(r);
          const int col = half * CPH + cc;  // column within the head
          const int kb = col / 64, ch = (col % 64) / 8;
          uint8_t* rowp = stage + kb * (BK * 128) + krow * 128;
          uint4 v0, v1;
          v0.x = pack_bf16(__uint_as_float(r[0]), __uint_as_float(r[1]));
          v0.y = pack_bf16(__uint_as_float(r[2]), __uint_as_float(r[3]));
          v0.z = pack_bf16(__uint_as_float(r[4]), __uint_as_float(r[5]));
          v0.w = pack_bf16(__uint_as_float(r[6]), __uint_as_float(r[7]));
          v1.x = pack_bf16(__uint_as_float(r[8]), __uint_as_float(r[9]));
          v1.y = pack_bf16(__uint_as_float(r[10]), __uint_as_float(r[11]));
          v1.z = pack_bf16(__uint_as_float(r[12]), __uint_as_float(r[13]));
          v1.w = pack_bf16(__uint_as_float(r[14]), __uint_as_float(r[15]));
          *reinterpret_cast<uint4*>(rowp + ((ch ^ (krow & 7)) * 16)) = v0;
          *reinterpret_cast<uint4*>(rowp + (((ch + 1) ^ (krow & 7)) * 16)) = v1;
        }
      }
      fence_proxy_async_smem();
    }
    // one named barrier for the 256 compute threads, reached on every path
    epi = bar_red_and(1, NCOMP, epi);
    if (epi && cw == 0 && lane == 0) {
      for (int kb = 0; kb < C::KB; ++kb) {
        tma_store_3d(&tmdV, sbase + C::OFF_EPI_V + kb * BK * 128, col0 + kb * 64, kt * BK, b);
        tma_store_3d(&tmdK, sbase + C::OFF_EPI_K + kb * BK * 128, col0 + kb * 64, kt * BK, b);
      }
      bulk_commit();
      bulk_wait<0>();
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
  if (threadIdx.x == 0 && abort_flag) atomicOr(prm.status, STATUS_BWD_TIMEOUT);
}

// Zeroes the dQ columns of the (batch, head) shard range.
__global__ void zero_dq_shard_kernel(float4* __restrict__ dQ, int T, int N, int D, int NH,
                                     int bh_begin, int bh_end) {
  const long long per_bh = (long long)T * (D / 4);
  const long long total = (long long)(bh_end - bh_begin) * per_bh;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < total;
       i += (long long)gridDim.x * blockDim.x) {
    const long long bh = bh_begin + i / per_bh;
    const long long rem = i % per_bh;
    const long long t = rem / (D / 4), c4 = rem % (D / 4);
    const long long bb = bh / NH, hh = bh % NH;
    dQ[((bb * T + t) * N + hh * D) / 4 + c4] = make_float4(0.f, 0.f, 0.f, 0.f);
  }
}

template <int HD>
cudaError_t launch_bwd(const __nv_bfloat16* dO, const __nv_bfloat16* Dv, const float* lse,
                       const __nv_bfloat16* q, const __nv_bfloat16* k, const __nv_bfloat16* v,
                       float* dQ, __nv_bfloat16* dK, __nv_bfloat16* dV, const AttnShape& s,
                       uint32_t* status, cudaStream_t st) {
  using C = BwdCfg<HD>;
  // The setmaxnreg split assumes the kernel was compiled to exactly
  // LAUNCH_REGS registers per thread; refuse to launch otherwise.
  static const cudaError_t reg_check = [] {
    cudaFuncAttributes a;
    cudaError_t e = cudaFuncGetAttributes(&a, flash_bwd_kernel<HD>);
    if (e != cudaSuccess) return e;
    return a.numRegs == LAUNCH_REGS ? cudaSuccess : cudaErrorInvalidKernelImage;
  }();
  if (reg_check != cudaSuccess) return reg_check;
  CUtensorMap tq, tk, tv, tdo, tdq, tdk, tdv;
  const CUtensorMapDataType bf = CU_TENSOR_MAP_DATA_TYPE_BFLOAT16;
  const CUtensorMapSwizzle sw = CU_TENSOR_MAP_SWIZZLE_128B;
  if (!make_tmap_3d(&tq, q, bf, 2, s.N, s.T, s.B, 64, BQ, sw) ||
      !make_tmap_3d(&tk, k, bf, 2, s.N, s.T, s.B, 64, BK, sw) ||
      !make_tmap_3d(&tv, v, bf, 2, s.N, s.T, s.B, 64, BK, sw) ||
      !make_tmap_3d(&tdo, dO, bf, 2, s.N, s.T, s.B, 64, BQ, sw) ||
      !make_tmap_3d(&tdq, dQ, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, s.N, s.T, s.B, 32, BQ, sw) ||
      !make_tmap_3d(&tdk, dK, bf, 2, s.N, s.T, s.B, 64, BK, sw) ||
      !make_tmap_3d(&tdv, dV, bf, 2, s.N, s.T, s.B, 64, BK, sw))
    return cudaErrorInvalidValue;
  // dQ is accumulated by bulk reductions: zero the shard's columns first
  const int nbh = s.bh_end - s.bh_begin;
  cudaError_t e;
  if (s.bh_begin == 0 && s.bh_end == s.B * s.NH) {
    e = cudaMemsetAsync(dQ, 0, (size_t)s.B * s.T * s.N * sizeof(float), st);
  } else {
    zero_dq_shard_kernel<<<1184, 256, 0, st>>>(reinterpret_cast<float4*>(dQ), s.T, s.N, s.D, s.NH,
                                              s.bh_begin, s.bh_end);
    count_launches(1);
    e = cudaGetLastError();
  }
  if (e != cudaSuccess) return e;
  BwdParams prm;
  prm.T = s.T;
  prm.N = s.N;
  prm.NH = s.NH;
  prm.bh_begin = s.bh_begin;
  prm.nbh = nbh;
  prm.nkt = (s.T + BK - 1) / BK;
  prm.scale = 1.0f / sqrtf((float)HD);
  prm.scale_log2 = LOG2E / sqrtf((float)HD);
  prm.lse = lse;
  prm.Dv = Dv;
  prm.status = status;
  e = cudaFuncSetAttribute(flash_bwd_kernel<HD>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                           C::SMEM_BYTES);
  if (e != cudaSuccess) return e;
  const long long nblocks = (long long)prm.nkt * nbh;
  flash_bwd_kernel<HD><<<(unsigned)nblocks, NUM_THREADS, C::SMEM_BYTES, st>>>(tq, tk, tv, tdo, tdq,
                                                                            tdk, tdv, prm);
  count_launches(1);
  return cudaGetLastError();
}

}  // namespace

cudaError_t launch_flash_bwd(const __nv_bfloat16* dO, const __nv_bfloat16* Dv,
                             const float* lse, const __nv_bfloat16* q,
                             const __nv_bfloat16* k, const __nv_bfloat16* v, float* dQ,
                             __nv_bfloat16* dK, __nv_bfloat16* dV, const AttnShape& s,
                             uint32_t* status, cudaStream_t st) {
  if (s.bh_end <= s.bh_begin) return cudaSuccess;
  return s.D == 64 ? launch_bwd<64>(dO, Dv, lse, q, k, v, dQ, dK, dV, s, status, st)
                   : launch_bwd<128>(dO, Dv, lse, q, k, v, dQ, dK, dV, s, status, st);
}

}  // namespace ma
