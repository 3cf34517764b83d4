// flash_fwd_sm100.cu -- flashAttentionForward (attention.metal:56-164) on
// sm_100a: tcgen05 UMMA with TMEM accumulators, TMA-staged Q/K/V tiles in
// 128-byte-swizzled shared memory, an mbarrier pipeline and warp-specialised
// roles; each CTA walks many work units (static rounds, or launch control for
// long sequences: see decode_unit).
//
// Work unit: one (batch*head, 256-row query pair) = two 128-row query tiles
// A (rows 256p..256p+127) and B (the next 128 rows), heaviest first (see
// decode_unit).  Per key tile j (128 keys) of a unit:
//   S_X  = Q_X K_j^T          UMMA 128x128xD, fp32 in TMEM      (X = A, B)
//   P_X  = exp2(S_X c - m_X)  softmax warpgroup X, c = log2(e)/sqrt(D), bf16
//   O_X += P_X V_j            UMMA 128xDx128, fp32 in TMEM
// Tile A needs key tiles 0..2p, tile B 0..2p+1 (causal).  The tensor core
// works on one tile while the other tile's softmax runs (ping-pong); at D=64
// S_X(j+1) is issued as soon as softmax X has read S_X(j) into registers, so
// each softmax warpgroup finds its next scores ready.  K_j/V_j are loaded once
// for both tiles.
// Roles (384 threads, three warpgroups):
//   warpgroup 0  warp 0 TMA producer (Q pair per unit, K/V tile rings);
//                warp 1 owns TMEM (S_A, S_B, O_A, O_B) and issues every UMMA;
//                runs on 120 registers per thread (setmaxnreg)
//   warpgroups 1, 2  softmax of tile A resp. B on 192 registers: thread =
//                query row = TMEM lane; row max/sum in registers, lazy O
//                rescaling (only when the running max grows by more than 2^8),
//                epilogue O/rowsum -> bf16 -> smem -> TMA store, and
//                l = m + ln(rowsum) in fp32.  Given dO (D=64), the leader
//                also TMA-loads the dO tile into the O staging during the
//                last key tile and the epilogue forms computeD's
//                D = sum(bf16(O) * dO) per row before writing O over it.
// Conventions match the reference: scale 1/sqrt(D) applied to Q K^T, key >
// query masked, l stored fp32 at [row*NH + head], O = (sum P V) / rowsum.  S
// stays fp32 (the reference rounds it to bf16); P is bf16 as in the reference
// (attention.metal:139,153).
//
// Every mbarrier wait is bounded (about 2 s); on time-out the CTA sets an
// abort flag that all roles poll, winds down, frees its TMEM and sets
// STATUS_FWD_TIMEOUT in the device status word.
#include <type_traits>

#include "common.cuh"
#include "sm100.cuh"
#include "tmap.h"

namespace ma {
namespace {

using namespace sm100;

constexpr int BM = 128;  // query rows per tile
constexpr int BN = 128;  // keys per tile
constexpr int NUM_THREADS = 384;
constexpr int LAUNCH_REGS = 168;    // 65536 / 384, rounded down to a multiple of 8
constexpr int REGS_PRODUCER = 120;  // warpgroup 0 after setmaxnreg.dec
constexpr int REGS_SOFTMAX = 192;  // warpgroups 1, 2 after setmaxnreg.inc
static_assert(128 * REGS_PRODUCER + 256 * REGS_SOFTMAX == NUM_THREADS * LAUNCH_REGS,
              "register split must equal the launch allocation");
constexpr float LOG2E = 1.4426950408889634f;
constexpr float LN2 = 0.6931471805599453f;
constexpr float RESCALE_THRESHOLD = 8.0f;  // log2 units

template <int HD, bool DYN = false>
struct FwdCfg {
  static constexpr int KB = HD / 64;  // 64-column blocks per row
  static constexpr int QST = HD == 64 ? 2 : 1;  // Q-pair stages
  static constexpr int KST = HD == 64 ? 3 : 2;  // K tile stages
  static constexpr int VST = HD == 64 ? 3 : 1;  // V tile stages
  // UMMA issue order: D=64 issues S_X(j+1) before PV_X(j) (softmax-bound: the
  // next scores should be ready early); D=128 interleaves PV_X(j), S_X(j+1)
  // (tensor-bound: keeps PV close to its P)
  static constexpr bool EARLY_S = HD == 64;
  // D=64: P_X lives in TMEM (bf16 pairs) and PV_X reads it from there, which
  // halves the shared-memory traffic of the tensor core; D=128 has no TMEM
  // columns left and stages P in shared memory
  static constexpr bool P_TMEM = HD == 64;
  static constexpr uint32_t QT_BYTES = BM * HD * 2;  // one query tile
  static constexpr uint32_t KV_BYTES = BN * HD * 2;
  static constexpr uint32_t P_BYTES = BM * BN * 2;
  // per tile X: P (shared-memory P) or only the epilogue's O staging
  static constexpr uint32_t STG_BYTES = P_TMEM ? BM * HD * 2 : P_BYTES;
  // shared memory map (offsets from a 1024-aligned base)
  static constexpr uint32_t OFF_Q = 0;                          // [QST][2 tiles]
  static constexpr uint32_t OFF_K = OFF_Q + QST * 2 * QT_BYTES;  // [KST]
  static constexpr uint32_t OFF_V = OFF_K + KST * KV_BYTES;      // [VST]
  static constexpr uint32_t OFF_P = OFF_V + VST * KV_BYTES;      // [2 tiles] P / O staging
  // D=64: an all-zero fp32 tile (128 rows x 32 columns) that TMA stores copy
  // into dQ when the forward zeroes it for an accumulating backward
  static constexpr uint32_t ZT_BYTES = P_TMEM ? BM * 32 * 4 : 0;
  static constexpr uint32_t OFF_ZT = OFF_P + 2 * STG_BYTES;
  // the unit schedule: NSCHED 16-byte launch-control responses
  static constexpr int NSCHED = DYN ? (int)kSchedSlots : 0;  // dynamic schedule only
  // dynamic schedule's unit order: blocks of HB (batch, head) pairs at D=128
  // (their query pairs share K/V in L2: C3 forward -4.6 %), one block at D=64
  // (C4: blocks of 8-32 heads measured 1-2 % slower)
  static constexpr int HB = (DYN && HD == 128) ? 16 : 0;
  static constexpr uint32_t OFF_SCHED = OFF_ZT + ZT_BYTES;
  static constexpr uint32_t OFF_BAR = OFF_SCHED + NSCHED * 16;
  // q_full/empty[QST], k_full/empty[KST], v_full/empty[VST], per tile X:
  // s_full, s_free, p_full, pv_done, o_free, do_full; then never (nothing
  // arrives: the time-out test hook), fin (the UMMA issuer's wind-down) and
  // sched_full/empty[NSCHED]
  static constexpr int NBAR = 2 * QST + 2 * KST + 2 * VST + 2 * 6 + 2 + 2 * NSCHED;
  static constexpr uint32_t OFF_TSLOT = OFF_BAR + NBAR * 8;
  static constexpr uint32_t SMEM_BYTES = OFF_TSLOT + 16 + 1024;  // + alignment slack
  static constexpr uint32_t TCOL_S = 0;     // S_A, S_B at columns 0, 128
  static constexpr uint32_t TCOL_O = 256;   // O_A, O_B at 256, 256+HD
  static constexpr uint32_t TCOL_P = 256 + 2 * HD;  // P_A, P_B (D=64): 64 columns each
  static_assert(!P_TMEM || TCOL_P + 2 * (BN / 2) <= 512, "TMEM columns");
  static_assert(OFF_BAR + NBAR * 8 + 16 + 1024 <= 232448, "shared memory");
};

struct FwdParams {
  int T, NH, bh_begin, nbh, npairs, nqt;
  int nunits;
  float scale_log2;
  float* lse;
  uint32_t* status;
  // fused computeD (D = 64 only, both or neither set): D[row][h] =
  // bf16(sum_c O[row][h*64+c] * dO[row][h*64+c]) from the bf16-rounded O
  const __nv_bfloat16* dO;
  __nv_bfloat16* D;
  // optional (D=64): zeros are written to dQ's slab of every query tile the
  // kernel computes (by TMA stores, tensor map tmdQz), for a backward that
  // then accumulates into dQ
  float* dQz;
  uint32_t expire_ns;  // time-out test hook (ma_debug_expire_next_wait), 0 = off
};

// sum over 8 bf16 pairs of a[i] * b[i], fp32 (products of bf16 values are
// exact in fp32)
__device__ __forceinline__ float dot_bf16x8(uint4 a, uint4 b) {
  const __nv_bfloat162* x = reinterpret_cast<const __nv_bfloat162*>(&a);
  const __nv_bfloat162* y = reinterpret_cast<const __nv_bfloat162*>(&b);
  float s = 0.0f;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float2 fx = __bfloat1622float2(x[i]), fy = __bfloat1622float2(y[i]);
    s = fmaf(fx.x, fy.x, s);
    s = fmaf(fx.y, fy.y, s);
  }
  return s;
}

// Work units, heaviest first (causal work grows with the pair index):
// k -> (pair = npairs-1 - k / nbh, bh = bh_begin + k % nbh), dealt in one of
// two ways.  Static (up to 16 query tiles): one CTA per SM, units in rounds of
// G = gridDim.x in alternating direction (round g gives CTA c unit g*G + c
// for even g and g*G + G-1-c for odd g), which balances the decreasing unit
// sizes across CTAs.  Dynamic (longer sequences, whose units differ more in
// size): one CTA per unit; a running CTA takes its own unit (k = blockIdx.x)
// and then, by cluster launch control, the units of CTAs that have not
// started yet, in launch order, so units go greedily to whichever SM is free.
// With HB > 0 (the dynamic schedule at D=128) the order is blocked instead:
// block k / (HB*npairs) holds HB (batch, head) pairs (fewer in the last
// block), heaviest pair first within it, so the units in flight share their
// heads' K/V tiles in L2 and the grid still ends on light units.
struct Unit {
  int pair, b, h, nA, nB, nkv;
};

template <int HB>
__device__ __forceinline__ Unit decode_unit(const FwdParams& prm, int k) {
  Unit x;
  int bh;
  if constexpr (HB > 0) {  // blocks of HB (batch, head) pairs, heaviest pair first in each
    const int per = HB * prm.npairs;
    const int blk = k / per, r = k % per;
    const int hb = min(HB, prm.nbh - blk * HB);
    x.pair = prm.npairs - 1 - r / hb;
    bh = prm.bh_begin + blk * HB + r % hb;
  } else {
    x.pair = prm.npairs - 1 - k / prm.nbh;
    bh = prm.bh_begin + k % prm.nbh;
  }
  x.b = bh / prm.NH;
  x.h = bh % prm.NH;
  x.nA = 2 * x.pair + 1;                                   // key tiles 0..2p
  x.nB = (2 * x.pair + 1 < prm.nqt) ? 2 * x.pair + 2 : 0;  // tile B inside T?
  x.nkv = x.nB > 0 ? x.nB : x.nA;
  return x;
}

// Static schedule: the g-th unit of this CTA, or -1 when it has none left.
__device__ __forceinline__ int unit_of_round(const FwdParams& prm, int g) {
  const int G = gridDim.x;
  const long long k = (long long)g * G + ((g & 1) ? G - 1 - (int)blockIdx.x : (int)blockIdx.x);
  // past the end only in the last (partial) round: nothing follows it
  return k < prm.nunits ? (int)k : -1;
}

template <int HD, bool DYN>
__global__ void __launch_bounds__(NUM_THREADS, 1)
    flash_fwd_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                     const __grid_constant__ CUtensorMap tmV, const __grid_constant__ CUtensorMap tmO,
                     const __grid_constant__ CUtensorMap tmdO, const __grid_constant__ CUtensorMap tmdQz,
                     const FwdParams prm) {
  pdl_wait_and_release();
  using C = FwdCfg<HD, DYN>;
  extern __shared__ uint8_t smem_raw[];
  __shared__ int abort_flag;
  const uint32_t raw = smem_u32(smem_raw);
  const uint32_t sbase = (raw + 1023u) & ~1023u;
  uint8_t* gbase = smem_raw + (sbase - raw);
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;

  const uint32_t bar0 = sbase + C::OFF_BAR;
  auto BAR_QF = [&](int s) { return bar0 + 8u * s; };
  auto BAR_QE = [&](int s) { return bar0 + 8u * (C::QST + s); };
  auto BAR_KF = [&](int s) { return bar0 + 8u * (2 * C::QST + s); };
  auto BAR_KE = [&](int s) { return bar0 + 8u * (2 * C::QST + C::KST + s); };
  auto BAR_VF = [&](int s) { return bar0 + 8u * (2 * C::QST + 2 * C::KST + s); };
  auto BAR_VE = [&](int s) { return bar0 + 8u * (2 * C::QST + 2 * C::KST + C::VST + s); };
  const uint32_t barX = bar0 + 8u * (2 * C::QST + 2 * C::KST + 2 * C::VST);
  // per tile X in {0: A, 1: B}
  auto BAR_SF = [&](int x) { return barX + 8u * (0 * 2 + x); };
  auto BAR_SE = [&](int x) { return barX + 8u * (1 * 2 + x); };
  auto BAR_PF = [&](int x) { return barX + 8u * (2 * 2 + x); };
  auto BAR_PV = [&](int x) { return barX + 8u * (3 * 2 + x); };
  auto BAR_OE = [&](int x) { return barX + 8u * (4 * 2 + x); };
  auto BAR_DO = [&](int x) { return barX + 8u * (5 * 2 + x); };  // dO tile of X landed (fused computeD)
  const uint32_t BAR_NEVER = barX + 8u * 12;  // nothing arrives (time-out test hook)
  const uint32_t BAR_FIN = barX + 8u * 13;    // the UMMA issuer's last commit (wind-down)
  auto BAR_UF = [&](int s) { return barX + 8u * (14 + s); };              // response s landed
  auto BAR_UE = [&](int s) { return barX + 8u * (14 + C::NSCHED + s); };  // response s read by all
  // dynamic schedule: unit g >= 1 of this CTA is the one launch-control
  // response g-1 names (requested by the TMA producer when it starts unit
  // g-1); readers: the producer, the UMMA issuer and the 8 softmax warps
  constexpr uint32_t SCHED_READERS = 10;
  const uint32_t tslot = sbase + C::OFF_TSLOT;

  if (threadIdx.x == 0) {
    abort_flag = 0;
    for (int s = 0; s < C::QST; ++s) {
      mbar_init(BAR_QF(s), 1);
      mbar_init(BAR_QE(s), 1);
    }
    for (int s = 0; s < C::KST; ++s) {
      mbar_init(BAR_KF(s), 1);
      mbar_init(BAR_KE(s), 1);
    }
    for (int s = 0; s < C::VST; ++s) {
      mbar_init(BAR_VF(s), 1);
      mbar_init(BAR_VE(s), 1);
    }
    for (int x = 0; x < 2; ++x) {
      mbar_init(BAR_SF(x), 1);
      mbar_init(BAR_SE(x), 128);
      mbar_init(BAR_PF(x), 128);
      mbar_init(BAR_PV(x), 1);
      mbar_init(BAR_OE(x), 128);
      mbar_init(BAR_DO(x), 1);
    }
    mbar_init(BAR_NEVER, 1);
    mbar_init(BAR_FIN, 1);
    for (int u = 0; u < C::NSCHED; ++u) {
      mbar_init(BAR_UF(u), 1);
      mbar_init(BAR_UE(u), SCHED_READERS);
    }
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc(tslot, 512);
    tmem_relinquish();
  }
  if (C::ZT_BYTES && prm.dQz) {  // the zero tile the dQ stores copy from
    for (uint32_t i = threadIdx.x; i < C::ZT_BYTES / 16; i += NUM_THREADS)
      reinterpret_cast<uint4*>(gbase + C::OFF_ZT)[i] = make_uint4(0u, 0u, 0u, 0u);
    fence_proxy_async_smem();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *reinterpret_cast<volatile uint32_t*>(gbase + C::OFF_TSLOT);
  volatile int* abort_p = &abort_flag;
  const Sched sch{sbase + C::OFF_SCHED, BAR_UF(0), BAR_UE(0), abort_p};

  if (warp < 4) {
    reg_dealloc<REGS_PRODUCER>();
    if (warp == 0 && lane == 0) {
      // ---------------------------------------------------- TMA producer
      tma_prefetch_desc(&tmQ);
      tma_prefetch_desc(&tmK);
      tma_prefetch_desc(&tmV);
      uint32_t qc = 0, kc = 0, vc = 0;
      uint32_t nreq = 0;  // launch-control requests issued (request r names unit r+1)
      bool ok = true;
      for (int g = 0; ok; ++g) {
        int k;
        if constexpr (DYN) k = sched_unit<false>(sch, g);
        else k = unit_of_round(prm, g);
        if (k < 0) break;
        // dynamic: request unit g+1 now, a unit ahead of every reader
        if constexpr (DYN) {
          if (!sched_request(sch, nreq)) break;
          ++nreq;
        }
        const Unit un = decode_unit<C::HB>(prm, k);
        const int col0 = un.h * HD;
        const int qs = qc % C::QST;
        if (qc >= C::QST && !mbar_wait(BAR_QE(qs), ((qc / C::QST) - 1) & 1, abort_p)) break;
        const int ntile = un.nB > 0 ? 2 : 1;
        mbar_arrive_expect_tx(BAR_QF(qs), ntile * C::QT_BYTES);
        for (int x = 0; x < ntile; ++x)
          for (int kb = 0; kb < C::KB; ++kb)
            tma_load_3d(sbase + C::OFF_Q + (qs * 2 + x) * C::QT_BYTES + kb * BM * 128, &tmQ,
                        BAR_QF(qs), col0 + kb * 64, (2 * un.pair + x) * BM, un.b);
        ++qc;
        for (int j = 0; j < un.nkv; ++j) {
          const int ks = kc % C::KST;
          if (kc >= C::KST && !mbar_wait(BAR_KE(ks), ((kc / C::KST) - 1) & 1, abort_p)) { ok = false; break; }
          mbar_arrive_expect_tx(BAR_KF(ks), C::KV_BYTES);
          for (int kb = 0; kb < C::KB; ++kb)
            tma_load_3d(sbase + C::OFF_K + ks * C::KV_BYTES + kb * BN * 128, &tmK, BAR_KF(ks),
                        col0 + kb * 64, j * BN, un.b);
          ++kc;
          const int vs = vc % C::VST;
          if (vc >= C::VST && !mbar_wait(BAR_VE(vs), ((vc / C::VST) - 1) & 1, abort_p)) { ok = false; break; }
          mbar_arrive_expect_tx(BAR_VF(vs), C::KV_BYTES);
          for (int kb = 0; kb < C::KB; ++kb)
            tma_load_3d(sbase + C::OFF_V + vs * C::KV_BYTES + kb * BN * 128, &tmV, BAR_VF(vs),
                        col0 + kb * 64, j * BN, un.b);
          ++vc;
        }
      }
      if (*abort_p) {  // wind-down: let the loads and the request still in flight land
        if (DYN) sched_drain(sch, nreq);
        drain_ring(BAR_QF, C::QST, qc);
        drain_ring(BAR_KF, C::KST, kc);
        drain_ring(BAR_VF, C::VST, vc);
      }
    } else if (warp == 1 && lane == 0) {
      // ----------------------------------------------------------- MMA
      constexpr uint32_t IDESC_S = idesc_bf16_f32(BM, BN, 0, 0);
      constexpr uint32_t IDESC_O = idesc_bf16_f32(BM, HD, 0, 1);
      uint32_t qc = 0, kc = 0, vc = 0;
      uint32_t sc[2] = {0, 0};   // S_X issued so far
      uint32_t pvc[2] = {0, 0};  // PV_X issued so far
      uint32_t uc[2] = {0, 0};   // units in which tile X was active
      bool ok = true;
      for (int g = 0; ok; ++g) {
        int k;
        if constexpr (DYN) k = sched_unit<false>(sch, g);
        else k = unit_of_round(prm, g);
        if (k < 0) break;
        const Unit un = decode_unit<C::HB>(prm, k);
        const int n[2] = {un.nA, un.nB};
        const int qs = qc % C::QST;
        if (!mbar_wait(BAR_QF(qs), (qc / C::QST) & 1, abort_p)) break;
        // S_X(j) = Q_X K_j^T
        auto issue_s = [&](int x, int j) -> bool {
          if (sc[x] >= 1 && !mbar_wait(BAR_SE(x), (sc[x] - 1) & 1, abort_p)) return false;
          tc_fence_after();
          const uint32_t sq = sbase + C::OFF_Q + (qs * 2 + x) * C::QT_BYTES;
          const uint32_t sk = sbase + C::OFF_K + ((kc + j) % C::KST) * C::KV_BYTES;
#pragma unroll
          for (int kk = 0; kk < HD / 16; ++kk) {
            const uint32_t off = (kk >> 2) * (BM * 128) + (kk & 3) * 32;
            umma_bf16_ss(tmem + C::TCOL_S + x * BN, smem_desc_sw128(sq + off, 16, 1024),
                         smem_desc_sw128(sk + off, 16, 1024), IDESC_S, kk > 0 ? 1u : 0u);
          }
          umma_commit(BAR_SF(x));
          ++sc[x];
          return true;
        };
        // O_X += P_X V_j
        auto issue_pv = [&](int x, int j) -> bool {
          if (!mbar_wait(BAR_PF(x), pvc[x] & 1, abort_p)) return false;
          if (j == 0 && uc[x] >= 1 && !mbar_wait(BAR_OE(x), (uc[x] - 1) & 1, abort_p)) return false;
          tc_fence_after();
          const uint32_t sp = sbase + C::OFF_P + x * C::STG_BYTES;
          const uint32_t sv = sbase + C::OFF_V + ((vc + j) % C::VST) * C::KV_BYTES;
#pragma unroll
          for (int kk = 0; kk < BN / 16; ++kk) {
            const uint64_t bd = smem_desc_sw128(sv + kk * 2048, BN * 128, 1024);
            if (C::P_TMEM) {  // A = P_X from TMEM: 8 columns per 16 keys
              umma_bf16_ts(tmem + C::TCOL_O + x * HD, tmem + C::TCOL_P + x * (BN / 2) + kk * 8, bd,
                           IDESC_O, (j > 0 || kk > 0) ? 1u : 0u);
            } else {
              const uint64_t ad = smem_desc_sw128(sp + (kk >> 2) * (BM * 128) + (kk & 3) * 32, 16, 1024);
              umma_bf16_ss(tmem + C::TCOL_O + x * HD, ad, bd, IDESC_O, (j > 0 || kk > 0) ? 1u : 0u);
            }
          }
          umma_commit(BAR_PV(x));
          ++pvc[x];
          return true;
        };
        auto wait_k = [&](int j) {
          const uint32_t k = kc + j;
          return mbar_wait(BAR_KF(k % C::KST), (k / C::KST) & 1, abort_p);
        };
        auto wait_v = [&](int j) {
          const uint32_t v = vc + j;
          return mbar_wait(BAR_VF(v % C::VST), (v / C::VST) & 1, abort_p);
        };
        // prologue: S_A(0), S_B(0); K_0 is consumed once both are done
        ok = wait_k(0) && issue_s(0, 0) && (n[1] == 0 || issue_s(1, 0));
        if (ok) umma_commit(BAR_KE(kc % C::KST));
        // time-out test hook: with the first products in flight, wait on a
        // barrier nothing arrives at until the hook's limit runs out
        if (ok && g == 0 && prm.expire_ns) ok = mbar_wait(BAR_NEVER, 0, abort_p, prm.expire_ns);
        for (int j = 0; ok && j < un.nkv; ++j) {
          if (C::EARLY_S) {
            // S_X(j+1) as soon as softmax X has read S_X(j) (issue_s waits for
            // that), so the next scores are ready before this tile's softmax ends
            if (j + 1 < un.nkv) {
              if (!wait_k(j + 1)) { ok = false; break; }
              if (j + 1 < n[0] && !issue_s(0, j + 1)) { ok = false; break; }
              if (j + 1 < n[1] && !issue_s(1, j + 1)) { ok = false; break; }
              umma_commit(BAR_KE((kc + j + 1) % C::KST));  // K_{j+1} consumed
            }
            if (!wait_v(j)) { ok = false; break; }
            if (j < n[0] && !issue_pv(0, j)) { ok = false; break; }
            if (j < n[1] && !issue_pv(1, j)) { ok = false; break; }
          } else {
            // PV_A(j) S_A(j+1) | PV_B(j) S_B(j+1)
            if (!wait_v(j)) { ok = false; break; }
            const bool lastA = (j + 1 >= n[0]);
            if (j < n[0]) {
              if (!issue_pv(0, j)) { ok = false; break; }
              if (!lastA && (!wait_k(j + 1) || !issue_s(0, j + 1))) { ok = false; break; }
            }
            if (j < n[1]) {
              if (!issue_pv(1, j)) { ok = false; break; }
              if (j + 1 < n[1] && ((lastA && !wait_k(j + 1)) || !issue_s(1, j + 1))) { ok = false; break; }
            }
            if (j + 1 < un.nkv) umma_commit(BAR_KE((kc + j + 1) % C::KST));  // K_{j+1} consumed
          }
          umma_commit(BAR_VE((vc + j) % C::VST));           // V_j consumed
          if (j + 1 == un.nkv) umma_commit(BAR_QE(qs));     // every S of the unit issued
        }
        kc += un.nkv;
        vc += un.nkv;
        ++qc;
        for (int x = 0; x < 2; ++x)
          if (n[x] > 0) ++uc[x];
      }
      if (*abort_p) {  // wind-down: every UMMA issued must complete before TMEM is freed
        umma_commit(BAR_FIN);
        mbar_wait_for(BAR_FIN, 0, kDrainLimitNs);
      }
    }
  } else {
    reg_alloc<REGS_SOFTMAX>();
    // --------------------------------------------------------- softmax
    const int x = (warp - 4) >> 2;               // 0: tile A (warps 4-7), 1: tile B (8-11)
    const uint32_t wg_bar = 1 + x;               // named barrier of this warpgroup
    const int quarter = warp & 3;                // TMEM lane quarter of this warp
    const int row = quarter * 32 + lane;         // query row within the tile
    const uint32_t trow = tmem + ((uint32_t)(quarter * 32) << 16);
    const uint32_t tcol_s = C::TCOL_S + x * BN, tcol_o = C::TCOL_O + x * HD;
    const float c = prm.scale_log2;
    const bool wg_leader = (warp == 4 + 4 * x) && lane == 0;
    uint8_t* pbuf = gbase + C::OFF_P + x * C::STG_BYTES;
    uint32_t sc = 0;  // S_X consumed so far (== P_X produced)
    uint32_t nd = 0;  // dO tiles of X consumed so far (fused computeD)
    uint32_t nd_armed = 0;  // dO tile loads issued (leader)
    bool ok = true;
    for (int g = 0; ok; ++g) {
      int k;
      if constexpr (DYN) k = sched_unit<true>(sch, g);
      else k = unit_of_round(prm, g);
      if (k < 0) break;
      const Unit un = decode_unit<C::HB>(prm, k);
      const int nt = x == 0 ? un.nA : un.nB;
      if (nt == 0) continue;
      const int qtile = 2 * un.pair + x;
      if (C::ZT_BYTES && prm.dQz && wg_leader) {
        // this query tile's dQ slab (128 rows x HD fp32; rows past T are
        // clipped) from the zero tile, by TMA stores that need no waiting for
        for (int box = 0; box < HD / 32; ++box)
          tma_store_3d(&tmdQz, sbase + C::OFF_ZT, un.h * HD + box * 32, qtile * BM, un.b);
        bulk_commit();
      }
      // the previous unit's O store must have read the staging before it is
      // written again: at D=128 it holds P from this unit's first tile on, so
      // wait here; at D=64 (P in TMEM) it is next written by this unit's dO
      // load or epilogue, which wait there instead, so this unit's first
      // tiles overlap the store
      if constexpr (!C::P_TMEM) {
        if (sc >= 1 && wg_leader) bulk_wait_read<0>();
        bar_sync_named(wg_bar, 128);
      }
      float m_used = -INFINITY, l_sum = 0.0f;
      // one key tile; DIAG: the diagonal tile (keys after the query masked).
      // Instantiated twice so that the other tiles carry no masking code.
      auto tile = [&](auto diag_tag, int j) -> bool {
        constexpr bool DIAG = decltype(diag_tag)::value;
        if constexpr (DIAG && C::P_TMEM) {
          // the unit's last key tile: the dO tile of X goes by TMA into the O
          // staging (idle until the epilogue; rows past T read as zero); the
          // epilogue reads each chunk back before writing O over it
          if (prm.dO && wg_leader) {
            bulk_wait_read<0>();  // the previous unit's O store has read the staging
            mbar_arrive_expect_tx(BAR_DO(x), BM * HD * 2);
            ++nd_armed;
            for (int kb = 0; kb < C::KB; ++kb)
              tma_load_3d(smem_u32(pbuf) + kb * BM * 128, &tmdO, BAR_DO(x), un.h * HD + kb * 64, qtile * BM,
                          un.b);
          }
        }
        if (!mbar_wait_warp(BAR_SF(x), sc & 1, abort_p)) return false;
        tc_fence_after();
        float s[BN];
#pragma unroll
        for (int cc = 0; cc < BN; cc += 64) {
          uint32_t ra[32], rb[32];
          tmem_ld32(trow + tcol_s + cc, ra);
          tmem_ld32(trow + tcol_s + cc + 32, rb);
          tmem_wait_ld_dep(ra, rb);
#pragma unroll
          for (int i = 0; i < 32; ++i) {
            s[cc + i] = __uint_as_float(ra[i]);
            s[cc + 32 + i] = __uint_as_float(rb[i]);
          }
        }
        tc_fence_before();
        mbar_arrive(BAR_SE(x));
        if constexpr (DIAG) {
#pragma unroll
          for (int i = 0; i < BN; ++i)
            if (i > row) s[i] = -INFINITY;
        }
        // row maximum: 8 independent partial maxima, 3-input max (short chains)
        float pm[8];
#pragma unroll
        for (int q = 0; q < 8; ++q) pm[q] = fmaxf(s[q], s[8 + q]);
#pragma unroll
        for (int i = 16; i < BN; i += 16)
#pragma unroll
          for (int q = 0; q < 8; ++q) pm[q] = fmax3(pm[q], s[i + q], s[i + 8 + q]);
        const float mx = fmax3(fmax3(pm[0], pm[1], pm[2]), fmax3(pm[3], pm[4], pm[5]),
                               fmaxf(pm[6], pm[7]));
        const float m_new = fmaxf(m_used, mx * c);
        // lazy rescaling: only rows whose maximum grew by more than 2^8 move
        // m_used; O_X is rescaled below, once PV_X(j-1) has completed
        bool rescale = false;
        float alpha = 1.0f;
        if (j == 0) {
          m_used = m_new;
        } else {
          const bool need = m_new > m_used + RESCALE_THRESHOLD;
          rescale = __any_sync(0xffffffffu, need);
          if (need) {
            alpha = ex2(m_used - m_new);
            l_sum *= alpha;
            m_used = m_new;
          }
        }
        // P = 2^(S*c - m) with packed fp32x2 FMAs; row sum in 4 packed partials
        const float2 c2 = make_float2(c, c), nm2 = make_float2(-m_used, -m_used);
        float2 ps[4] = {make_float2(0.f, 0.f), make_float2(0.f, 0.f), make_float2(0.f, 0.f),
                        make_float2(0.f, 0.f)};
        uint32_t pk[BN / 2];  // P as bf16 pairs, even key in the low half
#pragma unroll
        for (int i = 0; i < BN; i += 2) {
          const float2 t = __ffma2_rn(make_float2(s[i], s[i + 1]), c2, nm2);
          const float e0 = ex2(t.x), e1 = ex2(t.y);
          ps[(i >> 1) & 3] = __fadd2_rn(ps[(i >> 1) & 3], make_float2(e0, e1));
          pk[i / 2] = pack_bf16(e0, e1);
        }
        l_sum += (ps[0].x + ps[0].y) + (ps[1].x + ps[1].y) + (ps[2].x + ps[2].y) +
                 (ps[3].x + ps[3].y);
        // PV_X(j-1) must be complete before O_X is rescaled and before P_X(j)
        // overwrites P_X (waited for only now, so the exponentials overlap it)
        if (j >= 1) {
          if (!mbar_wait_warp(BAR_PV(x), (sc - 1) & 1, abort_p)) return false;
          tc_fence_after();
        }
        if (rescale) {
#pragma unroll
          for (int cc = 0; cc < HD; cc += 16) {
            uint32_t r[16];
            tmem_ld16(trow + tcol_o + cc, r);
            tmem_wait_ld_dep(r);
#pragma unroll
            for (int i = 0; i < 16; ++i) r[i] = __float_as_uint(__uint_as_float(r[i]) * alpha);
            tmem_st16(trow + tcol_o + cc, r);
          }
          tmem_wait_st();
        }
        if constexpr (C::P_TMEM) {
          // this lane's P row into P_X
#pragma unroll
          for (int q = 0; q < BN / 32; ++q) {
            uint32_t r[16];
#pragma unroll
            for (int i = 0; i < 16; ++i) r[i] = pk[q * 16 + i];
            tmem_st16(trow + C::TCOL_P + x * (BN / 2) + q * 16, r);
          }
          tmem_wait_st();
        } else {
#pragma unroll
          for (int kb = 0; kb < BN / 64; ++kb) {
#pragma unroll
            for (int ch = 0; ch < 8; ++ch) {
              const int c0 = (kb * 64 + ch * 8) / 2;
              const uint4 v = make_uint4(pk[c0], pk[c0 + 1], pk[c0 + 2], pk[c0 + 3]);
              *reinterpret_cast<uint4*>(pbuf + kb * (BM * 128) + row * 128 + ((ch ^ (row & 7)) * 16)) = v;
            }
          }
          fence_proxy_async_smem();
        }
        tc_fence_before();
        mbar_arrive(BAR_PF(x));
        ++sc;
        return true;
      };
      for (int j = 0; ok && j < nt; ++j)
        ok = (j == qtile) ? tile(std::true_type{}, j) : tile(std::false_type{}, j);
      // --------------------------------------------- epilogue of tile X
      const bool epi = ok && mbar_wait_warp(BAR_PV(x), (sc - 1) & 1, abort_p);
      if constexpr (C::P_TMEM) {
        // without dO the epilogue is the staging's first writer in this unit
        // (with dO the warpgroup waits for the dO load, issued after the wait)
        if (!prm.dO) {
          if (wg_leader) bulk_wait_read<0>();
          bar_sync_named(wg_bar, 128);
        }
      }
      if (epi) {
        tc_fence_after();
        const float inv = 1.0f / l_sum;
        const int grow = qtile * BM + row;
        const bool fuse_d = C::P_TMEM && prm.dO;
        bool dok = true;
        if (fuse_d) dok = mbar_wait_warp(BAR_DO(x), nd & 1, abort_p);
        float dsum = 0.0f;
        // stage O (bf16) in this tile's P buffer (free: its last PV is done);
        // O is read from TMEM 64 columns (two loads, one wait) at a time
#pragma unroll
        for (int c64 = 0; c64 < HD; c64 += 64) {
          uint32_t ra[32], rb[32];
          tmem_ld32(trow + tcol_o + c64, ra);
          tmem_ld32(trow + tcol_o + c64 + 32, rb);
          tmem_wait_ld_dep(ra, rb);
#pragma unroll
          for (int c16 = 0; c16 < 64; c16 += 16) {
            const uint32_t* r = c16 < 32 ? ra + c16 : rb + (c16 - 32);
            const int cc = c64 + c16;
            uint4 v0, v1;
            v0.x = pack_bf16(__uint_as_float(r[0]) * inv, __uint_as_float(r[1]) * inv);
            v0.y = pack_bf16(__uint_as_float(r[2]) * inv, __uint_as_float(r[3]) * inv);
            v0.z = pack_bf16(__uint_as_float(r[4]) * inv, __uint_as_float(r[5]) * inv);
            v0.w = pack_bf16(__uint_as_float(r[6]) * inv, __uint_as_float(r[7]) * inv);
            v1.x = pack_bf16(__uint_as_float(r[8]) * inv, __uint_as_float(r[9]) * inv);
            v1.y = pack_bf16(__uint_as_float(r[10]) * inv, __uint_as_float(r[11]) * inv);
            v1.z = pack_bf16(__uint_as_float(r[12]) * inv, __uint_as_float(r[13]) * inv);
            v1.w = pack_bf16(__uint_as_float(r[14]) * inv, __uint_as_float(r[15]) * inv);
            const int kb = cc / 64, ch = (cc % 64) / 8;
            uint8_t* blk = pbuf + kb * (BM * 128) + row * 128;
            uint4* p0 = reinterpret_cast<uint4*>(blk + ((ch ^ (row & 7)) * 16));
            uint4* p1 = reinterpret_cast<uint4*>(blk + (((ch + 1) ^ (row & 7)) * 16));
            if (fuse_d) dsum += dot_bf16x8(v0, *p0) + dot_bf16x8(v1, *p1);  // dO, then O over it
            *p0 = v0;
            *p1 = v1;
          }
        }
        tc_fence_before();
        mbar_arrive(BAR_OE(x));  // O_X may be overwritten by the next unit
        fence_proxy_async_smem();
        if (grow < prm.T) {
          const long long ri = ((long long)un.b * prm.T + grow) * prm.NH + un.h;
          prm.lse[ri] = (m_used + log2f(l_sum)) * LN2;
          if (fuse_d && dok) prm.D[ri] = __float2bfloat16_rn(dsum);
        }
        if (fuse_d) ++nd;
      }
      // every thread of the warpgroup takes this barrier and leaves it with the
      // same verdict, so the warpgroup stays in step after a failed wait
      ok = bar_red_and(wg_bar, 128, epi);
      if (ok && wg_leader) {
        for (int kb = 0; kb < C::KB; ++kb)
          tma_store_3d(&tmO, sbase + C::OFF_P + x * C::STG_BYTES + kb * BM * 128, un.h * HD + kb * 64,
                       qtile * BM, un.b);
        bulk_commit();
      }
    }
    if (wg_leader) {
      bulk_wait<0>();
      // wind-down: a dO tile load whose epilogue never ran must land first
      if (*abort_p && nd_armed > 0) mbar_wait_for(BAR_DO(x), (nd_armed - 1) & 1, kDrainLimitNs);
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
  if (threadIdx.x == 0 && abort_flag) atomicOr(prm.status, STATUS_FWD_TIMEOUT);
}

// Launches the instantiation DYN (dynamic schedule: one CTA per unit, else
// one per SM).
template <int HD, bool DYN>
cudaError_t launch_fwd_kernel(const CUtensorMap& tq, const CUtensorMap& tk, const CUtensorMap& tv,
                              const CUtensorMap& to, const CUtensorMap& tdo, const CUtensorMap& tdqz,
                              const FwdParams& prm, cudaStream_t st) {
  using C = FwdCfg<HD, DYN>;
  // The setmaxnreg split assumes the kernel was compiled to exactly
  // LAUNCH_REGS registers per thread; refuse to launch otherwise.
  static const cudaError_t reg_check = [] {
    cudaFuncAttributes a;
    cudaError_t e = cudaFuncGetAttributes(&a, flash_fwd_kernel<HD, DYN>);
    if (e != cudaSuccess) return e;
    return a.numRegs == LAUNCH_REGS ? cudaSuccess : cudaErrorInvalidKernelImage;
  }();
  if (reg_check != cudaSuccess) return reg_check;
  cudaError_t e = cudaFuncSetAttribute(flash_fwd_kernel<HD, DYN>,
                                       cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM_BYTES);
  if (e != cudaSuccess) return e;
  int grid = prm.nunits;  // dynamic: one CTA per unit (see decode_unit)
  if (!DYN) {
    int dev = 0, sms = 148;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    grid = prm.nunits < sms ? prm.nunits : sms;
  }
  launch_pdl(flash_fwd_kernel<HD, DYN>, grid, NUM_THREADS, C::SMEM_BYTES, st, tq, tk, tv, to, tdo, tdqz, prm);
  count_launches(1);
  return cudaGetLastError();
}

template <int HD>
cudaError_t launch_fwd(const __nv_bfloat16* q, const __nv_bfloat16* k, const __nv_bfloat16* v,
                       __nv_bfloat16* out, float* lse, const AttnShape& s, uint32_t* status,
                       cudaStream_t st, const __nv_bfloat16* dO, __nv_bfloat16* Dv, float* dQz) {
  using C = FwdCfg<HD>;
  CUtensorMap tq, tk, tv, to, tdo, tdqz;
  const CUtensorMapDataType bf = CU_TENSOR_MAP_DATA_TYPE_BFLOAT16;
  const CUtensorMapSwizzle sw = CU_TENSOR_MAP_SWIZZLE_128B;
  if (!make_tmap_3d(&tq, q, bf, 2, s.N, s.T, s.B, 64, BM, sw) ||
      !make_tmap_3d(&tk, k, bf, 2, s.N, s.T, s.B, 64, BN, sw) ||
      !make_tmap_3d(&tv, v, bf, 2, s.N, s.T, s.B, 64, BN, sw) ||
      !make_tmap_3d(&to, out, bf, 2, s.N, s.T, s.B, 64, BM, sw))
    return cudaErrorInvalidValue;
  if (dO) {
    if (!make_tmap_3d(&tdo, dO, bf, 2, s.N, s.T, s.B, 64, BM, sw)) return cudaErrorInvalidValue;
  } else {
    tdo = tq;  // not read without dO
  }
  if (dQz && C::ZT_BYTES) {
    if (!make_tmap_3d(&tdqz, dQz, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, s.N, s.T, s.B, 32, BM,
                      CU_TENSOR_MAP_SWIZZLE_128B))
      return cudaErrorInvalidValue;
  } else {
    tdqz = tq;  // not written without dQz
  }
  FwdParams prm;
  prm.T = s.T;
  prm.NH = s.NH;
  prm.bh_begin = s.bh_begin;
  prm.nbh = s.bh_end - s.bh_begin;
  prm.nqt = (s.T + BM - 1) / BM;
  prm.npairs = (prm.nqt + 1) / 2;
  prm.nunits = prm.npairs * prm.nbh;
  prm.scale_log2 = LOG2E / sqrtf((float)HD);
  prm.lse = lse;
  prm.status = status;
  prm.dO = dO;
  prm.D = Dv;
  prm.dQz = C::ZT_BYTES ? dQz : nullptr;
  prm.expire_ns = take_expire_request(STATUS_FWD_TIMEOUT);
  // static rounds up to 16 query tiles, the dynamic schedule beyond
  if (prm.nqt > 16) return launch_fwd_kernel<HD, true>(tq, tk, tv, to, tdo, tdqz, prm, st);
  return launch_fwd_kernel<HD, false>(tq, tk, tv, to, tdo, tdqz, prm, st);
}

}  // namespace

cudaError_t launch_flash_fwd(const __nv_bfloat16* q, const __nv_bfloat16* k,
                             const __nv_bfloat16* v, __nv_bfloat16* out, float* lse,
                             const AttnShape& s, uint32_t* status, cudaStream_t st,
                             const __nv_bfloat16* dO, __nv_bfloat16* Dv, float* dQz) {
  if (s.bh_end <= s.bh_begin) return cudaSuccess;
  if ((dO == nullptr) != (Dv == nullptr) || (dO && s.D != 64)) return cudaErrorInvalidValue;
  if (s.D == 64) return launch_fwd<64>(q, k, v, out, lse, s, status, st, dO, Dv, dQz);
  // D=128: no shared memory left for the zero tile; dQ is zeroed by the
  // separate pass, before the forward
  if (dQz) {
    const cudaError_t e = launch_zero_dq(dQz, s, st);
    if (e != cudaSuccess) return e;
  }
  return launch_fwd<128>(q, k, v, out, lse, s, status, st, nullptr, nullptr, nullptr);
}

}  // namespace ma
