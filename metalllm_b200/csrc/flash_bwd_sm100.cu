// flash_bwd_sm100.cu -- flashAttentionBackward (attention.metal:198-299) on
// sm_100a with tcgen05 UMMA, TMEM accumulators and TMA.
//
// Work unit, as in the reference (attention.metal:219-223): one 128-key tile
// of one (batch, head), walking the query tiles i from the diagonal to the end
// (causal: earlier queries never see these keys).  Per query tile (128
// queries):
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
// and P^T goes to shared memory like dS^T.  dK/dV are owned by the unit and
// stored once (bf16, straight from registers to global memory); dQ is
// accumulated in fp32 by the bulk reductions of every key tile into zeros:
// the launcher writes them first, unless the caller passes a dQ that already
// holds them (the accumulating entry point; the reference's host zeroes dQ,
// model.h:549).
//
// Scheduling: units are ordered in blocks of HB (batch, head) pairs, within
// a block by key tile (heaviest first), then head; HB = 1 is (batch,
// head)-major.  Short sequences at D=64 (PERSIST): one CTA per SM, HB = 1,
// units dealt in rounds of gridDim.x in alternating direction (CTA c takes
// position c in even rounds and gridDim.x-1-c in odd ones), so the units of
// a head start together and walk different query tiles, and the units in
// flight share a few heads' Q/dO in L2.  Longer sequences, whose units differ
// more in size: one CTA per unit; a running CTA takes its own unit and then,
// by cluster launch control, the units of CTAs that have not started yet, in
// launch order, so units go greedily to whichever SM is free.  Either way a
// unit's dK/dV epilogue runs after the next unit's first step has been handed
// to the tensor core.  At D=64 K/V are double-buffered, so the next unit's
// K/V, Q/dO tiles and first S^T/dP^T are fetched and computed while the
// current unit finishes; at D=128 (one K/V buffer) the next unit's K/V load
// and first S^T/dP^T wait for the current unit's last products.  (PERSIST,
// the template argument, selects the static schedule.)
//
// Roles (384 threads, three warpgroups):
//   warpgroup 0 (120 registers per thread after setmaxnreg):
//     warp 0   TMA producer: K/V per unit, Q_i/dO_i into a STAGES-deep ring
//     warp 1   TMEM owner; lane 0 issues every UMMA and commit
//     warp 2   statistics: -l_i*log2(e) and -D_i/sqrt(D) per query (strided
//              in global memory), loaded into registers a step ahead and
//              staged in shared memory for the compute warps
//     warp 3   lane 0 issues the dQ bulk reductions
//   warpgroups 1, 2 (192 registers): compute, thread = key row = TMEM lane;
//              warpgroup 1 takes query columns 0-63, warpgroup 2 columns
//              64-127; the dK/dV epilogue (each thread stores its key row's
//              slice of its part's columns) and, at D=128, the dQ drain into
//              the staging buffer.
// At D=64 a fourth warpgroup (warps 12-15, 64 registers) drains dQ, and the
// CTA has 512 threads (warpgroup 0 80 registers, compute 184).
// D=64 schedule ("early S"): S^T/dP^T of the next query tile are issued as
// soon as the compute warps have read the current one, so they run on the
// tensor core while the compute warps form P^T/dS^T; dV, dK and dQ follow, and
// dQ of a tile is drained after the next tile is handed over.  D=128 has no
// TMEM room for that (S^T, dP^T, dV, dK fill all 512 columns; dQ reuses the
// S^T columns) and runs the steps in order, draining dQ before the next S^T.
//
// Conventions as the reference: P = exp(S/sqrt(D) - l) with l read as stored,
// D read as stored (bf16), dS includes 1/sqrt(D).  The reference rounds S,
// dP, P, dS and the dQ tile to bf16 and accumulates dK/dV in bf16 memory;
// here S, dP, dQ and dK/dV stay fp32 until their single store, and P, dS are
// bf16 (the UMMA operand type).
//
// All mbarrier waits are bounded (about 2 s); on time-out the CTA winds down,
// frees its TMEM and sets STATUS_BWD_TIMEOUT.  Warps meet only at mbarriers
// (no named barriers), so a failed wait cannot leave a warp stuck at one.
#include "common.cuh"
#include "sm100.cuh"
#include "tmap.h"

namespace ma {
namespace {

using namespace sm100;

constexpr int BK = 128;  // keys per unit
constexpr int BQ = 128;  // queries per step
constexpr int PERSIST_MAX_NKT = 16;  // static schedule when T/128 <= this (D=64)
constexpr float LOG2E = 1.4426950408889634f;


template <int HD, bool PERSIST>
struct BwdCfg {
  static constexpr int KB = HD / 64;
  static constexpr bool D64 = HD == 64;
  // Compute warpgroups: each takes BQ / NPART query columns of every step.
  // D=64 with NPART=2: a fourth warpgroup drains dQ (register split per
  // thread after setmaxnreg: warpgroup 0 80, compute 184, drain 64).
  // Otherwise the compute warpgroups also drain dQ, each its share of the
  // columns: D=64 with NPART=4 (640 threads; 64 / 104; measured slower and
  // not used), D=128 (384 threads; 120 / 192).
  static constexpr int NPART = 2;
  static constexpr int CPP = BQ / NPART;       // query columns per part
  static constexpr int NCOMP = 128 * NPART;    // compute threads
  static constexpr bool DRAIN_WG = D64 && NPART == 2;
  static constexpr int NUM_THREADS = 128 + NCOMP + (DRAIN_WG ? 128 : 0);
  static constexpr int LAUNCH_REGS = (65536 / NUM_THREADS) & ~7;  // registers per thread at launch
  static constexpr int REGS_PRODUCER = NPART == 4 ? 64 : (DRAIN_WG ? 80 : 120);
  static constexpr int REGS_DRAIN = DRAIN_WG ? 64 : 0;
  static constexpr int REGS_COMPUTE =
      ((NUM_THREADS * LAUNCH_REGS - 128 * REGS_PRODUCER - 128 * REGS_DRAIN) / NCOMP) & ~7;
  static constexpr int NDRAIN = DRAIN_WG ? 128 : NCOMP;  // arrivals on DQE, DSF
  // The unit's dK/dV epilogue (TMEM -> bf16 -> global memory) is run by the
  // compute warps, each part its columns, once they have handed the next
  // unit's first step to the tensor core: they would otherwise wait there for
  // the step's products, and with all of them the accumulators are released
  // sooner than by the drain warpgroup alone.
  static constexpr bool EPI_COMPUTE = true;
  static_assert(EPI_COMPUTE, "the drain warpgroup drains dQ only");
  static constexpr int NACC = EPI_COMPUTE ? NCOMP : NDRAIN;  // arrivals on ACC
  static_assert(128 * REGS_PRODUCER + NCOMP * REGS_COMPUTE + 128 * REGS_DRAIN <=
                    NUM_THREADS * LAUNCH_REGS,
                "register split must fit the launch allocation");
  static_assert(CPP % 16 == 0 && (HD / NPART) % 16 == 0, "column split");
  // Q_i/dO_i stages and K/V buffers: at D=64 K/V are double-buffered to
  // prefetch the next unit (under launch control too, where a CTA also runs
  // many units: C4 backward 3.75 -> 3.64 ms against one K/V buffer and three
  // Q/dO stages); D=128 has room for one of each
  static constexpr int STAGES = D64 ? 2 : 1;
  static constexpr int KVB = D64 ? 2 : 1;
  static constexpr bool P_IN_TMEM = D64;         // P^T in TMEM (else smem)
  static constexpr bool EARLY_S = D64;           // next S^T before dV/dK/dQ
  static constexpr bool DQ_ALIAS = !D64;         // dQ accumulator reuses the S^T columns
  static constexpr bool DQS_ALIAS = !D64;        // dQ staging reuses the P^T/dS^T smem
  // dQ staging buffers (the code allows more than one; a second buffer was
  // measured slower: the extra shared-memory traffic in flight slows the
  // tensor core's operand reads more than the overlap gains).  Statistics
  // ring stages: the statistics warp loads a step's values into registers a
  // step ahead, so one stage suffices where the shared memory is tight.
  static constexpr int DQSB = 1;
  static constexpr int SSTG = (D64 && PERSIST) ? 1 : 8;
  static constexpr uint32_t KV_BYTES = BK * HD * 2;
  static constexpr uint32_t QD_BYTES = BQ * HD * 2;
  static constexpr uint32_t PT_BYTES = BK * BQ * 2;
  static constexpr uint32_t DQS_BYTES = BQ * HD * 4;
  static constexpr uint32_t STAT_BYTES = 2 * BQ * 4;  // -l*log2e[128], -D/sqrt(D)[128]
  static constexpr uint32_t OFF_K = 0;                                // [KVB]
  static constexpr uint32_t OFF_V = OFF_K + KVB * KV_BYTES;           // [KVB]
  static constexpr uint32_t OFF_Q = OFF_V + KVB * KV_BYTES;           // [STAGES]
  static constexpr uint32_t OFF_DO = OFF_Q + STAGES * QD_BYTES;       // [STAGES]
  static constexpr uint32_t OFF_PT = OFF_DO + STAGES * QD_BYTES;      // only without P_IN_TMEM
  static constexpr uint32_t OFF_DST = OFF_PT + (P_IN_TMEM ? 0 : PT_BYTES);
  static constexpr uint32_t OFF_DQS = DQS_ALIAS ? OFF_PT : OFF_DST + PT_BYTES;  // [DQSB]
  static constexpr uint32_t OFF_STAT = DQS_ALIAS ? OFF_DST + PT_BYTES : OFF_DQS + DQSB * DQS_BYTES;
  // the unit schedule: NSCHED 16-byte launch-control responses, read by the
  // producer, the UMMA issuer (twice: its look-ahead and current steps), the
  // statistics and reduce warps, and every compute and drain warp
  static constexpr bool DYN = !PERSIST;  // units taken by launch control
  // (batch, head) pairs per block of the unit order (measured: D=128 gains
  // from 16, D=64 at long sequences is fastest (batch, head)-major)
  static constexpr int HB = (DYN && !D64) ? 16 : 1;
  static constexpr int NSCHED = DYN ? (int)kSchedSlots : 0;
  static constexpr uint32_t SCHED_READERS = 5 + NCOMP / 32 + (DRAIN_WG ? 4 : 0);
  static constexpr uint32_t OFF_SCHED = OFF_STAT + SSTG * STAT_BYTES;
  static constexpr uint32_t OFF_BAR = OFF_SCHED + NSCHED * 16;
  // kv_full/empty[KVB], qd_full/empty[S], st_full/empty[8], then s_full,
  // s_free, p_ready, p_free, dq_full, dq_free, dqs_full, dqs_free, done,
  // acc_free, never (nothing arrives: the time-out test hook), fin (the
  // UMMA issuer's wind-down), sched_full/empty[NSCHED]
  static constexpr int NBAR = 2 * KVB + 2 * STAGES + 2 * SSTG + 12 + 2 * (DQSB - 1) + 2 * NSCHED;
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
  int T, N, NH, bh_begin, nbh, nkt, nunits;
  float scale, scale_log2;
  const float* lse;
  const __nv_bfloat16* Dv;
  uint32_t* status;
  uint32_t expire_ns;  // time-out test hook (ma_debug_expire_next_wait), 0 = off
};

// Unit k -> (batch, head, key tile); its query tiles are kt .. nkt-1.  Block
// k / (HB * nkt) holds the units of HB (batch, head) pairs (fewer in the last
// block), key tile-major; HB = 1 is (batch, head)-major.
struct BUnit {
  int b, h, kt, nq;
};

template <int HB>
__device__ __forceinline__ BUnit bwd_unit(const BwdParams& prm, int k) {
  BUnit u;
  int bh;
  if constexpr (HB > 1) {
    const int per = HB * prm.nkt;
    const int blk = k / per, r = k % per;
    const int hb = min(HB, prm.nbh - blk * HB);
    bh = prm.bh_begin + blk * HB + r % hb;
    u.kt = r / hb;
  } else {
    bh = prm.bh_begin + k / prm.nkt;
    u.kt = k % prm.nkt;
  }
  u.b = bh / prm.NH;
  u.h = bh % prm.NH;
  u.nq = prm.nkt - u.kt;
  return u;
}

// Static schedule: the unit of this CTA in round g, -1 when rounds are
// exhausted, -2 when this CTA has none in round g (last, partial round).
__device__ __forceinline__ int bwd_unit_of_round(const BwdParams& prm, int g) {
  const int G = gridDim.x;
  if ((long long)g * G >= prm.nunits) return -1;
  const int c = blockIdx.x;
  const int k = g * G + ((g & 1) ? G - 1 - c : c);
  return k < prm.nunits ? k : -2;
}

// Walks this CTA's (unit, query tile) steps in order.  t counts steps over
// all units, uc counts units.
struct StepIter {
  int g;        // dynamic: units fetched; static: next round to look at
  BUnit u;
  int i;        // query tile index within the unit
  uint32_t t;   // global step
  uint32_t uc;  // unit counter
  bool valid;
};

template <bool DYN, int HB, bool WARP>
__device__ __forceinline__ bool next_unit(const BwdParams& prm, StepIter& s, const Sched& sc) {
  if constexpr (DYN) {
    const int k = sched_unit<WARP>(sc, (uint32_t)s.g++);
    if (k < 0 || k >= prm.nunits) return false;
    s.u = bwd_unit<HB>(prm, k);
    return true;
  } else {
    for (;;) {
      const int k = bwd_unit_of_round(prm, s.g);
      if (k == -1) return false;
      ++s.g;
      if (k >= 0) {
        s.u = bwd_unit<HB>(prm, k);
        return true;
      }
    }
  }
}

template <bool DYN, int HB, bool WARP>
__device__ __forceinline__ StepIter first_step(const BwdParams& prm, const Sched& sc) {
  StepIter s;
  s.g = 0;
  s.i = 0;
  s.t = 0;
  s.uc = 0;
  s.valid = next_unit<DYN, HB, WARP>(prm, s, sc);
  return s;
}

template <bool DYN, int HB, bool WARP>
__device__ __forceinline__ void advance(const BwdParams& prm, StepIter& s, const Sched& sc) {
  ++s.t;
  if (s.i + 1 < s.u.nq) {
    ++s.i;
    return;
  }
  s.i = 0;
  ++s.uc;
  s.valid = next_unit<DYN, HB, WARP>(prm, s, sc);
}

// P^T and dS^T for N query columns of one key row.  s[] holds S^T on entry
// and P^T on exit; dp[] holds dP^T on entry and dS^T on exit.  nl = -l*log2e
// and nd = -D/sqrt(D) per query column (shared memory, broadcast reads).
template <bool DIAG, int N>
__device__ __forceinline__ void p_ds_row(float (&s)[N], float (&dp)[N], const float* nl,
                                         const float* nd, float c, float sc, int krow, int qcol0) {
  const float2 c2 = make_float2(c, c), sc2 = make_float2(sc, sc);
#pragma unroll
  for (int j = 0; j < N; j += 4) {
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

// N bf16 values of one row as N/8 swizzled 16-byte chunks of a K-major SW128
// row, starting at chunk ch0 (row base `rowp`, swizzle phase `row & 7`).
template <int N>
__device__ __forceinline__ void store_row_sw128(uint8_t* rowp, int row, const float (&v)[N], int ch0) {
#pragma unroll
  for (int k = 0; k < N / 8; ++k) {
    const int c0 = k * 8, ch = ch0 + k;
    uint4 w;
    w.x = pack_bf16(v[c0 + 0], v[c0 + 1]);
    w.y = pack_bf16(v[c0 + 2], v[c0 + 3]);
    w.z = pack_bf16(v[c0 + 4], v[c0 + 5]);
    w.w = pack_bf16(v[c0 + 6], v[c0 + 7]);
    *reinterpret_cast<uint4*>(rowp + ((ch ^ (row & 7)) * 16)) = w;
  }
}

template <int HD, bool PERSIST>
__global__ void __launch_bounds__(BwdCfg<HD, PERSIST>::NUM_THREADS, 1)
    flash_bwd_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                     const __grid_constant__ CUtensorMap tmV, const __grid_constant__ CUtensorMap tmdO,
                     const __grid_constant__ CUtensorMap tmdQ, __nv_bfloat16* __restrict__ dK,
                     __nv_bfloat16* __restrict__ dV, const BwdParams prm) {
  pdl_wait_and_release();
  using C = BwdCfg<HD, PERSIST>;
  extern __shared__ uint8_t smem_raw[];
  __shared__ int abort_flag;
  const uint32_t raw = smem_u32(smem_raw);
  const uint32_t sbase = (raw + 1023u) & ~1023u;
  uint8_t* gbase = smem_raw + (sbase - raw);
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;

  const uint32_t bar0 = sbase + C::OFF_BAR;
  auto BAR_KF = [&](int s) { return bar0 + 8u * s; };
  auto BAR_KE = [&](int s) { return bar0 + 8u * (C::KVB + s); };
  auto BAR_QF = [&](int s) { return bar0 + 8u * (2 * C::KVB + s); };
  auto BAR_QE = [&](int s) { return bar0 + 8u * (2 * C::KVB + C::STAGES + s); };
  auto BAR_TF = [&](int s) { return bar0 + 8u * (2 * C::KVB + 2 * C::STAGES + s); };
  auto BAR_TE = [&](int s) { return bar0 + 8u * (2 * C::KVB + 2 * C::STAGES + C::SSTG + s); };
  const uint32_t BAR_SF = bar0 + 8u * (2 * C::KVB + 2 * C::STAGES + 2 * C::SSTG);
  const uint32_t BAR_SE = BAR_SF + 8;
  const uint32_t BAR_PR = BAR_SF + 16;
  const uint32_t BAR_PE = BAR_SF + 24;
  const uint32_t BAR_DQF = BAR_SF + 32;
  const uint32_t BAR_DQE = BAR_SF + 40;
  // staging buffer b: BAR_DSF(b) written, BAR_DSE(b) read by its reduction
  auto BAR_DSF = [&](int b) { return b == 0 ? BAR_SF + 48 : BAR_SF + 96 + 16u * (b - 1); };
  auto BAR_DSE = [&](int b) { return b == 0 ? BAR_SF + 56 : BAR_SF + 104 + 16u * (b - 1); };
  const uint32_t BAR_DONE = BAR_SF + 64;  // a unit's last UMMA completed
  const uint32_t BAR_ACC = BAR_SF + 72;   // dK/dV TMEM read by the epilogue
  const uint32_t BAR_NEVER = BAR_SF + 80; // nothing arrives (time-out test hook)
  const uint32_t BAR_FIN = BAR_SF + 88;   // the UMMA issuer's last commit (wind-down)
  const uint32_t BAR_UF = BAR_SF + 96 + 16u * (C::DQSB - 1);  // sched_full[NSCHED], then sched_empty
  const uint32_t BAR_UE = BAR_UF + 8u * C::NSCHED;
  const uint32_t tslot = sbase + C::OFF_TSLOT;
  float* stat_base = reinterpret_cast<float*>(gbase + C::OFF_STAT);

  if (threadIdx.x == 0) {
    abort_flag = 0;
    for (int s = 0; s < C::KVB; ++s) {
      mbar_init(BAR_KF(s), 1);
      mbar_init(BAR_KE(s), 1);
    }
    for (int s = 0; s < C::STAGES; ++s) {
      mbar_init(BAR_QF(s), 1);
      mbar_init(BAR_QE(s), 1);
    }
    for (int s = 0; s < C::SSTG; ++s) {
      mbar_init(BAR_TF(s), 32);
      mbar_init(BAR_TE(s), C::NCOMP);
    }
    mbar_init(BAR_SF, 1);
    mbar_init(BAR_SE, C::NCOMP);
    mbar_init(BAR_PR, C::NCOMP);
    mbar_init(BAR_PE, 1);
    mbar_init(BAR_DQF, 1);
    mbar_init(BAR_DQE, C::NDRAIN);
    for (int b = 0; b < C::DQSB; ++b) {
      mbar_init(BAR_DSF(b), C::NDRAIN);
      mbar_init(BAR_DSE(b), 1);
    }
    mbar_init(BAR_DONE, 1);
    mbar_init(BAR_ACC, C::NACC);
    mbar_init(BAR_NEVER, 1);
    mbar_init(BAR_FIN, 1);
    for (int u = 0; u < C::NSCHED; ++u) {
      mbar_init(BAR_UF + 8u * u, 1);
      mbar_init(BAR_UE + 8u * u, C::SCHED_READERS);
    }
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
  const Sched sch{sbase + C::OFF_SCHED, BAR_UF, BAR_UE, abort_p};  // the unit schedule

  if (warp < 4) {
    reg_dealloc<C::REGS_PRODUCER>();
    if (warp == 0) {
      // --------------------------------------------------------- producer
      if (lane == 0) {
        tma_prefetch_desc(&tmQ);
        tma_prefetch_desc(&tmdO);
        uint32_t kv_armed = 0, q_armed = 0;  // loads issued into each ring
        uint32_t nreq = 0;                   // launch-control requests issued
        for (StepIter s = first_step<C::DYN, C::HB, false>(prm, sch); s.valid; advance<C::DYN, C::HB, false>(prm, s, sch)) {
          const int col0 = s.u.h * HD;
          if (s.i == 0) {  // K/V of a new unit
            const int kvs = s.uc % C::KVB;
            if (s.uc >= C::KVB && !mbar_wait(BAR_KE(kvs), ((s.uc / C::KVB) - 1) & 1, abort_p)) break;
            mbar_arrive_expect_tx(BAR_KF(kvs), 2 * C::KV_BYTES);
            ++kv_armed;
            for (int kb = 0; kb < C::KB; ++kb) {
              tma_load_3d(sbase + C::OFF_K + kvs * C::KV_BYTES + kb * BK * 128, &tmK, BAR_KF(kvs),
                          col0 + kb * 64, s.u.kt * BK, s.u.b);
              tma_load_3d(sbase + C::OFF_V + kvs * C::KV_BYTES + kb * BK * 128, &tmV, BAR_KF(kvs),
                          col0 + kb * 64, s.u.kt * BK, s.u.b);
            }
          }
          const int st = s.t % C::STAGES;
          if (s.t >= C::STAGES && !mbar_wait(BAR_QE(st), ((s.t / C::STAGES) - 1) & 1, abort_p)) break;
          const int qt = s.u.kt + s.i;
          mbar_arrive_expect_tx(BAR_QF(st), 2 * C::QD_BYTES);
          ++q_armed;
          for (int kb = 0; kb < C::KB; ++kb) {
            tma_load_3d(sbase + C::OFF_Q + st * C::QD_BYTES + kb * BQ * 128, &tmQ, BAR_QF(st),
                        col0 + kb * 64, qt * BQ, s.u.b);
            tma_load_3d(sbase + C::OFF_DO + st * C::QD_BYTES + kb * BQ * 128, &tmdO, BAR_QF(st),
                        col0 + kb * 64, qt * BQ, s.u.b);
          }
          // three steps before the unit's end (or at its start), ask for the
          // next unit, so that every reader finds the answer when it gets there
          if (C::DYN && s.i == max(0, s.u.nq - 3)) {
            if (!sched_request(sch, nreq)) break;
            ++nreq;
          }
        }
        if (*abort_p) {  // wind-down: let the loads and the request still in flight land
          if (C::DYN) sched_drain(sch, nreq);
          drain_ring(BAR_KF, C::KVB, kv_armed);
          drain_ring(BAR_QF, C::STAGES, q_armed);
        }
      }
    } else if (warp == 1) {
      // -------------------------------------------------------------- MMA
      if (lane == 0) {
        constexpr uint32_t IDESC_S = idesc_bf16_f32(BK, BQ, 0, 0);   // S^T, dP^T
        constexpr uint32_t IDESC_KV = idesc_bf16_f32(BK, HD, 0, 1);  // dV, dK
        constexpr uint32_t IDESC_Q = idesc_bf16_f32(BQ, HD, 1, 1);   // dQ
        const uint32_t spt = sbase + C::OFF_PT, sdst = sbase + C::OFF_DST;
        // S^T and dP^T of step s into their TMEM columns
        auto issue_s = [&](const StepIter& s) -> bool {
          const int st = s.t % C::STAGES;
          const int kvs = s.uc % C::KVB;
          if (s.i == 0 && !mbar_wait(BAR_KF(kvs), (s.uc / C::KVB) & 1, abort_p)) return false;
          if (!mbar_wait(BAR_QF(st), (s.t / C::STAGES) & 1, abort_p)) return false;
          if (s.t >= 1 && !mbar_wait(BAR_SE, (s.t - 1) & 1, abort_p)) return false;
          if (C::DQ_ALIAS && s.t >= 1 && !mbar_wait(BAR_DQE, (s.t - 1) & 1, abort_p)) return false;
          tc_fence_after();
          const uint32_t sk = sbase + C::OFF_K + kvs * C::KV_BYTES;
          const uint32_t sv = sbase + C::OFF_V + kvs * C::KV_BYTES;
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
        StepIter cur = first_step<C::DYN, C::HB, false>(prm, sch);
        StepIter la = cur;  // next step whose S^T/dP^T is to be issued
        bool ok = true;
        if (la.valid) {
          ok = issue_s(la);
          advance<C::DYN, C::HB, false>(prm, la, sch);
        }
        // time-out test hook: with the first products in flight, wait on a
        // barrier nothing arrives at until the hook's limit runs out
        if (ok && prm.expire_ns) ok = mbar_wait(BAR_NEVER, 0, abort_p, prm.expire_ns);
        for (; ok && cur.valid; advance<C::DYN, C::HB, false>(prm, cur, sch)) {
          // the next step's S^T/dP^T ahead of this step's products, except
          // where it starts a unit whose K/V can only be loaded into the
          // single K/V buffer once this step's products are done with it
          const bool early = C::EARLY_S && la.valid && (C::KVB > 1 || la.uc == cur.uc);
          if (early) {
            if (!issue_s(la)) break;
            advance<C::DYN, C::HB, false>(prm, la, sch);
          }
          const int st = cur.t % C::STAGES;
          const int kvs = cur.uc % C::KVB;
          const uint32_t sk = sbase + C::OFF_K + kvs * C::KV_BYTES;
          const uint32_t sq = sbase + C::OFF_Q + st * C::QD_BYTES;
          const uint32_t sdo = sbase + C::OFF_DO + st * C::QD_BYTES;
          if (!mbar_wait(BAR_PR, cur.t & 1, abort_p)) break;
          // the previous unit's epilogue must have read dK/dV out of TMEM
          if (cur.i == 0 && cur.uc >= 1 && !mbar_wait(BAR_ACC, (cur.uc - 1) & 1, abort_p)) break;
          tc_fence_after();
#pragma unroll
          for (int kk = 0; kk < BQ / 16; ++kk) {  // dV += P^T dO_i
            const uint64_t bd = smem_desc_sw128(sdo + kk * 2048, BQ * 128, 1024);
            if (C::P_IN_TMEM) {
              umma_bf16_ts(tmem + C::TCOL_DV, tmem + C::TCOL_PT + kk * 8, bd, IDESC_KV,
                           (cur.i > 0 || kk > 0) ? 1u : 0u);
            } else {
              const uint64_t ad = smem_desc_sw128(spt + (kk >> 2) * (BK * 128) + (kk & 3) * 32, 16, 1024);
              umma_bf16_ss(tmem + C::TCOL_DV, ad, bd, IDESC_KV, (cur.i > 0 || kk > 0) ? 1u : 0u);
            }
          }
#pragma unroll
          for (int kk = 0; kk < BQ / 16; ++kk) {  // dK += dS^T Q_i
            const uint64_t ad = smem_desc_sw128(sdst + (kk >> 2) * (BK * 128) + (kk & 3) * 32, 16, 1024);
            const uint64_t bd = smem_desc_sw128(sq + kk * 2048, BQ * 128, 1024);
            umma_bf16_ss(tmem + C::TCOL_DK, ad, bd, IDESC_KV, (cur.i > 0 || kk > 0) ? 1u : 0u);
          }
          umma_commit(BAR_QE(st));
          // the dQ columns must have been drained (previous step)
          if (cur.t >= 1 && !mbar_wait(BAR_DQE, (cur.t - 1) & 1, abort_p)) break;
          tc_fence_after();
#pragma unroll
          for (int kk = 0; kk < BK / 16; ++kk) {  // dQ_i = dS K (A = dS^T as MN-major)
            const uint64_t ad = smem_desc_sw128(sdst + kk * 2048, BK * 128, 1024);
            const uint64_t bd = smem_desc_sw128(sk + kk * 2048, BK * 128, 1024);
            umma_bf16_ss(tmem + C::TCOL_DQ, ad, bd, IDESC_Q, kk > 0 ? 1u : 0u);
          }
          umma_commit(BAR_DQF);
          umma_commit(BAR_PE);
          if (cur.i + 1 == cur.u.nq) {  // the unit's last UMMA
            umma_commit(BAR_KE(kvs));
            umma_commit(BAR_DONE);
          }
          // (after them: D=128, or a unit start with a single K/V buffer)
          if ((!C::EARLY_S || C::KVB == 1) && !early && la.valid) {
            if (!issue_s(la)) break;
            advance<C::DYN, C::HB, false>(prm, la, sch);
          }
        }
        if (*abort_p) {  // wind-down: every UMMA issued must complete before TMEM is freed
          umma_commit(BAR_FIN);
          mbar_wait_for(BAR_FIN, 0, kDrainLimitNs);
        }
      }
    } else if (warp == 2) {
      // ------------------------------------------------------- statistics
      // A step's 128 (-l*log2e, -D/sqrt(D)) pairs, four queries per lane,
      // are loaded into registers one step ahead, so the ring slot is filled
      // as soon as the compute warps free it, whatever the load latency.
      float nl[4], nd[4];
      auto load_stats = [&](const StepIter& s) {
        const int qt = s.u.kt + s.i;
        const long long rbase = (long long)s.u.b * prm.T;
#pragma unroll
        for (int v = 0; v < 4; ++v) {
          const int q = qt * BQ + lane * 4 + v;
          nl[v] = 0.0f;
          nd[v] = 0.0f;
          if (q < prm.T) {
            const long long si = (rbase + q) * prm.NH + s.u.h;
            nl[v] = -__ldg(prm.lse + si) * LOG2E;
            nd[v] = -__bfloat162float(prm.Dv[si]) * prm.scale;
          }
        }
      };
      StepIter s = first_step<C::DYN, C::HB, true>(prm, sch);
      if (s.valid) load_stats(s);
      while (s.valid) {
        const float cl[4] = {nl[0], nl[1], nl[2], nl[3]};
        const float cd[4] = {nd[0], nd[1], nd[2], nd[3]};
        StepIter nx = s;
        advance<C::DYN, C::HB, true>(prm, nx, sch);
        if (nx.valid) load_stats(nx);  // the next step's, in flight while this one waits
        const int st = s.t % C::SSTG;
        if (s.t >= C::SSTG && !mbar_wait_warp(BAR_TE(st), ((s.t / C::SSTG) - 1) & 1, abort_p)) break;
        float* stt = stat_base + st * (2 * BQ);
#pragma unroll
        for (int v = 0; v < 4; ++v) {
          stt[lane * 4 + v] = cl[v];
          stt[BQ + lane * 4 + v] = cd[v];
        }
        mbar_arrive(BAR_TF(st));
        s = nx;
      }
    } else {
      // ------------------------------------------------- dQ reduce issuer
      if (lane == 0) {
        for (StepIter s = first_step<C::DYN, C::HB, false>(prm, sch); s.valid; advance<C::DYN, C::HB, false>(prm, s, sch)) {
          const int b = s.t % C::DQSB;
          if (!mbar_wait(BAR_DSF(b), (s.t / C::DQSB) & 1, abort_p)) break;
          for (int box = 0; box < HD / 32; ++box)
            tma_reduce_add_3d(&tmdQ, sbase + C::OFF_DQS + b * C::DQS_BYTES + box * (BQ * 128),
                              s.u.h * HD + box * 32, (s.u.kt + s.i) * BQ, s.u.b);
          bulk_commit();
          // the reduction DQSB-1 steps back has read its buffer, which may
          // now be rewritten (with one buffer: this step's)
          bulk_wait_read<C::DQSB - 1>();
          if (s.t + 1 >= (uint32_t)C::DQSB) mbar_arrive(BAR_DSE((s.t + 1 - C::DQSB) % C::DQSB));
        }
        bulk_wait<0>();
      }
    }
  } else if (!C::DRAIN_WG || warp < 4 + C::NCOMP / 32) {
    reg_alloc<C::REGS_COMPUTE>();
    // ------------------------------------------------------------ compute
    constexpr int CPP = C::CPP;                // query columns per part
    const int cw = warp - 4;                   // 0 .. NCOMP/32 - 1
    const int quarter = warp & 3;              // TMEM lane quarter
    const int krow = quarter * 32 + lane;      // key row (and dQ query row) within the tile
    const int part = cw >> 2;                  // query columns part*CPP .. +CPP-1
    const uint32_t tl = tmem + ((uint32_t)(quarter * 32) << 16);
    const float c = prm.scale_log2, sc = prm.scale;
    bool ok = true;

    // dQ of global step t: TMEM -> fp32 staging (128-byte swizzle, 32-column
    // boxes); the reduce issuer (warp 3) sends it to global memory.  Each
    // part drains HD / NPART of the head dimension's columns.
    auto drain_dq = [&](uint32_t t) {
      const int b = t % C::DQSB;
      if (ok) ok = mbar_wait_warp(BAR_DQF, t & 1, abort_p);
      if (ok && t >= (uint32_t)C::DQSB) ok = mbar_wait_warp(BAR_DSE(b), ((t / C::DQSB) - 1) & 1, abort_p);
      if (!ok) return;
      tc_fence_after();
      constexpr int CPH = HD / C::NPART;  // dQ columns per part
      uint8_t* dqs = gbase + C::OFF_DQS + b * C::DQS_BYTES;
#pragma unroll
      for (int cc = 0; cc < CPH; cc += 16) {
        uint32_t r[16];
        tmem_ld16(tl + C::TCOL_DQ + part * CPH + cc, r);
        tmem_wait_ld_dep(r);
        const int col = part * CPH + cc;  // first column (fp32) of the 16
        uint8_t* rowp = dqs + (col / 32) * (BQ * 128) + krow * 128;
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          const int ch = (col % 32) / 4 + q;
          uint4 v = make_uint4(r[q * 4 + 0], r[q * 4 + 1], r[q * 4 + 2], r[q * 4 + 3]);
          *reinterpret_cast<uint4*>(rowp + ((ch ^ (krow & 7)) * 16)) = v;
        }
      }
      tc_fence_before();
      mbar_arrive(BAR_DQE);
      fence_proxy_async_smem();
      mbar_arrive(BAR_DSF(b));
    };

    // dK/dV of unit v (its UMMAs complete, BAR_DONE phase vuc): TMEM ->
    // registers; frees the accumulators (BAR_ACC) for the next unit, then
    // converts to bf16 and stores this thread's row slice straight to global
    // memory (rows past T are not stored)
    auto epilogue = [&](const BUnit& v, uint32_t vuc) {
      if (ok) ok = mbar_wait_warp(BAR_DONE, vuc & 1, abort_p);
      if (!ok) return;
      tc_fence_after();
      constexpr int CPH = HD / C::NPART;  // dV, dK columns per part
      uint32_t acc[2][CPH];
#pragma unroll
      for (int which = 0; which < 2; ++which) {
        const uint32_t tcol = which == 0 ? C::TCOL_DV : C::TCOL_DK;
#pragma unroll
        for (int cc = 0; cc < CPH; cc += 16) {
          uint32_t r[16];
          tmem_ld16(tl + tcol + part * CPH + cc, r);
          tmem_wait_ld_dep(r);
#pragma unroll
          for (int j = 0; j < 16; ++j) acc[which][cc + j] = r[j];
        }
      }
      tc_fence_before();
      mbar_arrive(BAR_ACC);  // the next unit may overwrite dK/dV in TMEM
      const int key = v.kt * BK + krow;
      if (key < prm.T) {
        const long long off = ((long long)v.b * prm.T + key) * prm.N + v.h * HD + part * CPH;
#pragma unroll
        for (int which = 0; which < 2; ++which) {
          uint4* dst = reinterpret_cast<uint4*>((which == 0 ? dV : dK) + off);
#pragma unroll
          for (int cc = 0; cc < CPH; cc += 8) {
            uint4 w;
            w.x = pack_bf16(__uint_as_float(acc[which][cc + 0]), __uint_as_float(acc[which][cc + 1]));
            w.y = pack_bf16(__uint_as_float(acc[which][cc + 2]), __uint_as_float(acc[which][cc + 3]));
            w.z = pack_bf16(__uint_as_float(acc[which][cc + 4]), __uint_as_float(acc[which][cc + 5]));
            w.w = pack_bf16(__uint_as_float(acc[which][cc + 6]), __uint_as_float(acc[which][cc + 7]));
            dst[cc / 8] = w;
          }
        }
      }
    };

    // A unit's last dQ drain and its dK/dV epilogue run after the first step
    // of the next unit has been handed to the tensor core (or after the last
    // step of the last unit), so they overlap the next unit's UMMAs.
    BUnit prev{};
    uint32_t t = 0, uc = 0;
    bool have_prev = false;
    for (StepIter st_it = first_step<C::DYN, C::HB, true>(prm, sch); ok && st_it.valid; advance<C::DYN, C::HB, true>(prm, st_it, sch)) {
      const BUnit& u = st_it.u;
      const int i = st_it.i;
      t = st_it.t;
      uc = st_it.uc;
      const int ss = t % C::SSTG;
      ok = mbar_wait_warp(BAR_SF, t & 1, abort_p);
      if (!ok) break;
      tc_fence_after();
      float s[CPP], dp[CPP];
      if constexpr (CPP == 64) {
        uint32_t ra[32], rb[32];
        tmem_ld32(tl + C::TCOL_S + part * 64, ra);
        tmem_ld32(tl + C::TCOL_S + part * 64 + 32, rb);
        tmem_wait_ld_dep(ra, rb);
#pragma unroll
        for (int j = 0; j < 32; ++j) {
          s[j] = __uint_as_float(ra[j]);
          s[32 + j] = __uint_as_float(rb[j]);
        }
        tmem_ld32(tl + C::TCOL_DP + part * 64, ra);
        tmem_ld32(tl + C::TCOL_DP + part * 64 + 32, rb);
        tmem_wait_ld_dep(ra, rb);
#pragma unroll
        for (int j = 0; j < 32; ++j) {
          dp[j] = __uint_as_float(ra[j]);
          dp[32 + j] = __uint_as_float(rb[j]);
        }
      } else {
        static_assert(CPP == 32, "column split");
        uint32_t ra[32], rb[32];
        tmem_ld32(tl + C::TCOL_S + part * 32, ra);
        tmem_ld32(tl + C::TCOL_DP + part * 32, rb);
        tmem_wait_ld_dep(ra, rb);
#pragma unroll
        for (int j = 0; j < 32; ++j) {
          s[j] = __uint_as_float(ra[j]);
          dp[j] = __uint_as_float(rb[j]);
        }
      }
      tc_fence_before();
      mbar_arrive(BAR_SE);
      ok = mbar_wait_warp(BAR_TF(ss), (t / C::SSTG) & 1, abort_p);
      if (!ok) break;
      const float* stt = stat_base + ss * (2 * BQ) + part * CPP;
      if (i == 0) p_ds_row<true, CPP>(s, dp, stt, stt + BQ, c, sc, krow, part * CPP);
      else p_ds_row<false, CPP>(s, dp, stt, stt + BQ, c, sc, krow, part * CPP);
      mbar_arrive(BAR_TE(ss));
      // the previous step's UMMAs must be done with P^T/dS^T, and when the dQ
      // staging shares their smem its reduction must have read it
      if (t >= 1) ok = mbar_wait_warp(BAR_PE, (t - 1) & 1, abort_p);
      if (ok && C::DQS_ALIAS && t >= 1) ok = mbar_wait_warp(BAR_DSE(0), (t - 1) & 1, abort_p);
      if (!ok) break;
      // this part's columns of the key row: P^T (bf16 pairs in TMEM, or smem),
      // dS^T (smem); chunk (part*CPP % 64) / 8 of 64-column block part*CPP / 64
      const int blk = (part * CPP) / 64, ch0 = ((part * CPP) % 64) / 8;
      if constexpr (C::P_IN_TMEM) {
        uint32_t pk[CPP / 2];
#pragma unroll
        for (int j = 0; j < CPP / 2; ++j) pk[j] = pack_bf16(s[2 * j], s[2 * j + 1]);
        if constexpr (CPP == 64) tmem_st32(tl + C::TCOL_PT + part * 32, pk);
        else tmem_st16(tl + C::TCOL_PT + part * 16, pk);
        tmem_wait_st();
      } else {
        store_row_sw128<CPP>(gbase + C::OFF_PT + blk * (BK * 128) + krow * 128, krow, s, ch0);
      }
      store_row_sw128<CPP>(gbase + C::OFF_DST + blk * (BK * 128) + krow * 128, krow, dp, ch0);
      fence_proxy_async_smem();
      tc_fence_before();
      mbar_arrive(BAR_PR);
      // on a unit's first step the previous unit's dK/dV epilogue comes
      // first: the UMMA issuer waits for it before this step's products,
      // the dQ product that drain_dq(t) waits for among them
      if constexpr (C::EPI_COMPUTE) {
        if (i == 0 && have_prev) epilogue(prev, uc - 1);
        prev = u;
        have_prev = true;
      }
      if constexpr (!C::DRAIN_WG) {
        if (C::EARLY_S) {
          if (t >= 1) drain_dq(t - 1);
        } else {
          drain_dq(t);
        }
      }
    }
    if (ok && have_prev) {  // the last unit of this CTA
      if constexpr (!C::DRAIN_WG && C::EARLY_S) drain_dq(t);
      if constexpr (C::EPI_COMPUTE) epilogue(prev, uc);
    }
  } else {
    reg_dealloc<C::REGS_DRAIN>();
    // ---------------------------------------------------------- dQ drain
    // (D=64, warps 12-15): thread = TMEM lane = dQ query row
    const int quarter = warp & 3;
    const int row = quarter * 32 + lane;
    const uint32_t tl = tmem + ((uint32_t)(quarter * 32) << 16);
    bool ok = true;
    for (StepIter s = first_step<C::DYN, C::HB, true>(prm, sch); ok && s.valid; advance<C::DYN, C::HB, true>(prm, s, sch)) {
      const uint32_t t = s.t;
      const int b = t % C::DQSB;
      uint8_t* dqs = gbase + C::OFF_DQS + b * C::DQS_BYTES;
      // dQ of step t: TMEM -> fp32 staging b (128-byte swizzle, 32-column
      // boxes); the reduce issuer (warp 3) adds it into global dQ
      ok = mbar_wait_warp(BAR_DQF, t & 1, abort_p);
      if (ok && t >= (uint32_t)C::DQSB) ok = mbar_wait_warp(BAR_DSE(b), ((t / C::DQSB) - 1) & 1, abort_p);
      if (!ok) break;
      tc_fence_after();
#pragma unroll
      for (int cc = 0; cc < HD; cc += 16) {
        uint32_t r[16];
        tmem_ld16(tl + C::TCOL_DQ + cc, r);
        tmem_wait_ld_dep(r);
        uint8_t* rowp = dqs + (cc / 32) * (BQ * 128) + row * 128;
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          const int ch = (cc % 32) / 4 + q;
          const uint4 v = make_uint4(r[q * 4 + 0], r[q * 4 + 1], r[q * 4 + 2], r[q * 4 + 3]);
          *reinterpret_cast<uint4*>(rowp + ((ch ^ (row & 7)) * 16)) = v;
        }
      }
      tc_fence_before();
      mbar_arrive(BAR_DQE);
      fence_proxy_async_smem();
      mbar_arrive(BAR_DSF(b));
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
  pdl_wait_and_release();
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

template <int HD, bool PERSIST>
cudaError_t launch_bwd_kernel(const __nv_bfloat16* dO, const __nv_bfloat16* q,
                              const __nv_bfloat16* k, const __nv_bfloat16* v, float* dQ,
                              __nv_bfloat16* dK, __nv_bfloat16* dV, const AttnShape& s,
                              const BwdParams& prm, int grid, cudaStream_t st) {
  using C = BwdCfg<HD, PERSIST>;
  // The setmaxnreg split assumes the kernel was compiled to exactly
  // LAUNCH_REGS registers per thread; refuse to launch otherwise.
  static const cudaError_t reg_check = [] {
    cudaFuncAttributes a;
    cudaError_t e = cudaFuncGetAttributes(&a, flash_bwd_kernel<HD, PERSIST>);
    if (e != cudaSuccess) return e;
    return a.numRegs == C::LAUNCH_REGS ? cudaSuccess : cudaErrorInvalidKernelImage;
  }();
  if (reg_check != cudaSuccess) return reg_check;
  CUtensorMap tq, tk, tv, tdo, tdq;
  const CUtensorMapDataType bf = CU_TENSOR_MAP_DATA_TYPE_BFLOAT16;
  const CUtensorMapSwizzle sw = CU_TENSOR_MAP_SWIZZLE_128B;
  if (!make_tmap_3d(&tq, q, bf, 2, s.N, s.T, s.B, 64, BQ, sw) ||
      !make_tmap_3d(&tk, k, bf, 2, s.N, s.T, s.B, 64, BK, sw) ||
      !make_tmap_3d(&tv, v, bf, 2, s.N, s.T, s.B, 64, BK, sw) ||
      !make_tmap_3d(&tdo, dO, bf, 2, s.N, s.T, s.B, 64, BQ, sw) ||
      !make_tmap_3d(&tdq, dQ, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, s.N, s.T, s.B, 32, BQ, sw))
    return cudaErrorInvalidValue;
  cudaError_t e = cudaFuncSetAttribute(flash_bwd_kernel<HD, PERSIST>,
                                       cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM_BYTES);
  if (e != cudaSuccess) return e;
  launch_pdl(flash_bwd_kernel<HD, PERSIST>, grid, C::NUM_THREADS, C::SMEM_BYTES, st, tq, tk, tv, tdo, tdq, dK,
                                                                        dV, prm);
  count_launches(1);
  return cudaGetLastError();
}

template <int HD>
cudaError_t launch_bwd(const __nv_bfloat16* dO, const __nv_bfloat16* Dv, const float* lse,
                       const __nv_bfloat16* q, const __nv_bfloat16* k, const __nv_bfloat16* v,
                       float* dQ, __nv_bfloat16* dK, __nv_bfloat16* dV, const AttnShape& s,
                       uint32_t* status, cudaStream_t st, bool accumulate_dq) {
  // dQ is accumulated by bulk reductions: zero the shard's columns first,
  // unless the caller asks for dQ += (it holds zeros or partial sums)
  const int nbh = s.bh_end - s.bh_begin;
  if (!accumulate_dq) {
    const cudaError_t e = launch_zero_dq(dQ, s, st);
    if (e != cudaSuccess) return e;
  }
  BwdParams prm;
  prm.T = s.T;
  prm.N = s.N;
  prm.NH = s.NH;
  prm.bh_begin = s.bh_begin;
  prm.nbh = nbh;
  prm.nkt = (s.T + BK - 1) / BK;
  prm.nunits = prm.nkt * nbh;
  prm.scale = 1.0f / sqrtf((float)HD);
  prm.scale_log2 = LOG2E / sqrtf((float)HD);
  prm.lse = lse;
  prm.Dv = Dv;
  prm.status = status;
  prm.expire_ns = take_expire_request(STATUS_BWD_TIMEOUT);
  // short sequences at D=64: static rounds over one CTA per SM, (batch,
  // head)-major; otherwise one CTA per unit, the running CTAs taking over the
  // rest (see bwd_unit)
  if (HD == 64 && prm.nkt <= PERSIST_MAX_NKT) {
    int dev = 0, sms = 148;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    const int grid = prm.nunits < sms ? prm.nunits : sms;
    return launch_bwd_kernel<HD, true>(dO, q, k, v, dQ, dK, dV, s, prm, grid, st);
  }
  return launch_bwd_kernel<HD, false>(dO, q, k, v, dQ, dK, dV, s, prm, prm.nunits, st);
}

}  // namespace

cudaError_t launch_zero_dq(float* dQ, const AttnShape& s, cudaStream_t st) {
  if (s.bh_begin == 0 && s.bh_end == s.B * s.NH)
    return cudaMemsetAsync(dQ, 0, (size_t)s.B * s.T * s.N * sizeof(float), st);
  launch_pdl(zero_dq_shard_kernel, 1184, 256, 0, st, reinterpret_cast<float4*>(dQ), s.T, s.N, s.D, s.NH,
             s.bh_begin, s.bh_end);
  count_launches(1);
  return cudaGetLastError();
}

cudaError_t launch_flash_bwd(const __nv_bfloat16* dO, const __nv_bfloat16* Dv,
                             const float* lse, const __nv_bfloat16* q,
                             const __nv_bfloat16* k, const __nv_bfloat16* v, float* dQ,
                             __nv_bfloat16* dK, __nv_bfloat16* dV, const AttnShape& s,
                             uint32_t* status, cudaStream_t st, bool accumulate_dq) {
  if (s.bh_end <= s.bh_begin) return cudaSuccess;
  return s.D == 64 ? launch_bwd<64>(dO, Dv, lse, q, k, v, dQ, dK, dV, s, status, st, accumulate_dq)
                   : launch_bwd<128>(dO, Dv, lse, q, k, v, dQ, dK, dV, s, status, st, accumulate_dq);
}

}  // namespace ma
