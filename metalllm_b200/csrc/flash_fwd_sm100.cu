// flash_fwd_sm100.cu -- flashAttentionForward (attention.metal:56-164) on
// sm_100a: tcgen05 UMMA with TMEM accumulators, TMA-staged Q/K/V tiles in
// 128-byte-swizzled shared memory, an mbarrier pipeline and warp-specialised
// roles.
//
// Work unit: one CTA per (batch*head, 128-row query tile); tiles with the most
// causal work are launched first.  Per key tile j (128 keys):
//   S_j  = Q K_j^T            UMMA 128x128xD, fp32 in TMEM (double-buffered)
//   P_j  = exp2(S_j*c - m)    softmax warps, c = log2(e)/sqrt(D), bf16 to smem
//   O   += P_j V_j            UMMA 128xDx128, fp32 in TMEM
// Roles (192 threads):
//   warp 0     TMA producer: Q once, K/V tiles into a STAGES-deep ring
//   warp 1     owns TMEM; lane 0 issues every UMMA and commit
//   warps 2-5  softmax: thread = query row = TMEM lane; row max/sum in
//              registers, lazy O rescaling (only when the running max grows by
//              more than 2^8), epilogue O/l -> bf16 via smem + TMA store, and
//              l = m + ln(rowsum) in fp32.
// Conventions match the reference: scale 1/sqrt(D) applied to Q K^T, key >
// query masked, l stored fp32 at [row*NH + head], O = (sum P V) / rowsum.
// S stays fp32 (the reference rounds it to bf16); P is bf16 as in the
// reference (attention.metal:139,153).
//
// Every mbarrier wait is bounded (about 2 s); on time-out the CTA sets an
// abort flag that all roles poll, winds down, frees its TMEM and sets
// STATUS_FWD_TIMEOUT in the device status word.
#include "common.cuh"
#include "sm100.cuh"
#include "tmap.h"

namespace ma {
namespace {

using namespace sm100;

constexpr int BM = 128;  // query rows per CTA
constexpr int BN = 128;  // keys per tile
constexpr int NUM_THREADS = 192;
constexpr float LOG2E = 1.4426950408889634f;
constexpr float LN2 = 0.6931471805599453f;
constexpr float RESCALE_THRESHOLD = 8.0f;  // log2 units

template <int HD>
struct FwdCfg {
  static constexpr int KB = HD / 64;                 // 64-column blocks per row
  static constexpr int STAGES = 2;
  static constexpr int PBUF = HD == 64 ? 2 : 1;
  static constexpr uint32_t Q_BYTES = BM * HD * 2;
  static constexpr uint32_t KV_BYTES = BN * HD * 2;
  static constexpr uint32_t P_BYTES = BM * BN * 2;
  // shared memory map (offsets from a 1024-aligned base)
  static constexpr uint32_t OFF_Q = 0;
  static constexpr uint32_t OFF_K = OFF_Q + Q_BYTES;
  static constexpr uint32_t OFF_V = OFF_K + STAGES * KV_BYTES;
  static constexpr uint32_t OFF_P = OFF_V + STAGES * KV_BYTES;
  static constexpr uint32_t OFF_BAR = OFF_P + PBUF * P_BYTES;
  // barriers: q_full, k_full[S], v_full[S], kv_empty[S], s_full[2], s_free[2],
  // p_full[PB], p_free[PB], o_full
  static constexpr int NBAR = 1 + 3 * STAGES + 4 + 2 * PBUF + 1;
  static constexpr uint32_t OFF_TSLOT = OFF_BAR + NBAR * 8;
  static constexpr uint32_t SMEM_BYTES = OFF_TSLOT + 16 + 1024;  // + alignment slack
  static constexpr uint32_t TMEM_COLS = 512;
  static constexpr uint32_t TCOL_S = 0;     // S buffers at columns 0, 128
  static constexpr uint32_t TCOL_O = 256;   // O at 256 .. 256+HD
};

struct FwdParams {
  int T, N, NH, bh_begin, nbh, nqt;
  float scale_log2;
  float* lse;
  uint32_t* status;
};

template <int HD>
__global__ void __launch_bounds__(NUM_THREADS, 1)
    flash_fwd_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                     const __grid_constant__ CUtensorMap tmV, const __grid_constant__ CUtensorMap tmO,
                     const FwdParams prm) {
  using C = FwdCfg<HD>;
  extern __shared__ uint8_t smem_raw[];
  __shared__ int abort_flag;
  const uint32_t raw = smem_u32(smem_raw);
  const uint32_t sbase = (raw + 1023u) & ~1023u;
  uint8_t* gbase = smem_raw + (sbase - raw);

  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  // heaviest query tiles first
  const int idx = blockIdx.x;
  const int qt = prm.nqt - 1 - idx / prm.nbh;
  const int bh = prm.bh_begin + idx % prm.nbh;
  const int b = bh / prm.NH, h = bh % prm.NH;
  const int ntiles = qt + 1;  // causal: key tiles 0..qt
  const int col0 = h * HD;

  const uint32_t bar0 = sbase + C::OFF_BAR;
  const uint32_t BAR_Q = bar0;
  auto BAR_KF = [&](int s) { return bar0 + 8u * (1 + s); };
  auto BAR_VF = [&](int s) { return bar0 + 8u * (1 + C::STAGES + s); };
  auto BAR_KVE = [&](int s) { return bar0 + 8u * (1 + 2 * C::STAGES + s); };
  auto BAR_SF = [&](int s) { return bar0 + 8u * (1 + 3 * C::STAGES + s); };
  auto BAR_SE = [&](int s) { return bar0 + 8u * (3 + 3 * C::STAGES + s); };
  auto BAR_PF = [&](int s) { return bar0 + 8u * (5 + 3 * C::STAGES + s); };
  auto BAR_PE = [&](int s) { return bar0 + 8u * (5 + 3 * C::STAGES + C::PBUF + s); };
  const uint32_t BAR_O = bar0 + 8u * (5 + 3 * C::STAGES + 2 * C::PBUF);
  const uint32_t tslot = sbase + C::OFF_TSLOT;

  if (threadIdx.x == 0) {
    abort_flag = 0;
    mbar_init(BAR_Q, 1);
    for (int s = 0; s < C::STAGES; ++s) {
      mbar_init(BAR_KF(s), 1);
      mbar_init(BAR_VF(s), 1);
      mbar_init(BAR_KVE(s), 1);
    }
    for (int s = 0; s < 2; ++s) {
      mbar_init(BAR_SF(s), 1);
      mbar_init(BAR_SE(s), 128);
    }
    for (int s = 0; s < C::PBUF; ++s) {
      mbar_init(BAR_PF(s), 128);
      mbar_init(BAR_PE(s), 1);
    }
    mbar_init(BAR_O, 1);
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
    // ------------------------------------------------------ TMA producer
    if (lane == 0) {
      tma_prefetch_desc(&tmQ);
      tma_prefetch_desc(&tmK);
      tma_prefetch_desc(&tmV);
      mbar_arrive_expect_tx(BAR_Q, C::Q_BYTES);
      for (int kb = 0; kb < C::KB; ++kb)
        tma_load_3d(sbase + C::OFF_Q + kb * BM * 128, &tmQ, BAR_Q, col0 + kb * 64, qt * BM, b);
      for (int j = 0; j < ntiles; ++j) {
        const int st = j % C::STAGES;
        if (j >= C::STAGES && !mbar_wait(BAR_KVE(st), ((j - C::STAGES) / C::STAGES) & 1, abort_p))
          break;
        const uint32_t sk = sbase + C::OFF_K + st * C::KV_BYTES;
        const uint32_t sv = sbase + C::OFF_V + st * C::KV_BYTES;
        mbar_arrive_expect_tx(BAR_KF(st), C::KV_BYTES);
        for (int kb = 0; kb < C::KB; ++kb)
          tma_load_3d(sk + kb * BN * 128, &tmK, BAR_KF(st), col0 + kb * 64, j * BN, b);
        mbar_arrive_expect_tx(BAR_VF(st), C::KV_BYTES);
        for (int kb = 0; kb < C::KB; ++kb)
          tma_load_3d(sv + kb * BN * 128, &tmV, BAR_VF(st), col0 + kb * 64, j * BN, b);
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------- MMA
    if (lane == 0) {
      constexpr uint32_t IDESC_S = idesc_bf16_f32(BM, BN, 0, 0);
      constexpr uint32_t IDESC_O = idesc_bf16_f32(BM, HD, 0, 1);
      const uint32_t sq = sbase + C::OFF_Q;
      bool ok = mbar_wait(BAR_Q, 0, abort_p);
      auto issue_s = [&](int j) -> bool {
        const int st = j % C::STAGES, sb = j & 1;
        if (!mbar_wait(BAR_KF(st), (j / C::STAGES) & 1, abort_p)) return false;
        if (j >= 2 && !mbar_wait(BAR_SE(sb), ((j - 2) >> 1) & 1, abort_p)) return false;
        tc_fence_after();
        const uint32_t sk = sbase + C::OFF_K + st * C::KV_BYTES;
#pragma unroll
        for (int kk = 0; kk < HD / 16; ++kk) {
          const uint32_t koff = (kk >> 2) * (BM * 128) + (kk & 3) * 32;
          const uint64_t ad = smem_desc_sw128(sq + koff, 16, 1024);
          const uint64_t bd = smem_desc_sw128(sk + (kk >> 2) * (BN * 128) + (kk & 3) * 32, 16, 1024);
          umma_bf16_ss(tmem + C::TCOL_S + sb * BN, ad, bd, IDESC_S, kk > 0 ? 1u : 0u);
        }
        umma_commit(BAR_SF(sb));
        return true;
      };
      if (ok) ok = issue_s(0);
      for (int j = 0; ok && j < ntiles; ++j) {
        if (j + 1 < ntiles && !issue_s(j + 1)) break;
        const int st = j % C::STAGES, pb = j % C::PBUF;
        if (!mbar_wait(BAR_PF(pb), (j / C::PBUF) & 1, abort_p)) break;
        if (!mbar_wait(BAR_VF(st), (j / C::STAGES) & 1, abort_p)) break;
        tc_fence_after();
        const uint32_t sp = sbase + C::OFF_P + pb * C::P_BYTES;
        const uint32_t sv = sbase + C::OFF_V + st * C::KV_BYTES;
#pragma unroll
        for (int kk = 0; kk < BN / 16; ++kk) {
          const uint64_t ad = smem_desc_sw128(sp + (kk >> 2) * (BM * 128) + (kk & 3) * 32, 16, 1024);
          const uint64_t bd = smem_desc_sw128(sv + kk * 2048, BN * 128, 1024);
          umma_bf16_ss(tmem + C::TCOL_O, ad, bd, IDESC_O, (j > 0 || kk > 0) ? 1u : 0u);
        }
        umma_commit(BAR_KVE(st));
        umma_commit(BAR_PE(pb));
        if (j + 1 == ntiles) umma_commit(BAR_O);
      }
    }
  } else {
    // --------------------------------------------------------- softmax
    const int quarter = warp & 3;                // TMEM lane quarter of this warp
    const int row = quarter * 32 + lane;         // query row within the tile
    const int grow = qt * BM + row;              // query position
    const uint32_t trow = tmem + ((uint32_t)(quarter * 32) << 16);
    const float c = prm.scale_log2;
    float m_used = -INFINITY, l_sum = 0.0f;
    bool ok = true;
    for (int j = 0; j < ntiles; ++j) {
      const int sb = j & 1, pb = j % C::PBUF;
      if (!mbar_wait_warp(BAR_SF(sb), (j >> 1) & 1, abort_p)) { ok = false; break; }
      tc_fence_after();
      float s[BN];
#pragma unroll
      for (int cc = 0; cc < BN; cc += 64) {
        uint32_t ra[32], rb[32];
        tmem_ld32(trow + C::TCOL_S + sb * BN + cc, ra);
        tmem_ld32(trow + C::TCOL_S + sb * BN + cc + 32, rb);
        tmem_wait_ld_dep(ra, rb);
#pragma unroll
        for (int i = 0; i < 32; ++i) {
          s[cc + i] = __uint_as_float(ra[i]);
          s[cc + 32 + i] = __uint_as_float(rb[i]);
        }
      }
      tc_fence_before();
      mbar_arrive(BAR_SE(sb));
      if (j == qt) {  // diagonal tile: mask keys after the query
#pragma unroll
        for (int i = 0; i < BN; ++i)
          if (i > row) s[i] = -INFINITY;
      }
      // row maximum with 8 independent partial maxima (short dependency chains)
      float pm[8];
#pragma unroll
      for (int u = 0; u < 8; ++u) pm[u] = s[u];
#pragma unroll
      for (int i = 8; i < BN; i += 8)
#pragma unroll
        for (int u = 0; u < 8; ++u) pm[u] = fmaxf(pm[u], s[i + u]);
      const float mx = fmaxf(fmaxf(fmaxf(pm[0], pm[1]), fmaxf(pm[2], pm[3])),
                             fmaxf(fmaxf(pm[4], pm[5]), fmaxf(pm[6], pm[7])));
      const float m_new = fmaxf(m_used, mx * c);
      if (j == 0) {
        m_used = m_new;
      } else {
        const bool need = m_new > m_used + RESCALE_THRESHOLD;
        if (__any_sync(0xffffffffu, need)) {
          const float alpha = need ? ex2(m_used - m_new) : 1.0f;
          if (need) {
            l_sum *= alpha;
            m_used = m_new;
          }
          // O must be stable: wait for PV_{j-1}
          const int pp = (j - 1) % C::PBUF;
          if (!mbar_wait_warp(BAR_PE(pp), ((j - 1) / C::PBUF) & 1, abort_p)) { ok = false; break; }
          tc_fence_after();
#pragma unroll
          for (int cc = 0; cc < HD; cc += 16) {
            uint32_t r[16];
            tmem_ld16(trow + C::TCOL_O + cc, r);
            tmem_wait_ld_dep(r);
#pragma unroll
            for (int i = 0; i < 16; ++i) r[i] = __float_as_uint(__uint_as_float(r[i]) * alpha);
            tmem_st16(trow + C::TCOL_O + cc, r);
          }
          tmem_wait_st();
        }
      }
      // P = 2^(S*c - m) with packed fp32x2 FMAs; row sum in 4 packed partials
      const float2 c2 = make_float2(c, c), nm2 = make_float2(-m_used, -m_used);
      float2 ps[4] = {make_float2(0.f, 0.f), make_float2(0.f, 0.f), make_float2(0.f, 0.f),
                      make_float2(0.f, 0.f)};
#pragma unroll
      for (int i = 0; i < BN; i += 2) {
        const float2 t = __ffma2_rn(make_float2(s[i], s[i + 1]), c2, nm2);
        s[i] = ex2(t.x);
        s[i + 1] = ex2(t.y);
        ps[(i >> 1) & 3] = __fadd2_rn(ps[(i >> 1) & 3], make_float2(s[i], s[i + 1]));
      }
      const float rs = (ps[0].x + ps[0].y) + (ps[1].x + ps[1].y) + (ps[2].x + ps[2].y) +
                       (ps[3].x + ps[3].y);
      l_sum += rs;
      if (j >= C::PBUF && !mbar_wait_warp(BAR_PE(pb), ((j - C::PBUF) / C::PBUF) & 1, abort_p)) { ok = false; break; }
      uint8_t* prow = gbase + C::OFF_P + pb * C::P_BYTES;
#pragma unroll
      for (int kb = 0; kb < BN / 64; ++kb) {
#pragma unroll
        for (int ch = 0; ch < 8; ++ch) {
          const int c0 = kb * 64 + ch * 8;
          uint4 v;
          v.x = pack_bf16(s[c0 + 0], s[c0 + 1]);
          v.y = pack_bf16(s[c0 + 2], s[c0 + 3]);
          v.z = pack_bf16(s[c0 + 4], s[c0 + 5]);
          v.w = pack_bf16(s[c0 + 6], s[c0 + 7]);
          *reinterpret_cast<uint4*>(prow + kb * (BM * 128) + row * 128 + ((ch ^ (row & 7)) * 16)) = v;
        }
      }
      fence_proxy_async_smem();
      tc_fence_before();
      mbar_arrive(BAR_PF(pb));
    }
    // ------------------------------------------------------- epilogue
    const bool epi = ok && mbar_wait_warp(BAR_O, 0, abort_p);
    if (epi) {
      tc_fence_after();
      const float inv = 1.0f / l_sum;
      // stage O (bf16) in the P buffer 0 region, laid out like a TMA box
      uint8_t* ostage = gbase + C::OFF_P;
#pragma unroll
      for (int cc = 0; cc < HD; cc += 16) {
        uint32_t r[16];
        tmem_ld16(trow + C::TCOL_O + cc, r);
        tmem_wait_ld_dep(r);
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
        uint8_t* blk = ostage + kb * (BM * 128) + row * 128;
        *reinterpret_cast<uint4*>(blk + ((ch ^ (row & 7)) * 16)) = v0;
        *reinterpret_cast<uint4*>(blk + (((ch + 1) ^ (row & 7)) * 16)) = v1;
      }
      fence_proxy_async_smem();
      if (grow < prm.T)
        prm.lse[((long long)b * prm.T + grow) * prm.NH + h] = (m_used + log2f(l_sum)) * LN2;
    }
    // every softmax thread reaches this barrier, whatever happened before
    asm volatile("bar.sync 1, 128;" ::: "memory");
    if (epi && warp == 2 && lane == 0) {
      for (int kb = 0; kb < C::KB; ++kb)
        tma_store_3d(&tmO, sbase + C::OFF_P + kb * BM * 128, col0 + kb * 64, qt * BM, b);
      bulk_commit();
      bulk_wait<0>();
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, C::TMEM_COLS);
  }
  if (threadIdx.x == 0 && abort_flag) atomicOr(prm.status, STATUS_FWD_TIMEOUT);
}

template <int HD>
cudaError_t launch_fwd(const __nv_bfloat16* q, const __nv_bfloat16* k, const __nv_bfloat16* v,
                       __nv_bfloat16* out, float* lse, const AttnShape& s, uint32_t* status,
                       cudaStream_t st) {
  using C = FwdCfg<HD>;
  CUtensorMap tq, tk, tv, to;
  const CUtensorMapDataType bf = CU_TENSOR_MAP_DATA_TYPE_BFLOAT16;
  const CUtensorMapSwizzle sw = CU_TENSOR_MAP_SWIZZLE_128B;
  if (!make_tmap_3d(&tq, q, bf, 2, s.N, s.T, s.B, 64, BM, sw) ||
      !make_tmap_3d(&tk, k, bf, 2, s.N, s.T, s.B, 64, BN, sw) ||
      !make_tmap_3d(&tv, v, bf, 2, s.N, s.T, s.B, 64, BN, sw) ||
      !make_tmap_3d(&to, out, bf, 2, s.N, s.T, s.B, 64, BM, sw))
    return cudaErrorInvalidValue;
  FwdParams prm;
  prm.T = s.T;
  prm.N = s.N;
  prm.NH = s.NH;
  prm.bh_begin = s.bh_begin;
  prm.nbh = s.bh_end - s.bh_begin;
  prm.nqt = (s.T + BM - 1) / BM;
  prm.scale_log2 = LOG2E / sqrtf((float)HD);
  prm.lse = lse;
  prm.status = status;
  cudaError_t e = cudaFuncSetAttribute(flash_fwd_kernel<HD>,
                                       cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM_BYTES);
  if (e != cudaSuccess) return e;
  const long long nblocks = (long long)prm.nqt * prm.nbh;
  flash_fwd_kernel<HD><<<(unsigned)nblocks, NUM_THREADS, C::SMEM_BYTES, st>>>(tq, tk, tv, to, prm);
  count_launches(1);
  return cudaGetLastError();
}

}  // namespace

cudaError_t launch_flash_fwd(const __nv_bfloat16* q, const __nv_bfloat16* k,
                             const __nv_bfloat16* v, __nv_bfloat16* out, float* lse,
                             const AttnShape& s, uint32_t* status, cudaStream_t st) {
  if (s.bh_end <= s.bh_begin) return cudaSuccess;
  return s.D == 64 ? launch_fwd<64>(q, k, v, out, lse, s, status, st)
                   : launch_fwd<128>(q, k, v, out, lse, s, status, st);
}

}  // namespace ma
