// gemm_sm100.cu -- the GEMMs around attention (attention.metal:301-455) on
// sm_100a with tcgen05 UMMA, TMEM accumulators and TMA:
//   projForward     out   = attnOut . Wp                 (attention.metal:395-416)
//   projBackwarddX  dAttn = dZ . Wp^T                    (attention.metal:432-455)
//   projBackwarddW  dWp   = attnOut^T . dZ               (attention.metal:418-430)
//   computeGradDx   dX    = dQ.Wq^T + dK.Wk^T + dV.Wv^T  (attention.metal:301-342)
//   computeGradDw   dWq, dWk, dWv = X^T.dQ, X^T.dK, X^T.dV (attention.metal:344-393)
// Rows of the activations are B*M (all sequences of the batch), so the weight
// gradients sum over every row, as the reference's accumulate into buffers
// zeroed once per step does (model.h:549-556).
//
// One kernel: C (128 x BN tile per CTA) = sum over "segments" of A_s . B_s,
// K swept in steps of 64.  A is K-major ([rows of C][K]) or MN-major
// ([K][rows of C]); B is K-major ([cols of C][K]) or MN-major ([K][cols of
// C]); both arrive by TMA into a ring of 128-byte-swizzled stages.  The
// segments accumulate into one TMEM accumulator (computeGradDx's three
// products, as the reference's three runs into one dX tile,
// attention.metal:338-340); independent products (computeGradDw) are grid.z.
// dQ is fp32 in the reference; an fp32 operand is loaded as fp32 and
// converted to bf16 in shared memory by the epilogue warps, which are idle
// during the main loop (the UMMA takes bf16 x bf16 -> fp32).
//
// Roles (192 threads): warp 0 TMA producer, warp 1 TMEM owner + UMMA issuer,
// warps 2-5 fp32->bf16 converter during the main loop, then the epilogue
// (TMEM -> bf16 or fp32 -> smem -> TMA store; rows/cols past the matrix are
// clipped).  All mbarrier waits are bounded; on time-out the CTA winds down
// and sets STATUS_GEMM_TIMEOUT.
#include <cstring>

#include "common.cuh"
#include "sm100.cuh"
#include "tmap.h"

namespace ma {
namespace {

using namespace sm100;

constexpr int BM = 128;
constexpr int BK = 64;
constexpr int NUM_THREADS = 192;

// Tensor maps and flags of one launch.  a[i] / b[i] for i < na / nb; the
// operand of step s is a[na > 1 ? seg : 0], b[nb > 1 ? seg : (nz > 1 ? z : 0)].
struct GemmMaps {
  CUtensorMap a[3];
  CUtensorMap b[3];
  CUtensorMap c[3];
};

struct GemmArgs {
  int M, N, K;        // C is M x N per output; each segment contracts K
  int nseg;           // segments accumulated into one output
  int na, nb;         // number of distinct A / B maps
  uint32_t a_f32;     // bit i: a[i] is fp32 (converted to bf16 on chip)
  uint32_t b_f32;
  uint32_t c_f32;     // bit z: output z is fp32 (else bf16)
  int ksplit;         // split-K: grid.z = outputs * ksplit; partials are added (fp32 outputs)
  int kchunk;         // K steps per split
  // fused computeD (FUSE_D): D[row][h] = bf16(sum over head h's columns of
  // bf16(C) * O), O [M][N] bf16, D [M][N / head_dim] bf16
  const __nv_bfloat16* o_in;
  __nv_bfloat16* d_out;
  int head_dim;
  // ReLU epilogue (ACT 1): mask [M][N] uint8 written, 1 where the rounded
  // output is > 0 (mlp.metal:45-51); mask-multiply epilogue (ACT 2): the
  // rounded output is zeroed where the mask is 0; residual epilogue (ACT 3):
  // C = bf16(res + bf16(A . B)), res [M][N] bf16 (elementwise.metal's
  // residualAdd after the GEMM)
  uint8_t* mask;
  const __nv_bfloat16* res;
  uint32_t* status;
};

template <int BN, bool HAS_F32>
struct GemmCfg {
  static constexpr uint32_t A_BYTES = BM * BK * 2;             // 16 KB
  static constexpr uint32_t B_BYTES = BN * BK * 2;             // 8 / 16 KB
  static constexpr uint32_t F32_BYTES = HAS_F32 ? 2 * (BM > BN ? BM : BN) * 128 : 0;  // 32 KB
  static constexpr uint32_t STAGE_BYTES = A_BYTES + B_BYTES + F32_BYTES;
  // three stages leave room for two CTAs per SM at BN = 128 (32 KB stages)
  // and three at BN = 64 (24 KB), so one CTA's epilogue overlaps another's
  // main loop
  static constexpr int STAGES = 3;
  static constexpr uint32_t OFF_BAR = STAGES * STAGE_BYTES;
  // full[S], empty[S], converted[S], done
  static constexpr uint32_t OFF_TSLOT = OFF_BAR + (3 * STAGES + 1) * 8;
  static constexpr uint32_t SMEM_BYTES = OFF_TSLOT + 16 + 1024;
  static constexpr uint32_t OUT_BYTES = BM * BN * 4;  // epilogue staging, fp32 worst case
  static_assert(OUT_BYTES <= STAGES * STAGE_BYTES, "epilogue staging must fit in the ring");
  static_assert(SMEM_BYTES <= 232448, "shared memory");
};

__device__ __forceinline__ int bit_of(uint32_t m, int i) { return (m >> i) & 1u; }

// bf16(float(a) + float(b)) elementwise over 8 bf16 values (round to nearest even)
__device__ __forceinline__ uint4 add_bf16x8(uint4 a, uint4 b) {
  const __nv_bfloat162* x = reinterpret_cast<const __nv_bfloat162*>(&a);
  const __nv_bfloat162* y = reinterpret_cast<const __nv_bfloat162*>(&b);
  uint4 r;
  __nv_bfloat162* o = reinterpret_cast<__nv_bfloat162*>(&r);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float2 fx = __bfloat1622float2(x[i]), fy = __bfloat1622float2(y[i]);
    o[i] = __floats2bfloat162_rn(fy.x + fx.x, fy.y + fx.y);
  }
  return r;
}

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

template <int BN, bool A_MN, bool B_MN, bool HAS_F32, bool FUSE_D = false, int ACT = 0>
__global__ void __launch_bounds__(NUM_THREADS, 1)
    gemm_kernel(const __grid_constant__ GemmMaps maps, const GemmArgs args) {
  pdl_wait_and_release();
  using C = GemmCfg<BN, HAS_F32>;
  extern __shared__ uint8_t smem_raw[];
  __shared__ int abort_flag;
  const uint32_t raw = smem_u32(smem_raw);
  const uint32_t sbase = (raw + 1023u) & ~1023u;
  uint8_t* gbase = smem_raw + (sbase - raw);
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const int row0 = blockIdx.x * BM, col0 = blockIdx.y * BN;
  const int z = blockIdx.z / args.ksplit, kz = blockIdx.z % args.ksplit;
  // split-K: this CTA sweeps K steps [kbeg, kbeg + nk) of its output (nseg == 1)
  const int nk_all = (args.K + BK - 1) / BK;
  const int kbeg = kz * args.kchunk;
  const int nk = args.ksplit > 1 ? min(args.kchunk, nk_all - kbeg) : nk_all;
  const int nsteps = args.nseg * nk;

  const uint32_t bar0 = sbase + C::OFF_BAR;
  auto BAR_F = [&](int s) { return bar0 + 8u * s; };
  auto BAR_E = [&](int s) { return bar0 + 8u * (C::STAGES + s); };
  auto BAR_C = [&](int s) { return bar0 + 8u * (2 * C::STAGES + s); };
  const uint32_t BAR_DONE = bar0 + 8u * (3 * C::STAGES);
  const uint32_t tslot = sbase + C::OFF_TSLOT;
  if (threadIdx.x == 0) {
    abort_flag = 0;
    for (int s = 0; s < C::STAGES; ++s) {
      mbar_init(BAR_F(s), 1);
      mbar_init(BAR_E(s), 1);
      mbar_init(BAR_C(s), 128);
    }
    mbar_init(BAR_DONE, 1);
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc(tslot, BN);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *reinterpret_cast<volatile uint32_t*>(gbase + C::OFF_TSLOT);
  volatile int* abort_p = &abort_flag;

  // operand maps of step s
  auto a_index = [&](int s) { return args.na > 1 ? s / nk : 0; };
  auto b_index = [&](int s) { return args.nb > 1 ? (args.nseg > 1 ? s / nk : z) : 0; };
  auto step_f32 = [&](int s) {
    return HAS_F32 && (bit_of(args.a_f32, a_index(s)) || bit_of(args.b_f32, b_index(s)));
  };

  if (warp == 0) {
    if (lane == 0) {
      // ------------------------------------------------------ TMA producer
      for (int s = 0; s < nsteps; ++s) {
        const int st = s % C::STAGES;
        if (s >= C::STAGES && !mbar_wait(BAR_E(st), ((s / C::STAGES) - 1) & 1, abort_p)) break;
        const int ai = a_index(s), bi = b_index(s), k0 = (kbeg * (args.ksplit > 1) + s % nk) * BK;
        const bool af = HAS_F32 && bit_of(args.a_f32, ai), bf = HAS_F32 && bit_of(args.b_f32, bi);
        const uint32_t sa = sbase + st * C::STAGE_BYTES;
        const uint32_t sb = sa + C::A_BYTES;
        const uint32_t sf = sb + C::B_BYTES;  // fp32 staging
        mbar_arrive_expect_tx(BAR_F(st), (af ? 2 : 1) * C::A_BYTES + (bf ? 2 : 1) * C::B_BYTES);
        const CUtensorMap* am = &maps.a[ai];
        const CUtensorMap* bm = &maps.b[bi];
        if (!A_MN) {  // [rows][K]: box {64 K, 128 rows} (fp32: two {32, 128})
          if (af) {
            tma_load_2d(sf, am, BAR_F(st), k0, row0);
            tma_load_2d(sf + BM * 128, am, BAR_F(st), k0 + 32, row0);
          } else {
            tma_load_2d(sa, am, BAR_F(st), k0, row0);
          }
        } else {      // [K][rows]: boxes {64 rows, 64 K} (fp32: {32 rows, 64 K})
          if (af) {
            for (int j = 0; j < BM / 32; ++j) tma_load_2d(sf + j * (BK * 128), am, BAR_F(st), row0 + 32 * j, k0);
          } else {
            for (int j = 0; j < BM / 64; ++j) tma_load_2d(sa + j * (BK * 128), am, BAR_F(st), row0 + 64 * j, k0);
          }
        }
        if (!B_MN) {  // [cols][K]: box {64 K, BN cols} (fp32: two {32, BN})
          if (bf) {
            tma_load_2d(sf, bm, BAR_F(st), k0, col0);
            tma_load_2d(sf + BN * 128, bm, BAR_F(st), k0 + 32, col0);
          } else {
            tma_load_2d(sb, bm, BAR_F(st), k0, col0);
          }
        } else {      // [K][cols]: boxes {64 cols, 64 K} (fp32: {32 cols, 64 K})
          if (bf) {
            for (int j = 0; j < BN / 32; ++j) tma_load_2d(sf + j * (BK * 128), bm, BAR_F(st), col0 + 32 * j, k0);
          } else {
            for (int j = 0; j < BN / 64; ++j) tma_load_2d(sb + j * (BK * 128), bm, BAR_F(st), col0 + 64 * j, k0);
          }
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      // ------------------------------------------------------------- UMMA
      constexpr uint32_t IDESC = idesc_bf16_f32(BM, BN, A_MN ? 1 : 0, B_MN ? 1 : 0);
      for (int s = 0; s < nsteps; ++s) {
        const int st = s % C::STAGES;
        const uint32_t ph = (s / C::STAGES) & 1;
        // conversion barriers complete only on fp32 steps, which come first
        // in a CTA's step sequence (checked on the host), so (s / STAGES)
        // also counts their phases
        if (!mbar_wait(step_f32(s) ? BAR_C(st) : BAR_F(st), ph, abort_p)) break;
        tc_fence_after();
        const uint32_t sa = sbase + st * C::STAGE_BYTES;
        const uint32_t sb = sa + C::A_BYTES;
#pragma unroll
        for (int kk = 0; kk < BK / 16; ++kk) {
          const uint64_t ad = A_MN ? smem_desc_sw128(sa + kk * 2048, BK * 128, 1024)
                                   : smem_desc_sw128(sa + kk * 32, 16, 1024);
          const uint64_t bd = B_MN ? smem_desc_sw128(sb + kk * 2048, BK * 128, 1024)
                                   : smem_desc_sw128(sb + kk * 32, 16, 1024);
          umma_bf16_ss(tmem, ad, bd, IDESC, (s > 0 || kk > 0) ? 1u : 0u);
        }
        umma_commit(BAR_E(st));
        if (s + 1 == nsteps) umma_commit(BAR_DONE);
      }
    }
  } else {
    // ------------------------------------------ fp32 -> bf16 conversion
    const int t = threadIdx.x - 64;  // 0..127
    bool ok = true;
    if (HAS_F32) {
      for (int s = 0; ok && s < nsteps; ++s) {
        if (!step_f32(s)) continue;
        const int st = s % C::STAGES;
        ok = mbar_wait_warp(BAR_F(st), (s / C::STAGES) & 1, abort_p);
        if (!ok) break;
        uint8_t* sa = gbase + st * C::STAGE_BYTES;
        uint8_t* sb = sa + C::A_BYTES;
        const uint8_t* sf = sb + C::B_BYTES;
        const bool af = bit_of(args.a_f32, a_index(s));
        // one 64-value row of a 128-byte-swizzled tile per thread:
        // src = two fp32 rows (32 values each), dst = one bf16 row
        auto convert_row = [&](const uint8_t* src0, const uint8_t* src1, int srow, uint8_t* dst, int drow) {
#pragma unroll
          for (int ch = 0; ch < 8; ++ch) {  // destination 16-byte chunk = 8 bf16
            const uint8_t* src = ch < 4 ? src0 : src1;
            const int c0 = (ch % 4) * 2;      // two source chunks of 4 fp32
            const float4 x = *reinterpret_cast<const float4*>(src + srow * 128 + (((c0) ^ (srow & 7)) * 16));
            const float4 y = *reinterpret_cast<const float4*>(src + srow * 128 + (((c0 + 1) ^ (srow & 7)) * 16));
            uint4 w;
            w.x = pack_bf16(x.x, x.y);
            w.y = pack_bf16(x.z, x.w);
            w.z = pack_bf16(y.x, y.y);
            w.w = pack_bf16(y.z, y.w);
            *reinterpret_cast<uint4*>(dst + drow * 128 + ((ch ^ (drow & 7)) * 16)) = w;
          }
        };
        if (af) {
          if (!A_MN) {  // K-major [128 rows][64 K]: row t from the two 32-wide fp32 boxes
            convert_row(sf, sf + BM * 128, t, sa, t);
          } else {      // MN-major [64 K][128 rows]: K row t%64 of row block t/64
            const int k = t % 64, blk = t / 64;
            convert_row(sf + (2 * blk) * (BK * 128), sf + (2 * blk + 1) * (BK * 128), k,
                        sa + blk * (BK * 128), k);
          }
        } else {
          if (!B_MN) {  // K-major [BN cols][64 K]
            if (t < BN) convert_row(sf, sf + BN * 128, t, sb, t);
          } else {      // MN-major [64 K][BN cols]
            const int k = t % 64, blk = t / 64;
            if (blk < BN / 64)
              convert_row(sf + (2 * blk) * (BK * 128), sf + (2 * blk + 1) * (BK * 128), k,
                          sb + blk * (BK * 128), k);
          }
        }
        fence_proxy_async_smem();
        mbar_arrive(BAR_C(st));
      }
    }
    // ------------------------------------------------------------ epilogue
    const int quarter = warp & 3;
    const int row = quarter * 32 + lane;
    const uint32_t trow = tmem + ((uint32_t)(quarter * 32) << 16);
    const bool leader = (warp == 2 && lane == 0);
    if (ok) ok = mbar_wait_warp(BAR_DONE, 0, abort_p);
    ok = bar_red_and(1, 128, ok);
    const bool out_f32 = (args.c_f32 >> z) & 1u;
    const int grow = row0 + row;
    float dsum = 0.0f;  // FUSE_D: this row's partial dot for the current head
    if (ok) {
      // the row's residual / mask / O slice, loaded in one burst before the
      // accumulator is read (one memory round trip instead of one per chunk)
      constexpr int NPF = (ACT == 3 || FUSE_D) ? BN / 8 : (ACT == 2 ? BN / 16 : 1);
      uint4 pf[NPF];
      if constexpr (ACT == 3 || ACT == 2 || FUSE_D) {
        if (grow < args.M) {
          const uint4* src = ACT == 3   ? reinterpret_cast<const uint4*>(args.res + (size_t)grow * args.N + col0)
                             : FUSE_D ? reinterpret_cast<const uint4*>(args.o_in + (size_t)grow * args.N + col0)
                                      : reinterpret_cast<const uint4*>(args.mask + (size_t)grow * args.N + col0);
#pragma unroll
          for (int i = 0; i < NPF; ++i) pf[i] = __ldg(src + i);
        }
      }
      tc_fence_after();
      uint8_t* stage = gbase;  // the ring is idle now
#pragma unroll
      for (int cc = 0; cc < BN; cc += 16) {
        uint32_t r[16];
        tmem_ld16(trow + cc, r);
        tmem_wait_ld_dep(r);
        if (out_f32) {  // boxes of 32 fp32 columns: [BN/32][128 rows][128 B]
          uint8_t* rowp = stage + (cc / 32) * (BM * 128) + row * 128;
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            const int ch = (cc % 32) / 4 + q;
            *reinterpret_cast<uint4*>(rowp + ((ch ^ (row & 7)) * 16)) =
                make_uint4(r[4 * q], r[4 * q + 1], r[4 * q + 2], r[4 * q + 3]);
          }
        } else {        // boxes of 64 bf16 columns: [BN/64][128 rows][128 B]
          uint8_t* rowp = stage + (cc / 64) * (BM * 128) + row * 128;
          uint4 v0, v1;
          v0.x = pack_bf16(__uint_as_float(r[0]), __uint_as_float(r[1]));
          v0.y = pack_bf16(__uint_as_float(r[2]), __uint_as_float(r[3]));
          v0.z = pack_bf16(__uint_as_float(r[4]), __uint_as_float(r[5]));
          v0.w = pack_bf16(__uint_as_float(r[6]), __uint_as_float(r[7]));
          v1.x = pack_bf16(__uint_as_float(r[8]), __uint_as_float(r[9]));
          v1.y = pack_bf16(__uint_as_float(r[10]), __uint_as_float(r[11]));
          v1.z = pack_bf16(__uint_as_float(r[12]), __uint_as_float(r[13]));
          v1.w = pack_bf16(__uint_as_float(r[14]), __uint_as_float(r[15]));
          if constexpr (ACT == 3) {  // residual add on the rounded values
            if (grow < args.M) {
              v0 = add_bf16x8(v0, pf[cc / 8]);
              v1 = add_bf16x8(v1, pf[cc / 8 + 1]);
            }
          }
          if constexpr (ACT == 1 || ACT == 2) {  // on the rounded values, as the separate kernels do
            if (grow < args.M) {
              uint8_t* mp = args.mask + (size_t)grow * args.N + col0 + cc;
              uint4 mk = ACT == 2 ? pf[ACT == 2 ? cc / 16 : 0] : make_uint4(0, 0, 0, 0);
              uint32_t* w = reinterpret_cast<uint32_t*>(&v0);  // v0, v1: 8 words, 16 values
              uint32_t* wb = reinterpret_cast<uint32_t*>(&v1);
              uint8_t* mb = reinterpret_cast<uint8_t*>(&mk);
#pragma unroll
              for (int j = 0; j < 16; ++j) {
                uint32_t& word = j < 8 ? w[j / 2] : wb[(j - 8) / 2];
                const int sh = 16 * (j & 1);
                const uint32_t h = (word >> sh) & 0xFFFFu;
                // ACT 1: x > 0 (not negative, not zero, not NaN); ACT 2: mask set
                const bool on = ACT == 1 ? (!(h & 0x8000u) && (h & 0x7FFFu) != 0 && (h & 0x7FFFu) <= 0x7F80u)
                                         : mb[j] != 0;
                if (!on) word &= ~(0xFFFFu << sh);
                if (ACT == 1) mb[j] = on ? 1 : 0;
              }
              if (ACT == 1) *reinterpret_cast<uint4*>(mp) = mk;
            }
          }
          const int ch = (cc % 64) / 8;
          *reinterpret_cast<uint4*>(rowp + ((ch ^ (row & 7)) * 16)) = v0;
          *reinterpret_cast<uint4*>(rowp + (((ch + 1) ^ (row & 7)) * 16)) = v1;
          if constexpr (FUSE_D) {  // D from the rounded bf16 values, as computeD reads them
            if (grow < args.M) {
              dsum += dot_bf16x8(v0, pf[cc / 8]) + dot_bf16x8(v1, pf[cc / 8 + 1]);
              if ((col0 + cc + 16) % args.head_dim == 0) {
                const int nh = args.N / args.head_dim;
                args.d_out[(size_t)grow * nh + (col0 + cc) / args.head_dim] = __float2bfloat16_rn(dsum);
                dsum = 0.0f;
              }
            }
          }
        }
      }
      fence_proxy_async_smem();
    }
    ok = bar_red_and(1, 128, ok);
    if (ok && leader) {
      const CUtensorMap* cm = &maps.c[z];
      if (args.ksplit > 1) {  // fp32 partial sums added into the (zeroed) output
        for (int b = 0; b < BN / 32; ++b) tma_reduce_add_2d(cm, sbase + b * (BM * 128), col0 + 32 * b, row0);
      } else if (out_f32) {
        for (int b = 0; b < BN / 32; ++b) tma_store_2d(cm, sbase + b * (BM * 128), col0 + 32 * b, row0);
      } else {
        for (int b = 0; b < BN / 64; ++b) tma_store_2d(cm, sbase + b * (BM * 128), col0 + 64 * b, row0);
      }
      bulk_commit();
      bulk_wait<0>();
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, BN);
  }
  if (threadIdx.x == 0 && abort_flag) atomicOr(args.status, STATUS_GEMM_TIMEOUT);
}

// ------------------------------------------------------------------ host
enum Major { K_MAJOR = 0, MN_MAJOR = 1 };

// One operand: a row-major matrix in global memory.  For a K-major operand it
// is [outer][K] (outer = rows of C for A, cols of C for B); for an MN-major
// one it is [K][outer].  `f32` selects fp32 elements (else bf16).
struct Operand {
  const void* ptr;
  bool f32;
};

bool make_operand_map(CUtensorMap* m, const Operand& o, bool mn_major, uint64_t outer, uint64_t K,
                      uint32_t box_outer) {
  const CUtensorMapDataType t = o.f32 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16;
  const uint32_t eb = o.f32 ? 4 : 2, inner_box = o.f32 ? 32 : 64;
  const CUtensorMapSwizzle sw = CU_TENSOR_MAP_SWIZZLE_128B;
  if (!mn_major) return make_tmap_2d(m, o.ptr, t, eb, K, outer, inner_box, box_outer, sw);
  return make_tmap_2d(m, o.ptr, t, eb, outer, K, inner_box, BK, sw);
}

template <int BN, bool A_MN, bool B_MN, bool HAS_F32, bool FUSE_D = false, int ACT = 0>
cudaError_t run_gemm(const Operand* A, int na, const Operand* Bop, int nb, void* const* Cptr,
                     const bool* c_f32, int nz, int nseg, int M, int N, int K, uint32_t* status,
                     cudaStream_t st, int ksplit = 1, const __nv_bfloat16* o_in = nullptr,
                     __nv_bfloat16* d_out = nullptr, int head_dim = 0, uint8_t* mask = nullptr,
                     const __nv_bfloat16* res = nullptr) {
  using Cfg = GemmCfg<BN, HAS_F32>;
  GemmMaps maps;
  memset(&maps, 0, sizeof(maps));
  GemmArgs args{};
  args.M = M;
  args.N = N;
  args.K = K;
  args.nseg = nseg;
  args.na = na;
  args.nb = nb;
  args.status = status;
  args.o_in = o_in;
  args.d_out = d_out;
  args.head_dim = head_dim;
  args.mask = mask;
  args.res = res;
  if (ACT == 3 && (!res || nz != 1 || c_f32[0] || ksplit > 1 || N % 16 || (reinterpret_cast<uintptr_t>(res) & 15)))
    return cudaErrorInvalidValue;
  if ((ACT == 1 || ACT == 2) && (!mask || nz != 1 || c_f32[0] || ksplit > 1 || N % 16 || (reinterpret_cast<uintptr_t>(mask) & 15)))
    return cudaErrorInvalidValue;
  if (FUSE_D && (!o_in || !d_out || head_dim <= 0 || BN % 16 || N % head_dim || head_dim % 16 ||
                 nz != 1 || c_f32[0]))
    return cudaErrorInvalidValue;
  // split-K only for single-segment products with fp32 outputs (the partial
  // sums are added by TMA reductions into outputs the caller has zeroed)
  const int nk_all = (K + BK - 1) / BK;
  if (ksplit < 1 || nseg > 1) ksplit = 1;
  if (ksplit > nk_all) ksplit = nk_all;
  args.kchunk = (nk_all + ksplit - 1) / ksplit;
  args.ksplit = (nk_all + args.kchunk - 1) / args.kchunk;
  if (args.ksplit > 1)
    for (int i = 0; i < nz; ++i)
      if (!c_f32[i]) return cudaErrorInvalidValue;
  for (int i = 0; i < na; ++i) {
    if (A[i].f32) args.a_f32 |= 1u << i;
    if (!make_operand_map(&maps.a[i], A[i], A_MN, M, K, BM)) return cudaErrorInvalidValue;
  }
  for (int i = 0; i < nb; ++i) {
    if (Bop[i].f32) args.b_f32 |= 1u << i;
    if (!make_operand_map(&maps.b[i], Bop[i], B_MN, N, K, BN)) return cudaErrorInvalidValue;
  }
  if ((args.a_f32 | args.b_f32) && !HAS_F32) return cudaErrorInvalidValue;
  // The UMMA issuer waits for stage s's conversion with parity (s / STAGES):
  // that is right only when a CTA's fp32 steps come first (segment 0 of a
  // sum, or every step of a product).
  if (nseg > 1 && (args.b_f32 | (args.a_f32 & ~1u))) return cudaErrorInvalidValue;
  for (int i = 0; i < nz; ++i) {
    if (c_f32[i]) args.c_f32 |= 1u << i;
    const bool ok = c_f32[i]
                        ? make_tmap_2d(&maps.c[i], Cptr[i], CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, N, M, 32, BM,
                                       CU_TENSOR_MAP_SWIZZLE_128B)
                        : make_tmap_2d(&maps.c[i], Cptr[i], CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, N, M, 64, BM,
                                       CU_TENSOR_MAP_SWIZZLE_128B);
    if (!ok) return cudaErrorInvalidValue;
  }
  auto kern = gemm_kernel<BN, A_MN, B_MN, HAS_F32, FUSE_D, ACT>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, Cfg::SMEM_BYTES);
  if (e != cudaSuccess) return e;
  const dim3 grid((M + BM - 1) / BM, (N + BN - 1) / BN, nz * args.ksplit);
  launch_pdl(kern, grid, NUM_THREADS, Cfg::SMEM_BYTES, st, maps, args);
  count_launches(1);
  return cudaGetLastError();
}

}  // namespace

// Generic bf16 GEMM C[M][N] = A . B (bf16 out, fp32 accumulation) for the
// training step's matmuls (mlp.metal, linear.metal): A is [M][K] (K-major) or
// [K][M] (a_mn); B is [N][K] (K-major) or [K][N] (b_mn).  64-wide column
// tiles when 128-wide ones would leave most SMs idle.
cudaError_t launch_gemm_bf16(const __nv_bfloat16* A, bool a_mn, const __nv_bfloat16* B, bool b_mn,
                             __nv_bfloat16* C, int M, int N, int K, uint32_t* status, cudaStream_t st) {
  const Operand a{A, false}, b{B, false};
  void* c[1] = {C};
  const bool cf[1] = {false};
  const bool wide = (long long)((M + 127) / 128) * ((N + 127) / 128) >= 148;
#define MA_GEMM_CASE(BN_, AM, BMN)                                                               \
  if (a_mn == AM && b_mn == BMN)                                                                 \
    return run_gemm<BN_, AM, BMN, false>(&a, 1, &b, 1, c, cf, 1, 1, M, N, K, status, st);
  if (wide) {
    MA_GEMM_CASE(128, false, false)
    MA_GEMM_CASE(128, false, true)
    MA_GEMM_CASE(128, true, true)
  } else {
    MA_GEMM_CASE(64, false, false)
    MA_GEMM_CASE(64, false, true)
    MA_GEMM_CASE(64, true, true)
  }
#undef MA_GEMM_CASE
  return cudaErrorInvalidValue;  // A MN-major with B K-major is not needed
}

// The training step's MLP GEMMs with their element-wise step in the epilogue
// (A K-major): act = 1, C = relu(A . B) and mask = (C > 0) (mlp.metal:45-51,
// B MN-major); act = 2, C = (A . B) where mask is set, else 0 (the backward's
// mask multiply, B K-major); act = 3, C = res + A . B (the residual add after
// projForward / mlpForwardTwo, B MN-major).  Same values as launch_gemm_bf16
// followed by the separate element-wise kernels.
cudaError_t launch_gemm_bf16_act(const __nv_bfloat16* A, const __nv_bfloat16* B, bool b_mn, __nv_bfloat16* C,
                                 uint8_t* mask, const __nv_bfloat16* res, int act, int M, int N, int K,
                                 uint32_t* status, cudaStream_t st) {
  const Operand a{A, false}, b{B, false};
  void* c[1] = {C};
  const bool cf[1] = {false};
  const bool wide = (long long)((M + 127) / 128) * ((N + 127) / 128) >= 148;
#define MA_GEMM_ACT(BN_, BMN, ACT_)                                                                         \
  if (b_mn == BMN && act == ACT_)                                                                          \
    return run_gemm<BN_, false, BMN, false, false, ACT_>(&a, 1, &b, 1, c, cf, 1, 1, M, N, K, status, st, 1, \
                                                         nullptr, nullptr, 0, mask, res);
  if (wide) {
    MA_GEMM_ACT(128, true, 1)
    MA_GEMM_ACT(128, false, 2)
    MA_GEMM_ACT(128, true, 3)
  } else {
    MA_GEMM_ACT(64, true, 1)
    MA_GEMM_ACT(64, false, 2)
    MA_GEMM_ACT(64, true, 3)
  }
#undef MA_GEMM_ACT
  return cudaErrorInvalidValue;
}

// Split-K GEMM into an fp32 output (zeroed here): C[M][N] = A . B with both
// operands MN-major ([K][M], [K][N]); used for weight gradients, whose K (the
// B*T activation rows) is long and whose M x N is small.  As many K chunks
// as fill the co-resident CTA slots (ctas_per_sm per SM) in one wave, never
// more: a grid just past the slots would run a nearly empty second wave.
int pick_ksplit(int tiles, int K, int ctas_per_sm) {
  int dev = 0, sms = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const int nk = (K + BK - 1) / BK;
  int s = (sms * ctas_per_sm) / tiles;
  if (s > nk / 4) s = nk / 4;  // at least 4 K steps per chunk
  return s < 1 ? 1 : s;
}

cudaError_t launch_gemm_splitk_f32(const __nv_bfloat16* A, const __nv_bfloat16* B, float* C, int M, int N,
                                   int K, uint32_t* status, cudaStream_t st, bool zero) {
  if (zero) {
    cudaError_t e = cudaMemsetAsync(C, 0, (size_t)M * N * sizeof(float), st);
    if (e != cudaSuccess) return e;
  }
  const Operand a{A, false}, b{B, false};
  void* c[1] = {C};
  const bool cf[1] = {true};
  if (N % 128 == 0) {  // 128-wide tiles: fewer operand re-reads, N = 128 UMMAs
    const int tiles = ((M + 127) / 128) * (N / 128);
    return run_gemm<128, true, true, false>(&a, 1, &b, 1, c, cf, 1, 1, M, N, K, status, st,
                                            pick_ksplit(tiles, K, 2));
  }
  const int tiles = ((M + 127) / 128) * ((N + 63) / 64);
  return run_gemm<64, true, true, false>(&a, 1, &b, 1, c, cf, 1, 1, M, N, K, status, st,
                                         pick_ksplit(tiles, K, 3));
}

// rows = B*M activations rows, n = N (= NH*D)
cudaError_t launch_proj_forward(const __nv_bfloat16* attn, const __nv_bfloat16* w, __nv_bfloat16* out,
                                int rows, int n, uint32_t* status, cudaStream_t st) {
  const Operand a{attn, false}, b{w, false};
  void* c[1] = {out};
  const bool cf[1] = {false};
  return run_gemm<128, false, true, false>(&a, 1, &b, 1, c, cf, 1, 1, rows, n, n, status, st);
}

cudaError_t launch_proj_backward_dx(const __nv_bfloat16* dz, const __nv_bfloat16* w, __nv_bfloat16* dattn,
                                    int rows, int n, uint32_t* status, cudaStream_t st) {
  const Operand a{dz, false}, b{w, false};
  void* c[1] = {dattn};
  const bool cf[1] = {false};
  return run_gemm<128, false, false, false>(&a, 1, &b, 1, c, cf, 1, 1, rows, n, n, status, st);
}

// projBackwarddX with computeD fused into its epilogue: dAttn = dZ . W^T and
// D[row][h] = bf16(sum_c bf16(dAttn[row][h*hd + c]) * attn[row][h*hd + c]).
cudaError_t launch_proj_backward_dx_d(const __nv_bfloat16* dz, const __nv_bfloat16* w, __nv_bfloat16* dattn,
                                      const __nv_bfloat16* attn, __nv_bfloat16* d, int rows, int n, int head_dim,
                                      uint32_t* status, cudaStream_t st) {
  const Operand a{dz, false}, b{w, false};
  void* c[1] = {dattn};
  const bool cf[1] = {false};
  return run_gemm<128, false, false, false, true>(&a, 1, &b, 1, c, cf, 1, 1, rows, n, n, status, st, 1, attn,
                                                  d, head_dim);
}

cudaError_t launch_proj_backward_dw(const __nv_bfloat16* attn, const __nv_bfloat16* dz, __nv_bfloat16* dw,
                                    int rows, int n, uint32_t* status, cudaStream_t st) {
  const Operand a{attn, false}, b{dz, false};
  void* c[1] = {dw};
  const bool cf[1] = {false};
  return run_gemm<64, true, true, false>(&a, 1, &b, 1, c, cf, 1, 1, n, n, rows, status, st);
}

cudaError_t launch_grad_dx(float* dx, const __nv_bfloat16* qw, const __nv_bfloat16* kw,
                           const __nv_bfloat16* vw, const float* dq, const __nv_bfloat16* dk,
                           const __nv_bfloat16* dv, int rows, int n, uint32_t* status, cudaStream_t st) {
  const Operand a[3] = {{dq, true}, {dk, false}, {dv, false}};
  const Operand b[3] = {{qw, false}, {kw, false}, {vw, false}};
  void* c[1] = {dx};
  const bool cf[1] = {true};
  return run_gemm<128, false, false, true>(a, 3, b, 3, c, cf, 1, 3, rows, n, n, status, st);
}

cudaError_t launch_grad_dw(const __nv_bfloat16* x, const float* dq, const __nv_bfloat16* dk,
                           const __nv_bfloat16* dv, float* dqw, __nv_bfloat16* dkw, __nv_bfloat16* dvw,
                           int rows, int n, uint32_t* status, cudaStream_t st) {
  const Operand a{x, false};
  const Operand b[3] = {{dq, true}, {dk, false}, {dv, false}};
  void* c[3] = {dqw, dkw, dvw};
  const bool cf[3] = {true, false, false};
  return run_gemm<64, true, true, true>(&a, 1, b, 3, c, cf, 3, 1, n, n, rows, status, st);
}

// The same two products with dQ already rounded to bf16 (the rounding the
// fp32-operand path applies in shared memory, so the results are identical):
// the all-bf16 kernel without the in-kernel conversion.  The weight
// gradients are split along K and added (TMA reductions) into fp32 outputs
// the caller has zeroed.
cudaError_t launch_grad_dw_splitk_f32(const __nv_bfloat16* x, const __nv_bfloat16* dq16, const __nv_bfloat16* dk,
                                      const __nv_bfloat16* dv, float* dqw, float* dkw, float* dvw, int rows, int n,
                                      uint32_t* status, cudaStream_t st) {
  const Operand a{x, false};
  const Operand b[3] = {{dq16, false}, {dk, false}, {dv, false}};
  void* c[3] = {dqw, dkw, dvw};
  const bool cf[3] = {true, true, true};
  if (n % 128 == 0) {
    const int tiles = 3 * ((n + 127) / 128) * (n / 128);
    return run_gemm<128, true, true, false>(&a, 1, b, 3, c, cf, 3, 1, n, n, rows, status, st,
                                            pick_ksplit(tiles, rows, 2));
  }
  const int tiles = 3 * ((n + 127) / 128) * ((n + 63) / 64);
  return run_gemm<64, true, true, false>(&a, 1, b, 3, c, cf, 3, 1, n, n, rows, status, st,
                                         pick_ksplit(tiles, rows, 3));
}

cudaError_t launch_grad_dx_bf16(void* dx, bool dx_f32, const __nv_bfloat16* qw, const __nv_bfloat16* kw,
                                const __nv_bfloat16* vw, const __nv_bfloat16* dq16, const __nv_bfloat16* dk,
                                const __nv_bfloat16* dv, int rows, int n, uint32_t* status, cudaStream_t st) {
  const Operand a[3] = {{dq16, false}, {dk, false}, {dv, false}};
  const Operand b[3] = {{qw, false}, {kw, false}, {vw, false}};
  void* c[1] = {dx};
  const bool cf[1] = {dx_f32};
  return run_gemm<128, false, false, false>(a, 3, b, 3, c, cf, 1, 3, rows, n, n, status, st);
}

}  // namespace ma
