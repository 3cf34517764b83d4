// attn_oracle.cpp -- TEST INFRASTRUCTURE ONLY (the checker, never the product).
//
// Scalar, multithreaded CPU restatement of metalLLM's causal attention hot path:
//   computeQKV             attention.metal:19-53   (dispatch model.h:446-458)
//   flashAttentionForward  attention.metal:56-164  (dispatch model.h:459-473)
//   computeD               attention.metal:166-195 (dispatch model.h:639-647)
//   flashAttentionBackward attention.metal:198-299 (dispatch model.h:648-665)
//   computeGradDx, computeGradDw, projForward, projBackwarddW, projBackwarddX
//                          attention.metal:301-455 (dispatch model.h:474-481,
//                          621-636, 666-691)
//
// PARITY UNPINNED: the reference runs only on Apple Metal and ships no tests,
// golden vectors or fixtures, and its contractions run inside the closed
// MetalPerformancePrimitives matmul2d.  This file is anchored instead on the
// reference's own documented known answer (README.md:132, "row 0 of a causal
// head must equal V row 0"), on closed-form cases and on an fp64
// finite-difference check of its own backward (tests/test_oracle.py).
//
// Layouts follow the reference, stacked over a batch dimension B:
//   Q, K, V, O, dO, dK, dV : bf16 [B][T][NH*D]   (head h = columns h*D .. h*D+D-1)
//   dQ                     : fp32 [B][T][NH*D]
//   lse                    : fp32 [B][T][NH]     (index row*NH + head, attention.metal:158)
//   Dvec                   : bf16 [B][T][NH]     (attention.metal:193)
// with T = params.M and NH*D = params.N (attention.metal:7-12).
//
// Modes:
//   MODE_EXACT (0)    fp32 math; bf16 only where the reference stores to a
//                     buffer.  The tolerance of the GPU parity tests applies
//                     against this mode.
//   MODE_FAITHFUL (1) additionally reproduces the reference's internal bf16
//                     roundings (S, P, dP, dS, the dQ tile, the bf16 dK/dV
//                     read-modify-write) and its 64x64 tile order.  Reported
//                     as information only.
//   MODE_FP64 (2)     double math everywhere; used by the finite-difference
//                     self-test of the backward and as a high-precision check.
//
// Every entry point takes a (bh_begin, bh_end) range of flat indices
// bh = b*NH + h so that a subset of (batch, head) shards can be checked or
// timed; rows of shards outside the range are left untouched.

#include <algorithm>
#include <atomic>
#include <cmath>
#include <cstdint>
#include <cstring>
#include <thread>
#include <functional>
#include <vector>

namespace {

enum { MODE_EXACT = 0, MODE_FAITHFUL = 1, MODE_FP64 = 2 };

// bf16 <-> fp32, round-to-nearest-even (NaN kept quiet).
inline float bf2f(uint16_t h) {
  uint32_t u = (uint32_t)h << 16;
  float f;
  std::memcpy(&f, &u, 4);
  return f;
}
inline uint16_t f2bf(float f) {
  uint32_t u;
  std::memcpy(&u, &f, 4);
  if ((u & 0x7fffffffu) > 0x7f800000u) return (uint16_t)((u >> 16) | 0x40);
  uint32_t lsb = (u >> 16) & 1u;
  u += 0x7fffu + lsb;
  return (uint16_t)(u >> 16);
}
inline float rbf(float f) { return bf2f(f2bf(f)); }

// Runs fn(i) for i in [0, n) on up to nthreads std::threads, handing out
// indices dynamically so that unequal work items balance.
template <class F>
void parallel_for(int64_t n, int nthreads, F fn) {
  if (n <= 0) return;
  if (nthreads <= 0) nthreads = (int)std::max(1u, std::thread::hardware_concurrency());
  nthreads = (int)std::min<int64_t>(nthreads, n);
  if (nthreads <= 1) {
    for (int64_t i = 0; i < n; ++i) fn(i);
    return;
  }
  std::atomic<int64_t> next{0};
  std::vector<std::thread> pool;
  pool.reserve(nthreads);
  for (int t = 0; t < nthreads; ++t)
    pool.emplace_back([&] {
      for (int64_t i = next.fetch_add(1); i < n; i = next.fetch_add(1)) fn(i);
    });
  for (auto& th : pool) th.join();
}

struct Shape {
  int64_t T, N, D, NH, B;
};

bool valid(const Shape& s, uint32_t bh_begin, uint32_t bh_end) {
  if (s.T <= 0 || s.D <= 0 || s.NH <= 0 || s.B <= 0) return false;
  if (s.N != s.NH * s.D) return false;
  if (bh_begin > bh_end || (int64_t)bh_end > s.B * s.NH) return false;
  return true;
}

// ----------------------------------------------------------------- forward
// Exact / fp64: plain two-pass softmax per query row (the tiling of the
// reference only changes summation order).  Acc is float or double.
template <class Acc>
void fwd_row_exact(const uint16_t* q, const uint16_t* k, const uint16_t* v,
                   uint16_t* out, float* lse, float* out32, const Shape& s,
                   int64_t b, int64_t h, int64_t i, std::vector<Acc>& sc,
                   std::vector<Acc>& acc) {
  const int64_t N = s.N, D = s.D;
  const uint16_t* qi = q + (b * s.T + i) * N + h * D;
  const Acc scale = Acc(1) / std::sqrt(Acc(D));  // 1/sqrt(D), attention.metal:109
  Acc m = -INFINITY;
  for (int64_t j = 0; j <= i; ++j) {  // causal: keys j <= i, attention.metal:111,119
    const uint16_t* kj = k + (b * s.T + j) * N + h * D;
    Acc dot = 0;
    for (int64_t c = 0; c < D; ++c) dot += Acc(bf2f(qi[c])) * Acc(bf2f(kj[c]));
    sc[j] = dot * scale;
    m = std::max(m, sc[j]);
  }
  Acc l = 0;
  for (int64_t c = 0; c < D; ++c) acc[c] = 0;
  for (int64_t j = 0; j <= i; ++j) {
    Acc p = std::exp(sc[j] - m);
    l += p;
    const uint16_t* vj = v + (b * s.T + j) * N + h * D;
    for (int64_t c = 0; c < D; ++c) acc[c] += p * Acc(bf2f(vj[c]));
  }
  const int64_t orow = (b * s.T + i) * N + h * D;
  for (int64_t c = 0; c < D; ++c) {
    Acc o = acc[c] / l;  // out = O / rowsum, attention.metal:157,161
    out[orow + c] = f2bf((float)o);
    if (out32) out32[orow + c] = (float)o;
  }
  lse[(b * s.T + i) * s.NH + h] = (float)(m + std::log(l));  // attention.metal:158
}

// Faithful: the reference's per-(head, 64-row tile) loop with its bf16
// roundings, attention.metal:74-163.
void fwd_tile_faithful(const uint16_t* q, const uint16_t* k, const uint16_t* v,
                       uint16_t* out, float* lse, float* out32, const Shape& s,
                       int64_t b, int64_t h, int64_t tile) {
  const int64_t TM = 64, N = s.N, D = s.D;
  const int64_t r0 = tile * TM;
  const int64_t rows = std::min<int64_t>(TM, s.T - r0);
  const float d_sqrt = 1.0f / std::sqrt((float)D);
  std::vector<float> O(TM * D, 0.0f), S(TM * TM), rmax(TM, -INFINITY), rsum(TM, 0.0f);
  for (int64_t kt = 0; kt <= tile; ++kt) {
    const int64_t c0 = kt * TM;
    const int64_t cols = std::min<int64_t>(TM, s.T - c0);
    // S = bf16(Q K^T), then bf16(S*scale + mask)   (attention.metal:113-121)
    for (int64_t r = 0; r < rows; ++r) {
      const uint16_t* qi = q + (b * s.T + r0 + r) * N + h * D;
      for (int64_t c = 0; c < TM; ++c) {
        float val = -INFINITY;
        if (c < cols) {
          const uint16_t* kj = k + (b * s.T + c0 + c) * N + h * D;
          float dot = 0.0f;
          for (int64_t e = 0; e < D; ++e) dot += bf2f(qi[e]) * bf2f(kj[e]);
          val = rbf(dot) * d_sqrt;
          if (r0 + r < c0 + c) val = -INFINITY;
        }
        S[r * TM + c] = rbf(val);
      }
    }
    // online softmax per row (attention.metal:125-150)
    for (int64_t r = 0; r < rows; ++r) {
      float nm = -INFINITY;
      for (int64_t c = 0; c < TM; ++c) nm = std::max(nm, S[r * TM + c]);
      const float om = rmax[r];
      nm = std::max(nm, om);
      const float ed = std::exp(om - nm);
      float ls = 0.0f;
      for (int64_t c = 0; c < TM; ++c) {
        float val = std::exp(S[r * TM + c] - nm);
        S[r * TM + c] = rbf(val);
        ls += val;
      }
      for (int64_t e = 0; e < D; ++e) O[r * D + e] *= ed;
      rmax[r] = nm;
      rsum[r] = rsum[r] * ed + ls;
    }
    // O += P V (fp32 accumulate, attention.metal:153)
    for (int64_t r = 0; r < rows; ++r)
      for (int64_t c = 0; c < cols; ++c) {
        const float p = S[r * TM + c];
        if (p == 0.0f) continue;
        const uint16_t* vj = v + (b * s.T + c0 + c) * N + h * D;
        for (int64_t e = 0; e < D; ++e) O[r * D + e] += p * bf2f(vj[e]);
      }
  }
  for (int64_t r = 0; r < rows; ++r) {
    const float inv = 1.0f / rsum[r];
    lse[(b * s.T + r0 + r) * s.NH + h] = rmax[r] + std::log(rsum[r]);
    const int64_t orow = (b * s.T + r0 + r) * N + h * D;
    for (int64_t e = 0; e < D; ++e) {
      const float o = O[r * D + e] * inv;
      out[orow + e] = f2bf(o);
      if (out32) out32[orow + e] = o;
    }
  }
}

// ---------------------------------------------------------------- backward
// Exact / fp64 backward of one (b, h) shard over a contiguous range of query
// rows [i0, i1).  dK/dV contributions go to the caller's private accumulators
// (T*D each); dQ rows of the range are complete on return.
template <class Acc>
void bwd_rows_exact(const uint16_t* dO, const uint16_t* Dv, const float* lse,
                    const uint16_t* q, const uint16_t* k, const uint16_t* v,
                    float* dQ, const Shape& s, int64_t b, int64_t h, int64_t i0,
                    int64_t i1, Acc* dKacc, Acc* dVacc) {
  const int64_t N = s.N, D = s.D;
  const Acc scale = Acc(1) / std::sqrt(Acc(D));
  std::vector<Acc> qi(D), doi(D), dqi(D);
  for (int64_t i = i0; i < i1; ++i) {
    const int64_t row = (b * s.T + i) * N + h * D;
    for (int64_t c = 0; c < D; ++c) {
      qi[c] = bf2f(q[row + c]);
      doi[c] = bf2f(dO[row + c]);
      dqi[c] = 0;
    }
    const Acc l = lse[(b * s.T + i) * s.NH + h];       // attention.metal:279
    const Acc dd = bf2f(Dv[(b * s.T + i) * s.NH + h]);  // D is read as bf16, :280
    for (int64_t j = 0; j <= i; ++j) {  // masked entries (j > i) have P = 0, :282
      const int64_t krow = (b * s.T + j) * N + h * D;
      Acc sdot = 0, pdot = 0;
      for (int64_t c = 0; c < D; ++c) {
        sdot += qi[c] * Acc(bf2f(k[krow + c]));
        pdot += doi[c] * Acc(bf2f(v[krow + c]));
      }
      const Acc p = std::exp(sdot * scale - l);        // P = exp(S/sqrt(D) - lse), :281
      const Acc ds = p * (pdot - dd) * scale;          // dS, :284
      Acc* dk = dKacc + j * D;
      Acc* dv = dVacc + j * D;
      for (int64_t c = 0; c < D; ++c) {
        dqi[c] += ds * Acc(bf2f(k[krow + c]));         // dQ = dS K, :288
        dk[c] += ds * qi[c];                           // dK = dS^T Q, :289
        dv[c] += p * doi[c];                           // dV = P^T dO, :290
      }
    }
    for (int64_t c = 0; c < D; ++c) dQ[row + c] = (float)dqi[c];
  }
}

// Faithful backward of one (b, h) shard: the reference's key-tile-owned loop
// with its bf16 roundings, attention.metal:219-298.  dQ is accumulated in the
// kt-ascending order (the reference's atomics have no fixed order).
void bwd_shard_faithful(const uint16_t* dO, const uint16_t* Dv, const float* lse,
                        const uint16_t* q, const uint16_t* k, const uint16_t* v,
                        float* dQ, uint16_t* dK, uint16_t* dV, float* dk32,
                        float* dv32, const Shape& s, int64_t b, int64_t h) {
  const int64_t TM = 64, N = s.N, D = s.D;
  const int64_t ntiles = (s.T + TM - 1) / TM;
  const float d_sqrt = 1.0f / std::sqrt((float)D);
  std::vector<float> P(TM * TM), dS(TM * TM);
  std::vector<float> dKb(TM * D), dVb(TM * D);
  for (int64_t i = 0; i < s.T; ++i)
    for (int64_t c = 0; c < D; ++c) dQ[(b * s.T + i) * N + h * D + c] = 0.0f;
  for (int64_t kt = 0; kt < ntiles; ++kt) {
    const int64_t c0 = kt * TM, cols = std::min<int64_t>(TM, s.T - c0);
    std::fill(dKb.begin(), dKb.end(), 0.0f);  // the bf16 dK/dV tiles (pre-zeroed)
    std::fill(dVb.begin(), dVb.end(), 0.0f);
    for (int64_t qt = kt; qt < ntiles; ++qt) {
      const int64_t r0 = qt * TM, rows = std::min<int64_t>(TM, s.T - r0);
      for (int64_t r = 0; r < rows; ++r) {
        const int64_t qrow = (b * s.T + r0 + r) * N + h * D;
        const float l = lse[(b * s.T + r0 + r) * s.NH + h];
        const float dd = bf2f(Dv[(b * s.T + r0 + r) * s.NH + h]);
        for (int64_t c = 0; c < cols; ++c) {
          const int64_t krow = (b * s.T + c0 + c) * N + h * D;
          float sdot = 0.0f, pdot = 0.0f;
          for (int64_t e = 0; e < D; ++e) {
            sdot += bf2f(q[qrow + e]) * bf2f(k[krow + e]);
            pdot += bf2f(dO[qrow + e]) * bf2f(v[krow + e]);
          }
          float val = std::exp(rbf(sdot) * d_sqrt - l);
          if (kt == qt && c > r) val = 0.0f;
          P[r * TM + c] = rbf(val);
          dS[r * TM + c] = rbf(val * (rbf(pdot) - dd) * d_sqrt);
        }
      }
      // dQ tile = bf16(dS K), added in fp32 (attention.metal:288-296)
      for (int64_t r = 0; r < rows; ++r) {
        const int64_t qrow = (b * s.T + r0 + r) * N + h * D;
        for (int64_t e = 0; e < D; ++e) {
          float acc = 0.0f;
          for (int64_t c = 0; c < cols; ++c)
            acc += dS[r * TM + c] * bf2f(k[(b * s.T + c0 + c) * N + h * D + e]);
          dQ[qrow + e] += rbf(acc);
        }
      }
      // dK += dS^T Q and dV += P^T dO on bf16 memory (attention.metal:289-290)
      for (int64_t c = 0; c < cols; ++c)
        for (int64_t e = 0; e < D; ++e) {
          float ak = 0.0f, av = 0.0f;
          for (int64_t r = 0; r < rows; ++r) {
            const int64_t qrow = (b * s.T + r0 + r) * N + h * D;
            ak += dS[r * TM + c] * bf2f(q[qrow + e]);
            av += P[r * TM + c] * bf2f(dO[qrow + e]);
          }
          dKb[c * D + e] = rbf(dKb[c * D + e] + ak);
          dVb[c * D + e] = rbf(dVb[c * D + e] + av);
        }
    }
    for (int64_t c = 0; c < cols; ++c) {
      const int64_t krow = (b * s.T + c0 + c) * N + h * D;
      for (int64_t e = 0; e < D; ++e) {
        dK[krow + e] = f2bf(dKb[c * D + e]);
        dV[krow + e] = f2bf(dVb[c * D + e]);
        if (dk32) dk32[krow + e] = dKb[c * D + e];
        if (dv32) dv32[krow + e] = dVb[c * D + e];
      }
    }
  }
}

// Splits the causal rows [0, T) of one shard into `parts` contiguous ranges of
// roughly equal work (row i costs i+1 key visits).
std::vector<int64_t> causal_splits(int64_t T, int parts) {
  std::vector<int64_t> cut(parts + 1, T);
  cut[0] = 0;
  const double total = 0.5 * (double)T * (double)(T + 1);
  int64_t i = 0;
  double acc = 0.0;
  for (int p = 1; p < parts; ++p) {
    const double target = total * p / parts;
    while (i < T && acc + (double)(i + 1) <= target) acc += (double)(++i);
    cut[p] = i;
  }
  return cut;
}

template <class Acc>
void bwd_exact(const uint16_t* dO, const uint16_t* Dv, const float* lse,
               const uint16_t* q, const uint16_t* k, const uint16_t* v, float* dQ,
               uint16_t* dK, uint16_t* dV, float* dk32, float* dv32, const Shape& s,
               uint32_t bh0, uint32_t bh1, int nthreads) {
  const int64_t nsh = bh1 - bh0;
  if (nthreads <= 0) nthreads = (int)std::max(1u, std::thread::hardware_concurrency());
  // Few shards: split each shard's rows across threads with private dK/dV
  // accumulators; many shards: one shard per work item.
  const int parts = nsh >= nthreads ? 1 : (int)std::max<int64_t>(1, nthreads / std::max<int64_t>(nsh, 1));
  const int64_t T = s.T, D = s.D;
  std::vector<std::vector<int64_t>> splits;
  const std::vector<int64_t> cut = causal_splits(T, parts);
  std::vector<std::vector<Acc>> accK(nsh * parts), accV(nsh * parts);
  parallel_for(nsh * parts, nthreads, [&](int64_t w) {
    const int64_t sh = w / parts, part = w % parts;
    const int64_t bh = bh0 + sh, b = bh / s.NH, h = bh % s.NH;
    accK[w].assign(T * D, Acc(0));
    accV[w].assign(T * D, Acc(0));
    bwd_rows_exact<Acc>(dO, Dv, lse, q, k, v, dQ, s, b, h, cut[part], cut[part + 1],
                        accK[w].data(), accV[w].data());
  });
  parallel_for(nsh, nthreads, [&](int64_t sh) {
    const int64_t bh = bh0 + sh, b = bh / s.NH, h = bh % s.NH;
    for (int64_t j = 0; j < T; ++j) {
      const int64_t krow = (b * T + j) * s.N + h * D;
      for (int64_t c = 0; c < D; ++c) {
        Acc sk = 0, sv = 0;
        for (int p = 0; p < parts; ++p) {
          sk += accK[sh * parts + p][j * D + c];
          sv += accV[sh * parts + p][j * D + c];
        }
        dK[krow + c] = f2bf((float)sk);
        dV[krow + c] = f2bf((float)sv);
        if (dk32) dk32[krow + c] = (float)sk;
        if (dv32) dv32[krow + c] = (float)sv;
      }
    }
  });
}

}  // namespace

extern "C" {

// Oracle of computeQKV (attention.metal:19-53): Q = bf16(X Wq), K = bf16(X Wk),
// V = bf16(X Wv) with fp32 accumulation.  X is [rows][N] with rows = B*M; the
// weights are [N][N] row-major, row = input feature, column = output feature
// (main.cpp:1595).  q32/k32/v32 (optional) receive the unrounded fp32 values.
int oracle_compute_qkv(const uint16_t* X, uint16_t* q, uint16_t* k, uint16_t* v,
                       const uint16_t* qw, const uint16_t* kw, const uint16_t* vw,
                       uint32_t M, uint32_t N, uint32_t B, int nthreads, float* q32,
                       float* k32, float* v32) {
  if (!X || !q || !k || !v || !qw || !kw || !vw || M == 0 || N == 0 || B == 0) return 1;
  const int64_t rows = (int64_t)M * B;
  parallel_for(rows, nthreads, [&](int64_t r) {
    std::vector<float> aq(N, 0.0f), ak(N, 0.0f), av(N, 0.0f);
    for (int64_t kk = 0; kk < N; ++kk) {
      const float x = bf2f(X[r * N + kk]);
      if (x == 0.0f) continue;
      const uint16_t* wq = qw + kk * N;
      const uint16_t* wk = kw + kk * N;
      const uint16_t* wv = vw + kk * N;
      for (int64_t n = 0; n < N; ++n) {
        aq[n] += x * bf2f(wq[n]);
        ak[n] += x * bf2f(wk[n]);
        av[n] += x * bf2f(wv[n]);
      }
    }
    for (int64_t n = 0; n < N; ++n) {
      q[r * N + n] = f2bf(aq[n]);
      k[r * N + n] = f2bf(ak[n]);
      v[r * N + n] = f2bf(av[n]);
      if (q32) q32[r * N + n] = aq[n];
      if (k32) k32[r * N + n] = ak[n];
      if (v32) v32[r * N + n] = av[n];
    }
  });
  return 0;
}

// Oracle of flashAttentionForward (attention.metal:56-164) for shards
// [bh_begin, bh_end).  out32 (optional) receives O before the bf16 store.
int oracle_flash_forward(const uint16_t* q, const uint16_t* k, const uint16_t* v,
                         uint16_t* out, float* lse, uint32_t M, uint32_t N, uint32_t D,
                         uint32_t NH, uint32_t B, uint32_t bh_begin, uint32_t bh_end,
                         int mode, int nthreads, float* out32) {
  const Shape s{M, N, D, NH, B};
  if (!q || !k || !v || !out || !lse || !valid(s, bh_begin, bh_end)) return 1;
  const int64_t nsh = bh_end - bh_begin;
  if (mode == MODE_FAITHFUL) {
    const int64_t nt = (s.T + 63) / 64;
    // longest tiles first for balance
    parallel_for(nsh * nt, nthreads, [&](int64_t w) {
      const int64_t sh = w / nt, tile = nt - 1 - (w % nt);
      const int64_t bh = bh_begin + sh;
      fwd_tile_faithful(q, k, v, out, lse, out32, s, bh / s.NH, bh % s.NH, tile);
    });
    return 0;
  }
  const int64_t chunk = 16;
  const int64_t nchunks = (s.T + chunk - 1) / chunk;
  parallel_for(nsh * nchunks, nthreads, [&](int64_t w) {
    const int64_t sh = w / nchunks, ch = nchunks - 1 - (w % nchunks);
    const int64_t bh = bh_begin + sh, b = bh / s.NH, h = bh % s.NH;
    const int64_t i0 = ch * chunk, i1 = std::min<int64_t>(s.T, i0 + chunk);
    if (mode == MODE_FP64) {
      std::vector<double> sc(s.T), acc(s.D);
      for (int64_t i = i0; i < i1; ++i) fwd_row_exact<double>(q, k, v, out, lse, out32, s, b, h, i, sc, acc);
    } else {
      std::vector<float> sc(s.T), acc(s.D);
      for (int64_t i = i0; i < i1; ++i) fwd_row_exact<float>(q, k, v, out, lse, out32, s, b, h, i, sc, acc);
    }
  });
  return 0;
}

// Oracle of computeD (attention.metal:166-195): D[r,h] = bf16(sum_c dO*O) with
// an fp32 sum (fp64 in MODE_FP64; bf16-rounded products in MODE_FAITHFUL).
// d32 (optional) receives the sum before the bf16 store.
int oracle_compute_d(const uint16_t* dO, const uint16_t* O, uint16_t* Dout, uint32_t M,
                     uint32_t N, uint32_t D, uint32_t NH, uint32_t B, uint32_t bh_begin,
                     uint32_t bh_end, int mode, int nthreads, float* d32) {
  const Shape s{M, N, D, NH, B};
  if (!dO || !O || !Dout || !valid(s, bh_begin, bh_end)) return 1;
  parallel_for((int64_t)(bh_end - bh_begin), nthreads, [&](int64_t sh) {
    const int64_t bh = bh_begin + sh, b = bh / s.NH, h = bh % s.NH;
    for (int64_t i = 0; i < s.T; ++i) {
      const int64_t row = (b * s.T + i) * s.N + h * s.D;
      double acc64 = 0.0;
      float acc = 0.0f;
      for (int64_t c = 0; c < s.D; ++c) {
        const float x = bf2f(dO[row + c]), y = bf2f(O[row + c]);
        if (mode == MODE_FP64) acc64 += (double)x * (double)y;
        else if (mode == MODE_FAITHFUL) acc += rbf(x * y);
        else acc += x * y;
      }
      const float r = mode == MODE_FP64 ? (float)acc64 : acc;
      const int64_t di = (b * s.T + i) * s.NH + h;
      Dout[di] = f2bf(r);
      if (d32) d32[di] = r;
    }
  });
  return 0;
}

// Oracle of flashAttentionBackward (attention.metal:198-299).  dQ is written
// (not accumulated) in fp32; dK/dV are written in bf16.  dk32/dv32 (optional)
// receive dK/dV before the bf16 store.
int oracle_flash_backward(const uint16_t* dO, const uint16_t* Dv, const float* lse,
                          const uint16_t* q, const uint16_t* k, const uint16_t* v,
                          float* dQ, uint16_t* dK, uint16_t* dV, uint32_t M, uint32_t N,
                          uint32_t D, uint32_t NH, uint32_t B, uint32_t bh_begin,
                          uint32_t bh_end, int mode, int nthreads, float* dk32,
                          float* dv32) {
  const Shape s{M, N, D, NH, B};
  if (!dO || !Dv || !lse || !q || !k || !v || !dQ || !dK || !dV || !valid(s, bh_begin, bh_end))
    return 1;
  if (mode == MODE_FAITHFUL) {
    parallel_for((int64_t)(bh_end - bh_begin), nthreads, [&](int64_t sh) {
      const int64_t bh = bh_begin + sh;
      bwd_shard_faithful(dO, Dv, lse, q, k, v, dQ, dK, dV, dk32, dv32, s, bh / s.NH, bh % s.NH);
    });
  } else if (mode == MODE_FP64) {
    bwd_exact<double>(dO, Dv, lse, q, k, v, dQ, dK, dV, dk32, dv32, s, bh_begin, bh_end, nthreads);
  } else {
    bwd_exact<float>(dO, Dv, lse, q, k, v, dQ, dK, dV, dk32, dv32, s, bh_begin, bh_end, nthreads);
  }
  return 0;
}

// ---------------------------------------------------------------- GEMMs
// The GEMMs around attention (attention.metal:301-455), fp32 accumulation.
// Activations are [rows][N] (rows = B*M), weights [N][N] with row = input
// feature.  Operands marked fp32 are read as fp32 (the reference's dQ);
// everything else is bf16.  `sel` / `nsel` (optional) restrict the work to
// those output rows (the rest is left untouched): large shapes are checked on
// a sample of rows.  c32 (optional) receives the unrounded fp32 results.
namespace {

inline float ld(const void* p, bool f32, int64_t i) {
  return f32 ? static_cast<const float*>(p)[i] : bf2f(static_cast<const uint16_t*>(p)[i]);
}

// C[r][n] = sum_p sum_k A_p[r][k] * W_p[n][k]   (A times W^T; row r of C)
void rows_times_wt(int np, const void* const* A, const bool* af32, const uint16_t* const* W,
                   int64_t rows, int64_t N, const int64_t* sel, int64_t nsel, int nthreads,
                   std::function<void(int64_t, int64_t, float)> put) {
  const int64_t nr = sel ? nsel : rows;
  parallel_for(nr, nthreads, [&](int64_t idx) {
    const int64_t r = sel ? sel[idx] : idx;
    for (int64_t n = 0; n < N; ++n) {
      float acc = 0.0f;
      for (int p = 0; p < np; ++p)
        for (int64_t k = 0; k < N; ++k) acc += ld(A[p], af32[p], r * N + k) * bf2f(W[p][n * N + k]);
      put(r, n, acc);
    }
  });
}

// C[i][j] = sum_r X[r][i] * G[r][j]   (X^T times G; row i of C)
void xt_times_g(const uint16_t* X, const void* G, bool gf32, int64_t rows, int64_t N,
                const int64_t* sel, int64_t nsel, int nthreads,
                std::function<void(int64_t, int64_t, float)> put) {
  const int64_t nr = sel ? nsel : N;
  parallel_for(nr, nthreads, [&](int64_t idx) {
    const int64_t i = sel ? sel[idx] : idx;
    std::vector<float> acc(N, 0.0f);
    for (int64_t r = 0; r < rows; ++r) {
      const float x = bf2f(X[r * N + i]);
      if (x == 0.0f) continue;
      for (int64_t j = 0; j < N; ++j) acc[j] += x * ld(G, gf32, r * N + j);
    }
    for (int64_t j = 0; j < N; ++j) put(i, j, acc[j]);
  });
}

}  // namespace

// projForward (attention.metal:395-416): out = attn_out . proj_w
int oracle_proj_forward(const uint16_t* attn, const uint16_t* w, uint16_t* out, uint32_t rows,
                        uint32_t N, const int64_t* sel, int64_t nsel, int nthreads, float* out32) {
  if (!attn || !w || !out || rows == 0 || N == 0) return 1;
  const int64_t nr = sel ? nsel : rows;
  parallel_for(nr, nthreads, [&](int64_t idx) {
    const int64_t r = sel ? sel[idx] : idx;
    std::vector<float> acc(N, 0.0f);
    for (int64_t k = 0; k < N; ++k) {
      const float a = bf2f(attn[r * N + k]);
      if (a == 0.0f) continue;
      for (int64_t n = 0; n < N; ++n) acc[n] += a * bf2f(w[k * N + n]);
    }
    for (int64_t n = 0; n < N; ++n) {
      out[r * N + n] = f2bf(acc[n]);
      if (out32) out32[r * N + n] = acc[n];
    }
  });
  return 0;
}

// projBackwarddX (attention.metal:432-455): dAttn = dZ . proj_w^T
int oracle_proj_backward_dx(const uint16_t* dz, const uint16_t* w, uint16_t* dattn, uint32_t rows,
                            uint32_t N, const int64_t* sel, int64_t nsel, int nthreads, float* d32) {
  if (!dz || !w || !dattn || rows == 0 || N == 0) return 1;
  const void* A[1] = {dz};
  const bool af[1] = {false};
  const uint16_t* W[1] = {w};
  rows_times_wt(1, A, af, W, rows, N, sel, nsel, nthreads, [&](int64_t r, int64_t n, float v) {
    dattn[r * N + n] = f2bf(v);
    if (d32) d32[r * N + n] = v;
  });
  return 0;
}

// projBackwarddW (attention.metal:418-430): dProjw = attn_out^T . dZ
int oracle_proj_backward_dw(const uint16_t* attn, const uint16_t* dz, uint16_t* dw, uint32_t rows,
                            uint32_t N, const int64_t* sel, int64_t nsel, int nthreads, float* dw32) {
  if (!attn || !dz || !dw || rows == 0 || N == 0) return 1;
  xt_times_g(attn, dz, false, rows, N, sel, nsel, nthreads, [&](int64_t i, int64_t j, float v) {
    dw[i * N + j] = f2bf(v);
    if (dw32) dw32[i * N + j] = v;
  });
  return 0;
}

// computeGradDx (attention.metal:301-342): dX = dQ.Wq^T + dK.Wk^T + dV.Wv^T
// (fp32 dQ and dX, the three products summed in one fp32 accumulator)
int oracle_grad_dx(float* dx, const uint16_t* qw, const uint16_t* kw, const uint16_t* vw,
                   const float* dq, const uint16_t* dk, const uint16_t* dv, uint32_t rows, uint32_t N,
                   const int64_t* sel, int64_t nsel, int nthreads) {
  if (!dx || !qw || !kw || !vw || !dq || !dk || !dv || rows == 0 || N == 0) return 1;
  const void* A[3] = {dq, dk, dv};
  const bool af[3] = {true, false, false};
  const uint16_t* W[3] = {qw, kw, vw};
  rows_times_wt(3, A, af, W, rows, N, sel, nsel, nthreads,
                [&](int64_t r, int64_t n, float v) { dx[r * N + n] = v; });
  return 0;
}

// computeGradDw (attention.metal:344-393): dQw = X^T.dQ (fp32), dKw = X^T.dK,
// dVw = X^T.dV (bf16; dk32/dv32 optional unrounded values)
int oracle_grad_dw(const uint16_t* x, const float* dq, const uint16_t* dk, const uint16_t* dv,
                   float* dqw, uint16_t* dkw, uint16_t* dvw, uint32_t rows, uint32_t N,
                   const int64_t* sel, int64_t nsel, int nthreads, float* dk32, float* dv32) {
  if (!x || !dq || !dk || !dv || !dqw || !dkw || !dvw || rows == 0 || N == 0) return 1;
  xt_times_g(x, dq, true, rows, N, sel, nsel, nthreads,
             [&](int64_t i, int64_t j, float v) { dqw[i * N + j] = v; });
  xt_times_g(x, dk, false, rows, N, sel, nsel, nthreads, [&](int64_t i, int64_t j, float v) {
    dkw[i * N + j] = f2bf(v);
    if (dk32) dk32[i * N + j] = v;
  });
  xt_times_g(x, dv, false, rows, N, sel, nsel, nthreads, [&](int64_t i, int64_t j, float v) {
    dvw[i * N + j] = f2bf(v);
    if (dv32) dv32[i * N + j] = v;
  });
  return 0;
}

// fp64 loss used by the finite-difference self-test of the backward:
// L = sum over rows/cols of dO * O with O the exact fp64 causal attention
// output computed from fp64 (not bf16) inputs.  Inputs are fp64 [T][D] for a
// single head; returns L.  Gradients of L with respect to q/k/v are what the
// backward computes when dO is the weight and D = rowsum(dO * O).
double oracle_fp64_loss(const double* q, const double* k, const double* v,
                        const double* dO, uint32_t T, uint32_t D) {
  const double scale = 1.0 / std::sqrt((double)D);
  std::vector<double> sc(T);
  double L = 0.0;
  for (uint32_t i = 0; i < T; ++i) {
    double m = -INFINITY;
    for (uint32_t j = 0; j <= i; ++j) {
      double dot = 0.0;
      for (uint32_t c = 0; c < D; ++c) dot += q[i * D + c] * k[j * D + c];
      sc[j] = dot * scale;
      m = std::max(m, sc[j]);
    }
    double l = 0.0;
    for (uint32_t j = 0; j <= i; ++j) l += std::exp(sc[j] - m);
    for (uint32_t c = 0; c < D; ++c) {
      double o = 0.0;
      for (uint32_t j = 0; j <= i; ++j) o += std::exp(sc[j] - m) * v[j * D + c];
      L += dO[i * D + c] * (o / l);
    }
  }
  return L;
}

}  // extern "C"
