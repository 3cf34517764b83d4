// flash_v0.cu -- first correct CUDA path of flashAttentionForward /
// flashAttentionBackward (attention.metal:56-164, 198-299) and computeQKV
// (attention.metal:19-53): plain fp32 FMA kernels with shared-memory tiles,
// one thread per query row (forward) or key row (backward).  Same math and
// conventions as the reference: scale 1/sqrt(D) after Q K^T, causal mask
// key > query, l = m + ln(rowsum) in fp32, dS includes the 1/sqrt(D) factor,
// dQ fp32.  Only P is not rounded to bf16 here.
#include "common.cuh"

namespace ma {
namespace {

constexpr int TILE = 64;

__device__ __forceinline__ float bf(const __nv_bfloat16 x) { return __bfloat162float(x); }

// Forward: block = 64 threads = 64 query rows of one (batch, head).
template <int D>
__global__ void __launch_bounds__(64) fwd_v0_kernel(const __nv_bfloat16* __restrict__ q,
                                                    const __nv_bfloat16* __restrict__ k,
                                                    const __nv_bfloat16* __restrict__ v,
                                                    __nv_bfloat16* __restrict__ out,
                                                    float* __restrict__ lse, AttnShape s) {
  extern __shared__ float smem[];
  float* qs = smem;                    // [64][D+1]
  float* ks = qs + TILE * (D + 1);     // [64][D+1]
  float* vs = ks + TILE * (D + 1);     // [64][D]
  float* os = vs + TILE * D;           // [64][D+1]
  const int tile = blockIdx.x;
  const int bh = s.bh_begin + blockIdx.y;
  const int b = bh / s.NH, h = bh % s.NH;
  const int r = threadIdx.x;
  const int row = tile * TILE + r;
  const long long base = (long long)b * s.T * s.N + (long long)h * D;
  const float scale = rsqrtf((float)D);
  for (int i = threadIdx.x; i < TILE * D; i += blockDim.x) {
    const int rr = i / D, c = i % D;
    qs[rr * (D + 1) + c] = bf(q[base + (long long)(tile * TILE + rr) * s.N + c]);
    os[rr * (D + 1) + c] = 0.0f;
  }
  float m = -INFINITY, l = 0.0f;
  float sc[TILE];
  for (int kt = 0; kt <= tile; ++kt) {
    __syncthreads();
    for (int i = threadIdx.x; i < TILE * D; i += blockDim.x) {
      const int rr = i / D, c = i % D;
      const long long g = base + (long long)(kt * TILE + rr) * s.N + c;
      ks[rr * (D + 1) + c] = bf(k[g]);
      vs[rr * D + c] = bf(v[g]);
    }
    __syncthreads();
    float tmax = -INFINITY;
#pragma unroll 1
    for (int j = 0; j < TILE; ++j) {
      float dot = -INFINITY;
      if (kt * TILE + j <= row) {
        dot = 0.0f;
        for (int c = 0; c < D; ++c) dot = fmaf(qs[r * (D + 1) + c], ks[j * (D + 1) + c], dot);
        dot *= scale;
      }
      sc[j] = dot;
      tmax = fmaxf(tmax, dot);
    }
    const float mnew = fmaxf(m, tmax);
    const float alpha = __expf(m - mnew);
    l *= alpha;
    for (int c = 0; c < D; ++c) os[r * (D + 1) + c] *= alpha;
#pragma unroll 1
    for (int j = 0; j < TILE; ++j) {
      const float p = __expf(sc[j] - mnew);
      l += p;
      if (p != 0.0f)
        for (int c = 0; c < D; ++c) os[r * (D + 1) + c] = fmaf(p, vs[j * D + c], os[r * (D + 1) + c]);
    }
    m = mnew;
  }
  const float inv = 1.0f / l;
  for (int c = 0; c < D; ++c)
    out[base + (long long)row * s.N + c] = __float2bfloat16_rn(os[r * (D + 1) + c] * inv);
  lse[((long long)b * s.T + row) * s.NH + h] = m + logf(l);
}

// Backward: block = 64 threads = 64 key rows of one (batch, head); the block
// owns dK/dV of its key tile (as attention.metal:220 does) and adds its dQ
// contributions with fp32 atomics (attention.metal:292-296).
template <int D>
__global__ void __launch_bounds__(64) bwd_v0_kernel(
    const __nv_bfloat16* __restrict__ dO, const __nv_bfloat16* __restrict__ Dv,
    const float* __restrict__ lse, const __nv_bfloat16* __restrict__ q,
    const __nv_bfloat16* __restrict__ k, const __nv_bfloat16* __restrict__ v,
    float* __restrict__ dQ, __nv_bfloat16* __restrict__ dK, __nv_bfloat16* __restrict__ dV,
    AttnShape s) {
  extern __shared__ float smem[];
  float* ks = smem;                    // [64][D+1]
  float* vs = ks + TILE * (D + 1);     // [64][D+1]
  float* dks = vs + TILE * (D + 1);    // [64][D+1]
  float* dvs = dks + TILE * (D + 1);   // [64][D+1]
  float* qs = dvs + TILE * (D + 1);    // [64][D]
  float* dos = qs + TILE * D;          // [64][D]
  float* dss = dos + TILE * D;         // [64][65]
  float* ls = dss + TILE * (TILE + 1); // [64]
  float* dd = ls + TILE;               // [64]
  const int kt = blockIdx.x;
  const int bh = s.bh_begin + blockIdx.y;
  const int b = bh / s.NH, h = bh % s.NH;
  const int j = threadIdx.x;
  const int key = kt * TILE + j;
  const long long base = (long long)b * s.T * s.N + (long long)h * D;
  const float scale = rsqrtf((float)D);
  for (int i = threadIdx.x; i < TILE * D; i += blockDim.x) {
    const int rr = i / D, c = i % D;
    const long long g = base + (long long)(kt * TILE + rr) * s.N + c;
    ks[rr * (D + 1) + c] = bf(k[g]);
    vs[rr * (D + 1) + c] = bf(v[g]);
    dks[rr * (D + 1) + c] = 0.0f;
    dvs[rr * (D + 1) + c] = 0.0f;
  }
  const int ntiles = s.T / TILE;
  for (int qt = kt; qt < ntiles; ++qt) {
    __syncthreads();
    for (int i = threadIdx.x; i < TILE * D; i += blockDim.x) {
      const int rr = i / D, c = i % D;
      const long long g = base + (long long)(qt * TILE + rr) * s.N + c;
      qs[rr * D + c] = bf(q[g]);
      dos[rr * D + c] = bf(dO[g]);
    }
    {
      const long long li = ((long long)b * s.T + qt * TILE + threadIdx.x) * s.NH + h;
      ls[threadIdx.x] = lse[li];
      dd[threadIdx.x] = bf(Dv[li]);
    }
    __syncthreads();
#pragma unroll 1
    for (int i = 0; i < TILE; ++i) {
      const int qrow = qt * TILE + i;
      float ds = 0.0f;
      if (key <= qrow) {
        float sdot = 0.0f, pdot = 0.0f;
        for (int c = 0; c < D; ++c) {
          sdot = fmaf(qs[i * D + c], ks[j * (D + 1) + c], sdot);
          pdot = fmaf(dos[i * D + c], vs[j * (D + 1) + c], pdot);
        }
        const float p = __expf(sdot * scale - ls[i]);
        ds = p * (pdot - dd[i]) * scale;
        for (int c = 0; c < D; ++c) {
          dvs[j * (D + 1) + c] = fmaf(p, dos[i * D + c], dvs[j * (D + 1) + c]);
          dks[j * (D + 1) + c] = fmaf(ds, qs[i * D + c], dks[j * (D + 1) + c]);
        }
      }
      dss[i * (TILE + 1) + j] = ds;
    }
    __syncthreads();
    for (int e = threadIdx.x; e < TILE * D; e += blockDim.x) {
      const int i = e / D, c = e % D;
      float acc = 0.0f;
      for (int jj = 0; jj < TILE; ++jj) acc = fmaf(dss[i * (TILE + 1) + jj], ks[jj * (D + 1) + c], acc);
      atomicAdd(dQ + base + (long long)(qt * TILE + i) * s.N + c, acc);
    }
  }
  __syncthreads();
  for (int i = threadIdx.x; i < TILE * D; i += blockDim.x) {
    const int rr = i / D, c = i % D;
    const long long g = base + (long long)(kt * TILE + rr) * s.N + c;
    dK[g] = __float2bfloat16_rn(dks[rr * (D + 1) + c]);
    dV[g] = __float2bfloat16_rn(dvs[rr * (D + 1) + c]);
  }
}

// Zeroes the dQ columns of the shard range (dQ is written by accumulation).
__global__ void zero_dq_kernel(float* __restrict__ dQ, AttnShape s) {
  const long long nbh = s.bh_end - s.bh_begin;
  const long long per_bh = (long long)s.T * s.D;
  const long long total = nbh * per_bh;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < total;
       i += (long long)gridDim.x * blockDim.x) {
    const long long bh = s.bh_begin + i / per_bh;
    const long long rem = i % per_bh;
    const long long t = rem / s.D, c = rem % s.D;
    const long long b = bh / s.NH, h = bh % s.NH;
    dQ[(b * s.T + t) * s.N + h * s.D + c] = 0.0f;
  }
}

// computeQKV: three GEMMs [rows, N] x [N, N] sharing the X tile, 64x64 output
// tiles, 256 threads with 4x4 outputs each.
__global__ void __launch_bounds__(256) qkv_v0_kernel(const __nv_bfloat16* __restrict__ X,
                                                     const __nv_bfloat16* __restrict__ W0,
                                                     const __nv_bfloat16* __restrict__ W1,
                                                     const __nv_bfloat16* __restrict__ W2,
                                                     __nv_bfloat16* __restrict__ Y0,
                                                     __nv_bfloat16* __restrict__ Y1,
                                                     __nv_bfloat16* __restrict__ Y2, int N) {
  __shared__ float xs[16][64 + 1];
  __shared__ float ws[16][64];
  const __nv_bfloat16* W = blockIdx.z == 0 ? W0 : (blockIdx.z == 1 ? W1 : W2);
  __nv_bfloat16* Y = blockIdx.z == 0 ? Y0 : (blockIdx.z == 1 ? Y1 : Y2);
  const int n0 = blockIdx.x * 64, m0 = blockIdx.y * 64;
  const int tx = threadIdx.x % 16, ty = threadIdx.x / 16;
  float acc[4][4] = {};
  for (int k0 = 0; k0 < N; k0 += 16) {
    for (int i = threadIdx.x; i < 16 * 64; i += 256) {
      const int kk = i % 16, mm = i / 16;
      xs[kk][mm] = bf(X[(long long)(m0 + mm) * N + k0 + kk]);
      const int nn = i % 64, k2 = i / 64;
      ws[k2][nn] = bf(W[(long long)(k0 + k2) * N + n0 + nn]);
    }
    __syncthreads();
#pragma unroll
    for (int kk = 0; kk < 16; ++kk)
#pragma unroll
      for (int a = 0; a < 4; ++a)
#pragma unroll
        for (int c = 0; c < 4; ++c) acc[a][c] = fmaf(xs[kk][ty * 4 + a], ws[kk][tx * 4 + c], acc[a][c]);
    __syncthreads();
  }
#pragma unroll
  for (int a = 0; a < 4; ++a)
#pragma unroll
    for (int c = 0; c < 4; ++c)
      Y[(long long)(m0 + ty * 4 + a) * N + n0 + tx * 4 + c] = __float2bfloat16_rn(acc[a][c]);
}

template <class K>
cudaError_t set_smem(K kernel, size_t bytes) {
  return cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)bytes);
}

}  // namespace

cudaError_t launch_flash_fwd(const __nv_bfloat16* q, const __nv_bfloat16* k,
                             const __nv_bfloat16* v, __nv_bfloat16* out, float* lse,
                             const AttnShape& s, uint32_t*, cudaStream_t st) {
  const dim3 grid(s.T / TILE, s.bh_end - s.bh_begin);
  if (grid.y == 0) return cudaSuccess;
  if (s.D == 64) {
    const size_t bytes = sizeof(float) * TILE * (3 * (64 + 1) + 64);
    cudaError_t e = set_smem(fwd_v0_kernel<64>, bytes);
    if (e != cudaSuccess) return e;
    fwd_v0_kernel<64><<<grid, TILE, bytes, st>>>(q, k, v, out, lse, s);
    count_launches(1);
  } else {
    const size_t bytes = sizeof(float) * TILE * (3 * (128 + 1) + 128);
    cudaError_t e = set_smem(fwd_v0_kernel<128>, bytes);
    if (e != cudaSuccess) return e;
    fwd_v0_kernel<128><<<grid, TILE, bytes, st>>>(q, k, v, out, lse, s);
    count_launches(1);
  }
  return cudaGetLastError();
}

cudaError_t launch_flash_bwd(const __nv_bfloat16* dO, const __nv_bfloat16* Dv,
                             const float* lse, const __nv_bfloat16* q,
                             const __nv_bfloat16* k, const __nv_bfloat16* v, float* dQ,
                             __nv_bfloat16* dK, __nv_bfloat16* dV, const AttnShape& s,
                             uint32_t*, cudaStream_t st) {
  const dim3 grid(s.T / TILE, s.bh_end - s.bh_begin);
  if (grid.y == 0) return cudaSuccess;
  zero_dq_kernel<<<1184, 256, 0, st>>>(dQ, s);
    count_launches(1);
  if (s.D == 64) {
    const size_t bytes = sizeof(float) * (TILE * (4 * (64 + 1) + 2 * 64 + (TILE + 1) + 2));
    cudaError_t e = set_smem(bwd_v0_kernel<64>, bytes);
    if (e != cudaSuccess) return e;
    bwd_v0_kernel<64><<<grid, TILE, bytes, st>>>(dO, Dv, lse, q, k, v, dQ, dK, dV, s);
    count_launches(1);
  } else {
    const size_t bytes = sizeof(float) * (TILE * (4 * (128 + 1) + 2 * 128 + (TILE + 1) + 2));
    cudaError_t e = set_smem(bwd_v0_kernel<128>, bytes);
    if (e != cudaSuccess) return e;
    bwd_v0_kernel<128><<<grid, TILE, bytes, st>>>(dO, Dv, lse, q, k, v, dQ, dK, dV, s);
    count_launches(1);
  }
  return cudaGetLastError();
}

cudaError_t launch_qkv(const __nv_bfloat16* X, __nv_bfloat16* q, __nv_bfloat16* k,
                       __nv_bfloat16* v, const __nv_bfloat16* qw, const __nv_bfloat16* kw,
                       const __nv_bfloat16* vw, int rows, int N, uint32_t*, cudaStream_t st) {
  const dim3 grid(N / 64, rows / 64, 3);
  qkv_v0_kernel<<<grid, 256, 0, st>>>(X, qw, kw, vw, q, k, v, N);
    count_launches(1);
  return cudaGetLastError();
}

}  // namespace ma
