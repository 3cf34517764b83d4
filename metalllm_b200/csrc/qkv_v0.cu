// qkv_v0.cu -- first correct CUDA path of computeQKV (attention.metal:19-53):
// three GEMMs [rows, N] x [N, N] with fp32 FMA accumulation in shared-memory
// tiles, bf16 outputs.
#include "common.cuh"

namespace ma {
namespace {

constexpr int TILE = 64;

__device__ __forceinline__ float bf(const __nv_bfloat16 x) { return __bfloat162float(x); }

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

}  // namespace

cudaError_t launch_qkv(const __nv_bfloat16* X, __nv_bfloat16* q, __nv_bfloat16* k,
                       __nv_bfloat16* v, const __nv_bfloat16* qw, const __nv_bfloat16* kw,
                       const __nv_bfloat16* vw, int rows, int N, uint32_t*, cudaStream_t st) {
  const dim3 grid(N / 64, rows / 64, 3);
  qkv_v0_kernel<<<grid, 256, 0, st>>>(X, qw, kw, vw, q, k, v, N);
    count_launches(1);
  return cudaGetLastError();
}

}  // namespace ma
