// compute_d.cu -- computeD (attention.metal:166-195):
//   D[row, h] = bf16( sum_{c<D} dO[row, h*D+c] * O[row, h*D+c] )
// with the products and the sum in fp32 (the sum rounds to bf16 once).
//
// HBM-bound: per (row, head) item it reads 2*D bf16 values and writes one
// bf16.  Because a row holds its NH head slabs back to back, item
// i = row*NH + h starts at element i*D of dO/O and its result is element i of
// D: the whole batch is one flat, contiguous stream of D-element items.  G
// lanes (G*16 bytes = one item of each tensor) cooperate on an item with
// 16-byte loads, then reduce with shuffles; a warp covers 32/G consecutive
// items, so every load instruction of a warp reads 512 contiguous bytes.
#include "common.cuh"

namespace ma {
namespace {

__device__ __forceinline__ float dot8_bf16(uint4 a, uint4 b) {
  const __nv_bfloat162* x = reinterpret_cast<const __nv_bfloat162*>(&a);
  const __nv_bfloat162* y = reinterpret_cast<const __nv_bfloat162*>(&b);
  float acc = 0.0f;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float2 fx = __bfloat1622float2(x[i]);
    const float2 fy = __bfloat1622float2(y[i]);
    acc = fmaf(fx.x, fy.x, acc);
    acc = fmaf(fx.y, fy.y, acc);
  }
  return acc;
}

// G lanes per item (G = D/8: 8 for D=64, 16 for D=128).  Items outside the
// (batch, head) shard range are skipped.
template <int G>
__global__ void __launch_bounds__(256) compute_d_kernel(const uint4* __restrict__ dO,
                                                        const uint4* __restrict__ O,
                                                        __nv_bfloat16* __restrict__ Dv,
                                                        long long item_begin,
                                                        long long item_end, int T, int NH,
                                                        int bh_begin, int bh_end) {
  pdl_wait_and_release();
  const int lane_in_item = threadIdx.x % G;
  const long long items_per_block = blockDim.x / G;
  const bool full_range = (bh_begin == 0 && bh_end < 0);
  // The loop bound is warp-uniform (the shuffles below need the full warp);
  // lanes past item_end only mask their loads and stores.
  const long long warp_first = (threadIdx.x / 32) * (32 / G);
  for (long long base = item_begin + blockIdx.x * items_per_block + warp_first;
       base < item_end; base += (long long)gridDim.x * items_per_block) {
    const long long it = base + (threadIdx.x % 32) / G;
    bool active = it < item_end;
    if (active && !full_range) {
      const long long row = it / NH;
      const int h = (int)(it - row * NH);
      const long long b = row / T;
      const long long bh = b * NH + h;
      active = bh >= bh_begin && bh < bh_end;
    }
    float acc = 0.0f;
    if (active) {
      const long long off = it * G + lane_in_item;
      acc = dot8_bf16(__ldcs(dO + off), __ldcs(O + off));
    }
#pragma unroll
    for (int m = G / 2; m >= 1; m >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, m);
    if (active && lane_in_item == 0) Dv[it] = __float2bfloat16_rn(acc);
  }
}

}  // namespace

cudaError_t launch_compute_d(const __nv_bfloat16* dO, const __nv_bfloat16* O,
                             __nv_bfloat16* Dv, const AttnShape& s, cudaStream_t st) {
  const long long rows_per_b = s.T;
  const int b0 = s.bh_begin / s.NH;
  const int b1 = (s.bh_end + s.NH - 1) / s.NH;
  const long long item_begin = (long long)b0 * rows_per_b * s.NH;
  const long long item_end = (long long)b1 * rows_per_b * s.NH;
  const bool full = (s.bh_begin % s.NH == 0) && (s.bh_end % s.NH == 0);
  const int bh_end_arg = full ? -1 : s.bh_end;
  const int bh_begin_arg = full ? 0 : s.bh_begin;
  const long long items = item_end - item_begin;
  if (items <= 0) return cudaSuccess;
  int dev = 0, sms = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const int threads = 256;
  if (s.D == 64) {
    const long long per_block = threads / 8;
    long long blocks = (items + per_block - 1) / per_block;
    blocks = blocks < (long long)sms * 16 ? blocks : (long long)sms * 16;
    launch_pdl(compute_d_kernel<8>, (unsigned)blocks, threads, 0, st, 
        reinterpret_cast<const uint4*>(dO), reinterpret_cast<const uint4*>(O), Dv, item_begin,
        item_end, s.T, s.NH, bh_begin_arg, bh_end_arg);
    count_launches(1);
  } else {
    const long long per_block = threads / 16;
    long long blocks = (items + per_block - 1) / per_block;
    blocks = blocks < (long long)sms * 16 ? blocks : (long long)sms * 16;
    launch_pdl(compute_d_kernel<16>, (unsigned)blocks, threads, 0, st, 
        reinterpret_cast<const uint4*>(dO), reinterpret_cast<const uint4*>(O), Dv, item_begin,
        item_end, s.T, s.NH, bh_begin_arg, bh_end_arg);
    count_launches(1);
  }
  return cudaGetLastError();
}

}  // namespace ma
