// train_sm100.cu -- the element-wise, row-wise and optimizer kernels of
// metalLLM's training step (config 5) around the attention path:
//   embedForward/Backward  embed.metal:9-34 (+ the positional residualAdd,
//                          model.h:438; the positional gradient is the batch
//                          sum of the embedding-output gradient, model.h:284)
//   layernormForward/Backward  layernorm.metal:10-127
//   castFloatToBfloat      elementwise.metal:7-71 (residualAdd is fused into
//                          the GEMM and LayerNorm-backward epilogues)
//   lossForward/Backward   loss.metal:9-75 (mean over rows)
//   MetalStep (Adam) with the gradient gather and weight scatter of
//   model.h:726-757 in one pass   optimstep.metal:15-42
// (the ReLU and mask multiply of mlp.metal:45-51, 116-121 are GEMM epilogues).
// They are memory-bound: 16-byte vector accesses, one warp per row for the
// row reductions (fp32 math), block partial sums + one atomic per column and
// block for the LayerNorm parameter gradients.
#include "common.cuh"

namespace ma {
namespace {

constexpr int EW_THREADS = 256;

inline int ew_blocks(long long n) {
  long long b = (n + EW_THREADS - 1) / EW_THREADS;
  if (b > 148LL * 16) b = 148LL * 16;
  return (int)(b < 1 ? 1 : b);
}

__device__ __forceinline__ float bf(__nv_bfloat16 x) { return __bfloat162float(x); }
__device__ __forceinline__ __nv_bfloat16 tobf(float x) { return __float2bfloat16_rn(x); }

// ---------------------------------------------------------------- embedding
// out[r] = bf16(E[tok[r]] + P[r % T])   (embedForward then residualAdd)
__global__ void embed_forward_kernel(const int* __restrict__ tok, const __nv_bfloat16* __restrict__ emb,
                                     const __nv_bfloat16* __restrict__ pos, __nv_bfloat16* __restrict__ out,
                                     int rows, int T, int E) {
  pdl_wait_and_release();
  const int r = blockIdx.x;
  if (r >= rows) return;
  const __nv_bfloat16* e = emb + (long long)tok[r] * E;
  const __nv_bfloat16* p = pos + (long long)(r % T) * E;
  __nv_bfloat16* o = out + (long long)r * E;
  for (int c = threadIdx.x; c < E; c += blockDim.x) o[c] = tobf(bf(e[c]) + bf(p[c]));
}

// dEmb[tok[r]] += dZ[r] (fp32 atomics; dEmb zeroed first)
__global__ void embed_backward_kernel(const int* __restrict__ tok, const __nv_bfloat16* __restrict__ dz,
                                      float* __restrict__ demb, int rows, int E) {
  pdl_wait_and_release();
  const int r = blockIdx.x;
  if (r >= rows) return;
  float* d = demb + (long long)tok[r] * E;
  const __nv_bfloat16* g = dz + (long long)r * E;
  for (int c = threadIdx.x; c < E; c += blockDim.x) atomicAdd(d + c, bf(g[c]));
}

// dPos[t][c] = bf16(sum_b dZ[b*T + t][c])
__global__ void pos_grad_kernel(const __nv_bfloat16* __restrict__ dz, __nv_bfloat16* __restrict__ dpos,
                                int B, int T, int E) {
  pdl_wait_and_release();
  const long long n = (long long)T * E;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n;
       i += (long long)gridDim.x * blockDim.x) {
    float s = 0.0f;
    for (int b = 0; b < B; ++b) s += bf(dz[(long long)b * n + i]);
    dpos[i] = tobf(s);
  }
}

// ---------------------------------------------------------------- layernorm
// One warp per row (fp32): mean, variance, stdev = sqrt(var + eps);
// x_norm = bf16((x - mean) / stdev); out = bf16(gamma * xn + beta) with the
// unrounded xn (layernorm.metal:10-71).
__global__ void layernorm_forward_kernel(const __nv_bfloat16* __restrict__ x, __nv_bfloat16* __restrict__ xn,
                                         __nv_bfloat16* __restrict__ out, const __nv_bfloat16* __restrict__ gamma,
                                         const __nv_bfloat16* __restrict__ beta, float* __restrict__ stdev,
                                         int rows, int cols, float eps) {
  pdl_wait_and_release();
  const int warp = (blockIdx.x * blockDim.x + threadIdx.x) / 32, lane = threadIdx.x % 32;
  if (warp >= rows) return;
  const __nv_bfloat16* xr = x + (long long)warp * cols;
  float s = 0.0f;
  for (int c = lane; c < cols; c += 32) s += bf(xr[c]);
#pragma unroll
  for (int o = 16; o; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
  const float mean = s / cols;
  float v = 0.0f;
  for (int c = lane; c < cols; c += 32) {
    const float d = bf(xr[c]) - mean;
    v += d * d;
  }
#pragma unroll
  for (int o = 16; o; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  const float sd = sqrtf(v / cols + eps);
  const float rs = 1.0f / sd;
  if (lane == 0) stdev[warp] = sd;
  for (int c = lane; c < cols; c += 32) {
    const float n = (bf(xr[c]) - mean) * rs;
    xn[(long long)warp * cols + c] = tobf(n);
    out[(long long)warp * cols + c] = tobf(bf(gamma[c]) * n + bf(beta[c]));
  }
}

// Backward (layernorm.metal:74-127), dZ rewritten in place with dX:
//   g = dZ * gamma; dX = (g - mean(g) - xn * mean(g * xn)) / stdev;
//   dGamma += dZ * xn, dBeta += dZ (block partial sums, one atomic per column).
// One warp per row, WARPS rows per block.
constexpr int LN_WARPS = 8;
__global__ void layernorm_backward_kernel(__nv_bfloat16* __restrict__ dz, const __nv_bfloat16* __restrict__ xn,
                                          const __nv_bfloat16* __restrict__ gamma, const float* __restrict__ stdev,
                                          float* __restrict__ dgamma, float* __restrict__ dbeta, int rows,
                                          int cols, const __nv_bfloat16* __restrict__ res) {
  pdl_wait_and_release();
  extern __shared__ float red[];  // [2][cols]
  for (int c = threadIdx.x; c < 2 * cols; c += blockDim.x) red[c] = 0.0f;
  __syncthreads();
  const int lane = threadIdx.x % 32, w = threadIdx.x / 32;
  for (int row = blockIdx.x * LN_WARPS + w; row < rows; row += gridDim.x * LN_WARPS) {
    __nv_bfloat16* dr = dz + (long long)row * cols;
    const __nv_bfloat16* nr = xn + (long long)row * cols;
    float s1 = 0.0f, s2 = 0.0f;
    for (int c = lane; c < cols; c += 32) {
      const float d = bf(dr[c]), n = bf(nr[c]), g = d * bf(gamma[c]);
      s1 += g;
      s2 += g * n;
      atomicAdd(&red[c], d * n);
      atomicAdd(&red[cols + c], d);
    }
#pragma unroll
    for (int o = 16; o; o >>= 1) {
      s1 += __shfl_xor_sync(0xffffffffu, s1, o);
      s2 += __shfl_xor_sync(0xffffffffu, s2, o);
    }
    const float m1 = s1 / cols, m2 = s2 / cols, rs = 1.0f / stdev[row];
    __syncwarp();
    for (int c = lane; c < cols; c += 32) {
      const float g = bf(dr[c]) * bf(gamma[c]);
      const __nv_bfloat16 x = tobf(rs * (g - m1 - bf(nr[c]) * m2));
      dr[c] = res ? tobf(bf(x) + bf(res[(long long)row * cols + c])) : x;
    }
  }
  __syncthreads();
  for (int c = threadIdx.x; c < cols; c += blockDim.x) {
    atomicAdd(dgamma + c, red[c]);
    atomicAdd(dbeta + c, red[cols + c]);
  }
}

// Row kernels for cols <= 256*NCH (cols a multiple of 8): one warp per row,
// lane l holding the 8-column chunks l, l+32, ... (16-byte loads and stores),
// the row kept in registers between its passes.
__device__ __forceinline__ void unpack8(const uint4 u, float (&f)[8]) {
  const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&u);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float2 t = __bfloat1622float2(h[i]);
    f[2 * i] = t.x;
    f[2 * i + 1] = t.y;
  }
}
__device__ __forceinline__ uint4 pack8(const float (&f)[8]) {
  uint4 u;
  __nv_bfloat162* h = reinterpret_cast<__nv_bfloat162*>(&u);
#pragma unroll
  for (int i = 0; i < 4; ++i) h[i] = __floats2bfloat162_rn(f[2 * i], f[2 * i + 1]);
  return u;
}

template <int NCH>
__global__ void layernorm_forward_vec_kernel(const uint4* __restrict__ x, uint4* __restrict__ xn,
                                             uint4* __restrict__ out, const uint4* __restrict__ gamma,
                                             const uint4* __restrict__ beta, float* __restrict__ stdev, int rows,
                                             int cols, float eps) {
  pdl_wait_and_release();
  const int warp = (blockIdx.x * blockDim.x + threadIdx.x) / 32, lane = threadIdx.x % 32;
  if (warp >= rows) return;
  const int c8 = cols / 8;
  const long long rb = (long long)warp * c8;
  float v[NCH][8];
  float s = 0.0f;
#pragma unroll
  for (int k = 0; k < NCH; ++k) {
    const int c = lane + 32 * k;
    if (c < c8) {
      unpack8(x[rb + c], v[k]);
#pragma unroll
      for (int i = 0; i < 8; ++i) s += v[k][i];
    }
  }
#pragma unroll
  for (int o = 16; o; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
  const float mean = s / cols;
  float q = 0.0f;
#pragma unroll
  for (int k = 0; k < NCH; ++k)
    if (lane + 32 * k < c8)
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const float d = v[k][i] - mean;
        q += d * d;
      }
#pragma unroll
  for (int o = 16; o; o >>= 1) q += __shfl_xor_sync(0xffffffffu, q, o);
  const float sd = sqrtf(q / cols + eps);
  const float rs = 1.0f / sd;
  if (lane == 0) stdev[warp] = sd;
#pragma unroll
  for (int k = 0; k < NCH; ++k) {
    const int c = lane + 32 * k;
    if (c < c8) {
      float g[8], b[8], n[8], o[8];
      unpack8(gamma[c], g);
      unpack8(beta[c], b);
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        n[i] = (v[k][i] - mean) * rs;
        o[i] = g[i] * n[i] + b[i];
      }
      xn[rb + c] = pack8(n);
      out[rb + c] = pack8(o);
    }
  }
}

// Backward, dZ rewritten in place with dX (layernorm.metal:74-127); each
// lane keeps its columns' dGamma/dBeta partial sums in registers over the
// rows its warp visits, then the block reduces them in shared memory and adds
// one value per column into the fp32 outputs.
template <int NCH>
__global__ void __launch_bounds__(LN_WARPS * 32, 2) layernorm_backward_vec_kernel(uint4* __restrict__ dz, const uint4* __restrict__ xn,
                                              const uint4* __restrict__ gamma, const float* __restrict__ stdev,
                                              float* __restrict__ dgamma, float* __restrict__ dbeta, int rows,
                                              int cols, const uint4* __restrict__ res) {
  pdl_wait_and_release();
  extern __shared__ float red[];  // [warps][2][cols]: each warp's column partial sums
  const int lane = threadIdx.x % 32, w = threadIdx.x / 32, nw = blockDim.x / 32;
  const int c8 = cols / 8;
  float gm[NCH][8], pg[NCH][8], pb[NCH][8];
#pragma unroll
  for (int k = 0; k < NCH; ++k) {
    if (lane + 32 * k < c8) unpack8(gamma[lane + 32 * k], gm[k]);
#pragma unroll
    for (int i = 0; i < 8; ++i) pg[k][i] = pb[k][i] = 0.0f;
  }
  // rows of this warp; the next row's loads are issued before the current
  // row is computed, so each warp keeps two rows in flight
  const int stride = gridDim.x * nw;
  uint4 ld[NCH], ln[NCH], lr[NCH];
  float lsd = 1.0f;
  auto load_row = [&](int row) {
    const long long rb = (long long)row * c8;
#pragma unroll
    for (int k = 0; k < NCH; ++k) {
      const int c = lane + 32 * k;
      if (c < c8) {
        ld[k] = dz[rb + c];
        ln[k] = __ldg(xn + rb + c);
        if (res) lr[k] = __ldg(res + rb + c);
      }
    }
    lsd = __ldg(stdev + row);
  };
  int row = blockIdx.x * nw + w;
  if (row < rows) load_row(row);
  for (; row < rows; row += stride) {
    const long long rb = (long long)row * c8;
    float d[NCH][8], n[NCH][8];
    uint4 qr[NCH];  // the residual, unpacked at the store
#pragma unroll
    for (int k = 0; k < NCH; ++k) {
      if (lane + 32 * k < c8) {
        unpack8(ld[k], d[k]);
        unpack8(ln[k], n[k]);
        qr[k] = lr[k];
      }
    }
    const float rs = 1.0f / lsd;
    if (row + stride < rows) load_row(row + stride);
    float s1 = 0.0f, s2 = 0.0f;
#pragma unroll
    for (int k = 0; k < NCH; ++k) {
      if (lane + 32 * k < c8) {
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          const float g = d[k][i] * gm[k][i];
          s1 += g;
          s2 += g * n[k][i];
          pg[k][i] += d[k][i] * n[k][i];
          pb[k][i] += d[k][i];
        }
      }
    }
#pragma unroll
    for (int o = 16; o; o >>= 1) {
      s1 += __shfl_xor_sync(0xffffffffu, s1, o);
      s2 += __shfl_xor_sync(0xffffffffu, s2, o);
    }
    const float m1 = s1 / cols, m2 = s2 / cols;
#pragma unroll
    for (int k = 0; k < NCH; ++k) {
      const int c = lane + 32 * k;
      if (c < c8) {
        float r[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) r[i] = rs * (d[k][i] * gm[k][i] - m1 - n[k][i] * m2);
        if (res) {  // the following residual add, on the rounded dX
          float q[8];
          unpack8(qr[k], q);
#pragma unroll
          for (int i = 0; i < 8; ++i) r[i] = __bfloat162float(__float2bfloat16_rn(r[i])) + q[i];
        }
        dz[rb + c] = pack8(r);
      }
    }
  }
  // this warp's partials to its own rows of the block buffer (16-byte
  // stores, no atomics), then one thread per column sums the warps and adds
  // the block's total into the output
  float* wr = red + (size_t)w * 2 * cols;
#pragma unroll
  for (int k = 0; k < NCH; ++k) {
    const int c = lane + 32 * k;
    if (c < c8) {
      float4* g4 = reinterpret_cast<float4*>(wr + c * 8);
      float4* b4 = reinterpret_cast<float4*>(wr + cols + c * 8);
      g4[0] = make_float4(pg[k][0], pg[k][1], pg[k][2], pg[k][3]);
      g4[1] = make_float4(pg[k][4], pg[k][5], pg[k][6], pg[k][7]);
      b4[0] = make_float4(pb[k][0], pb[k][1], pb[k][2], pb[k][3]);
      b4[1] = make_float4(pb[k][4], pb[k][5], pb[k][6], pb[k][7]);
    }
  }
  __syncthreads();
  for (int c = threadIdx.x; c < 2 * cols; c += blockDim.x) {
    float t = 0.0f;
    for (int q = 0; q < nw; ++q) t += red[(size_t)q * 2 * cols + c];
    atomicAdd(c < cols ? dgamma + c : dbeta + (c - cols), t);
  }
}

// ---------------------------------------------------------------- glue

__global__ void cast_kernel(const float4* __restrict__ in, uint2* __restrict__ out, long long n4) {
  pdl_wait_and_release();
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n4;
       i += (long long)gridDim.x * blockDim.x) {
    const float4 v = in[i];
    __nv_bfloat162 lo = __floats2bfloat162_rn(v.x, v.y), hi = __floats2bfloat162_rn(v.z, v.w);
    out[i] = make_uint2(*reinterpret_cast<uint32_t*>(&lo), *reinterpret_cast<uint32_t*>(&hi));
  }
}

// ---------------------------------------------------------------- loss
// One warp per row: lse = max + ln(sum exp(x - max)); out = lse - x[y]
// (loss.metal:9-59).
__global__ void loss_forward_kernel(const __nv_bfloat16* __restrict__ x, const int* __restrict__ y,
                                    float* __restrict__ out, float* __restrict__ lse, int rows, int cols) {
  pdl_wait_and_release();
  const int warp = (blockIdx.x * blockDim.x + threadIdx.x) / 32, lane = threadIdx.x % 32;
  if (warp >= rows) return;
  const __nv_bfloat16* xr = x + (long long)warp * cols;
  float m = -INFINITY;
  for (int c = lane; c < cols; c += 32) m = fmaxf(m, bf(xr[c]));
#pragma unroll
  for (int o = 16; o; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
  float s = 0.0f;
  for (int c = lane; c < cols; c += 32) s += expf(bf(xr[c]) - m);
#pragma unroll
  for (int o = 16; o; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
  if (lane == 0) {
    const float l = m + logf(s);
    lse[warp] = l;
    out[warp] = l - bf(xr[y[warp]]);
  }
}

// mean of the per-row losses into *mean (one block, fixed order)
__global__ void mean_kernel(const float* __restrict__ v, int n, float* __restrict__ mean) {
  pdl_wait_and_release();
  __shared__ float part[32];
  float s = 0.0f;
  for (int i = threadIdx.x; i < n; i += blockDim.x) s += v[i];
#pragma unroll
  for (int o = 16; o; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
  if (threadIdx.x % 32 == 0) part[threadIdx.x / 32] = s;
  __syncthreads();
  if (threadIdx.x < 32) {
    s = threadIdx.x < (int)(blockDim.x / 32) ? part[threadIdx.x] : 0.0f;
#pragma unroll
    for (int o = 16; o; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
    if (threadIdx.x == 0) *mean = s / n;
  }
}

// dZ = bf16((exp(x - lse) - [c == y]) / rows)   (loss.metal:61-75)
__global__ void loss_backward_kernel(const __nv_bfloat16* __restrict__ x, const int* __restrict__ y,
                                     const float* __restrict__ lse, __nv_bfloat16* __restrict__ dz, int rows,
                                     int cols) {
  pdl_wait_and_release();
  const long long n = (long long)rows * cols;
  const float inv = 1.0f / rows;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n;
       i += (long long)gridDim.x * blockDim.x) {
    const int r = (int)(i / cols), c = (int)(i % cols);
    const float p = expf(bf(x[i]) - lse[r]);
    dz[i] = tobf((p - (c == y[r] ? 1.0f : 0.0f)) * inv);
  }
}

// ---------------------------------------------------------------- optimizer
// Adam on the flat fp32 master parameters with bf16 gradients and moments
// (optimstep.metal:15-42): v = b2 v + (1-b2) g^2; m = b1 m + (1-b1) g;
// p -= lr_t * m * rsqrt(v + eps).
// The whole optimizer step in one pass: for parameter blockIdx.y, each
// element's gradient is rounded to bf16 (the gather into the flat gradient
// array of model.h:726-742), Adam updates the fp32 master and bf16 moments at
// the parameter's flat offset (optimstep.metal:15-42), and the rounded master
// is written back to the bf16 weight (the scatter) -- the same values as
// gather, adam_kernel and scatter in sequence, in one launch.
__global__ void adam_fused_kernel(const AdamSegment* __restrict__ segs, float* __restrict__ p,
                                  __nv_bfloat16* __restrict__ m, __nv_bfloat16* __restrict__ v, float b1,
                                  float b2, float lr_t, float ob1, float ob2, float eps) {
  pdl_wait_and_release();
  const AdamSegment sg = segs[blockIdx.y];
  // four elements per step (counts are multiples of 4, offsets of 8): 16-byte
  // fp32 and 8-byte bf16 accesses
  const long long n4 = sg.count / 4;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n4;
       i += (long long)gridDim.x * blockDim.x) {
    float g[4];
    if (sg.grad_f32) {
      const float4 gf = static_cast<const float4*>(sg.grad)[i];
      g[0] = bf(tobf(gf.x));
      g[1] = bf(tobf(gf.y));
      g[2] = bf(tobf(gf.z));
      g[3] = bf(tobf(gf.w));
    } else {
      const uint2 gb = static_cast<const uint2*>(sg.grad)[i];
      const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&gb);
      const float2 lo = __bfloat1622float2(h[0]), hi = __bfloat1622float2(h[1]);
      g[0] = lo.x;
      g[1] = lo.y;
      g[2] = hi.x;
      g[3] = hi.y;
    }
    const long long j = sg.offset / 4 + i;
    float4 pv = reinterpret_cast<float4*>(p)[j];
    const uint2 mv = reinterpret_cast<const uint2*>(m)[j], vv = reinterpret_cast<const uint2*>(v)[j];
    const __nv_bfloat16* mh = reinterpret_cast<const __nv_bfloat16*>(&mv);
    const __nv_bfloat16* vh = reinterpret_cast<const __nv_bfloat16*>(&vv);
    float* pp = reinterpret_cast<float*>(&pv);
    __nv_bfloat16 mo[4], vo[4], wo[4];
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const float vi = fmaf(b2, bf(vh[e]), ob2 * (g[e] * g[e]));
      const float mi = fmaf(b1, bf(mh[e]), ob1 * g[e]);
      vo[e] = tobf(vi);
      mo[e] = tobf(mi);
      pp[e] = pp[e] - lr_t * mi * rsqrtf(vi + eps);
      wo[e] = tobf(pp[e]);
    }
    reinterpret_cast<float4*>(p)[j] = pv;
    reinterpret_cast<uint2*>(m)[j] = *reinterpret_cast<const uint2*>(mo);
    reinterpret_cast<uint2*>(v)[j] = *reinterpret_cast<const uint2*>(vo);
    reinterpret_cast<uint2*>(sg.weight)[i] = *reinterpret_cast<const uint2*>(wo);
  }
}

}  // namespace

// ---------------------------------------------------------------- launchers
cudaError_t launch_embed_forward(const int* tok, const __nv_bfloat16* emb, const __nv_bfloat16* pos,
                                 __nv_bfloat16* out, int rows, int T, int E, cudaStream_t st) {
  launch_pdl(embed_forward_kernel, rows, 128, 0, st, tok, emb, pos, out, rows, T, E);
  count_launches(1);
  return cudaGetLastError();
}

cudaError_t launch_embed_backward(const int* tok, const __nv_bfloat16* dz, float* demb, __nv_bfloat16* dpos,
                                  int B, int T, int V, int E, cudaStream_t st) {
  cudaError_t e = cudaMemsetAsync(demb, 0, (size_t)V * E * sizeof(float), st);
  if (e != cudaSuccess) return e;
  launch_pdl(embed_backward_kernel, B * T, 128, 0, st, tok, dz, demb, B * T, E);
  launch_pdl(pos_grad_kernel, ew_blocks((long long)T * E), EW_THREADS, 0, st, dz, dpos, B, T, E);
  count_launches(2);
  return cudaGetLastError();
}

cudaError_t launch_layernorm_forward(const __nv_bfloat16* x, __nv_bfloat16* xn, __nv_bfloat16* out,
                                     const __nv_bfloat16* gamma, const __nv_bfloat16* beta, float* stdev,
                                     int rows, int cols, float eps, cudaStream_t st) {
  const int wpb = 8;
  const dim3 grid((rows + wpb - 1) / wpb), block(wpb * 32);
  const int nch = (cols + 255) / 256;
  auto u = [](const void* p) { return reinterpret_cast<const uint4*>(p); };
  auto um = [](void* p) { return reinterpret_cast<uint4*>(p); };
  if (cols % 8 == 0 && nch <= 4) {
    switch (nch) {
      case 1: launch_pdl(layernorm_forward_vec_kernel<1>, grid, block, 0, st, u(x), um(xn), um(out), u(gamma), u(beta), stdev, rows, cols, eps); break;
      case 2: launch_pdl(layernorm_forward_vec_kernel<2>, grid, block, 0, st, u(x), um(xn), um(out), u(gamma), u(beta), stdev, rows, cols, eps); break;
      case 3: launch_pdl(layernorm_forward_vec_kernel<3>, grid, block, 0, st, u(x), um(xn), um(out), u(gamma), u(beta), stdev, rows, cols, eps); break;
      default: launch_pdl(layernorm_forward_vec_kernel<4>, grid, block, 0, st, u(x), um(xn), um(out), u(gamma), u(beta), stdev, rows, cols, eps); break;
    }
  } else {
    launch_pdl(layernorm_forward_kernel, grid, block, 0, st, x, xn, out, gamma, beta, stdev, rows, cols, eps);
  }
  count_launches(1);
  return cudaGetLastError();
}

cudaError_t launch_layernorm_backward(__nv_bfloat16* dz, const __nv_bfloat16* xn, const __nv_bfloat16* gamma,
                                      const float* stdev, float* dgamma, float* dbeta, int rows, int cols,
                                      cudaStream_t st, const __nv_bfloat16* res) {
  cudaError_t e = cudaMemsetAsync(dgamma, 0, (size_t)cols * sizeof(float), st);
  if (e == cudaSuccess) e = cudaMemsetAsync(dbeta, 0, (size_t)cols * sizeof(float), st);
  if (e != cudaSuccess) return e;
  const int nch = (cols + 255) / 256;
  if (cols % 8 == 0 && nch <= 4) {
    // two blocks per SM (the register use allows two): enough rows in
    // flight, few column atomics at the end
    int blocks = (rows + LN_WARPS - 1) / LN_WARPS;
    if (blocks > 2 * 148) blocks = 2 * 148;
    const size_t sm = (size_t)LN_WARPS * 2 * cols * sizeof(float);
    uint4* d = reinterpret_cast<uint4*>(dz);
    const uint4* n = reinterpret_cast<const uint4*>(xn);
    const uint4* g = reinterpret_cast<const uint4*>(gamma);
    const uint4* rv = reinterpret_cast<const uint4*>(res);
    auto run = [&](auto kern) {
      if (sm > 48 * 1024) cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sm);
      launch_pdl(kern, blocks, LN_WARPS * 32, sm, st, d, n, g, stdev, dgamma, dbeta, rows, cols, rv);
    };
    switch (nch) {
      case 1: run(layernorm_backward_vec_kernel<1>); break;
      case 2: run(layernorm_backward_vec_kernel<2>); break;
      case 3: run(layernorm_backward_vec_kernel<3>); break;
      default: run(layernorm_backward_vec_kernel<4>); break;
    }
  } else {
    int blocks = (rows + LN_WARPS - 1) / LN_WARPS;
    if (blocks > 148 * 4) blocks = 148 * 4;
    launch_pdl(layernorm_backward_kernel, blocks, LN_WARPS * 32, 2 * cols * sizeof(float), st, dz, xn, gamma, stdev,
                                                                                         dgamma, dbeta, rows, cols,
                                                                                         res);
  }
  count_launches(1);
  return cudaGetLastError();
}

cudaError_t launch_cast_f32_bf16(const float* in, __nv_bfloat16* out, long long n, cudaStream_t st) {
  const long long n4 = n / 4;
  launch_pdl(cast_kernel, ew_blocks(n4), EW_THREADS, 0, st, reinterpret_cast<const float4*>(in),
                                                    reinterpret_cast<uint2*>(out), n4);
  count_launches(1);
  return cudaGetLastError();
}

cudaError_t launch_loss_forward(const __nv_bfloat16* x, const int* y, float* out, float* lse, float* mean,
                                int rows, int cols, cudaStream_t st) {
  const int wpb = 8;
  launch_pdl(loss_forward_kernel, (rows + wpb - 1) / wpb, wpb * 32, 0, st, x, y, out, lse, rows, cols);
  launch_pdl(mean_kernel, 1, 1024, 0, st, out, rows, mean);
  count_launches(2);
  return cudaGetLastError();
}

cudaError_t launch_loss_backward(const __nv_bfloat16* x, const int* y, const float* lse, __nv_bfloat16* dz,
                                 int rows, int cols, cudaStream_t st) {
  launch_pdl(loss_backward_kernel, ew_blocks((long long)rows * cols), EW_THREADS, 0, st, x, y, lse, dz, rows, cols);
  count_launches(1);
  return cudaGetLastError();
}

cudaError_t launch_adam_fused(const AdamSegment* segs, int nsegs, long long max_count, float* p,
                              __nv_bfloat16* m, __nv_bfloat16* v, float lr_t, cudaStream_t st) {
  if (nsegs <= 0) return cudaSuccess;
  long long bx = (max_count / 4 + 2 * EW_THREADS - 1) / (2 * EW_THREADS);
  if (bx < 1) bx = 1;
  launch_pdl(adam_fused_kernel, dim3((unsigned)bx, (unsigned)nsegs), EW_THREADS, 0, st, segs, p, m, v, 0.9f, 0.999f, lr_t,
                                                                             0.1f, 0.001f, 1e-8f);
  count_launches(1);
  return cudaGetLastError();
}
}  // namespace ma
