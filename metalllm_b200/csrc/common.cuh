// common.cuh -- helpers shared by the kernels of libmetalattn (sm_100a only).
#pragma once

#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <utility>

#include "../../include/metalattn.h"

namespace ma {

// Programmatic dependent launch: wait until the previous kernel in the stream
// has completed and its writes are visible (a no-op when the kernel was not
// launched as a dependent), then let the next kernel be scheduled.
__device__ __forceinline__ void pdl_wait_and_release() {
  asm volatile("griddepcontrol.wait;" ::: "memory");
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

// Kernel launch with programmatic dependent launch allowed: the kernel may be
// scheduled while the previous kernel in the stream is still draining; every
// kernel of this library starts with pdl_wait_and_release(), which waits for
// that kernel's completion before any memory is touched, so stream order is
// kept.  Errors are reported through cudaGetLastError as for <<<>>>.
template <typename... KArgs, typename... Args>
inline void launch_pdl(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st,
                       Args&&... args) {
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  cudaLaunchKernelEx(&cfg, kern, std::forward<Args>(args)...);
}


// Per-kernel bits of the device status word (ma_device_status).
enum : uint32_t {
  STATUS_FWD_TIMEOUT = MA_STATUS_FWD_TIMEOUT,
  STATUS_BWD_TIMEOUT = MA_STATUS_BWD_TIMEOUT,
  STATUS_QKV_TIMEOUT = MA_STATUS_QKV_TIMEOUT,
  STATUS_GEMM_TIMEOUT = MA_STATUS_GEMM_TIMEOUT,
};

// Test hook of the bounded waits' time-out path (ma_debug_expire_next_wait):
// returns the wait, in ns, that this launch of the kernel with status bit
// `kernel_bit` must let run out on a barrier nothing arrives at, or 0; a
// request is consumed by the launch that takes it.
uint32_t take_expire_request(uint32_t kernel_bit);

// Problem description shared by the attention kernels.  Row strides are in
// elements: a (batch, position) row of Q/K/V/O/dO/dK/dV/dQ holds N = NH*D
// values; l and D hold NH values per row.
struct AttnShape {
  int T;         // sequence length (AttentionParams.M)
  int N;         // NH*D
  int D;         // head size
  int NH;        // heads
  int B;         // batch
  int bh_begin;  // flat (b*NH + h) shard range
  int bh_end;
};

// Adds n to the process-wide kernel launch counter (ma_kernel_launch_count).
void count_launches(unsigned n);

// Launchers (each returns the cudaError_t of its launch).
cudaError_t launch_compute_d(const __nv_bfloat16* dO, const __nv_bfloat16* O,
                             __nv_bfloat16* Dv, const AttnShape& s, cudaStream_t st);
// dO, Dv (D = 64 only, both or neither): computeD fused into the epilogue.
// dQz (optional): the forward also writes zeros to the dQ columns of the
// shard's rows, for a following backward that accumulates into dQ.
cudaError_t launch_flash_fwd(const __nv_bfloat16* q, const __nv_bfloat16* k,
                             const __nv_bfloat16* v, __nv_bfloat16* out, float* lse,
                             const AttnShape& s, uint32_t* status, cudaStream_t st,
                             const __nv_bfloat16* dO = nullptr, __nv_bfloat16* Dv = nullptr,
                             float* dQz = nullptr);
// Zeroes the dQ columns of the shard's (batch, head) slabs (a memset for the
// whole batch).
cudaError_t launch_zero_dq(float* dQ, const AttnShape& s, cudaStream_t st);
// accumulate_dq: dQ += the backward's dQ (dQ holds zeros or earlier partial
// sums on entry); otherwise the launcher zeroes the shard's dQ first.
cudaError_t launch_flash_bwd(const __nv_bfloat16* dO, const __nv_bfloat16* Dv,
                             const float* lse, const __nv_bfloat16* q,
                             const __nv_bfloat16* k, const __nv_bfloat16* v, float* dQ,
                             __nv_bfloat16* dK, __nv_bfloat16* dV, const AttnShape& s,
                             uint32_t* status, cudaStream_t st, bool accumulate_dq = false);
cudaError_t launch_qkv(const __nv_bfloat16* X, __nv_bfloat16* q, __nv_bfloat16* k,
                       __nv_bfloat16* v, const __nv_bfloat16* qw, const __nv_bfloat16* kw,
                       const __nv_bfloat16* vw, int rows, int N, uint32_t* status,
                       cudaStream_t st);

// GEMMs around attention (gemm_sm100.cu); rows = B*M activation rows, n = N.
cudaError_t launch_proj_forward(const __nv_bfloat16* attn, const __nv_bfloat16* w, __nv_bfloat16* out,
                                int rows, int n, uint32_t* status, cudaStream_t st);
cudaError_t launch_proj_backward_dx(const __nv_bfloat16* dz, const __nv_bfloat16* w,
                                    __nv_bfloat16* dattn, int rows, int n, uint32_t* status,
                                    cudaStream_t st);
cudaError_t launch_proj_backward_dw(const __nv_bfloat16* attn, const __nv_bfloat16* dz,
                                    __nv_bfloat16* dw, int rows, int n, uint32_t* status,
                                    cudaStream_t st);
cudaError_t launch_proj_backward_dx_d(const __nv_bfloat16* dz, const __nv_bfloat16* w, __nv_bfloat16* dattn,
                                      const __nv_bfloat16* attn, __nv_bfloat16* d, int rows, int n, int head_dim,
                                      uint32_t* status, cudaStream_t st);
cudaError_t launch_grad_dx(float* dx, const __nv_bfloat16* qw, const __nv_bfloat16* kw,
                           const __nv_bfloat16* vw, const float* dq, const __nv_bfloat16* dk,
                           const __nv_bfloat16* dv, int rows, int n, uint32_t* status, cudaStream_t st);
cudaError_t launch_grad_dw(const __nv_bfloat16* x, const float* dq, const __nv_bfloat16* dk,
                           const __nv_bfloat16* dv, float* dqw, __nv_bfloat16* dkw, __nv_bfloat16* dvw,
                           int rows, int n, uint32_t* status, cudaStream_t st);

cudaError_t launch_gemm_bf16(const __nv_bfloat16* A, bool a_mn, const __nv_bfloat16* B, bool b_mn,
                             __nv_bfloat16* C, int M, int N, int K, uint32_t* status, cudaStream_t st);
cudaError_t launch_gemm_bf16_act(const __nv_bfloat16* A, const __nv_bfloat16* B, bool b_mn, __nv_bfloat16* C,
                                 uint8_t* mask, const __nv_bfloat16* res, int act, int M, int N, int K,
                                 uint32_t* status, cudaStream_t st);
cudaError_t launch_gemm_splitk_f32(const __nv_bfloat16* A, const __nv_bfloat16* B, float* C, int M, int N,
                                   int K, uint32_t* status, cudaStream_t st, bool zero = true);
// The training step's computeGradDx/Dw on a bf16 copy of dQ; the weight
// gradients are fp32, split along K and added into zeroed outputs.
cudaError_t launch_grad_dw_splitk_f32(const __nv_bfloat16* x, const __nv_bfloat16* dq16, const __nv_bfloat16* dk,
                                      const __nv_bfloat16* dv, float* dqw, float* dkw, float* dvw, int rows, int n,
                                      uint32_t* status, cudaStream_t st);
cudaError_t launch_grad_dx_bf16(void* dx, bool dx_f32, const __nv_bfloat16* qw, const __nv_bfloat16* kw,
                                const __nv_bfloat16* vw, const __nv_bfloat16* dq16, const __nv_bfloat16* dk,
                                const __nv_bfloat16* dv, int rows, int n, uint32_t* status, cudaStream_t st);

// Training-step kernels (train_sm100.cu).
cudaError_t launch_embed_forward(const int* tok, const __nv_bfloat16* emb, const __nv_bfloat16* pos,
                                 __nv_bfloat16* out, int rows, int T, int E, cudaStream_t st);
cudaError_t launch_embed_backward(const int* tok, const __nv_bfloat16* dz, float* demb, __nv_bfloat16* dpos,
                                  int B, int T, int V, int E, cudaStream_t st);
cudaError_t launch_layernorm_forward(const __nv_bfloat16* x, __nv_bfloat16* xn, __nv_bfloat16* out,
                                     const __nv_bfloat16* gamma, const __nv_bfloat16* beta, float* stdev,
                                     int rows, int cols, float eps, cudaStream_t st);
// res (optional): dX is rounded to bf16 and res added (the residualAdd that
// follows the LayerNorm backward in model.h), one more rounding.
cudaError_t launch_layernorm_backward(__nv_bfloat16* dz, const __nv_bfloat16* xn, const __nv_bfloat16* gamma,
                                      const float* stdev, float* dgamma, float* dbeta, int rows, int cols,
                                      cudaStream_t st, const __nv_bfloat16* res = nullptr);

cudaError_t launch_cast_f32_bf16(const float* in, __nv_bfloat16* out, long long n, cudaStream_t st);


cudaError_t launch_loss_forward(const __nv_bfloat16* x, const int* y, float* out, float* lse, float* mean,
                                int rows, int cols, cudaStream_t st);
cudaError_t launch_loss_backward(const __nv_bfloat16* x, const int* y, const float* lse, __nv_bfloat16* dz,
                                 int rows, int cols, cudaStream_t st);


// One optimizer segment per parameter: its gradient (fp32 or bf16), its bf16
// weight, its element count and its offset into the flat master/moment arrays.
struct AdamSegment {
  const void* grad;
  __nv_bfloat16* weight;
  long long count;
  long long offset;
  int grad_f32;
};
cudaError_t launch_adam_fused(const AdamSegment* segs, int nsegs, long long max_count, float* p,
                              __nv_bfloat16* m, __nv_bfloat16* v, float lr_t, cudaStream_t st);
}  // namespace ma
