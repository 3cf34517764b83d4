/*
 * metalattn.h -- C ABI of the B200 (sm_100a) causal attention hot path of
 * metalLLM.  Each entry point replaces one Metal kernel dispatch of the
 * reference and keeps that kernel's buffer order, buffer layouts and dtypes.
 *
 * Layouts (row-major, a batch of B sequences stacked along the row axis):
 *   X, Q, K, V, O (attnOut), dO (dZAttn), dK, dV : bf16 [B][M][N]
 *   dQ                                           : fp32 [B][M][N]
 *   l (row logsumexp)                            : fp32 [B][M][NH]
 *   D (rowsum(dO*O))                             : bf16 [B][M][NH]
 *   Wq, Wk, Wv                                   : bf16 [N][N], row = input feature
 * where M = sequence length, N = NH*D, and head h owns columns h*D .. h*D+D-1.
 *
 * Conventions shared by every entry point:
 *   - Pointers are device pointers on the current CUDA device, 16-byte aligned.
 *   - Work is enqueued on `stream` (NULL = legacy default stream); nothing
 *     synchronises the host.  Results are ready when the stream is.
 *   - The return value is MA_OK or an MA_ERR_* code; ma_last_error_string()
 *     describes the last failure of the calling host thread.  No entry point
 *     exits, traps or prints.
 *   - Outputs are written, never accumulated: callers need not pre-zero
 *     dQ/dK/dV or Q/K/V (a caller that does, as model.h:418-424 and
 *     model.h:549-551 do, gets identical results).
 *   - Supported shapes: D in {64, 128}; any M >= 1 (the reference needs a
 *     multiple of 64, attention.metal:74; partial tiles are zero-filled on
 *     load and clipped on store here); N == NH*D; B >= 1.  computeQKV needs
 *     N a multiple of 64.  Anything else returns MA_ERR_SHAPE and computes
 *     nothing.
 *   - The library allocates nothing per call on the device except a cached
 *     4-byte error word per device.
 */
#ifndef METALATTN_H_
#define METALATTN_H_

#include <stdint.h>

#if defined(__GNUC__)
#define MA_API __attribute__((visibility("default")))
#else
#define MA_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

/* Shape carrier, laid out exactly as the reference's AttentionParams
 * (attention.metal:7-12, host twin main.cpp:114-119, filled model.h:178):
 * M = sequence length (BLOCK_SIZE), N = n_embed = NH*D, D = head size,
 * NH = number of heads.  Four uint32, 16 bytes. */
typedef struct AttentionParams {
  uint32_t M;
  uint32_t N;
  uint32_t D;
  uint32_t NH;
} AttentionParams;

/* A CUDA stream; binary-compatible with cudaStream_t / CUstream. */
typedef struct CUstream_st* ma_stream_t;

/* Raw bf16 bits (1 sign, 8 exponent, 7 mantissa), as the reference's bfloat. */
typedef uint16_t ma_bf16;

enum {
  MA_OK = 0,
  MA_ERR_SHAPE = 1,          /* unsupported or inconsistent AttentionParams / batch */
  MA_ERR_NULL = 2,           /* a required pointer is NULL */
  MA_ERR_ALIGN = 3,          /* a pointer is not 16-byte aligned */
  MA_ERR_CUDA = 4,           /* a CUDA runtime/driver call or launch failed */
  MA_ERR_DEVICE_TIMEOUT = 5, /* a kernel gave up on a bounded wait (see ma_device_status) */
  MA_ERR_RANGE = 6,          /* bh_begin/bh_end outside [0, B*NH] or reversed */
  MA_ERR_NO_DEVICE = 7,      /* no usable sm_100 device is current */
  MA_ERR_LIMIT = 8           /* a size exceeds a documented fixed limit */
};

/* computeQKV: Q = X*Wq, K = X*Wk, V = X*Wv, fp32 accumulation, bf16 outputs.
 * Replaces attention.metal:19-27 (buffers 0..7) dispatched at model.h:446-458.
 * X has B*p->M rows. */
MA_API int ma_computeQKV(const ma_bf16* X, ma_bf16* q, ma_bf16* k, ma_bf16* v,
                  const ma_bf16* q_w, const ma_bf16* k_w, const ma_bf16* v_w,
                  const AttentionParams* p, uint32_t B, ma_stream_t stream);

/* flashAttentionForward: causal softmax(Q K^T / sqrt(D)) V per (batch, head);
 * writes O (bf16) and l = rowmax + ln(rowsum) (fp32, natural log).
 * Replaces attention.metal:56-66 (buffers 0..5; the threadgroup buffers are
 * internal) dispatched at model.h:459-473. */
MA_API int ma_flashAttentionForward(const ma_bf16* q, const ma_bf16* k, const ma_bf16* v,
                             ma_bf16* out, float* l, const AttentionParams* p,
                             uint32_t B, ma_stream_t stream);

/* flashAttentionForward followed by computeD when dO is already known (an
 * attention-only step, or a recomputing backward): writes out, l as
 * ma_flashAttentionForward and D as ma_computeD(dO, out) would.  At D = 64 the
 * dot products are formed in the forward's epilogue from the bf16-rounded O
 * (one launch, O is not read back; D may differ from ma_computeD's by one
 * bf16 rounding step, the fp32 sum running in another order); at D = 128 the
 * two kernels run back to back.  No counterpart in the reference (its host
 * calls computeD in the backward, model.h:639-647). */
MA_API int ma_flashAttentionForwardComputeD(const ma_bf16* q, const ma_bf16* k, const ma_bf16* v,
                                            const ma_bf16* dO, ma_bf16* out, float* l, ma_bf16* D,
                                            const AttentionParams* p, uint32_t B, ma_stream_t stream);
MA_API int ma_flashAttentionForwardComputeD_shard(const ma_bf16* q, const ma_bf16* k, const ma_bf16* v,
                                                  const ma_bf16* dO, ma_bf16* out, float* l, ma_bf16* D,
                                                  const AttentionParams* p, uint32_t B, uint32_t bh_begin,
                                                  uint32_t bh_end, ma_stream_t stream);

/* computeD: D[row, h] = bf16(sum_c dO[row, h*D+c] * O[row, h*D+c]), fp32 sum.
 * Replaces attention.metal:166-171 (buffers 0..3) dispatched at model.h:639-647. */
MA_API int ma_computeD(const ma_bf16* dO, const ma_bf16* O, ma_bf16* D,
                const AttentionParams* p, uint32_t B, ma_stream_t stream);

/* flashAttentionBackward: recomputes P = exp(Q K^T / sqrt(D) - l) and writes
 * dQ (fp32), dK and dV (bf16) for causal attention, given dZ = dO and d = D
 * from ma_computeD.  Replaces attention.metal:198-211 (buffers 0..9)
 * dispatched at model.h:648-665. */
MA_API int ma_flashAttentionBackward(const ma_bf16* dZ, const ma_bf16* d, const float* l,
                              const ma_bf16* q, const ma_bf16* k, const ma_bf16* v,
                              float* dQ, ma_bf16* dK, ma_bf16* dV,
                              const AttentionParams* p, uint32_t B, ma_stream_t stream);

/* Shard variants: the same computation restricted to the flat (batch, head)
 * indices bh = b*NH + h in [bh_begin, bh_end) of the B-batch tensors the
 * pointers describe.  Rows and columns outside the range are not touched.
 * Used to split the independent (batch, head) shards over several GPUs; they
 * have no counterpart in the single-device reference (model.h:459-473,
 * model.h:639-665 always dispatch every head). */
MA_API int ma_flashAttentionForward_shard(const ma_bf16* q, const ma_bf16* k, const ma_bf16* v,
                                   ma_bf16* out, float* l, const AttentionParams* p,
                                   uint32_t B, uint32_t bh_begin, uint32_t bh_end,
                                   ma_stream_t stream);
MA_API int ma_computeD_shard(const ma_bf16* dO, const ma_bf16* O, ma_bf16* D,
                      const AttentionParams* p, uint32_t B, uint32_t bh_begin,
                      uint32_t bh_end, ma_stream_t stream);
MA_API int ma_flashAttentionBackward_shard(const ma_bf16* dZ, const ma_bf16* d, const float* l,
                                    const ma_bf16* q, const ma_bf16* k, const ma_bf16* v,
                                    float* dQ, ma_bf16* dK, ma_bf16* dV,
                                    const AttentionParams* p, uint32_t B, uint32_t bh_begin,
                                    uint32_t bh_end, ma_stream_t stream);

/* ---- GEMMs around attention (the rest of the attention block).  The
 * activations have B*M rows; weights are [N][N] bf16 with row = input
 * feature; weight gradients sum over all B*M rows.  N must be a multiple of
 * 64.  Outputs are written (the reference accumulates into buffers its host
 * zeroes first, model.h:552-556, which gives the same values). */

/* projForward: out = attn_out * proj_w (bf16).  Replaces attention.metal:
 * 395-416 (buffers 0..3) dispatched at model.h:474-481. */
MA_API int ma_projForward(const ma_bf16* attn_out, const ma_bf16* proj_w, ma_bf16* out,
                          const AttentionParams* p, uint32_t B, ma_stream_t stream);

/* projBackwarddW: dProjw = attn_out^T * dZ (bf16, fp32 accumulation).
 * Replaces attention.metal:418-430 (buffers 0..3) dispatched at model.h:621-628. */
MA_API int ma_projBackwarddW(const ma_bf16* attn_out, const ma_bf16* dZ, ma_bf16* dProjw,
                             const AttentionParams* p, uint32_t B, ma_stream_t stream);

/* projBackwarddX: dAttn = dZ * proj_w^T (bf16).  Replaces attention.metal:
 * 432-455 (buffers 0..3) dispatched at model.h:629-636. */
MA_API int ma_projBackwarddX(const ma_bf16* dZ, const ma_bf16* proj_w, ma_bf16* dAttn,
                             const AttentionParams* p, uint32_t B, ma_stream_t stream);

/* projBackwarddX with computeD fused into the GEMM epilogue: dAttn as
 * ma_projBackwarddX, and D as ma_computeD(dAttn, attn_out) computed from the
 * tile while it is on chip (the bf16-rounded dAttn values, fp32 sums, one
 * bf16 rounding), which saves computeD's launch and its read of dAttn.
 * Needs the attention shape (D in {64, 128}).  Replaces the pair of
 * dispatches at model.h:629-647 (attention.metal:432-455 then 166-195). */
MA_API int ma_projBackwarddXComputeD(const ma_bf16* dZ, const ma_bf16* proj_w, ma_bf16* dAttn,
                                     const ma_bf16* attn_out, ma_bf16* D, const AttentionParams* p,
                                     uint32_t B, ma_stream_t stream);

/* computeGradDx: dX = dQ * Wq^T + dK * Wk^T + dV * Wv^T, fp32 (dQ fp32, the
 * rest bf16; dQ enters the tensor core rounded to bf16).  Replaces
 * attention.metal:301-342 (buffers 0..7) dispatched at model.h:666-678. */
MA_API int ma_computeGradDx(float* dX, const ma_bf16* qw, const ma_bf16* kw, const ma_bf16* vw,
                            const float* dQ, const ma_bf16* dK, const ma_bf16* dV,
                            const AttentionParams* p, uint32_t B, ma_stream_t stream);

/* computeGradDw: dQw = X^T * dQ (fp32), dKw = X^T * dK, dVw = X^T * dV
 * (bf16), fp32 accumulation (dQ rounded to bf16 on entry).  Replaces
 * attention.metal:344-393 (buffers 0..7) dispatched at model.h:679-691. */
MA_API int ma_computeGradDw(const ma_bf16* x, const float* dQ, const ma_bf16* dK,
                            const ma_bf16* dV, float* dQw, ma_bf16* dKw, ma_bf16* dVw,
                            const AttentionParams* p, uint32_t B, ma_stream_t stream);

/* ---- Training step (config 5): the CUDA counterpart of the reference's
 * Model (model.h:104-860) for a batch of B sequences: token + positional
 * embedding, `layers` pre-LayerNorm blocks (attention through the entry
 * points above, then a ReLU MLP of width E*mlp_scale), a final LayerNorm, the
 * vocabulary projection, mean cross-entropy, and Adam (beta1 0.9, beta2
 * 0.999, eps 1e-8, bias-corrected step size, fp32 master weights, bf16
 * gradients and moments; optimstep.metal, model.h:726-757).  The model
 * allocates and owns all its buffers at creation (cudaMalloc) and initialises
 * the weights from `seed` with the reference's distributions
 * (main.cpp:1594-1620).  forward/backward/step only enqueue work on `stream`.
 * The model belongs to the device current at create; its other calls return
 * MA_ERR_NO_DEVICE while another device is current.
 * No counterpart in the attention-only reference ABI: it replaces model.h's
 * orchestration.  Limits (else MA_ERR_LIMIT): B*T < 2^30, E <= 16384,
 * E*mlp_scale <= 65536, vocab <= 2^20, layers <= 4096. */
typedef struct MaModelConfig {
  uint32_t B;          /* sequences per step */
  uint32_t T;          /* sequence length (BLOCK_SIZE) */
  uint32_t E;          /* embedding width (N_EMBED), a multiple of 64 */
  uint32_t NH;         /* heads; E/NH must be 64 or 128 */
  uint32_t layers;     /* N_LAYERS */
  uint32_t mlp_scale;  /* MLP width = E*mlp_scale (MLP_SCALE) */
  uint32_t vocab;      /* vocabulary (padded), a multiple of 64 */
  float lr;            /* LR */
  uint64_t seed;
} MaModelConfig;

typedef struct ma_model ma_model;

MA_API int ma_model_create(const MaModelConfig* cfg, ma_model** model);
MA_API int ma_model_destroy(ma_model* model);
/* tokens, targets: device int32 [B][T]; they must stay valid until backward
 * has been enqueued.  The mean loss is the tensor "loss" (device fp32). */
MA_API int ma_model_forward(ma_model* model, const int32_t* tokens, const int32_t* targets,
                            ma_stream_t stream);
MA_API int ma_model_backward(ma_model* model, ma_stream_t stream);
MA_API int ma_model_step(ma_model* model, ma_stream_t stream);
/* Device pointer and size of a named buffer: a parameter ("embed", "pos",
 * "layer<n>.qw" ... "linw"), its gradient ("grad.<name>"), or "logits",
 * "loss", "loss_rows", "lse_rows", "embed_out", "master", "dstream". */
MA_API int ma_model_tensor(ma_model* model, const char* name, void** ptr, uint64_t* bytes);
/* Synchronous copies of a named tensor to / from host memory (bytes must be
 * its size).  Writing a parameter also resets its fp32 master copy. */
MA_API int ma_model_read(ma_model* model, const char* name, void* host, uint64_t bytes);
MA_API int ma_model_write(ma_model* model, const char* name, const void* host, uint64_t bytes);
MA_API uint32_t ma_model_param_count(ma_model* model);
MA_API const char* ma_model_param_name(ma_model* model, uint32_t index);
/* Copies the model's kernel status word (bounded-wait time-outs) to *status. */
MA_API int ma_model_status(ma_model* model, uint32_t* status);
/* Text for the last error of a ma_model_* call on the calling thread. */
MA_API const char* ma_model_last_error(void);

/* The pair ma_flashAttentionForwardComputeDZeroDQ + ma_flashAttentionBackwardAccumulate
 * is ma_flashAttentionForwardComputeD + ma_flashAttentionBackward with dQ
 * handled as the reference handles it: its backward adds each key tile's
 * contribution into dQ (attention.metal:292-296), which its host zeroes
 * first (model.h:549-551).  ma_flashAttentionBackward zeroes dQ itself, a
 * separate pass over the whole fp32 tensor (201 MB at config 2) before the
 * kernel; here the forward writes those zeros instead, each thread for the
 * query row it computes, overlapped with its work.  Results equal the
 * separate calls (dQ to fp32 rounding, as between any two runs).
 *
 * ForwardComputeDZeroDQ: as ma_flashAttentionForwardComputeD, and it also
 * writes zeros to dQ (fp32 [B][M][N], 16-byte aligned) for every (row, head)
 * it computes (the shard's, for _shard).  No counterpart in the reference
 * (the reference zeroes dQ on the host, model.h:549-551). */
MA_API int ma_flashAttentionForwardComputeDZeroDQ(const ma_bf16* q, const ma_bf16* k, const ma_bf16* v,
                                                  const ma_bf16* dO, ma_bf16* out, float* l, ma_bf16* D,
                                                  float* dQ, const AttentionParams* p, uint32_t B,
                                                  ma_stream_t stream);
MA_API int ma_flashAttentionForwardComputeDZeroDQ_shard(const ma_bf16* q, const ma_bf16* k,
                                                        const ma_bf16* v, const ma_bf16* dO, ma_bf16* out,
                                                        float* l, ma_bf16* D, float* dQ,
                                                        const AttentionParams* p, uint32_t B,
                                                        uint32_t bh_begin, uint32_t bh_end,
                                                        ma_stream_t stream);
/* flashAttentionBackward with the reference's dQ contract
 * (attention.metal:198-211, 292-296): dQ += the backward's dQ, so dQ must
 * hold zeros (or earlier partial sums) on entry; dK and dV are written as by
 * ma_flashAttentionBackward.  Same arguments and limits. */
MA_API int ma_flashAttentionBackwardAccumulate(const ma_bf16* dZ, const ma_bf16* d, const float* l,
                                               const ma_bf16* q, const ma_bf16* k, const ma_bf16* v,
                                               float* dQ, ma_bf16* dK, ma_bf16* dV,
                                               const AttentionParams* p, uint32_t B, ma_stream_t stream);
MA_API int ma_flashAttentionBackwardAccumulate_shard(const ma_bf16* dZ, const ma_bf16* d, const float* l,
                                                     const ma_bf16* q, const ma_bf16* k, const ma_bf16* v,
                                                     float* dQ, ma_bf16* dK, ma_bf16* dV,
                                                     const AttentionParams* p, uint32_t B,
                                                     uint32_t bh_begin, uint32_t bh_end, ma_stream_t stream);

/* Allocation-free backward pass: computeD followed by flashAttentionBackward,
 * for callers that cannot let a library allocate device memory (hosts whose
 * own arena or caching allocator owns all of the GPU's memory, processes under
 * a fixed device-memory budget, loops that must not take the implicit device
 * synchronisation of cudaMalloc/cudaFree).  It takes the attention output O
 * instead of D and writes the same dQ, dK, dV as ma_computeD +
 * ma_flashAttentionBackward.  D and a status word live in a scratch array
 * compiled into the library (about 4 MiB, held by every GPU that loads it
 * until the process exits); it calls no cudaMalloc or cudaFree.
 *   - B*M*NH must not exceed MA_NOALLOC_MAX_D_ENTRIES, else MA_ERR_LIMIT.
 *   - The first call on a device looks the scratch's device address up (and
 *     may load the library's device code); make that first call before any
 *     stream capture.
 *   - All calls on a device share the scratch: calls that overlap on the GPU
 *     (other streams, other host threads) race and give wrong results.
 *   - A bounded wait that runs out in its kernels sets a bit in a status
 *     word inside the scratch; ma_device_status (which allocates nothing)
 *     reads and clears it together with the other entry points' word, and
 *     the bit stays set until that read.
 * No counterpart in the reference. */
#define MA_NOALLOC_MAX_D_ENTRIES (1u << 21)
MA_API int ma_flashAttentionBackward_noalloc(const ma_bf16* dZ, const ma_bf16* O, const float* l,
                                             const ma_bf16* q, const ma_bf16* k, const ma_bf16* v,
                                             float* dQ, ma_bf16* dK, ma_bf16* dV,
                                             const AttentionParams* p, uint32_t B,
                                             ma_stream_t stream);

/* Text for the last MA_ERR_* returned on the calling host thread ("" if none).
 * Replaces the reference's printed command-buffer error (model.h:361-365). */
MA_API const char* ma_last_error_string(void);

/* Bits of the status word read by ma_device_status: the kernels whose bounded
 * waits ran out. */
#define MA_STATUS_FWD_TIMEOUT (1u << 0)  /* flashAttentionForward */
#define MA_STATUS_BWD_TIMEOUT (1u << 1)  /* flashAttentionBackward */
#define MA_STATUS_QKV_TIMEOUT (1u << 2)  /* computeQKV */
#define MA_STATUS_GEMM_TIMEOUT (1u << 3) /* the GEMMs around attention */

/* Reads and clears the current device's kernel status: 0 = no kernel gave
 * up; otherwise a bit mask (MA_STATUS_*) of the kernels whose bounded waits
 * ran out since the last read, by any entry point on this device, including
 * ma_flashAttentionBackward_noalloc.  Synchronises `stream` first.  Allocates
 * nothing.  Returns MA_OK or an MA_ERR_* code. */
MA_API int ma_device_status(uint32_t* status, ma_stream_t stream);

/* Test hook of the kernels' time-out path.  The next launch of each kernel
 * named in `kernels` (MA_STATUS_FWD_TIMEOUT and/or MA_STATUS_BWD_TIMEOUT) lets
 * one wait run out on purpose: once its first tensor-core products are in
 * flight, its UMMA-issuing thread waits on an mbarrier that nothing arrives
 * at, for `wait_ns` nanoseconds (1 .. 10^9).  The kernel then winds down as
 * after a real time-out: every role stops at its next wait, the copies and
 * products already in flight are waited for, TMEM is freed and the kernel's
 * bit is set in the status word ma_device_status reads.  That launch's
 * outputs are undefined; nothing faults or traps, and later launches are not
 * affected.  A request not yet taken is replaced by the next call; kernels = 0
 * cancels it.  Diagnostic; no counterpart in the reference, which only prints
 * a failed command buffer's error (model.h:358-366). */
MA_API int ma_debug_expire_next_wait(uint32_t kernels, uint32_t wait_ns);

/* Number of kernels this library has launched in this process (all devices,
 * all threads), for accounting of launches in timed regions.  Diagnostic;
 * no counterpart in the reference. */
MA_API uint64_t ma_kernel_launch_count(void);

/* ---- Host-resident batches.  The reference's buffers are shared CPU/GPU
 * memory (MTLResourceStorageModeShared, model.h:236-253): its host writes
 * inputs and reads results in place.  On a discrete GPU the batch must cross
 * PCIe, so a pipeline splits the batch into chunks of `chunk_B` sequences
 * and overlaps, on three internal streams, the host->device copy of chunk
 * c+1, the kernels of chunk c and the device->host copy of chunk c-1 (the
 * copy engines of the two directions run concurrently).  Results equal
 * ma_flashAttentionForward (forward only) or ma_flashAttentionForwardComputeD
 * then ma_flashAttentionBackward (forward and backward) on device buffers,
 * since every (batch, head) is independent: bit for bit, except dQ, whose
 * fp32 partial sums from different key tiles are added in no fixed order
 * (as by the reference's atomics, attention.metal:292-296).
 *   - Host pointers should be page-locked (cudaHostAlloc / cudaHostRegister);
 *     pageable memory gives the same results without the overlap.
 *   - A pipeline belongs to the device current at create and owns three
 *     chunk-sized sets of device buffers (allocated once, at create).
 *   - Calls are stream-ordered: the copies start after the work already on
 *     `stream` and `stream` waits for the last copy back; the host buffers
 *     must stay valid until then.  Calls that use one pipeline must be
 *     ordered (same stream, or synchronised).
 * No counterpart in the reference. */
typedef struct ma_host_pipeline ma_host_pipeline;
MA_API int ma_host_pipeline_create(const AttentionParams* p, uint32_t chunk_B, ma_host_pipeline** out);
MA_API int ma_host_pipeline_destroy(ma_host_pipeline* pl);
/* flashAttentionForward over B host-resident sequences: q, k, v -> out, l. */
MA_API int ma_flashAttentionForward_host(ma_host_pipeline* pl, const ma_bf16* q, const ma_bf16* k,
                                         const ma_bf16* v, ma_bf16* out, float* l, uint32_t B,
                                         ma_stream_t stream);
/* forward, computeD and backward over B host-resident sequences:
 * q, k, v, dO -> out, l, dQ, dK, dV (the attention core of one training step,
 * model.h:459-473 then model.h:639-665). */
MA_API int ma_attentionForwardBackward_host(ma_host_pipeline* pl, const ma_bf16* q, const ma_bf16* k,
                                            const ma_bf16* v, const ma_bf16* dO, ma_bf16* out, float* l,
                                            float* dQ, ma_bf16* dK, ma_bf16* dV, uint32_t B,
                                            ma_stream_t stream);

/* Library version as major*10000 + minor*100 + patch. */
MA_API int ma_version(void);

#ifdef __cplusplus
}
#endif

#endif /* METALATTN_H_ */
