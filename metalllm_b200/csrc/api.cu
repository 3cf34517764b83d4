// api.cu -- the extern "C" boundary of libmetalattn (include/metalattn.h).
//
// Each entry point replaces one Metal dispatch of the reference's host code
// (model.h:446-473 forward, model.h:639-665 backward): it validates the
// AttentionParams and pointers, then enqueues the kernel on the caller's
// stream.  Errors are returned as MA_ERR_* codes with a per-thread message
// instead of the reference's exit(1) (model.h:333-336) or printed-and-ignored
// command-buffer error (model.h:361-365).
#include <atomic>
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <mutex>
#include <string>

#include "common.cuh"

namespace {
std::atomic<unsigned long long> g_launches{0};
}  // namespace

void ma::count_launches(unsigned n) { g_launches.fetch_add(n, std::memory_order_relaxed); }

namespace {
// Pending ma_debug_expire_next_wait request: kernel bits and the wait in ns.
std::mutex g_expire_mu;
uint32_t g_expire_mask = 0, g_expire_ns = 0;
}  // namespace

uint32_t ma::take_expire_request(uint32_t kernel_bit) {
  std::lock_guard<std::mutex> lock(g_expire_mu);
  if (!(g_expire_mask & kernel_bit)) return 0;
  g_expire_mask &= ~kernel_bit;
  return g_expire_ns;
}

namespace {

thread_local std::string g_last_error;

int fail(int code, const char* fmt, ...) __attribute__((format(printf, 2, 3)));
int fail(int code, const char* fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  g_last_error = buf;
  return code;
}

int ok() {
  g_last_error.clear();
  return MA_OK;
}

int cuda_fail(cudaError_t e, const char* what) {
  return fail(MA_ERR_CUDA, "%s: %s (%s)", what, cudaGetErrorName(e), cudaGetErrorString(e));
}

// One 4-byte status word per device (bit mask of kernels whose bounded waits
// ran out), allocated on first use and kept for the life of the process.
constexpr int kMaxDevices = 64;
uint32_t* g_status[kMaxDevices] = {};
std::mutex g_status_mu;

int device_status_word(uint32_t** out) {
  int dev = -1;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return cuda_fail(e, "cudaGetDevice");
  if (dev < 0 || dev >= kMaxDevices) return fail(MA_ERR_NO_DEVICE, "device ordinal %d out of range", dev);
  std::lock_guard<std::mutex> lock(g_status_mu);
  if (!g_status[dev]) {
    int major = 0, minor = 0;
    cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev);
    cudaDeviceGetAttribute(&minor, cudaDevAttrComputeCapabilityMinor, dev);
    if (major != 10 || minor != 0)
      return fail(MA_ERR_NO_DEVICE, "device %d is sm_%d%d; libmetalattn is built for sm_100a only", dev,
                  major, minor);
    void* p = nullptr;
    e = cudaMalloc(&p, sizeof(uint32_t));
    if (e != cudaSuccess) return cuda_fail(e, "cudaMalloc(status word)");
    e = cudaMemset(p, 0, sizeof(uint32_t));
    if (e != cudaSuccess) {
      cudaFree(p);
      return cuda_fail(e, "cudaMemset(status word)");
    }
    g_status[dev] = static_cast<uint32_t*>(p);
  }
  *out = g_status[dev];
  return MA_OK;
}

// Device address of the allocation-free entry point's status word on `dev`,
// or nullptr while that entry point has not run there (defined with its
// scratch array below).
uint32_t* noalloc_status_word_if_set_up(int dev);

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// Validates AttentionParams + batch + shard range; fills the kernel shape.
int check_shape(const AttentionParams* p, uint32_t B, uint32_t bh_begin, uint32_t bh_end,
                bool is_range, ma::AttnShape* s) {
  if (!p) return fail(MA_ERR_NULL, "AttentionParams pointer is NULL");
  if (p->D != 64 && p->D != 128)
    return fail(MA_ERR_SHAPE, "head size D=%u unsupported (supported: 64, 128)", p->D);
  if (p->NH == 0 || p->M == 0 || B == 0)
    return fail(MA_ERR_SHAPE, "empty shape: M=%u NH=%u B=%u", p->M, p->NH, B);
  if ((uint64_t)p->NH * p->D != p->N)
    return fail(MA_ERR_SHAPE, "N=%u must equal NH*D=%u*%u", p->N, p->NH, p->D);
  const uint64_t nbh = (uint64_t)B * p->NH;
  if ((uint64_t)B * p->M * p->N >= (1ull << 40) || nbh >= (1ull << 30) || p->M > (1u << 24))
    return fail(MA_ERR_LIMIT, "problem too large: B=%u M=%u N=%u", B, p->M, p->N);
  if (is_range && (bh_begin > bh_end || bh_end > nbh))
    return fail(MA_ERR_RANGE, "shard range [%u, %u) outside [0, %llu]", bh_begin, bh_end,
                (unsigned long long)nbh);
  s->T = (int)p->M;
  s->N = (int)p->N;
  s->D = (int)p->D;
  s->NH = (int)p->NH;
  s->B = (int)B;
  s->bh_begin = is_range ? (int)bh_begin : 0;
  s->bh_end = is_range ? (int)bh_end : (int)nbh;
  return MA_OK;
}

#define MA_REQUIRE_PTR(ptr)                                                          \
  do {                                                                               \
    if (!(ptr)) return fail(MA_ERR_NULL, "pointer '%s' is NULL", #ptr);              \
    if (!aligned16(ptr)) return fail(MA_ERR_ALIGN, "pointer '%s' is not 16-byte aligned", #ptr); \
  } while (0)

using bf16p = const __nv_bfloat16*;
using bf16m = __nv_bfloat16*;

int forward_impl(const ma_bf16* q, const ma_bf16* k, const ma_bf16* v, ma_bf16* out, float* l,
                 const AttentionParams* p, uint32_t B, uint32_t b0, uint32_t b1, bool range,
                 ma_stream_t stream, const ma_bf16* dO = nullptr, ma_bf16* D = nullptr,
                 float* dQ = nullptr, bool want_dqz = false) {
  ma::AttnShape s;
  int rc = check_shape(p, B, b0, b1, range, &s);
  if (rc) return rc;
  MA_REQUIRE_PTR(q);
  MA_REQUIRE_PTR(k);
  MA_REQUIRE_PTR(v);
  MA_REQUIRE_PTR(out);
  MA_REQUIRE_PTR(l);
  const bool with_d = dO != nullptr || D != nullptr;
  if (with_d) {
    MA_REQUIRE_PTR(dO);
    if (!D) return fail(MA_ERR_NULL, "pointer 'D' is NULL");
    if (reinterpret_cast<uintptr_t>(D) & 1u) return fail(MA_ERR_ALIGN, "pointer 'D' is not 2-byte aligned");
  }
  if (want_dqz) MA_REQUIRE_PTR(dQ);  // the forward writes zeros to it
  uint32_t* status = nullptr;
  rc = device_status_word(&status);
  if (rc) return rc;
  if (s.bh_end == s.bh_begin) return ok();
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  // D = 64: computeD in the forward's epilogue; D = 128: the separate kernel after it
  const bool fused = with_d && s.D == 64;
  cudaError_t e = ma::launch_flash_fwd(reinterpret_cast<bf16p>(q), reinterpret_cast<bf16p>(k),
                                       reinterpret_cast<bf16p>(v), reinterpret_cast<bf16m>(out), l, s,
                                       status, st, fused ? reinterpret_cast<bf16p>(dO) : nullptr,
                                       fused ? reinterpret_cast<bf16m>(D) : nullptr, want_dqz ? dQ : nullptr);
  if (e != cudaSuccess) return cuda_fail(e, "flashAttentionForward launch");
  if (with_d && !fused) {
    e = ma::launch_compute_d(reinterpret_cast<bf16p>(dO), reinterpret_cast<bf16p>(out), reinterpret_cast<bf16m>(D),
                             s, st);
    if (e != cudaSuccess) return cuda_fail(e, "computeD launch");
  }
  return ok();
}

int compute_d_impl(const ma_bf16* dO, const ma_bf16* O, ma_bf16* D, const AttentionParams* p,
                   uint32_t B, uint32_t b0, uint32_t b1, bool range, ma_stream_t stream) {
  ma::AttnShape s;
  int rc = check_shape(p, B, b0, b1, range, &s);
  if (rc) return rc;
  MA_REQUIRE_PTR(dO);
  MA_REQUIRE_PTR(O);
  if (!D) return fail(MA_ERR_NULL, "pointer 'D' is NULL");
  if (reinterpret_cast<uintptr_t>(D) & 1u) return fail(MA_ERR_ALIGN, "pointer 'D' is not 2-byte aligned");
  uint32_t* status = nullptr;
  rc = device_status_word(&status);
  if (rc) return rc;
  if (s.bh_end == s.bh_begin) return ok();
  cudaError_t e = ma::launch_compute_d(reinterpret_cast<bf16p>(dO), reinterpret_cast<bf16p>(O),
                                       reinterpret_cast<bf16m>(D), s,
                                       reinterpret_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "computeD launch");
  return ok();
}

int backward_impl(const ma_bf16* dZ, const ma_bf16* d, const float* l, const ma_bf16* q,
                  const ma_bf16* k, const ma_bf16* v, float* dQ, ma_bf16* dK, ma_bf16* dV,
                  const AttentionParams* p, uint32_t B, uint32_t b0, uint32_t b1, bool range,
                  ma_stream_t stream, bool accumulate_dq = false) {
  ma::AttnShape s;
  int rc = check_shape(p, B, b0, b1, range, &s);
  if (rc) return rc;
  MA_REQUIRE_PTR(dZ);
  if (!d) return fail(MA_ERR_NULL, "pointer 'd' is NULL");
  if (reinterpret_cast<uintptr_t>(d) & 1u) return fail(MA_ERR_ALIGN, "pointer 'd' is not 2-byte aligned");
  MA_REQUIRE_PTR(l);
  MA_REQUIRE_PTR(q);
  MA_REQUIRE_PTR(k);
  MA_REQUIRE_PTR(v);
  MA_REQUIRE_PTR(dQ);
  MA_REQUIRE_PTR(dK);
  MA_REQUIRE_PTR(dV);
  uint32_t* status = nullptr;
  rc = device_status_word(&status);
  if (rc) return rc;
  if (s.bh_end == s.bh_begin) return ok();
  cudaError_t e = ma::launch_flash_bwd(
      reinterpret_cast<bf16p>(dZ), reinterpret_cast<bf16p>(d), l, reinterpret_cast<bf16p>(q),
      reinterpret_cast<bf16p>(k), reinterpret_cast<bf16p>(v), dQ, reinterpret_cast<bf16m>(dK),
      reinterpret_cast<bf16m>(dV), s, status, reinterpret_cast<cudaStream_t>(stream), accumulate_dq);
  if (e != cudaSuccess) return cuda_fail(e, "flashAttentionBackward launch");
  return ok();
}

}  // namespace

extern "C" {

int ma_computeQKV(const ma_bf16* X, ma_bf16* q, ma_bf16* k, ma_bf16* v, const ma_bf16* q_w,
                  const ma_bf16* k_w, const ma_bf16* v_w, const AttentionParams* p, uint32_t B,
                  ma_stream_t stream) {
  if (!p) return fail(MA_ERR_NULL, "AttentionParams pointer is NULL");
  if (p->N == 0 || p->M == 0 || B == 0) return fail(MA_ERR_SHAPE, "empty shape: M=%u N=%u B=%u", p->M, p->N, B);
  if (p->N % 64 != 0) return fail(MA_ERR_SHAPE, "N=%u must be a multiple of 64", p->N);
  if ((uint64_t)B * p->M >= (1ull << 31) || p->N > 16384)
    return fail(MA_ERR_LIMIT, "problem too large: B*M=%llu N=%u", (unsigned long long)B * p->M, p->N);
  MA_REQUIRE_PTR(X);
  MA_REQUIRE_PTR(q);
  MA_REQUIRE_PTR(k);
  MA_REQUIRE_PTR(v);
  MA_REQUIRE_PTR(q_w);
  MA_REQUIRE_PTR(k_w);
  MA_REQUIRE_PTR(v_w);
  uint32_t* status = nullptr;
  int rc = device_status_word(&status);
  if (rc) return rc;
  cudaError_t e = ma::launch_qkv(
      reinterpret_cast<bf16p>(X), reinterpret_cast<bf16m>(q), reinterpret_cast<bf16m>(k),
      reinterpret_cast<bf16m>(v), reinterpret_cast<bf16p>(q_w), reinterpret_cast<bf16p>(k_w),
      reinterpret_cast<bf16p>(v_w), (int)(B * p->M), (int)p->N, status,
      reinterpret_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "computeQKV launch");
  return ok();
}

int ma_flashAttentionForward(const ma_bf16* q, const ma_bf16* k, const ma_bf16* v, ma_bf16* out,
                             float* l, const AttentionParams* p, uint32_t B, ma_stream_t stream) {
  return forward_impl(q, k, v, out, l, p, B, 0, 0, false, stream);
}

int ma_flashAttentionForward_shard(const ma_bf16* q, const ma_bf16* k, const ma_bf16* v,
                                   ma_bf16* out, float* l, const AttentionParams* p, uint32_t B,
                                   uint32_t bh_begin, uint32_t bh_end, ma_stream_t stream) {
  return forward_impl(q, k, v, out, l, p, B, bh_begin, bh_end, true, stream);
}

int ma_flashAttentionForwardComputeD(const ma_bf16* q, const ma_bf16* k, const ma_bf16* v,
                                     const ma_bf16* dO, ma_bf16* out, float* l, ma_bf16* D,
                                     const AttentionParams* p, uint32_t B, ma_stream_t stream) {
  return forward_impl(q, k, v, out, l, p, B, 0, 0, false, stream, dO, D);
}

int ma_flashAttentionForwardComputeD_shard(const ma_bf16* q, const ma_bf16* k, const ma_bf16* v,
                                           const ma_bf16* dO, ma_bf16* out, float* l, ma_bf16* D,
                                           const AttentionParams* p, uint32_t B, uint32_t bh_begin,
                                           uint32_t bh_end, ma_stream_t stream) {
  return forward_impl(q, k, v, out, l, p, B, bh_begin, bh_end, true, stream, dO, D);
}

int ma_flashAttentionForwardComputeDZeroDQ(const ma_bf16* q, const ma_bf16* k, const ma_bf16* v,
                                           const ma_bf16* dO, ma_bf16* out, float* l, ma_bf16* D, float* dQ,
                                           const AttentionParams* p, uint32_t B, ma_stream_t stream) {
  return forward_impl(q, k, v, out, l, p, B, 0, 0, false, stream, dO, D, dQ, true);
}

int ma_flashAttentionForwardComputeDZeroDQ_shard(const ma_bf16* q, const ma_bf16* k, const ma_bf16* v,
                                                 const ma_bf16* dO, ma_bf16* out, float* l, ma_bf16* D,
                                                 float* dQ, const AttentionParams* p, uint32_t B,
                                                 uint32_t bh_begin, uint32_t bh_end, ma_stream_t stream) {
  return forward_impl(q, k, v, out, l, p, B, bh_begin, bh_end, true, stream, dO, D, dQ, true);
}

int ma_computeD(const ma_bf16* dO, const ma_bf16* O, ma_bf16* D, const AttentionParams* p,
                uint32_t B, ma_stream_t stream) {
  return compute_d_impl(dO, O, D, p, B, 0, 0, false, stream);
}

int ma_computeD_shard(const ma_bf16* dO, const ma_bf16* O, ma_bf16* D, const AttentionParams* p,
                      uint32_t B, uint32_t bh_begin, uint32_t bh_end, ma_stream_t stream) {
  return compute_d_impl(dO, O, D, p, B, bh_begin, bh_end, true, stream);
}

int ma_flashAttentionBackward(const ma_bf16* dZ, const ma_bf16* d, const float* l,
                              const ma_bf16* q, const ma_bf16* k, const ma_bf16* v, float* dQ,
                              ma_bf16* dK, ma_bf16* dV, const AttentionParams* p, uint32_t B,
                              ma_stream_t stream) {
  return backward_impl(dZ, d, l, q, k, v, dQ, dK, dV, p, B, 0, 0, false, stream);
}

int ma_flashAttentionBackward_shard(const ma_bf16* dZ, const ma_bf16* d, const float* l,
                                    const ma_bf16* q, const ma_bf16* k, const ma_bf16* v,
                                    float* dQ, ma_bf16* dK, ma_bf16* dV,
                                    const AttentionParams* p, uint32_t B, uint32_t bh_begin,
                                    uint32_t bh_end, ma_stream_t stream) {
  return backward_impl(dZ, d, l, q, k, v, dQ, dK, dV, p, B, bh_begin, bh_end, true, stream);
}

int ma_flashAttentionBackwardAccumulate(const ma_bf16* dZ, const ma_bf16* d, const float* l,
                                        const ma_bf16* q, const ma_bf16* k, const ma_bf16* v, float* dQ,
                                        ma_bf16* dK, ma_bf16* dV, const AttentionParams* p, uint32_t B,
                                        ma_stream_t stream) {
  return backward_impl(dZ, d, l, q, k, v, dQ, dK, dV, p, B, 0, 0, false, stream, true);
}

int ma_flashAttentionBackwardAccumulate_shard(const ma_bf16* dZ, const ma_bf16* d, const float* l,
                                              const ma_bf16* q, const ma_bf16* k, const ma_bf16* v,
                                              float* dQ, ma_bf16* dK, ma_bf16* dV, const AttentionParams* p,
                                              uint32_t B, uint32_t bh_begin, uint32_t bh_end,
                                              ma_stream_t stream) {
  return backward_impl(dZ, d, l, q, k, v, dQ, dK, dV, p, B, bh_begin, bh_end, true, stream, true);
}

// ---------------------------------------------------------------- GEMMs
// Shared validation of the GEMM entry points: N a positive multiple of 64
// (16-byte TMA strides, whole 64-column weight tiles), B*M rows >= 1.
static int gemm_shape(const AttentionParams* p, uint32_t B, int* rows, int* n) {
  if (!p) return fail(MA_ERR_NULL, "AttentionParams pointer is NULL");
  if (p->N == 0 || p->M == 0 || B == 0) return fail(MA_ERR_SHAPE, "empty shape: M=%u N=%u B=%u", p->M, p->N, B);
  if (p->N % 64 != 0) return fail(MA_ERR_SHAPE, "N=%u must be a multiple of 64", p->N);
  if ((uint64_t)B * p->M >= (1ull << 31) || p->N > 16384)
    return fail(MA_ERR_LIMIT, "problem too large: B*M=%llu N=%u", (unsigned long long)B * p->M, p->N);
  *rows = (int)(B * p->M);
  *n = (int)p->N;
  return MA_OK;
}

int ma_projForward(const ma_bf16* attn_out, const ma_bf16* proj_w, ma_bf16* out,
                   const AttentionParams* p, uint32_t B, ma_stream_t stream) {
  int rows = 0, n = 0;
  int rc = gemm_shape(p, B, &rows, &n);
  if (rc) return rc;
  MA_REQUIRE_PTR(attn_out);
  MA_REQUIRE_PTR(proj_w);
  MA_REQUIRE_PTR(out);
  uint32_t* status = nullptr;
  rc = device_status_word(&status);
  if (rc) return rc;
  cudaError_t e = ma::launch_proj_forward(reinterpret_cast<bf16p>(attn_out), reinterpret_cast<bf16p>(proj_w),
                                          reinterpret_cast<bf16m>(out), rows, n, status,
                                          reinterpret_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "projForward launch");
  return ok();
}

int ma_projBackwarddW(const ma_bf16* attn_out, const ma_bf16* dZ, ma_bf16* dProjw,
                      const AttentionParams* p, uint32_t B, ma_stream_t stream) {
  int rows = 0, n = 0;
  int rc = gemm_shape(p, B, &rows, &n);
  if (rc) return rc;
  MA_REQUIRE_PTR(attn_out);
  MA_REQUIRE_PTR(dZ);
  MA_REQUIRE_PTR(dProjw);
  uint32_t* status = nullptr;
  rc = device_status_word(&status);
  if (rc) return rc;
  cudaError_t e = ma::launch_proj_backward_dw(reinterpret_cast<bf16p>(attn_out), reinterpret_cast<bf16p>(dZ),
                                              reinterpret_cast<bf16m>(dProjw), rows, n, status,
                                              reinterpret_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "projBackwarddW launch");
  return ok();
}

int ma_projBackwarddX(const ma_bf16* dZ, const ma_bf16* proj_w, ma_bf16* dAttn,
                      const AttentionParams* p, uint32_t B, ma_stream_t stream) {
  int rows = 0, n = 0;
  int rc = gemm_shape(p, B, &rows, &n);
  if (rc) return rc;
  MA_REQUIRE_PTR(dZ);
  MA_REQUIRE_PTR(proj_w);
  MA_REQUIRE_PTR(dAttn);
  uint32_t* status = nullptr;
  rc = device_status_word(&status);
  if (rc) return rc;
  cudaError_t e = ma::launch_proj_backward_dx(reinterpret_cast<bf16p>(dZ), reinterpret_cast<bf16p>(proj_w),
                                              reinterpret_cast<bf16m>(dAttn), rows, n, status,
                                              reinterpret_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "projBackwarddX launch");
  return ok();
}

int ma_projBackwarddXComputeD(const ma_bf16* dZ, const ma_bf16* proj_w, ma_bf16* dAttn,
                              const ma_bf16* attn_out, ma_bf16* D, const AttentionParams* p, uint32_t B,
                              ma_stream_t stream) {
  ma::AttnShape s;
  int rc = check_shape(p, B, 0, 0, false, &s);
  if (rc) return rc;
  int rows = 0, n = 0;
  rc = gemm_shape(p, B, &rows, &n);
  if (rc) return rc;
  MA_REQUIRE_PTR(dZ);
  MA_REQUIRE_PTR(proj_w);
  MA_REQUIRE_PTR(dAttn);
  MA_REQUIRE_PTR(attn_out);
  if (!D) return fail(MA_ERR_NULL, "pointer 'D' is NULL");
  if (reinterpret_cast<uintptr_t>(D) & 1u) return fail(MA_ERR_ALIGN, "pointer 'D' is not 2-byte aligned");
  uint32_t* status = nullptr;
  rc = device_status_word(&status);
  if (rc) return rc;
  cudaError_t e = ma::launch_proj_backward_dx_d(reinterpret_cast<bf16p>(dZ), reinterpret_cast<bf16p>(proj_w),
                                                reinterpret_cast<bf16m>(dAttn), reinterpret_cast<bf16p>(attn_out),
                                                reinterpret_cast<bf16m>(D), rows, n, (int)p->D, status,
                                                reinterpret_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "projBackwarddX+computeD launch");
  return ok();
}

int ma_computeGradDx(float* dX, const ma_bf16* qw, const ma_bf16* kw, const ma_bf16* vw,
                     const float* dQ, const ma_bf16* dK, const ma_bf16* dV,
                     const AttentionParams* p, uint32_t B, ma_stream_t stream) {
  int rows = 0, n = 0;
  int rc = gemm_shape(p, B, &rows, &n);
  if (rc) return rc;
  MA_REQUIRE_PTR(dX);
  MA_REQUIRE_PTR(qw);
  MA_REQUIRE_PTR(kw);
  MA_REQUIRE_PTR(vw);
  MA_REQUIRE_PTR(dQ);
  MA_REQUIRE_PTR(dK);
  MA_REQUIRE_PTR(dV);
  uint32_t* status = nullptr;
  rc = device_status_word(&status);
  if (rc) return rc;
  cudaError_t e = ma::launch_grad_dx(dX, reinterpret_cast<bf16p>(qw), reinterpret_cast<bf16p>(kw),
                                     reinterpret_cast<bf16p>(vw), dQ, reinterpret_cast<bf16p>(dK),
                                     reinterpret_cast<bf16p>(dV), rows, n, status,
                                     reinterpret_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "computeGradDx launch");
  return ok();
}

int ma_computeGradDw(const ma_bf16* x, const float* dQ, const ma_bf16* dK, const ma_bf16* dV,
                     float* dQw, ma_bf16* dKw, ma_bf16* dVw, const AttentionParams* p, uint32_t B,
                     ma_stream_t stream) {
  int rows = 0, n = 0;
  int rc = gemm_shape(p, B, &rows, &n);
  if (rc) return rc;
  MA_REQUIRE_PTR(x);
  MA_REQUIRE_PTR(dQ);
  MA_REQUIRE_PTR(dK);
  MA_REQUIRE_PTR(dV);
  MA_REQUIRE_PTR(dQw);
  MA_REQUIRE_PTR(dKw);
  MA_REQUIRE_PTR(dVw);
  uint32_t* status = nullptr;
  rc = device_status_word(&status);
  if (rc) return rc;
  cudaError_t e = ma::launch_grad_dw(reinterpret_cast<bf16p>(x), dQ, reinterpret_cast<bf16p>(dK),
                                     reinterpret_cast<bf16p>(dV), dQw, reinterpret_cast<bf16m>(dKw),
                                     reinterpret_cast<bf16m>(dVw), rows, n, status,
                                     reinterpret_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "computeGradDw launch");
  return ok();
}

const char* ma_last_error_string(void) { return g_last_error.c_str(); }

int ma_device_status(uint32_t* status, ma_stream_t stream) {
  if (!status) return fail(MA_ERR_NULL, "status pointer is NULL");
  int dev = -1;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return cuda_fail(e, "cudaGetDevice");
  if (dev < 0 || dev >= kMaxDevices) return fail(MA_ERR_NO_DEVICE, "device ordinal %d out of range", dev);
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  e = cudaStreamSynchronize(st);
  if (e != cudaSuccess) return cuda_fail(e, "cudaStreamSynchronize");
  // Two words may exist on this device: the one the allocating entry points
  // use and the one in the allocation-free entry point's scratch.  Only words
  // already set up are read, so this call allocates nothing.
  uint32_t* words[2] = {nullptr, noalloc_status_word_if_set_up(dev)};
  {
    std::lock_guard<std::mutex> lock(g_status_mu);
    words[0] = g_status[dev];
  }
  uint32_t all = 0;
  for (uint32_t* word : words) {
    if (!word) continue;
    uint32_t host = 0;
    e = cudaMemcpy(&host, word, sizeof(uint32_t), cudaMemcpyDeviceToHost);
    if (e != cudaSuccess) return cuda_fail(e, "cudaMemcpy(status word)");
    e = cudaMemset(word, 0, sizeof(uint32_t));
    if (e != cudaSuccess) return cuda_fail(e, "cudaMemset(status word)");
    all |= host;
  }
  *status = all;
  return ok();
}

uint64_t ma_kernel_launch_count(void) { return g_launches.load(std::memory_order_relaxed); }

int ma_debug_expire_next_wait(uint32_t kernels, uint32_t wait_ns) {
  const uint32_t supported = MA_STATUS_FWD_TIMEOUT | MA_STATUS_BWD_TIMEOUT;
  if (kernels & ~supported)
    return fail(MA_ERR_RANGE, "ma_debug_expire_next_wait: kernel mask 0x%x names kernels without the hook "
                "(supported: MA_STATUS_FWD_TIMEOUT | MA_STATUS_BWD_TIMEOUT)", kernels);
  if (kernels && (wait_ns == 0 || wait_ns > 1000000000u))
    return fail(MA_ERR_RANGE, "ma_debug_expire_next_wait: wait_ns=%u outside 1 .. 10^9", wait_ns);
  std::lock_guard<std::mutex> lock(g_expire_mu);
  g_expire_mask = kernels;
  g_expire_ns = kernels ? wait_ns : 0;
  return ok();
}

int ma_version(void) { return 100; }

}  // extern "C"

// ---------------------------------------------------------------------------
// Allocation-free backward pass.
//
// Some callers cannot let a library allocate device memory: hosts that hand
// all of a GPU's memory to their own arena or caching allocator at start-up
// (so a cudaMalloc outside it fails or fragments the arena), processes run
// under a fixed device-memory budget, and latency-critical loops that must not
// take the implicit device-wide synchronisation cudaMalloc/cudaFree can cause.
// The entry points above allocate a 4-byte status word on their first call on
// each device, and the backward pass needs the caller to allocate the D
// buffer between computeD and flashAttentionBackward.
// ma_flashAttentionBackward_noalloc needs neither: its scratch (the D values
// and a status word) lives in the file-scope array below, which every GPU that
// loads the library holds until the process exits.
namespace {

constexpr size_t kNoallocHeaderBytes = 256;  // status word, padded to keep D 256-byte aligned
constexpr size_t kNoallocScratchBytes = kNoallocHeaderBytes + (size_t)MA_NOALLOC_MAX_D_ENTRIES * 2;

static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoallocScratchBytes];

// In host code g_noalloc_scratch names a host-side stand-in, not device
// memory: kernels get the device address looked up here, once per device.
void* g_noalloc_base[kMaxDevices] = {};
std::mutex g_noalloc_mu;

int noalloc_scratch(void** out) {
  int dev = -1;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return cuda_fail(e, "cudaGetDevice");
  if (dev < 0 || dev >= kMaxDevices) return fail(MA_ERR_NO_DEVICE, "device ordinal %d out of range", dev);
  std::lock_guard<std::mutex> lock(g_noalloc_mu);
  if (!g_noalloc_base[dev]) {
    int major = 0, minor = 0;
    cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev);
    cudaDeviceGetAttribute(&minor, cudaDevAttrComputeCapabilityMinor, dev);
    if (major != 10 || minor != 0)
      return fail(MA_ERR_NO_DEVICE, "device %d is sm_%d%d; libmetalattn is built for sm_100a only", dev,
                  major, minor);
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess) return cuda_fail(e, "cudaGetSymbolAddress(no-alloc scratch)");
    g_noalloc_base[dev] = p;
  }
  *out = g_noalloc_base[dev];
  return MA_OK;
}

// The status word is the first word of the scratch.  It starts at zero (the
// array is zero-initialised when the module loads), the kernels only set bits
// in it, and ma_device_status reads and clears it, so a time-out stays
// visible until it has been read, whatever calls come in between.
uint32_t* noalloc_status_word_if_set_up(int dev) {
  std::lock_guard<std::mutex> lock(g_noalloc_mu);
  return static_cast<uint32_t*>(g_noalloc_base[dev]);
}

}  // namespace

extern "C" int ma_flashAttentionBackward_noalloc(const ma_bf16* dZ, const ma_bf16* O,
                                                 const float* l, const ma_bf16* q,
                                                 const ma_bf16* k, const ma_bf16* v, float* dQ,
                                                 ma_bf16* dK, ma_bf16* dV,
                                                 const AttentionParams* p, uint32_t B,
                                                 ma_stream_t stream) {
  ma::AttnShape s;
  int rc = check_shape(p, B, 0, 0, false, &s);
  if (rc) return rc;
  MA_REQUIRE_PTR(dZ);
  MA_REQUIRE_PTR(O);
  MA_REQUIRE_PTR(l);
  MA_REQUIRE_PTR(q);
  MA_REQUIRE_PTR(k);
  MA_REQUIRE_PTR(v);
  MA_REQUIRE_PTR(dQ);
  MA_REQUIRE_PTR(dK);
  MA_REQUIRE_PTR(dV);
  const uint64_t entries = (uint64_t)B * p->M * p->NH;
  if (entries > MA_NOALLOC_MAX_D_ENTRIES)
    return fail(MA_ERR_LIMIT,
                "ma_flashAttentionBackward_noalloc: B*M*NH = %llu exceeds the scratch maximum of %u "
                "(row, head) entries; use ma_computeD + ma_flashAttentionBackward",
                (unsigned long long)entries, (unsigned)MA_NOALLOC_MAX_D_ENTRIES);
  void* base = nullptr;
  rc = noalloc_scratch(&base);
  if (rc) return rc;
  uint32_t* status = static_cast<uint32_t*>(base);
  __nv_bfloat16* Dv = reinterpret_cast<__nv_bfloat16*>(static_cast<unsigned char*>(base) + kNoallocHeaderBytes);
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  // The scratch keeps the previous call's contents.  D is overwritten in full
  // by computeD below; the status word is cleared only by ma_device_status,
  // which reads it (a time-out is not lost to a later call).
  cudaError_t e = ma::launch_compute_d(reinterpret_cast<bf16p>(dZ), reinterpret_cast<bf16p>(O), Dv, s, st);
  if (e != cudaSuccess) return cuda_fail(e, "computeD launch (no-alloc)");
  e = ma::launch_flash_bwd(reinterpret_cast<bf16p>(dZ), Dv, l, reinterpret_cast<bf16p>(q),
                           reinterpret_cast<bf16p>(k), reinterpret_cast<bf16p>(v), dQ,
                           reinterpret_cast<bf16m>(dK), reinterpret_cast<bf16m>(dV), s, status, st);
  if (e != cudaSuccess) return cuda_fail(e, "flashAttentionBackward launch (no-alloc)");
  return ok();
}

// ---------------------------------------------------------------------------
// Host-resident batches: chunked copy / compute / copy-back pipeline.
// Chunk c uses buffer slot c % kSlots.  Stream order per chunk:
//   h2d : [wait the slot's previous compute done: its inputs are consumed] copy in -> in_ready
//   comp: wait in_ready, [wait the slot's previous copy out done: outputs read] kernels -> comp_done
//   d2h : wait comp_done, copy out -> out_done
// so copies in, kernels and copies out of neighbouring chunks overlap.  The
// slot's previous use may belong to an earlier run of the pipeline, on any
// stream: the waits are on the slot's events, not on stream order.
struct ma_host_pipeline {
  static constexpr int kSlots = 3;
  int device = -1;
  AttentionParams p{};
  uint32_t chunk_B = 0;
  size_t act_elems = 0, row_elems = 0;  // per chunk: chunk_B*M*N, chunk_B*M*NH
  struct Slot {
    __nv_bfloat16 *q = nullptr, *k = nullptr, *v = nullptr, *dO = nullptr, *out = nullptr, *dK = nullptr,
                  *dV = nullptr, *D = nullptr;
    float *l = nullptr, *dQ = nullptr;
    cudaEvent_t in_ready = nullptr, comp_done = nullptr, out_done = nullptr;
    bool used = false;  // a chunk (of this or an earlier run) has recorded its events
  } slot[kSlots];
  cudaStream_t h2d = nullptr, comp = nullptr, d2h = nullptr;
  cudaEvent_t start = nullptr;
  void* block = nullptr;  // one allocation holds every slot's buffers
};

namespace {

void pipeline_free(ma_host_pipeline* pl) {
  for (auto& s : pl->slot) {
    if (s.in_ready) cudaEventDestroy(s.in_ready);
    if (s.comp_done) cudaEventDestroy(s.comp_done);
    if (s.out_done) cudaEventDestroy(s.out_done);
  }
  if (pl->start) cudaEventDestroy(pl->start);
  if (pl->h2d) cudaStreamDestroy(pl->h2d);
  if (pl->comp) cudaStreamDestroy(pl->comp);
  if (pl->d2h) cudaStreamDestroy(pl->d2h);
  if (pl->block) cudaFree(pl->block);
  delete pl;
}

size_t round256(size_t n) { return (n + 255) & ~size_t(255); }

// One chunk of rows [b0, b0 + bc) of a host batch through the pipeline.
int pipeline_chunk(ma_host_pipeline* pl, int c, uint32_t b0, uint32_t bc, bool backward, const ma_bf16* q,
                   const ma_bf16* k, const ma_bf16* v, const ma_bf16* dO, ma_bf16* out, float* l, float* dQ,
                   ma_bf16* dK, ma_bf16* dV) {
  auto& s = pl->slot[c % ma_host_pipeline::kSlots];
  const bool reuse = s.used;
  const size_t per_seq = (size_t)pl->p.M * pl->p.N, per_seq_rows = (size_t)pl->p.M * pl->p.NH;
  const size_t off = (size_t)b0 * per_seq, off_rows = (size_t)b0 * per_seq_rows;
  const size_t n = (size_t)bc * per_seq, n_rows = (size_t)bc * per_seq_rows;
  cudaError_t e = cudaSuccess;
  auto h2d = [&](void* dst, const void* src, size_t bytes) {
    if (e == cudaSuccess) e = cudaMemcpyAsync(dst, src, bytes, cudaMemcpyHostToDevice, pl->h2d);
  };
  auto d2h = [&](void* dst, const void* src, size_t bytes) {
    if (e == cudaSuccess) e = cudaMemcpyAsync(dst, src, bytes, cudaMemcpyDeviceToHost, pl->d2h);
  };
  if (reuse) e = cudaStreamWaitEvent(pl->h2d, s.comp_done, 0);
  h2d(s.q, q + off, n * 2);
  h2d(s.k, k + off, n * 2);
  h2d(s.v, v + off, n * 2);
  if (backward) h2d(s.dO, dO + off, n * 2);
  if (e == cudaSuccess) e = cudaEventRecord(s.in_ready, pl->h2d);
  if (e == cudaSuccess) e = cudaStreamWaitEvent(pl->comp, s.in_ready, 0);
  if (e == cudaSuccess && reuse) e = cudaStreamWaitEvent(pl->comp, s.out_done, 0);
  if (e != cudaSuccess) return cuda_fail(e, "host pipeline: copy in");

  ma::AttnShape sh;
  int rc = check_shape(&pl->p, bc, 0, 0, false, &sh);
  if (rc) return rc;
  uint32_t* status = nullptr;
  rc = device_status_word(&status);
  if (rc) return rc;
  // with the backward, dO is already here: computeD rides in the forward's
  // epilogue at D = 64
  const bool fuse_d = backward && sh.D == 64;
  // with the backward, the forward also writes the zeros the backward adds
  // dQ into (no separate zeroing pass over dQ)
  e = ma::launch_flash_fwd(s.q, s.k, s.v, s.out, s.l, sh, status, pl->comp, fuse_d ? s.dO : nullptr,
                           fuse_d ? s.D : nullptr, backward ? s.dQ : nullptr);
  if (e != cudaSuccess) return cuda_fail(e, "host pipeline: flashAttentionForward launch");
  if (backward) {
    if (!fuse_d) e = ma::launch_compute_d(s.dO, s.out, s.D, sh, pl->comp);
    if (e != cudaSuccess) return cuda_fail(e, "host pipeline: computeD launch");
    e = ma::launch_flash_bwd(s.dO, s.D, s.l, s.q, s.k, s.v, s.dQ, s.dK, s.dV, sh, status, pl->comp,
                             /*accumulate_dq=*/true);
    if (e != cudaSuccess) return cuda_fail(e, "host pipeline: flashAttentionBackward launch");
  }
  e = cudaEventRecord(s.comp_done, pl->comp);
  if (e == cudaSuccess) e = cudaStreamWaitEvent(pl->d2h, s.comp_done, 0);
  d2h(out + off, s.out, n * 2);
  d2h(l + off_rows, s.l, n_rows * 4);
  if (backward) {
    d2h(dQ + off, s.dQ, n * 4);
    d2h(dK + off, s.dK, n * 2);
    d2h(dV + off, s.dV, n * 2);
  }
  if (e == cudaSuccess) e = cudaEventRecord(s.out_done, pl->d2h);
  if (e != cudaSuccess) return cuda_fail(e, "host pipeline: copy out");
  s.used = true;
  return MA_OK;
}

// After a failed run: copies of the chunks already enqueued may still read or
// write the caller's host buffers; wait for them before returning the error,
// so the caller may free or reuse those buffers at once.
void pipeline_drain(ma_host_pipeline* pl) {
  cudaStreamSynchronize(pl->h2d);
  cudaStreamSynchronize(pl->comp);
  cudaStreamSynchronize(pl->d2h);
}

int pipeline_run(ma_host_pipeline* pl, bool backward, const ma_bf16* q, const ma_bf16* k, const ma_bf16* v,
                 const ma_bf16* dO, ma_bf16* out, float* l, float* dQ, ma_bf16* dK, ma_bf16* dV, uint32_t B,
                 ma_stream_t stream) {
  if (!pl) return fail(MA_ERR_NULL, "host pipeline is NULL");
  int dev = -1;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return cuda_fail(e, "cudaGetDevice");
  if (dev != pl->device)
    return fail(MA_ERR_NO_DEVICE, "host pipeline belongs to device %d, current device is %d", pl->device, dev);
  ma::AttnShape sh;
  int rc = check_shape(&pl->p, B, 0, 0, false, &sh);
  if (rc) return rc;
  if (!q || !k || !v || !out || !l || (backward && (!dO || !dQ || !dK || !dV)))
    return fail(MA_ERR_NULL, "a host buffer pointer is NULL");
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  e = cudaEventRecord(pl->start, st);
  if (e == cudaSuccess) e = cudaStreamWaitEvent(pl->h2d, pl->start, 0);
  if (e == cudaSuccess) e = cudaStreamWaitEvent(pl->comp, pl->start, 0);
  if (e == cudaSuccess) e = cudaStreamWaitEvent(pl->d2h, pl->start, 0);
  if (e != cudaSuccess) {
    pipeline_drain(pl);
    return cuda_fail(e, "host pipeline: start");
  }
  const uint32_t nchunks = (B + pl->chunk_B - 1) / pl->chunk_B;
  for (uint32_t c = 0; c < nchunks; ++c) {
    const uint32_t b0 = c * pl->chunk_B;
    const uint32_t bc = B - b0 < pl->chunk_B ? B - b0 : pl->chunk_B;
    rc = pipeline_chunk(pl, (int)c, b0, bc, backward, q, k, v, dO, out, l, dQ, dK, dV);
    if (rc) {
      pipeline_drain(pl);
      return rc;
    }
  }
  // the d2h stream is in order, so its last record covers every chunk (and,
  // through the waits, every kernel and copy in)
  e = cudaStreamWaitEvent(st, pl->slot[(nchunks - 1) % ma_host_pipeline::kSlots].out_done, 0);
  if (e != cudaSuccess) {
    pipeline_drain(pl);
    return cuda_fail(e, "host pipeline: finish");
  }
  return ok();
}

}  // namespace

extern "C" int ma_host_pipeline_create(const AttentionParams* p, uint32_t chunk_B, ma_host_pipeline** out) {
  if (!out) return fail(MA_ERR_NULL, "output pointer is NULL");
  *out = nullptr;
  ma::AttnShape sh;
  int rc = check_shape(p, chunk_B, 0, 0, false, &sh);
  if (rc) return rc;
  uint32_t* status = nullptr;
  rc = device_status_word(&status);  // also checks for an sm_100 device
  if (rc) return rc;
  auto* pl = new ma_host_pipeline();
  cudaGetDevice(&pl->device);
  pl->p = *p;
  pl->chunk_B = chunk_B;
  pl->act_elems = (size_t)chunk_B * p->M * p->N;
  pl->row_elems = (size_t)chunk_B * p->M * p->NH;
  const size_t a2 = round256(pl->act_elems * 2), a4 = round256(pl->act_elems * 4);
  const size_t r2 = round256(pl->row_elems * 2), r4 = round256(pl->row_elems * 4);
  const size_t per_slot = 7 * a2 + a4 + r2 + r4;
  cudaError_t e = cudaMalloc(&pl->block, per_slot * ma_host_pipeline::kSlots);
  if (e != cudaSuccess) {
    pipeline_free(pl);
    return cuda_fail(e, "cudaMalloc(host pipeline buffers)");
  }
  unsigned char* base = static_cast<unsigned char*>(pl->block);
  for (auto& s : pl->slot) {
    auto take = [&](size_t bytes) {
      void* r = base;
      base += bytes;
      return r;
    };
    s.q = static_cast<__nv_bfloat16*>(take(a2));
    s.k = static_cast<__nv_bfloat16*>(take(a2));
    s.v = static_cast<__nv_bfloat16*>(take(a2));
    s.dO = static_cast<__nv_bfloat16*>(take(a2));
    s.out = static_cast<__nv_bfloat16*>(take(a2));
    s.dK = static_cast<__nv_bfloat16*>(take(a2));
    s.dV = static_cast<__nv_bfloat16*>(take(a2));
    s.dQ = static_cast<float*>(take(a4));
    s.D = static_cast<__nv_bfloat16*>(take(r2));
    s.l = static_cast<float*>(take(r4));
    for (cudaEvent_t* ev : {&s.in_ready, &s.comp_done, &s.out_done})
      if (e == cudaSuccess) e = cudaEventCreateWithFlags(ev, cudaEventDisableTiming);
  }
  if (e == cudaSuccess) e = cudaEventCreateWithFlags(&pl->start, cudaEventDisableTiming);
  for (cudaStream_t* st : {&pl->h2d, &pl->comp, &pl->d2h})
    if (e == cudaSuccess) e = cudaStreamCreateWithFlags(st, cudaStreamNonBlocking);
  if (e != cudaSuccess) {
    pipeline_free(pl);
    return cuda_fail(e, "host pipeline streams/events");
  }
  *out = pl;
  return ok();
}

extern "C" int ma_host_pipeline_destroy(ma_host_pipeline* pl) {
  if (!pl) return ok();
  int prev = -1;
  cudaGetDevice(&prev);
  cudaSetDevice(pl->device);
  cudaStreamSynchronize(pl->h2d);
  cudaStreamSynchronize(pl->comp);
  cudaStreamSynchronize(pl->d2h);
  pipeline_free(pl);
  if (prev >= 0) cudaSetDevice(prev);
  return ok();
}

extern "C" int ma_flashAttentionForward_host(ma_host_pipeline* pl, const ma_bf16* q, const ma_bf16* k,
                                             const ma_bf16* v, ma_bf16* out, float* l, uint32_t B,
                                             ma_stream_t stream) {
  return pipeline_run(pl, false, q, k, v, nullptr, out, l, nullptr, nullptr, nullptr, B, stream);
}

extern "C" int ma_attentionForwardBackward_host(ma_host_pipeline* pl, const ma_bf16* q, const ma_bf16* k,
                                                const ma_bf16* v, const ma_bf16* dO, ma_bf16* out, float* l,
                                                float* dQ, ma_bf16* dK, ma_bf16* dV, uint32_t B,
                                                ma_stream_t stream) {
  return pipeline_run(pl, true, q, k, v, dO, out, l, dQ, dK, dV, B, stream);
}
