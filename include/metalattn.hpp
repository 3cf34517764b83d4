/*
 * metalattn.hpp -- C++ host-side mirror of the reference's MetalAttention
 * harness (main.cpp:955-1284) over the C ABI of metalattn.h: one attention
 * block (computeQKV, flashAttentionForward, projForward; and the backward
 * projBackwarddW, projBackwarddX, computeD, flashAttentionBackward,
 * computeGradDx, computeGradDw) on host bf16 matrices, with the same
 * constructor arguments (m = sequence length, n = embedding width, d = head
 * size) and the same forward / backward signatures, plus an optional batch
 * of B sequences stacked along the rows.
 *
 * Matrices are raw bf16 bits (uint16_t), row-major: x, out, dRes, dX are
 * [B*m][n]; the weights and their gradients [n][n] (row = input feature).  As
 * the reference's host does (main.cpp:1236-1239), the fp32 dX and dQw the
 * kernels produce are rounded to bf16 on the host (round to nearest even).
 * Device buffers are allocated once by the constructor.  Errors throw
 * std::runtime_error with the library's message (the reference exits).
 *
 * metalattn::Model mirrors the reference's Model (model.h) over ma_model_*.
 *
 * Header-only; needs cuda_runtime.h and linking with -lmetalattn -lcudart.
 */
#ifndef METALATTN_HPP_
#define METALATTN_HPP_

#include <cuda_runtime.h>

#include <cstdint>
#include <cstring>
#include <stdexcept>
#include <string>
#include <vector>

#include "metalattn.h"

namespace metalattn {

inline void check(int rc, const char* what) {
  if (rc != MA_OK) throw std::runtime_error(std::string(what) + ": " + ma_last_error_string());
}

inline void check_cuda(cudaError_t e, const char* what) {
  if (e != cudaSuccess) throw std::runtime_error(std::string(what) + ": " + cudaGetErrorString(e));
}

// fp32 -> bf16 bits, round to nearest even (NaN stays NaN)
inline uint16_t to_bf16(float f) {
  uint32_t u;
  std::memcpy(&u, &f, 4);
  if ((u & 0x7FFFFFFFu) > 0x7F800000u) return static_cast<uint16_t>((u >> 16) | 0x40u);
  u += 0x7FFFu + ((u >> 16) & 1u);
  return static_cast<uint16_t>(u >> 16);
}

class CudaAttention {
 public:
  CudaAttention(int m, int n, int d, int batch = 1)
      : B_(batch), params_{static_cast<uint32_t>(m), static_cast<uint32_t>(n), static_cast<uint32_t>(d),
                           static_cast<uint32_t>(d > 0 ? n / d : 0)} {
    if (m <= 0 || n <= 0 || d <= 0 || batch <= 0 || n % d != 0)
      throw std::runtime_error("CudaAttention: invalid shape");
    act_ = static_cast<size_t>(batch) * m * n;
    rows_ = static_cast<size_t>(batch) * m * (n / d);
    w_ = static_cast<size_t>(n) * n;
    check_cuda(cudaStreamCreateWithFlags(&stream_, cudaStreamNonBlocking), "cudaStreamCreate");
    for (void** p : {&x_, &q_, &k_, &v_, &out_, &projOut_, &dRes_, &dZ_, &dK_, &dV_}) alloc(p, act_ * 2);
    for (void** p : {&qw_, &kw_, &vw_, &projw_, &dProjw_, &dKw_, &dVw_}) alloc(p, w_ * 2);
    alloc(&dQ_, act_ * 4);
    alloc(&dX_, act_ * 4);
    alloc(&dQw_, w_ * 4);
    alloc(&l_, rows_ * 4);
    alloc(&D_, rows_ * 2);
  }

  CudaAttention(const CudaAttention&) = delete;
  CudaAttention& operator=(const CudaAttention&) = delete;

  ~CudaAttention() {
    if (stream_) cudaStreamSynchronize(stream_);
    for (void* p : owned_) cudaFree(p);
    if (stream_) cudaStreamDestroy(stream_);
  }

  // main.cpp:1066-1127: out = (causal attention of X Wq, X Wk, X Wv) Wp
  void forward(const uint16_t* x, const uint16_t* qw, const uint16_t* kw, const uint16_t* vw,
               const uint16_t* projw, uint16_t* out) {
    h2d(x_, x, act_ * 2);
    h2d(qw_, qw, w_ * 2);
    h2d(kw_, kw, w_ * 2);
    h2d(vw_, vw, w_ * 2);
    h2d(projw_, projw, w_ * 2);
    const ma_stream_t s = reinterpret_cast<ma_stream_t>(stream_);
    check(ma_computeQKV(bf(x_), bf(q_), bf(k_), bf(v_), bf(qw_), bf(kw_), bf(vw_), &params_, B_, s), "computeQKV");
    check(ma_flashAttentionForward(bf(q_), bf(k_), bf(v_), bf(out_), f32(l_), &params_, B_, s),
          "flashAttentionForward");
    check(ma_projForward(bf(out_), bf(projw_), bf(projOut_), &params_, B_, s), "projForward");
    d2h(out, projOut_, act_ * 2);
    sync();
  }

  // main.cpp:1129-1243: gradients of the block given dRes = dL/d(out)
  void backward(const uint16_t* dRes, uint16_t* dprojw, uint16_t* dX, uint16_t* dqw, uint16_t* dkw,
                uint16_t* dvw) {
    h2d(dRes_, dRes, act_ * 2);
    const ma_stream_t s = reinterpret_cast<ma_stream_t>(stream_);
    check(ma_projBackwarddW(bf(out_), bf(dRes_), bf(dProjw_), &params_, B_, s), "projBackwarddW");
    check(ma_projBackwarddX(bf(dRes_), bf(projw_), bf(dZ_), &params_, B_, s), "projBackwarddX");
    check(ma_computeD(bf(dZ_), bf(out_), bf(D_), &params_, B_, s), "computeD");
    check(ma_flashAttentionBackward(bf(dZ_), bf(D_), f32(l_), bf(q_), bf(k_), bf(v_), f32(dQ_), bf(dK_), bf(dV_),
                                    &params_, B_, s),
          "flashAttentionBackward");
    check(ma_computeGradDx(f32(dX_), bf(qw_), bf(kw_), bf(vw_), f32(dQ_), bf(dK_), bf(dV_), &params_, B_, s),
          "computeGradDx");
    check(ma_computeGradDw(bf(x_), f32(dQ_), bf(dK_), bf(dV_), f32(dQw_), bf(dKw_), bf(dVw_), &params_, B_, s),
          "computeGradDw");
    std::vector<float> dx(act_), dq(w_);
    d2h(dprojw, dProjw_, w_ * 2);
    d2h(dx.data(), dX_, act_ * 4);
    d2h(dq.data(), dQw_, w_ * 4);
    d2h(dkw, dKw_, w_ * 2);
    d2h(dvw, dVw_, w_ * 2);
    sync();
    for (size_t i = 0; i < act_; ++i) dX[i] = to_bf16(dx[i]);
    for (size_t i = 0; i < w_; ++i) dqw[i] = to_bf16(dq[i]);
  }

  const AttentionParams& params() const { return params_; }
  cudaStream_t stream() const { return stream_; }

 private:
  void alloc(void** p, size_t bytes) {
    check_cuda(cudaMalloc(p, bytes), "cudaMalloc");
    owned_.push_back(*p);
  }
  void h2d(void* dst, const void* src, size_t bytes) {
    check_cuda(cudaMemcpyAsync(dst, src, bytes, cudaMemcpyHostToDevice, stream_), "cudaMemcpyAsync");
  }
  void d2h(void* dst, const void* src, size_t bytes) {
    check_cuda(cudaMemcpyAsync(dst, src, bytes, cudaMemcpyDeviceToHost, stream_), "cudaMemcpyAsync");
  }
  void sync() {
    check_cuda(cudaStreamSynchronize(stream_), "cudaStreamSynchronize");
    uint32_t status = 0;
    check(ma_device_status(&status, reinterpret_cast<ma_stream_t>(stream_)), "ma_device_status");
    if (status) throw std::runtime_error("a kernel gave up on a bounded wait (device status word set)");
  }
  static ma_bf16* bf(void* p) { return static_cast<ma_bf16*>(p); }
  static float* f32(void* p) { return static_cast<float*>(p); }

  uint32_t B_;
  AttentionParams params_;
  size_t act_ = 0, rows_ = 0, w_ = 0;
  cudaStream_t stream_ = nullptr;
  std::vector<void*> owned_;
  void *x_ = nullptr, *q_ = nullptr, *k_ = nullptr, *v_ = nullptr, *out_ = nullptr, *projOut_ = nullptr;
  void *dRes_ = nullptr, *dZ_ = nullptr, *dK_ = nullptr, *dV_ = nullptr;
  void *qw_ = nullptr, *kw_ = nullptr, *vw_ = nullptr, *projw_ = nullptr, *dProjw_ = nullptr, *dKw_ = nullptr,
       *dVw_ = nullptr;
  void *dQ_ = nullptr, *dX_ = nullptr, *dQw_ = nullptr, *l_ = nullptr, *D_ = nullptr;
};

// The reference's Model (model.h:17-860): the whole training step (embedding,
// layers of LayerNorm + attention + MLP, final LayerNorm, vocabulary
// projection, loss, Adam) with the constructor's shape arguments (m = block
// size, v = vocabulary, e = embedding width, s = MLP scale, d = head size)
// plus the layer count, a batch of B sequences, the learning rate and the
// initialisation seed.  forward() takes host token ids and targets
// ([B][m] uint32, as model.h:414 reads them) and returns the mean loss.
class Model {
 public:
  Model(int m, int v, int e, int s, int d, int layers, int batch = 1, float lr = 0.003f, uint64_t seed = 0)
      : B_(batch), m_(m) {
    if (m <= 0 || v <= 0 || e <= 0 || s <= 0 || d <= 0 || layers <= 0 || batch <= 0 || e % d != 0)
      throw std::runtime_error("Model: invalid shape");
    MaModelConfig cfg{static_cast<uint32_t>(batch), static_cast<uint32_t>(m), static_cast<uint32_t>(e),
                      static_cast<uint32_t>(e / d), static_cast<uint32_t>(layers), static_cast<uint32_t>(s),
                      static_cast<uint32_t>(v), lr, seed};
    if (ma_model_create(&cfg, &model_) != MA_OK)
      throw std::runtime_error(std::string("ma_model_create: ") + ma_model_last_error());
    check_cuda(cudaStreamCreateWithFlags(&stream_, cudaStreamNonBlocking), "cudaStreamCreate");
    const size_t n = static_cast<size_t>(batch) * m;
    check_cuda(cudaMalloc(&tokens_, n * 4), "cudaMalloc");
    check_cuda(cudaMalloc(&targets_, n * 4), "cudaMalloc");
  }

  Model(const Model&) = delete;
  Model& operator=(const Model&) = delete;

  ~Model() {
    if (stream_) cudaStreamSynchronize(stream_);
    if (tokens_) cudaFree(tokens_);
    if (targets_) cudaFree(targets_);
    if (model_) ma_model_destroy(model_);
    if (stream_) cudaStreamDestroy(stream_);
  }

  // model.h:414-536
  float forward(const uint32_t* tokens, const uint32_t* targets) {
    const size_t n = static_cast<size_t>(B_) * m_;
    check_cuda(cudaMemcpyAsync(tokens_, tokens, n * 4, cudaMemcpyHostToDevice, stream_), "cudaMemcpyAsync");
    check_cuda(cudaMemcpyAsync(targets_, targets, n * 4, cudaMemcpyHostToDevice, stream_), "cudaMemcpyAsync");
    run(ma_model_forward(model_, static_cast<const int32_t*>(tokens_), static_cast<const int32_t*>(targets_),
                         reinterpret_cast<ma_stream_t>(stream_)),
        "ma_model_forward");
    check_cuda(cudaStreamSynchronize(stream_), "cudaStreamSynchronize");
    float loss = 0.0f;
    run(ma_model_read(model_, "loss", &loss, sizeof(loss)), "ma_model_read");
    return loss;
  }

  // model.h:538-712
  void backward() { run(ma_model_backward(model_, reinterpret_cast<ma_stream_t>(stream_)), "ma_model_backward"); }

  // model.h:726-757 (Adam)
  void step() {
    run(ma_model_step(model_, reinterpret_cast<ma_stream_t>(stream_)), "ma_model_step");
    check_cuda(cudaStreamSynchronize(stream_), "cudaStreamSynchronize");
    uint32_t status = 0;
    run(ma_model_status(model_, &status), "ma_model_status");
    if (status) throw std::runtime_error("a kernel gave up on a bounded wait (model status word set)");
  }

  // synchronous copies of a named tensor (a parameter, "grad.<name>", "logits", ...)
  void read(const char* name, void* host, uint64_t bytes) {
    check_cuda(cudaStreamSynchronize(stream_), "cudaStreamSynchronize");
    run(ma_model_read(model_, name, host, bytes), "ma_model_read");
  }
  void write(const char* name, const void* host, uint64_t bytes) {
    check_cuda(cudaStreamSynchronize(stream_), "cudaStreamSynchronize");
    run(ma_model_write(model_, name, host, bytes), "ma_model_write");
  }

  ma_model* handle() const { return model_; }
  cudaStream_t stream() const { return stream_; }

 private:
  static void run(int rc, const char* what) {
    if (rc != MA_OK) throw std::runtime_error(std::string(what) + ": " + ma_model_last_error());
  }

  int B_, m_;
  ma_model* model_ = nullptr;
  cudaStream_t stream_ = nullptr;
  void* tokens_ = nullptr;
  void* targets_ = nullptr;
};

}  // namespace metalattn

#endif  // METALATTN_HPP_
