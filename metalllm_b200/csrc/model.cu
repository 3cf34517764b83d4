// model.cu -- metalLLM's training step (config 5) on CUDA: the counterpart of
// the reference's Model (model.h:104-860) for a batch of B sequences.  It owns
// the weights, gradients, Adam state and activation buffers (allocated once,
// like model.h:210-330) and enqueues forward (model.h:414-523), backward
// (model.h:537-711) and the Adam step (model.h:726-757) on a stream with the
// library's kernels: the attention path (computeQKV, flashAttention*,
// computeD, the GEMMs of attention.metal:301-455) plus train_sm100.cu's
// element-wise kernels and the tcgen05 GEMM for the MLP and the vocabulary
// projection.  Nothing synchronises the host, so a whole step can be captured
// into a CUDA graph once the model has run one step.
#include <algorithm>
#include <cmath>
#include <cstring>
#include <random>
#include <string>
#include <vector>

#include "common.cuh"

namespace ma {
namespace {

using bf16 = __nv_bfloat16;

struct Param {
  std::string name;
  size_t count;
  bf16* weight;       // what the forward reads
  void* grad;         // where the backward writes the gradient
  bool grad_f32;      // fp32 gradient (converted when gathered) or bf16
  size_t offset;      // into the flat optimizer arrays
};

struct LayerNormBufs {
  bf16 *gamma, *beta, *xn, *out;
  float *stdev, *dgamma, *dbeta;
};

struct Layer {
  LayerNormBufs ln1, ln2;
  bf16 *qw, *kw, *vw, *projw, *up, *dp;
  bf16 *q, *k, *v, *attn, *res1, *mlp_v, *res2;
  float* l;
  uint8_t* mask;
  // fp32 weight gradients (parts of the model's zeroed-per-step block)
  float *dqw, *dkw, *dvw, *dprojw, *dup, *ddp;
};

}  // namespace
}  // namespace ma

struct ma_model {
  MaModelConfig cfg{};
  int device = -1;  // the device current at create; every buffer lives there
  int R = 0, T = 0, E = 0, H = 0, V = 0, NH = 0, D = 0, L = 0, Bt = 0;
  std::vector<void*> allocs;
  std::vector<ma::Param> params;
  std::vector<ma::Layer> layers;
  ma::LayerNormBufs lnf{};
  __nv_bfloat16 *embed = nullptr, *pos = nullptr, *linw = nullptr;
  __nv_bfloat16 *embed_out = nullptr, *logits = nullptr, *dlogits = nullptr;
  __nv_bfloat16 *dstream = nullptr, *dbranch = nullptr, *dzattn = nullptr, *dattnd = nullptr;
  __nv_bfloat16 *dk = nullptr, *dv = nullptr, *dmlpv = nullptr, *dpos = nullptr;
  float* dlinw = nullptr;
  // every split-K weight gradient, contiguous, zeroed by one memset per backward
  float* wgrads = nullptr;
  size_t wgrads_count = 0;
  __nv_bfloat16* dq16 = nullptr;  // dQ rounded to bf16 for computeGradDx/Dw
  float *dq = nullptr, *demb = nullptr;
  float *loss_rows = nullptr, *lse_rows = nullptr, *loss_mean = nullptr;
  const int* tokens = nullptr;   // last forward's inputs (device)
  const int* targets = nullptr;
  float* master = nullptr;
  __nv_bfloat16 *mom = nullptr, *var = nullptr;
  ma::AdamSegment* segs = nullptr;  // device table, one entry per parameter
  long long max_count = 0;
  size_t nparam = 0;
  float step_count = 0.0f;
  uint32_t* status = nullptr;
};

namespace ma {
namespace {

template <typename T>
cudaError_t alloc(ma_model* m, T** p, size_t count) {
  void* q = nullptr;
  cudaError_t e = cudaMalloc(&q, count * sizeof(T) + 16);
  if (e != cudaSuccess) return e;
  m->allocs.push_back(q);
  *p = static_cast<T*>(q);
  return cudaMemset(q, 0, count * sizeof(T) + 16);
}

void fill_normal(std::vector<uint16_t>& w, float sd, std::mt19937_64& gen) {
  std::normal_distribution<float> dist(0.0f, sd);
  for (auto& x : w) {
    const float f = dist(gen);
    uint32_t u;
    std::memcpy(&u, &f, 4);
    u += 0x7FFFu + ((u >> 16) & 1u);  // round to nearest even
    x = (uint16_t)(u >> 16);
  }
}

cudaError_t upload(const std::vector<uint16_t>& h, bf16* d) {
  return cudaMemcpy(d, h.data(), h.size() * 2, cudaMemcpyHostToDevice);
}

}  // namespace
}  // namespace ma

namespace {

thread_local std::string g_model_error;

int merr(int code, const std::string& msg) {
  g_model_error = msg;
  return code;
}

#define MA_M_CUDA(call, what)                                                                    \
  do {                                                                                          \
    cudaError_t e_ = (call);                                                                    \
    if (e_ != cudaSuccess)                                                                      \
      return merr(MA_ERR_CUDA, std::string(what) + ": " + cudaGetErrorName(e_) + " (" +          \
                                   cudaGetErrorString(e_) + ")");                              \
  } while (0)

// Work for a model must be enqueued with its own device current: from another
// device the kernels would run there on this device's pointers.
int check_device(const ma_model* m) {
  int dev = -1;
  MA_M_CUDA(cudaGetDevice(&dev), "cudaGetDevice");
  if (dev != m->device)
    return merr(MA_ERR_NO_DEVICE, "the model lives on device " + std::to_string(m->device) +
                                      ", the current device is " + std::to_string(dev));
  return MA_OK;
}

}  // namespace

extern "C" {

const char* ma_model_last_error(void) { return g_model_error.c_str(); }

int ma_model_create(const MaModelConfig* c, ma_model** out) {
  using namespace ma;
  if (!c || !out) return merr(MA_ERR_NULL, "NULL argument");
  *out = nullptr;
  if (c->B == 0 || c->T == 0 || c->E == 0 || c->NH == 0 || c->layers == 0 || c->mlp_scale == 0 ||
      c->vocab == 0)
    return merr(MA_ERR_SHAPE, "empty model configuration");
  if (c->E % c->NH != 0 || (c->E / c->NH != 64 && c->E / c->NH != 128))
    return merr(MA_ERR_SHAPE, "head size E/NH must be 64 or 128");
  if (c->E % 64 != 0 || c->vocab % 64 != 0 || ((uint64_t)c->E * c->mlp_scale) % 64 != 0)
    return merr(MA_ERR_SHAPE, "E, vocab and the MLP width must be multiples of 64");
  if ((uint64_t)c->B * c->T >= (1u << 30)) return merr(MA_ERR_LIMIT, "B*T too large");
  if (c->E > 16384 || (uint64_t)c->E * c->mlp_scale > 65536 || c->vocab > (1u << 20) || c->layers > 4096)
    return merr(MA_ERR_LIMIT, "E <= 16384, E*mlp_scale <= 65536, vocab <= 2^20 and layers <= 4096");
  int dev = 0, major = 0;
  MA_M_CUDA(cudaGetDevice(&dev), "cudaGetDevice");
  MA_M_CUDA(cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev), "device attribute");
  if (major != 10) return merr(MA_ERR_NO_DEVICE, "libmetalattn needs an sm_100 device");

  ma_model* m = new ma_model();
  m->cfg = *c;
  m->device = dev;
  m->Bt = (int)c->B;
  m->T = (int)c->T;
  m->E = (int)c->E;
  m->R = m->Bt * m->T;
  m->H = (int)(c->E * c->mlp_scale);
  m->V = (int)c->vocab;
  m->NH = (int)c->NH;
  m->D = m->E / m->NH;
  m->L = (int)c->layers;
  const size_t R = m->R, E = m->E, H = m->H, V = m->V, T = m->T;
  std::mt19937_64 gen(c->seed);
  auto fail = [&](cudaError_t e, const char* what) {
    for (void* p : m->allocs) cudaFree(p);
    delete m;
    return merr(MA_ERR_CUDA, std::string(what) + ": " + cudaGetErrorName(e));
  };
  cudaError_t e = cudaSuccess;
#define ALLOC(ptr, n)                                    \
  do {                                                   \
    if ((e = alloc(m, &(ptr), (n))) != cudaSuccess) return fail(e, "cudaMalloc"); \
  } while (0)
  // parameters, initialised as main.cpp:1594-1620 (normal, Xavier, Kaiming)
  auto param = [&](const char* name, bf16** w, size_t rows, size_t cols, float sd, bool ones,
                   void* grad, bool grad_f32) -> cudaError_t {
    cudaError_t e2 = alloc(m, w, rows * cols);
    if (e2 != cudaSuccess) return e2;
    std::vector<uint16_t> h(rows * cols, ones ? 0x3F80 : 0);
    if (sd > 0.0f) fill_normal(h, sd, gen);
    e2 = upload(h, *w);
    if (e2 != cudaSuccess) return e2;
    m->params.push_back({name, rows * cols, *w, grad, grad_f32, 0});
    return cudaSuccess;
  };
  ALLOC(m->demb, V * E);
  ALLOC(m->dpos, T * E);
  if ((e = param("embed", &m->embed, V, E, 0.02f, false, m->demb, true)) != cudaSuccess) return fail(e, "param");
  if ((e = param("pos", &m->pos, T, E, 0.02f, false, m->dpos, false)) != cudaSuccess) return fail(e, "param");
  m->layers.resize(m->L);
  // the weight gradients that split-K GEMMs add into, in one block
  m->wgrads_count = (size_t)m->L * (4 * (size_t)E * E + 2 * (size_t)E * H) + (size_t)E * V;
  ALLOC(m->wgrads, m->wgrads_count);
  float* wg_next = m->wgrads;
  auto wg_take = [&](size_t n) {
    float* p = wg_next;
    wg_next += n;
    return p;
  };
  const float small = 0.02f / std::sqrt(2.0f * m->L);
  auto ln_bufs = [&](LayerNormBufs& ln) -> cudaError_t {
    cudaError_t e2;
    if ((e2 = alloc(m, &ln.xn, R * E)) || (e2 = alloc(m, &ln.out, R * E)) || (e2 = alloc(m, &ln.stdev, R)) ||
        (e2 = alloc(m, &ln.dgamma, E)) || (e2 = alloc(m, &ln.dbeta, E)))
      return e2;
    return cudaSuccess;
  };
  for (int n = 0; n < m->L; ++n) {
    Layer& y = m->layers[n];
    const std::string pre = "layer" + std::to_string(n) + ".";
    if ((e = ln_bufs(y.ln1)) || (e = ln_bufs(y.ln2))) return fail(e, "cudaMalloc");
    y.dqw = wg_take(E * E);
    y.dkw = wg_take(E * E);
    y.dvw = wg_take(E * E);
    y.dprojw = wg_take(E * E);
    y.dup = wg_take(E * H);
    y.ddp = wg_take(H * E);
    const float xav = std::sqrt(2.0f / (float)(E + E)), kai = std::sqrt(2.0f / (float)E);
    if ((e = param((pre + "ln1_gamma").c_str(), &y.ln1.gamma, 1, E, 0.0f, true, y.ln1.dgamma, true)) ||
        (e = param((pre + "ln1_beta").c_str(), &y.ln1.beta, 1, E, 0.0f, false, y.ln1.dbeta, true)) ||
        (e = param((pre + "qw").c_str(), &y.qw, E, E, xav, false, y.dqw, true)) ||
        (e = param((pre + "kw").c_str(), &y.kw, E, E, xav, false, y.dkw, true)) ||
        (e = param((pre + "vw").c_str(), &y.vw, E, E, xav, false, y.dvw, true)) ||
        (e = param((pre + "projw").c_str(), &y.projw, E, E, small, false, y.dprojw, true)) ||
        (e = param((pre + "ln2_gamma").c_str(), &y.ln2.gamma, 1, E, 0.0f, true, y.ln2.dgamma, true)) ||
        (e = param((pre + "ln2_beta").c_str(), &y.ln2.beta, 1, E, 0.0f, false, y.ln2.dbeta, true)) ||
        (e = param((pre + "up").c_str(), &y.up, E, H, kai, false, y.dup, true)) ||
        (e = param((pre + "dp").c_str(), &y.dp, H, E, small, false, y.ddp, true)))
      return fail(e, "param");
    ALLOC(y.q, R * E);
    ALLOC(y.k, R * E);
    ALLOC(y.v, R * E);
    ALLOC(y.attn, R * E);
    ALLOC(y.l, R * m->NH);
    ALLOC(y.res1, R * E);
    ALLOC(y.mlp_v, R * H);
    ALLOC(y.mask, R * H);
    ALLOC(y.res2, R * E);
  }
  if ((e = ln_bufs(m->lnf))) return fail(e, "cudaMalloc");
  m->dlinw = wg_take(E * V);
  if ((e = param("lnf_gamma", &m->lnf.gamma, 1, E, 0.0f, true, m->lnf.dgamma, true)) ||
      (e = param("lnf_beta", &m->lnf.beta, 1, E, 0.0f, false, m->lnf.dbeta, true)) ||
      (e = param("linw", &m->linw, E, V, 0.02f, false, m->dlinw, true)))
    return fail(e, "param");
  ALLOC(m->embed_out, R * E);
  ALLOC(m->logits, R * V);
  ALLOC(m->dlogits, R * V);
  ALLOC(m->dstream, R * E);
  ALLOC(m->dbranch, R * E);
  ALLOC(m->dzattn, R * E);
  ALLOC(m->dattnd, R * m->NH);
  ALLOC(m->dq, R * E);
  ALLOC(m->dq16, R * E);
  ALLOC(m->dk, R * E);
  ALLOC(m->dv, R * E);
  ALLOC(m->dmlpv, R * H);
  ALLOC(m->loss_rows, R);
  ALLOC(m->lse_rows, R);
  ALLOC(m->loss_mean, 1);
  ALLOC(m->status, 1);
  // flat optimizer state (model.h:300-325): fp32 master copy of the bf16
  // weights and bf16 moments (the gradients are read where the backward
  // wrote them)
  size_t off = 0;
  for (auto& p : m->params) {
    p.offset = off;
    off += (p.count + 7) & ~(size_t)7;
  }
  m->nparam = off;
  ALLOC(m->master, off);

  ALLOC(m->mom, off);
  ALLOC(m->var, off);
  for (auto& p : m->params) {
    std::vector<uint16_t> h(p.count);
    std::vector<float> f(p.count);
    if ((e = cudaMemcpy(h.data(), p.weight, p.count * 2, cudaMemcpyDeviceToHost))) return fail(e, "cudaMemcpy");
    for (size_t i = 0; i < p.count; ++i) {
      const uint32_t u = (uint32_t)h[i] << 16;
      std::memcpy(&f[i], &u, 4);
    }
    if ((e = cudaMemcpy(m->master + p.offset, f.data(), p.count * 4, cudaMemcpyHostToDevice)))
      return fail(e, "cudaMemcpy");
  }
  // the optimizer's segment table (one fused launch per step)
  std::vector<ma::AdamSegment> segs;
  for (const auto& p : m->params) {
    if (p.count % 4 != 0) return fail(cudaErrorInvalidValue, "parameter size not a multiple of 4");
    segs.push_back({p.grad, p.weight, (long long)p.count, (long long)p.offset, p.grad_f32 ? 1 : 0});
    m->max_count = std::max(m->max_count, (long long)p.count);
  }
  ALLOC(m->segs, segs.size());
  if ((e = cudaMemcpy(m->segs, segs.data(), segs.size() * sizeof(ma::AdamSegment), cudaMemcpyHostToDevice)))
    return fail(e, "cudaMemcpy");
#undef ALLOC
  *out = m;
  return MA_OK;
}

int ma_model_destroy(ma_model* m) {
  if (!m) return MA_OK;
  for (void* p : m->allocs) cudaFree(p);
  delete m;
  return MA_OK;
}

int ma_model_forward(ma_model* m, const int32_t* tokens, const int32_t* targets, ma_stream_t stream) {
  using namespace ma;
  if (!m || !tokens || !targets) return merr(MA_ERR_NULL, "NULL argument");
  if (int rc = check_device(m)) return rc;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  m->tokens = tokens;
  m->targets = targets;
  const int R = m->R, E = m->E, H = m->H, V = m->V;
  AttnShape s{m->T, E, m->D, m->NH, m->Bt, 0, m->Bt * m->NH};
  MA_M_CUDA(launch_embed_forward(tokens, m->embed, m->pos, m->embed_out, R, m->T, E, st), "embedForward");
  bf16* hidden = m->embed_out;
  for (Layer& y : m->layers) {
    MA_M_CUDA(launch_layernorm_forward(hidden, y.ln1.xn, y.ln1.out, y.ln1.gamma, y.ln1.beta, y.ln1.stdev, R, E,
                                       1e-5f, st), "layernormForward");
    MA_M_CUDA(launch_qkv(y.ln1.out, y.q, y.k, y.v, y.qw, y.kw, y.vw, R, E, m->status, st), "computeQKV");
    MA_M_CUDA(launch_flash_fwd(y.q, y.k, y.v, y.attn, y.l, s, m->status, st), "flashAttentionForward");
    // projForward with the residual add in its epilogue: res1 = hidden + attn . projw
    MA_M_CUDA(launch_gemm_bf16_act(y.attn, y.projw, true, y.res1, nullptr, hidden, 3, R, E, E, m->status, st),
              "projForward + residualAdd");
    MA_M_CUDA(launch_layernorm_forward(y.res1, y.ln2.xn, y.ln2.out, y.ln2.gamma, y.ln2.beta, y.ln2.stdev, R, E,
                                       1e-5f, st), "layernormForward");
    MA_M_CUDA(launch_gemm_bf16_act(y.ln2.out, y.up, true, y.mlp_v, y.mask, nullptr, 1, R, H, E, m->status, st),
              "mlpForwardOne + relu");
    MA_M_CUDA(launch_gemm_bf16_act(y.mlp_v, y.dp, true, y.res2, nullptr, y.res1, 3, R, E, H, m->status, st),
              "mlpForwardTwo + residualAdd");
    hidden = y.res2;
  }
  MA_M_CUDA(launch_layernorm_forward(hidden, m->lnf.xn, m->lnf.out, m->lnf.gamma, m->lnf.beta, m->lnf.stdev, R,
                                     E, 1e-5f, st), "layernormForward");
  MA_M_CUDA(launch_gemm_bf16(m->lnf.out, false, m->linw, true, m->logits, R, V, E, m->status, st),
            "linearForward");
  MA_M_CUDA(launch_loss_forward(m->logits, targets, m->loss_rows, m->lse_rows, m->loss_mean, R, V, st),
            "lossForward");
  return MA_OK;
}

// Weight gradient G[M][N] (fp32, zeroed at the start of the backward) =
// X^T . Y over all B*T rows (X [rows][M], Y [rows][N], bf16), split along K
// with the partial sums added by TMA reductions; Adam rounds it to bf16, as
// the reference's bf16 gradient buffers hold it.
static cudaError_t wgrad(ma_model* m, const __nv_bfloat16* X, const __nv_bfloat16* Y, float* G, int M, int N,
                         cudaStream_t st) {
  return ma::launch_gemm_splitk_f32(X, Y, G, M, N, m->R, m->status, st, /*zero=*/false);
}

int ma_model_backward(ma_model* m, ma_stream_t stream) {
  using namespace ma;
  if (!m || !m->tokens) return merr(MA_ERR_NULL, "backward before forward");
  if (int rc = check_device(m)) return rc;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  const int R = m->R, E = m->E, H = m->H, V = m->V;
  AttnShape s{m->T, E, m->D, m->NH, m->Bt, 0, m->Bt * m->NH};
  MA_M_CUDA(cudaMemsetAsync(m->wgrads, 0, m->wgrads_count * sizeof(float), st), "zero weight gradients");
  MA_M_CUDA(launch_loss_backward(m->logits, m->targets, m->lse_rows, m->dlogits, R, V, st), "lossBackward");
  // linearBackward: dStream = dLogits . W^T ; dW = lnf.out^T . dLogits
  MA_M_CUDA(launch_gemm_bf16(m->dlogits, false, m->linw, false, m->dstream, R, E, V, m->status, st),
            "linearBackward dX");
  MA_M_CUDA(wgrad(m, m->lnf.out, m->dlogits, m->dlinw, E, V, st), "linearBackward dW");
  MA_M_CUDA(launch_layernorm_backward(m->dstream, m->lnf.xn, m->lnf.gamma, m->lnf.stdev, m->lnf.dgamma,
                                      m->lnf.dbeta, R, E, st), "layernormBackward");
  for (int n = m->L - 1; n >= 0; --n) {
    Layer& y = m->layers[n];
    // MLP: dV = (dStream . Dp^T) * mask; dUp = ln2.out^T . dV; dDp = V^T . dStream;
    // dBranch = dV . Up^T
    MA_M_CUDA(launch_gemm_bf16_act(m->dstream, y.dp, false, m->dmlpv, y.mask, nullptr, 2, R, H, E, m->status, st),
              "mlpBackwardOne + mask");
    MA_M_CUDA(wgrad(m, y.ln2.out, m->dmlpv, y.dup, E, H, st), "mlpBackwardTwo dUp");
    MA_M_CUDA(wgrad(m, y.mlp_v, m->dstream, y.ddp, H, E, st), "mlpBackwardTwo dDp");
    MA_M_CUDA(launch_gemm_bf16(m->dmlpv, false, y.up, false, m->dbranch, R, E, H, m->status, st),
              "mlpBackwardTwo dX");
    // LayerNorm backward with the residual add: dbranch = dLN2 + dstream
    MA_M_CUDA(launch_layernorm_backward(m->dbranch, y.ln2.xn, y.ln2.gamma, y.ln2.stdev, y.ln2.dgamma,
                                        y.ln2.dbeta, R, E, st, m->dstream), "layernormBackward + residualAdd");
    // attention block
    MA_M_CUDA(wgrad(m, y.attn, m->dbranch, y.dprojw, E, E, st), "projBackwarddW");
    // projBackwarddX with computeD fused into its epilogue
    MA_M_CUDA(launch_proj_backward_dx_d(m->dbranch, y.projw, m->dzattn, y.attn, m->dattnd, R, E, m->D, m->status,
                                        st), "projBackwarddX + computeD");
    MA_M_CUDA(launch_flash_bwd(m->dzattn, m->dattnd, y.l, y.q, y.k, y.v, m->dq, m->dk, m->dv, s, m->status, st),
              "flashAttentionBackward");
    // dQ rounded to bf16 once for both products (their fp32-operand kernels
    // apply the same rounding on chip)
    MA_M_CUDA(launch_cast_f32_bf16(m->dq, m->dq16, (long long)R * E, st), "castFloatToBfloat dQ");
    // dX straight to bf16 (the fp32 dX rounded by castFloatToBfloat gives the same values)
    MA_M_CUDA(launch_grad_dx_bf16(m->dstream, false, y.qw, y.kw, y.vw, m->dq16, m->dk, m->dv, R, E, m->status, st),
              "computeGradDx + castFloatToBfloat");
    MA_M_CUDA(launch_grad_dw_splitk_f32(y.ln1.out, m->dq16, m->dk, m->dv, y.dqw, y.dkw, y.dvw, R, E, m->status,
                                        st), "computeGradDw");
    MA_M_CUDA(launch_layernorm_backward(m->dstream, y.ln1.xn, y.ln1.gamma, y.ln1.stdev, y.ln1.dgamma,
                                        y.ln1.dbeta, R, E, st, m->dbranch), "layernormBackward + residualAdd");
  }
  MA_M_CUDA(launch_embed_backward(m->tokens, m->dstream, m->demb, m->dpos, m->Bt, m->T, V, E, st),
            "embedBackward");
  return MA_OK;
}

int ma_model_step(ma_model* m, ma_stream_t stream) {
  using namespace ma;
  if (!m) return merr(MA_ERR_NULL, "NULL model");
  if (int rc = check_device(m)) return rc;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  m->step_count += 1.0f;
  const float t = m->step_count;
  const float lr_t = m->cfg.lr * std::sqrt(1.0f - std::pow(0.999f, t)) / (1.0f - std::pow(0.9f, t));
  MA_M_CUDA(launch_adam_fused(m->segs, (int)m->params.size(), m->max_count, m->master, m->mom, m->var, lr_t, st),
            "MetalStep");
  return MA_OK;
}

int ma_model_tensor(ma_model* m, const char* name, void** ptr, uint64_t* bytes) {
  if (!m || !name || !ptr || !bytes) return merr(MA_ERR_NULL, "NULL argument");
  const std::string n(name);
  const size_t R = m->R, E = m->E, V = m->V;
  for (const auto& p : m->params) {
    if (n == p.name) {
      *ptr = p.weight;
      *bytes = p.count * 2;
      return MA_OK;
    }
    if (n == "grad." + p.name) {
      *ptr = p.grad;
      *bytes = p.count * (p.grad_f32 ? 4 : 2);
      return MA_OK;
    }
  }
  struct Named {
    const char* name;
    void* p;
    size_t bytes;
  } named[] = {{"logits", m->logits, R * V * 2},   {"loss_rows", m->loss_rows, R * 4},
               {"loss", m->loss_mean, 4},         {"lse_rows", m->lse_rows, R * 4},
               {"embed_out", m->embed_out, R * E * 2}, {"master", m->master, m->nparam * 4},
               {"dstream", m->dstream, R * E * 2}};
  for (const auto& x : named) {
    if (n == x.name) {
      *ptr = x.p;
      *bytes = x.bytes;
      return MA_OK;
    }
  }
  const size_t H = m->H;
  struct Named2 {
    const char* name;
    void* p;
    size_t bytes;
  } scratch[] = {{"dmlpv", m->dmlpv, R * H * 2}, {"dbranch", m->dbranch, R * E * 2},
                 {"dzattn", m->dzattn, R * E * 2},
                 {"dlogits", m->dlogits, R * V * 2}};
  for (const auto& x : scratch) {
    if (n == x.name) {
      *ptr = x.p;
      *bytes = x.bytes;
      return MA_OK;
    }
  }
  for (int i = 0; i < m->L; ++i) {  // per-layer activations "layer<i>.<buffer>"
    const ma::Layer& y = m->layers[i];
    const std::string pre = "layer" + std::to_string(i) + ".";
    struct Named3 {
      const char* name;
      void* p;
      size_t bytes;
    } act[] = {{"mlp_v", y.mlp_v, R * H * 2}, {"mask", y.mask, R * H}, {"ln2_out", y.ln2.out, R * E * 2},
               {"ln2_xn", y.ln2.xn, R * E * 2}, {"attn", y.attn, R * E * 2}, {"res1", y.res1, R * E * 2},
               {"res2", y.res2, R * E * 2}, {"ln1_out", y.ln1.out, R * E * 2}};
    for (const auto& x : act) {
      if (n == pre + x.name) {
        *ptr = x.p;
        *bytes = x.bytes;
        return MA_OK;
      }
    }
  }
  return merr(MA_ERR_RANGE, "no tensor named " + n);
}

// Synchronous host copies of a named tensor (tests, checkpoints).  Writing a
// parameter also refreshes its fp32 master copy, so the optimizer continues
// from the written values.
int ma_model_read(ma_model* m, const char* name, void* host, uint64_t bytes) {
  void* p = nullptr;
  uint64_t n = 0;
  int rc = ma_model_tensor(m, name, &p, &n);
  if (rc) return rc;
  if (!host || bytes != n) return merr(MA_ERR_RANGE, std::string("size mismatch for ") + name);
  if ((rc = check_device(m))) return rc;
  MA_M_CUDA(cudaMemcpy(host, p, n, cudaMemcpyDeviceToHost), "cudaMemcpy");
  return MA_OK;
}

int ma_model_write(ma_model* m, const char* name, const void* host, uint64_t bytes) {
  void* p = nullptr;
  uint64_t n = 0;
  int rc = ma_model_tensor(m, name, &p, &n);
  if (rc) return rc;
  if (!host || bytes != n) return merr(MA_ERR_RANGE, std::string("size mismatch for ") + name);
  if ((rc = check_device(m))) return rc;
  MA_M_CUDA(cudaMemcpy(p, host, n, cudaMemcpyHostToDevice), "cudaMemcpy");
  for (const auto& q : m->params) {
    if (q.name == name) {
      std::vector<float> f(q.count);
      const uint16_t* h = static_cast<const uint16_t*>(host);
      for (size_t i = 0; i < q.count; ++i) {
        const uint32_t u = (uint32_t)h[i] << 16;
        std::memcpy(&f[i], &u, 4);
      }
      MA_M_CUDA(cudaMemcpy(m->master + q.offset, f.data(), q.count * 4, cudaMemcpyHostToDevice), "cudaMemcpy");
    }
  }
  return MA_OK;
}

uint32_t ma_model_param_count(ma_model* m) { return m ? (uint32_t)m->params.size() : 0; }

const char* ma_model_param_name(ma_model* m, uint32_t i) {
  return (m && i < m->params.size()) ? m->params[i].name.c_str() : nullptr;
}

int ma_model_status(ma_model* m, uint32_t* status) {
  if (!m || !status) return merr(MA_ERR_NULL, "NULL argument");
  if (int rc = check_device(m)) return rc;
  MA_M_CUDA(cudaMemcpy(status, m->status, 4, cudaMemcpyDeviceToHost), "cudaMemcpy");
  return MA_OK;
}

}  // extern "C"
