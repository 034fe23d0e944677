// C++17 device-side mirror of the NeuralSuite GPT API.
//
// The classes keep the reference's names and calling conventions --
// Tensor / Parameter / Module::Register / Layer::Forward / Layer::Backward /
// CrossEntropyLoss / AdamW, GPTBlock, GPTModel -- but their tensors live in
// HBM and every computation is a call into the C ABI of include/ns_b200.h.
// Differences from the CPU reference, all deliberate:
//  * Forward returns a view of a buffer the layer owns (sized once for the
//    largest batch), not a fresh deep copy; it stays valid until the layer's
//    next Forward, which is what the training loop needs and what keeps the
//    step free of allocations after the first one.
//  * Layers remember a view of their input instead of deep-copying it
//    (reference: last_input_ = input); callers keep inputs alive until
//    Backward, as GPTBlock / GPTModel do.
//  * GPTBlock fuses what the reference does in separate passes: each residual
//    add into the LayerNorm that reads the sum (ln_2 for the first, the next
//    block's ln_1 or ln_f for the second) and the residual gradient adds into
//    LayerNorm backward; GELU runs with its lo part as one pass after the
//    mlp_fc GEMM, and the GELU backward inside mlp_fc's bias-gradient pass.
//  * Errors surface as the reference's exception types (std::invalid_argument,
//    std::out_of_range) from the C++ layer; the C ABI turns them into status
//    codes.
#pragma once

#include <cuda_runtime.h>

#include <algorithm>
#include <cmath>
#include <cstdint>
#include <memory>
#include <stdexcept>
#include <string>
#include <utility>
#include <vector>

#include "ns_b200.h"

namespace neuralsuite {
namespace cuda {

// Throws the reference-style exception for a non-OK status.
inline void Check(ns_status s) {
  if (s == NS_OK) return;
  const std::string msg = ns_last_error();
  if (s == NS_ERR_INVALID_ARGUMENT) throw std::invalid_argument(msg);
  if (s == NS_ERR_OUT_OF_RANGE) throw std::out_of_range(msg);
  throw std::runtime_error(msg);
}

inline void CheckCuda(cudaError_t e, const char* what) {
  if (e != cudaSuccess)
    throw std::runtime_error(std::string(what) + ": " + cudaGetErrorString(e));
}

// Owning device allocation.
class DeviceBuffer {
 public:
  DeviceBuffer() = default;
  explicit DeviceBuffer(size_t bytes) : bytes_(bytes) {
    if (bytes > 0) CheckCuda(cudaMalloc(&ptr_, bytes), "cudaMalloc");
  }
  ~DeviceBuffer() {
    if (ptr_) cudaFree(ptr_);
  }
  DeviceBuffer(const DeviceBuffer&) = delete;
  DeviceBuffer& operator=(const DeviceBuffer&) = delete;
  void* get() const { return ptr_; }
  size_t bytes() const { return bytes_; }

 private:
  void* ptr_ = nullptr;
  size_t bytes_ = 0;
};

// fp32 device tensor: shape + pointer, possibly a view of shared storage
// (include/tensor.h:45-148 keeps the same View/Shape/TotalSize vocabulary).
class Tensor {
 public:
  Tensor() = default;
  Tensor(float* data, std::vector<int> shape) : data_(data), shape_(std::move(shape)) {}
  static Tensor Empty(const std::vector<int>& shape) {
    Tensor t;
    t.shape_ = shape;
    const size_t n = t.TotalSize();
    t.owner_ = std::make_shared<DeviceBuffer>(n * sizeof(float));
    t.data_ = static_cast<float*>(t.owner_->get());
    return t;
  }
  float* Data() const { return data_; }
  const std::vector<int>& Shape() const { return shape_; }
  size_t TotalSize() const {
    if (shape_.empty()) return 0;
    size_t n = 1;
    for (int d : shape_) n *= static_cast<size_t>(d);
    return n;
  }
  Tensor View(const std::vector<int>& shape) const {
    Tensor v(data_, shape);
    if (v.TotalSize() > Capacity())
      throw std::invalid_argument("View: the requested shape is larger than the tensor");
    v.owner_ = owner_;
    v.capacity_ = capacity_ ? capacity_ : TotalSize();
    return v;
  }
  size_t Capacity() const { return capacity_ ? capacity_ : TotalSize(); }

 private:
  std::shared_ptr<DeviceBuffer> owner_;
  float* data_ = nullptr;
  std::vector<int> shape_;
  size_t capacity_ = 0;
};

// Value + gradient of the same shape (include/parameter.h:30-59); both are
// views into the owning model's flat buffers once the model binds them.
class Parameter {
 public:
  Parameter() = default;
  explicit Parameter(std::vector<int> dims) : dims_(std::move(dims)) {}
  Tensor& Value() { return value_; }
  Tensor& Grad() { return grad_; }
  const std::vector<int>& Shape() const { return dims_; }
  size_t TotalSize() const {
    size_t n = 1;
    for (int d : dims_) n *= static_cast<size_t>(d);
    return dims_.empty() ? 0 : n;
  }
  void Bind(float* value, float* grad) {
    value_ = Tensor(value, dims_);
    grad_ = Tensor(grad, dims_);
  }
  // The value's tf32 lo part, kept by the owning model (refreshed at the
  // start of every forward pass); nullptr when no model keeps one.
  void BindLo(const float* lo) { lo_ = lo; }
  const float* Lo() const { return lo_; }

 private:
  std::vector<int> dims_;
  Tensor value_, grad_;
  const float* lo_ = nullptr;
};

// Execution context shared by the layers of one model: stream + scratch.
struct Context {
  cudaStream_t stream = nullptr;
  void* scratch = nullptr;
  size_t scratch_bytes = 0;
};

// Module tree with registration-ordered parameters (include/module.h:33-96).
class Module {
 public:
  Module() = default;
  virtual ~Module() = default;
  Module(const Module&) = delete;
  Module& operator=(const Module&) = delete;

  std::vector<Parameter*> Parameters() {
    std::vector<Parameter*> all;
    for (auto& e : own_) all.push_back(e.second);
    for (auto& c : children_) {
      auto sub = c.second->Parameters();
      all.insert(all.end(), sub.begin(), sub.end());
    }
    return all;
  }
  std::vector<std::pair<std::string, Parameter*>> NamedParameters(const std::string& prefix = "") {
    std::vector<std::pair<std::string, Parameter*>> all;
    for (auto& e : own_) all.emplace_back(prefix + e.first, e.second);
    for (auto& c : children_) {
      auto sub = c.second->NamedParameters(prefix + c.first + ".");
      all.insert(all.end(), sub.begin(), sub.end());
    }
    return all;
  }
  void SetContext(Context* ctx) {
    ctx_ = ctx;
    for (auto& c : children_) c.second->SetContext(ctx);
  }

 protected:
  void Register(Parameter* p, const std::string& name) { own_.emplace_back(name, p); }
  void Register(Module* m, const std::string& name) { children_.emplace_back(name, m); }
  cudaStream_t stream() const { return ctx_ ? ctx_->stream : nullptr; }
  Context* ctx_ = nullptr;

 private:
  std::vector<std::pair<std::string, Parameter*>> own_;
  std::vector<std::pair<std::string, Module*>> children_;
};

// include/layer.h:26-60
class Layer : public Module {
 public:
  virtual Tensor Forward(const Tensor& input) = 0;
  virtual Tensor Backward(const Tensor& grad_output) = 0;
};

// Rows of the flattened [N, features] view of a tensor whose last axis is `features`.
inline int Rows(const Tensor& t, int features) {
  return static_cast<int>(t.TotalSize() / static_cast<size_t>(features));
}

// Grows `buf` to hold at least rows x cols floats and returns a [rows, cols] view.
inline Tensor Scratch(Tensor& buf, int rows, int cols) {
  const size_t need = static_cast<size_t>(rows) * cols;
  if (buf.Capacity() < need || buf.Data() == nullptr) buf = Tensor::Empty({rows, cols});
  return buf.View({rows, cols});
}

// include/layers/linear.h:23-131: Y = X W + b with W stored [in, out].
class Linear : public Layer {
 public:
  Linear(int in, int out) : in_(in), out_(out), weight_({in, out}), bias_({out}) {
    Register(&weight_, "weight");
    Register(&bias_, "bias");
  }
  Tensor Forward(const Tensor& x) override { return Run(x, NS_EPI_BIAS, nullptr, nullptr); }
  // Forward with the 3xTF32 operand splits shared with the neighbours: x_lo
  // (or null) is X's tf32 lo part, made by X's producer (it must stay intact
  // until Backward); y_lo (or null) receives Y's, written by the epilogue.
  Tensor ForwardLo(const Tensor& x, const float* x_lo, float* y_lo) {
    return Run(x, NS_EPI_BIAS, nullptr, nullptr, x_lo, y_lo);
  }
  // Y = X W + b, and post = gelu(Y); post_lo (or null) receives post's tf32
  // lo part.  With post_lo the GELU runs as one streaming pass after the
  // GEMM (cheaper than GELU and two more stores in the GEMM epilogue, which
  // hold up its tensor core); without, it is fused into the epilogue.
  Tensor ForwardGelu(const Tensor& x, Tensor* post, float* post_lo = nullptr,
                     const float* x_lo = nullptr) {
    const int n = Rows(x, in_);
    Tensor g = Scratch(post_, n, out_);
    Tensor y;
    if (post_lo) {
      y = Run(x, NS_EPI_BIAS, nullptr, nullptr, x_lo);
      Check(ns_gelu_fwd_lo(y.Data(), g.Data(), post_lo, static_cast<int64_t>(n) * out_, stream()));
    } else {
      y = Run(x, NS_EPI_BIAS_GELU, nullptr, g.Data(), x_lo);
    }
    *post = g;
    return y;
  }
  // X W alone, bias not added: for a consumer that adds bias and residual in
  // its own pass (ns_layernorm_fwd_ex).
  Tensor ForwardNoBias(const Tensor& x, const float* x_lo = nullptr) {
    return Run(x, NS_EPI_STORE, nullptr, nullptr, x_lo);
  }
  // Y = resid + (X W + b)  (the GPTBlock residual ElementwiseAdd fused).
  Tensor ForwardResidual(const Tensor& x, const Tensor& resid, const float* x_lo = nullptr) {
    return Run(x, NS_EPI_BIAS_RESID, resid.Data(), nullptr, x_lo);
  }
  Tensor Backward(const Tensor& dy) override { return BackwardImpl(dy, nullptr); }
  // GeluBackward then Linear::Backward: `dpost` is the gradient at gelu(Y)
  // for this layer's output Y = `pre`; it is overwritten by dpost * gelu'(pre),
  // the gradient at Y (in the same pass as the bias sum and the operand split).
  Tensor BackwardThroughGelu(const Tensor& dpost, const Tensor& pre) {
    return BackwardImpl(dpost, pre.Data());
  }
  Parameter& WeightParam() { return weight_; }
  Parameter& BiasParam() { return bias_; }
  int In() const { return in_; }
  int Out() const { return out_; }

 private:
  // The 3xTF32 GEMMs read each operand's tf32 lo part.  The input X feeds the
  // forward product and the dW product, the weight W the forward and dX
  // products, dY the dX and dW products: each is split once (ns_split_lo)
  // and the copy passed to every product that reads it (ns_gemm_lo).
  bool SplitOk() const { return in_ % 4 == 0 && out_ % 4 == 0; }
  // W's lo part kept by the owning model, when there is one the GEMM can read
  // (16-byte aligned); otherwise the layer splits W itself.
  const float* WeightLo() const {
    const float* lo = weight_.Lo();
    return (lo && (reinterpret_cast<uintptr_t>(lo) & 15) == 0) ? lo : nullptr;
  }

  Tensor Run(const Tensor& x, int epi, const float* aux, float* aux_out,
             const float* x_lo_in = nullptr, float* out_lo = nullptr) {
    if (x.Shape().empty() || x.Shape().back() != in_)
      throw std::invalid_argument("Linear: the last axis of the input is not in_features");
    const int n = Rows(x, in_);
    last_input_ = x;
    const float* x_lo = nullptr;
    const float* w_lo = nullptr;
    if (SplitOk()) {
      if (WeightLo()) {
        w_lo = WeightLo();
      } else {
        Tensor wl = Scratch(w_lo_buf_, in_, out_);
        Check(ns_split_lo(weight_.Value().Data(), in_, out_, out_, wl.Data(), stream()));
        w_lo = wl.Data();
      }
      if (x_lo_in) {
        x_lo = x_lo_in;
      } else {
        Tensor xl = Scratch(x_lo_buf_, n, in_);
        Check(ns_split_lo(x.Data(), n, in_, in_, xl.Data(), stream()));
        x_lo = xl.Data();
      }
    }
    last_x_lo_ = x_lo;
    Tensor y = Scratch(out_buf_, n, out_);
    Check(ns_gemm_lo_out(n, out_, in_, x.Data(), in_, 0, x_lo, weight_.Value().Data(), out_, 0,
                         w_lo, y.Data(), out_, 0.0f, epi, bias_.Value().Data(), aux, aux_out,
                         out_lo, ctx_->scratch, ctx_->scratch_bytes, stream()));
    std::vector<int> shape = x.Shape();
    shape.back() = out_;
    return y.View(shape);
  }
  Tensor BackwardImpl(const Tensor& dy, const float* gelu_pre) {
    const int n = Rows(last_input_, in_);
    if (Rows(dy, out_) != n) throw std::invalid_argument("Linear::Backward: batch mismatch");
    Tensor dx = Scratch(dx_buf_, n, in_);
    // The lo copies of X and W made (or taken) by the forward pass are still current.
    const bool lo = SplitOk();
    const float* x_lo = lo ? last_x_lo_ : nullptr;
    const float* w_lo = lo ? (WeightLo() ? WeightLo() : w_lo_buf_.Data()) : nullptr;
    const float* dy_lo = nullptr;
    if (lo) {
      // db and dY's lo part from one pass over dY (with the GELU backward).
      Tensor dl = Scratch(dy_lo_buf_, n, out_);
      if (gelu_pre)
        Check(ns_bias_grad_split_gelu(dy.Data(), gelu_pre, n, out_, bias_.Grad().Data(), dl.Data(),
                                      ctx_->scratch, ctx_->scratch_bytes, stream()));
      else
        Check(ns_bias_grad_split(dy.Data(), n, out_, bias_.Grad().Data(), dl.Data(), ctx_->scratch,
                                 ctx_->scratch_bytes, stream()));
      dy_lo = dl.Data();
    } else if (gelu_pre) {
      Check(ns_gelu_bwd(dy.Data(), gelu_pre, dy.Data(), static_cast<int64_t>(n) * out_, stream()));
    }
    // dX = dY W^T  (W read transposed in place: no Transpose copy)
    Check(ns_gemm_lo(n, in_, out_, dy.Data(), out_, 0, dy_lo, weight_.Value().Data(), out_, 1, w_lo,
                     dx.Data(), in_, 0.0f, NS_EPI_STORE, nullptr, nullptr, nullptr, ctx_->scratch,
                     ctx_->scratch_bytes, stream()));
    // dW = X^T dY, overwritten (MatMul's Resize+Zeros), X read transposed in place.
    Check(ns_gemm_lo(in_, out_, n, last_input_.Data(), in_, 1, x_lo, dy.Data(), out_, 0, dy_lo,
                     weight_.Grad().Data(), out_, 0.0f, NS_EPI_STORE, nullptr, nullptr, nullptr,
                     ctx_->scratch, ctx_->scratch_bytes, stream()));
    // db = column sums of dY, overwritten (with the split above when it ran).
    if (!lo)
      Check(ns_bias_grad(dy.Data(), n, out_, bias_.Grad().Data(), ctx_->scratch, ctx_->scratch_bytes,
                         stream()));
    return dx.View(last_input_.Shape());
  }

  int in_, out_;
  Parameter weight_, bias_;
  Tensor last_input_;
  Tensor out_buf_, post_, dx_buf_;
  Tensor x_lo_buf_, w_lo_buf_, dy_lo_buf_;  // tf32 lo parts of X, W and dY
  const float* last_x_lo_ = nullptr;        // X's lo part used by the last Forward
};

// include/layers/layernorm.h:22-59 (eps 1e-5, gamma = 1, beta = 0).
class LayerNormLayer : public Layer {
 public:
  explicit LayerNormLayer(int dim, float eps = 1e-5f) : dim_(dim), eps_(eps), gamma_({dim}), beta_({dim}) {
    Register(&gamma_, "gamma");
    Register(&beta_, "beta");
  }
  Tensor Forward(const Tensor& x) override {
    const int n = Rows(x, dim_);
    last_input_ = x;
    Tensor y = Scratch(out_buf_, n, dim_);
    Tensor mean = Scratch(mean_, n, 1), rstd = Scratch(rstd_, n, 1);
    Check(ns_layernorm_fwd(x.Data(), gamma_.Value().Data(), beta_.Value().Data(), y.Data(),
                           mean.Data(), rstd.Data(), n, dim_, eps_, stream()));
    return y.View(x.Shape());
  }
  // Forward with the neighbours fused (ns_layernorm_fwd_ex): with resid, the
  // input is formed as resid + (raw + bias) and written over `raw` (the layer
  // input kept for backward); y_lo (or null) receives the output's tf32 lo part.
  Tensor ForwardEx(const Tensor& raw, const float* bias, const Tensor* resid, float* y_lo) {
    const int n = Rows(raw, dim_);
    last_input_ = raw;
    Tensor y = Scratch(out_buf_, n, dim_);
    Tensor mean = Scratch(mean_, n, 1), rstd = Scratch(rstd_, n, 1);
    Check(ns_layernorm_fwd_ex(raw.Data(), bias, resid ? resid->Data() : nullptr,
                              resid ? raw.Data() : nullptr, gamma_.Value().Data(),
                              beta_.Value().Data(), y.Data(), y_lo, mean.Data(), rstd.Data(), n,
                              dim_, eps_, stream()));
    return y.View(raw.Shape());
  }
  Tensor Backward(const Tensor& dy) override { return BackwardAdd(dy, nullptr); }
  // dx = dresid + LayerNormBackward(dy): the residual ElementwiseAdd fused.
  Tensor BackwardAdd(const Tensor& dy, const Tensor* dresid) {
    const int n = Rows(last_input_, dim_);
    Tensor dx = Scratch(dx_buf_, n, dim_);
    Check(ns_layernorm_bwd(dy.Data(), last_input_.Data(), gamma_.Value().Data(), mean_.Data(),
                           rstd_.Data(), dresid ? dresid->Data() : nullptr, dx.Data(),
                           gamma_.Grad().Data(), beta_.Grad().Data(), n, dim_, ctx_->scratch,
                           ctx_->scratch_bytes, stream()));
    return dx.View(last_input_.Shape());
  }

 private:
  int dim_;
  float eps_;
  Parameter gamma_, beta_;
  Tensor last_input_, out_buf_, mean_, rstd_, dx_buf_;
};

// GELU activation layer (include/activations.h:23-55, kGelu only).
class GeluActivation : public Layer {
 public:
  Tensor Forward(const Tensor& x) override {
    last_input_ = x;
    Tensor y = Scratch(out_buf_, 1, static_cast<int>(x.TotalSize()));
    Check(ns_gelu_fwd(x.Data(), y.Data(), static_cast<int64_t>(x.TotalSize()), stream()));
    return y.View(x.Shape());
  }
  Tensor Backward(const Tensor& dy) override {
    Tensor dx = Scratch(dx_buf_, 1, static_cast<int>(last_input_.TotalSize()));
    Check(ns_gelu_bwd(dy.Data(), last_input_.Data(), dx.Data(),
                      static_cast<int64_t>(last_input_.TotalSize()), stream()));
    return dx.View(last_input_.Shape());
  }

 private:
  Tensor last_input_, out_buf_, dx_buf_;
};

// include/layers/attention.h:330-588 (Forward / Backward; no KV cache).
class MultiHeadAttention : public Layer {
 public:
  MultiHeadAttention(int n_embd, int n_head)
      : n_embd_(n_embd), n_head_(n_head), head_dim_(n_head > 0 ? n_embd / n_head : 0),
        c_attn_(n_embd, 3 * n_embd), c_proj_(n_embd, n_embd) {
    if (n_head <= 0 || n_embd <= 0)
      throw std::invalid_argument("MultiHeadAttention: n_embd and n_head must be positive");
    if (n_embd % n_head != 0)
      throw std::invalid_argument("MultiHeadAttention: n_embd (" + std::to_string(n_embd) +
                                  ") must be divisible by n_head (" + std::to_string(n_head) + ")");
    Register(&c_attn_, "c_attn");
    Register(&c_proj_, "c_proj");
  }
  Tensor Forward(const Tensor& x) override { return ForwardImpl(x, nullptr, nullptr, false); }
  // c_proj output added to `resid` (GPTBlock's first residual add fused).
  Tensor ForwardResidual(const Tensor& x, const Tensor& resid) {
    return ForwardImpl(x, &resid, nullptr, false);
  }
  // c_proj's product without its bias (the caller adds bias and residual in
  // the next LayerNorm); x_lo (or null) is x's tf32 lo part.
  Tensor ForwardNoBias(const Tensor& x, const float* x_lo) { return ForwardImpl(x, nullptr, x_lo, true); }
  const float* OutBias() { return c_proj_.BiasParam().Value().Data(); }
  Tensor Backward(const Tensor& dy) override {
    const int B = batch_, T = seq_, M = B * T;
    Tensor datt = c_proj_.Backward(dy);
    Tensor dqkv = Scratch(dqkv_buf_, M, 3 * n_embd_);
    Check(ns_attn_bwd_lo(qkv_.Data(), qkv_lo_, att_.Data(), datt.Data(), lse_.Data(), B, T, n_head_,
                         head_dim_, dqkv.Data(), ctx_->scratch, ctx_->scratch_bytes, stream()));
    Tensor dx = c_attn_.Backward(dqkv);
    return dx.View({B, T, n_embd_});
  }
  Linear& AttnProjection() { return c_attn_; }
  Linear& OutProjection() { return c_proj_; }
  // The last forward's c_attn output [B*T, 3C] (the KV-cache prefill reads
  // its K and V columns).
  const Tensor& Qkv() const { return qkv_; }

 private:
  Tensor ForwardImpl(const Tensor& x, const Tensor* resid, const float* x_lo, bool no_bias) {
    if (x.Shape().size() != 3 || x.Shape()[2] != n_embd_)
      throw std::invalid_argument("MultiHeadAttention: input must be [B, T, n_embd]");
    batch_ = x.Shape()[0];
    seq_ = x.Shape()[1];
    const int M = batch_ * seq_;
    // qkv's lo part comes out of the c_attn epilogue (the attention kernels'
    // K/V/Q operand split) and the attention output's out of the attention
    // epilogue (c_proj's X split), when rows stay 16-byte aligned.
    const bool lo = n_embd_ % 4 == 0;
    qkv_lo_ = lo ? Scratch(qkv_lo_buf_, M, 3 * n_embd_).Data() : nullptr;
    float* att_lo = lo ? Scratch(att_lo_buf_, M, n_embd_).Data() : nullptr;
    qkv_ = c_attn_.ForwardLo(x.View({M, n_embd_}), x_lo, qkv_lo_);
    att_ = Scratch(att_buf_, M, n_embd_);
    lse_ = Scratch(lse_buf_, batch_ * n_head_, seq_);
    Check(ns_attn_fwd_lo(qkv_.Data(), qkv_lo_, batch_, seq_, n_head_, head_dim_, att_.Data(), att_lo,
                         lse_.Data(), ctx_->scratch, ctx_->scratch_bytes, stream()));
    Tensor y = no_bias ? c_proj_.ForwardNoBias(att_, att_lo)
               : resid ? c_proj_.ForwardResidual(att_, resid->View({M, n_embd_}), att_lo)
                       : c_proj_.ForwardLo(att_, att_lo, nullptr);
    return y.View({batch_, seq_, n_embd_});
  }

  int n_embd_, n_head_, head_dim_;
  Linear c_attn_, c_proj_;
  int batch_ = 0, seq_ = 0;
  Tensor qkv_, att_, lse_;
  Tensor att_buf_, lse_buf_, dqkv_buf_, qkv_lo_buf_, att_lo_buf_;
  float* qkv_lo_ = nullptr;
};

// include/layers/embedding.h:24-92, the table only; GPTModel drives the
// fused token+position kernels.
class Embedding : public Module {
 public:
  Embedding(int num, int dim) : num_(num), dim_(dim), weight_({num, dim}) { Register(&weight_, "weight"); }
  Parameter& WeightParam() { return weight_; }
  int Num() const { return num_; }

 private:
  int num_, dim_;
  Parameter weight_;
};

// include/gpt.h:33-39
struct GPTConfig {
  int vocab_size = 54;
  int block_size = 64;
  int n_layer = 4;
  int n_head = 4;
  int n_embd = 128;
};

// include/gpt.h:45-130: pre-LN block, registration order ln_1, attn, ln_2,
// mlp_fc, mlp_proj (12 parameters).
class GPTBlock : public Layer {
 public:
  explicit GPTBlock(const GPTConfig& c)
      : ln_1_(c.n_embd), attn_(c.n_embd, c.n_head), ln_2_(c.n_embd),
        mlp_fc_(c.n_embd, 4 * c.n_embd), mlp_proj_(4 * c.n_embd, c.n_embd) {
    Register(&ln_1_, "ln_1");
    Register(&attn_, "attn");
    Register(&ln_2_, "ln_2");
    Register(&mlp_fc_, "mlp_fc");
    Register(&mlp_proj_, "mlp_proj");
  }
  // x1 = x + attn(ln_1(x)); x2 = x1 + mlp_proj(gelu(mlp_fc(ln_2(x1))))
  // The operand lo parts come from the producers: ln_1 -> c_attn, ln_2 ->
  // mlp_fc, the GELU pass -> mlp_proj (attention handles its own); the first
  // residual add runs inside ln_2 on c_proj's plain product.
  Tensor Forward(const Tensor& x) override {
    const int C = x.Shape().back(), M = Rows(x, C);
    const float* gelu_lo = ForwardToGelu(x, nullptr, nullptr);
    Tensor x2 = mlp_proj_.ForwardResidual(gelu_, x1_.View({M, C}), gelu_lo);
    return x2.View(x.Shape());
  }
  // The block with its last residual add left open: the input arrives as
  // in_resid + (x + in_bias) (the previous block's open output; in_bias and
  // in_resid null: x as it is) and ln_1 closes it, writing the sum over x.
  // Returns mlp_proj's plain product; the block's output is
  // OpenResid() + (product + OpenBias()), formed by the consumer's LayerNorm
  // (the next block's ln_1 or ln_f) in its own pass, with the same rounding.
  Tensor ForwardOpen(const Tensor& x, const float* in_bias, const Tensor* in_resid) {
    const int C = x.Shape().back(), M = Rows(x, C);
    const float* gelu_lo = ForwardToGelu(x, in_bias, in_resid);
    x1_ = x1_.View({M, C});
    return mlp_proj_.ForwardNoBias(gelu_, gelu_lo).View(x.Shape());
  }
  const float* OpenBias() { return mlp_proj_.BiasParam().Value().Data(); }
  const Tensor& OpenResid() const { return x1_; }
  MultiHeadAttention& Attn() { return attn_; }
  // GPTBlock::Backward (gpt.h:82-100) with the GELU backward fused into the
  // mlp_fc bias-gradient pass and both residual adds fused into LayerNorm
  // backward.
  Tensor Backward(const Tensor& dout) override {
    const int C = dout.Shape().back();
    const int M = Rows(dout, C);
    Tensor dgelu = mlp_proj_.Backward(dout.View({M, C}));
    Tensor dh2 = mlp_fc_.BackwardThroughGelu(dgelu, fc_pre_);
    Tensor dx1 = ln_2_.BackwardAdd(dh2, &dout);
    Tensor dh1 = attn_.Backward(dx1.View(dout.Shape()));
    Tensor dx = ln_1_.BackwardAdd(dh1, &dx1);
    return dx.View(dout.Shape());
  }

 private:
  // ln_1 .. GELU (x1 = x + attn(ln_1(x)) kept in x1_, gelu(mlp_fc(ln_2(x1)))
  // in gelu_); returns the GELU output's lo part (or null).
  const float* ForwardToGelu(const Tensor& x, const float* in_bias, const Tensor* in_resid) {
    const int C = x.Shape().back(), M = Rows(x, C);
    const bool lo = C % 4 == 0;
    float* h1_lo = lo ? Scratch(h1_lo_buf_, M, C).Data() : nullptr;
    Tensor h1 = ln_1_.ForwardEx(x, in_bias, in_resid, h1_lo);
    Tensor raw1 = attn_.ForwardNoBias(h1, h1_lo);
    float* h2_lo = lo ? Scratch(h2_lo_buf_, M, C).Data() : nullptr;
    const Tensor x2d = x.View({M, C});
    Tensor h2 = ln_2_.ForwardEx(raw1, attn_.OutBias(), &x2d, h2_lo);
    x1_ = raw1;  // now x + attn(ln_1(x)), written by ln_2
    float* gelu_lo = mlp_fc_.Out() % 4 == 0 ? Scratch(gelu_lo_buf_, M, mlp_fc_.Out()).Data() : nullptr;
    fc_pre_ = mlp_fc_.ForwardGelu(h2.View({M, C}), &gelu_, gelu_lo, h2_lo);
    return gelu_lo;
  }

  LayerNormLayer ln_1_;
  MultiHeadAttention attn_;
  LayerNormLayer ln_2_;
  Linear mlp_fc_;
  Linear mlp_proj_;
  Tensor x1_, fc_pre_, gelu_, gelu_lo_buf_, h1_lo_buf_, h2_lo_buf_;
};

// Sizes of GPTModel's parameters in registration order (include/gpt.h:143-149,
// 59-63, layers' Register calls): wte, wpe, per block 12 tensors, ln_f 2.
struct ParamSpec {
  int64_t numel;
  int rank;
};
inline std::vector<ParamSpec> GPTParamSpecs(const GPTConfig& c) {
  const int64_t C = c.n_embd;
  std::vector<ParamSpec> v = {{(int64_t)c.vocab_size * C, 2}, {(int64_t)c.block_size * C, 2}};
  for (int l = 0; l < c.n_layer; ++l) {
    const ParamSpec blk[12] = {{C, 1},         {C, 1},     {C * 3 * C, 2}, {3 * C, 1},
                               {C * C, 2},     {C, 1},     {C, 1},         {C, 1},
                               {C * 4 * C, 2}, {4 * C, 1}, {4 * C * C, 2}, {C, 1}};
    v.insert(v.end(), blk, blk + 12);
  }
  v.push_back({C, 1});
  v.push_back({C, 1});
  return v;
}

// Gradient buckets for the data-parallel all-reduce, in launch order.  A
// bucket can be launched once every gradient in it is final, so the natural
// groups follow the backward order: [block L-1 .. ln_f], block L-2, ...,
// block 0, [wte, wpe] (wte's is final only after the embedding backward).
// Each group is cut into pieces of at most `cap` floats (0 = no cap).
struct Bucket {
  int64_t begin, end;
  int group;  // index of the readiness group (0 = first launched)
};
inline std::vector<Bucket> PlanBuckets(const GPTConfig& c, int64_t cap) {
  const auto specs = GPTParamSpecs(c);
  std::vector<int64_t> off(specs.size() + 1, 0);
  for (size_t i = 0; i < specs.size(); ++i) off[i + 1] = off[i] + specs[i].numel;
  auto block_begin = [&](int l) { return off[2 + 12 * l]; };
  std::vector<std::pair<int64_t, int64_t>> groups;
  const int64_t total = off.back();
  if (c.n_layer > 0) {
    groups.emplace_back(block_begin(c.n_layer - 1), total);
    for (int l = c.n_layer - 2; l >= 0; --l) groups.emplace_back(block_begin(l), block_begin(l + 1));
    groups.emplace_back(0, block_begin(0));
  } else {
    groups.emplace_back(off[2], total);
    groups.emplace_back(0, off[2]);
  }
  std::vector<Bucket> out;
  for (size_t g = 0; g < groups.size(); ++g) {
    int64_t b = groups[g].first;
    const int64_t e = groups[g].second;
    while (b < e) {
      const int64_t n = (cap > 0) ? std::min<int64_t>(cap, e - b) : (e - b);
      out.push_back({b, b + n, (int)g});
      b += n;
    }
  }
  return out;
}

// include/losses.h:32-91 on device: Forward computes the mean loss into a
// device float and the gradient (softmax - onehot) / denom in one pass;
// Backward returns that gradient.
class CrossEntropyLoss {
 public:
  void Forward(const Tensor& logits, const int32_t* targets, float denom, float* loss_out,
               int32_t* err_flag, Context* ctx) {
    const int V = logits.Shape().back();
    const int n = Rows(logits, V);
    Tensor d = Scratch(dlogits_, n, V);
    Check(ns_cross_entropy(logits.Data(), targets, n, V, denom, loss_out, d.Data(), err_flag,
                           ctx->scratch, ctx->scratch_bytes, ctx->stream));
    last_ = d;
  }
  Tensor Backward() { return last_; }

 private:
  Tensor dlogits_, last_;
};

// include/gpt.h:136-327.  Parameters and gradients are two flat device
// buffers in registration order, bound into the layers' Parameter views.
class GPTModel : public Module {
 public:
  GPTModel(const GPTConfig& cfg, int max_batch)
      : config_(cfg), max_batch_(max_batch), wte_(cfg.vocab_size, cfg.n_embd),
        wpe_(cfg.block_size, cfg.n_embd), ln_f_(cfg.n_embd) {
    if (cfg.vocab_size <= 0 || cfg.block_size <= 0 || cfg.n_layer < 0 || cfg.n_embd <= 0 ||
        max_batch <= 0)
      throw std::invalid_argument("GPTModel: sizes must be positive");
    Register(&wte_, "wte");
    Register(&wpe_, "wpe");
    for (int i = 0; i < cfg.n_layer; ++i) {
      blocks_.push_back(std::make_unique<GPTBlock>(cfg));
      Register(blocks_.back().get(), "blocks." + std::to_string(i));
    }
    Register(&ln_f_, "ln_f");
    auto params = Parameters();
    offsets_.assign(params.size() + 1, 0);
    for (size_t i = 0; i < params.size(); ++i) {
      offsets_[i + 1] = offsets_[i] + (int64_t)params[i]->TotalSize();
      ranks_.push_back((int)params[i]->Shape().size());
    }
    // Every tensor starts on a 16-byte boundary only if the sizes allow it;
    // the kernels check alignment and fall back to scalar paths otherwise.
    const int64_t total = offsets_.back();
    values_ = std::make_shared<DeviceBuffer>(total * sizeof(float));
    grads_ = std::make_shared<DeviceBuffer>(total * sizeof(float));
    CheckCuda(cudaMemset(grads_->get(), 0, total * sizeof(float)), "cudaMemset");
    // The values' tf32 lo parts, one flat copy split in one pass at the start
    // of every forward (instead of one split per weight per product).
    values_lo_ = std::make_shared<DeviceBuffer>(total * sizeof(float));
    for (size_t i = 0; i < params.size(); ++i) {
      params[i]->Bind(Values() + offsets_[i], Grads() + offsets_[i]);
      params[i]->BindLo(static_cast<const float*>(values_lo_->get()) + offsets_[i]);
    }
    // One scratch area sized for the largest workspace any kernel of the step needs.
    const int M = max_batch * cfg.block_size, C = cfg.n_embd, V = cfg.vocab_size;
    size_t ws = 0;
    auto gw = [&](int m, int n, int k) { ws = std::max(ws, ns_gemm_workspace_size(m, n, k)); };
    gw(M, 3 * C, C); gw(M, C, C); gw(M, 4 * C, C); gw(M, C, 4 * C); gw(M, V, C);
    gw(M, C, 3 * C); gw(M, C, V); gw(C, 3 * C, M); gw(C, C, M); gw(C, 4 * C, M);
    gw(4 * C, C, M); gw(V, C, M);
    ws = std::max(ws, ns_layernorm_bwd_workspace_size(M, C));
    for (int n : {3 * C, C, 4 * C}) ws = std::max(ws, ns_bias_grad_workspace_size(M, n));
    if (cfg.n_head > 0) {
      ws = std::max(ws, ns_attn_fwd_workspace_size(max_batch, cfg.block_size, cfg.n_head,
                                                   C / cfg.n_head));
      ws = std::max(ws, ns_attn_bwd_workspace_size(max_batch, cfg.block_size, cfg.n_head,
                                                   C / cfg.n_head));
    }
    ws = std::max(ws, ns_cross_entropy_workspace_size(M, V));
    ws = std::max(ws, ns_sumsq_workspace_size(total));
    scratch_ = std::make_shared<DeviceBuffer>(std::max<size_t>(ws, 256));
    ctx_storage_.scratch = scratch_->get();
    ctx_storage_.scratch_bytes = scratch_->bytes();
    SetContext(&ctx_storage_);
    small_ = std::make_shared<DeviceBuffer>(64 * sizeof(float));
    CheckCuda(cudaMemset(small_->get(), 0, 64 * sizeof(float)), "cudaMemset");
    tokens_ = std::make_shared<DeviceBuffer>((size_t)M * sizeof(int32_t));
    x0_ = Tensor::Empty({M, C});
  }

  const GPTConfig& Config() const { return config_; }
  int MaxBatch() const { return max_batch_; }
  GPTBlock& Block(int i) { return *blocks_[i]; }
  float* Values() { return static_cast<float*>(values_->get()); }
  float* Grads() { return static_cast<float*>(grads_->get()); }
  int64_t NumParams() const { return offsets_.back(); }
  const std::vector<int64_t>& Offsets() const { return offsets_; }
  const std::vector<int>& Ranks() const { return ranks_; }
  // Device scalars: [0] loss, [1] token error flag (int bits), [2] target error flag,
  // [3] grad sum of squares, [8..15] AdamW hyper-parameters.
  float* Small() { return static_cast<float*>(small_->get()); }
  Tensor& Logits() { return logits_; }
  void SetStream(cudaStream_t s) { ctx_storage_.stream = s; }
  const Context& Ctx() const { return ctx_storage_; }
  cudaStream_t Stream() const { return ctx_storage_.stream; }

  // GPTModel::Forward (gpt.h:192-232) on device int32 tokens [B, T].
  Tensor Forward(const int32_t* tokens, int B, int T) {
    if (B <= 0 || B > max_batch_) throw std::invalid_argument("GPTModel::Forward: batch exceeds max_batch");
    if (T <= 0) throw std::invalid_argument("GPTModel::Forward: empty sequence");
    if (T > config_.block_size)
      throw std::out_of_range("GPTModel::Forward: sequence longer than block_size");
    B_ = B;
    T_ = T;
    const int M = B * T, C = config_.n_embd;
    CheckCuda(cudaMemcpyAsync(tokens_->get(), tokens, (size_t)M * sizeof(int32_t),
                              cudaMemcpyDeviceToDevice, Stream()),
              "token copy");
    // Parameter lo parts for this pass (the values may have changed since the
    // last one: optimizer step, broadcast, or a write through ns_gpt_params).
    constexpr int64_t kSplitChunk = int64_t(1) << 30;
    for (int64_t o = 0; o < NumParams(); o += kSplitChunk) {
      const int n = (int)std::min(kSplitChunk, NumParams() - o);
      Check(ns_split_lo(Values() + o, 1, n, n, static_cast<float*>(values_lo_->get()) + o, Stream()));
    }
    Tensor x = x0_.View({B, T, C});
    Check(ns_embedding_fwd(Tokens(), B, T, wte_.WeightParam().Value().Data(), config_.vocab_size,
                           wpe_.WeightParam().Value().Data(), config_.block_size, C, x.Data(),
                           reinterpret_cast<int32_t*>(Small() + 1), Stream()));
    // Each block's last residual add stays open and is formed by the next
    // LayerNorm (the next block's ln_1, or ln_f) in its own pass.
    const float* open_bias = nullptr;
    Tensor open_resid;
    for (auto& blk : blocks_) {
      x = blk->ForwardOpen(x, open_bias, open_bias ? &open_resid : nullptr);
      open_bias = blk->OpenBias();
      open_resid = blk->OpenResid();
    }
    float* xf_lo = C % 4 == 0 ? Scratch(xf_lo_buf_, M, C).Data() : nullptr;
    xf_ = ln_f_.ForwardEx(x, open_bias, open_bias ? &open_resid : nullptr, xf_lo).View({M, C});
    xf_lo_ = xf_lo;
    // logits = x_2d . wte^T (gpt.h:226-228): wte read as a K-major operand, no transpose copy.
    logits_ = Scratch(logits_buf_, M, config_.vocab_size);
    Check(ns_gemm_lo(M, config_.vocab_size, C, xf_.Data(), C, 0, xf_lo_,
                     wte_.WeightParam().Value().Data(), C, 1, WteLo(), logits_.Data(),
                     config_.vocab_size, 0.0f, NS_EPI_STORE, nullptr, nullptr, nullptr,
                     ctx_storage_.scratch, ctx_storage_.scratch_bytes, Stream()));
    return logits_;
  }

  // CrossEntropyLoss on the last logits; denom = rows * world_size.
  void LossBackward(const int32_t* targets, float denom) {
    criterion_.Forward(logits_, targets, denom, Small(), reinterpret_cast<int32_t*>(Small() + 2),
                       &ctx_storage_);
  }

  // GPTModel::Backward (gpt.h:234-272).  `on_group_ready(g)` is called in
  // stream order when every gradient of bucket group g is final.
  template <typename OnReady>
  void Backward(OnReady&& on_group_ready) {
    const int M = B_ * T_, C = config_.n_embd, V = config_.vocab_size;
    Tensor dlogits = criterion_.Backward();
    // dlogits' lo part, split once for both head products.
    const float* dl_lo = nullptr;
    if (V % 4 == 0 && C % 4 == 0) {
      Tensor dl = Scratch(dlogits_lo_buf_, M, V);
      Check(ns_split_lo(dlogits.Data(), M, V, V, dl.Data(), Stream()));
      dl_lo = dl.Data();
    }
    // dx = dlogits . wte  (wte read N-major in place)
    Tensor dx = Scratch(dx_head_, M, C);
    Check(ns_gemm_lo(M, C, V, dlogits.Data(), V, 0, dl_lo, wte_.WeightParam().Value().Data(), C,
                     0, WteLo(), dx.Data(), C, 0.0f, NS_EPI_STORE, nullptr, nullptr, nullptr,
                     ctx_storage_.scratch, ctx_storage_.scratch_bytes, Stream()));
    // head term of the tied wte gradient, dlogits^T . x, written first (the
    // embedding backward adds its own sum to it at the end, gpt.h:262-269).
    Check(ns_gemm_lo(V, C, M, dlogits.Data(), V, 1, dl_lo, xf_.Data(), C, 0, xf_lo_,
                     wte_.WeightParam().Grad().Data(), C, 0.0f, NS_EPI_STORE, nullptr, nullptr,
                     nullptr, ctx_storage_.scratch, ctx_storage_.scratch_bytes, Stream()));
    Tensor d = ln_f_.Backward(dx.View({B_, T_, C}));
    int group = 0;
    for (int l = (int)blocks_.size() - 1; l >= 0; --l) {
      d = blocks_[l]->Backward(d);
      on_group_ready(group++);
    }
    if (blocks_.empty()) on_group_ready(group++);
    Check(ns_embedding_bwd(Tokens(), B_, T_, d.Data(), V, config_.block_size, C,
                           wte_.WeightParam().Grad().Data(), 1, wpe_.WeightParam().Grad().Data(),
                           Stream()));
    on_group_ready(group++);
  }
  void Backward() {
    Backward([](int) {});
  }

  int32_t* Tokens() { return static_cast<int32_t*>(tokens_->get()); }

 private:
  // wte's lo part for the tied head's products (it needs C % 4 == 0 and a
  // 16-byte aligned start; otherwise the GEMM splits wte itself).
  const float* WteLo() {
    const float* lo = wte_.WeightParam().Lo();
    return (config_.n_embd % 4 == 0 && (reinterpret_cast<uintptr_t>(lo) & 15) == 0) ? lo : nullptr;
  }

  GPTConfig config_;
  int max_batch_;
  Embedding wte_, wpe_;
  std::vector<std::unique_ptr<GPTBlock>> blocks_;
  LayerNormLayer ln_f_;
  CrossEntropyLoss criterion_;
  std::vector<int64_t> offsets_;
  std::vector<int> ranks_;
  std::shared_ptr<DeviceBuffer> values_, grads_, values_lo_, scratch_, small_, tokens_;
  Context ctx_storage_;
  Tensor x0_, xf_, logits_, logits_buf_, dx_head_, xf_lo_buf_, dlogits_lo_buf_;
  const float* xf_lo_ = nullptr;  // ln_f output's lo part (the head's A operand)
  int B_ = 0, T_ = 0;
};

// include/optimizers.h:143-253 over the model's flat buffers: one launch per
// step, decay wd on rank >= 2 tensors (the reference's heuristic without
// parameter groups), hyper-parameters in device memory.
class AdamW {
 public:
  AdamW(GPTModel& model, float lr = 1e-3f, float b1 = 0.9f, float b2 = 0.95f, float eps = 1e-8f,
        float wd = 0.01f)
      : model_(model) {
    const int64_t n = model.NumParams();
    m_ = std::make_shared<DeviceBuffer>(n * sizeof(float));
    v_ = std::make_shared<DeviceBuffer>(n * sizeof(float));
    CheckCuda(cudaMemset(m_->get(), 0, n * sizeof(float)), "cudaMemset");
    CheckCuda(cudaMemset(v_->get(), 0, n * sizeof(float)), "cudaMemset");
    wd_ = wd;
    for (int r : model.Ranks()) decay_.push_back(r >= 2 ? wd : 0.0f);
    const float h[7] = {lr, b1, b2, eps, 1.0f, 1.0f, 0.0f};
    CheckCuda(cudaMemcpy(Hyper(), h, sizeof(h), cudaMemcpyHostToDevice), "cudaMemcpy");
  }
  void SetLearningRate(float lr) {
    lr_host_ = lr;
    CheckCuda(cudaMemcpyAsync(Hyper(), &lr_host_, sizeof(float), cudaMemcpyHostToDevice,
                              model_.Stream()),
              "cudaMemcpyAsync");
    CheckCuda(cudaStreamSynchronize(model_.Stream()), "cudaStreamSynchronize");
  }
  void Step() {
    Check(ns_adamw_flat_device(model_.Values(), model_.Grads(), static_cast<float*>(m_->get()),
                               static_cast<float*>(v_->get()), model_.NumParams(),
                               model_.Offsets().data(), decay_.data(), (int)decay_.size(), Hyper(),
                               model_.Stream()));
  }
  void ZeroGrad() {
    CheckCuda(cudaMemsetAsync(model_.Grads(), 0, model_.NumParams() * sizeof(float), model_.Stream()),
              "cudaMemsetAsync");
  }
  float* Hyper() { return model_.Small() + 8; }
  // Optimizer state, for checkpoints: first and second moments (flat, the
  // parameters' offsets) and the weight decay given to rank >= 2 tensors.
  float* M() { return static_cast<float*>(m_->get()); }
  float* V() { return static_cast<float*>(v_->get()); }
  float WeightDecay() const { return wd_; }

 private:
  GPTModel& model_;
  std::shared_ptr<DeviceBuffer> m_, v_;
  std::vector<float> decay_;
  float wd_ = 0.0f;
  float lr_host_ = 0.0f;
};

}  // namespace cuda
}  // namespace neuralsuite
