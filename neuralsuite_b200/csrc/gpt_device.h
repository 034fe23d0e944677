// C++17 device-side mirror of the NeuralSuite GPT API.
//
// The classes keep the reference's names and calling conventions --
// Tensor / Parameter / Module::Register / Layer::Forward / Layer::Backward /
// CrossEntropyLoss / AdamW, GPTBlock, GPTModel -- but their tensors live in
// HBM and every computation is a call into the C ABI of include/ns_b200.h.
// Differences from the CPU reference, all deliberate:
//  * Forward returns a view of a buffer the layer owns (sized once for the
//    largest batch), not a fresh deep copy; it stays valid until the layer's
//    next Forward, which is what the training loop needs and what makes the
//    step free of allocations (so it can be captured in a CUDA graph).
//  * Layers remember a view of their input instead of deep-copying it
//    (reference: last_input_ = input); callers keep inputs alive until
//    Backward, as GPTBlock / GPTModel do.
//  * GPTBlock fuses what the reference does in separate passes: GELU into
//    the mlp_fc GEMM, the residual adds into the c_proj / mlp_proj GEMMs and
//    into LayerNorm backward, the GELU backward into the mlp_proj dX GEMM.
//  * Errors surface as the reference's exception types (std::invalid_argument,
//    std::out_of_range) from the C++ layer; the C ABI turns them into status
//    codes.
#pragma once

#include <cuda_runtime.h>

#include <cmath>
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

 private:
  std::vector<int> dims_;
  Tensor value_, grad_;
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
  // Y = X W + b, and post = gelu(Y) (GeluForward fused into the epilogue).
  Tensor ForwardGelu(const Tensor& x, Tensor* post) {
    const int n = Rows(x, in_);
    Tensor g = Scratch(post_, n, out_);
    Tensor y = Run(x, NS_EPI_BIAS_GELU, nullptr, g.Data());
    *post = g;
    return y;
  }
  // Y = resid + (X W + b)  (the GPTBlock residual ElementwiseAdd fused).
  Tensor ForwardResidual(const Tensor& x, const Tensor& resid) {
    return Run(x, NS_EPI_BIAS_RESID, resid.Data(), nullptr);
  }
  Tensor Backward(const Tensor& dy) override { return BackwardImpl(dy, NS_EPI_STORE, nullptr); }
  // dX = (dY W^T) * gelu'(pre): Linear::Backward followed by GeluBackward.
  Tensor BackwardGelu(const Tensor& dy, const Tensor& gelu_input) {
    return BackwardImpl(dy, NS_EPI_GELU_BWD, gelu_input.Data());
  }
  Parameter& WeightParam() { return weight_; }
  Parameter& BiasParam() { return bias_; }
  int In() const { return in_; }
  int Out() const { return out_; }

 private:
  Tensor Run(const Tensor& x, int epi, const float* aux, float* aux_out) {
    if (x.Shape().empty() || x.Shape().back() != in_)
      throw std::invalid_argument("Linear: the last axis of the input is not in_features");
    const int n = Rows(x, in_);
    last_input_ = x;
    Tensor y = Scratch(out_buf_, n, out_);
    Check(ns_gemm(n, out_, in_, x.Data(), in_, 0, weight_.Value().Data(), out_, 0, y.Data(), out_,
                  0.0f, epi, bias_.Value().Data(), aux, aux_out, ctx_->scratch,
                  ctx_->scratch_bytes, stream()));
    std::vector<int> shape = x.Shape();
    shape.back() = out_;
    return y.View(shape);
  }
  Tensor BackwardImpl(const Tensor& dy, int epi, const float* aux) {
    const int n = Rows(last_input_, in_);
    if (Rows(dy, out_) != n) throw std::invalid_argument("Linear::Backward: batch mismatch");
    Tensor dx = Scratch(dx_buf_, n, in_);
    // dX = dY W^T  (W read transposed in place: no Transpose copy)
    Check(ns_gemm(n, in_, out_, dy.Data(), out_, 0, weight_.Value().Data(), out_, 1, dx.Data(), in_,
                  0.0f, epi, nullptr, aux, nullptr, ctx_->scratch, ctx_->scratch_bytes, stream()));
    // dW = X^T dY, overwritten (MatMul's Resize+Zeros), X read transposed in place.
    Check(ns_gemm(in_, out_, n, last_input_.Data(), in_, 1, dy.Data(), out_, 0,
                  weight_.Grad().Data(), out_, 0.0f, NS_EPI_STORE, nullptr, nullptr, nullptr,
                  ctx_->scratch, ctx_->scratch_bytes, stream()));
    // db = column sums of dY, overwritten.
    Check(ns_bias_grad(dy.Data(), n, out_, bias_.Grad().Data(), ctx_->scratch, ctx_->scratch_bytes,
                       stream()));
    return dx.View(last_input_.Shape());
  }

  int in_, out_;
  Parameter weight_, bias_;
  Tensor last_input_;
  Tensor out_buf_, post_, dx_buf_;
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
  Tensor Forward(const Tensor& x) override { return ForwardImpl(x, nullptr); }
  // c_proj output added to `resid` (GPTBlock's first residual add fused).
  Tensor ForwardResidual(const Tensor& x, const Tensor& resid) { return ForwardImpl(x, &resid); }
  Tensor Backward(const Tensor& dy) override {
    const int B = batch_, T = seq_, M = B * T;
    Tensor datt = c_proj_.Backward(dy);
    Tensor dqkv = Scratch(dqkv_buf_, M, 3 * n_embd_);
    Check(ns_attn_bwd(qkv_.Data(), att_.Data(), datt.Data(), lse_.Data(), B, T, n_head_, head_dim_,
                      dqkv.Data(), ctx_->scratch, ctx_->scratch_bytes, stream()));
    Tensor dx = c_attn_.Backward(dqkv);
    return dx.View({B, T, n_embd_});
  }
  Linear& AttnProjection() { return c_attn_; }
  Linear& OutProjection() { return c_proj_; }

 private:
  Tensor ForwardImpl(const Tensor& x, const Tensor* resid) {
    if (x.Shape().size() != 3 || x.Shape()[2] != n_embd_)
      throw std::invalid_argument("MultiHeadAttention: input must be [B, T, n_embd]");
    batch_ = x.Shape()[0];
    seq_ = x.Shape()[1];
    const int M = batch_ * seq_;
    qkv_ = c_attn_.Forward(x.View({M, n_embd_}));
    att_ = Scratch(att_buf_, M, n_embd_);
    lse_ = Scratch(lse_buf_, batch_ * n_head_, seq_);
    Check(ns_attn_fwd(qkv_.Data(), batch_, seq_, n_head_, head_dim_, att_.Data(), lse_.Data(),
                      stream()));
    Tensor y = resid ? c_proj_.ForwardResidual(att_, resid->View({M, n_embd_}))
                     : c_proj_.Forward(att_);
    return y.View({batch_, seq_, n_embd_});
  }

  int n_embd_, n_head_, head_dim_;
  Linear c_attn_, c_proj_;
  int batch_ = 0, seq_ = 0;
  Tensor qkv_, att_, lse_;
  Tensor att_buf_, lse_buf_, dqkv_buf_;
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
  Tensor Forward(const Tensor& x) override {
    Tensor h1 = ln_1_.Forward(x);
    x1_ = attn_.ForwardResidual(h1, x);
    Tensor h2 = ln_2_.Forward(x1_);
    fc_pre_ = mlp_fc_.ForwardGelu(h2.View({Rows(h2, h2.Shape().back()), h2.Shape().back()}), &gelu_);
    Tensor x2 = mlp_proj_.ForwardResidual(gelu_, x1_.View({Rows(x1_, x1_.Shape().back()), x1_.Shape().back()}));
    return x2.View(x.Shape());
  }
  // GPTBlock::Backward (gpt.h:82-100) with the GELU backward fused into the
  // mlp_proj dX GEMM and both residual adds fused into LayerNorm backward.
  Tensor Backward(const Tensor& dout) override {
    const int C = dout.Shape().back();
    const int M = Rows(dout, C);
    Tensor dfc = mlp_proj_.BackwardGelu(dout.View({M, C}), fc_pre_);
    Tensor dh2 = mlp_fc_.Backward(dfc);
    Tensor dx1 = ln_2_.BackwardAdd(dh2, &dout);
    Tensor dh1 = attn_.Backward(dx1.View(dout.Shape()));
    Tensor dx = ln_1_.BackwardAdd(dh1, &dx1);
    return dx.View(dout.Shape());
  }

 private:
  LayerNormLayer ln_1_;
  MultiHeadAttention attn_;
  LayerNormLayer ln_2_;
  Linear mlp_fc_;
  Linear mlp_proj_;
  Tensor x1_, fc_pre_, gelu_;
};

}  // namespace cuda
}  // namespace neuralsuite
