// Test infrastructure: NOT part of the product.
//
// A thin C ABI over the NeuralSuite reference's own C++ classes, so the tests
// and the CPU-baseline leg of bench.py can run the reference implementation of
// the GPT training step on identical inputs.  It is compiled (by
// oracle/Makefile) against the reference's headers and its src/tensor.cpp +
// src/tokenizer.cpp, with the reference's Release flags, into
// oracle/_ref/libnsref.so.  Nothing here re-implements arithmetic: every
// number comes from the reference's MatMul / LayerNorm* / Gelu* /
// MultiHeadAttention / Embedding / GPTModel / CrossEntropyLoss / AdamW.
//
// Reference entry points wrapped (paths inside the NeuralSuite project):
//   MatMul                  src/tensor.cpp:198-271
//   LayerNormForward/Bwd    src/tensor.cpp:290-359
//   GeluForward/Backward    src/tensor.cpp:428-461
//   CausalSoftmaxForward    src/tensor.cpp:394-426
//   CrossEntropyLoss        include/losses.h:32-91
//   Embedding               include/layers/embedding.h:24-92
//   MultiHeadAttention      include/layers/attention.h:330-588
//   GPTModel                include/gpt.h:136-327
//   AdamW                   include/optimizers.h:143-253
//   SaveWeights/LoadWeights include/gpt.h:293-306 (NSF, include/serialization.h)
//   ForwardWithKVCache      include/gpt.h:153-190, include/layers/attention.h:481-546
//   Conv2D                  include/layers/conv2d.h:192-414
//   ResidualBlock           include/layers/residual.h:23-64
//   MSELoss                 include/losses.h:97-124
//   LSTM / BiLSTM           include/layers/lstm.h:320-664
//   ClipGradients           train_llm.cpp:112-129 (restated: it is a static
//                           function of the training program, not a library
//                           symbol)
//   parallel::ThreadCount   include/parallel.h:58-64

#include <chrono>
#include <cmath>
#include <cstring>
#include <exception>
#include <memory>
#include <string>
#include <vector>

#include "gpt.h"
#include "layers/conv2d.h"
#include "layers/layernorm.h"
#include "layers/lstm.h"
#include "layers/residual.h"
#include "losses.h"
#include "optimizers.h"
#include "parallel.h"
#include "tensor.h"

using namespace neuralsuite;

namespace {

thread_local std::string g_last_error;

template <typename Fn>
int Guard(Fn&& fn) {
  try {
    fn();
    return 0;
  } catch (const std::out_of_range& e) {
    g_last_error = std::string("out_of_range: ") + e.what();
    return 3;
  } catch (const std::invalid_argument& e) {
    g_last_error = std::string("invalid_argument: ") + e.what();
    return 2;
  } catch (const std::exception& e) {
    g_last_error = std::string("exception: ") + e.what();
    return 1;
  }
}

Tensor FromHost(const float* p, std::vector<int> shape) {
  Tensor t(shape);
  if (t.TotalSize() > 0) std::memcpy(t.Data(), p, t.TotalSize() * sizeof(float));
  return t;
}

void ToHost(const Tensor& t, float* p) {
  if (p != nullptr && t.TotalSize() > 0) std::memcpy(p, t.Data(), t.TotalSize() * sizeof(float));
}

struct GptHandle {
  GPTConfig cfg;
  std::unique_ptr<GPTModel> model;
  std::unique_ptr<AdamW> opt;
  CrossEntropyLoss criterion;
};

}  // namespace

extern "C" {

const char* nsref_last_error(void) { return g_last_error.c_str(); }

void nsref_set_threads(int n) { parallel::ThreadCount() = n > 0 ? n : 1; }
int nsref_threads(void) { return parallel::ThreadCount(); }

int nsref_matmul(const float* A, const float* B, float* C, int M, int K, int N) {
  return Guard([&] {
    Tensor a = FromHost(A, {M, K});
    Tensor b = FromHost(B, {K, N});
    Tensor c;
    MatMul(a, b, c);
    ToHost(c, C);
  });
}

int nsref_layernorm_fwd(const float* x, const float* gamma, const float* beta, float* out,
                        float* mean, float* rstd, int rows, int dim, float eps) {
  return Guard([&] {
    Tensor tx = FromHost(x, {rows, dim});
    Tensor g = FromHost(gamma, {dim});
    Tensor b = FromHost(beta, {dim});
    Tensor o, m, r;
    LayerNormForward(tx, g, b, o, m, r, eps);
    ToHost(o, out);
    ToHost(m, mean);
    ToHost(r, rstd);
  });
}

int nsref_layernorm_bwd(const float* dout, const float* x, const float* gamma, const float* mean,
                        const float* rstd, float* dx, float* dgamma, float* dbeta, int rows,
                        int dim) {
  return Guard([&] {
    Tensor td = FromHost(dout, {rows, dim});
    Tensor tx = FromHost(x, {rows, dim});
    Tensor g = FromHost(gamma, {dim});
    Tensor m = FromHost(mean, {rows});
    Tensor r = FromHost(rstd, {rows});
    Tensor o, dg, db;
    LayerNormBackward(td, tx, g, m, r, o, dg, db);
    ToHost(o, dx);
    ToHost(dg, dgamma);
    ToHost(db, dbeta);
  });
}

int nsref_gelu_fwd(const float* x, float* y, int n) {
  return Guard([&] {
    Tensor tx = FromHost(x, {n});
    Tensor ty;
    GeluForward(tx, ty);
    ToHost(ty, y);
  });
}

int nsref_gelu_bwd(const float* dout, const float* x, float* dx, int n) {
  return Guard([&] {
    Tensor td = FromHost(dout, {n});
    Tensor tx = FromHost(x, {n});
    Tensor o;
    GeluBackward(td, tx, o);
    ToHost(o, dx);
  });
}

int nsref_causal_softmax(const float* in, float* out, int batch, int T) {
  return Guard([&] {
    Tensor ti = FromHost(in, {batch, T, T});
    Tensor to;
    CausalSoftmaxForward(ti, to, T);
    ToHost(to, out);
  });
}

// CrossEntropyLoss::Forward then ::Backward on [rows, classes] logits.
int nsref_cross_entropy(const float* logits, const float* targets, int rows, int classes,
                        float* loss, float* dlogits) {
  return Guard([&] {
    Tensor tl = FromHost(logits, {rows, classes});
    Tensor tt = FromHost(targets, {rows});
    CrossEntropyLoss ce;
    *loss = ce.Forward(tl, tt);
    Tensor d = ce.Backward();
    ToHost(d, dlogits);
  });
}

// Embedding::Forward followed by Embedding::Backward with `dout`.
int nsref_embedding(const float* weight, int num, int dim, const float* idx, int batch, int T,
                    const float* dout, float* out, float* dweight) {
  return Guard([&] {
    Embedding emb(num, dim);
    std::memcpy(emb.Weight().Data(), weight, sizeof(float) * num * dim);
    Tensor ti = FromHost(idx, {batch, T});
    Tensor o = emb.Forward(ti);
    ToHost(o, out);
    if (dout != nullptr) {
      Tensor td = FromHost(dout, {batch, T, dim});
      emb.Backward(td);
      ToHost(emb.WeightParam().Grad(), dweight);
    }
  });
}

// MultiHeadAttention::Forward + ::Backward with the given projection weights.
// grads: c_attn.weight, c_attn.bias, c_proj.weight, c_proj.bias (registration order).
int nsref_mha(int B, int T, int C, int H, const float* w_attn, const float* b_attn,
              const float* w_proj, const float* b_proj, const float* x, const float* dout,
              float* y, float* dx, float* g_w_attn, float* g_b_attn, float* g_w_proj,
              float* g_b_proj) {
  return Guard([&] {
    MultiHeadAttention attn(C, H);
    std::vector<Tensor*> p = attn.GetParameters();
    std::memcpy(p[0]->Data(), w_attn, sizeof(float) * C * 3 * C);
    std::memcpy(p[1]->Data(), b_attn, sizeof(float) * 3 * C);
    std::memcpy(p[2]->Data(), w_proj, sizeof(float) * C * C);
    std::memcpy(p[3]->Data(), b_proj, sizeof(float) * C);
    Tensor tx = FromHost(x, {B, T, C});
    Tensor ty = attn.Forward(tx);
    ToHost(ty, y);
    Tensor td = FromHost(dout, {B, T, C});
    Tensor tdx = attn.Backward(td);
    ToHost(tdx, dx);
    std::vector<Tensor*> g = attn.GetGradients();
    ToHost(*g[0], g_w_attn);
    ToHost(*g[1], g_b_attn);
    ToHost(*g[2], g_w_proj);
    ToHost(*g[3], g_b_proj);
  });
}

// Conv2D::Forward + ::Backward (include/layers/conv2d.h:192-414) with the
// given weights: y [B, OC, OH, OW], dx, dweight, dbias.
int nsref_conv2d(int B, int IC, int H, int W, int OC, int k, int stride, int pad,
                 const float* weight, const float* bias, const float* x, const float* dout,
                 float* y, float* dx, float* dweight, float* dbias) {
  return Guard([&] {
    Conv2D conv(IC, OC, k, stride, pad);
    std::memcpy(conv.Weight().Data(), weight, sizeof(float) * OC * IC * k * k);
    std::memcpy(conv.Bias().Data(), bias, sizeof(float) * OC);
    Tensor tx = FromHost(x, {B, IC, H, W});
    Tensor ty = conv.Forward(tx);
    ToHost(ty, y);
    if (dout != nullptr) {
      Tensor td = FromHost(dout, ty.Shape());
      Tensor tdx = conv.Backward(td);
      ToHost(tdx, dx);
      std::vector<Tensor*> g = conv.GetGradients();
      ToHost(*g[0], dweight);
      ToHost(*g[1], dbias);
    }
  });
}

// LSTM (bidir = 0) or BiLSTM (bidir = 1) Forward + Backward
// (include/layers/lstm.h:320-664) with the flat parameters in registration
// order (weight_ih, weight_hh, bias_ih, bias_hh; BiLSTM: forward's then
// reverse's); grads likewise.
int nsref_lstm(int T, int B, int IN, int H, int bidir, const float* params, const float* x,
               const float* dout, float* out, float* dx, float* grads) {
  return Guard([&] {
    std::unique_ptr<Layer> layer;
    if (bidir) layer = std::make_unique<BiLSTM>(IN, H);
    else layer = std::make_unique<LSTM>(IN, H);
    size_t off = 0;
    for (Tensor* t : layer->GetParameters()) {
      std::memcpy(t->Data(), params + off, t->TotalSize() * sizeof(float));
      off += t->TotalSize();
    }
    Tensor tx = FromHost(x, {T, B, IN});
    Tensor ty = layer->Forward(tx);
    ToHost(ty, out);
    Tensor td = FromHost(dout, ty.Shape());
    ToHost(layer->Backward(td), dx);
    off = 0;
    for (Tensor* t : layer->GetGradients()) {
      std::memcpy(grads + off, t->Data(), t->TotalSize() * sizeof(float));
      off += t->TotalSize();
    }
  });
}

// ------------------------------------------------------ diffusion U-Net
//
// The U-Net of the diffusion training step (the reference has none): two
// stride-2 levels down and two nearest-neighbour levels up with skip sums,
// each level Conv2D -> ResidualBlock(Conv2D 3x3) -> LayerNormLayer (last
// axis, as the reference's LayerNorm normalises), a 3x3 head and MSELoss.
// Every layer is the reference's own class (include/layers/conv2d.h,
// residual.h, layernorm.h, include/losses.h:97-124); only the nearest
// upsample, which the reference lacks, is written here (UpNearest2x).
namespace {

// y[b][c][i][j] = x[b][c][i/2][j/2]; backward sums each 2x2 block in
// (0,0), (0,1), (1,0), (1,1) order.
Tensor UpNearest2x(const Tensor& x) {
  const int B = x.Shape()[0], C = x.Shape()[1], H = x.Shape()[2], W = x.Shape()[3];
  Tensor y({B, C, 2 * H, 2 * W});
  for (int bc = 0; bc < B * C; ++bc)
    for (int i = 0; i < 2 * H; ++i)
      for (int j = 0; j < 2 * W; ++j)
        y[((size_t)bc * 2 * H + i) * 2 * W + j] = x[((size_t)bc * H + i / 2) * W + j / 2];
  return y;
}
Tensor UpNearest2xBackward(const Tensor& dy) {
  const int B = dy.Shape()[0], C = dy.Shape()[1], H = dy.Shape()[2] / 2, W = dy.Shape()[3] / 2;
  Tensor dx({B, C, H, W});
  for (int bc = 0; bc < B * C; ++bc)
    for (int i = 0; i < H; ++i)
      for (int j = 0; j < W; ++j) {
        const size_t r0 = ((size_t)bc * 2 * H + 2 * i) * 2 * W + 2 * j, r1 = r0 + 2 * W;
        float s = 0.0f;
        s += dy[r0];
        s += dy[r0 + 1];
        s += dy[r1];
        s += dy[r1 + 1];
        dx[((size_t)bc * H + i) * W + j] = s;
      }
  return dx;
}
Tensor Add(const Tensor& a, const Tensor& b) {
  Tensor out(a.Shape());
  ElementwiseAdd(a, b, out);
  return out;
}

struct UNet {
  int C0, HW;
  std::shared_ptr<Conv2D> conv_in, down1, down2, up1, up0, conv_out;
  std::shared_ptr<ResidualBlock> res[5];
  std::shared_ptr<LayerNormLayer> ln[5];
  std::vector<Parameter*> params;
  MSELoss mse;
  std::unique_ptr<AdamW> opt;
  Tensor e0, e1;

  UNet(int in_ch, int base, int hw) : C0(base), HW(hw) {
    const int c[3] = {base, 2 * base, 4 * base};
    const int w[3] = {hw, hw / 2, hw / 4};
    conv_in = std::make_shared<Conv2D>(in_ch, c[0], 3, 1, 1);
    down1 = std::make_shared<Conv2D>(c[0], c[1], 3, 2, 1);
    down2 = std::make_shared<Conv2D>(c[1], c[2], 3, 2, 1);
    up1 = std::make_shared<Conv2D>(c[2], c[1], 3, 1, 1);
    up0 = std::make_shared<Conv2D>(c[1], c[0], 3, 1, 1);
    conv_out = std::make_shared<Conv2D>(c[0], in_ch, 3, 1, 1);
    const int rc[5] = {c[0], c[1], c[2], c[1], c[0]};
    const int rw[5] = {w[0], w[1], w[2], w[1], w[0]};
    for (int i = 0; i < 5; ++i) {
      res[i] = std::make_shared<ResidualBlock>(std::make_shared<Conv2D>(rc[i], rc[i], 3, 1, 1));
      ln[i] = std::make_shared<LayerNormLayer>(rw[i]);
    }
    // Registration order: conv_in, res0, ln0, down1, res1, ln1, down2, res2,
    // ln2, up1, res3, ln3, up0, res4, ln4, conv_out.
    auto add = [&](Layer* l) {
      for (Parameter* p : l->Parameters()) params.push_back(p);
    };
    add(conv_in.get()); add(res[0].get()); add(ln[0].get());
    add(down1.get()); add(res[1].get()); add(ln[1].get());
    add(down2.get()); add(res[2].get()); add(ln[2].get());
    add(up1.get()); add(res[3].get()); add(ln[3].get());
    add(up0.get()); add(res[4].get()); add(ln[4].get());
    add(conv_out.get());
  }

  Tensor Forward(const Tensor& x) {
    e0 = ln[0]->Forward(res[0]->Forward(conv_in->Forward(x)));
    e1 = ln[1]->Forward(res[1]->Forward(down1->Forward(e0)));
    Tensor m = ln[2]->Forward(res[2]->Forward(down2->Forward(e1)));
    Tensor u1 = ln[3]->Forward(res[3]->Forward(Add(up1->Forward(UpNearest2x(m)), e1)));
    Tensor u0 = ln[4]->Forward(res[4]->Forward(Add(up0->Forward(UpNearest2x(u1)), e0)));
    return conv_out->Forward(u0);
  }

  void Backward(const Tensor& dout) {
    Tensor du0 = conv_out->Backward(dout);
    Tensor ds0 = res[4]->Backward(ln[4]->Backward(du0));           // d(up0 out + e0)
    Tensor du1 = UpNearest2xBackward(up0->Backward(ds0));
    Tensor ds1 = res[3]->Backward(ln[3]->Backward(du1));           // d(up1 out + e1)
    Tensor dm = UpNearest2xBackward(up1->Backward(ds1));
    Tensor de1 = Add(down2->Backward(res[2]->Backward(ln[2]->Backward(dm))), ds1);
    Tensor de0 = Add(down1->Backward(res[1]->Backward(ln[1]->Backward(de1))), ds0);
    conv_in->Backward(res[0]->Backward(ln[0]->Backward(de0)));
  }
};

}  // namespace

void* nsref_unet_create(int in_ch, int base, int hw) {
  UNet* u = nullptr;
  Guard([&] { u = new UNet(in_ch, base, hw); });
  return u;
}
void nsref_unet_destroy(void* h) { delete static_cast<UNet*>(h); }
int nsref_unet_num_tensors(void* h) { return (int)static_cast<UNet*>(h)->params.size(); }
long long nsref_unet_tensor_numel(void* h, int i) {
  return (long long)static_cast<UNet*>(h)->params[i]->Value().TotalSize();
}
void nsref_unet_set_params(void* h, const float* flat) {
  size_t off = 0;
  for (Parameter* p : static_cast<UNet*>(h)->params) {
    std::memcpy(p->Value().Data(), flat + off, p->Value().TotalSize() * sizeof(float));
    off += p->Value().TotalSize();
  }
}
void nsref_unet_get(void* h, int grads, float* flat) {
  size_t off = 0;
  for (Parameter* p : static_cast<UNet*>(h)->params) {
    const Tensor& t = grads ? p->Grad() : p->Value();
    std::memcpy(flat + off, t.Data(), t.TotalSize() * sizeof(float));
    off += t.TotalSize();
  }
}
// Forward -> MSELoss -> Backward on x, target [B, in_ch, hw, hw]; out = the
// prediction.
int nsref_unet_fwd_bwd(void* h, int B, const float* x, const float* target, float* loss,
                       float* out) {
  UNet* u = static_cast<UNet*>(h);
  return Guard([&] {
    const int ic = u->conv_in->Weight().Shape()[1];
    Tensor tx = FromHost(x, {B, ic, u->HW, u->HW});
    Tensor tt = FromHost(target, {B, ic, u->HW, u->HW});
    Tensor y = u->Forward(tx);
    ToHost(y, out);
    *loss = u->mse.Forward(y, tt);
    u->Backward(u->mse.Backward());
  });
}
int nsref_unet_adamw_init(void* h, float lr) {
  UNet* u = static_cast<UNet*>(h);
  return Guard([&] { u->opt = std::make_unique<AdamW>(u->params, lr); });
}
int nsref_unet_adamw_step(void* h) {
  return Guard([&] { static_cast<UNet*>(h)->opt->Step(); });
}

// ---------------------------------------------------------------- GPT model

void* nsref_gpt_create(int vocab, int block, int n_layer, int n_head, int n_embd) {
  GptHandle* h = nullptr;
  int rc = Guard([&] {
    auto owned = std::make_unique<GptHandle>();
    owned->cfg.vocab_size = vocab;
    owned->cfg.block_size = block;
    owned->cfg.n_layer = n_layer;
    owned->cfg.n_head = n_head;
    owned->cfg.n_embd = n_embd;
    owned->model = std::make_unique<GPTModel>(owned->cfg);
    h = owned.release();
  });
  return rc == 0 ? h : nullptr;
}

void nsref_gpt_destroy(void* handle) { delete static_cast<GptHandle*>(handle); }

int nsref_gpt_num_tensors(void* handle) {
  return static_cast<int>(static_cast<GptHandle*>(handle)->model->Parameters().size());
}

long long nsref_gpt_tensor_numel(void* handle, int i) {
  return static_cast<long long>(
      static_cast<GptHandle*>(handle)->model->Parameters()[i]->TotalSize());
}

int nsref_gpt_tensor_rank(void* handle, int i) {
  return static_cast<int>(static_cast<GptHandle*>(handle)->model->Parameters()[i]->Shape().size());
}

// Copies the registration-order parameter list into / out of one flat buffer.
void nsref_gpt_set_params(void* handle, const float* flat) {
  size_t off = 0;
  for (Tensor* t : static_cast<GptHandle*>(handle)->model->GetParameters()) {
    std::memcpy(t->Data(), flat + off, t->TotalSize() * sizeof(float));
    off += t->TotalSize();
  }
}

void nsref_gpt_get_params(void* handle, float* flat) {
  size_t off = 0;
  for (Tensor* t : static_cast<GptHandle*>(handle)->model->GetParameters()) {
    std::memcpy(flat + off, t->Data(), t->TotalSize() * sizeof(float));
    off += t->TotalSize();
  }
}

void nsref_gpt_get_grads(void* handle, float* flat) {
  size_t off = 0;
  for (Tensor* t : static_cast<GptHandle*>(handle)->model->GetGradients()) {
    std::memcpy(flat + off, t->Data(), t->TotalSize() * sizeof(float));
    off += t->TotalSize();
  }
}

// One Forward -> CrossEntropy -> Backward, the sequence of
// tools/parity/parity_gpt.cpp:86-97 and train_llm.cpp:216-226.
int nsref_gpt_fwd_bwd(void* handle, const float* idx, const float* targets, int B, int T,
                      float* loss, float* logits_out) {
  GptHandle* h = static_cast<GptHandle*>(handle);
  return Guard([&] {
    const int V = h->cfg.vocab_size;
    Tensor ti = FromHost(idx, {B, T});
    Tensor tt = FromHost(targets, {B * T});
    Tensor logits = h->model->Forward(ti);
    ToHost(logits, logits_out);
    Tensor logits_2d({B * T, V});
    std::memcpy(logits_2d.Data(), logits.Data(), logits.TotalSize() * sizeof(float));
    *loss = h->criterion.Forward(logits_2d, tt);
    Tensor d2 = h->criterion.Backward();
    Tensor dlogits({B, T, V});
    std::memcpy(dlogits.Data(), d2.Data(), d2.TotalSize() * sizeof(float));
    h->model->Backward(dlogits);
  });
}

// Global-norm clip with the serial float sum of train_llm.cpp:112-129.
float nsref_gpt_clip_gradients(void* handle, float max_norm) {
  GptHandle* h = static_cast<GptHandle*>(handle);
  float total = 0.0f;
  for (Parameter* p : h->model->Parameters()) {
    const Tensor& g = p->Grad();
    for (size_t i = 0; i < g.TotalSize(); ++i) total += g[i] * g[i];
  }
  const float norm = std::sqrt(total);
  if (norm > max_norm && norm > 0.0f) {
    const float scale = max_norm / norm;
    for (Parameter* p : h->model->Parameters()) {
      Tensor& g = p->Grad();
      for (size_t i = 0; i < g.TotalSize(); ++i) g[i] *= scale;
    }
  }
  return norm;
}

int nsref_gpt_adamw_init(void* handle, float lr, float b1, float b2, float eps, float wd) {
  GptHandle* h = static_cast<GptHandle*>(handle);
  return Guard([&] {
    h->opt = std::make_unique<AdamW>(h->model->Parameters(), lr, b1, b2, eps, wd);
  });
}

void nsref_gpt_adamw_set_lr(void* handle, float lr) {
  static_cast<GptHandle*>(handle)->opt->SetLearningRate(lr);
}

int nsref_gpt_adamw_step(void* handle) {
  GptHandle* h = static_cast<GptHandle*>(handle);
  return Guard([&] { h->opt->Step(); });
}

// GPTModel::SaveWeights / LoadWeights (include/gpt.h:293-306): the NSF file
// of include/serialization.h.  1 on success, 0 on failure (the reference
// returns bool and prints the reason).
int nsref_gpt_save_weights(void* handle, const char* path) {
  return static_cast<GptHandle*>(handle)->model->SaveWeights(path) ? 1 : 0;
}

int nsref_gpt_load_weights(void* handle, const char* path) {
  return static_cast<GptHandle*>(handle)->model->LoadWeights(path) ? 1 : 0;
}

// GPTModel::ForwardWithKVCache(token, pos) (include/gpt.h:159-190): one
// token through the cached model; logits_out receives vocab floats.
int nsref_gpt_decode(void* handle, int token, int pos, float* logits_out) {
  GptHandle* h = static_cast<GptHandle*>(handle);
  return Guard([&] { ToHost(h->model->ForwardWithKVCache(token, pos), logits_out); });
}

// GPTModel::ClearKVCache (include/gpt.h:153-157).
void nsref_gpt_clear_kv(void* handle) { static_cast<GptHandle*>(handle)->model->ClearKVCache(); }

int nsref_gpt_zero_grad(void* handle) {
  GptHandle* h = static_cast<GptHandle*>(handle);
  return Guard([&] { h->model->ZeroGrad(); });
}

}  // extern "C"
