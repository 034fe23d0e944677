// Model-level C ABI: the device GPTModel + CrossEntropyLoss + AdamW of
// gpt_device.h behind ns_gpt_*, plus the data-parallel gradient all-reduce.
//
// Data parallel: each process owns one GPU and a full replica.  The backward
// hands every bucket group to a second stream as soon as its gradients are
// final (an event recorded after the group's last kernel), and NCCL sums it
// there while the backward of the earlier blocks continues; the compute
// stream joins the comm stream before the optimizer.  Because the
// cross-entropy gradient is divided by rows * world_size, the sum over ranks
// is the gradient of the global-batch mean loss.
#include <cstdio>
#include <cstring>
#include <exception>
#include <map>
#include <string>
#include <memory>
#include <vector>

#include "comm.h"
#include "common.cuh"
#include "gpt_device.h"
#include "gemm_tc.cuh"
#include "gpt_handle.h"
#include "nsf.h"

using neuralsuite::cuda::AdamW;
using neuralsuite::cuda::Bucket;
using neuralsuite::cuda::GPTConfig;
using neuralsuite::cuda::GPTModel;


namespace {

template <typename Fn>
ns_status Guard(Fn&& fn) {
  try {
    return fn();
  } catch (const std::out_of_range& e) {
    return nsb::fail(NS_ERR_OUT_OF_RANGE, e.what());
  } catch (const std::invalid_argument& e) {
    return nsb::fail(NS_ERR_INVALID_ARGUMENT, e.what());
  } catch (const std::exception& e) {
    return nsb::fail(NS_ERR_CUDA, e.what());
  }
}

GPTConfig ToConfig(const ns_gpt_config* c) {
  GPTConfig g;
  g.vocab_size = c->vocab_size;
  g.block_size = c->block_size;
  g.n_layer = c->n_layer;
  g.n_head = c->n_head;
  g.n_embd = c->n_embd;
  return g;
}

void release_comm_resources(ns_gpt* h) {
  for (cudaEvent_t e : h->group_ready) cudaEventDestroy(e);
  h->group_ready.clear();
  if (h->comm_done) cudaEventDestroy(h->comm_done);
  h->comm_done = nullptr;
  for (cudaEvent_t* e : {&h->t_bwd_end, &h->t_comm_begin, &h->t_comm_end}) {
    if (*e) cudaEventDestroy(*e);
    *e = nullptr;
  }
  h->comm_timed = false;
  if (h->comm_stream) cudaStreamDestroy(h->comm_stream);
  h->comm_stream = nullptr;
}

ns_status backward_impl(ns_gpt* h, cudaStream_t s) {
  GPTModel& m = *h->model;
  m.SetStream(s);
  if (!h->comm || h->world == 1) {
    m.Backward();
    return NS_OK;
  }
  ns_status rc = NS_OK;
  const bool timing = h->comm_timing && h->t_bwd_end;
  m.Backward([&](int g) {
    if (rc != NS_OK) return;
    cudaEvent_t ev = h->group_ready[g];
    if (cudaEventRecord(ev, s) != cudaSuccess || cudaStreamWaitEvent(h->comm_stream, ev, 0) != cudaSuccess) {
      rc = nsb::fail(NS_ERR_CUDA, "bucket event");
      return;
    }
    if (timing && g == 0 && cudaEventRecord(h->t_comm_begin, h->comm_stream) != cudaSuccess) {
      rc = nsb::fail(NS_ERR_CUDA, "timing event");
      return;
    }
    for (const Bucket& b : h->buckets) {
      if (b.group != g) continue;
      rc = nsb::comm::allreduce(h->comm, m.Grads() + b.begin, b.end - b.begin, h->comm_stream);
      if (rc != NS_OK) return;
    }
  });
  if (rc != NS_OK) return rc;
  // The per-rank mean losses are summed too; the host divides by world.
  rc = nsb::comm::allreduce(h->comm, m.Small(), 1, h->comm_stream);
  if (rc != NS_OK) return rc;
  NS_TRY_CUDA(cudaEventRecord(h->comm_done, h->comm_stream), "comm join");
  if (timing) {
    NS_TRY_CUDA(cudaEventRecord(h->t_comm_end, h->comm_stream), "timing event");
    NS_TRY_CUDA(cudaEventRecord(h->t_bwd_end, s), "timing event");
    h->comm_timed = true;
  }
  NS_TRY_CUDA(cudaStreamWaitEvent(s, h->comm_done, 0), "comm join");
  return NS_OK;
}

// ------------------------------------------------------------ checkpoints
//
// Names and shapes of GPTModel::NamedParameters() in registration order
// (include/module.h:62-73 over the Register calls of include/gpt.h:59-63,
// 143-149 and the layers'), and the architecture metadata of
// GPTModel::ArchitectureMetadata() (include/gpt.h:309-316).
std::vector<nsb::nsf::Entry> gpt_entries(const ns_gpt_config& c) {
  const int V = c.vocab_size, B = c.block_size, C = c.n_embd;
  std::vector<nsb::nsf::Entry> e;
  auto add = [&](const std::string& name, std::vector<int> dims) { e.push_back({name, dims}); };
  add("wte.weight", {V, C});
  add("wpe.weight", {B, C});
  for (int i = 0; i < c.n_layer; ++i) {
    const std::string p = "blocks." + std::to_string(i) + ".";
    add(p + "ln_1.gamma", {C});
    add(p + "ln_1.beta", {C});
    add(p + "attn.c_attn.weight", {C, 3 * C});
    add(p + "attn.c_attn.bias", {3 * C});
    add(p + "attn.c_proj.weight", {C, C});
    add(p + "attn.c_proj.bias", {C});
    add(p + "ln_2.gamma", {C});
    add(p + "ln_2.beta", {C});
    add(p + "mlp_fc.weight", {C, 4 * C});
    add(p + "mlp_fc.bias", {4 * C});
    add(p + "mlp_proj.weight", {4 * C, C});
    add(p + "mlp_proj.bias", {C});
  }
  add("ln_f.gamma", {C});
  add("ln_f.beta", {C});
  return e;
}

std::map<std::string, std::string> gpt_meta(const ns_gpt_config& c) {
  return {{"arch", "gpt"},
          {"vocab_size", std::to_string(c.vocab_size)},
          {"block_size", std::to_string(c.block_size)},
          {"n_layer", std::to_string(c.n_layer)},
          {"n_head", std::to_string(c.n_head)},
          {"n_embd", std::to_string(c.n_embd)}};
}

ns_gpt_config config_of(const ns_gpt* h) {
  const GPTConfig& g = h->model->Config();
  return ns_gpt_config{g.vocab_size, g.block_size, g.n_layer, g.n_head, g.n_embd, 1};
}

// Points entries at consecutive slices of `base` (the flat registration-order
// buffer); false if the table does not cover exactly n floats.
bool bind_flat(std::vector<nsb::nsf::Entry>& e, float* base, int64_t n) {
  int64_t off = 0;
  for (auto& x : e) {
    x.data = base + off;
    x.out = base + off;
    off += (int64_t)x.numel();
  }
  return off == n;
}

std::string fmt_float(float v) {
  char b[32];
  std::snprintf(b, sizeof(b), "%.9g", (double)v);
  return b;
}

}  // namespace

extern "C" {

ns_status ns_nsf_save_gpt(const ns_gpt_config* cfg, const float* host_params, const char* path) {
  NS_REQUIRE(cfg && host_params && path, "ns_nsf_save_gpt: NULL argument");
  auto e = gpt_entries(*cfg);
  int64_t n = 0;
  for (auto& x : e) n += (int64_t)x.numel();
  bind_flat(e, const_cast<float*>(host_params), n);
  const std::string err = nsb::nsf::Write(path, gpt_meta(*cfg), e);
  if (!err.empty()) return nsb::fail(NS_ERR_INVALID_ARGUMENT, "ns_nsf_save_gpt: " + err);
  return NS_OK;
}

ns_status ns_nsf_load_gpt(const ns_gpt_config* cfg, const char* path, float* host_params) {
  NS_REQUIRE(cfg && host_params && path, "ns_nsf_load_gpt: NULL argument");
  auto e = gpt_entries(*cfg);
  int64_t n = 0;
  for (auto& x : e) n += (int64_t)x.numel();
  // Read into a private buffer: the caller's array changes only on success.
  std::vector<float> tmp((size_t)n);
  bind_flat(e, tmp.data(), n);
  const std::string err = nsb::nsf::Read(path, gpt_meta(*cfg), e);
  if (!err.empty()) return nsb::fail(NS_ERR_INVALID_ARGUMENT, "ns_nsf_load_gpt: " + err);
  std::memcpy(host_params, tmp.data(), tmp.size() * sizeof(float));
  return NS_OK;
}

ns_status ns_gpt_save_weights(ns_gpt* h, const char* path, void* stream) {
  NS_REQUIRE(h && path, "ns_gpt_save_weights: NULL argument");
  return Guard([&]() -> ns_status {
    GPTModel& m = *h->model;
    std::vector<float> host((size_t)m.NumParams());
    cudaStream_t s = nsb::as_stream(stream);
    NS_TRY_CUDA(cudaMemcpyAsync(host.data(), m.Values(), host.size() * sizeof(float),
                                cudaMemcpyDeviceToHost, s),
                "ns_gpt_save_weights copy");
    NS_TRY_CUDA(cudaStreamSynchronize(s), "ns_gpt_save_weights sync");
    const ns_gpt_config c = config_of(h);
    return ns_nsf_save_gpt(&c, host.data(), path);
  });
}

ns_status ns_gpt_load_weights(ns_gpt* h, const char* path, void* stream) {
  NS_REQUIRE(h && path, "ns_gpt_load_weights: NULL argument");
  return Guard([&]() -> ns_status {
    GPTModel& m = *h->model;
    std::vector<float> host((size_t)m.NumParams());
    const ns_gpt_config c = config_of(h);
    ns_status rc = ns_nsf_load_gpt(&c, path, host.data());
    if (rc != NS_OK) return rc;  // the device parameters are untouched
    cudaStream_t s = nsb::as_stream(stream);
    NS_TRY_CUDA(cudaMemcpyAsync(m.Values(), host.data(), host.size() * sizeof(float),
                                cudaMemcpyHostToDevice, s),
                "ns_gpt_load_weights copy");
    NS_TRY_CUDA(cudaStreamSynchronize(s), "ns_gpt_load_weights sync");
    return NS_OK;
  });
}

ns_status ns_gpt_save_optimizer(ns_gpt* h, const char* path, void* stream) {
  NS_REQUIRE(h && path, "ns_gpt_save_optimizer: NULL argument");
  NS_REQUIRE(h->opt, "ns_gpt_save_optimizer: optimizer not initialised");
  return Guard([&]() -> ns_status {
    GPTModel& m = *h->model;
    const size_t n = (size_t)m.NumParams();
    std::vector<float> host(2 * n);
    float hyper[7];
    cudaStream_t s = nsb::as_stream(stream);
    NS_TRY_CUDA(cudaMemcpyAsync(host.data(), h->opt->M(), n * 4, cudaMemcpyDeviceToHost, s), "copy");
    NS_TRY_CUDA(cudaMemcpyAsync(host.data() + n, h->opt->V(), n * 4, cudaMemcpyDeviceToHost, s), "copy");
    NS_TRY_CUDA(cudaMemcpyAsync(hyper, h->opt->Hyper(), sizeof(hyper), cudaMemcpyDeviceToHost, s), "copy");
    NS_TRY_CUDA(cudaStreamSynchronize(s), "ns_gpt_save_optimizer sync");
    const ns_gpt_config c = config_of(h);
    auto pm = gpt_entries(c), pv = gpt_entries(c);
    bind_flat(pm, host.data(), (int64_t)n);
    bind_flat(pv, host.data() + n, (int64_t)n);
    std::vector<nsb::nsf::Entry> e;
    for (auto& x : pm) e.push_back({"m." + x.name, x.dims, x.data, x.out});
    for (auto& x : pv) e.push_back({"v." + x.name, x.dims, x.data, x.out});
    int32_t step = 0;
    std::memcpy(&step, &hyper[6], 4);
    auto meta = gpt_meta(c);
    meta["arch"] = "gpt-adamw";
    meta["step"] = std::to_string(step);
    meta["lr"] = fmt_float(hyper[0]);
    meta["beta1"] = fmt_float(hyper[1]);
    meta["beta2"] = fmt_float(hyper[2]);
    meta["eps"] = fmt_float(hyper[3]);
    meta["weight_decay"] = fmt_float(h->opt->WeightDecay());
    const std::string err = nsb::nsf::Write(path, meta, e);
    if (!err.empty()) return nsb::fail(NS_ERR_INVALID_ARGUMENT, "ns_gpt_save_optimizer: " + err);
    return NS_OK;
  });
}

ns_status ns_gpt_load_optimizer(ns_gpt* h, const char* path, void* stream) {
  NS_REQUIRE(h && path, "ns_gpt_load_optimizer: NULL argument");
  NS_REQUIRE(h->opt, "ns_gpt_load_optimizer: call ns_gpt_adamw_init first");
  return Guard([&]() -> ns_status {
    GPTModel& m = *h->model;
    const size_t n = (size_t)m.NumParams();
    std::vector<float> host(2 * n);
    const ns_gpt_config c = config_of(h);
    auto pm = gpt_entries(c), pv = gpt_entries(c);
    bind_flat(pm, host.data(), (int64_t)n);
    bind_flat(pv, host.data() + n, (int64_t)n);
    std::vector<nsb::nsf::Entry> e;
    for (auto& x : pm) e.push_back({"m." + x.name, x.dims, x.data, x.out});
    for (auto& x : pv) e.push_back({"v." + x.name, x.dims, x.data, x.out});
    auto expect = gpt_meta(c);
    expect["arch"] = "gpt-adamw";
    expect["weight_decay"] = fmt_float(h->opt->WeightDecay());
    std::map<std::string, std::string> meta;
    const std::string err = nsb::nsf::Read(path, expect, e, &meta);
    if (!err.empty()) return nsb::fail(NS_ERR_INVALID_ARGUMENT, "ns_gpt_load_optimizer: " + err);
    float hyper[7];
    try {
      hyper[0] = std::stof(meta.at("lr"));
      hyper[1] = std::stof(meta.at("beta1"));
      hyper[2] = std::stof(meta.at("beta2"));
      hyper[3] = std::stof(meta.at("eps"));
      hyper[4] = hyper[5] = 1.0f;  // bias corrections: recomputed by the next step
      const int32_t step = (int32_t)std::stol(meta.at("step"));
      std::memcpy(&hyper[6], &step, 4);
    } catch (const std::exception&) {
      return nsb::fail(NS_ERR_INVALID_ARGUMENT,
                       "ns_gpt_load_optimizer: missing or malformed step / lr / beta / eps");
    }
    cudaStream_t s = nsb::as_stream(stream);
    NS_TRY_CUDA(cudaMemcpyAsync(h->opt->M(), host.data(), n * 4, cudaMemcpyHostToDevice, s), "copy");
    NS_TRY_CUDA(cudaMemcpyAsync(h->opt->V(), host.data() + n, n * 4, cudaMemcpyHostToDevice, s), "copy");
    NS_TRY_CUDA(cudaMemcpyAsync(h->opt->Hyper(), hyper, sizeof(hyper), cudaMemcpyHostToDevice, s), "copy");
    NS_TRY_CUDA(cudaStreamSynchronize(s), "ns_gpt_load_optimizer sync");
    return NS_OK;
  });
}

ns_status ns_gpt_create(const ns_gpt_config* cfg, ns_gpt** out) {
  NS_REQUIRE(cfg && out, "ns_gpt_create: NULL argument");
  return Guard([&]() -> ns_status {
    auto h = std::make_unique<ns_gpt>();
    h->model = std::make_unique<GPTModel>(ToConfig(cfg), cfg->max_batch);
    NS_TRY_CUDA(cudaMallocHost(reinterpret_cast<void**>(&h->host_small), 16 * sizeof(float)),
                "cudaMallocHost");
    NS_TRY_CUDA(cudaEventCreateWithFlags(&h->step_done, cudaEventDisableTiming), "event");
    *out = h.release();
    return NS_OK;
  });
}

ns_status ns_gpt_destroy(ns_gpt* h) {
  if (!h) return NS_OK;
  cudaDeviceSynchronize();
  release_comm_resources(h);
  if (h->step_done) cudaEventDestroy(h->step_done);
  if (h->host_small) cudaFreeHost(h->host_small);
  delete h;
  return NS_OK;
}

int ns_gpt_num_tensors(const ns_gpt* h) { return h ? (int)h->model->Ranks().size() : 0; }
// Getters: 0 / NULL for a NULL handle or a tensor index out of range.
static bool valid_tensor(const ns_gpt* h, int i) {
  return h && i >= 0 && i < (int)h->model->Ranks().size();
}
int64_t ns_gpt_tensor_numel(const ns_gpt* h, int i) {
  return valid_tensor(h, i) ? h->model->Offsets()[i + 1] - h->model->Offsets()[i] : 0;
}
int ns_gpt_tensor_rank(const ns_gpt* h, int i) { return valid_tensor(h, i) ? h->model->Ranks()[i] : 0; }
int64_t ns_gpt_tensor_offset(const ns_gpt* h, int i) {
  return valid_tensor(h, i) ? h->model->Offsets()[i] : 0;
}
int64_t ns_gpt_num_params(const ns_gpt* h) { return h ? h->model->NumParams() : 0; }
float* ns_gpt_params(ns_gpt* h) { return h ? h->model->Values() : nullptr; }
float* ns_gpt_grads(ns_gpt* h) { return h ? h->model->Grads() : nullptr; }
float* ns_gpt_logits(ns_gpt* h) { return h ? h->model->Logits().Data() : nullptr; }
float* ns_gpt_loss(ns_gpt* h) { return h ? h->model->Small() : nullptr; }

ns_status ns_gpt_forward(ns_gpt* h, const int32_t* tokens, int B, int T, void* stream) {
  NS_REQUIRE(h, "ns_gpt_forward: NULL model");
  return Guard([&]() -> ns_status {
    h->model->SetStream(nsb::as_stream(stream));
    h->model->Forward(tokens, B, T);
    h->B = B;
    h->T = T;
    return NS_OK;
  });
}

ns_status ns_gpt_loss_backward(ns_gpt* h, const int32_t* targets, void* stream) {
  NS_REQUIRE(h, "ns_gpt_loss_backward: NULL model");
  return Guard([&]() -> ns_status {
    NS_REQUIRE(h->B > 0, "ns_gpt_loss_backward: no forward pass yet");
    h->model->SetStream(nsb::as_stream(stream));
    h->model->LossBackward(targets, (float)((double)h->B * h->T * h->world));
    return NS_OK;
  });
}

ns_status ns_gpt_backward(ns_gpt* h, void* stream) {
  NS_REQUIRE(h, "ns_gpt_backward: NULL model");
  // The all-reduce of earlier buckets runs beside these GEMMs: dynamic order.
  const nsb::tc::PairScheduleScope sched(h->comm && h->world > 1);
  return Guard([&]() -> ns_status { return backward_impl(h, nsb::as_stream(stream)); });
}

ns_status ns_gpt_adamw_init(ns_gpt* h, float lr, float b1, float b2, float eps, float wd) {
  NS_REQUIRE(h, "ns_gpt_adamw_init: NULL model");
  return Guard([&]() -> ns_status {
    h->opt = std::make_unique<AdamW>(*h->model, lr, b1, b2, eps, wd);
    return NS_OK;
  });
}

ns_status ns_gpt_adamw_set_lr(ns_gpt* h, float lr) {
  NS_REQUIRE(h, "ns_gpt_adamw_set_lr: NULL model");
  NS_REQUIRE(h->opt, "ns_gpt_adamw_set_lr: optimizer not initialised");
  return Guard([&]() -> ns_status {
    h->opt->SetLearningRate(lr);
    return NS_OK;
  });
}

ns_status ns_gpt_adamw_step(ns_gpt* h, void* stream) {
  NS_REQUIRE(h, "ns_gpt_adamw_step: NULL model");
  NS_REQUIRE(h->opt, "ns_gpt_adamw_step: optimizer not initialised");
  return Guard([&]() -> ns_status {
    h->model->SetStream(nsb::as_stream(stream));
    h->opt->Step();
    return NS_OK;
  });
}

ns_status ns_gpt_clip_gradients(ns_gpt* h, float max_norm, void* stream) {
  NS_REQUIRE(h, "ns_gpt_clip_gradients: NULL model");
  GPTModel& m = *h->model;
  cudaStream_t s = nsb::as_stream(stream);
  float* sumsq = m.Small() + 3;
  ns_status rc = ns_sumsq(m.Grads(), m.NumParams(), sumsq, m.Ctx().scratch, m.Ctx().scratch_bytes, s);
  if (rc != NS_OK) return rc;
  return ns_clip_scale(m.Grads(), m.NumParams(), sumsq, max_norm, s);
}

ns_status ns_gpt_train_step(ns_gpt* h, const int32_t* tokens, const int32_t* targets, int B, int T,
                            float max_norm, float* host_loss, void* stream) {
  NS_REQUIRE(h, "ns_gpt_train_step: NULL model");
  NS_REQUIRE(h->opt, "ns_gpt_train_step: call ns_gpt_adamw_init first");
  cudaStream_t s = nsb::as_stream(stream);
  ns_status rc = ns_gpt_forward(h, tokens, B, T, stream);
  if (rc != NS_OK) return rc;
  rc = ns_gpt_loss_backward(h, targets, stream);
  if (rc != NS_OK) return rc;
  rc = ns_gpt_backward(h, stream);
  if (rc != NS_OK) return rc;
  if (max_norm > 0.0f) {
    rc = ns_gpt_clip_gradients(h, max_norm, stream);
    if (rc != NS_OK) return rc;
  }
  rc = ns_gpt_adamw_step(h, stream);
  if (rc != NS_OK) return rc;
  if (host_loss) {
    NS_TRY_CUDA(cudaMemcpyAsync(h->host_small, h->model->Small(), 4 * sizeof(float),
                                cudaMemcpyDeviceToHost, s),
                "loss copy");
    NS_TRY_CUDA(cudaEventRecord(h->step_done, s), "step event");
    rc = nsb::comm::wait_event(h->comm, h->step_done, 600.0);
    if (rc != NS_OK) return rc;
    int32_t tok_err, tgt_err;
    std::memcpy(&tok_err, h->host_small + 1, 4);
    std::memcpy(&tgt_err, h->host_small + 2, 4);
    if (tok_err || tgt_err)
      return nsb::fail(NS_ERR_OUT_OF_RANGE, "a token or target id is outside [0, vocab_size)");
    *host_loss = h->host_small[0] / (float)h->world;
  }
  return NS_OK;
}

ns_status ns_gpt_set_comm(ns_gpt* h, ns_comm* comm, int world_size, int64_t bucket_floats) {
  NS_REQUIRE(h, "ns_gpt_set_comm: NULL model");
  NS_REQUIRE(world_size >= 1, "ns_gpt_set_comm: world_size < 1");
  NS_TRY_CUDA(cudaDeviceSynchronize(), "ns_gpt_set_comm sync");
  release_comm_resources(h);
  h->comm = comm;
  h->world = comm ? world_size : 1;
  if (!comm) return NS_OK;
  h->buckets = neuralsuite::cuda::PlanBuckets(h->model->Config(), bucket_floats);
  int groups = 0;
  for (const Bucket& b : h->buckets) groups = std::max(groups, b.group + 1);
  NS_TRY_CUDA(cudaStreamCreateWithFlags(&h->comm_stream, cudaStreamNonBlocking), "comm stream");
  for (int g = 0; g < groups; ++g) {
    cudaEvent_t e;
    NS_TRY_CUDA(cudaEventCreateWithFlags(&e, cudaEventDisableTiming), "event");
    h->group_ready.push_back(e);
  }
  NS_TRY_CUDA(cudaEventCreateWithFlags(&h->comm_done, cudaEventDisableTiming), "event");
  return NS_OK;
}

ns_status ns_gpt_set_comm_timing(ns_gpt* h, int enable) {
  NS_REQUIRE(h, "ns_gpt_set_comm_timing: NULL model");
  NS_REQUIRE(h->comm && h->world > 1, "ns_gpt_set_comm_timing: no communicator attached");
  h->comm_timing = enable != 0;
  h->comm_timed = false;
  for (cudaEvent_t* e : {&h->t_bwd_end, &h->t_comm_begin, &h->t_comm_end})
    if (!*e) NS_TRY_CUDA(cudaEventCreate(e), "ns_gpt_set_comm_timing");
  return NS_OK;
}

ns_status ns_gpt_comm_times(ns_gpt* h, float* exposed_ms, float* span_ms) {
  NS_REQUIRE(h, "ns_gpt_comm_times: NULL model");
  NS_REQUIRE(exposed_ms && span_ms, "ns_gpt_comm_times: NULL argument");
  NS_REQUIRE(h->comm_timed, "ns_gpt_comm_times: no timed backward since timing was enabled");
  NS_TRY_CUDA(cudaEventSynchronize(h->t_comm_end), "ns_gpt_comm_times");
  NS_TRY_CUDA(cudaEventSynchronize(h->t_bwd_end), "ns_gpt_comm_times");
  float exposed = 0.0f, span = 0.0f;
  // Negative when the compute stream reached its join after the last
  // all-reduce had finished: nothing was exposed.
  NS_TRY_CUDA(cudaEventElapsedTime(&exposed, h->t_bwd_end, h->t_comm_end), "ns_gpt_comm_times");
  NS_TRY_CUDA(cudaEventElapsedTime(&span, h->t_comm_begin, h->t_comm_end), "ns_gpt_comm_times");
  *exposed_ms = exposed > 0.0f ? exposed : 0.0f;
  *span_ms = span;
  return NS_OK;
}

int ns_gpt_plan_buckets(const ns_gpt_config* cfg, int64_t bucket_floats, int64_t* begin,
                        int64_t* end, int max_buckets) {
  if (!cfg) return 0;
  const auto b = neuralsuite::cuda::PlanBuckets(ToConfig(cfg), bucket_floats);
  const int n = (int)b.size();
  for (int i = 0; i < n && i < max_buckets; ++i) {
    if (begin) begin[i] = b[i].begin;
    if (end) end[i] = b[i].end;
  }
  return n;
}

}  // extern "C"
