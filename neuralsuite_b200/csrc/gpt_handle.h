// The model handle behind the ns_gpt_* C ABI (shared by gpt.cu and the
// KV-cache decoder in decode.cu).
#pragma once

#include <memory>
#include <vector>

#include "comm.h"
#include "gpt_device.h"

struct ns_gpt {
  std::unique_ptr<neuralsuite::cuda::GPTModel> model;
  std::unique_ptr<neuralsuite::cuda::AdamW> opt;
  ns_comm* comm = nullptr;
  int world = 1;
  std::vector<neuralsuite::cuda::Bucket> buckets;
  cudaStream_t comm_stream = nullptr;
  std::vector<cudaEvent_t> group_ready;
  cudaEvent_t comm_done = nullptr;
  cudaEvent_t step_done = nullptr;
  // Communication timing (ns_gpt_set_comm_timing): the compute stream's end
  // of backward, the comm stream's start of the first bucket and its end.
  bool comm_timing = false;
  bool comm_timed = false;  // the events hold a backward's marks
  cudaEvent_t t_bwd_end = nullptr, t_comm_begin = nullptr, t_comm_end = nullptr;
  float* host_small = nullptr;  // pinned: loss + error flags
  int B = 0, T = 0;
};
