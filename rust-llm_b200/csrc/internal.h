// Handle layout and workspace management shared by the C ABI sources.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include "rl_sampler.h"
#include "spec_kernel.cuh"

struct rl_sampler {
  int device = 0;
  int max_batch = 0;
  int max_vocab = 0;
  int max_history = 0;
  int num_sms = 0;
  uint32_t flags = 0;
  uint32_t debug = 0;             // rl_sampler_set_debug switches
  cudaEvent_t ev[3] = {};         // RL_DEBUG_TIMING: around the last call's kernels
  int ev_n = 0;                   // kernels timed by the last call
  cudaStream_t stream = nullptr;  // used by the host-buffer entry points
  // device staging buffers of rl_sample_host (allocated at create)
  float* stage_logits = nullptr;
  int32_t* stage_hist = nullptr;
  int32_t* stage_hist_len = nullptr;
  uint32_t* stage_mask = nullptr;
  int mask_words = 0;
  rl_row_params* stage_params = nullptr;
  float* stage_u = nullptr;
  float* stage_T = nullptr;       // rl_decoder_sample_host: temperatures and top_p
  float* stage_p = nullptr;
  int32_t* stage_tok = nullptr;
  float* stage_prob = nullptr;
  int32_t* stage_status = nullptr;
  // workspace of the chunked spec kernel (arrival counters zeroed at create)
  rl::Workspace ws = {};
  // partial results of rl_beam_step (allocated at create, [max_batch])
  uint64_t* part_keys = nullptr;      // [max_batch * kN]
  rl::PartStats* part_stats = nullptr;
  rl_row_params* beam_params = nullptr;
  // rl_sample_sharded (RL_CREATE_SHARDED): this rank's packed records and the
  // gathered records of all ranks
  uint64_t* shard_send = nullptr;  // [max_batch * kRec]
  uint64_t* shard_recv = nullptr;  // [kMergeMaxShards * max_batch * kRec]
  float* zero_u = nullptr;            // uniforms of partial launches (unused, zero)
  // LM head (rl_lmhead_*): per-CTA row maxima [min(max_batch, 256) * num_sms]
  // and the GEMM's timeout flag
  uint64_t* lm_part = nullptr;
  int* lm_err = nullptr;
};

namespace rl {
rl_status alloc_workspace(rl_sampler* h);
void free_workspace(rl_sampler* h);
rl_status set_error(rl_status st, const char* msg);
rl_status nccl_gather_records(void* comm, const uint64_t* send, uint64_t* recv, int B, int* G, cudaStream_t stream);
void clear_error();
}  // namespace rl
