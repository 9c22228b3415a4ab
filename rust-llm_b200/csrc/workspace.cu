// Device buffers owned by a sampler handle: allocated once at create, never
// in a sampling call.
#include <cuda_runtime.h>

#include <cstdio>

#include "internal.h"

namespace rl {

template <typename T>
static bool dalloc(T** p, size_t n) {
  return cudaMalloc(reinterpret_cast<void**>(p), sizeof(T) * (n ? n : 1)) == cudaSuccess;
}

rl_status alloc_workspace(rl_sampler* h) {
  if (cudaStreamCreateWithFlags(&h->stream, cudaStreamNonBlocking) != cudaSuccess)
    return set_error(RL_ERR_CUDA, "rl_sampler_create: cudaStreamCreate failed");
  const size_t B = static_cast<size_t>(h->max_batch);
  h->mask_words = (h->max_vocab + 31) / 32;
  bool ok = dalloc(&h->stage_logits, B * static_cast<size_t>(h->max_vocab)) &&
            dalloc(&h->stage_hist, B * static_cast<size_t>(h->max_history)) &&
            dalloc(&h->stage_hist_len, B) && dalloc(&h->stage_mask, B * h->mask_words) &&
            dalloc(&h->stage_params, B) && dalloc(&h->stage_u, B) && dalloc(&h->stage_T, B) &&
            dalloc(&h->stage_p, B) && dalloc(&h->stage_tok, B) &&
            dalloc(&h->stage_prob, B) && dalloc(&h->stage_status, B);
  // spec kernel workspace: per-item summaries, candidate lists and
  // histograms that the streaming kernel hands to the finish kernel (one
  // item per row, or up to spec_max_ws_items segments of small batches)
  const size_t items = static_cast<size_t>(spec_max_ws_items(h->num_sms, h->max_batch));
  h->ws.max_items = static_cast<int>(items);
  ok = ok && dalloc(&h->ws.row_done, B) && dalloc(&h->ws.sums, items) && dalloc(&h->ws.cands, items * kN) &&
       dalloc(&h->ws.hcnt, items * kNB) && dalloc(&h->ws.hmass, items * kNB) &&
       dalloc(&h->ws.tabs, items * kHmax) && dalloc(&h->ws.tabn, items) &&
       dalloc(&h->ws.wovf, static_cast<size_t>(spec_max_ctas(h->num_sms)) * kCW * kWovf);
  if (h->flags & RL_CREATE_SHARDED)
    ok = ok && dalloc(&h->shard_send, B * kRec) && dalloc(&h->shard_recv, static_cast<size_t>(kMergeMaxShards) * B * kRec);
  ok = ok && dalloc(&h->part_keys, B * kN) && dalloc(&h->part_stats, B) && dalloc(&h->beam_params, B) &&
       dalloc(&h->zero_u, B);
  ok = ok && dalloc(&h->lm_part, (B < 256 ? B : 256) * static_cast<size_t>(h->num_sms)) && dalloc(&h->lm_err, 1);
  for (int i = 0; i < 3 && ok; ++i) ok = cudaEventCreate(&h->ev[i]) == cudaSuccess;
  if (ok) ok = cudaMemset(h->ws.row_done, 0, sizeof(int32_t) * B) == cudaSuccess &&
               cudaMemset(h->zero_u, 0, sizeof(float) * B) == cudaSuccess &&
               cudaDeviceSynchronize() == cudaSuccess;
  if (!ok) {
    cudaGetLastError();
    return set_error(RL_ERR_OOM, "rl_sampler_create: device allocation failed");
  }
  return RL_OK;
}

void free_workspace(rl_sampler* h) {
  cudaFree(h->stage_logits);
  cudaFree(h->stage_hist);
  cudaFree(h->stage_hist_len);
  cudaFree(h->stage_mask);
  cudaFree(h->stage_params);
  cudaFree(h->stage_u);
  cudaFree(h->stage_T);
  cudaFree(h->stage_p);
  cudaFree(h->stage_tok);
  cudaFree(h->stage_prob);
  cudaFree(h->stage_status);
  cudaFree(h->ws.row_done);
  cudaFree(h->ws.sums);
  cudaFree(h->ws.cands);
  cudaFree(h->ws.hcnt);
  cudaFree(h->ws.hmass);
  cudaFree(h->ws.wovf);
  cudaFree(h->ws.tabs);
  cudaFree(h->ws.tabn);
  h->ws = {};
  cudaFree(h->shard_send);
  cudaFree(h->shard_recv);
  h->shard_send = nullptr;
  h->shard_recv = nullptr;
  cudaFree(h->part_keys);
  cudaFree(h->part_stats);
  cudaFree(h->beam_params);
  cudaFree(h->zero_u);
  cudaFree(h->lm_part);
  cudaFree(h->lm_err);
  h->part_keys = nullptr;
  h->part_stats = nullptr;
  h->beam_params = nullptr;
  h->zero_u = nullptr;
  h->lm_part = nullptr;
  h->lm_err = nullptr;
  for (int i = 0; i < 3; ++i)
    if (h->ev[i]) cudaEventDestroy(h->ev[i]);
  if (h->stream) cudaStreamDestroy(h->stream);
  h->stage_logits = nullptr;
  h->stream = nullptr;
}

}  // namespace rl
