// Launch interface of the cluster-per-row spec sampling kernel.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include "rl_sampler.h"

namespace rl {

constexpr int kNT = 512;               // threads per CTA
constexpr int kNWarp = kNT / 32;
constexpr int kNB = 1024;              // histogram bins over l = (x - m) / T
constexpr float kRbin = 16.0f;         // bins per nat: the window covers 64 nats
constexpr int kCap = 2048;             // rank-0 collection buffer (keys)
constexpr int kHmax = 1024;            // max history entries per row
constexpr int kCmax = 16;              // max CTAs per cluster
constexpr int kNPiece = 4;             // bulk-copy pieces per slice
constexpr int kMaxRounds = 16;         // collection rounds per row
constexpr double kMassScale = 1099511627776.0;  // 2^40 fixed point for bin masses
constexpr float kMassScaleF = 1099511627776.0f;

// Output modes of the kernel.
enum SpecMode : int {
  kModeSample = 0,  // draw one token per row
};

struct SpecArgs {
  const void* logits;
  int64_t ld;
  int B;
  int V;
  const int32_t* hist;
  const int32_t* hist_len;
  int hist_stride;
  const uint32_t* mask;
  int64_t mask_stride;
  const rl_row_params* params;
  const float* uniforms;
  int32_t* out_tok;
  float* out_prob;
  int32_t* row_status;
  int32_t* list_ids;
  float* list_probs;
  int32_t* list_len;
  int list_cap;
  int L;             // slice length per CTA (elements, multiple of 128)
  int vocab_offset;  // global id of local id 0 (vocabulary shards)
  int mode;
};

int spec_smem_bytes(int L, int es);
int spec_pick_cluster(int B, int V, int es, int num_sms);
cudaError_t launch_spec(const SpecArgs& args, int dtype, int num_sms, cudaStream_t stream);

}  // namespace rl
