// Launch interface of the chunked spec sampling kernel.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include "rl_sampler.h"

namespace rl {

constexpr int kCT = 512;             // threads per chunk CTA
constexpr int kCW = kCT / 32;        // warps per chunk CTA
constexpr int kChunkBytes = 65536;   // logits bytes per chunk (16384 f32 / 32768 bf16)
constexpr int kNB = 1024;            // histogram bins per chunk (absolute grid)
constexpr float kRbin = 16.0f;       // bins per nat of (x - m) / T
constexpr int kKthr = 128;           // top_k <= kKthr: thread-maximum threshold path
constexpr int kKbig = 512;           // histogram path: each chunk keeps its top kKbig
constexpr int kCapC = 1024;          // candidate keys per chunk in the workspace
constexpr int kSmax = 64;            // max chunks per row
constexpr int kHmax = 1024;          // max history entries per row
constexpr int kNPiece = 4;           // bulk-copy pieces per chunk
constexpr int kMaxRounds = 16;       // bin rounds of the finishing walk
constexpr int kMergeCap = 8192;      // merged keys the finishing CTA holds (64 KB)
constexpr double kMassScale = 1099511627776.0;  // 2^40 fixed point for bin masses
constexpr float kMassScaleF = 1099511627776.0f;

// Per-chunk summary written by every chunk CTA.
struct ChunkSum {
  float m;       // chunk max over allowed finite (penalised) logits
  int argmax;    // lowest row-local id at that max
  int nallow;    // allowed finite logits in the chunk
  int flags;     // bit0 non-finite input, bit1 copy timeout, bit2 candidate overflow
  double z;      // sum of exp((x - m) / T) over the chunk, relative to m
  int ncand;     // candidate keys written
  int babs_m;    // absolute bin of m
  int athr;      // histogram path: every element with absolute bin >= athr was kept
  float tau;     // threshold path: every element >= tau was kept
};

// Device workspace owned by the handle (allocated at create).
struct Workspace {
  int32_t* row_done;           // [max_batch] arrival counters, reset by the finisher
  ChunkSum* sums;              // [max_batch * smax]
  uint64_t* cands;             // [max_batch * smax * kCapC]
  uint32_t* hcnt;              // [max_batch * smax * kNB]
  unsigned long long* hmass;   // [max_batch * smax * kNB]
  int smax;
};

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
  int vocab_offset;  // global id of local id 0 (vocabulary shards)
  int mode;
  int chunk_elems;   // elements per chunk
  Workspace ws;
};

int spec_smem_bytes(int es);
int spec_chunks(int V, int es);
cudaError_t launch_spec(const SpecArgs& args, int dtype, cudaStream_t stream);

}  // namespace rl
