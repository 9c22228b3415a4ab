// Launch interface of the chunked spec sampling kernel.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include "rl_sampler.h"

namespace rl {

constexpr int kCT = 384;             // threads per chunk CTA (three CTAs per SM)
constexpr int kCW = kCT / 32;        // warps per chunk CTA
constexpr int kCE = 12288;           // logits per chunk (48 KB f32, 24 KB bf16)
constexpr int kGPT = kCE / kCT / 4;  // groups of 4 logits per thread (8)
constexpr int kNB = 1024;            // histogram bins per chunk (absolute grid)
constexpr float kRbin = 16.0f;       // bins per nat of (x - m) / T
constexpr int kKthr = 128;           // top_k <= kKthr: thread-maximum threshold path
constexpr int kKbig = 512;           // histogram path: each chunk keeps its top kKbig
constexpr int kCapC = 1024;          // candidate keys per chunk in the workspace
constexpr int kSmax = 64;            // max chunks per row
constexpr int kHmax = 1024;          // max history entries per row
constexpr int kNPiece = 4;           // bulk-copy pieces per chunk
constexpr int kMaxRounds = 16;       // bin rounds of the finishing walk
constexpr int kMergeCap = 4096;      // keys the finishing CTA holds (32 KB)
constexpr float kMassQ = 1048576.0f; // 2^20 fixed point of bin-relative masses (u32)
constexpr int kBinCntSafe = 3800;    // a bin holding more elements may overflow its u32 mass

// Per-chunk summary written by every chunk CTA.
struct ChunkSum {
  float m;       // chunk max over allowed finite (penalised) logits (-inf: none)
  int argmax;    // lowest row-local id at that max
  int nallow;    // allowed finite logits in the chunk
  int flags;     // bit0 non-finite, bit1 copy timeout, bit2 candidate overflow, bit3 bin overflow
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
  uint32_t* hcnt;              // [max_batch * smax * kNB] counts per chunk bin
  uint32_t* hmass;             // [max_batch * smax * kNB] bin-relative masses, 2^20 fixed point
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
  Workspace ws;
};

int spec_smem_bytes(int es);
int spec_chunks(int V);
cudaError_t launch_spec(const SpecArgs& args, int dtype, cudaStream_t stream);

}  // namespace rl
