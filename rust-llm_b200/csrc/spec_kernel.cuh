// Launch interface of the streaming spec sampling kernel.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include <climits>

#include "rl_sampler.h"

namespace rl {

constexpr int kCW = 8;                     // consumer warps per CTA
constexpr int kConsumers = kCW * 32;       // consumer threads (named barrier 1)
constexpr int kThreads = kConsumers + 64;  // + the copy-issuing warp + the row-preparation warp
constexpr int kProdWarp = kCW;
constexpr int kMetaWarp = kCW + 1;
constexpr int kCE = 4096;                  // logits per chunk
constexpr int kSlice = kCE / kCW;          // logits of one consumer warp per chunk (512)
constexpr int kNS = 3;                     // chunk stages in flight per CTA
constexpr int kStageBytes = kCE * 4;       // one stage (f32 chunk; bf16 uses half)
constexpr int kMaskWords = kCE / 32;       // allowed-token mask words per chunk (128)
constexpr int kN = 128;                    // candidate keys kept per (row, segment)
constexpr int kWcap = 512;                 // per-warp candidate buffer (shared memory)
constexpr int kWovf = 512;                 // per-warp overflow (global): one chunk slice of appends
constexpr int kWcompact = 384;             // a warp compacts before a chunk when it holds more keys
constexpr int kNB = 1024;                  // histogram bins (window)
constexpr float kRbin = 16.0f;             // bins per nat of x / T
constexpr int kHead = 128;                 // window bins above the anchoring max (8 nats)
constexpr int kHmax = 1024;                // history entries per row
constexpr int kCollect = 2048;             // finisher: keys of one bin being resolved
constexpr float kMassQ = 1048576.0f;       // 2^20 fixed point of bin-relative masses
constexpr int kSmax = 64;                  // segments per row

constexpr int kFlagBad = 1;       // NaN / +inf among the allowed logits
constexpr int kFlagTimeout = 2;   // a wait ran out of its budget
constexpr int kFlagHistBad = 4;   // histogram unusable (overflow, no anchor)
constexpr int kNoAnchor = INT_MIN;

// Summary of one (row, segment) item.
struct ItemSum {
  float m;        // max over allowed finite (penalised) logits, -inf if none
  int argmax;     // lowest row-local id at m
  int nallow;     // allowed finite logits
  int flags;      // kFlag*
  double z;       // sum of exp((x - m) / T) over the item
  int ncand;      // sorted candidate keys written (<= kN)
  int atop;       // histogram window top (absolute bin), kNoAnchor if none
  int wlo;        // lowest absolute bin in the window
  int pad;
  unsigned long long qsum;  // sum of the fixed-point masses added
};

// Device workspace owned by the handle (allocated at create).
struct Workspace {
  int32_t* row_done;  // [max_batch] arrival counters, reset by the finisher
  ItemSum* sums;      // [max_items]
  uint64_t* cands;    // [max_items * kN]
  uint32_t* hmass;    // [max_items * kNB]
  uint32_t* hcnt;     // [max_items * kNB]
  uint64_t* wovf;     // [max_ctas * kCW * kWovf] per-warp candidate overflow
  uint32_t* tabs;     // [max_items * kHmax] the item's sorted history table (split launch)
  int32_t* tabn;      // [max_items] its entry count
  int max_items;      // items of a launch with more than one segment per row
};

// Per-row result of a partial launch (vocabulary shards, beam candidates):
// the row's sorted top list goes to part_keys[row * kN ...], keys carrying
// global ids (local id + vocab_offset).
struct PartStats {  // layout of rl_part_stats
  float m;       // max over allowed finite logits (-inf if none)
  int argmax;    // lowest global id at m
  int nallow;    // allowed finite logits
  int flags;     // kFlagBad / kFlagTimeout
  double z;      // sum of exp((x - m) / T) over the shard
  int nt;        // keys written (min(top_k, nallow) on the threshold path, else 0)
  int pad;
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
  int32_t* list_cut;  // [B, 3] debug: K, position of the last kept entry, its id
  int vocab_offset;  // global id of local id 0 (vocabulary shards)
  int debug_flags;   // RL_DEBUG_* switches of the handle
  uint64_t* part_keys;   // non-null: partial launch, no draw (see PartStats)
  PartStats* part_stats;
  int part_packed;       // 1: row r's keys at part_keys + r * kRec, its stats right after them
  int nseg;          // segments per row
  int cps;           // chunks per segment
  int nitems;        // B * nseg
  Workspace ws;
};

// Beam step: the rows' partial results combined per item.
constexpr int kBeamMaxBeams = 16;
constexpr int kBeamMaxCand = kBeamMaxBeams * 2 * kBeamMaxBeams;
struct BeamArgs {
  const uint64_t* keys;    // [items * beams * kN] partial top lists
  const PartStats* stats;  // [items * beams]
  int items, beams;
  const float* scores;     // [items * beams]
  const uint8_t* done;     // [items * beams]
  const int32_t* lens;     // [items * beams]
  float alpha;
  int eos, log_softmax, n_out;
  int32_t* out_beam;
  int32_t* out_tok;
  float* out_score;
  uint8_t* out_done;
};
cudaError_t launch_beam_combine(const BeamArgs& b, cudaStream_t stream);
// rows' params of a beam step: T = 1, top_p = 1, top_k, no penalties
cudaError_t launch_fill_params(rl_row_params* p, int n, int top_k, cudaStream_t stream);

// Vocabulary shards: the G partial results of each row merged and drawn.
constexpr int kMergeMaxShards = 16;
// A packed partial record: kN keys then the 32-byte PartStats (u64 units).
constexpr int kRec = kN + 4;
constexpr int kMergeMax = kMergeMaxShards * kN;
struct MergeArgs {
  const uint64_t* keys;    // [G, B, kN], or packed records [G, B, kRec] (stats == nullptr)
  const PartStats* stats;  // [G, B]
  int G, B;
  const rl_row_params* params;
  const float* uniforms;
  int32_t* out_tok;
  float* out_prob;
  int32_t* row_status;
};
cudaError_t launch_shard_merge(const MergeArgs& m, cudaStream_t stream);

int spec_smem_bytes();
__host__ __device__ inline int spec_chunks(int V) { return (V + kCE - 1) / kCE; }
// Segments per row, chunks per segment and CTAs for a batch (host side).
void spec_plan(int B, int V, int num_sms, int* nseg, int* cps, int* nctas);
// Items of the largest launch that uses the workspace (more than one segment).
int spec_max_ws_items(int num_sms, int max_batch);
// CTAs of the largest launch (the per-warp overflow areas).
inline int spec_max_ctas(int num_sms) { return 2 * num_sms; }
// ev (nullable): three events recorded before the streaming kernel, between
// it and the finish kernel, and after the finish kernel.
cudaError_t launch_spec(const SpecArgs& args, int dtype, int num_sms, cudaStream_t stream,
                        cudaEvent_t* ev = nullptr);

// One segment per row (no per-item workspace: only ws.wovf is used), at most
// max_ctas CTAs (the persistent CTAs loop over the rows).
cudaError_t launch_spec_single(const SpecArgs& args, int dtype, int num_sms, int max_ctas, cudaStream_t stream);
// Sets the single-kernel launch's shared-memory limit for both dtypes on the
// current device (what its first launch per dtype would do otherwise).
cudaError_t spec_configure_single();

// The short-row kernel (sample_small.cu): one CTA per row with the row in
// shared memory, for rows of at most 45056 logits; plain unmasked
// sampling calls only (no list, cutoff, partial or debug outputs).
bool small_rows_ok(int V);
cudaError_t launch_small_rows(const SpecArgs& args, int dtype, cudaStream_t stream);

}  // namespace rl
