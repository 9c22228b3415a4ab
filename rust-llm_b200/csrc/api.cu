// C ABI of the sampler (include/rl_sampler.h): handle lifetime, argument
// validation, error reporting and the launches.
#include <cuda_runtime.h>

#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <cstddef>
#include <cstdint>
#include <string>

#include "rl_sampler.h"
#include "spec_kernel.cuh"
#include "internal.h"

static_assert(sizeof(rl_part_stats) == sizeof(rl::PartStats) && offsetof(rl_part_stats, z) == offsetof(rl::PartStats, z) &&
                  offsetof(rl_part_stats, n) == offsetof(rl::PartStats, nt),
              "rl_part_stats layout");
static_assert(RL_PART_KEYS == rl::kN, "partial list length");

namespace {

thread_local std::string g_err;

rl_status fail(rl_status st, const char* fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  g_err = buf;
  return st;
}

rl_status cuda_fail(cudaError_t e, const char* what) {
  return fail(RL_ERR_CUDA, "%s: %s", what, cudaGetErrorString(e));
}

// Makes the handle's device current for the scope of a call.
struct DeviceGuard {
  int prev = -1;
  bool ok = true;
  explicit DeviceGuard(int dev) {
    if (cudaGetDevice(&prev) != cudaSuccess) prev = -1;
    if (prev != dev) ok = cudaSetDevice(dev) == cudaSuccess;
  }
  ~DeviceGuard() {
    int cur = -1;
    if (prev >= 0 && cudaGetDevice(&cur) == cudaSuccess && cur != prev) cudaSetDevice(prev);
  }
};

}  // namespace

namespace rl {
rl_status set_error(rl_status st, const char* msg) { return fail(st, "%s", msg); }
void clear_error() { g_err.clear(); }
}  // namespace rl

extern "C" {
#pragma GCC visibility push(default)

const char* rl_last_error(void) { return g_err.c_str(); }

const char* rl_version(void) { return "rl_sampler 0.1 (sm_100a)"; }

rl_status rl_sampler_create(rl_sampler** out, int device, int max_batch, int max_vocab,
                            int max_history, uint32_t flags) {
  if (!out) return fail(RL_ERR_INVALID_ARG, "rl_sampler_create: out is NULL");
  *out = nullptr;
  if (max_batch <= 0 || max_vocab <= 0 || max_history < 0)
    return fail(RL_ERR_INVALID_ARG, "rl_sampler_create: limits must be positive");
  if (max_batch > 65535) return fail(RL_ERR_SHAPE, "rl_sampler_create: max_batch > 65535");
  if (max_vocab > (1 << 21) - rl::kCE)
    return fail(RL_ERR_SHAPE, "rl_sampler_create: max_vocab %d > %d", max_vocab, (1 << 21) - rl::kCE);
  if (max_history > rl::kHmax)
    return fail(RL_ERR_SHAPE, "rl_sampler_create: max_history %d > %d", max_history, rl::kHmax);
  if (flags & ~RL_CREATE_SHARDED) return fail(RL_ERR_INVALID_ARG, "rl_sampler_create: unknown flags 0x%x", flags);
  int ndev = 0;
  cudaError_t e = cudaGetDeviceCount(&ndev);
  if (e != cudaSuccess) return cuda_fail(e, "cudaGetDeviceCount");
  if (device < 0 || device >= ndev)
    return fail(RL_ERR_INVALID_ARG, "rl_sampler_create: device %d not present (%d devices)", device, ndev);
  DeviceGuard g(device);
  if (!g.ok) return fail(RL_ERR_CUDA, "rl_sampler_create: cudaSetDevice(%d) failed", device);
  cudaDeviceProp prop;
  e = cudaGetDeviceProperties(&prop, device);
  if (e != cudaSuccess) return cuda_fail(e, "cudaGetDeviceProperties");
  if (prop.major < 10)
    return fail(RL_ERR_UNSUPPORTED, "rl_sampler_create: device %d is sm_%d%d; this library is built for sm_100a",
                device, prop.major, prop.minor);
  rl_sampler* h = new (std::nothrow) rl_sampler();
  if (!h) return fail(RL_ERR_OOM, "rl_sampler_create: host allocation failed");
  h->device = device;
  h->max_batch = max_batch;
  h->max_vocab = max_vocab;
  h->max_history = max_history;
  h->num_sms = prop.multiProcessorCount;
  h->flags = flags;
  rl_status st = rl::alloc_workspace(h);
  if (st != RL_OK) {
    rl::free_workspace(h);
    delete h;
    return st;
  }
  *out = h;
  rl::clear_error();
  return RL_OK;
}

rl_status rl_sampler_set_debug(rl_sampler* h, uint32_t flags) {
  if (!h) return fail(RL_ERR_INVALID_ARG, "rl_sampler_set_debug: handle is NULL");
  if (flags & ~(RL_DEBUG_EXPIRE_WAIT | RL_DEBUG_TIMING))
    return fail(RL_ERR_INVALID_ARG, "rl_sampler_set_debug: unknown flags 0x%x", flags);
  h->debug = flags;
  return RL_OK;
}

rl_status rl_sampler_kernel_times(rl_sampler* h, float* ms, int cap, int* n) {
  if (!h || !n || (cap > 0 && !ms)) return fail(RL_ERR_INVALID_ARG, "rl_sampler_kernel_times: NULL pointer");
  *n = 0;
  if (h->ev_n == 0) return RL_OK;
  DeviceGuard g(h->device);
  cudaError_t e = cudaEventSynchronize(h->ev[h->ev_n]);
  if (e != cudaSuccess) return cuda_fail(e, "rl_sampler_kernel_times");
  const int k = h->ev_n < cap ? h->ev_n : cap;
  for (int i = 0; i < k; ++i) {
    e = cudaEventElapsedTime(&ms[i], h->ev[i], h->ev[i + 1]);
    if (e != cudaSuccess) return cuda_fail(e, "rl_sampler_kernel_times");
  }
  *n = k;
  return RL_OK;
}

rl_status rl_sampler_destroy(rl_sampler* h) {
  if (!h) return RL_OK;
  DeviceGuard g(h->device);
  rl::free_workspace(h);
  delete h;
  return RL_OK;
}

static rl_status sample_common(rl_sampler* h, const void* logits, rl_dtype dtype, int B, int V,
                               int64_t ld, const int32_t* hist, const int32_t* hist_len,
                               int hist_stride, const uint32_t* mask, int64_t mask_stride,
                               const rl_row_params* params, const float* uniforms, int32_t* out_tok,
                               float* out_prob, int32_t* row_status, int32_t* list_ids,
                               float* list_probs, int32_t* list_len, int list_cap, void* stream,
                               int vocab_offset, uint64_t* part_keys = nullptr,
                               rl::PartStats* part_stats = nullptr, int32_t* list_cut = nullptr,
                               int part_packed = 0) {
  if (!h) return fail(RL_ERR_INVALID_ARG, "rl_sample_batch: handle is NULL");
  if (B < 0 || V <= 0) return fail(RL_ERR_INVALID_ARG, "rl_sample_batch: B=%d V=%d", B, V);
  if (B == 0) return RL_OK;
  if (!logits || !params || !uniforms || !(out_tok || part_keys))
    return fail(RL_ERR_INVALID_ARG, "rl_sample_batch: logits, params, uniforms and out_tok are required");
  if (dtype != RL_F32 && dtype != RL_BF16) return fail(RL_ERR_INVALID_ARG, "rl_sample_batch: bad dtype %d", dtype);
  if (ld < V) return fail(RL_ERR_INVALID_ARG, "rl_sample_batch: ld %lld < V %d", (long long)ld, V);
  if (B > h->max_batch || V > h->max_vocab)
    return fail(RL_ERR_SHAPE, "rl_sample_batch: B=%d V=%d beyond the handle's limits (%d, %d)", B, V,
                h->max_batch, h->max_vocab);
  if (hist) {
    if (!hist_len) return fail(RL_ERR_INVALID_ARG, "rl_sample_batch: hist without hist_len");
    if (hist_stride < 0 || hist_stride > h->max_history)
      return fail(RL_ERR_SHAPE, "rl_sample_batch: hist_stride %d beyond max_history %d", hist_stride,
                  h->max_history);
  }
  if (mask && mask_stride < (V + 31) / 32)
    return fail(RL_ERR_INVALID_ARG, "rl_sample_batch: mask_stride %lld < ceil(V/32)", (long long)mask_stride);
  if (list_len && (!list_ids || !list_probs || list_cap <= 0))
    return fail(RL_ERR_INVALID_ARG, "rl_sample_batch_debug: list buffers required");
  DeviceGuard g(h->device);
  if (!g.ok) return fail(RL_ERR_CUDA, "cudaSetDevice(%d) failed", h->device);
  rl::SpecArgs a = {};
  a.logits = logits;
  a.ld = ld;
  a.B = B;
  a.V = V;
  a.hist = hist;
  a.hist_len = hist_len;
  a.hist_stride = hist ? hist_stride : 0;
  a.mask = mask;
  a.mask_stride = mask_stride;
  a.params = params;
  a.uniforms = uniforms;
  a.out_tok = out_tok;
  a.out_prob = out_prob;
  a.row_status = row_status;
  a.list_ids = list_ids;
  a.list_probs = list_probs;
  a.list_len = list_len;
  a.list_cap = list_cap;
  a.list_cut = list_cut;
  a.vocab_offset = vocab_offset;
  a.debug_flags = static_cast<int>(h->debug);
  a.part_keys = part_keys;
  a.part_stats = part_stats;
  a.part_packed = part_packed;
  a.ws = h->ws;
  const bool timed = (h->debug & RL_DEBUG_TIMING) != 0;
  cudaError_t e;
  // short unmasked rows without inspection outputs: the one-kernel short-row
  // sampler (measured faster there; masked rows stay on the streaming
  // kernels, where a sparse allowed set makes the short-row threshold search
  // slower than the two-kernel path)
  const bool small = rl::small_rows_ok(V) && !mask && !list_len && !list_cut && !part_keys && vocab_offset == 0 &&
                     (h->debug & RL_DEBUG_EXPIRE_WAIT) == 0;
  if (small) {
    if (timed) cudaEventRecord(h->ev[0], static_cast<cudaStream_t>(stream));
    e = rl::launch_small_rows(a, dtype, static_cast<cudaStream_t>(stream));
    if (timed) cudaEventRecord(h->ev[1], static_cast<cudaStream_t>(stream));
    h->ev_n = timed ? 1 : 0;
  } else {
    e = rl::launch_spec(a, dtype, h->num_sms, static_cast<cudaStream_t>(stream), timed ? h->ev : nullptr);
    h->ev_n = timed ? 2 : 0;
  }
  if (e != cudaSuccess) return cuda_fail(e, "rl_sample_batch launch");
  return RL_OK;
}

rl_status rl_sample_batch(rl_sampler* h, const void* logits, rl_dtype dtype, int B, int V, int64_t ld,
                          const int32_t* hist, const int32_t* hist_len, int hist_stride,
                          const uint32_t* mask, int64_t mask_stride, const rl_row_params* params,
                          const float* uniforms, int32_t* out_tok, float* out_prob, int32_t* row_status,
                          void* stream) {
  return sample_common(h, logits, dtype, B, V, ld, hist, hist_len, hist_stride, mask, mask_stride, params,
                       uniforms, out_tok, out_prob, row_status, nullptr, nullptr, nullptr, 0, stream, 0);
}

rl_status rl_sample_batch_debug(rl_sampler* h, const void* logits, rl_dtype dtype, int B, int V,
                                int64_t ld, const int32_t* hist, const int32_t* hist_len,
                                int hist_stride, const uint32_t* mask, int64_t mask_stride,
                                const rl_row_params* params, const float* uniforms, int32_t* out_tok,
                                float* out_prob, int32_t* row_status, int32_t* list_ids,
                                float* list_probs, int32_t* list_len, int list_cap, int32_t* out_cut,
                                void* stream) {
  if (!list_len) return fail(RL_ERR_INVALID_ARG, "rl_sample_batch_debug: list_len is NULL");
  return sample_common(h, logits, dtype, B, V, ld, hist, hist_len, hist_stride, mask, mask_stride, params,
                       uniforms, out_tok, out_prob, row_status, list_ids, list_probs, list_len, list_cap,
                       stream, 0, nullptr, nullptr, out_cut);
}

rl_status rl_sample_partial(rl_sampler* h, const void* logits, rl_dtype dtype, int B, int V, int64_t ld,
                            int vocab_offset, const int32_t* hist, const int32_t* hist_len, int hist_stride,
                            const uint32_t* mask, int64_t mask_stride, const rl_row_params* params,
                            uint64_t* out_keys, rl_part_stats* out_stats, void* stream) {
  if (!h) return fail(RL_ERR_INVALID_ARG, "rl_sample_partial: handle is NULL");
  if (!out_keys || !out_stats) return fail(RL_ERR_INVALID_ARG, "rl_sample_partial: out_keys and out_stats are required");
  if (vocab_offset < 0 || static_cast<int64_t>(vocab_offset) + V > INT32_MAX)
    return fail(RL_ERR_INVALID_ARG, "rl_sample_partial: vocab_offset %d out of range", vocab_offset);
  if (B > h->max_batch) return fail(RL_ERR_SHAPE, "rl_sample_partial: B=%d > max_batch %d", B, h->max_batch);
  return sample_common(h, logits, dtype, B, V, ld, hist, hist_len, hist_stride, mask, mask_stride, params,
                       h->zero_u, nullptr, nullptr, nullptr, nullptr, nullptr, nullptr, 0, stream, vocab_offset,
                       out_keys, reinterpret_cast<rl::PartStats*>(out_stats));
}

rl_status rl_sample_merge(rl_sampler* h, int G, int B, const uint64_t* keys, const rl_part_stats* stats,
                          const rl_row_params* params, const float* uniforms, int32_t* out_tok, float* out_prob,
                          int32_t* row_status, void* stream) {
  if (!h) return fail(RL_ERR_INVALID_ARG, "rl_sample_merge: handle is NULL");
  if (G <= 0 || B < 0) return fail(RL_ERR_INVALID_ARG, "rl_sample_merge: G=%d B=%d", G, B);
  if (G > rl::kMergeMaxShards) return fail(RL_ERR_SHAPE, "rl_sample_merge: G=%d > %d", G, rl::kMergeMaxShards);
  if (B == 0) return RL_OK;
  if (!keys || !stats || !params || !uniforms || !out_tok)
    return fail(RL_ERR_INVALID_ARG, "rl_sample_merge: keys, stats, params, uniforms and out_tok are required");
  DeviceGuard g(h->device);
  if (!g.ok) return fail(RL_ERR_CUDA, "cudaSetDevice(%d) failed", h->device);
  rl::MergeArgs m = {};
  m.keys = keys;
  m.stats = reinterpret_cast<const rl::PartStats*>(stats);
  m.G = G;
  m.B = B;
  m.params = params;
  m.uniforms = uniforms;
  m.out_tok = out_tok;
  m.out_prob = out_prob;
  m.row_status = row_status;
  cudaError_t e = rl::launch_shard_merge(m, static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "rl_sample_merge launch");
  return RL_OK;
}

rl_status rl_sample_sharded(rl_sampler* h, void* comm, const void* logits, rl_dtype dtype, int B, int V_local,
                            int64_t ld, int vocab_offset, int V_global, const int32_t* hist, const int32_t* hist_len,
                            int hist_stride, const uint32_t* mask, int64_t mask_stride, const rl_row_params* params,
                            const float* uniforms, int32_t* out_tok, float* out_prob, int32_t* row_status,
                            void* stream) {
  if (!h) return fail(RL_ERR_INVALID_ARG, "rl_sample_sharded: handle is NULL");
  if (!comm) return fail(RL_ERR_INVALID_ARG, "rl_sample_sharded: comm is NULL");
  if (!h->shard_send) return fail(RL_ERR_UNSUPPORTED, "rl_sample_sharded: handle created without RL_CREATE_SHARDED");
  if (B < 0 || V_local <= 0) return fail(RL_ERR_INVALID_ARG, "rl_sample_sharded: B=%d V_local=%d", B, V_local);
  if (vocab_offset < 0 || static_cast<int64_t>(vocab_offset) + V_local > V_global)
    return fail(RL_ERR_INVALID_ARG, "rl_sample_sharded: columns [%d, %lld) outside the vocabulary of %d", vocab_offset,
                static_cast<long long>(vocab_offset) + V_local, V_global);
  if (B > h->max_batch) return fail(RL_ERR_SHAPE, "rl_sample_sharded: B=%d > max_batch %d", B, h->max_batch);
  if (B == 0) return RL_OK;
  if (!out_tok || !uniforms || !params) return fail(RL_ERR_INVALID_ARG, "rl_sample_sharded: a required pointer is NULL");
  DeviceGuard g(h->device);
  if (!g.ok) return fail(RL_ERR_CUDA, "cudaSetDevice(%d) failed", h->device);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  // 1. this rank's columns -> its packed records
  rl_status st = sample_common(h, logits, dtype, B, V_local, ld, hist, hist_len, hist_stride, mask, mask_stride,
                               params, h->zero_u, nullptr, nullptr, nullptr, nullptr, nullptr, nullptr, 0, stream,
                               vocab_offset, h->shard_send, nullptr, nullptr, 1);
  if (st != RL_OK) return st;
  // 2. one all-gather of the records of every rank
  int G = 0;
  st = rl::nccl_gather_records(comm, h->shard_send, h->shard_recv, B, &G, s);
  if (st != RL_OK) return st;
  // 3. the same merge and draw on every rank
  rl::MergeArgs m = {};
  m.keys = h->shard_recv;
  m.stats = nullptr;  // packed records
  m.G = G;
  m.B = B;
  m.params = params;
  m.uniforms = uniforms;
  m.out_tok = out_tok;
  m.out_prob = out_prob;
  m.row_status = row_status;
  cudaError_t e = rl::launch_shard_merge(m, s);
  if (e != cudaSuccess) return cuda_fail(e, "rl_sample_sharded: merge launch");
  return RL_OK;
}

rl_status rl_beam_step(rl_sampler* h, const float* logits, int items, int beams, int V, int64_t ld,
                       const float* beam_scores, const uint8_t* beam_done, const int32_t* beam_len, float alpha,
                       int eos, int log_softmax, int n_out, int32_t* out_beam, int32_t* out_tok, float* out_score,
                       uint8_t* out_done, void* stream) {
  if (!h) return fail(RL_ERR_INVALID_ARG, "rl_beam_step: handle is NULL");
  if (items < 0 || beams < 1 || beams > rl::kBeamMaxBeams)
    return fail(RL_ERR_INVALID_ARG, "rl_beam_step: items=%d beams=%d (1 <= beams <= %d)", items, beams,
                rl::kBeamMaxBeams);
  if (n_out < 1 || n_out > 2 * beams)
    return fail(RL_ERR_INVALID_ARG, "rl_beam_step: n_out=%d not in [1, 2*beams]", n_out);
  if (items == 0) return RL_OK;
  if (!logits || !beam_scores || !beam_done || !out_beam || !out_tok || !out_score || !out_done ||
      (alpha != 1.0f && !beam_len))
    return fail(RL_ERR_INVALID_ARG, "rl_beam_step: a required pointer is NULL");
  const int rows = items * beams;
  if (static_cast<int64_t>(items) * beams > h->max_batch)
    return fail(RL_ERR_SHAPE, "rl_beam_step: items*beams=%lld > max_batch %d",
                static_cast<long long>(items) * beams, h->max_batch);
  DeviceGuard g(h->device);
  if (!g.ok) return fail(RL_ERR_CUDA, "cudaSetDevice(%d) failed", h->device);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  // every row: T = 1, top_k = 2*beams, no nucleus cut, no penalties
  cudaError_t e = rl::launch_fill_params(h->beam_params, rows, 2 * beams, s);
  if (e != cudaSuccess) return cuda_fail(e, "rl_beam_step: params");
  rl_status st = sample_common(h, logits, RL_F32, rows, V, ld, nullptr, nullptr, 0, nullptr, 0, h->beam_params,
                               h->zero_u, nullptr, nullptr, nullptr, nullptr, nullptr, nullptr, 0, stream, 0,
                               h->part_keys, h->part_stats);
  if (st != RL_OK) return st;
  rl::BeamArgs b = {};
  b.keys = h->part_keys;
  b.stats = h->part_stats;
  b.items = items;
  b.beams = beams;
  b.scores = beam_scores;
  b.done = beam_done;
  b.lens = beam_len;
  b.alpha = alpha;
  b.eos = eos;
  b.log_softmax = log_softmax;
  b.n_out = n_out;
  b.out_beam = out_beam;
  b.out_tok = out_tok;
  b.out_score = out_score;
  b.out_done = out_done;
  e = rl::launch_beam_combine(b, s);
  if (e != cudaSuccess) return cuda_fail(e, "rl_beam_step: combine launch");
  return RL_OK;
}

rl_status rl_sample_host(rl_sampler* h, const float* logits, int B, int V, const int32_t* hist,
                         const int32_t* hist_len, int hist_stride, const uint32_t* mask,
                         int64_t mask_stride, const rl_row_params* params, const float* uniforms,
                         int32_t* out_tok, float* out_prob) {
  if (!h) return fail(RL_ERR_INVALID_ARG, "rl_sample_host: handle is NULL");
  if (B < 0 || V <= 0) return fail(RL_ERR_INVALID_ARG, "rl_sample_host: B=%d V=%d", B, V);
  if (B == 0) return RL_OK;
  if (!logits || !params || !uniforms || !out_tok)
    return fail(RL_ERR_INVALID_ARG, "rl_sample_host: logits, params, uniforms and out_tok are required");
  if (!h->stage_logits) return fail(RL_ERR_UNSUPPORTED, "rl_sample_host: handle created without staging buffers");
  if (B > h->max_batch || V > h->max_vocab)
    return fail(RL_ERR_SHAPE, "rl_sample_host: B=%d V=%d beyond the handle's limits", B, V);
  if (hist && (!hist_len || hist_stride < 0 || hist_stride > h->max_history))
    return fail(RL_ERR_SHAPE, "rl_sample_host: bad history arguments");
  if (mask && (mask_stride < (V + 31) / 32 || mask_stride > h->mask_words))
    return fail(RL_ERR_INVALID_ARG, "rl_sample_host: mask_stride must be in [ceil(V/32), ceil(max_vocab/32)]");
  DeviceGuard g(h->device);
  if (!g.ok) return fail(RL_ERR_CUDA, "cudaSetDevice(%d) failed", h->device);
  cudaStream_t s = h->stream;
  cudaError_t e;
#define RL_TRY(call, what)                   \
  do {                                       \
    e = (call);                              \
    if (e != cudaSuccess) return cuda_fail(e, what); \
  } while (0)
  RL_TRY(cudaMemcpyAsync(h->stage_logits, logits, sizeof(float) * (size_t)B * V, cudaMemcpyHostToDevice, s),
         "rl_sample_host: copy logits");
  if (hist) {
    RL_TRY(cudaMemcpyAsync(h->stage_hist, hist, sizeof(int32_t) * (size_t)B * hist_stride, cudaMemcpyHostToDevice, s),
           "rl_sample_host: copy history");
    RL_TRY(cudaMemcpyAsync(h->stage_hist_len, hist_len, sizeof(int32_t) * B, cudaMemcpyHostToDevice, s),
           "rl_sample_host: copy history lengths");
  }
  if (mask)
    RL_TRY(cudaMemcpyAsync(h->stage_mask, mask, sizeof(uint32_t) * (size_t)B * mask_stride, cudaMemcpyHostToDevice, s),
           "rl_sample_host: copy mask");
  RL_TRY(cudaMemcpyAsync(h->stage_params, params, sizeof(rl_row_params) * B, cudaMemcpyHostToDevice, s),
         "rl_sample_host: copy params");
  RL_TRY(cudaMemcpyAsync(h->stage_u, uniforms, sizeof(float) * B, cudaMemcpyHostToDevice, s),
         "rl_sample_host: copy uniforms");
  rl_status st = sample_common(h, h->stage_logits, RL_F32, B, V, V, hist ? h->stage_hist : nullptr,
                               hist ? h->stage_hist_len : nullptr, hist_stride, mask ? h->stage_mask : nullptr,
                               mask_stride, h->stage_params, h->stage_u, h->stage_tok, h->stage_prob,
                               h->stage_status, nullptr, nullptr, nullptr, 0, s, 0);
  if (st != RL_OK) return st;
  RL_TRY(cudaMemcpyAsync(out_tok, h->stage_tok, sizeof(int32_t) * B, cudaMemcpyDeviceToHost, s),
         "rl_sample_host: copy tokens");
  if (out_prob)
    RL_TRY(cudaMemcpyAsync(out_prob, h->stage_prob, sizeof(float) * B, cudaMemcpyDeviceToHost, s),
           "rl_sample_host: copy probabilities");
  RL_TRY(cudaStreamSynchronize(s), "rl_sample_host: synchronize");
#undef RL_TRY
  return RL_OK;
}

}  // extern "C"
