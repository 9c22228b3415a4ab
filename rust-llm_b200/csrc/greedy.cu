// Greedy entry points of the reference's live API, one CTA per row.
//   rl_greedy          Decoder::greedy_sample        src/decoder.rs:160-167
//                      argmax; Iterator::max_by keeps the LAST maximum.
//   rl_grammar_greedy  Sampler::sample_with_grammar  src/decoder.rs:359-376
//                      stable descending sort of the allowed (id, logit)
//                      pairs, first entry: the LOWEST allowed id among the
//                      maxima; an empty allowed set allows every id.
// Both are a single HBM pass with 16-byte loads; rows are independent.
#include <climits>

#include "common.cuh"
#include "internal.h"

namespace rl {

constexpr int kGNT = 256;

// Packs (value, index) so that a larger u64 is the preferred candidate.
// last_wins: ties prefer the larger index (greedy_sample); otherwise the
// smaller index (sample_with_grammar). -0.0 and +0.0 tie (v + 0 maps -0.0
// to +0.0), as partial_cmp has them.
__device__ __forceinline__ uint64_t pack_vi(float v, int i, bool last_wins) {
  const uint32_t lo = last_wins ? static_cast<uint32_t>(i) : 0xffffffffu - static_cast<uint32_t>(i);
  return (static_cast<uint64_t>(ord_key(__fadd_rn(v, 0.0f))) << 32) | lo;
}

__device__ __forceinline__ uint64_t block_max_u64(uint64_t v, uint64_t* red) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const uint64_t n = __shfl_xor_sync(0xffffffffu, v, o);
    v = n > v ? n : v;
  }
  if (lane == 0) red[warp] = v;
  __syncthreads();
  if (warp == 0) {
    v = lane < kGNT / 32 ? red[lane] : 0ull;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const uint64_t n = __shfl_xor_sync(0xffffffffu, v, o);
      v = n > v ? n : v;
    }
    if (lane == 0) red[0] = v;
  }
  __syncthreads();
  return red[0];
}

__global__ void __launch_bounds__(kGNT) greedy_kernel(const float* __restrict__ logits, int V, int64_t ld,
                                                      const uint32_t* __restrict__ mask, int64_t mask_stride,
                                                      int last_wins, int32_t* __restrict__ out_tok) {
  __shared__ uint64_t red[kGNT / 32];
  __shared__ int any_allowed;
  const int row = blockIdx.x;
  const float* x = logits + static_cast<int64_t>(row) * ld;
  const uint32_t* mrow = mask ? mask + static_cast<int64_t>(row) * mask_stride : nullptr;
  bool use_mask = false;
  if (mrow) {
    if (threadIdx.x == 0) any_allowed = 0;
    __syncthreads();
    int found = 0;
    const int nw = (V + 31) >> 5;
    for (int w = threadIdx.x; w < nw && !found; w += kGNT) {
      uint32_t bits = mrow[w];
      const int rem = V - w * 32;
      if (rem < 32) bits &= (1u << rem) - 1u;
      found = bits != 0u;
    }
    if (found) any_allowed = 1;
    __syncthreads();
    use_mask = any_allowed != 0;
  }
  const bool lw = last_wins != 0;
  uint64_t best = 0ull;
  const bool vec = ((reinterpret_cast<uintptr_t>(x) & 15u) == 0);
  const int nv = vec ? V / 4 : 0;
  for (int g = threadIdx.x; g < nv; g += kGNT) {
    const float4 q = reinterpret_cast<const float4*>(x)[g];
    const float v[4] = {q.x, q.y, q.z, q.w};
    uint32_t bits = 0xfu;
    if (use_mask) bits = (mrow[(g * 4) >> 5] >> ((g * 4) & 31)) & 0xfu;
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      if ((bits >> k) & 1u) {
        const uint64_t c = pack_vi(v[k], g * 4 + k, lw);
        best = c > best ? c : best;
      }
    }
  }
  for (int i = nv * 4 + threadIdx.x; i < V; i += kGNT) {
    if (use_mask && !((mrow[i >> 5] >> (i & 31)) & 1u)) continue;
    const uint64_t c = pack_vi(x[i], i, lw);
    best = c > best ? c : best;
  }
  best = block_max_u64(best, red);
  if (threadIdx.x == 0) {
    const uint32_t lo = static_cast<uint32_t>(best & 0xffffffffu);
    out_tok[row] = lw ? static_cast<int32_t>(lo) : static_cast<int32_t>(0xffffffffu - lo);
  }
}

}  // namespace rl

namespace {
rl_status check_common(rl_sampler* h, const float* logits, int B, int V, int64_t ld, int32_t* out_tok,
                       const char* who) {
  if (!h) return rl::set_error(RL_ERR_INVALID_ARG, "greedy: handle is NULL");
  if (B < 0 || V <= 0 || ld < V) return rl::set_error(RL_ERR_INVALID_ARG, "greedy: bad B / V / ld");
  if (B > 0 && (!logits || !out_tok)) return rl::set_error(RL_ERR_INVALID_ARG, "greedy: logits and out_tok are required");
  (void)who;
  return RL_OK;
}
}  // namespace

extern "C" {
#pragma GCC visibility push(default)

rl_status rl_greedy(rl_sampler* h, const float* logits, int B, int V, int64_t ld, int32_t* out_tok,
                    void* stream) {
  rl_status st = check_common(h, logits, B, V, ld, out_tok, "rl_greedy");
  if (st != RL_OK || B == 0) return st;
  int prev = -1;
  cudaGetDevice(&prev);
  if (prev != h->device) cudaSetDevice(h->device);
  rl::greedy_kernel<<<B, rl::kGNT, 0, static_cast<cudaStream_t>(stream)>>>(logits, V, ld, nullptr, 0, 1, out_tok);
  cudaError_t e = cudaGetLastError();
  if (prev >= 0 && prev != h->device) cudaSetDevice(prev);
  if (e != cudaSuccess) return rl::set_error(RL_ERR_CUDA, cudaGetErrorString(e));
  return RL_OK;
}

rl_status rl_grammar_greedy(rl_sampler* h, const float* logits, int B, int V, int64_t ld, const uint32_t* mask,
                            int64_t mask_stride, int32_t* out_tok, void* stream) {
  rl_status st = check_common(h, logits, B, V, ld, out_tok, "rl_grammar_greedy");
  if (st != RL_OK || B == 0) return st;
  if (mask && mask_stride < (V + 31) / 32)
    return rl::set_error(RL_ERR_INVALID_ARG, "rl_grammar_greedy: mask_stride < ceil(V/32)");
  int prev = -1;
  cudaGetDevice(&prev);
  if (prev != h->device) cudaSetDevice(h->device);
  rl::greedy_kernel<<<B, rl::kGNT, 0, static_cast<cudaStream_t>(stream)>>>(logits, V, ld, mask, mask_stride, 0,
                                                                            out_tok);
  cudaError_t e = cudaGetLastError();
  if (prev >= 0 && prev != h->device) cudaSetDevice(prev);
  if (e != cudaSuccess) return rl::set_error(RL_ERR_CUDA, cudaGetErrorString(e));
  return RL_OK;
}

// Host-buffer forms (synchronous, on the handle's stream): the rows are
// copied into the handle's staging buffers (logits at stride max_vocab, mask
// rows at stride ceil(max_vocab / 32)), reduced, and the tokens copied back.
static rl_status greedy_host(rl_sampler* h, const float* logits, int B, int V, const uint32_t* mask,
                             int64_t mask_stride, int lastmax, int32_t* out_tok, const char* who) {
  rl::clear_error();
  if (!h) return rl::set_error(RL_ERR_INVALID_ARG, "greedy (host): handle is NULL");
  if (B < 0 || V <= 0) return rl::set_error(RL_ERR_INVALID_ARG, "greedy (host): bad B or V");
  if (B == 0) return RL_OK;
  if (!logits || !out_tok) return rl::set_error(RL_ERR_INVALID_ARG, "greedy (host): logits and out_tok are required");
  if (B > h->max_batch || V > h->max_vocab) return rl::set_error(RL_ERR_SHAPE, "greedy (host): B or V beyond the handle");
  const int64_t words = (V + 31) / 32;
  if (mask && mask_stride < words) return rl::set_error(RL_ERR_INVALID_ARG, "greedy (host): mask_stride < ceil(V/32)");
  if (!h->stage_logits || (mask && !h->stage_mask))
    return rl::set_error(RL_ERR_UNSUPPORTED, "greedy (host): no staging buffers");
  int prev = -1;
  cudaGetDevice(&prev);
  if (prev != h->device && cudaSetDevice(h->device) != cudaSuccess)
    return rl::set_error(RL_ERR_CUDA, "greedy (host): cudaSetDevice failed");
  cudaStream_t s = h->stream;
  const int64_t ld = h->max_vocab;
  cudaError_t e = cudaMemcpy2DAsync(h->stage_logits, sizeof(float) * ld, logits, sizeof(float) * V, sizeof(float) * V,
                                    B, cudaMemcpyHostToDevice, s);
  if (e == cudaSuccess && mask)
    e = cudaMemcpy2DAsync(h->stage_mask, sizeof(uint32_t) * h->mask_words, mask, sizeof(uint32_t) * mask_stride,
                          sizeof(uint32_t) * words, B, cudaMemcpyHostToDevice, s);
  if (e == cudaSuccess) {
    rl::greedy_kernel<<<B, rl::kGNT, 0, s>>>(h->stage_logits, V, ld, mask ? h->stage_mask : nullptr,
                                             mask ? h->mask_words : 0, lastmax, h->stage_tok);
    e = cudaGetLastError();
  }
  if (e == cudaSuccess) e = cudaMemcpyAsync(out_tok, h->stage_tok, sizeof(int32_t) * B, cudaMemcpyDeviceToHost, s);
  if (e == cudaSuccess) e = cudaStreamSynchronize(s);
  if (prev >= 0 && prev != h->device) cudaSetDevice(prev);
  if (e != cudaSuccess) return rl::set_error(RL_ERR_CUDA, who);
  return RL_OK;
}

rl_status rl_greedy_host(rl_sampler* h, const float* logits, int B, int V, int32_t* out_tok) {
  return greedy_host(h, logits, B, V, nullptr, 0, 1, out_tok, "rl_greedy_host: CUDA error");
}

rl_status rl_grammar_greedy_host(rl_sampler* h, const float* logits, int B, int V, const uint32_t* mask,
                                 int64_t mask_stride, int32_t* out_tok) {
  return greedy_host(h, logits, B, V, mask, mask_stride, 0, out_tok, "rl_grammar_greedy_host: CUDA error");
}

}  // extern "C"
