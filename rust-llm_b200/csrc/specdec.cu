// Speculative decoding's sampling arithmetic (SpeculativeDecoder,
// src/inference.rs:238-438) on the device, bit for bit:
//
//   sample      :376-414  T <= 0: argmax of the ids >= offset (Iterator::
//                         max_by: the LAST maximum; 0 when none). T > 0:
//                         v / T, max from f32::MIN, exp(v - max), sequential
//                         f32 sum, divided out when > 0, then the id-order
//                         draw r <= cumsum, else V - 1. Ids include offset.
//   softmax_at  :416-429  max from f32::MIN, exp(v - max) summed left to
//                         right, exp(v[idx] - max) / sum (0 outside the row)
//   verify_and_accept
//               :335-374  the leading drafts with r < min(p / p, 1) where
//                         p = softmax_at(draft) (both of the reference's
//                         probabilities are the target's), then one draw of
//                         sample(target, 1.0, n_draft): the bonus token when
//                         every draft was accepted (kept when > 0 and not the
//                         last draft), the fallback token of generate
//                         (:293-300) when none was (kept when > 0)
//
// One CTA of kXT threads per row; every left-to-right sum is the bit-exact
// xsum of exact_sum.cuh and exp is the correctly rounded f32 exponential
// (float)exp((double)y), so the tokens match the reference's for the same
// uniforms (the reference draws them with rand_simple(), :432-438).
//
// Deviation: a row holding NaN or +inf (where the reference either panics in
// partial_cmp().unwrap() or walks NaN sums) gives token -1 and, for verify,
// accepted -1. -inf logits are ordinary (exp gives 0).
#include <cuda_runtime.h>

#include <cstdio>

#include "common.cuh"
#include "exact_sum.cuh"
#include "internal.h"

namespace rl {
namespace {

struct SDArgs {
  const float* logits;
  int64_t ld;
  int V;
  // sample
  const float* temperature;
  const int32_t* offset;
  const float* uniforms;
  // verify
  const int32_t* drafts;
  int draft_stride;
  const int32_t* n_draft;
  const float* accept_u;
  const int32_t* room;
  const float* draw_u;
  int32_t* out_tok;
  int32_t* out_accepted;
};

__device__ __forceinline__ float exp_f32(float y) { return static_cast<float>(exp(static_cast<double>(y))); }

// Block-wide max of v (f32::max: NaN ignored) and OR of bad.
__device__ __forceinline__ float bmax_or(float v, int& bad, XShared& sh) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  bad = __any_sync(0xffffffffu, bad) ? 1 : 0;
  __syncthreads();  // sh.bins / sh.red may still be read by an earlier step
  if ((threadIdx.x & 31) == 0) {
    reinterpret_cast<float*>(sh.bins)[threadIdx.x >> 5] = v;
    sh.red[0][threadIdx.x >> 5] = bad;
  }
  __syncthreads();
  float m = -3.40282347e38f;
  int b = 0;
#pragma unroll
  for (int w = 0; w < kXW; ++w) {
    m = fmaxf(m, reinterpret_cast<float*>(sh.bins)[w]);
    b |= sh.red[0][w];
  }
  bad = b;
  __syncthreads();
  return m;
}

// SpeculativeDecoder::sample of the row x (every thread returns the token).
__device__ int sd_sample(const float* x, int V, float T, int off, float r, XShared& sh, int& par) {
  const int tid = threadIdx.x;
  if (off < 0) return -1;  // a usize in the reference
  const int n = V - off;
  if (T != T) return V - 1;  // every adjusted value is NaN: the draw falls through
  if (!(T > 0.0f)) {
    // argmax over the ids >= offset, the last maximum; NaN panics there
    if (n <= 0) return 0;
    uint64_t best = 0;
    int nan = 0;
    for (int i = off + tid; i < V; i += kXT) {
      const float v = x[i];
      nan |= v != v;
      const uint64_t k = (static_cast<uint64_t>(ord_key(v == 0.0f ? 0.0f : v)) << 32) | static_cast<uint32_t>(i);
      best = k > best ? k : best;
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const uint64_t t = __shfl_xor_sync(0xffffffffu, best, o);
      best = t > best ? t : best;
    }
    nan = __any_sync(0xffffffffu, nan) ? 1 : 0;
    __syncthreads();
    if ((tid & 31) == 0) {
      sh.wtot[tid >> 5] = best;
      sh.red[1][tid >> 5] = nan;
    }
    __syncthreads();
    uint64_t b = 0;
    int bad = 0;
#pragma unroll
    for (int w = 0; w < kXW; ++w) {
      b = sh.wtot[w] > b ? sh.wtot[w] : b;
      bad |= sh.red[1][w];
    }
    __syncthreads();
    return bad ? -1 : static_cast<int>(b & 0xffffffffu);
  }
  if (n <= 0) return V - 1;
  // adjusted = v / T, its max from f32::MIN
  float mx = -3.40282347e38f;
  int bad = 0;
  for (int i = off + tid; i < V; i += kXT) {
    const float a = __fdiv_rn(x[i], T);
    bad |= (a != a) || (a == RL_POS_INF);
    mx = fmaxf(mx, a);
  }
  mx = bmax_or(mx, bad, sh);
  if (bad) return -1;
  auto e_of = [&](int j) { return exp_f32(__fsub_rn(__fdiv_rn(x[off + j], T), mx)); };
  float sum = 0.0f;
  xsum(
      [&](int j, bool& ok) {
        ok = true;
        return e_of(j);
      },
      n, false, 0.0f, &sum, sh, par);
  const bool norm = sum > 0.0f;
  float cs = 0.0f;
  const int j = xsum(
      [&](int j, bool& ok) {
        ok = true;
        const float e = e_of(j);
        return norm ? __fdiv_rn(e, sum) : e;
      },
      n, true, r, &cs, sh, par);
  return j < n ? j + off : V - 1;
}

__global__ void __launch_bounds__(kXT, 1) specdec_sample_kernel(const __grid_constant__ SDArgs a) {
  __shared__ XShared sh;
  int par = 0;
  const int row = blockIdx.x;
  const float* x = a.logits + static_cast<int64_t>(row) * a.ld;
  const int tok = sd_sample(x, a.V, a.temperature[row], a.offset[row], a.uniforms[row], sh, par);
  if (threadIdx.x == 0) a.out_tok[row] = tok;
}

__global__ void __launch_bounds__(kXT, 1) specdec_verify_kernel(const __grid_constant__ SDArgs a) {
  __shared__ XShared sh;
  __shared__ int acc_sh;
  int par = 0;
  const int row = blockIdx.x, tid = threadIdx.x;
  const int V = a.V;
  const float* x = a.logits + static_cast<int64_t>(row) * a.ld;
  const int D = a.n_draft[row];
  const int32_t* dr = a.drafts + static_cast<int64_t>(row) * a.draft_stride;
  if (D < 1 || D > a.draft_stride) {
    if (tid == 0) {
      a.out_accepted[row] = -1;
      a.out_tok[row] = -1;
    }
    return;
  }
  // softmax_at: the row's max from f32::MIN and its sequential exp sum
  float mx = -3.40282347e38f;
  int bad = 0;
  for (int i = tid; i < V; i += kXT) {
    const float v = x[i];
    bad |= (v != v) || (v == RL_POS_INF);
    mx = fmaxf(mx, v);
  }
  mx = bmax_or(mx, bad, sh);
  if (bad) {
    if (tid == 0) {
      a.out_accepted[row] = -1;
      a.out_tok[row] = -1;
    }
    return;
  }
  float esum = 0.0f;
  xsum(
      [&](int i, bool& ok) {
        ok = true;
        return exp_f32(__fsub_rn(x[i], mx));
      },
      V, false, 0.0f, &esum, sh, par);
  if (tid == 0) {
    int acc = 0;
    const float* au = a.accept_u + static_cast<int64_t>(row) * a.draft_stride;
    for (int i = 0; i < D; ++i) {
      const int id = dr[i];
      float p = 0.0f;
      if (id >= 0 && id < V) p = esum > 0.0f ? __fdiv_rn(exp_f32(__fsub_rn(x[id], mx)), esum) : 0.0f;
      const float acceptance = p > 0.0f ? fminf(__fdiv_rn(p, p), 1.0f) : 0.0f;
      if (au[i] < acceptance) {
        acc = i + 1;
      } else {
        break;
      }
    }
    acc_sh = acc;
  }
  __syncthreads();
  const int acc = acc_sh;
  int tok = -1;
  if ((acc == D && a.room[row] > 0) || acc == 0) {
    const int s = sd_sample(x, V, 1.0f, D, a.draw_u[row], sh, par);
    if (acc == D) tok = (s > 0 && s != dr[D - 1]) ? s : -1;
    else tok = s > 0 ? s : -1;
  }
  if (tid == 0) {
    a.out_accepted[row] = acc;
    a.out_tok[row] = tok;
  }
}

// Makes the handle's device current for the scope of a call.
struct SDDeviceGuard {
  int prev = -1;
  bool ok = true;
  explicit SDDeviceGuard(int dev) {
    if (cudaGetDevice(&prev) != cudaSuccess) prev = -1;
    if (prev != dev) ok = cudaSetDevice(dev) == cudaSuccess;
  }
  ~SDDeviceGuard() {
    int cur = -1;
    if (prev >= 0 && cudaGetDevice(&cur) == cudaSuccess && cur != prev) cudaSetDevice(prev);
  }
};

}  // namespace
}  // namespace rl

extern "C" {
#pragma GCC visibility push(default)

rl_status rl_specdec_sample(rl_sampler* h, const float* logits, int B, int V, int64_t ld, const float* temperature,
                            const int32_t* offset, const float* uniforms, int32_t* out_tok, void* stream) {
  rl::clear_error();
  if (!h) return rl::set_error(RL_ERR_INVALID_ARG, "rl_specdec_sample: handle is NULL");
  if (B < 0 || V <= 0 || ld < V) return rl::set_error(RL_ERR_INVALID_ARG, "rl_specdec_sample: bad B, V or ld");
  if (B == 0) return RL_OK;
  if (!logits || !temperature || !offset || !uniforms || !out_tok)
    return rl::set_error(RL_ERR_INVALID_ARG, "rl_specdec_sample: a required pointer is NULL");
  rl::SDDeviceGuard g(h->device);
  if (!g.ok) return rl::set_error(RL_ERR_CUDA, "rl_specdec_sample: cudaSetDevice failed");
  rl::SDArgs a = {};
  a.logits = logits;
  a.ld = ld;
  a.V = V;
  a.temperature = temperature;
  a.offset = offset;
  a.uniforms = uniforms;
  a.out_tok = out_tok;
  rl::specdec_sample_kernel<<<B, rl::kXT, 0, static_cast<cudaStream_t>(stream)>>>(a);
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return rl::set_error(RL_ERR_CUDA, cudaGetErrorString(e));
  return RL_OK;
}

rl_status rl_specdec_verify(rl_sampler* h, const float* logits, int B, int V, int64_t ld, const int32_t* drafts,
                            int draft_stride, const int32_t* n_draft, const float* accept_u, const int32_t* room,
                            const float* draw_u, int32_t* out_accepted, int32_t* out_tok, void* stream) {
  rl::clear_error();
  if (!h) return rl::set_error(RL_ERR_INVALID_ARG, "rl_specdec_verify: handle is NULL");
  if (B < 0 || V <= 0 || ld < V || draft_stride < 1)
    return rl::set_error(RL_ERR_INVALID_ARG, "rl_specdec_verify: bad B, V, ld or draft_stride");
  if (B == 0) return RL_OK;
  if (!logits || !drafts || !n_draft || !accept_u || !room || !draw_u || !out_accepted || !out_tok)
    return rl::set_error(RL_ERR_INVALID_ARG, "rl_specdec_verify: a required pointer is NULL");
  rl::SDDeviceGuard g(h->device);
  if (!g.ok) return rl::set_error(RL_ERR_CUDA, "rl_specdec_verify: cudaSetDevice failed");
  rl::SDArgs a = {};
  a.logits = logits;
  a.ld = ld;
  a.V = V;
  a.drafts = drafts;
  a.draft_stride = draft_stride;
  a.n_draft = n_draft;
  a.accept_u = accept_u;
  a.room = room;
  a.draw_u = draw_u;
  a.out_accepted = out_accepted;
  a.out_tok = out_tok;
  rl::specdec_verify_kernel<<<B, rl::kXT, 0, static_cast<cudaStream_t>(stream)>>>(a);
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return rl::set_error(RL_ERR_CUDA, cudaGetErrorString(e));
  return RL_OK;
}

#pragma GCC visibility pop
}  // extern "C"
