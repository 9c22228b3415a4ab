// ref_exact profile on the device: Decoder::sample_with_params
// (src/decoder.rs:35-100), quirk for quirk, one CTA per row with the row in
// shared memory -- or, for a row too long for it, in a global scratch row
// (the handle's staging buffer), read and written through L1/L2.
//
//   decoder.rs:44-55  T > 0: max (f32::max, NaN-ignoring), (x - max) / T,
//                     exp, sequential f32 sum, divide by the sum if > 0
//   decoder.rs:57-81  top_p < 1: stable descending sort, sequential f32
//                     cumsum, cutoff = first position with cumsum >= top_p
//                     (else V); ORIGINAL ids i > cutoff are zeroed; the sum
//                     is taken again and divided out if > 0
//   decoder.rs:83-90  id-order draw: first i with r <= cumsum_i
//   decoder.rs:92-97  no such i: the LAST maximum (Iterator::max_by)
//
// Every sum of the reference is a left-to-right f32 accumulation. The device
// reproduces those sums bit for bit without a serial loop (xsum below): while
// the running sum s stays inside one binade [2^e, 2^(e+1)), every f32 add
// RN(s + x) rounds x to a multiple of the binade's ulp u = 2^(e-23)
// independently of s -- except for exact ties, which round to the even
// multiple and so depend on s's last bit. The sum is then an integer prefix
// scan of the per-element units, with the rare ties resolved in order and
// the add that leaves the binade done as a real f32 add. exp is
// (float)exp((double)y): the correctly rounded f32 exponential, which is what
// a libm expf returns except in rare near-halfway cases.
//
// Deviation (documented in the header): a row holding NaN or +-inf returns
// token -1 and probability 0.
#include <climits>
#include <cstdio>

#include "common.cuh"
#include "exact_sum.cuh"
#include "internal.h"

static thread_local char g_xerr[256];

namespace rl {
namespace {

// The need-th largest (1-based) value key among those < prev; *n_gt the
// count of keys above it (< prev), *n_eq the count equal to it.
__device__ uint32_t select_key(const float* vals, int V, uint64_t prev, int need, int* n_gt, int* n_eq, XShared& sh) {
  const int tid = threadIdx.x, lane = tid & 31;
  uint32_t prefix = 0, known = 0;
  int gt = 0, eq = 0;
  for (int pass = 0; pass < 4; ++pass) {
    const int shift = 24 - 8 * pass;
    if (tid < 256) sh.bins[tid] = 0;
    __syncthreads();
    for (int i = tid; i < V; i += kXT) {
      const uint32_t o = vkey32(vals[i]);
      if (static_cast<uint64_t>(o) < prev && (o & known) == prefix) atomicAdd(&sh.bins[(o >> shift) & 255u], 1);
    }
    __syncthreads();
    if (tid < 32) {
      int c = 0;
#pragma unroll
      for (int b = 0; b < 8; ++b) c += sh.bins[lane * 8 + b];
      int suf = c;  // sum over lanes >= lane
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int t = __shfl_down_sync(0xffffffffu, suf, o);
        if (lane + o < 32) suf += t;
      }
      const unsigned hit = __ballot_sync(0xffffffffu, suf >= need);
      const int L = 31 - __clz(hit);
      if (lane == L) {
        int cum = suf - c;
        for (int b = 7; b >= 0; --b) {
          const int cb = sh.bins[lane * 8 + b];
          if (cum + cb >= need) {
            sh.sel = lane * 8 + b;
            sh.gt = cum;
            sh.eq = cb;
            break;
          }
          cum += cb;
        }
      }
    }
    __syncthreads();
    const int sel = sh.sel;
    gt += sh.gt;
    need -= sh.gt;
    eq = sh.eq;
    prefix |= static_cast<uint32_t>(sel) << shift;
    known |= 0xffu << shift;
    __syncthreads();
  }
  *n_gt = gt;
  *n_eq = eq;
  return prefix;
}

__device__ void bitonic_desc(uint64_t* a, int n) {
  for (int k = 2; k <= n; k <<= 1)
    for (int j = k >> 1; j > 0; j >>= 1) {
      for (int i = threadIdx.x; i < n; i += kXT) {
        const int l = i ^ j;
        if (l > i) {
          const uint64_t x = a[i], y = a[l];
          const bool desc = (i & k) == 0;
          if (desc ? (x < y) : (x > y)) {
            a[i] = y;
            a[l] = x;
          }
        }
      }
      __syncthreads();
    }
}

struct XArgs {
  const float* logits;
  int64_t ld;
  int V;
  int cap;  // keys of a sorted batch (power of two)
  float* scratch;      // non-null: the row's working copy lives here (row r at r * scratch_ld)
  int64_t scratch_ld;
  const float* temperature;
  const float* top_p;
  const float* uniforms;
  int32_t* out_tok;
  float* out_prob;
};

__global__ void __launch_bounds__(kXT, 1) decoder_exact_kernel(const __grid_constant__ XArgs a) {
  extern __shared__ __align__(16) unsigned char xsm[];
  __shared__ XShared sh;
  const int V = a.V;
  const int row = blockIdx.x, tid = threadIdx.x;
  // the working copy of the row: shared memory, or the global scratch row
  // (then the sorted batches take the start of shared memory)
  float* vals = a.scratch ? a.scratch + static_cast<int64_t>(row) * a.scratch_ld : reinterpret_cast<float*>(xsm);
  uint64_t* list = reinterpret_cast<uint64_t*>(
      a.scratch ? xsm : xsm + ((static_cast<size_t>(V) * 4 + 15) & ~static_cast<size_t>(15)));
  int par = 0;
  const float* x = a.logits + static_cast<int64_t>(row) * a.ld;
  // ---- load, max (f32::max from f32::MIN), finiteness ----
  float mx = -3.40282347e38f;
  int bad = 0;
  for (int i = tid; i < V; i += kXT) {
    const float v = __ldg(x + i);
    vals[i] = v;
    mx = fmaxf(mx, v);
    bad |= (fabsf(v) < RL_POS_INF) ? 0 : 1;
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
  bad = __any_sync(0xffffffffu, bad) ? 1 : 0;
  if ((tid & 31) == 0) {
    sh.red[0][tid >> 5] = bad;
    reinterpret_cast<float*>(sh.bins)[tid >> 5] = mx;
  }
  __syncthreads();
  {
    int b2 = 0;
    float m2 = -3.40282347e38f;
    for (int w = 0; w < kXW; ++w) {
      b2 |= sh.red[0][w];
      m2 = fmaxf(m2, reinterpret_cast<float*>(sh.bins)[w]);
    }
    bad = b2;
    mx = m2;
  }
  __syncthreads();
  if (bad) {
    if (tid == 0) {
      a.out_tok[row] = -1;
      if (a.out_prob) a.out_prob[row] = 0.0f;
    }
    return;
  }
  const float T = a.temperature[row];
  const float top_p = a.top_p[row];
  const float r = a.uniforms[row];
  const bool mono = T > 0.0f;
  // ---- decoder.rs:44-55 ----
  if (mono) {
    for (int i = tid; i < V; i += kXT) {
      const float y = __fdiv_rn(__fsub_rn(vals[i], mx), T);
      vals[i] = static_cast<float>(exp(static_cast<double>(y)));
    }
    __syncthreads();
    float sum = 0.0f;
    xsum([&](int i, bool& ok) { ok = true; return vals[i]; }, V, false, 0.0f, &sum, sh, par);
    if (sum > 0.0f) {
      for (int i = tid; i < V; i += kXT) vals[i] = __fdiv_rn(vals[i], sum);
    }
    __syncthreads();
  }
  // ---- decoder.rs:57-81 ----
  int cutoff = V;  // no cut
  if (top_p < 1.0f) {
    uint64_t prev = 1ull << 32;
    int pos = 0;
    float cum = 0.0f;
    bool found = false;
    while (pos < V && !found) {
      const int need = min(a.cap, V - pos);
      int n_gt = 0, n_eq = 0;
      const uint32_t t = select_key(vals, V, prev, need, &n_gt, &n_eq, sh);
      const bool all_eq = n_gt + n_eq <= a.cap;
      if (tid == 0) sh.cnt = 0;
      __syncthreads();
      for (int i = tid; i < V; i += kXT) {
        const float v = vals[i];
        const uint32_t o = vkey32(v);
        if (static_cast<uint64_t>(o) < prev && (o > t || (all_eq && o == t))) list[atomicAdd(&sh.cnt, 1)] = vkey64(v, i);
      }
      __syncthreads();
      const int nl = sh.cnt;
      int p2 = 1;
      while (p2 < nl) p2 <<= 1;
      for (int i = nl + tid; i < p2; i += kXT) list[i] = 0ull;
      __syncthreads();
      bitonic_desc(list, p2);
      const int j = xsum_any(mono, [&](int i, bool& ok) { ok = true; return key_val(list[i]); }, nl, true, top_p,
                             &cum, sh, par);
      if (j < nl) {
        cutoff = pos + j;
        found = true;
        break;
      }
      pos += nl;
      if (!all_eq) {
        // a tie group too large to sort: it follows in id order
        const int f = xsum_any(mono,
                               [&](int i, bool& ok) {
                                 const float v = vals[i];
                                 ok = vkey32(v) == t;
                                 return v;
                               },
                               V, true, top_p, &cum, sh, par);
        if (f < V) {
          int c = 0;
          for (int i = tid; i < f; i += kXT) c += vkey32(vals[i]) == t ? 1 : 0;
          cutoff = pos + xsum_i(c, sh, par);
          found = true;
          break;
        }
        pos += n_eq;
      }
      prev = t;
    }
    // ORIGINAL ids beyond the cutoff position are zeroed, then renormalised
    for (int i = cutoff + 1 + tid; i < V; i += kXT) vals[i] = 0.0f;
    __syncthreads();
    const int nz = min(V, cutoff + 1);
    float sum = 0.0f;
    xsum_any(mono, [&](int i, bool& ok) { ok = true; return vals[i]; }, nz, false, 0.0f, &sum, sh, par);
    if (sum > 0.0f) {
      for (int i = tid; i < nz; i += kXT) vals[i] = __fdiv_rn(vals[i], sum);
    }
    __syncthreads();
  }
  // ---- decoder.rs:83-97 ----
  const int nd = min(V, cutoff + 1);  // zeros past the cutoff cannot reach r
  float cs = 0.0f;
  int tok = xsum_any(mono, [&](int i, bool& ok) { ok = true; return vals[i]; }, nd, true, r, &cs, sh, par);
  if (tok >= nd) {
    // last maximum of the final array
    uint64_t best = 0;
    for (int i = tid; i < V; i += kXT) {
      const uint64_t k = (static_cast<uint64_t>(vkey32(vals[i])) << 32) | static_cast<uint32_t>(i);
      best = k > best ? k : best;
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const uint64_t n2 = __shfl_xor_sync(0xffffffffu, best, o);
      best = n2 > best ? n2 : best;
    }
    if ((tid & 31) == 0) sh.wtot[tid >> 5] = best;
    __syncthreads();
    uint64_t b = 0;
    for (int w = 0; w < kXW; ++w) b = sh.wtot[w] > b ? sh.wtot[w] : b;
    tok = static_cast<int>(b & 0xffffffffu);
  }
  if (tid == 0) {
    a.out_tok[row] = tok;
    if (a.out_prob) a.out_prob[row] = vals[tok];
  }
}

}  // namespace

// Dynamic shared memory of a launch (-1: does not fit); in_global: the row
// lives in a global scratch row, only the sorted batches in shared memory.
int decoder_exact_smem(int V, int max_optin, int* cap, bool in_global) {
  const size_t base = in_global ? 0 : (static_cast<size_t>(V) * 4 + 15) & ~static_cast<size_t>(15);
  const size_t fixed = sizeof(XShared) + 1024;  // static shared memory and reserve
  for (int c = 2048; c >= 1024; c >>= 1)
    if (base + static_cast<size_t>(c) * 8 + fixed <= static_cast<size_t>(max_optin)) {
      *cap = c;
      return static_cast<int>(base + static_cast<size_t>(c) * 8);
    }
  return -1;
}

cudaError_t launch_decoder_exact(const float* logits, int B, int V, int64_t ld, const float* temperature,
                                 const float* top_p, const float* uniforms, int32_t* out_tok, float* out_prob,
                                 int smem, int cap, float* scratch, int64_t scratch_ld, cudaStream_t stream) {
  cudaError_t e = cudaFuncSetAttribute(decoder_exact_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  if (e != cudaSuccess) return e;
  XArgs a;
  a.logits = logits;
  a.ld = ld;
  a.V = V;
  a.cap = cap;
  a.temperature = temperature;
  a.top_p = top_p;
  a.uniforms = uniforms;
  a.out_tok = out_tok;
  a.out_prob = out_prob;
  a.scratch = scratch;
  a.scratch_ld = scratch_ld;
  decoder_exact_kernel<<<B, kXT, smem, stream>>>(a);
  return cudaGetLastError();
}

}  // namespace rl

extern "C" {
#pragma GCC visibility push(default)

// The launch behind rl_decoder_sample and rl_decoder_sample_host (the
// handle's device is current). A row that does not fit in shared memory is
// worked on in the handle's staging buffer (row r at r * max_vocab), which
// may be the logits themselves (the host entry copies them there first).
static rl_status decoder_sample_dev(rl_sampler* h, const float* logits, int B, int V, int64_t ld,
                                   const float* temperature, const float* top_p, const float* uniforms,
                                   int32_t* out_tok, float* out_prob, cudaStream_t stream, const char* who) {
  int optin = 0;
  cudaError_t e = cudaDeviceGetAttribute(&optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, h->device);
  if (e != cudaSuccess) return rl::set_error(RL_ERR_CUDA, cudaGetErrorString(e));
  int cap = 0;
  int smem = rl::decoder_exact_smem(V, optin, &cap, false);
  float* scratch = nullptr;
  if (smem <= 0) {
    if (!h->stage_logits) {
      std::snprintf(g_xerr, sizeof(g_xerr), "%s: V=%d exceeds shared memory and the handle has no staging buffer", who, V);
      return rl::set_error(RL_ERR_SHAPE, g_xerr);
    }
    smem = rl::decoder_exact_smem(V, optin, &cap, true);
    scratch = h->stage_logits;
    if (smem <= 0) return rl::set_error(RL_ERR_SHAPE, "rl_decoder_sample: shared memory too small");
  }
  e = rl::launch_decoder_exact(logits, B, V, ld, temperature, top_p, uniforms, out_tok, out_prob, smem, cap, scratch,
                               h->max_vocab, stream);
  if (e != cudaSuccess) return rl::set_error(RL_ERR_CUDA, cudaGetErrorString(e));
  return RL_OK;
}

// Makes the handle's device current for the scope of a call.
struct XDeviceGuard {
  int prev = -1;
  bool ok = true;
  explicit XDeviceGuard(int dev) {
    if (cudaGetDevice(&prev) != cudaSuccess) prev = -1;
    if (prev != dev) ok = cudaSetDevice(dev) == cudaSuccess;
  }
  ~XDeviceGuard() {
    int cur = -1;
    if (prev >= 0 && cudaGetDevice(&cur) == cudaSuccess && cur != prev) cudaSetDevice(prev);
  }
};

rl_status rl_decoder_sample(rl_sampler* h, const float* logits, int B, int V, int64_t ld, const float* temperature,
                            const float* top_p, const float* uniforms, int32_t* out_tok, float* out_prob,
                            void* stream) {
  rl::clear_error();
  if (!h) return rl::set_error(RL_ERR_INVALID_ARG, "rl_decoder_sample: handle is NULL");
  if (B < 0 || V <= 0) return rl::set_error(RL_ERR_INVALID_ARG, "rl_decoder_sample: bad B or V");
  if (B == 0) return RL_OK;
  if (!logits || !temperature || !top_p || !uniforms || !out_tok)
    return rl::set_error(RL_ERR_INVALID_ARG, "rl_decoder_sample: a required pointer is NULL");
  if (ld < V) return rl::set_error(RL_ERR_INVALID_ARG, "rl_decoder_sample: ld < V");
  if (B > h->max_batch || V > h->max_vocab)
    return rl::set_error(RL_ERR_SHAPE, "rl_decoder_sample: B or V beyond the handle's limits");
  XDeviceGuard g(h->device);
  if (!g.ok) return rl::set_error(RL_ERR_CUDA, "rl_decoder_sample: cudaSetDevice failed");
  return decoder_sample_dev(h, logits, B, V, ld, temperature, top_p, uniforms, out_tok, out_prob,
                            static_cast<cudaStream_t>(stream), "rl_decoder_sample");
}

rl_status rl_decoder_sample_host(rl_sampler* h, const float* logits, int B, int V, const float* temperature,
                                 const float* top_p, const float* uniforms, int32_t* out_tok, float* out_prob) {
  rl::clear_error();
  if (!h) return rl::set_error(RL_ERR_INVALID_ARG, "rl_decoder_sample_host: handle is NULL");
  if (B < 0 || V <= 0) return rl::set_error(RL_ERR_INVALID_ARG, "rl_decoder_sample_host: bad B or V");
  if (B == 0) return RL_OK;
  if (!logits || !temperature || !top_p || !uniforms || !out_tok)
    return rl::set_error(RL_ERR_INVALID_ARG, "rl_decoder_sample_host: a required pointer is NULL");
  if (B > h->max_batch || V > h->max_vocab)
    return rl::set_error(RL_ERR_SHAPE, "rl_decoder_sample_host: B or V beyond the handle's limits");
  if (!h->stage_logits) return rl::set_error(RL_ERR_UNSUPPORTED, "rl_decoder_sample_host: no staging buffers");
  XDeviceGuard g(h->device);
  if (!g.ok) return rl::set_error(RL_ERR_CUDA, "rl_decoder_sample_host: cudaSetDevice failed");
  cudaStream_t s = h->stream;
  // the rows are staged at stride max_vocab, where a long row is also worked on
  const int64_t ld = h->max_vocab;
  cudaError_t e = cudaMemcpy2DAsync(h->stage_logits, sizeof(float) * ld, logits, sizeof(float) * V,
                                    sizeof(float) * V, B, cudaMemcpyHostToDevice, s);
  if (e == cudaSuccess)
    e = cudaMemcpyAsync(h->stage_T, temperature, sizeof(float) * B, cudaMemcpyHostToDevice, s);
  if (e == cudaSuccess)
    e = cudaMemcpyAsync(h->stage_p, top_p, sizeof(float) * B, cudaMemcpyHostToDevice, s);
  if (e == cudaSuccess)
    e = cudaMemcpyAsync(h->stage_u, uniforms, sizeof(float) * B, cudaMemcpyHostToDevice, s);
  if (e != cudaSuccess) return rl::set_error(RL_ERR_CUDA, "rl_decoder_sample_host: copy to the device failed");
  rl_status st = decoder_sample_dev(h, h->stage_logits, B, V, ld, h->stage_T, h->stage_p, h->stage_u, h->stage_tok,
                                    h->stage_prob, s, "rl_decoder_sample_host");
  if (st != RL_OK) return st;
  e = cudaMemcpyAsync(out_tok, h->stage_tok, sizeof(int32_t) * B, cudaMemcpyDeviceToHost, s);
  if (e == cudaSuccess && out_prob)
    e = cudaMemcpyAsync(out_prob, h->stage_prob, sizeof(float) * B, cudaMemcpyDeviceToHost, s);
  if (e == cudaSuccess) e = cudaStreamSynchronize(s);
  if (e != cudaSuccess) return rl::set_error(RL_ERR_CUDA, "rl_decoder_sample_host: copy back failed");
  return RL_OK;
}

}  // extern "C"
