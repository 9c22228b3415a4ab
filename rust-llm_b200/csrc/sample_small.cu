// The spec sampler for short rows: one CTA of 512 threads per row, the
// whole row in shared memory, no pipeline and no second kernel.
//
// Same semantics as the streaming sampler (sample_spec.cu) and the CPU
// restatement it is tested against, step by step:
//   1. penalties on the row's distinct history ids in [0, V) (the first
//      kHmax entries), with their counts: x < 0 ? x * rp : x / rp, then
//      - count * freq - pres (src/decoder.rs:102-110 for the repetition rule)
//   2. mask: an empty mask row allows every id
//   3. a NaN or +inf allowed logit, no allowed finite logit or a non-finite
//      temperature: row_status RL_ERR_NONFINITE; -inf logits are excluded
//   4. temperature <= 0: the argmax (lowest id on ties), probability 1
//   5. e = exp((x - max) / T) in f32, Z = their sum (double)
//   6. order (x desc, id asc), K = top_k > 0 ? min(top_k, allowed) : allowed
//   7. cutoff = first position whose cumulative probability >= top_p (when
//      top_p < 1), else K - 1; S = the cumulative probability there
//   8. draw: first position <= cutoff whose cumulative probability > u * S
//
// The ordered list is built in batches of up to kQBatch keys: a radix
// select over the row in shared memory finds the batch's smallest key, the
// batch is gathered, sorted and scanned; batches continue below it until the
// cutoff and the draw are both found. Short rows are where the streaming
// kernel's fixed per-item costs (its row preparation, the item end and the
// finish kernel) outweigh the data; here a row of 32000 logits is one pass
// into shared memory and a few block-wide steps.
#include <cuda_runtime.h>

#include <climits>

#include "common.cuh"
#include "internal.h"
#include "spec_kernel.cuh"
#include "spec_row.cuh"

namespace rl {
namespace {

constexpr int kQT = 512;
constexpr int kQW = kQT / 32;
constexpr int kQBatch = 1024;     // keys ordered per batch
constexpr int kQMaxBatch = 64;    // batch records kept for the draw
constexpr int kQGather = 2048;    // keys gathered at or above a batch's threshold
constexpr int kQMaxV = 45056;     // longest row held in shared memory (f32)

struct QShared {
  uint32_t bins[256];
  double dred[kQW];
  unsigned long long ured[kQW];
  float fred[kQW];
  int ired[kQW];
  uint64_t bprev[kQMaxBatch];  // batch b: the keys below bprev[b]
  double bcum[kQMaxBatch];     // cumulative probability before batch b
  int bpos[kQMaxBatch];        // list position of batch b's first key
  int sel, above, cntb, cnt;
};

__device__ __forceinline__ float q_f32(float v) { return v; }
__device__ __forceinline__ float q_f32(uint16_t v) { return bf16_bits_to_f32(v); }

// Block reductions: every thread returns the result.
__device__ __forceinline__ int q_sum_i(int v, QShared& sh) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  __syncthreads();
  if ((threadIdx.x & 31) == 0) sh.ired[threadIdx.x >> 5] = v;
  __syncthreads();
  int m = 0;
  for (int w = 0; w < kQW; ++w) m += sh.ired[w];
  return m;
}
__device__ __forceinline__ int q_min_i(int v, QShared& sh) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = min(v, __shfl_xor_sync(0xffffffffu, v, o));
  __syncthreads();
  if ((threadIdx.x & 31) == 0) sh.ired[threadIdx.x >> 5] = v;
  __syncthreads();
  int m = INT_MAX;
  for (int w = 0; w < kQW; ++w) m = min(m, sh.ired[w]);
  return m;
}
__device__ __forceinline__ double q_sum_d(double v, QShared& sh) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  __syncthreads();
  if ((threadIdx.x & 31) == 0) sh.dred[threadIdx.x >> 5] = v;
  __syncthreads();
  double m = 0.0;
  for (int w = 0; w < kQW; ++w) m += sh.dred[w];
  return m;
}
__device__ __forceinline__ uint64_t q_minmax_u64(uint64_t v, bool want_max, QShared& sh) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const uint64_t t = __shfl_xor_sync(0xffffffffu, v, o);
    v = want_max ? (t > v ? t : v) : (t < v ? t : v);
  }
  __syncthreads();
  if ((threadIdx.x & 31) == 0) sh.ured[threadIdx.x >> 5] = v;
  __syncthreads();
  uint64_t m = sh.ured[0];
  for (int w = 1; w < kQW; ++w) m = want_max ? (sh.ured[w] > m ? sh.ured[w] : m) : (sh.ured[w] < m ? sh.ured[w] : m);
  return m;
}
// Inclusive block scan of doubles; *total gets the sum.
__device__ __forceinline__ double q_scan_d(double v, QShared& sh, double* total) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  double inc = v;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const double t = __shfl_up_sync(0xffffffffu, inc, o);
    if (lane >= o) inc += t;
  }
  __syncthreads();
  if (lane == 31) sh.dred[warp] = inc;
  __syncthreads();
  double before = 0.0, tot = 0.0;
  for (int w = 0; w < kQW; ++w) {
    if (w < warp) before += sh.dred[w];
    tot += sh.dred[w];
  }
  *total = tot;
  return before + inc;
}

// The key of position i from the row's value keys kv (ord_key of the
// logit, 0 for an excluded id): (value key, then lower id first).
__device__ __forceinline__ bool q_key(const uint32_t* kv, int i, uint64_t prev, uint64_t* k) {
  const uint32_t k32 = kv[i];
  if (k32 == 0u) return false;
  *k = (static_cast<uint64_t>(k32) << 32) | static_cast<uint64_t>(0xffffffffu - static_cast<uint32_t>(i));
  return *k < prev;
}

// The need-th largest key among the keys below prev (1 <= need <= their
// count): a radix select from the first byte where the keys differ.
__device__ __noinline__ uint64_t q_select(const uint32_t* kv, int V, uint64_t prev, int need, QShared& sh) {
  const int tid = threadIdx.x;
  uint64_t kmin = ~0ull, kmax = 0ull;
  for (int i = tid; i < V; i += kQT) {
    uint64_t k;
    if (q_key(kv, i, prev, &k)) {
      kmin = k < kmin ? k : kmin;
      kmax = k > kmax ? k : kmax;
    }
  }
  kmin = q_minmax_u64(kmin, false, sh);
  kmax = q_minmax_u64(kmax, true, sh);
  if (kmin == kmax) return kmax;
  int shift = 64 - (__clzll(static_cast<long long>(kmin ^ kmax)) & ~7);
  uint64_t prefix = shift >= 64 ? 0ull : ((kmax >> shift) << shift);
  while (true) {
    shift -= 8;
    if (tid < 256) sh.bins[tid] = 0u;
    __syncthreads();
    for (int i = tid; i < V; i += kQT) {
      uint64_t k;
      if (q_key(kv, i, prev, &k) && (shift + 8 >= 64 || (k >> (shift + 8)) == (prefix >> (shift + 8))))
        atomicAdd(&sh.bins[(k >> shift) & 255u], 1u);
    }
    __syncthreads();
    // warp 0: bucket 255 - 8 * lane - j held by lane, descending
    if (tid < 32) {
      uint32_t c[8], ls = 0;
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        c[j] = sh.bins[255 - 8 * tid - j];
        ls += c[j];
      }
      uint32_t inc = ls;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const uint32_t t = __shfl_up_sync(0xffffffffu, inc, o);
        if (tid >= o) inc += t;
      }
      const uint32_t exc = inc - ls;
      const bool hit = exc < static_cast<uint32_t>(need) && inc >= static_cast<uint32_t>(need);
      if (hit) {
        uint32_t run = exc;
        for (int j = 0; j < 8; ++j) {
          if (run + c[j] >= static_cast<uint32_t>(need)) {
            sh.sel = 255 - 8 * tid - j;
            sh.above = static_cast<int>(run);
            sh.cntb = static_cast<int>(c[j]);
            break;
          }
          run += c[j];
        }
      }
    }
    __syncthreads();
    const int bucket = sh.sel, above = sh.above, cntb = sh.cntb;
    __syncthreads();
    prefix |= static_cast<uint64_t>(bucket) << shift;
    need -= above;
    if (shift == 0) return prefix;
    if (cntb == need) {
      // the whole bucket is taken: its smallest key
      uint64_t mn = ~0ull;
      for (int i = tid; i < V; i += kQT) {
        uint64_t k;
        if (q_key(kv, i, prev, &k) && (k >> shift) == (prefix >> shift)) mn = k < mn ? k : mn;
      }
      return q_minmax_u64(mn, false, sh);
    }
  }
}

// Descending bitonic sort of a[0, P) (P a power of two <= kQGather).
__device__ __noinline__ void q_sort_desc(uint64_t* a, int P) {
  for (int k = 2; k <= P; k <<= 1)
    for (int j = k >> 1; j > 0; j >>= 1) {
      for (int i = threadIdx.x; i < P; i += kQT) {
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

// Descending bitonic sort of kQT keys, one per thread (thread t holds
// position t before and after): shuffles within a warp, the shared scratch
// xs across warps.
__device__ __noinline__ uint64_t q_sort_regs(uint64_t v, uint64_t* xs) {
  const int tid = threadIdx.x;
#pragma unroll 1
  for (int k = 2; k <= kQT; k <<= 1)
#pragma unroll 1
    for (int j = k >> 1; j > 0; j >>= 1) {
      uint64_t y;
      if (j < 32) {
        y = __shfl_xor_sync(0xffffffffu, v, j);
      } else {
        __syncthreads();
        xs[tid] = v;
        __syncthreads();
        y = xs[tid ^ j];
      }
      const bool keep_max = ((tid & j) == 0) == ((tid & k) == 0);
      v = keep_max ? (v > y ? v : y) : (v > y ? y : v);
    }
  __syncthreads();
  return v;
}

// Sorts keys[0, c) descending (c <= kQGather); positions up to the next
// power of two get 0.
__device__ void q_sort_keys(uint64_t* keys, int c) {
  const int tid = threadIdx.x;
  if (c <= kQT) {
    const uint64_t v = tid < c ? keys[tid] : 0ull;
    const uint64_t r = q_sort_regs(v, keys + kQT);  // scratch past the keys
    keys[tid] = r;
    __syncthreads();
    return;
  }
  int P = 1;
  while (P < c) P <<= 1;
  for (int i = c + tid; i < P; i += kQT) keys[i] = 0ull;
  __syncthreads();
  q_sort_desc(keys, P);
}

// Keys >= tau and below prev into keys[0, c) (unordered); returns c (the
// writes stop at kQGather, the count does not).
__device__ __noinline__ int q_gather(const uint32_t* kv, int V, uint64_t prev, uint64_t tau, uint64_t* keys, QShared& sh) {
  __syncthreads();
  if (threadIdx.x == 0) sh.cnt = 0;
  __syncthreads();
  for (int i = threadIdx.x; i < V; i += kQT) {
    uint64_t k;
    if (q_key(kv, i, prev, &k) && k >= tau) {
      const int j = atomicAdd(&sh.cnt, 1);
      if (j < kQGather) keys[j] = k;
    }
  }
  __syncthreads();
  return sh.cnt;
}

// Count of the keys >= tau below prev.
__device__ __noinline__ int q_count(const uint32_t* kv, int V, uint64_t prev, uint64_t tau, QShared& sh) {
  int c = 0;
  for (int i = threadIdx.x; i < V; i += kQT) {
    uint64_t k;
    c += (q_key(kv, i, prev, &k) && k >= tau) ? 1 : 0;
  }
  return q_sum_i(c, sh);
}

// One batch: the n = min(kQBatch, left) largest keys below prev, sorted
// descending into keys[0, n), and their cumulative probabilities (from
// base) into cum[0, n); left = the list positions still to order, elig =
// the count of keys below prev (>= left). Returns n.
//
// The batch's keys are those at or above a threshold: taken from a sorted
// sample of the row (every s-th position) at the rank where about 1.5 n
// keys are expected above it, checked by a count, and moved (up to three
// times) until n <= count <= kQGather; then one gather and one sort. An
// exact radix select sets the threshold when the sample cannot (heavy
// ties, or the keys below prev spread unevenly over the sample).
__device__ __noinline__ int q_batch(const uint32_t* kv, int V, uint64_t prev, int left, int elig, float M, const RowT& rt,
                       double Z, double base, uint64_t* keys, double* cum, QShared& sh) {
  const int tid = threadIdx.x;
  const int n = min(kQBatch, left);
  uint64_t tau = 0ull;
  bool ok = elig <= kQT;  // every key below prev: one small sort, no threshold
  if (!ok) {
    // the sample: position t * st for thread t, sorted descending
    const int st = (V + kQT - 1) / kQT;
    uint64_t sk = 0ull;
    if (tid * st < V) {
      uint64_t k;
      if (q_key(kv, tid * st, prev, &k)) sk = k;
    }
    const int ns = q_sum_i(sk != 0ull ? 1 : 0, sh);
    keys[tid] = q_sort_regs(sk, keys + kQT);
    __syncthreads();
    if (ns > 0) {
      long long r = (static_cast<long long>(3 * n / 2 + 16) * ns) / elig;
      for (int tries = 0; tries < 4 && !ok; ++tries) {
        const int rr = static_cast<int>(min(r, static_cast<long long>(ns - 1)));
        const uint64_t t = keys[rr];
        const int c = q_count(kv, V, prev, t, sh);
        if (c >= n && c <= kQGather) {
          tau = t;
          ok = true;
        } else if (c < n) {
          if (rr == ns - 1) break;
          r = 2 * r + 1;
        } else {
          if (rr == 0) break;
          r = r / 2;
        }
      }
    }
  }
  if (!ok) tau = q_select(kv, V, prev, n, sh);
  const int ng = min(q_gather(kv, V, prev, tau, keys, sh), kQGather);
  q_sort_keys(keys, ng);
  // cumulative probabilities, kQT positions per round
  double run = base;
  for (int t0 = 0; t0 < n; t0 += kQT) {
    const int t = t0 + tid;
    const double p = t < n ? static_cast<double>(expf(exact_l(key_val(keys[t]), M, rt))) / Z : 0.0;
    double tot;
    const double c = q_scan_d(p, sh, &tot);
    if (t < n) cum[t] = run + c;
    run += tot;
  }
  __syncthreads();
  return n;
}

struct QArgs {
  const void* logits;
  int64_t ld;
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
};

template <typename E>
__global__ void __launch_bounds__(kQT, 1) small_rows_kernel(const __grid_constant__ QArgs a) {
  extern __shared__ __align__(16) unsigned char qsm[];
  __shared__ QShared sh;
  const int row = blockIdx.x, tid = threadIdx.x;
  const int V = a.V;
  float* vals = reinterpret_cast<float*>(qsm);
  uint64_t* keys = reinterpret_cast<uint64_t*>(qsm + ((static_cast<size_t>(V) * 4 + 15) & ~static_cast<size_t>(15)));
  double* cum = reinterpret_cast<double*>(keys + kQGather);
  int32_t* hs = reinterpret_cast<int32_t*>(cum + kQBatch);
  uint32_t* ms = reinterpret_cast<uint32_t*>(hs + kHmax);  // the row's mask words
  const rl_row_params prm = a.params[row];
  const float u = a.uniforms[row];
  auto finish = [&](int st, int tok, float prob) {
    if (tid == 0) {
      a.out_tok[row] = tok;
      if (a.out_prob) a.out_prob[row] = prob;
      if (a.row_status) a.row_status[row] = st;
    }
  };
  // ---- the row and its history into shared memory ----
  const E* x = reinterpret_cast<const E*>(a.logits) + static_cast<int64_t>(row) * a.ld;
  {
    // 16-byte loads, eight in flight per thread, then the unaligned tail
    constexpr int EPV = 16 / static_cast<int>(sizeof(E));  // elements per load
    const bool al = (reinterpret_cast<uintptr_t>(x) & 15u) == 0;
    const int nv = al ? V / EPV : 0;
    const uint4* xv = reinterpret_cast<const uint4*>(x);
    for (int b0 = tid; b0 < nv; b0 += 8 * kQT) {
      uint4 r[8];
#pragma unroll
      for (int j = 0; j < 8; ++j)
        if (b0 + j * kQT < nv) r[j] = __ldcs(xv + b0 + j * kQT);
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const int q = b0 + j * kQT;
        if (q >= nv) break;
        const uint32_t w[4] = {r[j].x, r[j].y, r[j].z, r[j].w};
        if constexpr (sizeof(E) == 4) {
#pragma unroll
          for (int e = 0; e < 4; ++e) vals[q * 4 + e] = __uint_as_float(w[e]);
        } else {
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            vals[q * 8 + 2 * e] = __uint_as_float(w[e] << 16);
            vals[q * 8 + 2 * e + 1] = __uint_as_float(w[e] & 0xffff0000u);
          }
        }
      }
    }
    for (int i = nv * EPV + tid; i < V; i += kQT) vals[i] = q_f32(x[i]);
  }
  const uint32_t* mrow = a.mask ? a.mask + static_cast<int64_t>(row) * a.mask_stride : nullptr;
  const int nw = (V + 31) / 32;
  int any = 0;
  if (mrow)
    for (int w = tid; w < nw; w += kQT) {
      const uint32_t m = mrow[w];
      ms[w] = m;
      any |= m != 0u;
    }
  const bool pen = !(prm.repeat_penalty == 1.0f && prm.frequency_penalty == 0.0f && prm.presence_penalty == 0.0f);
  int hl = 0;
  if (a.hist && a.hist_len && pen) hl = max(0, min(a.hist_len[row], min(a.hist_stride, kHmax)));
  const int32_t* hrow = a.hist ? a.hist + static_cast<int64_t>(row) * a.hist_stride : nullptr;
  for (int j = tid; j < hl; j += kQT) hs[j] = hrow[j];
  __syncthreads();
  // ---- 1. penalties: each distinct id once, at its first occurrence ----
  for (int j = tid; j < hl; j += kQT) {
    const int id = hs[j];
    if (id < 0 || id >= V) continue;
    bool first = true;
    int c = 0;
    for (int i = 0; i < hl; ++i) {
      if (hs[i] != id) continue;
      if (i < j) {
        first = false;
        break;
      }
      ++c;
    }
    if (first) {
      const float v = vals[id];
      const float x1 = (v < 0.0f) ? __fmul_rn(v, prm.repeat_penalty) : __fdiv_rn(v, prm.repeat_penalty);
      vals[id] = __fsub_rn(__fsub_rn(x1, __fmul_rn(static_cast<float>(c), prm.frequency_penalty)), prm.presence_penalty);
    }
  }
  __syncthreads();
  // ---- 2./3. mask, validity, max, argmax, allowed count ----
  const bool masked = q_sum_i(any, sh) > 0;
  float mx = RL_NEG_INF;
  int bad = 0, nal = 0;
  for (int i = tid; i < V; i += kQT) {
    float v = vals[i];
    const bool allowed = !masked || ((ms[i >> 5] >> (i & 31)) & 1u);
    if (allowed) bad |= (v != v) || (v == RL_POS_INF);
    if (!allowed || !(v > RL_NEG_INF)) v = RL_NEG_INF;  // excluded
    vals[i] = v;
    nal += v > RL_NEG_INF ? 1 : 0;
    mx = fmaxf(mx, v);
  }
  // one reduction round for the three
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    nal += __shfl_xor_sync(0xffffffffu, nal, o);
    bad |= __shfl_xor_sync(0xffffffffu, bad, o);
  }
  __syncthreads();
  if ((tid & 31) == 0) {
    sh.fred[tid >> 5] = mx;
    sh.ired[tid >> 5] = nal;
    sh.bins[tid >> 5] = static_cast<uint32_t>(bad);
  }
  __syncthreads();
  float M = RL_NEG_INF;
  nal = 0;
  bad = 0;
#pragma unroll
  for (int w = 0; w < kQW; ++w) {
    M = fmaxf(M, sh.fred[w]);
    nal += sh.ired[w];
    bad |= static_cast<int>(sh.bins[w]);
  }
  const float T = prm.temperature;
  if (bad || nal == 0 || !(fabsf(T) < RL_POS_INF)) {
    finish(RL_ERR_NONFINITE, -1, 0.0f);
    return;
  }
  int am = INT_MAX;
  for (int i = tid; i < V; i += kQT)
    if (vals[i] == M) am = min(am, i);
  am = q_min_i(am, sh);
  // ---- 4. greedy ----
  if (T <= 0.0f) {
    finish(0, am, 1.0f);
    return;
  }
  // ---- 5. softmax sum ----
  const RowT rt = make_rowt(T);
  // the softmax sum: a per-thread f32 sum of 2^((x - M) log2(e) / T) (each
  // term within a few ulps of the list's exact exponentials), added in double
  float zf = 0.0f;
  for (int i = tid; i < V; i += kQT)
    if (vals[i] > RL_NEG_INF) {
      float y;
      asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(__fmul_rn(__fsub_rn(vals[i], M), rt.c)));
      zf += y;
    }
  const double Z = q_sum_d(static_cast<double>(zf), sh);
  // the row as value keys from here on (ord_key of the logit with -0 read as
  // +0; 0, which no finite logit maps to, marks an excluded id)
  uint32_t* kv = reinterpret_cast<uint32_t*>(vals);
  for (int i = tid; i < V; i += kQT) {
    const float v = vals[i];
    kv[i] = v > RL_NEG_INF ? ord_key(__fadd_rn(v, 0.0f)) : 0u;
  }
  __syncthreads();
  // ---- 6.-8. the ordered list in batches: cutoff, then the draw ----
  const int K = (prm.top_k > 0) ? min(prm.top_k, nal) : nal;
  const bool mass = prm.top_p < 1.0f;
  const double tp = static_cast<double>(prm.top_p);
  uint64_t prev = ~0ull;
  int pos = 0, nb = 0, cutoff = -1;
  double base = 0.0, S = 0.0;
  if (!mass && K == nal) {
    // every allowed id is kept: S is the whole mass, Z / Z
    cutoff = K - 1;
    S = 1.0;
  }
  bool drawn = false;  // the draw target lies in a batch already ordered
  while (pos < K && !drawn && nb < kQMaxBatch) {
    if (tid == 0) {
      sh.bprev[nb] = prev;
      sh.bcum[nb] = base;
      sh.bpos[nb] = pos;
    }
    const int n = q_batch(kv, V, prev, K - pos, nal - pos, M, rt, Z, base, keys, cum, sh);
    ++nb;
    if (cutoff < 0) {
      int c = INT_MAX;
      if (mass)
        for (int t = tid; t < n; t += kQT)
          if (cum[t] >= tp) c = min(c, t);
      c = q_min_i(c, sh);
      if (c != INT_MAX) cutoff = min(pos + c, K - 1);
      else if (pos + n == K) cutoff = K - 1;
      if (cutoff >= 0) S = cum[cutoff - pos];
    }
    // the target u * S <= S is below the end of this batch once the cutoff
    // is known inside it, or once the batch's cumulative mass passes it
    if (cutoff >= 0 && (cutoff < pos + n || cum[n - 1] > static_cast<double>(u) * S)) drawn = true;
    base = cum[n - 1];
    prev = keys[n - 1];
    pos += n;
    __syncthreads();
  }
  if (cutoff < 0 || (!drawn && pos < K)) {
    // more batches than kept records (a draw past 64 * kQBatch keys)
    finish(RL_ERR_UNSUPPORTED, -1, 0.0f);
    return;
  }
  // the draw: the batch whose range holds the target, re-ordered when it is
  // not the last one
  const double target = static_cast<double>(u) * S;
  int b = nb - 1;
  while (b > 0 && sh.bcum[b] > target) --b;
  if (b != nb - 1) {
    q_batch(kv, V, sh.bprev[b], K - sh.bpos[b], nal - sh.bpos[b], M, rt, Z, sh.bcum[b], keys, cum, sh);
  }
  const int p0 = sh.bpos[b];
  const int lim = min(cutoff - p0, kQBatch - 1);  // last position of this batch the draw may take
  int d = INT_MAX;
  for (int t = tid; t <= lim; t += kQT)
    if (cum[t] > target) d = min(d, t);
  d = q_min_i(d, sh);
  if (d == INT_MAX) d = lim;
  const uint64_t kd = keys[d];
  const float e = expf(exact_l(key_val(kd), M, rt));
  finish(0, static_cast<int>(key_id(kd)), static_cast<float>((static_cast<double>(e) / Z) / S));
}

}  // namespace

bool small_rows_ok(int V) { return V >= 1 && V <= kQMaxV; }

cudaError_t launch_small_rows(const SpecArgs& s, int dtype, cudaStream_t stream) {
  QArgs a;
  a.logits = s.logits;
  a.ld = s.ld;
  a.V = s.V;
  a.hist = s.hist;
  a.hist_len = s.hist_len;
  a.hist_stride = s.hist_stride;
  a.mask = s.mask;
  a.mask_stride = s.mask_stride;
  a.params = s.params;
  a.uniforms = s.uniforms;
  a.out_tok = s.out_tok;
  a.out_prob = s.out_prob;
  a.row_status = s.row_status;
  const size_t smem = ((static_cast<size_t>(s.V) * 4 + 15) & ~static_cast<size_t>(15)) + kQGather * 8 + kQBatch * 8 +
                      static_cast<size_t>(kHmax) * 4 + static_cast<size_t>(kQMaxV / 32) * 4;
  cudaError_t e;
  if (dtype == RL_BF16) {
    e = cudaFuncSetAttribute(small_rows_kernel<uint16_t>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             static_cast<int>(smem));
    if (e != cudaSuccess) return e;
    small_rows_kernel<uint16_t><<<s.B, kQT, smem, stream>>>(a);
  } else {
    e = cudaFuncSetAttribute(small_rows_kernel<float>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             static_cast<int>(smem));
    if (e != cudaSuccess) return e;
    small_rows_kernel<float><<<s.B, kQT, smem, stream>>>(a);
  }
  return cudaGetLastError();
}

}  // namespace rl
