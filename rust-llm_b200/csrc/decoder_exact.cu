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
#include "internal.h"

static thread_local char g_xerr[256];

namespace rl {
namespace {

constexpr int kXT = 512;               // threads per row
constexpr int kXW = kXT / 32;
constexpr int kXPer = 4;               // elements per thread per scan chunk
constexpr int kXChunk = kXT * kXPer;   // 2048
constexpr int kXTies = 64;             // ties resolved per chunk; the next one ends the chunk

struct XShared {
  unsigned long long wtot[kXW];
  int red[2][kXW];
  int bins[256];
  uint32_t tie_base[kXTies];  // units of s before the tie's element (ties rounded down)
  uint32_t tie_q[kXTies];     // the tie's own units rounded down
  int tie_up[kXTies];         // round-ups up to and including each tie
  float s;
  int idx;
  int cnt;
  int sel, gt, eq;
};

__device__ __forceinline__ uint32_t vkey32(float v) { return ord_key(v == 0.0f ? 0.0f : v); }
__device__ __forceinline__ uint64_t vkey64(float v, int i) {
  return (static_cast<uint64_t>(vkey32(v)) << 32) | static_cast<uint64_t>(0xffffffffu - static_cast<uint32_t>(i));
}

// Block-wide minimum (alternating scratch rows: one barrier per call).
__device__ __forceinline__ int xmin(int v, XShared& sh, int& par) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = min(v, __shfl_xor_sync(0xffffffffu, v, o));
  int* r = sh.red[par];
  par ^= 1;
  if ((threadIdx.x & 31) == 0) r[threadIdx.x >> 5] = v;
  __syncthreads();
  int m = r[0];
#pragma unroll
  for (int w = 1; w < kXW; ++w) m = min(m, r[w]);
  return m;
}

__device__ __forceinline__ int xsum_i(int v, XShared& sh, int& par) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  int* r = sh.red[par];
  par ^= 1;
  if ((threadIdx.x & 31) == 0) r[threadIdx.x >> 5] = v;
  __syncthreads();
  int m = 0;
#pragma unroll
  for (int w = 0; w < kXW; ++w) m += r[w];
  return m;
}

// The float with `units` ulps of binade E (biased exponent, 0 = subnormal):
// value = units * 2^(max(E,1) - 150), units < 2^24.
__device__ __forceinline__ float from_units(uint32_t units, int E) {
  return __uint_as_float((static_cast<uint32_t>(max(E, 1) - 1) << 23) + units);
}

// Left-to-right f32 sum s <- RN(s + x_i), i in [0, n), of non-negative x,
// bit-exact. get(i, ok) returns x_i; ok == false: the element adds nothing and
// is no stop position. With use_thr, returns the first ok index i with
// s_i >= thr (the sum after adding x_i), else n. *s_io: the starting sum on
// entry, the sum at the returned index (or after n) on exit. Every thread of
// the block calls it; all return the same values.
template <typename Get>
__device__ int xsum(const Get& get, int n, bool use_thr, float thr, float* s_io, XShared& sh, int& par) {
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  float s = *s_io;
  int base = 0;
  while (base < n) {
    float xv[kXPer];
    bool ok[kXPer];
#pragma unroll
    for (int q = 0; q < kXPer; ++q) {
      const int i = base + tid * kXPer + q;
      bool k = false;
      float x = 0.0f;
      if (i < n) x = get(i, k);
      ok[q] = k;
      xv[q] = k ? x : 0.0f;
    }
    if (s == 0.0f) {
      // 0 + x = x exactly: the sum is the first positive element
      int fpos = INT_MAX, fstop = INT_MAX;
#pragma unroll
      for (int q = 0; q < kXPer; ++q) {
        const int i = base + tid * kXPer + q;
        if (ok[q] && xv[q] > 0.0f) fpos = min(fpos, i);
        if (use_thr && ok[q] && 0.0f >= thr) fstop = min(fstop, i);
      }
      fpos = xmin(fpos, sh, par);
      fstop = xmin(fstop, sh, par);
      if (fstop != INT_MAX && fstop <= fpos) {
        *s_io = 0.0f;
        return fstop;
      }
      if (fpos == INT_MAX) {
        base += kXChunk;
        continue;
      }
#pragma unroll
      for (int q = 0; q < kXPer; ++q)
        if (base + tid * kXPer + q == fpos) sh.s = xv[q];
      __syncthreads();
      s = sh.s;
      __syncthreads();
      if (use_thr && s >= thr) {
        *s_io = s;
        return fpos;
      }
      base = fpos + 1;
      continue;
    }
    // the binade of s: value = S ulps of 2^(e-23)
    const uint32_t sb = __float_as_uint(s);
    const int E = static_cast<int>((sb >> 23) & 0xffu);
    const int e = E ? E - 127 : -126;
    const uint32_t S = E ? ((sb & 0x7fffffu) | 0x800000u) : (sb & 0x7fffffu);
    // per element: units rounded half down (bits 63..16) and the tie flag
    uint64_t pk[kXPer];
    uint64_t tsum = 0;
#pragma unroll
    for (int q = 0; q < kXPer; ++q) {
      uint32_t d = 0, tie = 0;
      const float x = xv[q];
      if (x > 0.0f) {
        const uint32_t xb = __float_as_uint(x);
        const int Ex = static_cast<int>((xb >> 23) & 0xffu);
        const int ex = Ex ? Ex - 127 : -126;
        const uint32_t mx = Ex ? ((xb & 0x7fffffu) | 0x800000u) : (xb & 0x7fffffu);
        if (ex > e) {
          d = 1u << 25;  // x alone leaves the binade
        } else {
          const int sh2 = e - ex;
          if (sh2 == 0) {
            d = mx;
          } else if (sh2 <= 24) {
            const uint32_t half = 1u << (sh2 - 1);
            const uint32_t rem = mx & ((1u << sh2) - 1u);
            d = (mx >> sh2) + (rem > half ? 1u : 0u);
            tie = rem == half ? 1u : 0u;
          }
        }
      }
      pk[q] = (static_cast<uint64_t>(d) << 16) | tie;
      tsum += pk[q];
    }
    // block exclusive scan of tsum
    uint64_t inc = tsum;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const uint64_t t = __shfl_up_sync(0xffffffffu, inc, o);
      if (lane >= o) inc += t;
    }
    if (lane == 31) sh.wtot[warp] = inc;
    __syncthreads();
    uint64_t excl = inc - tsum, total = 0;
#pragma unroll
    for (int w = 0; w < kXW; ++w) {
      const uint64_t t = sh.wtot[w];
      if (w < warp) excl += t;
      total += t;
    }
    // first element that may leave the binade (ties counted up), or the
    // tie past the resolvable count: it is added with a real f32 add
    int jc = INT_MAX;
    {
      uint64_t run = excl;
#pragma unroll
      for (int q = 0; q < kXPer; ++q) {
        const int i = base + tid * kXPer + q;
        const uint64_t before = run;
        run += pk[q];
        const uint64_t ub = static_cast<uint64_t>(S) + (run >> 16) + (run & 0xffffu);
        const bool tie_over = (pk[q] & 1u) && (before & 0xffffu) >= static_cast<uint64_t>(kXTies);
        if (i < n && (ub > 0xffffffull || tie_over)) jc = min(jc, i);
      }
    }
    jc = xmin(jc, sh, par);
    // ties before jc, in index order: round to the even multiple
    const bool any_tie = (total & 0xffffu) != 0;
    if (any_tie) {
      uint64_t run = excl;
#pragma unroll
      for (int q = 0; q < kXPer; ++q) {
        const int i = base + tid * kXPer + q;
        if ((pk[q] & 1u) && i < jc) {
          const int o = static_cast<int>(run & 0xffffu);
          sh.tie_base[o] = S + static_cast<uint32_t>(run >> 16);
          sh.tie_q[o] = static_cast<uint32_t>(pk[q] >> 16);
        }
        run += pk[q];
      }
      __syncthreads();
      if (tid == 0) {
        // ties before jc hold ordinals 0.. in index order (a tie past kXTies
        // ends the chunk); entries past them are never read
        const int nt = min(static_cast<int>(total & 0xffffu), kXTies);
        int ups = 0;
        for (int o = 0; o < nt; ++o) {
          const uint32_t lower = sh.tie_base[o] + static_cast<uint32_t>(ups) + sh.tie_q[o];
          ups += (lower & 1u) ? 1 : 0;
          sh.tie_up[o] = ups;
        }
      }
      __syncthreads();
    }
    // exact sums s_i for i < jc; the first one reaching thr
    int fstop = INT_MAX;
    uint32_t units_jc = 0;
    bool own_jc = false;
    float x_jc = 0.0f;
    {
      uint64_t run = excl;
#pragma unroll
      for (int q = 0; q < kXPer; ++q) {
        const int i = base + tid * kXPer + q;
        const uint64_t before = run;
        run += pk[q];
        if (i == jc) {
          const int tb = static_cast<int>(before & 0xffffu);
          const int ub = (any_tie && tb > 0) ? sh.tie_up[min(tb, kXTies) - 1] : 0;
          units_jc = S + static_cast<uint32_t>(before >> 16) + static_cast<uint32_t>(ub);
          own_jc = true;
          x_jc = xv[q];
        }
        if (use_thr && ok[q] && i < jc) {
          const int ti = static_cast<int>(run & 0xffffu);
          const int up = (any_tie && ti > 0) ? sh.tie_up[ti - 1] : 0;
          const uint32_t units = S + static_cast<uint32_t>(run >> 16) + static_cast<uint32_t>(up);
          if (from_units(units, E) >= thr) fstop = min(fstop, i);
        }
      }
    }
    if (use_thr) {
      fstop = xmin(fstop, sh, par);
      if (fstop != INT_MAX) {
        uint64_t run = excl;
#pragma unroll
        for (int q = 0; q < kXPer; ++q) {
          const int i = base + tid * kXPer + q;
          run += pk[q];
          if (i == fstop) {
            const int ti = static_cast<int>(run & 0xffffu);
            const int up = (any_tie && ti > 0) ? sh.tie_up[ti - 1] : 0;
            sh.s = from_units(S + static_cast<uint32_t>(run >> 16) + static_cast<uint32_t>(up), E);
          }
        }
        __syncthreads();
        *s_io = sh.s;
        __syncthreads();
        return fstop;
      }
    }
    if (jc != INT_MAX) {
      // the add that leaves the binade (or ends the tie list): a real f32 add
      if (own_jc) sh.s = __fadd_rn(from_units(units_jc, E), x_jc);
      __syncthreads();
      s = sh.s;
      __syncthreads();
      bool okj = false;
      if (use_thr) {
        float dummy = get(jc, okj);
        (void)dummy;
      }
      if (use_thr && okj && s >= thr) {
        *s_io = s;
        return jc;
      }
      base = jc + 1;
      continue;
    }
    {
      const int tt = static_cast<int>(total & 0xffffu);
      const int up = (any_tie && tt > 0) ? sh.tie_up[min(tt, kXTies) - 1] : 0;
      s = from_units(S + static_cast<uint32_t>(total >> 16) + static_cast<uint32_t>(up), E);
    }
    __syncthreads();  // tie lists and wtot are rewritten by the next chunk
    base += kXChunk;
  }
  *s_io = s;
  return n;
}

// The same contract for values of either sign (T <= 0 rows): one thread adds.
template <typename Get>
__device__ int xsum_serial(const Get& get, int n, bool use_thr, float thr, float* s_io, XShared& sh) {
  if (threadIdx.x == 0) {
    float s = *s_io;
    int res = n;
    for (int i = 0; i < n; ++i) {
      bool ok = false;
      const float x = get(i, ok);
      if (!ok) continue;
      s = __fadd_rn(s, x);
      if (use_thr && s >= thr) {
        res = i;
        break;
      }
    }
    sh.s = s;
    sh.idx = res;
  }
  __syncthreads();
  const int r = sh.idx;
  *s_io = sh.s;
  __syncthreads();
  return r;
}

template <typename Get>
__device__ __forceinline__ int xsum_any(bool mono, const Get& get, int n, bool use_thr, float thr, float* s_io,
                                        XShared& sh, int& par) {
  return mono ? xsum(get, n, use_thr, thr, s_io, sh, par) : xsum_serial(get, n, use_thr, thr, s_io, sh);
}

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
