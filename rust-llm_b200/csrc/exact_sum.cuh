// Bit-exact left-to-right f32 sums on the device (one CTA of kXT threads),
// shared by the reference-semantics samplers (decoder_exact.cu: Decoder::
// sample_with_params, src/decoder.rs:35-100; specdec.cu: SpeculativeDecoder::
// sample / softmax_at, src/inference.rs:376-429). Every sum in those
// functions is an f32 fold from 0; xsum reproduces it without a serial loop:
// while the running sum s stays inside one binade [2^e, 2^(e+1)), every f32
// add RN(s + x) rounds x to a multiple of the binade's ulp u = 2^(e-23)
// independently of s -- except for exact ties, which round to the even
// multiple and so depend on s's last bit. The sum is then an integer prefix
// scan of the per-element units, with the rare ties resolved in order and the
// add that leaves the binade done as a real f32 add.
#pragma once

#include <climits>
#include <cstdint>

#include "common.cuh"

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

}  // namespace
}  // namespace rl
