// Batched spec sampling: penalties -> mask -> temperature -> softmax ->
// top-k -> top-p -> draw.
//
// Reference behaviour (chenyusolar/rust-llm, src/decoder.rs):
//   temperature softmax        Decoder::sample_with_params   decoder.rs:44-55
//   repetition penalty rule    Decoder::apply_repeat_penalty decoder.rs:102-110
//   top-k order                Decoder::top_k_logits         decoder.rs:112-122
//   inclusive top-p cutoff     Decoder::sample_top_p         decoder.rs:124-144
//   strict '<' draw            Decoder::sample_multinomial   decoder.rs:146-158
//   empty allowed set -> all   Sampler::sample_with_grammar  decoder.rs:362-364
//
// Design (B200, sm_100a). A persistent launch of at most two CTAs per SM; a
// row is split into segments of 4096-logit chunks and each CTA owns a list of
// (row, segment) items. A CTA has three roles:
//   * one copy warp streams the chunks through a ring of kNS shared-memory
//     stages with bulk async copies (cp.async.bulk + full/empty mbarrier
//     pairs) -- the only HBM read of the logits;
//   * one preparation warp builds each item's row data one item ahead:
//     parameters, the allowed-mask flag and the history table (sorted,
//     de-duplicated ids with their counts, for the penalties);
//   * eight consumer warps each own a fixed 512-logit slice of every chunk
//     and keep their running state in registers, with no block barrier per
//     chunk: max, allowed count, non-finite check, the softmax sum (per-lane
//     reference, ex2), the candidate keys of the row's top list (per-warp
//     buffer compacted by a warp radix select, bound shared across warps)
//     and, for rows without a small top_k, a windowed histogram of
//     bin-relative masses (16 bins per nat) for deep top-p cutoffs.
// At the end of an item the consumers select the item's top-128 keys; the
// last CTA of a row to finish (the only one when a row is one segment)
// merges the row and writes its token: exact exp over the sorted list, the
// inclusive top-p cutoff and the draw. When the cutoff or the draw lies
// below the list, the merged histogram locates its bin and the row is
// re-read for that bin's logits; an exact radix walk over re-reads of the
// row covers what the histogram cannot.
#include <atomic>
#include <climits>

#include "common.cuh"
#include "spec_kernel.cuh"
#include "spec_row.cuh"

namespace rl {

__device__ __forceinline__ float ex2_approx(float t) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(t));
  return y;
}
// 1.5 * 2^23: adding it to a float f with |f| < 2^22 rounds f to the nearest
// integer n (ties to even), and the sum's bit pattern is 0x4B400000 + n.
constexpr float kMagic = 12582912.0f;
constexpr uint32_t kMagicBits = 0x4B400000u;
// Absolute histogram bin of x, about floor(x * kRbin / T): the nearest integer
// to x * cb - 1/2 by the magic-number add (full-rate float adds, no
// conversion instruction). Non-decreasing in x; equal to the floor except
// that x * cb within rounding of an integer may land one bin lower. Valid for
// |x * cb| < 2^22 (histogram windows anchor well inside that range).
__device__ __forceinline__ int bin_int(float x, const RowT& r) {
  return static_cast<int>(__float_as_uint(__fadd_rn(__fmaf_rn(x, r.cb_hi, -0.5f), kMagic)) - kMagicBits);
}
__device__ __forceinline__ float bin_of(float x, const RowT& r) { return static_cast<float>(bin_int(x, r)); }
// kMassQ exp((u - 1) / kRbin) for the position u in [0, 1] of a logit in its
// bin: the mass relative to the bin's top edge in 2^20 fixed point. A cubic in
// u, the degree-3 Taylor polynomial of the exponential about u = 1/2 expanded
// in powers of u (relative error < 6e-8 on [0, 1]).
constexpr float kMq0 = 985045.9375f, kMq1 = 61565.6953125f, kMq2 = 1922.958740234375f, kMq3 = 41.35395050048828f;
__device__ __forceinline__ float pen_value(float v, int cnt, float rp, float freq, float pres) {
  const float x1 = (v < 0.0f) ? mul_rn(v, rp) : div_rn(v, rp);
  return sub_rn(sub_rn(x1, mul_rn(static_cast<float>(cnt), freq)), pres);
}

// ---------------------------------------------------------------------------
// Shared-memory layout
// ---------------------------------------------------------------------------
struct ItemMeta {
  int item, row, seg, c0, c1;
  int mode;        // 0 greedy, 1 threshold (top_k <= kN), 2 histogram
  int nkeep;       // candidate keys kept
  int need_count;  // histogram counts (top_k > kN)
  int mask_on;     // the row's allowed set is not empty
  int ntab;        // history table entries
  int wbins;       // window depth below the anchor top (bins)
  int top_k;
  float top_p, u, rp, pres, freq;
  RowT rt;
};

struct Ctl {
  unsigned long long tau_shared;  // item-level candidate bound (max over warps)
  unsigned long long res_key;
  long long res_c;
  double res_d;
  int abort;
  int is_last;
  int cnt;
  int sel_bucket;
  uint32_t sel_above, sel_cnt;
  int res_i, res_j;
  float cx_lo, cx_hi;    // value interval of the bin being collected
  float cx_lo2, cx_hi2;  // a second bin collected by the same re-read (empty: +inf, -inf)
  int tab_seq;         // split streaming kernel: item sequence + 1 whose table is sorted
};

struct Red {
  double d[kCW];
  unsigned long long q[kCW];
  float f[kCW];
  int i[kCW];
  uint32_t u[kCW];
};

constexpr int kOffBar = 0;                         // up to 16 mbarriers
constexpr int kOffCtl = 128;
constexpr int kOffRed = 256;
constexpr int kOffWcnt = 512;                      // per-warp candidate counts
constexpr int kOffMeta = 640;                      // 2 ItemMeta
constexpr int kOffTopE = 896;                      // kN floats: exact e of the list
constexpr int kOffTopC = kOffTopE + kN * 4;        // kN doubles: cumulative probabilities
constexpr int kOffTop = kOffTopC + kN * 8;         // kN keys: the sorted list
constexpr int kOffSumS = kOffTop + kN * 8;         // kSmax ItemSum (finisher)
constexpr int kOffSegN = kOffSumS + kSmax * static_cast<int>(sizeof(ItemSum));  // kSmax ints
constexpr int kOffTab = kOffSegN + kSmax * 4;      // 2 x kHmax u32
constexpr int kOffHist = kOffTab + 2 * kHmax * 4;  // mass[kNB] + cnt[kNB] u32
constexpr int kOffRadix = kOffHist + 2 * kNB * 4;  // kCW x 256 u32 radix bins
constexpr int kOffWbuf = kOffRadix + kCW * 256 * 4;   // kCW x kWcap keys
constexpr int kOffMask = kOffWbuf + kCW * kWcap * 8;  // kNS x kMaskWords u32
constexpr int kOffStage = ((kOffMask + kNS * kMaskWords * 4 + 127) / 128) * 128;
constexpr int kSmemBytes = kOffStage + kNS * kStageBytes;
// Finisher reuse: the collect buffer spans the histogram and the radix bins;
// the merged histogram (two kNB double arrays) the warp buffers.
static_assert(kOffRadix + kCW * 256 * 4 - kOffHist >= kCollect * 8, "collect buffer");
static_assert(kCW * kWcap * 8 >= 2 * kNB * 8, "merged histogram");
static_assert(256 * (4 + 8 + 8) <= kCW * 256 * 4, "radix walk bins");
static_assert(kCW * kWcap >= 2 * kNB + 8 * kConsumers && kCollect <= 8 * kConsumers, "sort scratch");
static_assert(kCW * kN <= 4 * kConsumers && kCW * kN * 8 <= kCW * 256 * 4, "item-end sort of the kept keys");
static_assert(sizeof(ItemMeta) <= 128 && sizeof(Ctl) <= 128 && sizeof(Red) <= 256, "smem header");
static_assert(3 * kNS + 5 <= 16, "mbarriers");
static_assert(kOffMeta + 2 * 128 <= kOffTopE, "meta");
static_assert(kOffWcnt + 32 + kCW * 8 + kCW * 4 <= kOffMeta && (kOffWcnt + 32) % 8 == 0,
              "per-warp counts, histogram totals and published bounds");
static_assert(kOffStage % 128 == 0 && kOffMask % 16 == 0 && kOffSumS % 8 == 0 && kOffHist % 16 == 0, "alignment");
static_assert(kSmemBytes <= 113 * 1024, "two CTAs per SM");

int spec_smem_bytes() { return kSmemBytes; }

struct Smem {
  uint64_t* full;    // [kNS]
  uint64_t* empty;   // [kNS]
  uint64_t* mfull;   // [2]
  uint64_t* mempty;  // [2]
  uint64_t* ready;   // [kNS] split kernel: the chunk in the stage is patched
  uint64_t* never;   // a barrier nothing completes (RL_DEBUG_EXPIRE_WAIT)
  Ctl* ctl;
  Red* red;
  int* wcnt;
  ItemMeta* meta;
  float* tope;
  double* topc;
  uint64_t* top;
  ItemSum* sums;
  int* segn;
  uint32_t* tab;
  uint32_t* hmass;
  uint32_t* hcnt;
  uint32_t* radix;
  uint64_t* wbuf;
  uint32_t* maskst;
  unsigned char* stage;
};
extern __shared__ __align__(128) unsigned char g_smem[];
struct Smem;
__device__ __forceinline__ uint32_t* wk_of(const Smem& sm);
__device__ __forceinline__ Smem smem_map() {
  unsigned char* s = g_smem;
  Smem m;
  m.full = reinterpret_cast<uint64_t*>(s + kOffBar);
  m.empty = m.full + kNS;
  m.mfull = m.empty + kNS;
  m.mempty = m.mfull + 2;
  m.ready = m.mempty + 2;
  m.never = m.ready + kNS;
  m.ctl = reinterpret_cast<Ctl*>(s + kOffCtl);
  m.red = reinterpret_cast<Red*>(s + kOffRed);
  m.wcnt = reinterpret_cast<int*>(s + kOffWcnt);
  m.meta = reinterpret_cast<ItemMeta*>(s + kOffMeta);
  m.tope = reinterpret_cast<float*>(s + kOffTopE);
  m.topc = reinterpret_cast<double*>(s + kOffTopC);
  m.top = reinterpret_cast<uint64_t*>(s + kOffTop);
  m.sums = reinterpret_cast<ItemSum*>(s + kOffSumS);
  m.segn = reinterpret_cast<int*>(s + kOffSegN);
  m.tab = reinterpret_cast<uint32_t*>(s + kOffTab);
  m.hmass = reinterpret_cast<uint32_t*>(s + kOffHist);
  m.hcnt = m.hmass + kNB;
  m.radix = reinterpret_cast<uint32_t*>(s + kOffRadix);
  m.wbuf = reinterpret_cast<uint64_t*>(s + kOffWbuf);
  m.maskst = reinterpret_cast<uint32_t*>(s + kOffMask);
  m.stage = s + kOffStage;
  return m;
}
// Per-warp published bounds of compact_warp_buf (kCW u32), after the
// per-warp counts (kCW ints) and histogram totals (kCW u64).
__device__ __forceinline__ uint32_t* wk_of(const Smem& sm) { return reinterpret_cast<uint32_t*>(sm.wcnt + kCW + 2 * kCW); }

// ---------------------------------------------------------------------------
// Small helpers
// ---------------------------------------------------------------------------
__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}
// Barrier of the 256 consumer threads (the other two warps never join it).
__device__ __forceinline__ void cbar() { asm volatile("bar.sync 1, 256;" ::: "memory"); }
__device__ __forceinline__ uint64_t warp_min_u64(uint64_t v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const uint64_t t = __shfl_xor_sync(0xffffffffu, v, o);
    v = t < v ? t : v;
  }
  return v;
}
__device__ __forceinline__ uint64_t warp_max_u64(uint64_t v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const uint64_t t = __shfl_xor_sync(0xffffffffu, v, o);
    v = t > v ? t : v;
  }
  return v;
}
// k agrees with prefix on every bit at or above bit s
__device__ __forceinline__ bool hi_match(uint64_t k, uint64_t prefix, int s) {
  return s >= 64 || ((k ^ prefix) >> s) == 0;
}
template <typename E>
__device__ __forceinline__ float to_f32(E v);
template <>
__device__ __forceinline__ float to_f32<float>(float v) { return v; }
template <>
__device__ __forceinline__ float to_f32<uint16_t>(uint16_t v) { return bf16_bits_to_f32(v); }

__device__ __forceinline__ float pick16(const float (&v)[4][4], int idx) {
  float r = 0.0f;
#pragma unroll
  for (int q = 0; q < 4; ++q)
#pragma unroll
    for (int k = 0; k < 4; ++k)
      if (q * 4 + k == idx) r = v[q][k];
  return r;
}
__device__ __forceinline__ void put16(float (&v)[4][4], int idx, float x) {
#pragma unroll
  for (int q = 0; q < 4; ++q)
#pragma unroll
    for (int k = 0; k < 4; ++k)
      if (q * 4 + k == idx) v[q][k] = x;
}

// Consumer-group reductions: every consumer thread returns the result, and
// the final combination runs in a fixed order, so all threads agree.
__device__ __forceinline__ double csum_d(double v, Red* r) {
  v = warp_sum_d(v);
  v = __shfl_sync(0xffffffffu, v, 0);
  if ((threadIdx.x & 31) == 0) r->d[threadIdx.x >> 5] = v;
  cbar();
  double t = 0.0;
#pragma unroll
  for (int w = 0; w < kCW; ++w) t += r->d[w];
  cbar();
  return t;
}
__device__ __forceinline__ unsigned long long csum_u64(unsigned long long v, Red* r) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  if ((threadIdx.x & 31) == 0) r->q[threadIdx.x >> 5] = v;
  cbar();
  unsigned long long t = 0;
#pragma unroll
  for (int w = 0; w < kCW; ++w) t += r->q[w];
  cbar();
  return t;
}
__device__ __forceinline__ int csum_i(int v, Red* r) {
  v = warp_sum_i(v);
  if ((threadIdx.x & 31) == 0) r->i[threadIdx.x >> 5] = v;
  cbar();
  int t = 0;
#pragma unroll
  for (int w = 0; w < kCW; ++w) t += r->i[w];
  cbar();
  return t;
}
__device__ __forceinline__ int cmin_i(int v, Red* r) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = min(v, __shfl_xor_sync(0xffffffffu, v, o));
  if ((threadIdx.x & 31) == 0) r->i[threadIdx.x >> 5] = v;
  cbar();
  int t = INT_MAX;
#pragma unroll
  for (int w = 0; w < kCW; ++w) t = min(t, r->i[w]);
  cbar();
  return t;
}
__device__ __forceinline__ int cor_i(int v, Red* r) {
  v = __any_sync(0xffffffffu, v) ? 1 : 0;
  if ((threadIdx.x & 31) == 0) r->i[threadIdx.x >> 5] = v;
  cbar();
  int t = 0;
#pragma unroll
  for (int w = 0; w < kCW; ++w) t |= r->i[w];
  cbar();
  return t;
}
__device__ __forceinline__ float cmax_f(float v, Red* r) {
  v = warp_max(v);
  if ((threadIdx.x & 31) == 0) r->f[threadIdx.x >> 5] = v;
  cbar();
  float t = RL_NEG_INF;
#pragma unroll
  for (int w = 0; w < kCW; ++w) t = fmaxf(t, r->f[w]);
  cbar();
  return t;
}
__device__ __forceinline__ uint64_t cmin_u64(uint64_t v, Red* r) {
  v = warp_min_u64(v);
  if ((threadIdx.x & 31) == 0) r->q[threadIdx.x >> 5] = v;
  cbar();
  uint64_t t = ~0ull;
#pragma unroll
  for (int w = 0; w < kCW; ++w) t = r->q[w] < t ? r->q[w] : t;
  cbar();
  return t;
}
__device__ __forceinline__ uint64_t cmax_u64(uint64_t v, Red* r) {
  v = warp_max_u64(v);
  if ((threadIdx.x & 31) == 0) r->q[threadIdx.x >> 5] = v;
  cbar();
  uint64_t t = 0;
#pragma unroll
  for (int w = 0; w < kCW; ++w) t = r->q[w] > t ? r->q[w] : t;
  cbar();
  return t;
}
// Inclusive scans over consumer threads 0..255 (thread order).
__device__ __forceinline__ double cscan_d(double v, Red* r, double* total) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  double s = v;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const double t = __shfl_up_sync(0xffffffffu, s, o);
    if (lane >= o) s += t;
  }
  if (lane == 31) r->d[warp] = s;
  cbar();
  double before = 0.0, tot = 0.0;
#pragma unroll
  for (int w = 0; w < kCW; ++w) {
    if (w < warp) before += r->d[w];
    tot += r->d[w];
  }
  cbar();
  *total = tot;
  return before + s;
}
__device__ __forceinline__ uint32_t cscan_u32(uint32_t v, Red* r) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  uint32_t s = v;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const uint32_t t = __shfl_up_sync(0xffffffffu, s, o);
    if (lane >= o) s += t;
  }
  if (lane == 31) r->u[warp] = s;
  cbar();
  uint32_t before = 0;
#pragma unroll
  for (int w = 0; w < kCW; ++w)
    if (w < warp) before += r->u[w];
  cbar();
  return before + s;
}

// Descending bitonic sort of a[0..n) (n <= P, P a power of two) by the
// consumer threads; a[n..P) is padded with 0 (the smallest key).
// Descending bitonic sort of KPT keys per consumer thread (positions
// tid * KPT + e): compare-exchanges within a thread in registers, within a
// warp by shuffles, across warps through the shared scratch xs (256 * KPT
// keys) -- six block barriers pairs at most for 2048 keys.
template <int KPT>
__device__ __forceinline__ void bitonic_desc_regs(uint64_t (&r)[KPT], uint64_t* xs) {
  const int tid = threadIdx.x;
  constexpr int NPOS = kConsumers * KPT;
  for (int k = 2; k <= NPOS; k <<= 1) {
    for (int j = k >> 1; j > 0; j >>= 1) {
      if (j < KPT) {
#pragma unroll
        for (int e = 0; e < KPT; ++e) {
          const int f = e ^ j;
          if (f > e) {
            const bool desc = ((tid * KPT + e) & k) == 0;
            const uint64_t x = r[e], y = r[f];
            if (desc ? (x < y) : (x > y)) {
              r[e] = y;
              r[f] = x;
            }
          }
        }
      } else {
        uint64_t y[KPT];
        if (j < 32 * KPT) {
#pragma unroll
          for (int e = 0; e < KPT; ++e) y[e] = __shfl_xor_sync(0xffffffffu, r[e], j / KPT);
        } else {
#pragma unroll
          for (int e = 0; e < KPT; ++e) xs[tid * KPT + e] = r[e];
          cbar();
#pragma unroll
          for (int e = 0; e < KPT; ++e) y[e] = xs[(tid * KPT + e) ^ j];
          cbar();
        }
#pragma unroll
        for (int e = 0; e < KPT; ++e) {
          const int i = tid * KPT + e;
          const bool keep_max = ((i & j) == 0) == ((i & k) == 0);
          const uint64_t hi = r[e] > y[e] ? r[e] : y[e];
          const uint64_t lo = r[e] > y[e] ? y[e] : r[e];
          r[e] = keep_max ? hi : lo;
        }
      }
    }
  }
}

template <int KPT>
__device__ __forceinline__ void csort_kpt(uint64_t* a, int n, int P, uint64_t* xs) {
  const int tid = threadIdx.x;
  uint64_t r[KPT];
#pragma unroll
  for (int e = 0; e < KPT; ++e) {
    const int i = tid * KPT + e;
    r[e] = i < n ? a[i] : 0ull;
  }
  cbar();
  bitonic_desc_regs<KPT>(r, xs);
#pragma unroll
  for (int e = 0; e < KPT; ++e) {
    const int i = tid * KPT + e;
    if (i < P) a[i] = r[e];
  }
  cbar();
}

// Sorts a[0, n) descending (keys are > 0); positions [n, P) get 0. P is a
// power of two <= kCollect. Consumer threads only.
__device__ __noinline__ void csort_desc(uint64_t* a, int n, int P) {
  if (P <= 32) {
    // one warp, one key per lane
    if (threadIdx.x < 32) {
      const int lane = threadIdx.x;
      uint64_t r = lane < n ? a[lane] : 0ull;
#pragma unroll
      for (int k = 2; k <= 32; k <<= 1)
#pragma unroll
        for (int j = k >> 1; j > 0; j >>= 1) {
          const uint64_t y = __shfl_xor_sync(0xffffffffu, r, j);
          const bool keep_max = ((lane & j) == 0) == ((lane & k) == 0);
          r = keep_max ? (r > y ? r : y) : (r > y ? y : r);
        }
      if (lane < P) a[lane] = r;
    }
    cbar();
    return;
  }
  // scratch: the second half of the warp-buffer area (the finisher keeps its
  // merged histogram in the first half)
  uint64_t* xs = smem_map().wbuf + 2 * kNB;
  if (P <= kConsumers) csort_kpt<1>(a, n, P, xs);
  else if (P <= 2 * kConsumers) csort_kpt<2>(a, n, P, xs);
  else if (P <= 4 * kConsumers) csort_kpt<4>(a, n, P, xs);
  else csort_kpt<8>(a, n, P, xs);
}
__device__ __forceinline__ int pow2_at_least(int n) {
  int p = 1;
  while (p < n) p <<= 1;
  return p;
}

// ---------------------------------------------------------------------------
// Radix selection of the need-th largest key (keys are distinct, need >= 1)
// ---------------------------------------------------------------------------
// Warp version over a warp's candidates: keys [0, min(n, kWcap)) in shared
// memory (buf), the rest in its global overflow area (gov); n <= kWcap + kWovf.
// bins: 256 u32 of this warp.
__device__ __forceinline__ uint64_t wkey(const uint64_t* buf, const uint64_t* gov, int i) {
  return i < kWcap ? buf[i] : __ldcg(reinterpret_cast<const unsigned long long*>(gov + (i - kWcap)));
}
// With min_shift > 0 the walk stops once the bits above min_shift are
// fixed and returns the lowest key of that bucket: a lower bound that keeps
// at least need keys (the bucket's other keys too).
__device__ __forceinline__ uint64_t warp_select(const uint64_t* buf, const uint64_t* gov, int n, int need,
                                                uint32_t* bins, int min_shift = 0) {
  const int lane = threadIdx.x & 31;
  __syncwarp();
  uint64_t kmin = ~0ull, kmax = 0ull;
#pragma unroll 1
  for (int i = lane; i < n; i += 32) {
    const uint64_t k = wkey(buf, gov, i);
    kmin = k < kmin ? k : kmin;
    kmax = k > kmax ? k : kmax;
  }
  kmin = warp_min_u64(kmin);
  kmax = warp_max_u64(kmax);
  if (kmin == kmax) return kmax;
  const int lead = __clzll(static_cast<long long>(kmin ^ kmax));
  int shift = 64 - (lead & ~7);
  uint64_t prefix = shift >= 64 ? 0ull : ((kmax >> shift) << shift);
#pragma unroll 1
  for (int pass = 0; pass < 8; ++pass) {
    shift -= 8;
    for (int b = lane; b < 256; b += 32) bins[b] = 0u;
    __syncwarp();
  #pragma unroll 1
  for (int i = lane; i < n; i += 32) {
      const uint64_t k = wkey(buf, gov, i);
      if (hi_match(k, prefix, shift + 8)) atomicAdd(&bins[static_cast<int>((k >> shift) & 255u)], 1u);
    }
    __syncwarp();
    // lane L owns buckets 255 - 8L - j, j = 0..7 (descending)
    uint32_t c[8];
    uint32_t ls = 0;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      c[j] = bins[255 - 8 * lane - j];
      ls += c[j];
    }
    uint32_t inc = ls;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const uint32_t t = __shfl_up_sync(0xffffffffu, inc, o);
      if (lane >= o) inc += t;
    }
    const uint32_t exc = inc - ls;
    const bool hit = exc < static_cast<uint32_t>(need) && inc >= static_cast<uint32_t>(need);
    const int hl = __ffs(__ballot_sync(0xffffffffu, hit)) - 1;
    int bucket = 0;
    uint32_t above = 0, cntb = 0;
    if (lane == hl) {
      uint32_t run = exc;
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        if (cntb == 0 && run + c[j] >= static_cast<uint32_t>(need)) {
          bucket = 255 - 8 * lane - j;
          above = run;
          cntb = c[j];
        }
        run += c[j];
      }
    }
    bucket = __shfl_sync(0xffffffffu, bucket, hl);
    above = __shfl_sync(0xffffffffu, above, hl);
    cntb = __shfl_sync(0xffffffffu, cntb, hl);
    __syncwarp();
    prefix |= static_cast<uint64_t>(bucket) << shift;
    need -= static_cast<int>(above);
    if (shift <= min_shift) return prefix;
    if (cntb == 1u || static_cast<uint32_t>(need) == cntb) {
      uint64_t mn = ~0ull;
#pragma unroll 1
      for (int i = lane; i < n; i += 32) {
        const uint64_t k = wkey(buf, gov, i);
        if (hi_match(k, prefix, shift) && k < mn) mn = k;
      }
      return warp_min_u64(mn);
    }
  }
  return prefix;
}

// The need-th largest value among the 512 f32 logits of a warp's slice in
// shared memory (NaN and -inf ignored; -inf when fewer than need remain),
// by a radix select on the ordered bits; bins: 256 u32 of this warp.
__device__ __noinline__ float warp_kth_stage(const float* slice, int need, uint32_t* bins) {
  const int lane = threadIdx.x & 31;
  float v[4][4];
#pragma unroll
  for (int q = 0; q < 4; ++q)
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const float x = slice[(q * 4 + k) * 32 + lane];
      v[q][k] = (x != x) ? RL_NEG_INF : x;
    }
  int cnt = 0;
  uint32_t kmin = 0xffffffffu, kmax = 0u;
#pragma unroll
  for (int q = 0; q < 4; ++q)
#pragma unroll
    for (int k = 0; k < 4; ++k)
      if (v[q][k] > RL_NEG_INF) {
        const uint32_t u = ord_key(v[q][k]);
        ++cnt;
        kmin = min(kmin, u);
        kmax = max(kmax, u);
      }
  if (warp_sum_i(cnt) < need) return RL_NEG_INF;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    kmin = min(kmin, __shfl_xor_sync(0xffffffffu, kmin, o));
    kmax = max(kmax, __shfl_xor_sync(0xffffffffu, kmax, o));
  }
  if (kmin == kmax) return ord_key_inv(kmax);
  const int lead = __clz(static_cast<int>(kmin ^ kmax));
  int shift = 32 - (lead & ~7);
  uint32_t prefix = shift >= 32 ? 0u : ((kmax >> shift) << shift);
  for (int pass = 0; pass < 4; ++pass) {
    shift -= 8;
    for (int b = lane; b < 256; b += 32) bins[b] = 0u;
    __syncwarp();
#pragma unroll
    for (int q = 0; q < 4; ++q)
#pragma unroll
      for (int k = 0; k < 4; ++k)
        if (v[q][k] > RL_NEG_INF) {
          const uint32_t u = ord_key(v[q][k]);
          if (shift + 8 >= 32 || ((u ^ prefix) >> (shift + 8)) == 0u) atomicAdd(&bins[(u >> shift) & 255u], 1u);
        }
    __syncwarp();
    uint32_t c[8];
    uint32_t ls = 0;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      c[j] = bins[255 - 8 * lane - j];
      ls += c[j];
    }
    uint32_t inc = ls;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const uint32_t t = __shfl_up_sync(0xffffffffu, inc, o);
      if (lane >= o) inc += t;
    }
    const uint32_t exc = inc - ls;
    const bool hit = exc < static_cast<uint32_t>(need) && inc >= static_cast<uint32_t>(need);
    const int hl = __ffs(__ballot_sync(0xffffffffu, hit)) - 1;
    int bucket = 0;
    uint32_t above = 0, cntb = 0;
    if (lane == hl) {
      uint32_t run = exc;
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        if (cntb == 0 && run + c[j] >= static_cast<uint32_t>(need)) {
          bucket = 255 - 8 * lane - j;
          above = run;
          cntb = c[j];
        }
        run += c[j];
      }
    }
    bucket = __shfl_sync(0xffffffffu, bucket, hl);
    above = __shfl_sync(0xffffffffu, above, hl);
    cntb = __shfl_sync(0xffffffffu, cntb, hl);
    __syncwarp();
    prefix |= static_cast<uint32_t>(bucket) << shift;
    need -= static_cast<int>(above);
    if (shift == 0) return ord_key_inv(prefix);
    if (static_cast<uint32_t>(need) == cntb) {
      uint32_t mn = 0xffffffffu;
#pragma unroll
      for (int q = 0; q < 4; ++q)
#pragma unroll
        for (int k = 0; k < 4; ++k)
          if (v[q][k] > RL_NEG_INF) {
            const uint32_t u = ord_key(v[q][k]);
            if (((u ^ prefix) >> shift) == 0u) mn = min(mn, u);
          }
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) mn = min(mn, __shfl_xor_sync(0xffffffffu, mn, o));
      return ord_key_inv(mn);
    }
  }
  return ord_key_inv(prefix);
}

// Keeps the keys >= T of a warp's buffer buf[0..n) (n <= kWcap), in order,
// compacted to the front; returns their count.
__device__ __forceinline__ int warp_filter(uint64_t* buf, int n, uint64_t T) {
  const int lane = threadIdx.x & 31;
  int pos = 0;
#pragma unroll 1
  for (int i0 = 0; i0 < n; i0 += 32) {
    const int i = i0 + lane;
    const uint64_t k = i < n ? buf[i] : 0ull;
    const bool kf = i < n && k >= T;
    const unsigned b = __ballot_sync(0xffffffffu, kf);
    __syncwarp();
    if (kf) buf[pos + __popc(b & ((1u << lane) - 1u))] = k;
    pos += __popc(b);
  }
  __syncwarp();
  return pos;
}

// Keys >= T among a warp's n candidates (shared buffer and overflow).
__device__ __forceinline__ int warp_count_ge(const uint64_t* buf, const uint64_t* gov, int n, uint64_t T) {
  const int lane = threadIdx.x & 31;
  __syncwarp();
  int c = 0;
#pragma unroll 1
  for (int i = lane; i < n; i += 32) c += wkey(buf, gov, i) >= T ? 1 : 0;
  return warp_sum_i(c);
}
// Moves the keys >= T of a warp's n candidates to buf[0..), in order; the
// caller has checked that they fit in buf.
__device__ __forceinline__ void warp_keep_ge(uint64_t* buf, const uint64_t* gov, int n, uint64_t T) {
  const int lane = threadIdx.x & 31;
  int pos = 0;
#pragma unroll 1
  for (int i0 = 0; i0 < n; i0 += 32) {
    const int i = i0 + lane;
    const uint64_t k = i < n ? wkey(buf, gov, i) : 0ull;
    const bool kf = i < n && k >= T;
    const unsigned b = __ballot_sync(0xffffffffu, kf);
    __syncwarp();
    if (kf) buf[pos + __popc(b & ((1u << lane) - 1u))] = k;
    pos += __popc(b);
  }
  __syncwarp();
}

// Descending bitonic sort of a warp's buffer buf[0..n) (n <= kN) in place;
// positions n..pow2 are padded with 0 and not read back.
__device__ __forceinline__ void warp_sort_desc(uint64_t* buf, int n) {
  const int lane = threadIdx.x & 31;
  int P = 1;
  while (P < n) P <<= 1;
  for (int i = n + lane; i < P; i += 32) buf[i] = 0ull;
  __syncwarp();
  for (int k = 2; k <= P; k <<= 1) {
    for (int j = k >> 1; j > 0; j >>= 1) {
      for (int i = lane; i < P; i += 32) {
        const int l = i ^ j;
        if (l > i) {
          const uint64_t x = buf[i], y = buf[l];
          const bool desc = (i & k) == 0;
          if (desc ? (x < y) : (x > y)) {
            buf[i] = y;
            buf[l] = x;
          }
        }
      }
      __syncwarp();
    }
  }
}

// The need-th largest value among the kCE f32 logits of a stage (NaN and
// -inf ignored; -inf when fewer than need remain), by the consumer threads:
// a radix select on the ordered bits; bins: 256 u32.
// E: f32 or bf16 stage; excl (nullable): kCE bits, set for the positions to
// leave out (a bf16 stage holds raw values, so its history ids are skipped).
template <typename E>
__device__ __noinline__ float block_kth_stage(const E* stg, int need, uint32_t* bins, Red* rs, Ctl* ctl,
                                              const uint32_t* excl) {
  const int tid = threadIdx.x;
  constexpr int R = kCE / kConsumers;
  uint32_t u[R];
  int cnt = 0;
  uint32_t kmin = 0xffffffffu, kmax = 0u;
#pragma unroll
  for (int r = 0; r < R; ++r) {
    const int e = r * kConsumers + tid;
    const float x = to_f32<E>(stg[e]);
    const bool ok = x > RL_NEG_INF && !(excl && ((excl[e >> 5] >> (e & 31)) & 1u));  // false for NaN
    u[r] = ok ? ord_key(x) : 0u;
    if (ok) {
      ++cnt;
      kmin = min(kmin, u[r]);
      kmax = max(kmax, u[r]);
    }
  }
  if (csum_i(cnt, rs) < need) return RL_NEG_INF;
  kmin = static_cast<uint32_t>(cmin_u64(kmin, rs));
  kmax = static_cast<uint32_t>(cmax_u64(kmax, rs));
  if (kmin == kmax) return ord_key_inv(kmax);
  const int lead = __clz(static_cast<int>(kmin ^ kmax));
  int shift = 32 - (lead & ~7);
  uint32_t prefix = shift >= 32 ? 0u : ((kmax >> shift) << shift);
#pragma unroll 1
  for (int pass = 0; pass < 4; ++pass) {
    shift -= 8;
    bins[tid] = 0u;
    cbar();
#pragma unroll
    for (int r = 0; r < R; ++r)
      if (u[r] != 0u && (shift + 8 >= 32 || ((u[r] ^ prefix) >> (shift + 8)) == 0u))
        atomicAdd(&bins[(u[r] >> shift) & 255u], 1u);
    cbar();
    const uint32_t c = bins[255 - tid];
    const uint32_t inc = cscan_u32(c, rs);
    const uint32_t exc = inc - c;
    if (exc < static_cast<uint32_t>(need) && inc >= static_cast<uint32_t>(need)) {
      ctl->sel_bucket = 255 - tid;
      ctl->sel_above = exc;
      ctl->sel_cnt = c;
    }
    cbar();
    const int bucket = ctl->sel_bucket;
    const uint32_t above = ctl->sel_above, cntb = ctl->sel_cnt;
    cbar();
    prefix |= static_cast<uint32_t>(bucket) << shift;
    need -= static_cast<int>(above);
    if (shift == 0) return ord_key_inv(prefix);
    if (static_cast<uint32_t>(need) == cntb) {
      uint32_t mn = 0xffffffffu;
#pragma unroll
      for (int r = 0; r < R; ++r)
        if (u[r] != 0u && ((u[r] ^ prefix) >> shift) == 0u) mn = min(mn, u[r]);
      return ord_key_inv(static_cast<uint32_t>(cmin_u64(mn, rs)));
    }
  }
  return ord_key_inv(prefix);
}

// Keeps the top `keep` keys of a warp's candidates (n > keep) in buf[0, keep);
// returns the bound (the keep-th largest key). The kept keys are written in
// 32-key windows after the window has been read, so the in-place move is safe.
__device__ __forceinline__ uint64_t warp_compact(uint64_t* buf, const uint64_t* gov, int n, int keep,
                                                 uint32_t* bins, int min_shift = 0) {
  const int lane = threadIdx.x & 31;
  const uint64_t T = warp_select(buf, gov, n, keep, bins, min_shift);
  int pos = 0;
#pragma unroll 1
  for (int i0 = 0; i0 < n; i0 += 32) {
    const int i = i0 + lane;
    const uint64_t k = i < n ? wkey(buf, gov, i) : 0ull;
    const bool kf = i < n && k >= T;
    const unsigned b = __ballot_sync(0xffffffffu, kf);
    __syncwarp();
    if (kf) buf[pos + __popc(b & ((1u << lane) - 1u))] = k;
    pos += __popc(b);
  }
  __syncwarp();
  return T;
}

// Consumer-group version over segments of keys: segment s holds cnts[s]
// valid keys at base[s * seg_size ...]. G: the keys are in global memory
// written by other CTAs (read through L2).
template <bool G>
__device__ __forceinline__ uint64_t ldkey(const uint64_t* p) {
  if constexpr (G) {
    return __ldcg(reinterpret_cast<const unsigned long long*>(p));
  } else {
    return *p;
  }
}
template <bool G>
__device__ uint64_t block_select(const uint64_t* base, int nsegs, int seg_size, const int* cnts, int need,
                                 uint32_t* bins, Red* rs, Ctl* ctl) {
  const int tid = threadIdx.x;
  const int slots = nsegs * seg_size;
  uint64_t kmin = ~0ull, kmax = 0ull;
  for (int f = tid; f < slots; f += kConsumers) {
    const int s = f / seg_size;
    if (f - s * seg_size < cnts[s]) {
      const uint64_t k = ldkey<G>(base + f);
      kmin = k < kmin ? k : kmin;
      kmax = k > kmax ? k : kmax;
    }
  }
  kmin = cmin_u64(kmin, rs);
  kmax = cmax_u64(kmax, rs);
  if (kmin == kmax) return kmax;
  const int lead = __clzll(static_cast<long long>(kmin ^ kmax));
  int shift = 64 - (lead & ~7);
  uint64_t prefix = shift >= 64 ? 0ull : ((kmax >> shift) << shift);
  for (int pass = 0; pass < 8; ++pass) {
    shift -= 8;
    bins[tid] = 0u;
    cbar();
    for (int f = tid; f < slots; f += kConsumers) {
      const int s = f / seg_size;
      if (f - s * seg_size < cnts[s]) {
        const uint64_t k = ldkey<G>(base + f);
        if (hi_match(k, prefix, shift + 8)) atomicAdd(&bins[static_cast<int>((k >> shift) & 255u)], 1u);
      }
    }
    cbar();
    const uint32_t c = bins[255 - tid];
    const uint32_t inc = cscan_u32(c, rs);
    const uint32_t exc = inc - c;
    if (exc < static_cast<uint32_t>(need) && inc >= static_cast<uint32_t>(need)) {
      ctl->sel_bucket = 255 - tid;
      ctl->sel_above = exc;
      ctl->sel_cnt = c;
    }
    cbar();
    const int bucket = ctl->sel_bucket;
    const uint32_t above = ctl->sel_above, cntb = ctl->sel_cnt;
    cbar();
    prefix |= static_cast<uint64_t>(bucket) << shift;
    need -= static_cast<int>(above);
    if (shift == 0) return prefix;
    if (cntb == 1u || static_cast<uint32_t>(need) == cntb) {
      uint64_t mn = ~0ull;
      for (int f = tid; f < slots; f += kConsumers) {
        const int s = f / seg_size;
        if (f - s * seg_size < cnts[s]) {
          const uint64_t k = ldkey<G>(base + f);
          if (hi_match(k, prefix, shift) && k < mn) mn = k;
        }
      }
      return cmin_u64(mn, rs);
    }
  }
  return prefix;
}

// Gathers the keys >= T of the segments into out (<= kN) and sorts them.
template <bool G>
__device__ int gather_sorted(const uint64_t* base, int nsegs, int seg_size, const int* cnts, uint64_t T,
                             uint64_t* out, Ctl* ctl) {
  const int tid = threadIdx.x;
  if (tid == 0) ctl->cnt = 0;
  cbar();
  const int slots = nsegs * seg_size;
  for (int f = tid; f < slots; f += kConsumers) {
    const int s = f / seg_size;
    if (f - s * seg_size < cnts[s]) {
      const uint64_t k = ldkey<G>(base + f);
      if (k >= T) {
        const int i = atomicAdd(&ctl->cnt, 1);
        if (i < kN) out[i] = k;
      }
    }
  }
  cbar();
  const int n = min(ctl->cnt, kN);
  cbar();
  csort_desc(out, n, kN);
  return n;
}

// ---------------------------------------------------------------------------
// Chunk geometry shared by the copy warp and the consumers
// ---------------------------------------------------------------------------
template <typename E>
__device__ __forceinline__ uint32_t chunk_bytes(const SpecArgs& a, int row, int start, int len) {
  const E* src = reinterpret_cast<const E*>(a.logits) + static_cast<int64_t>(row) * a.ld + start;
  if (reinterpret_cast<uintptr_t>(src) & 15u) return 0u;
  return static_cast<uint32_t>(len * static_cast<int>(sizeof(E))) & ~15u;
}
__device__ __forceinline__ uint32_t mask_bytes(const SpecArgs& a, int row, int start, int len) {
  if (!a.mask) return 0u;
  const uint32_t* src = a.mask + static_cast<int64_t>(row) * a.mask_stride + (start >> 5);
  if (reinterpret_cast<uintptr_t>(src) & 15u) return 0u;
  return (static_cast<uint32_t>((len + 31) >> 5) * 4u) & ~15u;
}

// ---------------------------------------------------------------------------
// Copy warp
// ---------------------------------------------------------------------------
// Bulk copy with an L2 eviction-priority hint (rows the finisher may re-read
// are kept in L2 with evict_last).
__device__ __forceinline__ void bulk_g2s_hint(void* dst_smem, const void* src_gmem, uint32_t bytes, uint64_t* bar,
                                              uint64_t policy) {
  asm volatile(
      "cp.async.bulk.shared::cta.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1], %2, [%3], %4;" ::"r"(
          smem_u32(dst_smem)),
      "l"(src_gmem), "r"(bytes), "r"(smem_u32(bar)), "l"(policy)
      : "memory");
}
__device__ __forceinline__ uint64_t evict_last_policy() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_last.b64 %0, 1.0;" : "=l"(p));
  return p;
}
__device__ __forceinline__ uint64_t evict_first_policy() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
  return p;
}
template <typename E>
__device__ __noinline__ void producer_loop(const SpecArgs& a) {
  if ((threadIdx.x & 31) != 0) return;
  const Smem sm = smem_map();
  const int S = spec_chunks(a.V);
  const uint64_t keep_l2 = evict_last_policy();
  const uint64_t drop_l2 = evict_first_policy();
  int seq = 0;
  bool ok = true;
  for (int item = blockIdx.x; item < a.nitems && ok; item += gridDim.x) {
    const int row = item / a.nseg;
    const int seg = item - row * a.nseg;
    const int c0 = seg * a.cps, c1 = min(S, c0 + a.cps);
    // rows on the histogram path may be re-read by their finisher
    const float T = a.params[row].temperature;
    const int tk = a.params[row].top_k;
    const bool hint = (fabsf(T) < RL_POS_INF) && T > 0.0f && !(tk > 0 && tk <= kN);
    for (int c = c0; c < c1; ++c, ++seq) {
      const int s = seq % kNS;
      const uint32_t ph = static_cast<uint32_t>((seq / kNS) & 1);
      if (!mbar_wait(&sm.empty[s], ph ^ 1u, kWaitBudget) || *reinterpret_cast<volatile int*>(&sm.ctl->abort)) {
        atomicExch(&sm.ctl->abort, 1);
        ok = false;
        break;
      }
      const int start = c * kCE;
      const int len = min(kCE, a.V - start);
      const uint32_t db = chunk_bytes<E>(a, row, start, len);
      const uint32_t mb = mask_bytes(a, row, start, len);
      mbar_expect_tx(&sm.full[s], db + mb);
      if (db) {
        const E* src = reinterpret_cast<const E*>(a.logits) + static_cast<int64_t>(row) * a.ld + start;
        // rows that are read once leave L2 first, so that the histogram
        // rows stay for their finisher's re-read
        bulk_g2s_hint(sm.stage + s * kStageBytes, src, db, &sm.full[s], hint ? keep_l2 : drop_l2);
      }
      if (mb)
        bulk_g2s(sm.maskst + s * kMaskWords, a.mask + static_cast<int64_t>(row) * a.mask_stride + (start >> 5), mb,
                 &sm.full[s]);
    }
  }
  if (!ok) {
    // never leave with a copy still landing in this CTA's shared memory
    for (int i = max(0, seq - kNS); i < seq; ++i)
      mbar_wait(&sm.full[i % kNS], static_cast<uint32_t>((i / kNS) & 1), kWaitBudget);
  }
}

// ---------------------------------------------------------------------------
// Row-preparation warp
// ---------------------------------------------------------------------------
// The row's history ids in [lo, hi) (row-local ids), in history order, into
// tab. Returns the count. PRE: the row's first 512 entries are in pre[]
// already (lane l holds entries r * 32 + l).
template <bool PRE>
__device__ __forceinline__ int gather_history_impl(const SpecArgs& a, int row, int hl, uint32_t* tab, int lo, int hi,
                                                   const int (&pre)[16]) {
  const int lane = threadIdx.x & 31;
  const int32_t* h = a.hist + static_cast<int64_t>(row) * a.hist_stride;
  int n = 0;
  for (int g0 = 0; g0 < hl; g0 += 512) {
    // 16 loads in flight per lane: a 512-token history in one round trip
    int ids[16];
#pragma unroll
    for (int r = 0; r < 16; ++r) {
      const int i = g0 + r * 32 + lane;
      ids[r] = (PRE && g0 == 0) ? pre[r] : (i < hl ? __ldg(h + i) : -1);
    }
#pragma unroll
    for (int r = 0; r < 16; ++r) {
      const int i = g0 + r * 32 + lane;
      const int id = ids[r] - a.vocab_offset;
      const bool ok = i < hl && id >= lo && id < hi;
      const unsigned b = __ballot_sync(0xffffffffu, ok);
      if (ok) tab[n + __popc(b & ((1u << lane) - 1u))] = static_cast<uint32_t>(id);
      n += __popc(b);
    }
  }
  __syncwarp();
  return n;
}
__device__ __noinline__ int gather_history(const SpecArgs& a, int row, int hl, uint32_t* tab, int lo, int hi) {
  const int none[16] = {};
  return gather_history_impl<false>(a, row, hl, tab, lo, hi, none);
}

// Consumers: sorts the raw history ids tab[0, n) (n <= kHmax) with the
// register bitonic sort (64-bit keys ~id in the radix area, descending =
// ascending ids) and packs (id << 11) | count like sort_table.
__device__ __noinline__ void block_sort_table(uint32_t* tab, int n) {
  const Smem sm = smem_map();
  const int tid = threadIdx.x;
  // Fast path: one counting pass into at most kCW * 256 id ranges, then
  // each range (a few entries) put in order by one thread. A range with
  // more than 64 entries (a history that repeats a few ids many times)
  // takes the bitonic sort below instead.
  {
    constexpr int kBuckets = kCW * 256;
    constexpr int BPT = kBuckets / kConsumers;
    uint32_t mx = 0u;
    for (int i = tid; i < n; i += kConsumers) mx = max(mx, tab[i]);
    mx = static_cast<uint32_t>(cmax_u64(mx, sm.red));
    int sh = 0;
    while ((mx >> sh) >= static_cast<uint32_t>(kBuckets)) ++sh;
    const int nb = static_cast<int>(mx >> sh) + 1;
    uint32_t* cnt = sm.radix;                               // [nb] range sizes, then starts
    uint32_t* tmp = reinterpret_cast<uint32_t*>(sm.wbuf);  // [kHmax] ids, [kHmax] ranks
    for (int i = tid; i < nb; i += kConsumers) cnt[i] = 0u;
    cbar();
    for (int i = tid; i < n; i += kConsumers) {
      const uint32_t id = tab[i];
      tmp[i] = id;
      tmp[kHmax + i] = atomicAdd(&cnt[id >> sh], 1u);
    }
    cbar();
    uint32_t loc[BPT];
    uint32_t sum = 0u, big = 0u;
#pragma unroll
    for (int r = 0; r < BPT; ++r) {
      const int b = tid * BPT + r;
      loc[r] = b < nb ? cnt[b] : 0u;
      sum += loc[r];
      big = max(big, loc[r]);
    }
    if (cmax_u64(big, sm.red) <= 64u) {
      uint32_t run = cscan_u32(sum, sm.red) - sum;
      uint32_t st[BPT];
#pragma unroll
      for (int r = 0; r < BPT; ++r) {
        const int b = tid * BPT + r;
        st[r] = run;
        if (b < nb) cnt[b] = run;
        run += loc[r];
      }
      cbar();
      for (int i = tid; i < n; i += kConsumers) {
        const uint32_t id = tmp[i];
        tab[cnt[id >> sh] + tmp[kHmax + i]] = id;
      }
      cbar();
      // insertion sort of this thread's ranges (sizes <= 64, mostly 0 or 1)
#pragma unroll 1
      for (int r = 0; r < BPT; ++r) {
        uint32_t* t = tab + st[r];
        for (int i = 1; i < static_cast<int>(loc[r]); ++i) {
          const uint32_t x = t[i];
          int j = i - 1;
          while (j >= 0 && t[j] > x) {
            t[j + 1] = t[j];
            --j;
          }
          t[j + 1] = x;
        }
      }
      cbar();
    } else {
      uint64_t* k64 = reinterpret_cast<uint64_t*>(sm.radix);
      for (int i = tid; i < n; i += kConsumers) k64[i] = static_cast<uint64_t>(~tab[i]);
      int P = 1;
      while (P < n) P <<= 1;
      cbar();
      csort_desc(k64, n, P);
#pragma unroll
      for (int r = 0; r < kHmax / kConsumers; ++r) {
        const int p = tid + r * kConsumers;
        if (p < n) tab[p] = ~static_cast<uint32_t>(k64[p]);
      }
      cbar();
    }
  }
  uint32_t packed[kHmax / kConsumers];
#pragma unroll
  for (int r = 0; r < kHmax / kConsumers; ++r) {
    const int p = tid + r * kConsumers;
    packed[r] = 0u;
    if (p < n) {
      const uint32_t id = tab[p];
      uint32_t c = 0u;
      if (p == 0 || tab[p - 1] != id) {
        int q = p + 1;
        while (q < n && tab[q] == id) ++q;
        c = static_cast<uint32_t>(min(q - p, 2047));
      }
      packed[r] = (id << 11) | c;
    }
  }
  cbar();
#pragma unroll
  for (int r = 0; r < kHmax / kConsumers; ++r) {
    const int p = tid + r * kConsumers;
    if (p < n) tab[p] = packed[r];
  }
  cbar();
}

// Consumers: sorts the slot's raw history ids and packs them as
// (id << 11) | count -- the first copy of an id carries its count, later
// copies count 0 (skipped).
__device__ __noinline__ void sort_table(uint32_t* tab, int n) {
  const int tid = threadIdx.x;
  int P = 1;
  while (P < n) P <<= 1;
  for (int i = n + tid; i < P; i += kConsumers) tab[i] = 0x7fffffffu;
  cbar();
  for (int k = 2; k <= P; k <<= 1) {
    for (int j = k >> 1; j > 0; j >>= 1) {
      for (int i = tid; i < P; i += kConsumers) {
        const int l = i ^ j;
        if (l > i) {
          const uint32_t x = tab[i], y = tab[l];
          const bool up = (i & k) == 0;
          if (up ? (x > y) : (x < y)) {
            tab[i] = y;
            tab[l] = x;
          }
        }
      }
      cbar();
    }
  }
  uint32_t packed[kHmax / kConsumers];
#pragma unroll
  for (int r = 0; r < kHmax / kConsumers; ++r) {
    const int p = tid + r * kConsumers;
    packed[r] = 0u;
    if (p < n) {
      const uint32_t id = tab[p];
      uint32_t c = 0u;
      if (p == 0 || tab[p - 1] != id) {
        int q = p + 1;
        while (q < n && tab[q] == id) ++q;
        c = static_cast<uint32_t>(min(q - p, 2047));
      }
      packed[r] = (id << 11) | c;
    }
  }
  cbar();
#pragma unroll
  for (int r = 0; r < kHmax / kConsumers; ++r) {
    const int p = tid + r * kConsumers;
    if (p < n) tab[p] = packed[r];
  }
  cbar();
}

// Cursor start: the number of table entries with id < lo.
__device__ __forceinline__ int tab_lower_bound(const uint32_t* tab, int ntab, int lo) {
  const int lane = threadIdx.x & 31;
  int c = 0;
  for (int j0 = 0; j0 < ntab; j0 += 32) {
    const int j = j0 + lane;
    const bool lt = j < ntab && static_cast<int>(tab[j] >> 11) < lo;
    c += __popc(__ballot_sync(0xffffffffu, lt));
  }
  return c;
}

// The metadata of an item and the raw (unsorted) history table of its row,
// written by one warp. defer_tab: the table is not gathered; ntab holds minus
// the history length to gather when a re-read of the row needs the table
// (lazy_table).
__device__ __noinline__ void build_meta(const SpecArgs& a, int item, ItemMeta& mt, uint32_t* tab, bool defer_tab) {
  const int lane = threadIdx.x & 31;
  const int S = spec_chunks(a.V);
  const int row = item / a.nseg;
  const int seg = item - row * a.nseg;
  // every global read of the row issued up front: parameters, the first
  // 512 history entries (entries past hist_len are read but not used) and
  // the allowed mask, in one round trip
  const rl_row_params prm = a.params[row];
  const float u = a.uniforms[row];
  const int hl_raw = a.hist ? a.hist_len[row] : 0;
  int pre[16];
  {
    const int hs = a.hist ? min(a.hist_stride, kHmax) : 0;
    const int32_t* h = a.hist + static_cast<int64_t>(row) * a.hist_stride;
#pragma unroll
    for (int r = 0; r < 16; ++r) {
      const int i = r * 32 + lane;
      pre[r] = (!defer_tab && i < hs) ? __ldg(h + i) : -1;
    }
  }
  const float T = prm.temperature;
  int mode;
  if (!(fabsf(T) < RL_POS_INF) || !(T > 0.0f)) mode = 0;  // greedy; a non-finite T is reported at the end
  else if (prm.top_k > 0 && prm.top_k <= kN) mode = 1;
  else mode = 2;
  // allowed-mask flag: an empty allowed set means every id is allowed
  int mask_on = 0;
  if (a.mask) {
    const uint32_t* mrow = a.mask + static_cast<int64_t>(row) * a.mask_stride;
    const int nw = (a.V + 31) >> 5;
    const int nfull = a.V >> 5;  // words with no bit past the row end
    uint32_t any = 0u;
    if ((reinterpret_cast<uintptr_t>(mrow) & 15u) == 0) {
      // 16-byte loads, eight in flight per lane
      const uint4* m4 = reinterpret_cast<const uint4*>(mrow);
      const int n4 = nfull >> 2;
      for (int w0 = 0; w0 < n4; w0 += 256) {
        uint4 q[8];
#pragma unroll
        for (int r = 0; r < 8; ++r) {
          const int w = w0 + r * 32 + lane;
          q[r] = w < n4 ? __ldg(m4 + w) : make_uint4(0u, 0u, 0u, 0u);
        }
#pragma unroll
        for (int r = 0; r < 8; ++r) any |= q[r].x | q[r].y | q[r].z | q[r].w;
      }
      for (int w = (n4 << 2) + lane; w < nw; w += 32) {
        uint32_t bits = __ldg(mrow + w);
        const int rem = a.V - w * 32;
        if (rem < 32) bits &= (1u << rem) - 1u;
        any |= bits;
      }
    } else {
      for (int w0 = 0; w0 < nw; w0 += 256) {
        uint32_t q[8];
#pragma unroll
        for (int r = 0; r < 8; ++r) {
          const int w = w0 + r * 32 + lane;
          q[r] = w < nw ? __ldg(mrow + w) : 0u;
          const int rem = a.V - w * 32;
          if (w < nw && rem < 32) q[r] &= (1u << rem) - 1u;
        }
#pragma unroll
        for (int r = 0; r < 8; ++r) any |= q[r];
      }
    }
    mask_on = __any_sync(0xffffffffu, any != 0u) ? 1 : 0;
  }
  // history table (only when the penalties are not the identity)
  const bool pen = !(prm.repeat_penalty == 1.0f && prm.frequency_penalty == 0.0f && prm.presence_penalty == 0.0f);
  int ntab = 0;
  if (a.hist && pen) {
    const int hl = max(0, min(hl_raw, min(a.hist_stride, kHmax)));
    if (hl > 0) ntab = defer_tab ? -hl : gather_history_impl<true>(a, row, hl, tab, 0, a.V, pre);
  }
  // Histogram window depth W (nats below the anchor): the mass below it is
  // at most V e^-W of the row max, kept under a quarter of the tail mass
  // that the top-p cutoff leaves (or, without a cutoff, that the draw
  // leaves). A draw that still lands below the window is resolved by the
  // exact radix walk.
  int wbins = kNB - 1;
  if (mode == 2 && prm.top_k <= 0) {
    const double p = static_cast<double>(prm.top_p);
    const double tail = (p < 1.0) ? 1.0 - p : 1.0 - static_cast<double>(u);
    if (tail > 0.0 && p > 0.0) {
      const double W = log(4.0 * static_cast<double>(a.V) / tail) + 1.0;
      wbins = min(wbins, kHead + max(64, static_cast<int>(ceil(W * kRbin))));
    }
  }
  if (lane == 0) {
    mt.item = item;
    mt.row = row;
    mt.seg = seg;
    mt.c0 = seg * a.cps;
    mt.c1 = min(S, mt.c0 + a.cps);
    mt.mode = mode;
    mt.nkeep = mode == 1 ? prm.top_k : kN;
    // bins count logits too where a position is needed: top_k beyond the
    // list, or a debug launch reporting the cutoff position
    mt.need_count = (mode == 2 && (prm.top_k > 0 || a.list_cut != nullptr)) ? 1 : 0;
    mt.mask_on = mask_on;
    mt.ntab = ntab;
    mt.wbins = wbins;
    mt.top_k = prm.top_k;
    mt.top_p = prm.top_p;
    mt.u = u;
    mt.rp = prm.repeat_penalty;
    mt.pres = prm.presence_penalty;
    mt.freq = prm.frequency_penalty;
    mt.rt = make_rowt(mode == 0 ? 1.0f : T);
    mt.rt.T = T;  // the raw temperature (greedy rows check it at the end)
  }
}

template <typename E, bool SPLIT>
__device__ __noinline__ void meta_loop(const SpecArgs& a) {
  const Smem sm = smem_map();
  const int lane = threadIdx.x & 31;
  const int S = spec_chunks(a.V);
  int cseq = 0;
  for (int mseq = 0;; ++mseq) {
    const int slot = mseq & 1;
    ItemMeta& mt = sm.meta[slot];
    const int item = blockIdx.x + mseq * gridDim.x;
    if (item >= a.nitems) return;
    if (!mbar_wait(&sm.mempty[slot], static_cast<uint32_t>(((mseq >> 1) & 1) ^ 1), kWaitBudget) ||
        *reinterpret_cast<volatile int*>(&sm.ctl->abort)) {
      if (lane == 0) atomicExch(&sm.ctl->abort, 1);
      return;
    }
    uint32_t* tab = sm.tab + slot * kHmax;
    build_meta(a, item, mt, tab, false);
    __syncwarp();
    if (lane == 0) mbar_arrive(&sm.mfull[slot]);
    if constexpr (SPLIT) {
      // each chunk of the item: penalties patched into the stage (f32 slices
      // wholly in the stage; the rest is penalised in registers by the
      // consumers), then released to the consumers
      const int row = item / a.nseg;
      const int seg = item - row * a.nseg;
      const int c0 = seg * a.cps, c1 = min(S, c0 + a.cps);
      const int ntab = mt.ntab;
      const float rp = mt.rp, fq = mt.freq, pr = mt.pres;
      const bool row_al = (reinterpret_cast<uintptr_t>(reinterpret_cast<const E*>(a.logits) +
                                                       static_cast<int64_t>(row) * a.ld) & 15u) == 0;
      bool tab_ok = true;
      if (sizeof(E) == 4 && ntab > 0 && row_al) {
        // the consumers sort the table; wait (bounded) for their signal
        const long long t0 = clock64();
        while (*reinterpret_cast<volatile int*>(&sm.ctl->tab_seq) != mseq + 1) {
          if (clock64() - t0 > kWaitBudget || *reinterpret_cast<volatile int*>(&sm.ctl->abort)) {
            tab_ok = false;
            break;
          }
          __nanosleep(128);  // leave the issue slots to the sorting warps
        }
        __syncwarp();
        __threadfence_block();
      }
      if (!tab_ok) {
        if (lane == 0) atomicExch(&sm.ctl->abort, 1);
        return;
      }
      int hp = ntab > 0 ? tab_lower_bound(tab, ntab, c0 * kCE) : 0;
      for (int c = c0; c < c1; ++c, ++cseq) {
        const int s = cseq % kNS;
        if (!mbar_wait(&sm.full[s], static_cast<uint32_t>((cseq / kNS) & 1), kWaitBudget)) {
          if (lane == 0) atomicExch(&sm.ctl->abort, 1);
          return;
        }
        if (sizeof(E) == 4 && ntab > 0 && row_al) {
          const int start = c * kCE;
          const int len = min(kCE, a.V - start);
          const int nfast = ((len * 4) & ~15) / 4;
          const int hi = start + (nfast / kSlice) * kSlice;  // whole slices in the stage
          float* f = reinterpret_cast<float*>(sm.stage + s * kStageBytes);
          bool wrote = false;
          while (true) {
            const int j = hp + lane;
            const uint32_t ent = j < ntab ? tab[j] : 0xffffffffu;
            const int id = static_cast<int>(ent >> 11);
            const bool below = j < ntab && id < hi;
            if (below && id >= start && (ent & 2047u) != 0u) {
              f[id - start] = pen_value(f[id - start], static_cast<int>(ent & 2047u), rp, fq, pr);
              wrote = true;
            }
            const int adv = __popc(__ballot_sync(0xffffffffu, below));
            hp += adv;
            if (adv < 32) break;
          }
          // generic writes ordered before the next bulk copy into this stage
          if (__any_sync(0xffffffffu, wrote)) fence_proxy_async();
          __syncwarp();
        }
        if (lane == 0) mbar_arrive(&sm.ready[s]);
      }
    }
  }
}

// ---------------------------------------------------------------------------
// Consumer side: penalties and row re-reads
// ---------------------------------------------------------------------------
// Penalties of the table entries in [lo, hi) applied to the registers of the
// slice that starts at lo (logit lo + (q*32+lane)*4 + k is v[q][k]); hp is
// the warp's cursor in the table.
__device__ __forceinline__ void pen_regs(float (&v)[4][4], int lo, int hi, const uint32_t* tab, int ntab, int& hp,
                                         const ItemMeta& mt) {
  const int lane = threadIdx.x & 31;
  while (true) {
    const int j = hp + lane;
    const uint32_t ent = j < ntab ? tab[j] : 0xffffffffu;
    const int id = static_cast<int>(ent >> 11);
    const bool below = j < ntab && id < hi;
    const bool mine = below && id >= lo && (ent & 2047u) != 0u;
    unsigned mb = __ballot_sync(0xffffffffu, mine);
    while (mb) {
      const int src = __ffs(mb) - 1;
      mb &= mb - 1u;
      const int e = __shfl_sync(0xffffffffu, id, src) - lo;
      const int cn = __shfl_sync(0xffffffffu, static_cast<int>(ent & 2047u), src);
      if (((e >> 2) & 31) == lane) {
        const int idx = ((e >> 7) << 2) | (e & 3);
        put16(v, idx, pen_value(pick16(v, idx), cn, mt.rp, mt.freq, mt.pres));
      }
    }
    const int adv = __popc(__ballot_sync(0xffffffffu, below));
    hp += adv;
    if (adv < 32) break;
  }
}
// Row re-read: the warp's slice of chunk `start` from global memory,
// penalised and masked (-inf outside the row or disallowed).
// Raw logits of a warp's slice of chunk `start` (-inf past the row end):
// 16-byte vector loads when the chunk is whole and aligned.
template <typename E>
__device__ __forceinline__ void load_slice_raw(const E* rowp, int V, int start, int base, float (&v)[4][4]) {
  const int lane = threadIdx.x & 31;
  const int len = min(kCE, V - start);
  const bool vec = len == kCE && (reinterpret_cast<uintptr_t>(rowp) & 15u) == 0;
  if (vec) {
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      const int el0 = base + (q * 32 + lane) * 4;
      if constexpr (sizeof(E) == 4) {
        const float4 f = __ldcs(reinterpret_cast<const float4*>(rowp + start + el0));
        v[q][0] = f.x;
        v[q][1] = f.y;
        v[q][2] = f.z;
        v[q][3] = f.w;
      } else {
        const uint2 h = __ldcs(reinterpret_cast<const uint2*>(rowp + start + el0));
        v[q][0] = __uint_as_float(h.x << 16);
        v[q][1] = __uint_as_float(h.x & 0xffff0000u);
        v[q][2] = __uint_as_float(h.y << 16);
        v[q][3] = __uint_as_float(h.y & 0xffff0000u);
      }
    }
  } else {
#pragma unroll
    for (int q = 0; q < 4; ++q)
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        const int el = base + (q * 32 + lane) * 4 + k;
        v[q][k] = el < len ? to_f32<E>(__ldcg(rowp + start + el)) : RL_NEG_INF;
      }
  }
}
// Penalties and mask applied to a raw slice (row re-reads).
template <typename E>
__device__ __forceinline__ void finish_slice(const SpecArgs& a, const ItemMeta& mt, const uint32_t* tab, int& hp,
                                             int start, int base, float (&v)[4][4]) {
  const int lane = threadIdx.x & 31;
  const int len = min(kCE, a.V - start);
  if (mt.ntab > 0) pen_regs(v, start + base, start + base + kSlice, tab, mt.ntab, hp, mt);
  if (mt.mask_on) {
    const uint32_t* mrow = a.mask + static_cast<int64_t>(mt.row) * a.mask_stride;
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      const int e0 = base + (q * 32 + lane) * 4;
      const uint32_t word = e0 < len ? __ldcg(mrow + ((start + e0) >> 5)) : 0u;
      const uint32_t bits = (word >> ((start + e0) & 31)) & 15u;
#pragma unroll
      for (int k = 0; k < 4; ++k)
        if (!((bits >> k) & 1u)) v[q][k] = RL_NEG_INF;
    }
  }
}
template <typename E>
__device__ __forceinline__ void load_slice_global(const SpecArgs& a, const ItemMeta& mt, const uint32_t* tab, int& hp,
                                                  int start, int base, float (&v)[4][4]) {
  const E* rowp = reinterpret_cast<const E*>(a.logits) + static_cast<int64_t>(mt.row) * a.ld;
  load_slice_raw<E>(rowp, a.V, start, base, v);
  finish_slice<E>(a, mt, tab, hp, start, base, v);
}
// The raw slices of a row (warp w: slice w of every chunk) with three chunks
// of loads in flight in fixed registers: the loop is unrolled by three, so no
// register copy waits on a load still in flight. f(v, start) per slice, in
// chunk order.
template <typename E, typename F>
__device__ __forceinline__ void stream_raw3(const E* rowp, int V, int base, F f) {
  const int S = spec_chunks(V);
  float b0[4][4], b1[4][4], b2[4][4];
  load_slice_raw<E>(rowp, V, 0, base, b0);
  if (S > 1) load_slice_raw<E>(rowp, V, kCE, base, b1);
  if (S > 2) load_slice_raw<E>(rowp, V, 2 * kCE, base, b2);
#pragma unroll 1
  for (int c = 0; c < S; c += 3) {
    f(b0, c * kCE);
    if (c + 3 < S) load_slice_raw<E>(rowp, V, (c + 3) * kCE, base, b0);
    if (c + 1 < S) {
      f(b1, (c + 1) * kCE);
      if (c + 4 < S) load_slice_raw<E>(rowp, V, (c + 4) * kCE, base, b1);
    }
    if (c + 2 < S) {
      f(b2, (c + 2) * kCE);
      if (c + 5 < S) load_slice_raw<E>(rowp, V, (c + 5) * kCE, base, b2);
    }
  }
}
// Streams a row with penalties and mask applied; f(x, id) for every allowed
// finite logit. DEEP: three chunks in flight (the finish kernel, which has the
// registers); otherwise one chunk ahead (inside the streaming kernel).
template <typename E, bool DEEP, typename F>
__device__ __forceinline__ void stream_row(const SpecArgs& a, const ItemMeta& mt, const uint32_t* tab, F f) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int base = warp * kSlice;
  const E* rowp = reinterpret_cast<const E*>(a.logits) + static_cast<int64_t>(mt.row) * a.ld;
  int hp = 0;
  auto slice = [&](float (&v)[4][4], int start) {
    finish_slice<E>(a, mt, tab, hp, start, base, v);
#pragma unroll
    for (int q = 0; q < 4; ++q)
#pragma unroll
      for (int k = 0; k < 4; ++k)
        if (v[q][k] > RL_NEG_INF) f(v[q][k], start + base + (q * 32 + lane) * 4 + k);
  };
  if constexpr (DEEP) {
    stream_raw3<E>(rowp, a.V, base, slice);
  } else {
    const int S = spec_chunks(a.V);
    float n1[4][4];
    load_slice_raw<E>(rowp, a.V, 0, base, n1);
#pragma unroll 1
    for (int c = 0; c < S; ++c) {
      float v[4][4];
#pragma unroll
      for (int q = 0; q < 4; ++q)
#pragma unroll
        for (int k = 0; k < 4; ++k) v[q][k] = n1[q][k];
      if (c + 1 < S) load_slice_raw<E>(rowp, a.V, (c + 1) * kCE, base, n1);
      slice(v, c * kCE);
    }
  }
}

// ---------------------------------------------------------------------------
// Finisher
// ---------------------------------------------------------------------------
// Where a partial launch puts row r's sorted keys and its summary.
__device__ __forceinline__ uint64_t* part_keys_of(const SpecArgs& a, int row) {
  return a.part_keys + static_cast<int64_t>(row) * (a.part_packed ? kRec : kN);
}
__device__ __forceinline__ PartStats* part_stats_of(const SpecArgs& a, int row) {
  return a.part_packed ? reinterpret_cast<PartStats*>(part_keys_of(a, row) + kN) : a.part_stats + row;
}

__device__ __forceinline__ void write_row(const SpecArgs& a, int row, int status, int token, float prob) {
  if (a.part_keys) {
    // partial launch: an unfinished row is reported through its summary
    PartStats ps;
    ps.m = RL_NEG_INF;
    ps.argmax = -1;
    ps.nallow = 0;
    ps.flags = status == RL_ERR_TIMEOUT ? kFlagTimeout : kFlagBad;
    ps.z = 0.0;
    ps.nt = 0;
    ps.pad = 0;
    *part_stats_of(a, row) = ps;
    return;
  }
  const bool ok = status == 0;
  a.out_tok[row] = ok ? token + a.vocab_offset : -1;
  if (a.out_prob) a.out_prob[row] = ok ? prob : 0.0f;
  if (a.row_status) a.row_status[row] = status;
}

// Whether the sorted history table holds `id` (entries (id << 11) | count).
__device__ __forceinline__ bool tab_has(const uint32_t* tab, int ntab, int id) {
  int lo = 0, hi = ntab;
  while (lo < hi) {
    const int mid = (lo + hi) >> 1;
    if (static_cast<int>(tab[mid] >> 11) < id) lo = mid + 1;
    else hi = mid;
  }
  return lo < ntab && static_cast<int>(tab[lo] >> 11) == id;
}

// The smallest float x with bin_of(x) >= A. bin_of is non-decreasing in x
// over |x * cb| < 2^22 (the range that histogram windows accept), so this is
// a binary search (32 steps) over the order-preserving integer image of that
// range. Near 0 a bin edge can lie many ulps away from A / cb (x * cb - 1/2
// rounds to -1/2 for every |x * cb| < 2^-25), so no stepping from a guess.
__device__ float bin_floor_x(float A, const RowT& rt) {
  const float lim = 4190000.0f / rt.cb_hi;
  if (bin_of(-lim, rt) >= A) return RL_NEG_INF;
  if (bin_of(lim, rt) < A) return RL_POS_INF;
  uint32_t lo = ord_key(-lim), hi = ord_key(lim);  // bin(lo) < A <= bin(hi)
  while (hi - lo > 1u) {
    const uint32_t mid = lo + ((hi - lo) >> 1);
    if (bin_of(ord_key_inv(mid), rt) >= A) hi = mid;
    else lo = mid;
  }
  return ord_key_inv(hi);
}

// Keys of the allowed logits of absolute bin A (and of bin A2 unless A2 is
// NaN), gathered from one re-read of the row into buf; returns the count
// (> kCollect: too many). The stream compares raw logits against the bins'
// value intervals and leaves out the history ids, which are then tested with
// their penalised values.
// With explicit edges (expl): the logits in [xlo_o, xhi_o) instead of bin A
// (A2 must be NaN then).
template <typename E, bool SPLIT>
__device__ __noinline__ int collect_bin(const SpecArgs& a, const ItemMeta& mt, const uint32_t* tab, float A, float A2,
                                        uint64_t* buf, Ctl* ctl, float xlo_o = 0.0f, float xhi_o = 0.0f,
                                        bool expl = false) {
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const RowT rt = mt.rt;
  // the four bin edges, one thread each
  if (tid == 0) {
    ctl->cnt = 0;
    ctl->cx_lo = expl ? xlo_o : bin_floor_x(A, rt);
  } else if (tid == 32) {
    ctl->cx_hi = expl ? xhi_o : bin_floor_x(A + 1.0f, rt);
  } else if (tid == 64) {
    ctl->cx_lo2 = (!expl && A2 == A2) ? bin_floor_x(A2, rt) : RL_POS_INF;
  } else if (tid == 96) {
    ctl->cx_hi2 = (!expl && A2 == A2) ? bin_floor_x(A2 + 1.0f, rt) : RL_NEG_INF;
  }
  cbar();
  const float xlo = ctl->cx_lo;
  const float xhi = ctl->cx_hi;
  const float xlo2 = ctl->cx_lo2;
  const float xhi2 = ctl->cx_hi2;
  if constexpr (!SPLIT) {
    // inside the streaming kernel: the penalised stream (few registers)
    stream_row<E, false>(a, mt, tab, [&](float x, int id) {
      if ((x >= xlo && x < xhi) || (x >= xlo2 && x < xhi2)) {
        const int i = atomicAdd(&ctl->cnt, 1);
        if (i < kCollect) buf[i] = cand_key(x, static_cast<uint32_t>(id));
      }
    });
    cbar();
    const int n0 = ctl->cnt;
    cbar();
    return n0;
  }
  const int ntab = mt.ntab;
  const int V = a.V;
  const int S = spec_chunks(V);
  const int base = warp * kSlice;
  const E* rowp = reinterpret_cast<const E*>(a.logits) + static_cast<int64_t>(mt.row) * a.ld;
  const uint32_t* mrow = mt.mask_on ? a.mask + static_cast<int64_t>(mt.row) * a.mask_stride : nullptr;
  // While the row streams, hits are only noted: a per-warp queue of
  // (chunk, lane, 16-bit mask) words filled by a ballot, no atomics and no
  // loads in the loop (either would hold up the loads in flight); the keys
  // are built from the queue afterwards. The queue lives in the sort
  // scratch of the warp-buffer area, free until the keys are sorted.
  constexpr int kQcap = 512;
  static_assert(2 * kNB * 8 + kCW * kQcap * 4 <= kCW * kWcap * 8, "collect queue");
  uint32_t* wq = reinterpret_cast<uint32_t*>(smem_map().wbuf + 2 * kNB) + warp * kQcap;
  int nq = 0;  // warp-uniform
  auto note = [&](unsigned hm, int start) {
    const unsigned ball = __ballot_sync(0xffffffffu, hm != 0u);
    if (ball) {
      const int j = nq + __popc(ball & ((1u << lane) - 1u));
      if (hm && j < kQcap)
        wq[j] = (static_cast<uint32_t>(start / kCE) << 21) | (static_cast<uint32_t>(lane) << 16) | hm;
      nq += __popc(ball);
    }
  };
  if (!(xlo2 < xhi2)) {
    // one bin: two compares per logit
    stream_raw3<E>(rowp, V, base, [&](float (&v)[4][4], int start) {
      unsigned hm = 0u;
#pragma unroll
      for (int q = 0; q < 4; ++q)
#pragma unroll
        for (int k = 0; k < 4; ++k) hm |= (v[q][k] >= xlo && v[q][k] < xhi) ? (1u << (q * 4 + k)) : 0u;
      note(hm, start);
    });
  } else {
    // two bins (xhi <= xlo2): one compare against the lower edge, the exact
    // test only where a lane of the warp passes it
    stream_raw3<E>(rowp, V, base, [&](float (&v)[4][4], int start) {
      unsigned hm = 0u;
#pragma unroll
      for (int q = 0; q < 4; ++q)
#pragma unroll
        for (int k = 0; k < 4; ++k) hm |= (v[q][k] >= xlo) ? (1u << (q * 4 + k)) : 0u;
      if (!__any_sync(0xffffffffu, hm != 0u)) return;
      hm = 0u;
#pragma unroll
      for (int q = 0; q < 4; ++q)
#pragma unroll
        for (int k = 0; k < 4; ++k)
          hm |= ((v[q][k] >= xlo && v[q][k] < xhi) || (v[q][k] >= xlo2 && v[q][k] < xhi2)) ? (1u << (q * 4 + k)) : 0u;
      note(hm, start);
    });
  }
  __syncwarp();
  // the queued hits: keys from (cached) reloads, one queue word per lane
  for (int e = lane; e < min(nq, kQcap); e += 32) {
    const uint32_t w = wq[e];
    const int c = static_cast<int>(w >> 21), l = static_cast<int>((w >> 16) & 31u);
    unsigned hm = w & 0xffffu;
    while (hm) {
      const int b = __ffs(hm) - 1;
      hm &= hm - 1u;
      const int id = c * kCE + base + ((b >> 2) * 32 + l) * 4 + (b & 3);
      if (mrow && !((__ldcg(mrow + (id >> 5)) >> (id & 31)) & 1u)) continue;
      const float x = to_f32<E>(rowp[id]);
      const int i = atomicAdd(&ctl->cnt, 1);
      if (i < kCollect) buf[i] = cand_key(x, static_cast<uint32_t>(id));
    }
  }
  // a full queue (or a row too long for the chunk field) reports too many keys
  if (lane == 0 && (nq > kQcap || spec_chunks(V) > 2048)) atomicMax(&ctl->cnt, kCollect + 1);
  cbar();
  const int n_all = ctl->cnt;
  if (ntab > 0 && n_all <= kCollect) {
    // history ids were taken with their raw values: drop them (one search
    // per collected key), then test their penalised values (an overflowing
    // bin keeps its count above kCollect and is not filtered)
    const int n0 = n_all;
    cbar();
    if (tid == 0) ctl->cnt = 0;
    cbar();
    uint64_t keep[kCollect / kConsumers];
    int nk = 0;
#pragma unroll
    for (int r = 0; r < kCollect / kConsumers; ++r) {
      const int i = tid + r * kConsumers;
      if (i < n0) {
        const uint64_t key = buf[i];
        if (!tab_has(tab, ntab, static_cast<int>(key_id(key)))) keep[nk++] = key;
      }
    }
    cbar();
    for (int r = 0; r < nk; ++r) buf[atomicAdd(&ctl->cnt, 1)] = keep[r];
  }
  // history ids: their penalised values
  for (int j = tid; j < ntab; j += kConsumers) {
    const uint32_t ent = tab[j];
    const int cnt = static_cast<int>(ent & 2047u);
    const int id = static_cast<int>(ent >> 11);
    if (cnt == 0 || id >= V) continue;
    if (mrow && !((__ldcg(mrow + (id >> 5)) >> (id & 31)) & 1u)) continue;
    const float raw = to_f32<E>(rowp[id]);
    if (raw != raw) continue;
    const float x = pen_value(raw, cnt, mt.rp, mt.freq, mt.pres);
    if ((x >= xlo && x < xhi) || (x >= xlo2 && x < xhi2)) {
      const int i = atomicAdd(&ctl->cnt, 1);
      if (i < kCollect) buf[i] = cand_key(x, static_cast<uint32_t>(id));
    }
  }
  cbar();
  const int n = ctl->cnt;
  cbar();
  return n;
}

// A bin too full for the collect buffer, split by one re-read: its allowed
// logits grouped by order key into kSub sub-ranges of the bin's key range
// [klo, klo + span), sub-range 0 the highest; per sub-range the count
// (sm.radix[s]) and the exact mass in probability units (the doubles after
// the counts). All consumer threads return the bin's klo, span and top edge.
constexpr int kSub = 256;
static_assert(kSub == kConsumers, "one sub-range per consumer thread");
template <typename E, bool SPLIT>
__device__ __noinline__ void sub_hist(const SpecArgs& a, const ItemMeta& mt, const uint32_t* tab, float A, float M,
                                      double Z, uint32_t* klo_out, uint32_t* span_out, float* xhi_out) {
  const Smem sm = smem_map();
  const int tid = threadIdx.x;
  const RowT rt = mt.rt;
  uint32_t* bcnt = sm.radix;
  double* bmass = reinterpret_cast<double*>(sm.radix + 256);
  if (tid == 0) sm.ctl->cx_lo = bin_floor_x(A, rt);
  else if (tid == 32) sm.ctl->cx_hi = bin_floor_x(A + 1.0f, rt);
  bcnt[tid] = 0u;
  bmass[tid] = 0.0;
  cbar();
  const float xlo = sm.ctl->cx_lo, xhi = sm.ctl->cx_hi;
  cbar();
  const uint32_t klo = ord_key(__fadd_rn(xlo, 0.0f));
  const uint32_t span = ord_key(xhi) - klo;  // > 0: xlo < xhi
  auto add = [&](float x) {
    const uint32_t j = static_cast<uint32_t>(
        (static_cast<uint64_t>(ord_key(__fadd_rn(x, 0.0f)) - klo) * static_cast<uint64_t>(kSub)) / span);
    const int sb = kSub - 1 - static_cast<int>(j);
    atomicAdd(&bcnt[sb], 1u);
    atomicAdd(&bmass[sb], static_cast<double>(exact_e(x, M, rt)) / Z);
  };
  // raw values of the ids outside the history (plain loads: the re-read is
  // mostly an L2 hit), then the history ids with their penalised values
  const E* rowp = reinterpret_cast<const E*>(a.logits) + static_cast<int64_t>(mt.row) * a.ld;
  const uint32_t* mrow = mt.mask_on ? a.mask + static_cast<int64_t>(mt.row) * a.mask_stride : nullptr;
  const int ntab = mt.ntab;
  const int V = a.V;
  for (int i0 = 0; i0 < V; i0 += kConsumers * 8) {
    float v[8];
#pragma unroll
    for (int u = 0; u < 8; ++u) {
      const int i = i0 + u * kConsumers + tid;
      v[u] = i < V ? to_f32<E>(__ldcg(rowp + i)) : RL_NEG_INF;
    }
#pragma unroll
    for (int u = 0; u < 8; ++u) {
      const int i = i0 + u * kConsumers + tid;
      const float x = v[u];
      if (!(x >= xlo && x < xhi && x > RL_NEG_INF)) continue;
      if (mrow && !((__ldcg(mrow + (i >> 5)) >> (i & 31)) & 1u)) continue;
      if (ntab > 0 && tab_has(tab, ntab, i)) continue;
      add(x);
    }
  }
  for (int j = tid; j < ntab; j += kConsumers) {
    const uint32_t ent = tab[j];
    const int cnt = static_cast<int>(ent & 2047u);
    const int id = static_cast<int>(ent >> 11);
    if (cnt == 0 || id >= V) continue;
    if (mrow && !((__ldcg(mrow + (id >> 5)) >> (id & 31)) & 1u)) continue;
    const float raw = to_f32<E>(rowp[id]);
    if (raw != raw) continue;
    const float x = pen_value(raw, cnt, mt.rp, mt.freq, mt.pres);
    if (x >= xlo && x < xhi && x > RL_NEG_INF) add(x);
  }
  cbar();
  *klo_out = klo;
  *span_out = span;
  *xhi_out = xhi;
}

// A bin too full for the collect buffer, resolved to one sub-range: after
// sub_hist, the first sub-range (highest first) at whose end the running
// count c0 + n / mass m0 + m passes the test (kind 0, the cutoff: count >= K
// when count_mode, or mass >= p when mass_mode; kind 1, the draw: mass > p);
// its logits are collected into buf (*ntot keys, > kCollect: too many).
// s = INT_MAX when the test passes nowhere in the bin; the bin's exact count
// and mass are returned either way. Out of line: only rows whose bins
// overflow the buffer come here.
struct SubPick {
  int s;
  int n_total;
  double m_total;
  long long c_before;
  double m_before;
};
template <typename E, bool SPLIT>
__device__ __noinline__ SubPick split_bin(const SpecArgs& a, const ItemMeta& mt, const uint32_t* tab, float A, float M,
                                          double Z, long long c0, double m0, int kind, long long K, double p,
                                          bool count_mode, bool mass_mode, uint64_t* buf, int* ntot) {
  const Smem sm = smem_map();
  const int tid = threadIdx.x;
  uint32_t klo, span;
  float xhi;
  sub_hist<E, SPLIT>(a, mt, tab, A, M, Z, &klo, &span, &xhi);
  const uint32_t n = sm.radix[tid];
  const double m = reinterpret_cast<const double*>(sm.radix + 256)[tid];
  const long long ci = c0 + static_cast<long long>(cscan_u32(n, sm.red));
  double mtot;
  const double mi = m0 + cscan_d(m, sm.red, &mtot);
  SubPick r;
  r.n_total = csum_i(static_cast<int>(n), sm.red);
  r.m_total = mtot;
  const bool pass = kind == 0 ? ((count_mode && ci >= K) || (mass_mode && mi >= p)) : (mi > p);
  r.s = cmin_i((n > 0u && pass) ? tid : INT_MAX, sm.red);
  r.c_before = 0;
  r.m_before = 0.0;
  *ntot = 0;
  if (r.s == INT_MAX) return r;
  if (tid == r.s) {
    // keys k of sub-range j: floor((k - klo) kSub / span) = j
    const uint64_t j = static_cast<uint64_t>(kSub - 1 - tid);
    const uint64_t kSubU = static_cast<uint64_t>(kSub);
    const uint32_t ka = klo + static_cast<uint32_t>((j * span + kSubU - 1) / kSubU);
    const uint32_t kb = klo + static_cast<uint32_t>(((j + 1) * span + kSubU - 1) / kSubU);
    sm.ctl->res_c = ci - static_cast<long long>(n);
    sm.ctl->res_d = mi - m;
    sm.ctl->cx_lo2 = ord_key_inv(ka);
    sm.ctl->cx_hi2 = (j + 1 == kSubU) ? xhi : ord_key_inv(kb);
  }
  cbar();
  r.c_before = sm.ctl->res_c;
  r.m_before = sm.ctl->res_d;
  const float x1 = sm.ctl->cx_lo2, x2 = sm.ctl->cx_hi2;
  cbar();
  *ntot = collect_bin<E, SPLIT>(a, mt, tab, 0.0f, __int_as_float(0x7fc00000), buf, sm.ctl, x1, x2, true);
  return r;
}

// Exact radix walk over re-reads of the row: the first logit in list order
// at which the running count reaches cnt_target (kind 0) or the running
// mass (e units, relative to M) reaches target (kind 1: >=, kind 2: >).
// Returns its key and its exclusive cumulative count and mass; when the
// target is never reached, *cnt_before = -1 and *mass_before = the total.
template <typename E, bool SPLIT>
__device__ __noinline__ uint64_t radix_walk(const SpecArgs& a, const ItemMeta& mt, const uint32_t* tab, float M, int kind,
                               long long cnt_target, double target, long long* cnt_before, double* mass_before) {
  const Smem sm = smem_map();
  const int tid = threadIdx.x;
  uint32_t* bcnt = sm.radix;
  double* bmass = reinterpret_cast<double*>(sm.radix + 256);
  unsigned long long* bmax = reinterpret_cast<unsigned long long*>(bmass + 256);
  uint64_t prefix = 0ull;
  for (int shift = 56; shift >= 0; shift -= 8) {
    bcnt[tid] = 0u;
    bmass[tid] = 0.0;
    bmax[tid] = 0ull;
    cbar();
    long long my_c = 0;
    double my_m = 0.0;
    const RowT rt = mt.rt;
    stream_row<E, SPLIT>(a, mt, tab, [&](float x, int id) {
      const uint64_t key = cand_key(x, static_cast<uint32_t>(id));
      const double e = static_cast<double>(exact_e(x, M, rt));
      if (hi_match(key, prefix, shift + 8)) {
        const int b = static_cast<int>((key >> shift) & 255u);
        atomicAdd(&bcnt[b], 1u);
        atomicAdd(&bmass[b], e);
        atomicMax(&bmax[b], static_cast<unsigned long long>(key));
      } else if (key > prefix) {
        my_c += 1;
        my_m += e;
      }
    });
    cbar();
    // logits above the current prefix range
    const long long ca = static_cast<long long>(csum_u64(static_cast<unsigned long long>(my_c), sm.red));
    const double ma = csum_d(my_m, sm.red);
    // thread t owns bucket 255 - t; inclusive scans from the top bucket
    const int b = 255 - tid;
    double mtot;
    const uint32_t nb = bcnt[b];
    const double mbk = bmass[b];
    const uint32_t cinc = cscan_u32(nb, sm.red);
    const double minc = cscan_d(mbk, sm.red, &mtot);
    bool hit = false;
    if (nb > 0u) {
      if (kind == 0) hit = ca + static_cast<long long>(cinc) >= cnt_target;
      else if (kind == 1) hit = ma + minc >= target;
      else hit = ma + minc > target;
    }
    const int first = cmin_i(hit ? tid : INT_MAX, sm.red);
    if (first == INT_MAX) {
      *cnt_before = -1;
      *mass_before = ma + mtot;
      return 0ull;
    }
    if (tid == first) {
      sm.ctl->res_i = static_cast<int>(nb);
      sm.ctl->res_j = b;
      sm.ctl->res_key = bmax[b];
      sm.ctl->res_c = ca + static_cast<long long>(cinc - nb);
      sm.ctl->res_d = ma + (minc - mbk);
    }
    cbar();
    const int cnt_b = sm.ctl->res_i;
    const int bsel = sm.ctl->res_j;
    const uint64_t kmaxb = sm.ctl->res_key;
    const long long ce = sm.ctl->res_c;
    const double me = sm.ctl->res_d;
    cbar();
    prefix |= static_cast<uint64_t>(bsel) << shift;
    if (cnt_b == 1 || shift == 0) {
      *cnt_before = ce;
      *mass_before = me;
      return cnt_b == 1 ? kmaxb : prefix;
    }
  }
  *cnt_before = -1;
  *mass_before = 0.0;
  return 0ull;
}

// First index j in [0, n) of sorted keys (exact e, probability units,
// starting at `run`) where cond(j, cum_j) holds; INT_MAX if none. *cum_at
// gets the inclusive cumulative there, *run_end the total.
template <typename F>
__device__ int sweep_sorted(const uint64_t* keys, int n, float M, double Z, const RowT& rt, double run, F cond,
                            Red* rs, Ctl* ctl, double* cum_at, double* run_end) {
  const int tid = threadIdx.x;
  for (int c0 = 0; c0 < n; c0 += kConsumers) {
    const int j = c0 + tid;
    double pj = 0.0;
    if (j < n) pj = static_cast<double>(exact_e(key_val(keys[j]), M, rt)) / Z;
    double tot;
    const double cum = run + cscan_d(pj, rs, &tot);
    const int g = cmin_i((j < n && cond(j, cum)) ? j : INT_MAX, rs);
    if (g != INT_MAX) {
      if (j == g) ctl->res_d = cum;
      cbar();
      *cum_at = ctl->res_d;
      cbar();
      *run_end = run + tot;
      return g;
    }
    run += tot;
  }
  *run_end = run;
  return INT_MAX;
}

// The finish kernel's history table, when a re-read of the row first needs
// it (build_meta left minus the history length in ntab): the sorted table
// the streaming kernel left for the row's first item, else gathered and
// sorted here.
__device__ __noinline__ void lazy_table(const SpecArgs& a, const ItemMeta& mt, const uint32_t* tab_c, int first_item) {
  ItemMeta& m = const_cast<ItemMeta&>(mt);
  uint32_t* tab = const_cast<uint32_t*>(tab_c);
  const int hl = -m.ntab;
  if (hl <= 0) return;
  cbar();
  if (a.ws.tabs) {
    const int n = __ldcg(a.ws.tabn + first_item);
    const uint32_t* src = a.ws.tabs + static_cast<int64_t>(first_item) * kHmax;
    for (int i = threadIdx.x; i < n; i += kConsumers) tab[i] = __ldcg(src + i);
    cbar();
    if (threadIdx.x == 0) m.ntab = n;
    cbar();
    return;
  }
  if (threadIdx.x < 32) {
    const int n = gather_history(a, m.row, hl, tab, 0, a.V);
    if (threadIdx.x == 0) m.ntab = n;
  }
  cbar();
  if (m.ntab > 0) block_sort_table(tab, m.ntab);
}

// Softmax sum of a row from its segment summaries, relative to the row max.
__device__ __forceinline__ double row_z(const ItemSum* sums, int nseg, float M, float T) {
  const double cd = kLog2e / static_cast<double>(T);
  double Z = 0.0;
  for (int s = 0; s < nseg; ++s) {
    const ItemSum& q = sums[s];
    if (q.nallow > 0 && q.m > RL_NEG_INF) Z += q.z * exp2((static_cast<double>(q.m) - static_cast<double>(M)) * cd);
  }
  return Z;
}

// Summary of a partial launch's row (global argmax id, -1 if none).
__device__ __forceinline__ void write_part(const SpecArgs& a, int row, float M, int argmax, int nallow, int flags,
                                           double Z, int nt) {
  PartStats ps;
  ps.m = M;
  ps.argmax = (argmax == INT_MAX) ? -1 : argmax + a.vocab_offset;
  ps.nallow = nallow;
  ps.flags = flags & (kFlagBad | kFlagTimeout);
  ps.z = Z;
  ps.nt = nt;
  ps.pad = 0;
  *part_stats_of(a, row) = ps;
}

// The finisher of a row (consumer threads). On entry sm.sums[0..nseg) hold
// the segment summaries; for a one-segment row sm.top holds the sorted list
// and the histogram is in shared memory.
template <typename E, bool SPLIT>
__device__ __noinline__ void finish_row(const SpecArgs& a, const ItemMeta& mt, const uint32_t* tab, int first_item) {
  const Smem sm = smem_map();
  const int tid = threadIdx.x;
  const int row = mt.row;
  const int nseg = a.nseg;
  Ctl* ctl = sm.ctl;
  Red* rs = sm.red;
  // ---- row summary ----
  float M = RL_NEG_INF;
  int argmax = INT_MAX, nallow = 0, flags = 0;
  for (int s = 0; s < nseg; ++s) {
    const ItemSum& q = sm.sums[s];
    nallow += q.nallow;
    flags |= q.flags;
    if (q.m > M) {
      M = q.m;
      argmax = q.argmax;
    } else if (q.m == M) {
      argmax = min(argmax, q.argmax);
    }
  }
  const float T = mt.rt.T;
  int status = 0;
  if (flags & kFlagTimeout) status = RL_ERR_TIMEOUT;
  else if ((flags & kFlagBad) || nallow == 0 || !(fabsf(T) < RL_POS_INF)) status = RL_ERR_NONFINITE;
  const bool want_list = a.list_len != nullptr;
  if (a.part_keys && (status != 0 || mt.mode != 1)) {
    // partial launch of a row without a list (greedy, or not a top-k row)
    if (tid == 0) write_part(a, row, M, argmax, nallow, flags, mt.mode == 0 ? 0.0 : row_z(sm.sums, nseg, M, T), 0);
    return;
  }
  if (status != 0 || mt.mode == 0) {
    if (tid == 0) {
      write_row(a, row, status, argmax, 1.0f);
      if (a.list_cut) {
        a.list_cut[static_cast<int64_t>(row) * 3 + 0] = status == 0 ? 1 : 0;
        a.list_cut[static_cast<int64_t>(row) * 3 + 1] = status == 0 ? 0 : -1;
        a.list_cut[static_cast<int64_t>(row) * 3 + 2] = status == 0 ? argmax + a.vocab_offset : -1;
      }
      if (want_list) {
        const bool ok = status == 0 && a.list_cap > 0;
        a.list_len[row] = ok ? 1 : 0;
        if (ok) {
          a.list_ids[static_cast<int64_t>(row) * a.list_cap] = argmax + a.vocab_offset;
          a.list_probs[static_cast<int64_t>(row) * a.list_cap] = 1.0f;
        }
      }
    }
    return;
  }
  const RowT& rt = mt.rt;
  const double Z = row_z(sm.sums, nseg, M, T);
  // ---- the row's sorted list ----
  int nt = 0;
  if (nseg == 1) {
    nt = sm.sums[0].ncand;
  } else {
    int total = 0;
    for (int s = 0; s < nseg; ++s) total += sm.sums[s].ncand;
    for (int s = tid; s < nseg; s += kConsumers) sm.segn[s] = sm.sums[s].ncand;
    cbar();
    const uint64_t* base = a.ws.cands + static_cast<int64_t>(first_item) * kN;
    const int need = min(total, mt.nkeep);
    if (need > 0) {
      // a segment holding nkeep keys bounds the row's nkeep-th key by its last
      // one (lists are sorted); the keys above the bound go to shared memory
      uint64_t b0 = 0ull;
      if (tid < nseg && sm.segn[tid] >= mt.nkeep)
        b0 = __ldcg(reinterpret_cast<const unsigned long long*>(base + static_cast<int64_t>(tid) * kN + mt.nkeep - 1));
      const uint64_t bound = cmax_u64(b0, rs);
      uint64_t* buf = reinterpret_cast<uint64_t*>(sm.hmass);  // collect area (the histogram is in global)
      if (tid == 0) ctl->cnt = 0;
      cbar();
      const int slots = nseg * kN;
      for (int f0 = 0; f0 < slots; f0 += 4 * kConsumers) {
        uint64_t k4[4];
        bool ok4[4];
#pragma unroll
        for (int r = 0; r < 4; ++r) {
          const int f = f0 + r * kConsumers + tid;
          const int sg = f / kN;
          ok4[r] = f < slots && (f - sg * kN) < sm.segn[sg];
          k4[r] = ok4[r] ? __ldcg(reinterpret_cast<const unsigned long long*>(base + f)) : 0ull;
        }
#pragma unroll
        for (int r = 0; r < 4; ++r)
          if (ok4[r] && k4[r] >= bound) {
            const int i = atomicAdd(&ctl->cnt, 1);
            if (i < kCollect) buf[i] = k4[r];
          }
      }
      cbar();
      const int ncol = ctl->cnt;
      cbar();
      if (ncol <= kCollect) {
        csort_desc(buf, ncol, pow2_at_least(max(ncol, 1)));
        for (int i = tid; i < need; i += kConsumers) sm.top[i] = buf[i];
        cbar();
        nt = need;
      } else {
        const uint64_t Tk = block_select<true>(base, nseg, kN, sm.segn, need, sm.radix, rs, ctl);
        nt = gather_sorted<true>(base, nseg, kN, sm.segn, Tk, sm.top, ctl);
      }
    }
  }
  if (a.part_keys) {
    // partial launch: the row's (shard's) sorted list with global ids
    for (int i = tid; i < nt; i += kConsumers) {
      const uint64_t k = sm.top[i];
      part_keys_of(a, row)[i] =
          cand_key(key_val(k), key_id(k) + static_cast<uint32_t>(a.vocab_offset));
    }
    if (tid == 0) write_part(a, row, M, argmax, nallow, flags, Z, nt);
    return;
  }
  const int K = (mt.top_k > 0 && mt.top_k < nallow) ? mt.top_k : nallow;
  const bool mass_mode = mt.top_p < 1.0f;
  const bool count_mode = K < nallow;
  const double pd = static_cast<double>(mt.top_p);
  const double ud = static_cast<double>(mt.u);
  // exact e and cumulative probabilities of the list
  {
    float e = 0.0f;
    double pr = 0.0;
    if (tid < nt) {
      e = exact_e(key_val(sm.top[tid]), M, rt);
      pr = static_cast<double>(e) / Z;
    }
    double tot;
    const double cum = cscan_d(pr, rs, &tot);
    if (tid < nt) {
      sm.tope[tid] = e;
      sm.topc[tid] = cum;
    }
    cbar();
  }
  // complete prefix: list entries whose whole bin is in the list
  int complete = nt;
  float amin = 0.0f;
  if (mt.mode == 2 && nt < nallow && nt > 0) {
    amin = bin_of(key_val(sm.top[nt - 1]), rt);
    complete = cmin_i((tid < nt && bin_of(key_val(sm.top[tid]), rt) == amin) ? tid : INT_MAX, rs);
  }
  if (want_list) {
    const bool listed = K <= nt;
    const int nl = listed ? min(K, a.list_cap) : 0;
    if (tid == 0) a.list_len[row] = listed ? nl : -1;
    for (int i = tid; i < nl; i += kConsumers) {
      a.list_ids[static_cast<int64_t>(row) * a.list_cap + i] = static_cast<int>(key_id(sm.top[i])) + a.vocab_offset;
      a.list_probs[static_cast<int64_t>(row) * a.list_cap + i] =
          static_cast<float>(static_cast<double>(sm.tope[i]) / Z);
    }
  }
  int token = -1, st = 0;
  float prob = 0.0f;
  bool done = false;
  // position of the last kept entry in list order and its id (debug
  // launches; -2: the id is not resolved)
  long long dbg_pos = -1;
  int dbg_id = -2;
  // cutoff inside the complete prefix
  const int cut = cmin_i(
      (tid < complete && (tid == K - 1 || (mass_mode && sm.topc[tid] >= pd))) ? tid : INT_MAX, rs);
  if (cut != INT_MAX) {
    dbg_pos = cut;
    dbg_id = static_cast<int>(key_id(sm.top[cut]));
    const double Sx = sm.topc[cut];
    const double tgt = ud * Sx;
    int d = cmin_i((tid <= cut && sm.topc[tid] > tgt) ? tid : INT_MAX, rs);
    if (d == INT_MAX) d = cut;
    token = static_cast<int>(key_id(sm.top[d]));
    prob = static_cast<float>((static_cast<double>(sm.tope[d]) / Z) / Sx);
    done = true;
  } else if (!mass_mode && !count_mode) {
    // the list is every allowed id: S is the whole mass (1)
    dbg_pos = K - 1;
    dbg_id = (nt == nallow && nt > 0) ? static_cast<int>(key_id(sm.top[nt - 1])) : -2;
    const int d = cmin_i((tid < complete && sm.topc[tid] > ud) ? tid : INT_MAX, rs);
    if (d != INT_MAX) {
      token = static_cast<int>(key_id(sm.top[d]));
      prob = static_cast<float>(static_cast<double>(sm.tope[d]) / Z);
      done = true;
    }
  }

  if (!done) {
    if constexpr (SPLIT) lazy_table(a, mt, tab, first_item);
    // ---- below the list: the merged histogram, then the exact radix walk ----
    const double base_m = complete > 0 ? sm.topc[complete - 1] : 0.0;  // probability units
    const long long base_c = complete;
    bool hist_ok = mt.mode == 2 && nt > 0;
    int A_hi = 0, A_lo = INT_MIN;
    if (hist_ok) {
      // Logits above the list's last bin A_hi are all in the list. Below it
      // every segment's histogram must be complete: its window reaches up to
      // A_hi, or its maximum lies inside its window (segments later in a row
      // anchor lower, and hold nothing above their window top then).
      A_hi = static_cast<int>(amin);
      for (int s = 0; s < nseg; ++s) {
        const ItemSum& q = sm.sums[s];
        if (q.nallow == 0) continue;
        if (q.atop == kNoAnchor || (q.flags & kFlagHistBad)) {
          hist_ok = false;
          continue;
        }
        A_lo = max(A_lo, q.wlo);
        if (q.atop < A_hi && static_cast<int>(bin_of(q.m, rt)) > q.atop) hist_ok = false;
      }
      if (A_hi < A_lo || A_hi - A_lo >= kNB) hist_ok = false;
    }
    bool resolved = false;
    if (hist_ok) {
      // merged bins i = A_hi - A in probability units: inclusive prefix sums
      double* cm = reinterpret_cast<double*>(sm.wbuf);
      double* cc = cm + kNB;
      const int nb = A_hi - A_lo + 1;
      constexpr int BPT = kNB / kConsumers;
      {
        double lm[BPT], lc[BPT];
        double sm_ = 0.0, sc_ = 0.0;
        // bin A's mass unit exp((A+1)/kRbin - M/T) / (kMassQ Z): one exp2 per
        // thread, then the ratio between neighbouring bins
        const double rho = exp2(-kLog2e / static_cast<double>(kRbin));
        double fac = exp2(((static_cast<double>(A_hi - tid * BPT) + 1.0) / static_cast<double>(kRbin) -
                           static_cast<double>(M) / static_cast<double>(T)) * kLog2e) /
                     (static_cast<double>(kMassQ) * Z);
#pragma unroll
        for (int r = 0; r < BPT; ++r, fac *= rho) {
          const int i = tid * BPT + r;
          double mq = 0.0, cq = 0.0;
          if (i < nb) {
            const int A = A_hi - i;
            for (int s = 0; s < nseg; ++s) {
              const ItemSum& q = sm.sums[s];
              if (q.nallow == 0) continue;
              const int off = q.atop - A;
              if (off < 0 || off >= kNB) continue;
              if (nseg == 1) {
                mq += static_cast<double>(sm.hmass[off]);
                cq += static_cast<double>(sm.hcnt[off]);
              } else {
                const int64_t gb = static_cast<int64_t>(first_item + s) * kNB + off;
                mq += static_cast<double>(__ldcg(a.ws.hmass + gb));
                if (mt.need_count) cq += static_cast<double>(__ldcg(a.ws.hcnt + gb));
              }
            }
            mq *= fac;
          }
          lm[r] = mq;
          lc[r] = cq;
          sm_ += mq;
          sc_ += cq;
        }
        double tm, tc;
        double im = cscan_d(sm_, rs, &tm) - sm_;
        double ic = cscan_d(sc_, rs, &tc) - sc_;
#pragma unroll
        for (int r = 0; r < BPT; ++r) {
          const int i = tid * BPT + r;
          im += lm[r];
          ic += lc[r];
          if (i < nb) {
            cm[i] = im;
            cc[i] = ic;
          }
        }
        cbar();
      }
      uint64_t* buf = reinterpret_cast<uint64_t*>(sm.hmass);  // collect buffer (the histogram is merged)
      // sorted keys in buf: bin held at [off1, off1 + n1), bin held2 (read
      // with it, higher values) at [0, n2)
      int held = -1, held2 = -1, off1 = 0, n1 = 0, n2 = 0;
      double corr = 0.0;  // exact minus histogram mass of the bins passed so far
      long long ccorr = 0;
      // -- the cutoff bin --
      int i_c = nb, cut_pos = -1;
      double Sx = 0.0, bm_cut = 0.0;
      double bm_bin = 0.0;    // mass before the cutoff bin
      bool held_sub = false;  // the held keys are one sub-range of their bin
      bool cut_ok = false;
      int i0 = 0;
      // a lower bound on the logits of bin i: its mass over the mass of a
      // logit at its top edge (each of its logits has at most that mass)
      auto bin_min_count = [&](int i) {
        const double e_top = exp2((static_cast<double>(A_hi - i + 1) / static_cast<double>(kRbin) -
                                   static_cast<double>(M) / static_cast<double>(T)) * kLog2e) / Z;
        return (cm[i] - (i > 0 ? cm[i - 1] : 0.0)) / e_top;
      };
      for (int guard = 0; guard < nb && !cut_ok && (mass_mode || count_mode); ++guard) {
        int best = INT_MAX;
#pragma unroll
        for (int r = 0; r < BPT; ++r) {
          const int i = tid * BPT + r;
          if (i >= i0 && i < nb) {
            const bool hc = count_mode && base_c + ccorr + static_cast<long long>(cc[i]) >= K;
            const bool hm = mass_mode && base_m + corr + cm[i] >= pd;
            if ((hc || hm) && i < best) best = i;
          }
        }
        const int f = cmin_i(best, rs);
        if (f == INT_MAX) break;
        const double mb = base_m + corr + (f > 0 ? cm[f - 1] : 0.0);
        const long long cb = base_c + ccorr + (f > 0 ? static_cast<long long>(cc[f - 1]) : 0);
        // the draw bin, when a cutoff in bin f already fixes it: read in the
        // same pass. S lies in [bin start, bin end]; with top_p alone, in
        // [top_p, top_p + the mass of one logit at the bin's top edge]
        int fd = -1;
        {
          const bool p_only = mass_mode && !count_mode;
          const double e_top = exp2((static_cast<double>(A_hi - f + 1) / static_cast<double>(kRbin) -
                                     static_cast<double>(M) / static_cast<double>(T)) * kLog2e) / Z;
          const double s_end = base_m + corr + cm[f];
          const double t_lo = ud * (p_only ? fmax(mb, pd) : mb);
          const double t_hi = ud * (p_only ? fmin(s_end, fmax(mb, pd) + e_top) : s_end);
          if (t_lo >= base_m) {
            int b_lo = INT_MAX, b_hi = INT_MAX;
#pragma unroll
            for (int r = 0; r < BPT; ++r) {
              const int i = tid * BPT + r;
              if (i < f) {
                const double e_i = base_m + corr + cm[i];
                if (e_i > t_lo && i < b_lo) b_lo = i;
                if (e_i > t_hi && i < b_hi) b_hi = i;
              }
            }
            b_lo = cmin_i(b_lo, rs);
            b_hi = cmin_i(b_hi, rs);
            if (b_lo == b_hi && b_lo < f) fd = b_lo;
          }
        }
        const double nmin_f = bin_min_count(f);
        if (fd >= 0 && nmin_f + bin_min_count(fd) > static_cast<double>(kCollect)) fd = -1;
        // a bin sure to overflow the buffer goes straight to its sub-ranges
        int ntot = nmin_f > static_cast<double>(kCollect)
                       ? kCollect + 1
                       : collect_bin<E, SPLIT>(a, mt, tab, static_cast<float>(A_hi - f),
                                               fd >= 0 ? static_cast<float>(A_hi - fd) : __int_as_float(0x7fc00000),
                                               buf, ctl);
        if (ntot > kCollect && fd >= 0) {
          // the two bins together overflow the buffer: the cutoff bin alone
          // (the draw bin is collected by its own re-read below)
          fd = -1;
          ntot = collect_bin<E, SPLIT>(a, mt, tab, static_cast<float>(A_hi - f), __int_as_float(0x7fc00000), buf, ctl);
        }
        double mbs = mb;     // mass and count before the held keys
        long long cbs = cb;
        bool sub = false;
        if (ntot > kCollect) {
          // the bin alone overflows the buffer: its sub-ranges, then the
          // one where the cutoff falls
          const SubPick sp = split_bin<E, SPLIT>(a, mt, tab, static_cast<float>(A_hi - f), M, Z, cb, mb, 0,
                                                 static_cast<long long>(K), pd, count_mode, mass_mode, buf, &ntot);
          if (sp.s == INT_MAX) {
            // not in this bin: continue with its exact mass and count
            corr += sp.m_total - (cm[f] - (f > 0 ? cm[f - 1] : 0.0));
            ccorr += static_cast<long long>(sp.n_total) - static_cast<long long>(cc[f] - (f > 0 ? cc[f - 1] : 0.0));
            i0 = f + 1;
            continue;
          }
          if (ntot > kCollect) break;
          mbs = sp.m_before;
          cbs = sp.c_before;
          sub = true;
        }
        csort_desc(buf, ntot, pow2_at_least(max(ntot, 1)));
        n2 = 0;
        if (fd >= 0) {
          const float lo_d = ctl->cx_lo2;
          int j0 = INT_MAX;
          for (int j = tid; j < ntot; j += kConsumers)
            if (key_val(buf[j]) < lo_d) j0 = min(j0, j);
          j0 = cmin_i(j0, rs);
          n2 = j0 == INT_MAX ? ntot : j0;
        }
        held = f;
        held2 = fd;
        off1 = n2;
        n1 = ntot - n2;
        double cum_at = 0.0, run_end = 0.0;
        const int g = sweep_sorted(
            buf + off1, n1, M, Z, rt, mbs,
            [&](int j, double cum) {
              return (count_mode && cbs + j == static_cast<long long>(K) - 1) || (mass_mode && cum >= pd);
            },
            rs, ctl, &cum_at, &run_end);
        if (g != INT_MAX) {
          i_c = f;
          cut_pos = g;
          Sx = cum_at;
          bm_cut = mbs;
          bm_bin = mb;
          held_sub = sub;
          cut_ok = true;
          dbg_pos = cbs + g;  // exact when the bins carry counts (debug launches)
          dbg_id = static_cast<int>(key_id(buf[off1 + g]));
        } else if (sub) {
          break;  // the sub-range's sums disagree at rounding level: exact walk
        } else {
          // the histogram overstated this bin: continue with its exact mass
          corr += (run_end - mb) - (cm[f] - (f > 0 ? cm[f - 1] : 0.0));
          ccorr += static_cast<long long>(n1) - static_cast<long long>(cc[f] - (f > 0 ? cc[f - 1] : 0.0));
          i0 = f + 1;
        }
      }
      if (!cut_ok && !mass_mode && !count_mode) {
        cut_ok = true;  // no cutoff: S is the whole mass
        Sx = 1.0;
        dbg_pos = K - 1;
        dbg_id = -2;
      }
      if (cut_ok) {
        const double tgt = ud * Sx;
        if (complete > 0 && tgt < base_m) {
          int d = cmin_i((tid < complete && sm.topc[tid] > tgt) ? tid : INT_MAX, rs);
          if (d == INT_MAX) d = complete - 1;
          token = static_cast<int>(key_id(sm.top[d]));
          prob = static_cast<float>((static_cast<double>(sm.tope[d]) / Z) / Sx);
          resolved = true;
        } else {
          // the draw bin: the first bin whose end exceeds the target, at or
          // above the cutoff bin
          int i_d = 0;
          for (int guard = 0; guard < nb && !resolved; ++guard) {
            int best = INT_MAX;
#pragma unroll
            for (int r = 0; r < BPT; ++r) {
              const int i = tid * BPT + r;
              if (i >= i_d && i < nb && base_m + corr + cm[i] > tgt && i < best) best = i;
            }
            int f = cmin_i(best, rs);
            if (cut_pos >= 0 && (f == INT_MAX || f > i_c)) f = i_c;
            if (f == INT_MAX) break;
            const uint64_t* kb = buf + off1;
            int kn = n1;
            bool at_cut = cut_pos >= 0 && f == i_c;
            double mb = at_cut ? bm_cut : base_m + corr + (f > 0 ? cm[f - 1] : 0.0);
            bool dsub = false;  // the keys swept are one sub-range of bin f
            if (at_cut && held == f && held_sub && tgt < bm_cut) {
              // the cutoff bin was split and the draw lies above the
              // sub-range held: the sub-range of the bin that holds it
              int ntot = 0;
              const SubPick sp = split_bin<E, SPLIT>(a, mt, tab, static_cast<float>(A_hi - f), M, Z, 0, bm_bin, 1, 0,
                                                     tgt, false, false, buf, &ntot);
              if (sp.s == INT_MAX || !(sp.m_before < bm_cut) || ntot > kCollect) break;
              csort_desc(buf, ntot, pow2_at_least(max(ntot, 1)));
              held = -1;  // the cutoff's keys are gone
              kb = buf;
              kn = ntot;
              mb = sp.m_before;
              at_cut = false;
              dsub = true;
            } else if (held2 == f) {
              kb = buf;
              kn = n2;
            } else if (held != f) {
              if (at_cut && held_sub) break;  // the cutoff's sub-range is gone: exact walk
              int ntot = bin_min_count(f) > static_cast<double>(kCollect)
                             ? kCollect + 1
                             : collect_bin<E, SPLIT>(a, mt, tab, static_cast<float>(A_hi - f),
                                                     __int_as_float(0x7fc00000), buf, ctl);
              if (ntot > kCollect) {
                if (at_cut) break;
                // the bin overflows the buffer: the sub-range where the draw falls
                const SubPick sp = split_bin<E, SPLIT>(a, mt, tab, static_cast<float>(A_hi - f), M, Z, 0, mb, 1, 0,
                                                       tgt, false, false, buf, &ntot);
                if (sp.s == INT_MAX) {
                  held = -1;
                  i_d = f + 1;
                  continue;
                }
                if (ntot > kCollect) break;
                mb = sp.m_before;
                dsub = true;
              }
              csort_desc(buf, ntot, pow2_at_least(max(ntot, 1)));
              held = dsub ? -1 : f;
              held2 = -1;
              off1 = 0;
              n1 = ntot;
              kb = buf;
              kn = ntot;
            }
            const int lim = at_cut ? cut_pos + 1 : kn;
            double cum_at = 0.0, run_end = 0.0;
            int g = sweep_sorted(
                kb, lim, M, Z, rt, mb, [&](int, double cum) { return cum > tgt; }, rs, ctl, &cum_at, &run_end);
            if (g == INT_MAX && at_cut) g = cut_pos;
            if (g == INT_MAX && dsub) break;  // sums disagree at rounding level: exact walk
            if (g != INT_MAX) {
              const uint64_t key = kb[g];
              token = static_cast<int>(key_id(key));
              prob = static_cast<float>((static_cast<double>(exact_e(key_val(key), M, rt)) / Z) / Sx);
              resolved = true;
            } else {
              i_d = f + 1;
            }
          }
        }
      }
    }
    if (!resolved) {
      // ---- exact radix walk over re-reads of the row ----
      long long cb1 = -1, cb2 = -1;
      double mb1 = 0.0, mb2 = 0.0;
      uint64_t kc = 0ull;
      double Sx_e = 0.0;
      bool have_cut = false;
      if (count_mode) {
        const uint64_t kk = radix_walk<E, SPLIT>(a, mt, tab, M, 0, K, 0.0, &cb1, &mb1);
        if (cb1 >= 0) {
          kc = kk;
          Sx_e = mb1 + static_cast<double>(exact_e(key_val(kk), M, rt));
          have_cut = true;
          dbg_pos = cb1;
        }
      }
      if (mass_mode) {
        const uint64_t kp = radix_walk<E, SPLIT>(a, mt, tab, M, 1, 0, pd * Z, &cb2, &mb2);
        if (cb2 >= 0 && (!have_cut || kp > kc)) {
          kc = kp;
          Sx_e = mb2 + static_cast<double>(exact_e(key_val(kp), M, rt));
          have_cut = true;
          dbg_pos = cb2;
        }
      }
      if (have_cut) {
        dbg_id = static_cast<int>(key_id(kc));
      } else {
        dbg_pos = K - 1;
        dbg_id = -2;
      }
      if (!have_cut) {
        long long cbt;
        double tot;
        radix_walk<E, SPLIT>(a, mt, tab, M, 0, LLONG_MAX, 0.0, &cbt, &tot);
        Sx_e = tot;
      }
      long long cbd;
      double mbd;
      uint64_t kd = radix_walk<E, SPLIT>(a, mt, tab, M, 2, 0, ud * Sx_e, &cbd, &mbd);
      if (cbd < 0 || (have_cut && kd < kc)) kd = kc;
      if (kd == 0ull || !(Sx_e > 0.0)) {
        st = RL_ERR_UNSUPPORTED;
      } else {
        token = static_cast<int>(key_id(kd));
        prob = static_cast<float>(static_cast<double>(exact_e(key_val(kd), M, rt)) / Sx_e);
      }
    }
  }
  if (tid == 0) {
    write_row(a, row, st, token, prob);
    if (a.list_cut) {
      a.list_cut[static_cast<int64_t>(row) * 3 + 0] = st == 0 ? K : 0;
      a.list_cut[static_cast<int64_t>(row) * 3 + 1] = st == 0 ? static_cast<int>(dbg_pos) : -1;
      a.list_cut[static_cast<int64_t>(row) * 3 + 2] = (st == 0 && dbg_id >= 0) ? dbg_id + a.vocab_offset : dbg_id;
    }
  }
}

// Per-thread accumulators of an item, handed to its end.
struct ItemAcc {
  float m_run;
  int arg_run;
  int nal, bad, tmo;
  float zref, zs;
  unsigned long long qs;
  int wcnt;
  int atop;
  int hist_on;
  int cseq;
};

// End of an item (consumer threads): the item's summary and top list, then
// the row's finisher when this CTA is the last of the row to arrive.
template <typename E, bool SPLIT>
__device__ __noinline__ void item_end(const SpecArgs& a, int item, int slot, ItemAcc acc) {
  const Smem sm = smem_map();
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const ItemMeta& mt = sm.meta[slot];
  const uint32_t* tab = sm.tab + slot * kHmax;
  const int mode = mt.mode;
  const int row = mt.row;
  const int nkeep = mt.nkeep;
  const RowT& rt = mt.rt;
  uint32_t* bins_w = sm.radix + warp * 256;
  uint64_t* wbuf = sm.wbuf + warp * kWcap;
  const uint64_t* gov = a.ws.wovf + (static_cast<int64_t>(blockIdx.x) * kCW + warp) * kWovf;
  const float m_run = acc.m_run;
  const int arg_run = acc.arg_run;
  const int nal = acc.nal, bad = acc.bad, tmo = acc.tmo;
  const float zref = acc.zref, zs = acc.zs;
  const unsigned long long qs = acc.qs;
  int wcnt = acc.wcnt;
  const int atop = acc.atop;
  const bool hist_on = acc.hist_on != 0;
  if (mode != 0) {
    // each warp: drop the keys below the item's shared bound; a warp still
    // holding more than nkeep keeps its exact top-nkeep and shares its bound
    unsigned long long* tsh = &sm.ctl->tau_shared;
    if (wcnt <= kWcap) wcnt = warp_filter(wbuf, wcnt, *reinterpret_cast<volatile unsigned long long*>(tsh));
    if (wcnt > nkeep) {
      const uint64_t T = warp_compact(wbuf, gov, wcnt, nkeep, bins_w);
      wcnt = nkeep;
      if (lane == 0) atomicMax(tsh, static_cast<unsigned long long>(T));
    }
    cbar();
    // every bound is in: each warp keeps its keys >= the item's bound (<= nkeep)
    wcnt = warp_filter(wbuf, wcnt, sm.ctl->tau_shared);
  }
  // ---- one reduction round: per warp its max, allowed count, flags, mass
  // sums, and its softmax sum relative to its own max (sampled rows) or its
  // argmax (greedy rows); thread 0 combines the warps ----
  Red* rs = sm.red;
  unsigned long long* wq2 = reinterpret_cast<unsigned long long*>(sm.wcnt + 8);  // per-warp histogram totals
  {
    const float wm = warp_max(m_run);
    const int wn = warp_sum_i(nal);
    const uint32_t wf = (__any_sync(0xffffffffu, bad) ? 1u : 0u) | (__any_sync(0xffffffffu, tmo) ? 2u : 0u);
    unsigned long long q = qs, bsum = 0ull;
    if (mode == 2)
      for (int i = tid; i < kNB; i += kConsumers) bsum += sm.hmass[i];
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      q += __shfl_xor_sync(0xffffffffu, q, o);
      bsum += __shfl_xor_sync(0xffffffffu, bsum, o);
    }
    double wz = 0.0;
    if (mode == 0) {
      int wa = (m_run == wm && wm > RL_NEG_INF) ? arg_run : INT_MAX;
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) wa = min(wa, __shfl_xor_sync(0xffffffffu, wa, o));
      wz = static_cast<double>(wa);
    } else {
      double zl = 0.0;
      if (zref > RL_NEG_INF && wm > RL_NEG_INF)
        zl = static_cast<double>(zs) *
             exp2((static_cast<double>(zref) - static_cast<double>(wm)) * (kLog2e / static_cast<double>(rt.T)));
      wz = warp_sum_d(zl);
    }
    if (lane == 0) {
      rs->f[warp] = wm;
      rs->i[warp] = wn;
      rs->u[warp] = wf;
      rs->q[warp] = q;
      rs->d[warp] = wz;
      wq2[warp] = bsum;
      sm.wcnt[warp] = wcnt;
    }
  }
  cbar();
  float m_item = RL_NEG_INF;
  int nallow = 0;
  uint32_t fl = 0u;
  unsigned long long tq = 0ull, tb = 0ull;
#pragma unroll
  for (int w = 0; w < kCW; ++w) {
    m_item = fmaxf(m_item, rs->f[w]);
    nallow += rs->i[w];
    fl |= rs->u[w];
    tq += rs->q[w];
    tb += wq2[w];
  }
  const int badf = fl & 1u, tmof = (fl >> 1) & 1u;
  int argmax = INT_MAX;
  double z_item = 0.0;
  if (tid == 0) {
    // (only thread 0 writes the item's summary)
#pragma unroll
    for (int w = 0; w < kCW; ++w) {
      const float wm = rs->f[w];
      if (mode == 0) {
        if (wm == m_item && m_item > RL_NEG_INF) argmax = min(argmax, static_cast<int>(rs->d[w]));
      } else if (wm > RL_NEG_INF) {
        z_item += rs->d[w] * exp2((static_cast<double>(wm) - static_cast<double>(m_item)) *
                                  (kLog2e / static_cast<double>(rt.T)));
      }
    }
  }
  int hflags = 0;
  if (mode == 2 && (tq != tb || !hist_on)) hflags = kFlagHistBad;
  int ncand = 0;
  if (mode != 0) {
    // the warps' kept keys, flattened into the (free) radix area
    uint64_t* flat = reinterpret_cast<uint64_t*>(sm.radix);
    int total = 0, off = 0;
#pragma unroll
    for (int w = 0; w < kCW; ++w) {
      if (w < warp) off += sm.wcnt[w];
      total += sm.wcnt[w];
    }
    for (int i = lane; i < wcnt; i += 32) flat[off + i] = wbuf[i];
    cbar();
    const int need = min(total, nkeep);
    if (need > 0 && total <= kN) {
      // few keys: sorted in registers, in place
      csort_desc(flat, total, pow2_at_least(total));
      for (int t = tid; t < need; t += kConsumers) sm.top[t] = flat[t];
      cbar();
      ncand = need;
    } else if (need > 0) {
      // the need-th largest by a radix select over the kept keys, then
      // only the keys at or above it sorted
      if (tid == 0) sm.segn[0] = total;
      cbar();
      const uint64_t T = block_select<false>(flat, 1, total, sm.segn, need, reinterpret_cast<uint32_t*>(sm.wbuf),
                                             rs, sm.ctl);
      ncand = gather_sorted<false>(flat, 1, total, sm.segn, T, sm.top, sm.ctl);
    }
  }
  ItemSum is;
  is.m = m_item;
  is.argmax = argmax;
  is.nallow = nallow;
  is.flags = (badf ? kFlagBad : 0) | (tmof ? kFlagTimeout : 0) | hflags;
  is.z = z_item;
  is.ncand = ncand;
  is.atop = (mode == 2) ? atop : kNoAnchor;
  is.wlo = (mode == 2 && atop != kNoAnchor) ? atop - mt.wbins : 0;
  is.pad = 0;
  is.qsum = qs;
  const int first_item = row * a.nseg;
  if constexpr (SPLIT) {
    // the finish kernel merges the row's items: every item goes to the
    // workspace (with its sorted history table, for the rows that re-read)
    if (tid == 0) {
      a.ws.sums[item] = is;
      a.ws.tabn[item] = mt.ntab;
    }
    if (mode != 0) {
      uint32_t* gt = a.ws.tabs + static_cast<int64_t>(item) * kHmax;
      for (int i = tid; i < mt.ntab; i += kConsumers) gt[i] = tab[i];
    }
    uint64_t* gc = a.ws.cands + static_cast<int64_t>(item) * kN;
    for (int i = tid; i < ncand; i += kConsumers) gc[i] = sm.top[i];
    if (mode == 2) {
      uint32_t* gm = a.ws.hmass + static_cast<int64_t>(item) * kNB;
      uint32_t* gk = a.ws.hcnt + static_cast<int64_t>(item) * kNB;
      for (int i = tid; i < kNB; i += kConsumers) {
        gm[i] = sm.hmass[i];
        if (mt.need_count) gk[i] = sm.hcnt[i];
      }
    }
    (void)first_item;
    cbar();
    return;
  }
  bool run_finisher;
  if (a.nseg == 1) {
    if (tid == 0) sm.sums[0] = is;
    cbar();
    run_finisher = true;
  } else {
    if (tid == 0) a.ws.sums[item] = is;
    uint64_t* gc = a.ws.cands + static_cast<int64_t>(item) * kN;
    for (int i = tid; i < ncand; i += kConsumers) gc[i] = sm.top[i];
    if (mode == 2) {
      uint32_t* gm = a.ws.hmass + static_cast<int64_t>(item) * kNB;
      uint32_t* gk = a.ws.hcnt + static_cast<int64_t>(item) * kNB;
      for (int i = tid; i < kNB; i += kConsumers) {
        gm[i] = sm.hmass[i];
        if (mt.need_count) gk[i] = sm.hcnt[i];
      }
    }
    // the CTA's writes are ordered before the barrier; one thread's fence
    // then publishes them at device scope before the arrival
    cbar();
    if (tid == 0) {
      __threadfence();
      const int prev = atomicAdd(&a.ws.row_done[row], 1);
      __threadfence();
      sm.ctl->is_last = (prev == a.nseg - 1) ? 1 : 0;
    }
    cbar();
    run_finisher = sm.ctl->is_last != 0;
    if (run_finisher) {
      for (int s2 = tid; s2 < a.nseg; s2 += kConsumers) {
        const ItemSum* src = a.ws.sums + first_item + s2;
        ItemSum t;
        t.m = __ldcg(&src->m);
        t.argmax = __ldcg(&src->argmax);
        t.nallow = __ldcg(&src->nallow);
        t.flags = __ldcg(&src->flags);
        t.z = __ldcg(&src->z);
        t.ncand = __ldcg(&src->ncand);
        t.atop = __ldcg(&src->atop);
        t.wlo = __ldcg(&src->wlo);
        t.pad = 0;
        t.qsum = __ldcg(&src->qsum);
        sm.sums[s2] = t;
      }
      cbar();
    }
  }
  if (run_finisher) {
    finish_row<E, false>(a, mt, tab, first_item);
    if (a.nseg > 1 && tid == 0) a.ws.row_done[row] = 0;  // ready for the next launch
  }
  cbar();
}

// A warp's candidate buffer brought back to (about) nkeep keys: a bound from
// the top 16 value bits (two radix passes) keeps nkeep keys and the rest of
// their bucket; exact only when that is too many. Returns the new bound,
// shared through tau_shared.
//
// The warp also publishes a lower bound wk[warp] on the value key of its
// kw-th largest key (kw = ceil(nkeep / kCW)); the warps' elements are
// disjoint, so the union of every warp's top kw holds at least nkeep keys,
// all at or above min over the warps of wk: a bound on the item's nkeep-th
// largest key much closer to it than any one warp's nkeep-th (the warps see
// an eighth of the item each). wk only grows; a warp that has not published
// yet holds 0, which leaves the bound alone.
__device__ __noinline__ uint64_t compact_warp_buf(uint64_t* wbuf, const uint64_t* gov, int* wcnt, int nkeep,
                                                  uint32_t* bins_w, int* wc, unsigned long long* tau_shared,
                                                  uint32_t* wk) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int n = *wcnt;
  uint64_t tau = warp_select(wbuf, gov, n, nkeep, bins_w, 48);
  int kept = warp_count_ge(wbuf, gov, n, tau);
  if (kept > kWcompact - 64) {
    tau = warp_select(wbuf, gov, n, nkeep, bins_w);
    kept = nkeep;
  }
  warp_keep_ge(wbuf, gov, n, tau);
  *wcnt = kept;
  const int kw = (nkeep + kCW - 1) / kCW;
  uint64_t bw = 0ull;
  if (kept >= kw) bw = warp_select(wbuf, gov, kept, kw, bins_w, 48);  // <= the kw-th largest kept key
  if (lane == 0) {
    *wc = kept;
    atomicMax(tau_shared, static_cast<unsigned long long>(tau));
    volatile uint32_t* w = wk;
    const uint32_t v = static_cast<uint32_t>(bw >> 32);
    if (v > w[warp]) w[warp] = v;
    uint32_t u = 0xffffffffu;
#pragma unroll
    for (int i = 0; i < kCW; ++i) u = min(u, w[i]);
    if (u != 0u) atomicMax(tau_shared, static_cast<unsigned long long>(u) << 32);
  }
  __syncwarp();
  return tau;
}

// ---------------------------------------------------------------------------
// Consumer warps
// ---------------------------------------------------------------------------
// The chunks of one item (consumer threads), specialised per row mode so
// that each mode keeps only the state it needs in registers.
template <typename E, int MODE, bool SPLIT>
__device__ __noinline__ ItemAcc run_item(const SpecArgs& a, int slot, int cseq) {
  const Smem sm = smem_map();
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  constexpr int es = static_cast<int>(sizeof(E));
  const int V = a.V;
  const int base = warp * kSlice;
  uint32_t* bins_w = sm.radix + warp * 256;
  uint64_t* wbuf = sm.wbuf + warp * kWcap;
  uint64_t* gov = a.ws.wovf + (static_cast<int64_t>(blockIdx.x) * kCW + warp) * kWovf;
  const ItemMeta& mt = sm.meta[slot];
  const uint32_t* tab = sm.tab + slot * kHmax;
  constexpr int mode = MODE;
  const int row = mt.row;
  const RowT rt = mt.rt;
  const int nkeep = mt.nkeep;
  const int ntab = mt.ntab;
  const bool mask_on = mt.mask_on != 0;
  const E* rowp = reinterpret_cast<const E*>(a.logits) + static_cast<int64_t>(row) * a.ld;
  const uint32_t* mrow = a.mask ? a.mask + static_cast<int64_t>(row) * a.mask_stride : nullptr;
  // every chunk of the row shares the row's 16-byte alignment (chunks are
  // multiples of 16 bytes), so the copy warp's byte counts follow from it
  const bool row_al = (reinterpret_cast<uintptr_t>(rowp) & 15u) == 0;
  const bool mrow_al = mrow && (reinterpret_cast<uintptr_t>(mrow) & 15u) == 0;
  // running state
  float m_run = RL_NEG_INF;
  int arg_run = INT_MAX;
  int nal = 0, bad = 0, tmo = 0;
  float zref = RL_NEG_INF, zs = 0.0f;
  unsigned long long qs = 0ull;
  int wcnt = 0;
  uint64_t tau = 0ull;
  float tau_v = RL_NEG_INF;
  int atop = kNoAnchor;
  float atop_f = 0.0f, x_lo = RL_POS_INF;
  const float wb_f = static_cast<float>(mt.wbins);
  // item fields the loop needs live in registers: a shared-memory read after
  // a shared atomic waits for the atomic to complete
  const bool need_cnt = mt.need_count != 0;
  const uint32_t wb_u = static_cast<uint32_t>(mt.wbins);
  const int c0 = mt.c0, c1 = mt.c1;
  bool hist_on = MODE == 2;
  const int wtrig = min(kWcompact, max(2 * nkeep + 32, 128));
  int hp = ntab > 0 ? tab_lower_bound(tab, ntab, mt.c0 * kCE) : 0;
  if (mode == 2)
    for (int i = tid; i < kNB; i += kConsumers) {
      sm.hmass[i] = 0u;
      sm.hcnt[i] = 0u;
    }
  if (tid == 0) sm.ctl->tau_shared = 0ull;
  if (lane == 0) {
    sm.wcnt[warp] = 0;
    wk_of(sm)[warp] = 0u;
  }
  cbar();
  // RL_DEBUG_EXPIRE_WAIT: a bounded wait on a barrier that nothing
  // completes runs out, and the item reports a timeout like any wait would
  if ((a.debug_flags & 1) && !mbar_wait(sm.never, 0u, 2000)) tmo = 1;
  bool pre_patched = false;
  if constexpr (MODE != 0 && es == 4) {
    // bound from the item's first chunk (f32, whole in the stage, no mask):
    // its nkeep-th largest penalised value over all kCE logits, so that the
    // item appends about nkeep ln(n / kCE) keys in all
    const int start = mt.c0 * kCE;
    const int len = min(kCE, V - start);
    const int nfast = row_al ? ((len * es) & ~15) / es : 0;
    if (!mask_on && nfast == kCE) {
      const int s = cseq % kNS;
      float* f = reinterpret_cast<float*>(sm.stage + s * kStageBytes);
      // (split kernel: the row-preparation warp patched the stage already)
      if (mbar_wait(SPLIT ? &sm.ready[s] : &sm.full[s], static_cast<uint32_t>((cseq / kNS) & 1), kWaitBudget)) {
        const int lo = start + base, hi = lo + kSlice;
        while (!SPLIT && ntab > 0) {
          const int j = hp + lane;
          const uint32_t ent = j < ntab ? tab[j] : 0xffffffffu;
          const int id = static_cast<int>(ent >> 11);
          const bool below = j < ntab && id < hi;
          const bool mine = below && id >= lo && (ent & 2047u) != 0u;
          if (mine) f[id - start] = pen_value(f[id - start], static_cast<int>(ent & 2047u), mt.rp, mt.freq, mt.pres);
          pre_patched |= __any_sync(0xffffffffu, mine);
          const int adv = __popc(__ballot_sync(0xffffffffu, below));
          hp += adv;
          if (adv < 32) break;
        }
      }
      __syncwarp();
      cbar();  // every warp's penalties are in the stage
      const float t0 = block_kth_stage<float>(f, nkeep, sm.radix, sm.red, sm.ctl, nullptr);
      if (t0 > tau_v) {
        tau_v = t0;
        // every logit equal to t0 is kept (the key of +0.0 for a zero bound)
        tau = static_cast<uint64_t>(ord_key(__fadd_rn(t0, 0.0f))) << 32;
        if (tid == 0) atomicMax(&sm.ctl->tau_shared, static_cast<unsigned long long>(tau));
      }
    }
  }
  if constexpr (MODE != 0 && es == 2) {
    // the same bound for a bf16 item: the stage holds raw values (penalties
    // are applied in registers), so the chunk's history ids are left out --
    // the nkeep-th largest of the other logits, whose values are final, is
    // still a lower bound on the row's nkeep-th largest penalised value
    const int start = mt.c0 * kCE;
    const int len = min(kCE, V - start);
    const int nfast = row_al ? ((len * es) & ~15) / es : 0;
    if (!mask_on && nfast == kCE) {
      const int s = cseq % kNS;
      uint32_t* excl = sm.radix + 256;  // kCE bits, past the 256 select bins
      for (int i = tid; i < kCE / 32; i += kConsumers) excl[i] = 0u;
      cbar();
      if (ntab > 0) {
        const int j0 = tab_lower_bound(tab, ntab, start);
        for (int j = j0 + tid; j < ntab; j += kConsumers) {
          const int id = static_cast<int>(tab[j] >> 11);
          if (id >= start + kCE) break;  // the table is sorted by id
          atomicOr(&excl[(id - start) >> 5], 1u << ((id - start) & 31));
        }
      }
      cbar();
      if (mbar_wait(SPLIT ? &sm.ready[s] : &sm.full[s], static_cast<uint32_t>((cseq / kNS) & 1), kWaitBudget)) {
        const uint16_t* h = reinterpret_cast<const uint16_t*>(sm.stage + s * kStageBytes);
        const float t0 = block_kth_stage<uint16_t>(h, nkeep, sm.radix, sm.red, sm.ctl, excl);
        if (t0 > tau_v) {
          tau_v = t0;
          tau = static_cast<uint64_t>(ord_key(__fadd_rn(t0, 0.0f))) << 32;
          if (tid == 0) atomicMax(&sm.ctl->tau_shared, static_cast<unsigned long long>(tau));
        }
      } else {
        tmo = 1;
      }
    }
  }

  for (int c = c0; c < c1; ++c, ++cseq) {
    if (MODE != 0 && wcnt > wtrig) {
      // room for a whole slice of appends (no logits are live here); small
      // lists compact early, so that the union bound rises early
      tau = compact_warp_buf(wbuf, gov, &wcnt, nkeep, bins_w, sm.wcnt + warp, &sm.ctl->tau_shared, wk_of(sm));
      tau_v = key_val(tau);
    }
    const int s = cseq % kNS;
    const uint32_t ph = static_cast<uint32_t>((cseq / kNS) & 1);
    if (!mbar_wait(SPLIT ? &sm.ready[s] : &sm.full[s], ph, kWaitBudget)) tmo = 1;
    const int start = c * kCE;
    const int len = min(kCE, V - start);
    const int nfast = row_al ? ((len * es) & ~15) / es : 0;
    const int mfast = mrow_al ? ((((len + 31) >> 5) * 4) & ~15) / 4 : 0;
    E* stg = reinterpret_cast<E*>(sm.stage + s * kStageBytes);
    const uint32_t* mst = sm.maskst + s * kMaskWords;
    const int lo = start + base, hi = lo + kSlice;
    float v[4][4];
    // penalties patched into the stage (f32 slices entirely in the stage)
    const bool patch = (es == 4) && (base + kSlice <= nfast);
    bool patched = false;
    if (!SPLIT && ntab > 0 && patch) {
      float* f = reinterpret_cast<float*>(stg);
      while (true) {
        const int j = hp + lane;
        const uint32_t ent = j < ntab ? tab[j] : 0xffffffffu;
        const int id = static_cast<int>(ent >> 11);
        const bool below = j < ntab && id < hi;
        const bool mine = below && id >= lo && (ent & 2047u) != 0u;
        if (mine) f[id - start] = pen_value(f[id - start], static_cast<int>(ent & 2047u), mt.rp, mt.freq, mt.pres);
        patched |= __any_sync(0xffffffffu, mine);
        const int adv = __popc(__ballot_sync(0xffffffffu, below));
        hp += adv;
        if (adv < 32) break;
      }
      __syncwarp();
    }
    if (nfast == kCE) {
      // a whole aligned chunk: straight shared-memory loads
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const int el0 = base + (q * 32 + lane) * 4;
        if constexpr (es == 4) {
          const float4 f = *reinterpret_cast<const float4*>(reinterpret_cast<const float*>(stg) + el0);
          v[q][0] = f.x;
          v[q][1] = f.y;
          v[q][2] = f.z;
          v[q][3] = f.w;
        } else {
          const uint2 h = *reinterpret_cast<const uint2*>(reinterpret_cast<const uint16_t*>(stg) + el0);
          v[q][0] = __uint_as_float(h.x << 16);
          v[q][1] = __uint_as_float(h.x & 0xffff0000u);
          v[q][2] = __uint_as_float(h.y << 16);
          v[q][3] = __uint_as_float(h.y & 0xffff0000u);
        }
      }
    } else {
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      const int el0 = base + (q * 32 + lane) * 4;
      if (el0 < nfast) {
        if constexpr (es == 4) {
          const float4 f = *reinterpret_cast<const float4*>(reinterpret_cast<const float*>(stg) + el0);
          v[q][0] = f.x;
          v[q][1] = f.y;
          v[q][2] = f.z;
          v[q][3] = f.w;
        } else {
          const uint2 h = *reinterpret_cast<const uint2*>(reinterpret_cast<const uint16_t*>(stg) + el0);
          v[q][0] = __uint_as_float(h.x << 16);
          v[q][1] = __uint_as_float(h.x & 0xffff0000u);
          v[q][2] = __uint_as_float(h.y << 16);
          v[q][3] = __uint_as_float(h.y & 0xffff0000u);
        }
      } else {
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          const int el = el0 + k;
          v[q][k] = el < len ? to_f32<E>(__ldcg(rowp + start + el)) : RL_NEG_INF;
        }
      }
    }
    }
    uint32_t mbits[4] = {15u, 15u, 15u, 15u};
    if (mask_on) {
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const int el0 = base + (q * 32 + lane) * 4;
        const int wi = el0 >> 5;
        uint32_t word = 0u;
        if (wi < mfast) word = mst[wi];
        else if (el0 < len) word = __ldcg(mrow + (start >> 5) + wi);
        mbits[q] = (word >> ((lane & 7) * 4)) & 15u;
      }
    }
    // the stage is released: generic writes ordered before the next bulk copy
    if (patched || (c == c0 && pre_patched)) asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    __syncwarp();
    if (lane == 0) mbar_arrive(&sm.empty[s]);
    // penalties in registers (bf16, or slices partly outside the stage)
    if (ntab > 0 && !patch) pen_regs(v, lo, hi, tab, ntab, hp, mt);

    // ---- per-slice statistics ----
    float lm = RL_NEG_INF;
    if (mask_on) {
#pragma unroll
      for (int q = 0; q < 4; ++q)
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          const int el = base + (q * 32 + lane) * 4 + k;
          const bool allowed = el < len && ((mbits[q] >> k) & 1u);
          float x = allowed ? v[q][k] : RL_NEG_INF;
          if (allowed) {
            bad |= (x != x) || (x == RL_POS_INF);
            nal += (x > RL_NEG_INF) ? 1 : 0;
          }
          if (x != x) x = RL_NEG_INF;
          v[q][k] = x;
          lm = fmaxf(lm, x);
        }
    } else {
      // trees (depth 4) rather than 16-long dependent chains; the sum is
      // finite exactly when every logit is (or a huge finite sum overflows,
      // which the exact check below sorts out)
      float mx[8], sx[8];
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        mx[j] = fmaxf(v[j >> 1][(j & 1) * 2], v[j >> 1][(j & 1) * 2 + 1]);
        sx[j] = v[j >> 1][(j & 1) * 2] + v[j >> 1][(j & 1) * 2 + 1];
      }
#pragma unroll
      for (int w2 = 4; w2 > 0; w2 >>= 1)
#pragma unroll
        for (int j = 0; j < w2; ++j) {
          mx[j] = fmaxf(mx[j], mx[j + w2]);
          sx[j] = sx[j] + sx[j + w2];
        }
      lm = mx[0];
      if (fabsf(sx[0]) < RL_POS_INF) {
        nal += 16;
      } else {
        lm = RL_NEG_INF;
#pragma unroll
        for (int q = 0; q < 4; ++q)
#pragma unroll
          for (int k = 0; k < 4; ++k) {
            const int el = base + (q * 32 + lane) * 4 + k;
            float x = v[q][k];
            if (el < len) {
              bad |= (x != x) || (x == RL_POS_INF);
              nal += (x > RL_NEG_INF) ? 1 : 0;
            }
            if (x != x) x = RL_NEG_INF;
            v[q][k] = x;
            lm = fmaxf(lm, x);
          }
      }
    }
    if (mode == 0) {
      // a strictly larger maximum moves the lane's argmax (lowest id of it)
      if (lm > m_run) {
        int la = INT_MAX;
#pragma unroll
        for (int q = 3; q >= 0; --q)
#pragma unroll
          for (int k = 3; k >= 0; --k)
            if (v[q][k] == lm) la = start + base + (q * 32 + lane) * 4 + k;
        m_run = lm;
        arg_run = la;
      }
      continue;
    }
    m_run = fmaxf(m_run, lm);
    // ---- softmax sum (per-lane reference) ----
    if (lm > RL_NEG_INF) {
      if (zref == RL_NEG_INF) {
        zref = lm;
      } else if ((lm - zref) * rt.c > 8.0f) {
        zs *= ex2_approx((zref - lm) * rt.c);
        zref = lm;
      }
      const float zc = zref * rt.c;
      float z4[4] = {0.0f, 0.0f, 0.0f, 0.0f};
#pragma unroll
      for (int q = 0; q < 4; ++q)
#pragma unroll
        for (int k = 0; k < 4; ++k) z4[k] += ex2_approx(fmaf(v[q][k], rt.c, -zc));
      zs += (z4[0] + z4[1]) + (z4[2] + z4[3]);
    }
    // ---- candidates ----
    {
      const uint64_t ts = *reinterpret_cast<volatile unsigned long long*>(&sm.ctl->tau_shared);
      if (ts > tau) {
        tau = ts;
        tau_v = key_val(ts);
      }
      if (__any_sync(0xffffffffu, lm > RL_NEG_INF && lm >= tau_v)) {
        // the lane's takers as a 16-bit mask (every slot statically
        // indexed), their places in the warp's buffer from a warp scan of
        // the counts: no atomics
        unsigned hm = 0u;
#pragma unroll
        for (int q = 0; q < 4; ++q)
#pragma unroll
          for (int k = 0; k < 4; ++k) {
            const float x = v[q][k];
            bool take = x > RL_NEG_INF && x >= tau_v;
            if (take && !(x > tau_v))
              take = cand_key(x, static_cast<uint32_t>(start + base + (q * 32 + lane) * 4 + k)) >= tau;
            hm |= take ? (1u << (q * 4 + k)) : 0u;
          }
        const int nh = __popc(hm);
        int inc = nh;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
          const int t = __shfl_up_sync(0xffffffffu, inc, o);
          if (lane >= o) inc += t;
        }
        int idx = wcnt + inc - nh;
        wcnt += __shfl_sync(0xffffffffu, inc, 31);
        while (hm) {
          const int b = __ffs(hm) - 1;
          hm &= hm - 1u;
          const uint64_t key = cand_key(pick16(v, b), static_cast<uint32_t>(start + base + ((b >> 2) * 32 + lane) * 4 + (b & 3)));
          if (idx < kWcap) wbuf[idx] = key;
          else __stcg(reinterpret_cast<unsigned long long*>(gov + (idx - kWcap)), key);
          ++idx;
        }
        __syncwarp();
      }
    }
    // ---- windowed histogram ----
    if (hist_on) {
      if (atop == kNoAnchor) {
        // anchor on the first chunk with an allowed finite logit
        const float bm = cmax_f(lm, sm.red);
        if (bm > RL_NEG_INF) {
          const float af = bin_of(bm, rt);
          if (fabsf(af) < 4190000.0f) {
            atop = static_cast<int>(af) + kHead;
            atop_f = static_cast<float>(atop);
            x_lo = (atop_f - wb_f - 2.0f) / rt.cb_hi;  // logits below are outside the window
          } else {
            hist_on = false;
          }
        }
      }
      if (atop != kNoAnchor && __any_sync(0xffffffffu, lm >= x_lo)) {
        // straight-line per logit, only the atomics predicated: the window
        // offset r of the bin (bin_int), the position u of x in its bin and
        // the fixed-point mass from the cubic, rounded by the magic add; no
        // exp, floor or conversion instructions (quarter-rate pipes)
        const uint32_t K = static_cast<uint32_t>(atop) + kMagicBits;
        uint32_t q32 = 0u;  // <= 16 * 2^20 per chunk
        uint32_t rr[16], qq[16];
#pragma unroll
        for (int j = 0; j < 16; ++j) {
          const float x = v[j >> 2][j & 3];
          const float sb = __fadd_rn(__fmaf_rn(x, rt.cb_hi, -0.5f), kMagic);
          rr[j] = K - __float_as_uint(sb);
          const float u = __fmaf_rn(x, rt.cb_lo, __fmaf_rn(x, rt.cb_hi, -__fsub_rn(sb, kMagic)));
          const float pm = __fmaf_rn(__fmaf_rn(__fmaf_rn(kMq3, u, kMq2), u, kMq1), u, kMq0);
          qq[j] = __float_as_uint(__fadd_rn(pm, kMagic)) - kMagicBits;
          q32 += rr[j] <= wb_u ? qq[j] : 0u;
        }
        // the window's atomics back to back, predicated (no branches)
        const uint32_t hb = smem_u32(sm.hmass);
#pragma unroll
        for (int j = 0; j < 16; ++j)
          asm volatile("{ .reg .pred p; setp.le.u32 p, %0, %1; @p red.shared.add.u32 [%2], %3; }" ::"r"(rr[j]), "r"(wb_u),
                       "r"(hb + 4u * rr[j]), "r"(qq[j])
                       : "memory");
        if (need_cnt) {
          const uint32_t cb = smem_u32(sm.hcnt);
#pragma unroll
          for (int j = 0; j < 16; ++j)
            asm volatile("{ .reg .pred p; setp.le.u32 p, %0, %1; @p red.shared.add.u32 [%2], 1; }" ::"r"(rr[j]), "r"(wb_u),
                         "r"(cb + 4u * rr[j])
                         : "memory");
        }
        qs += q32;
      }
    }
  }

  ItemAcc acc;
  acc.m_run = m_run;
  acc.arg_run = arg_run;
  acc.nal = nal;
  acc.bad = bad;
  acc.tmo = tmo;
  acc.zref = zref;
  acc.zs = zs;
  acc.qs = qs;
  acc.wcnt = wcnt;
  acc.atop = atop;
  acc.hist_on = hist_on ? 1 : 0;
  acc.cseq = cseq;
  return acc;
}

template <typename E, bool SPLIT>
__device__ __noinline__ void consumer_loop(const SpecArgs& a) {
  const Smem sm = smem_map();
  const int tid = threadIdx.x;
  int cseq = 0;
  for (int mseq = 0;; ++mseq) {
    const int item = blockIdx.x + mseq * gridDim.x;
    if (item >= a.nitems) return;
    const int slot = mseq & 1;
    const bool timeout = !mbar_wait(&sm.mfull[slot], static_cast<uint32_t>((mseq >> 1) & 1), kWaitBudget);
    if (cor_i(timeout || *reinterpret_cast<volatile int*>(&sm.ctl->abort), sm.red)) {
      if (tid == 0) {
        atomicExch(&sm.ctl->abort, 1);
        // items of this CTA that will not be streamed
        for (int it = item; it < a.nitems; it += gridDim.x) {
          if constexpr (SPLIT) {
            ItemSum t = {};
            t.m = RL_NEG_INF;
            t.argmax = INT_MAX;
            t.flags = kFlagTimeout;
            t.atop = kNoAnchor;
            a.ws.sums[it] = t;
          } else if ((it % a.nseg) == 0) {
            write_row(a, it / a.nseg, RL_ERR_TIMEOUT, -1, 0.0f);
          }
        }
      }
      return;
    }
    const int mode = sm.meta[slot].mode;
    if (sm.meta[slot].ntab > 0) {
      if constexpr (SPLIT) {
        block_sort_table(sm.tab + slot * kHmax, sm.meta[slot].ntab);
        // the row-preparation warp patches the stages with this table
        if (tid == 0) {
          __threadfence_block();
          *reinterpret_cast<volatile int*>(&sm.ctl->tab_seq) = mseq + 1;
        }
      } else {
        sort_table(sm.tab + slot * kHmax, sm.meta[slot].ntab);
      }
    }
    ItemAcc acc;
    if (mode == 0) acc = run_item<E, 0, SPLIT>(a, slot, cseq);
    else if (mode == 1) acc = run_item<E, 1, SPLIT>(a, slot, cseq);
    else acc = run_item<E, 2, SPLIT>(a, slot, cseq);
    cseq = acc.cseq;
    item_end<E, SPLIT>(a, item, slot, acc);
    // the row data of this slot may be rebuilt
    if ((tid & 31) == 0) mbar_arrive(&sm.mempty[slot]);
  }
}

// ---------------------------------------------------------------------------
// The kernel
// ---------------------------------------------------------------------------
template <typename E, bool SPLIT>
__global__ void __launch_bounds__(kThreads, 2) spec_pipe_kernel(const __grid_constant__ SpecArgs a) {
  const Smem sm = smem_map();
  if (threadIdx.x == 0) {
    for (int s = 0; s < kNS; ++s) {
      mbar_init(&sm.full[s], 1);
      mbar_init(&sm.empty[s], kCW);
    }
    for (int s = 0; s < 2; ++s) {
      mbar_init(&sm.mfull[s], 1);
      mbar_init(&sm.mempty[s], kCW);
    }
    for (int s = 0; s < kNS; ++s) mbar_init(&sm.ready[s], 1);
    mbar_init(sm.never, 1);
    sm.ctl->abort = 0;
    sm.ctl->tab_seq = 0;
    fence_mbar_init();
  }
  __syncthreads();
  // a dependent finish grid may be scheduled as soon as resources free up
  // (it waits for this grid's completion before reading its outputs)
  if (SPLIT) asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  const int warp = threadIdx.x >> 5;
  if (warp == kProdWarp) producer_loop<E>(a);
  else if (warp == kMetaWarp) meta_loop<E, SPLIT>(a);
  else consumer_loop<E, SPLIT>(a);
}

// The finish kernel: one CTA of kConsumers threads per row merges the row's
// item summaries, top lists and histograms written by the streaming kernel
// and draws the token (the same finisher the single-kernel path runs inline).
template <typename E>
__global__ void __launch_bounds__(kConsumers, 2) spec_finish_kernel(const __grid_constant__ SpecArgs a) {
  const Smem sm = smem_map();
  const int tid = threadIdx.x;
  const int row = blockIdx.x;
  const int first_item = row * a.nseg;
  if (tid < 32) build_meta(a, first_item, sm.meta[0], sm.tab, true);
  // the row's parameters come from the caller; everything below comes from
  // the streaming kernel
  asm volatile("griddepcontrol.wait;" ::: "memory");
  for (int s2 = tid; s2 < a.nseg; s2 += kConsumers) {
    const ItemSum* src = a.ws.sums + first_item + s2;
    ItemSum t;
    t.m = __ldcg(&src->m);
    t.argmax = __ldcg(&src->argmax);
    t.nallow = __ldcg(&src->nallow);
    t.flags = __ldcg(&src->flags);
    t.z = __ldcg(&src->z);
    t.ncand = __ldcg(&src->ncand);
    t.atop = __ldcg(&src->atop);
    t.wlo = __ldcg(&src->wlo);
    t.pad = 0;
    t.qsum = __ldcg(&src->qsum);
    sm.sums[s2] = t;
  }
  __syncthreads();
  const ItemMeta& mt = sm.meta[0];
  if (mt.ntab > 0) sort_table(sm.tab, mt.ntab);
  if (a.nseg == 1) {
    // a one-segment row: its list and histogram where the finisher expects
    // them (shared memory)
    const int nc = sm.sums[0].ncand;
    for (int i = tid; i < nc; i += kConsumers) sm.top[i] = __ldcg(a.ws.cands + static_cast<int64_t>(first_item) * kN + i);
    if (mt.mode == 2) {
      const uint32_t* gm = a.ws.hmass + static_cast<int64_t>(first_item) * kNB;
      const uint32_t* gk = a.ws.hcnt + static_cast<int64_t>(first_item) * kNB;
      for (int i = tid; i < kNB; i += kConsumers) {
        sm.hmass[i] = __ldcg(gm + i);
        sm.hcnt[i] = mt.need_count ? __ldcg(gk + i) : 0u;
      }
    }
  }
  __syncthreads();
  finish_row<E, true>(a, mt, sm.tab, first_item);
}

// ---------------------------------------------------------------------------
// Host side
// ---------------------------------------------------------------------------
void spec_plan(int B, int V, int num_sms, int* nseg, int* cps, int* nctas) {
  const int slots = 2 * num_sms;
  const int S = spec_chunks(V);
  int ns = 1;
  if (B > 0 && B < slots) ns = max(1, min(min(S, kSmax), slots / B));
  const int c = (S + ns - 1) / ns;
  ns = (S + c - 1) / c;
  *nseg = ns;
  *cps = c;
  *nctas = max(1, min(B * ns, slots));
}

int spec_max_ws_items(int num_sms, int max_batch) { return max(2 * (2 * num_sms), max_batch); }

template <typename E, bool SPLIT>
static cudaError_t launch_typed(const SpecArgs& a, int nctas, cudaStream_t stream, cudaEvent_t* ev = nullptr) {
  // the kernels' shared-memory limit, set once per device (a per-device
  // flag read and written atomically: several host threads may launch)
  static std::atomic<int> configured[64];
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64 || !configured[dev].load(std::memory_order_acquire)) {
    cudaError_t e =
        cudaFuncSetAttribute(spec_pipe_kernel<E, SPLIT>, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemBytes);
    if (e == cudaSuccess && SPLIT)
      e = cudaFuncSetAttribute(spec_finish_kernel<E>, cudaFuncAttributeMaxDynamicSharedMemorySize, kOffStage);
    if (e != cudaSuccess) return e;
    if (dev >= 0 && dev < 64) configured[dev].store(1, std::memory_order_release);
  }
  if (ev) cudaEventRecord(ev[0], stream);
  spec_pipe_kernel<E, SPLIT><<<nctas, kThreads, kSmemBytes, stream>>>(a);
  if (ev) cudaEventRecord(ev[1], stream);
  if (SPLIT) {
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return e;
    // programmatic dependent launch: the finish kernel's CTAs are scheduled
    // as the streaming kernel's CTAs retire and prepare their row while the
    // last ones run; they read the streaming kernel's outputs only after
    // the grid-dependency wait (which waits for that grid to complete)
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(static_cast<unsigned>(a.B));
    cfg.blockDim = dim3(kConsumers);
    cfg.dynamicSmemBytes = kOffStage;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    e = cudaLaunchKernelEx(&cfg, spec_finish_kernel<E>, a);
    if (e != cudaSuccess) return e;
    if (ev) cudaEventRecord(ev[2], stream);
  }
  return cudaGetLastError();
}

cudaError_t spec_configure_single() {
  cudaError_t e = cudaFuncSetAttribute(spec_pipe_kernel<float, false>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       kSmemBytes);
  if (e == cudaSuccess)
    e = cudaFuncSetAttribute(spec_pipe_kernel<uint16_t, false>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             kSmemBytes);
  return e;
}

cudaError_t launch_spec(const SpecArgs& args, int dtype, int num_sms, cudaStream_t stream, cudaEvent_t* ev) {
  if (args.B == 0) return cudaSuccess;
  SpecArgs a = args;
  int nctas = 0;
  spec_plan(a.B, a.V, num_sms, &a.nseg, &a.cps, &nctas);
  a.nitems = a.B * a.nseg;
  if (a.nitems > a.ws.max_items) return cudaErrorInvalidValue;
  return dtype == RL_BF16 ? launch_typed<uint16_t, true>(a, nctas, stream, ev)
                          : launch_typed<float, true>(a, nctas, stream, ev);
}

cudaError_t launch_spec_single(const SpecArgs& args, int dtype, int num_sms, int max_ctas, cudaStream_t stream) {
  if (args.B == 0) return cudaSuccess;
  SpecArgs a = args;
  a.nseg = 1;
  a.cps = spec_chunks(a.V);
  a.nitems = a.B;
  const int nctas = max(1, min(min(a.B, 2 * num_sms), max_ctas));
  return dtype == RL_BF16 ? launch_typed<uint16_t, false>(a, nctas, stream)
                          : launch_typed<float, false>(a, nctas, stream);
}

// ---------------------------------------------------------------------------
// Beam step: the rows' partial results combined per item (BeamSearch::search,
// src/decoder.rs:227-270). One CTA of kConsumers threads per item.
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(kConsumers) beam_combine_kernel(const __grid_constant__ BeamArgs b) {
  __shared__ float cs[kBeamMaxCand];
  __shared__ int co[kBeamMaxCand];
  __shared__ int ct[kBeamMaxCand];
  __shared__ unsigned char cdn[kBeamMaxCand];
  __shared__ int nc;
  const int item = blockIdx.x, tid = threadIdx.x;
  const int k = 2 * b.beams;
  if (tid == 0) nc = 0;
  __syncthreads();
  // candidates in the reference's push order: beam ascending, then the beam's
  // list order (value desc, id asc); order key = beam * 64 + position
  for (int f = tid; f < b.beams * k; f += blockDim.x) {
    const int bm = f / k, j = f - bm * k;
    const int row = item * b.beams + bm;
    if (b.done[row]) {
      if (j == 0) {
        const int i = atomicAdd(&nc, 1);
        cs[i] = b.scores[row];
        co[i] = bm * 64;
        ct[i] = -1;
        cdn[i] = 1;
      }
      continue;
    }
    const PartStats ps = b.stats[row];
    if (j >= ps.nt) continue;
    const uint64_t key = b.keys[static_cast<int64_t>(row) * kN + j];
    const float x = key_val(key);
    float v = x;
    if (b.log_softmax) {
      const float lse = static_cast<float>(static_cast<double>(ps.m) + log(ps.z));
      v = __fsub_rn(x, lse);
    }
    float lp = 1.0f;
    if (b.alpha != 1.0f) lp = powf(__fdiv_rn(__fadd_rn(static_cast<float>(b.lens[row] + 1), 6.0f), 6.0f), b.alpha);
    const int id = static_cast<int>(key_id(key));
    const int i = atomicAdd(&nc, 1);
    cs[i] = __fdiv_rn(__fadd_rn(b.scores[row], v), lp);
    co[i] = bm * 64 + j;
    ct[i] = id;
    cdn[i] = id == b.eos ? 1 : 0;
  }
  __syncthreads();
  const int n = nc;
  for (int i = tid; i < n; i += blockDim.x) {
    const float sc = cs[i];
    const int oi = co[i];
    int rank = 0;
    for (int j = 0; j < n; ++j) rank += (cs[j] > sc || (!(cs[j] < sc) && !(cs[j] > sc) && co[j] < oi)) ? 1 : 0;
    if (rank < b.n_out) {
      const int64_t o = static_cast<int64_t>(item) * b.n_out + rank;
      b.out_beam[o] = oi >> 6;
      b.out_tok[o] = ct[i];
      b.out_score[o] = sc;
      b.out_done[o] = cdn[i];
    }
  }
  for (int r = n + tid; r < b.n_out; r += blockDim.x) {
    const int64_t o = static_cast<int64_t>(item) * b.n_out + r;
    b.out_beam[o] = -1;
    b.out_tok[o] = -1;
    b.out_score[o] = RL_NEG_INF;
    b.out_done[o] = 0;
  }
}

cudaError_t launch_beam_combine(const BeamArgs& b, cudaStream_t stream) {
  if (b.items == 0) return cudaSuccess;
  beam_combine_kernel<<<b.items, kConsumers, 0, stream>>>(b);
  return cudaGetLastError();
}

// ---------------------------------------------------------------------------
// Vocabulary shards: the G partial results of each row merged, then the
// finisher's cutoff and draw. One CTA of kConsumers threads per row.
// ---------------------------------------------------------------------------
// Shard g's keys and summary of row r (separate arrays, or packed records
// as one all-gather lays them out).
__device__ __forceinline__ const uint64_t* merge_keys(const MergeArgs& m, int g, int row) {
  return m.keys + (static_cast<int64_t>(g) * m.B + row) * (m.stats ? kN : kRec);
}
__device__ __forceinline__ PartStats merge_stats(const MergeArgs& m, int g, int row) {
  if (m.stats) return m.stats[static_cast<int64_t>(g) * m.B + row];
  return *reinterpret_cast<const PartStats*>(merge_keys(m, g, row) + kN);
}

__global__ void __launch_bounds__(kConsumers) shard_merge_kernel(const __grid_constant__ MergeArgs m) {
  __shared__ uint64_t keys[kMergeMax];
  __shared__ uint64_t top[kN];
  __shared__ double cum[kN];
  __shared__ float ev[kN];
  __shared__ double wsum[kCW];
  __shared__ int cnt;
  const int row = blockIdx.x, tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const rl_row_params prm = m.params[row];
  const float T = prm.temperature;
  // row summary over the shards (argmax: lowest global id at the max)
  float M = RL_NEG_INF;
  int argmax = INT_MAX, nallow = 0, flags = 0;
  for (int g = 0; g < m.G; ++g) {
    const PartStats ps = merge_stats(m, g, row);
    nallow += ps.nallow;
    flags |= ps.flags;
    if (ps.nallow == 0) continue;
    if (ps.m > M) {
      M = ps.m;
      argmax = ps.argmax;
    } else if (ps.m == M) {
      argmax = min(argmax, ps.argmax);
    }
  }
  int status = 0;
  if (flags & kFlagTimeout) status = RL_ERR_TIMEOUT;
  else if ((flags & kFlagBad) || nallow == 0 || !(fabsf(T) < RL_POS_INF)) status = RL_ERR_NONFINITE;
  const bool greedy = !(T > 0.0f);
  if (!greedy && status == 0 && !(prm.top_k > 0 && prm.top_k <= kN)) status = RL_ERR_UNSUPPORTED;
  if (status != 0 || greedy) {
    if (tid == 0) {
      m.out_tok[row] = status == 0 ? argmax : -1;
      if (m.out_prob) m.out_prob[row] = status == 0 ? 1.0f : 0.0f;
      if (m.row_status) m.row_status[row] = status;
    }
    return;
  }
  const RowT rt = make_rowt(T);
  const double cd = kLog2e / static_cast<double>(T);
  double Z = 0.0;
  for (int g = 0; g < m.G; ++g) {
    const PartStats ps = merge_stats(m, g, row);
    if (ps.nallow > 0 && ps.m > RL_NEG_INF) Z += ps.z * exp2((static_cast<double>(ps.m) - static_cast<double>(M)) * cd);
  }
  const int K = min(prm.top_k, nallow);
  // a shard list holding K keys bounds the row's K-th key by its K-th one
  uint64_t bound = 0ull;
  for (int g = 0; g < m.G; ++g) {
    const PartStats ps = merge_stats(m, g, row);
    if (ps.nt >= K) {
      const uint64_t kk = merge_keys(m, g, row)[K - 1];
      bound = kk > bound ? kk : bound;
    }
  }
  if (tid == 0) cnt = 0;
  __syncthreads();
  for (int f = tid; f < m.G * kN; f += blockDim.x) {
    const int g = f / kN, j = f - g * kN;
    const PartStats ps = merge_stats(m, g, row);
    if (j >= ps.nt) continue;
    const uint64_t kk = merge_keys(m, g, row)[j];
    if (kk >= bound) keys[atomicAdd(&cnt, 1)] = kk;  // at most G * kN keys
  }
  __syncthreads();
  const int n = cnt;
  for (int i = tid; i < n; i += blockDim.x) {
    const uint64_t kk = keys[i];
    int r = 0;
    for (int j = 0; j < n; ++j) r += keys[j] > kk ? 1 : 0;
    if (r < K) top[r] = kk;
  }
  __syncthreads();
  // exact e and the inclusive cumulative probabilities of the K keys
  float e = 0.0f;
  double s = 0.0;
  if (tid < K) {
    e = exact_e(key_val(top[tid]), M, rt);
    s = static_cast<double>(e) / Z;
  }
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const double t = __shfl_up_sync(0xffffffffu, s, o);
    if (lane >= o) s += t;
  }
  if (lane == 31) wsum[warp] = s;
  __syncthreads();
  double before = 0.0;
  for (int w = 0; w < warp; ++w) before += wsum[w];
  if (tid < K) {
    cum[tid] = before + s;
    ev[tid] = e;
  }
  __syncthreads();
  if (tid == 0) {
    // inclusive top-p cutoff (first cum >= p), then the strict draw
    // (first cum > u * S), as the one-row finisher does
    int cut = K - 1;
    if (prm.top_p < 1.0f) {
      const double pd = static_cast<double>(prm.top_p);
      for (int j = 0; j < K; ++j)
        if (cum[j] >= pd) {
          cut = j;
          break;
        }
    }
    const double S = cum[cut];
    const double tgt = static_cast<double>(m.uniforms[row]) * S;
    int d = cut;
    for (int j = 0; j <= cut; ++j)
      if (cum[j] > tgt) {
        d = j;
        break;
      }
    m.out_tok[row] = static_cast<int>(key_id(top[d]));
    if (m.out_prob) m.out_prob[row] = static_cast<float>((static_cast<double>(ev[d]) / Z) / S);
    if (m.row_status) m.row_status[row] = 0;
  }
}

cudaError_t launch_shard_merge(const MergeArgs& m, cudaStream_t stream) {
  if (m.B == 0) return cudaSuccess;
  shard_merge_kernel<<<m.B, kConsumers, 0, stream>>>(m);
  return cudaGetLastError();
}

__global__ void fill_params_kernel(rl_row_params* p, int n, int top_k) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i < n) {
    rl_row_params q;
    q.temperature = 1.0f;
    q.top_p = 1.0f;
    q.top_k = top_k;
    q.repeat_penalty = 1.0f;
    q.presence_penalty = 0.0f;
    q.frequency_penalty = 0.0f;
    p[i] = q;
  }
}

cudaError_t launch_fill_params(rl_row_params* p, int n, int top_k, cudaStream_t stream) {
  fill_params_kernel<<<(n + 255) / 256, 256, 0, stream>>>(p, n, top_k);
  return cudaGetLastError();
}

}  // namespace rl
