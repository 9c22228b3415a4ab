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
// Design (B200, sm_100a). One launch; the grid is (chunks, rows). Every CTA
// streams one 64 KB chunk of one row into shared memory with bulk async
// copies (cp.async.bulk + mbarrier) -- the only HBM read of those logits --
// and reduces it to a small summary in the handle's workspace:
//   P1  chunk max / lowest argmax / allowed count / per-thread maxima
//   P2  Z partial sum of exp((x - m_c)/T) (ex2 on a split log2(e)/T), and for
//       rows without a small top_k, count + mass histograms on an absolute
//       bin grid (16 bins per nat)
//   P3  candidate keys (value desc, id asc) of everything that can be in the
//       row's top-k: x >= tau, tau = k-th largest per-thread maximum (k <= 128),
//       or the chunk's top 512 by the histogram.
// The last CTA of a row to finish (arrival counter) merges the summaries:
// global max, Z, the exact top-k list (sorted keys, exact exp), the inclusive
// top-p cutoff and the draw. Rows without a small top_k walk the merged
// histogram bin by bin; a bin not covered by the candidate lists is re-read
// from the (L2-resident) row.
#include <climits>

#include "common.cuh"
#include "spec_kernel.cuh"

namespace rl {

constexpr uint16_t kBf16Marker = 0x7fc1;  // bf16 slot whose penalised value is in the side table
constexpr uint16_t kBf16NegInf = 0xff80;
constexpr double kLog2e = 1.4426950408889634074;

// ---------------------------------------------------------------------------
// Row arithmetic
// ---------------------------------------------------------------------------
struct RowT {
  float T, rT;       // temperature, RN(1/T)
  bool fast_div;     // Markstein division valid for T
  float c_hi, c_lo;  // log2(e)/T split in two floats
  float cb;          // absolute bins per logit unit: kRbin / T
};

__device__ __forceinline__ RowT make_rowt(float T) {
  RowT r;
  r.T = T;
  r.rT = __frcp_rn(T);
  r.fast_div = (T >= 9.5367431640625e-07f) && (T <= 1048576.0f);
  const double c = kLog2e / static_cast<double>(T);
  r.c_hi = static_cast<float>(c);
  r.c_lo = static_cast<float>(c - static_cast<double>(r.c_hi));
  r.cb = div_rn(kRbin, T);
  return r;
}
// l = (x - m) / T with IEEE rounding, as the CPU restatement computes it.
__device__ __forceinline__ float exact_l(float x, float m, const RowT& r) {
  const float d = sub_rn(x, m);
  if (r.fast_div && (d == 0.0f || fabsf(d) >= 8.077935669e-28f)) return div_fixed(d, r.T, r.rT);
  return div_rn(d, r.T);
}
__device__ __forceinline__ float exact_e(float x, float m, const RowT& r) { return expf(exact_l(x, m, r)); }
__device__ __forceinline__ float ex2_approx(float t) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(t));
  return y;
}
// exp((x - m)/T) for bulk sums: split-constant exponent, hardware ex2.
__device__ __forceinline__ float fast_e(float x, float m, const RowT& r) {
  const float d = sub_rn(x, m);
  return ex2_approx(fmaf(d, r.c_lo, d * r.c_hi));
}
// Absolute bin of a logit: monotone in x, identical wherever it is computed.
__device__ __forceinline__ int babs(float x, const RowT& r) {
  return __float2int_rd(__fmul_rn(x, r.cb));
}

// ---------------------------------------------------------------------------
// Chunk access: values of G consecutive elements per 16-byte shared load.
// ---------------------------------------------------------------------------
template <typename E>
struct Slice;

template <>
struct Slice<float> {
  static constexpr int G = 4;
  const float* data;
  __device__ __forceinline__ void load(int g, float (&v)[4]) const {
    const float4 q = reinterpret_cast<const float4*>(data)[g];
    v[0] = q.x;
    v[1] = q.y;
    v[2] = q.z;
    v[3] = q.w;
  }
};

template <>
struct Slice<uint16_t> {
  static constexpr int G = 8;
  const uint16_t* data;
  const int32_t* pen_id;  // local ids of penalised entries (-1: duplicate)
  const float* pen_val;
  int n_pen;
  __device__ __noinline__ float lookup(int local) const {
    for (int t = 0; t < n_pen; ++t)
      if (pen_id[t] == local) return pen_val[t];
    return __int_as_float(0x7fffffff);
  }
  __device__ __forceinline__ void load(int g, float (&v)[8]) const {
    const uint4 q = reinterpret_cast<const uint4*>(data)[g];
    const uint32_t w[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const uint32_t lo = w[k] & 0xffffu, hi = w[k] >> 16;
      v[2 * k] = (lo == kBf16Marker) ? lookup(g * 8 + 2 * k) : bf16_bits_to_f32(lo);
      v[2 * k + 1] = (hi == kBf16Marker) ? lookup(g * 8 + 2 * k + 1) : bf16_bits_to_f32(hi);
    }
  }
};

// ---------------------------------------------------------------------------
// Block helpers (kCT threads)
// ---------------------------------------------------------------------------
struct RedScratch {
  double d[kCW];
  float f[kCW];
  int i[kCW];
  int j[kCW];
  int k[kCW];
  double bcast_d;
  int bcast_i;
  int pad;
};

__device__ __forceinline__ double block_sum_d(double v, RedScratch* rs) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  v = warp_sum_d(v);
  __syncthreads();
  if (lane == 0) rs->d[warp] = v;
  __syncthreads();
  if (warp == 0) {
    double t = lane < kCW ? rs->d[lane] : 0.0;
    t = warp_sum_d(t);
    if (lane == 0) rs->bcast_d = t;
  }
  __syncthreads();
  return rs->bcast_d;
}

__device__ __forceinline__ int block_min_i(int v, RedScratch* rs) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = min(v, __shfl_xor_sync(0xffffffffu, v, o));
  __syncthreads();
  if (lane == 0) rs->i[warp] = v;
  __syncthreads();
  if (warp == 0) {
    int t = lane < kCW ? rs->i[lane] : INT_MAX;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) t = min(t, __shfl_xor_sync(0xffffffffu, t, o));
    if (lane == 0) rs->bcast_i = t;
  }
  __syncthreads();
  return rs->bcast_i;
}

__device__ __forceinline__ int block_or_i(int v, RedScratch* rs) {
  v = __any_sync(0xffffffffu, v != 0);
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  __syncthreads();
  if (lane == 0) rs->i[warp] = v;
  __syncthreads();
  if (warp == 0) {
    int t = lane < kCW ? rs->i[lane] : 0;
    t = __any_sync(0xffffffffu, t != 0);
    if (lane == 0) rs->bcast_i = t;
  }
  __syncthreads();
  return rs->bcast_i;
}

// Inclusive block scan of doubles (one value per thread); *total = block sum.
__device__ __forceinline__ double block_scan_d(double v, RedScratch* rs, double* total) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const double n = __shfl_up_sync(0xffffffffu, v, o);
    if (lane >= o) v += n;
  }
  __syncthreads();
  if (lane == 31) rs->d[warp] = v;
  __syncthreads();
  if (warp == 0) {
    double t = lane < kCW ? rs->d[lane] : 0.0;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const double n = __shfl_up_sync(0xffffffffu, t, o);
      if (lane >= o) t += n;
    }
    if (lane < kCW) rs->d[lane] = t;
  }
  __syncthreads();
  const double off = warp > 0 ? rs->d[warp - 1] : 0.0;
  *total = rs->d[kCW - 1];
  return v + off;
}

// Descending bitonic sort of P (power of two) keys in shared memory.
template <typename K>
__device__ void block_sort_desc(K* s, int P) {
  for (int k = 2; k <= P; k <<= 1) {
    for (int j = k >> 1; j > 0; j >>= 1) {
      for (int i = threadIdx.x; i < P; i += kCT) {
        const int ixj = i ^ j;
        if (ixj > i) {
          const K a = s[i], b = s[ixj];
          const bool desc = (i & k) == 0;
          if (desc ? (a < b) : (a > b)) {
            s[i] = b;
            s[ixj] = a;
          }
        }
      }
      __syncthreads();
    }
  }
}

__device__ __forceinline__ int pow2_ceil(int n) {
  int p = 1;
  while (p < n) p <<= 1;
  return p;
}

// ---------------------------------------------------------------------------
// Shared-memory layout
// ---------------------------------------------------------------------------
struct Ctrl {
  int n_local;   // history entries inside the chunk
  int ncand;     // candidate keys written
  int is_last;
  int mask_on;
  int overflow;
  int nbin;      // keys gathered for the current bin (finisher)
  int pad[2];
};

// Finisher walk state (rank of the row's list, masses relative to the row max).
struct Walk {
  int phase;              // 0: find the cutoff, 1: find the draw, 2: done
  int K;                  // list length
  int mass_mode;          // top_p < 1
  int cut_in_seg;         // the cutoff element is in the current segment
  int cut_idx;
  int status;
  int token;
  float prob;
  long long count_before;
  double mass_before;
  double Z, t2, S, t3;
};

constexpr int kOffMbar = 0;
constexpr int kOffCtrl = 64;
constexpr int kOffWalk = 128;
constexpr int kOffRed = 256;
constexpr int kOffTmax = 1024;                 // kCT floats
constexpr int kOffCnt = kOffTmax + kCT * 4;    // kNB u32 / finisher: kNB doubles (counts)
constexpr int kOffMass = kOffCnt + kNB * 8;    // kNB u64 / finisher: kNB doubles (masses)
constexpr int kOffHist = kOffMass + kNB * 8;   // kHmax ints
constexpr int kOffPen = kOffHist + kHmax * 4;  // kHmax floats
constexpr int kOffSums = kOffPen + kHmax * 4;  // kSmax ChunkSum (finisher)
constexpr int kOffData = ((kOffSums + kSmax * static_cast<int>(sizeof(ChunkSum)) + 127) / 128) * 128;
static_assert(sizeof(Walk) <= 128, "walk");
static_assert(kOffRed + sizeof(RedScratch) <= kOffTmax, "smem header");

int spec_smem_bytes(int /*es*/) { return kOffData + kChunkBytes; }
int spec_chunks(int V, int es) {
  const int ce = kChunkBytes / es;
  return (V + ce - 1) / ce;
}

// ---------------------------------------------------------------------------
// Finisher pieces
// ---------------------------------------------------------------------------
// Sweep over n sorted keys: first index j whose cumulative mass
// (w.mass_before + e_0 + ... + e_j, e exact) meets the condition. mode 0:
// cutoff (list position K-1, or cum >= t2 in mass mode); mode 1: cum > t3.
__device__ int sweep(const uint64_t* keys, int n, const Walk& w, float m, const RowT& rt, int mode,
                     RedScratch* rs, double* cum_at) {
  double run = w.mass_before;
  for (int c0 = 0; c0 < n; c0 += kCT) {
    const int j = c0 + threadIdx.x;
    const bool valid = j < n;
    float e = 0.0f;
    if (valid) e = exact_e(key_val(keys[j]), m, rt);
    double tot;
    const double cum = run + block_scan_d(static_cast<double>(e), rs, &tot);
    bool cond = false;
    if (valid) {
      if (mode == 0)
        cond = (w.count_before + j == static_cast<long long>(w.K) - 1) || (w.mass_mode && cum >= w.t2);
      else
        cond = cum > w.t3;
    }
    const int f = block_min_i(cond ? j : INT_MAX, rs);
    if (f != INT_MAX) {
      if (j == f) rs->bcast_d = cum;
      __syncthreads();
      *cum_at = rs->bcast_d;
      __syncthreads();
      return f;
    }
    run += tot;
  }
  return INT_MAX;
}

// Penalised value of history id `id` from the finisher's sorted history
// table (ids hid[0..nh), values hval), or `x` if not in the history.
__device__ __forceinline__ float hist_value(float x, int id, const int32_t* hid, const float* hval, int nh) {
  int lo = 0, hi = nh - 1;
  while (lo <= hi) {
    const int mid = (lo + hi) >> 1;
    const int v = hid[mid];
    if (v == id) return hval[mid];
    if (v < id) lo = mid + 1;
    else hi = mid - 1;
  }
  return x;
}

// ---------------------------------------------------------------------------
// The kernel
// ---------------------------------------------------------------------------
template <typename E>
__global__ void __launch_bounds__(kCT, 2) spec_chunk_kernel(const SpecArgs a) {
  extern __shared__ __align__(128) unsigned char smem[];
  const int chunk = blockIdx.x;
  const int row = blockIdx.y;
  const int S = gridDim.x;
  const int tid = threadIdx.x;
  const int lane = tid & 31;
  const int warp = tid >> 5;

  uint64_t* mbar = reinterpret_cast<uint64_t*>(smem + kOffMbar);
  Ctrl* ctrl = reinterpret_cast<Ctrl*>(smem + kOffCtrl);
  Walk* wk = reinterpret_cast<Walk*>(smem + kOffWalk);
  RedScratch* rs = reinterpret_cast<RedScratch*>(smem + kOffRed);
  float* tmax = reinterpret_cast<float*>(smem + kOffTmax);
  uint32_t* cnt = reinterpret_cast<uint32_t*>(smem + kOffCnt);
  unsigned long long* mass = reinterpret_cast<unsigned long long*>(smem + kOffMass);
  int32_t* hist_local = reinterpret_cast<int32_t*>(smem + kOffHist);
  float* pen_val = reinterpret_cast<float*>(smem + kOffPen);
  ChunkSum* sums_s = reinterpret_cast<ChunkSum*>(smem + kOffSums);
  E* data = reinterpret_cast<E*>(smem + kOffData);

  const int V = a.V;
  const int CE = a.chunk_elems;
  const int start = chunk * CE;
  const int len = max(0, min(CE, V - start));
  constexpr int es = static_cast<int>(sizeof(E));
  constexpr int G = Slice<E>::G;
  const int ngroups = CE / G;
  const Workspace& ws = a.ws;

  const rl_row_params prm = a.params[row];
  const float T = prm.temperature;
  const bool greedy = !(T > 0.0f);  // also NaN: reported as non-finite by the finisher
  const bool thr_path = prm.top_k > 0 && prm.top_k <= kKthr;
  const bool hist_path = !greedy && !thr_path;

  // ---- prologue: mbarriers, bulk copy ----
  const E* src = reinterpret_cast<const E*>(a.logits) + static_cast<int64_t>(row) * a.ld + start;
  const uint32_t bulk_bytes = static_cast<uint32_t>(len * es) & ~15u;
  const bool use_bulk = ((reinterpret_cast<uintptr_t>(src) & 15u) == 0) && bulk_bytes > 0;
  if (tid == 0) {
    for (int p = 0; p < kNPiece; ++p) mbar_init(&mbar[p], 1);
    fence_mbar_init();
    ctrl->n_local = 0;
    ctrl->ncand = 0;
    ctrl->overflow = 0;
  }
  if (hist_path)
    for (int b = tid; b < kNB; b += kCT) {
      cnt[b] = 0u;
      mass[b] = 0ull;
    }
  __syncthreads();
  if (tid == 0 && use_bulk) {
    const uint32_t piece = ((bulk_bytes / kNPiece) + 15u) & ~15u;
    uint32_t off = 0;
    for (int p = 0; p < kNPiece; ++p) {
      const uint32_t nb = off < bulk_bytes ? min(piece, bulk_bytes - off) : 0u;
      mbar_expect_tx(&mbar[p], nb);
      if (nb > 0)
        bulk_g2s(reinterpret_cast<unsigned char*>(data) + off,
                 reinterpret_cast<const unsigned char*>(src) + off, nb, &mbar[p]);
      off += nb;
    }
  }

  // history ids inside this chunk, overlapping the copy
  const int vstart = a.vocab_offset + start;
  int hl = a.hist ? a.hist_len[row] : 0;
  hl = max(0, min(hl, min(a.hist_stride, kHmax)));
  for (int j = tid; j < hl; j += kCT) {
    const int h = a.hist[static_cast<int64_t>(row) * a.hist_stride + j];
    const int loc = h - vstart;
    if (h >= a.vocab_offset && loc >= 0 && loc < len) hist_local[atomicAdd(&ctrl->n_local, 1)] = loc;
  }
  // does the row's mask allow anything? (an all-zero mask allows every id)
  const uint32_t* mrow = a.mask ? a.mask + static_cast<int64_t>(row) * a.mask_stride : nullptr;
  int mask_on = 0;
  if (mrow) {
    const int nw = (V + 31) >> 5;
    int any = 0;
    for (int w0 = 0; w0 < nw && !any; w0 += kCT) {
      const int w = w0 + tid;
      uint32_t bits = 0u;
      if (w < nw) {
        bits = mrow[w];
        const int rem = V - w * 32;
        if (rem < 32) bits &= (1u << rem) - 1u;
      }
      any = block_or_i(bits != 0u, rs);
    }
    mask_on = any;
  }

  // ---- wait for the chunk, unaligned remainder, tail padding ----
  int timed_out = 0;
  if (use_bulk) {
    bool ok = true;
    for (int p = 0; p < kNPiece; ++p) ok &= mbar_wait(&mbar[p], 0, kWaitBudget);
    timed_out = !ok;
  }
  {
    const int first_plain = use_bulk ? static_cast<int>(bulk_bytes / es) : 0;
    for (int i = first_plain + tid; i < len; i += kCT) data[i] = src[i];
    E neg;
    if constexpr (sizeof(E) == 4) {
      neg = RL_NEG_INF;
    } else {
      neg = kBf16NegInf;
    }
    for (int i = len + tid; i < CE; i += kCT) data[i] = neg;
  }
  __syncthreads();

  // ---- penalties (first occurrence of an id applies them) ----
  const int n_local = min(ctrl->n_local, kHmax);
  for (int t = tid; t < n_local; t += kCT) {
    const int h = hist_local[t];
    int c = 0;
    bool first = true;
    for (int j = 0; j < n_local; ++j) {
      if (hist_local[j] == h) {
        ++c;
        if (j < t) first = false;
      }
    }
    if (first) {
      float v;
      if constexpr (sizeof(E) == 4) {
        v = data[h];
      } else {
        v = bf16_bits_to_f32(data[h]);
      }
      const float x1 = (v < 0.0f) ? mul_rn(v, prm.repeat_penalty) : div_rn(v, prm.repeat_penalty);
      const float x3 = sub_rn(sub_rn(x1, mul_rn(static_cast<float>(c), prm.frequency_penalty)), prm.presence_penalty);
      if constexpr (sizeof(E) == 4) {
        data[h] = x3;
      } else {
        pen_val[t] = x3;
      }
    }
  }
  __syncthreads();
  Slice<E> sl;
  sl.data = data;
  if constexpr (sizeof(E) == 2) {
    for (int t = tid; t < n_local; t += kCT) {
      const int h = hist_local[t];
      bool first = true;
      for (int j = 0; j < t; ++j)
        if (hist_local[j] == h) first = false;
      if (first) data[h] = kBf16Marker;
    }
    __syncthreads();
    for (int t = tid; t < n_local; t += kCT) {
      const int h = hist_local[t];
      bool first = true;
      for (int j = 0; j < t; ++j)
        if (hist_local[j] == h) first = false;
      if (!first) hist_local[t] = -1;
    }
    __syncthreads();
    sl.pen_id = hist_local;
    sl.pen_val = pen_val;
    sl.n_pen = n_local;
  }
  // masked ids -> -inf in place
  if (mask_on) {
    for (int g = tid; g < ngroups; g += kCT) {
      const int id0 = start + g * G;
      const uint32_t bits = id0 < V ? (mrow[id0 >> 5] >> (id0 & 31)) : 0u;
#pragma unroll
      for (int k = 0; k < G; ++k) {
        if (!((bits >> k) & 1u)) {
          if constexpr (sizeof(E) == 4) {
            data[g * G + k] = RL_NEG_INF;
          } else {
            data[g * G + k] = kBf16NegInf;
          }
        }
      }
    }
    __syncthreads();
  }

  // ---- P1: chunk max / lowest argmax / allowed count / non-finite; thread maxima ----
  float mx = RL_NEG_INF;
  int amx = INT_MAX;
  int nallow = 0;
  int bad = 0;
  for (int g = tid; g < ngroups; g += kCT) {
    float v[G];
    sl.load(g, v);
#pragma unroll
    for (int k = 0; k < G; ++k) {
      const float x = v[k];
      if (x > RL_NEG_INF) {
        if (!(x < RL_POS_INF)) bad = 1;
        ++nallow;
        if (x > mx) {
          mx = x;
          amx = g * G + k;
        }
      } else if (x != x) {
        bad = 1;
      }
    }
  }
  tmax[tid] = mx;
  float m_c;
  int argmax_c, nallow_c, bad_c;
  {
    const float wm = warp_max(mx);
    int wa = (mx == wm) ? amx : INT_MAX;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) wa = min(wa, __shfl_xor_sync(0xffffffffu, wa, o));
    const int wn = warp_sum_i(nallow);
    const int wb = warp_sum_i(bad);
    __syncthreads();
    if (lane == 0) {
      rs->f[warp] = wm;
      rs->i[warp] = wa;
      rs->j[warp] = wn;
      rs->k[warp] = wb;
    }
    __syncthreads();
    float bm = RL_NEG_INF;
    int ba = INT_MAX, bn = 0, bb = 0;
    for (int w = 0; w < kCW; ++w) {
      bn += rs->j[w];
      bb |= rs->k[w];
      if (rs->f[w] > bm) {
        bm = rs->f[w];
        ba = rs->i[w];
      } else if (rs->f[w] == bm) {
        ba = min(ba, rs->i[w]);
      }
    }
    m_c = bm;
    argmax_c = ba == INT_MAX ? INT_MAX : ba + start;
    nallow_c = bn;
    bad_c = bb ? 1 : 0;
  }

  double z_c = 0.0;
  int babs_m = 0;
  int athr = INT_MIN;
  float tau = RL_NEG_INF;
  const RowT rt = make_rowt(greedy ? 1.0f : T);
  if (!greedy && nallow_c > 0 && !bad_c) {
    babs_m = babs(m_c, rt);
    // ---- P2: Z partial (+ histograms) ----
    float zsum = 0.0f;
    for (int g = tid; g < ngroups; g += kCT) {
      float v[G];
      sl.load(g, v);
#pragma unroll
      for (int k = 0; k < G; ++k) {
        const float x = v[k];
        if (x > RL_NEG_INF) {
          const float e = fast_e(x, m_c, rt);
          zsum += e;
          if (hist_path) {
            const int b = babs_m - babs(x, rt);
            if (b < kNB) {
              atomicAdd(&cnt[b], 1u);
              atomicAdd(&mass[b], __float2ull_rn(e * kMassScaleF));
            }
          }
        }
      }
    }
    z_c = block_sum_d(static_cast<double>(zsum), rs);
    // ---- collection threshold ----
    if (thr_path) {
      // k-th largest per-thread maximum: a lower bound of the chunk's k-th value
      block_sort_desc(tmax, kCT);
      tau = tmax[prm.top_k - 1];
      if (!(tau > RL_NEG_INF)) tau = -3.402823466e38f;  // fewer than k threads hold a value: keep all
    } else {
      // first bin whose cumulative count reaches kKbig
      uint32_t c0 = cnt[2 * tid], c1 = cnt[2 * tid + 1];
      double tot;
      const double incl = block_scan_d(static_cast<double>(c0 + c1), rs, &tot);
      const double excl = incl - static_cast<double>(c0 + c1);
      int bfound = INT_MAX;
      if (excl < kKbig && excl + c0 >= kKbig) bfound = 2 * tid;
      else if (excl + c0 < kKbig && incl >= kKbig) bfound = 2 * tid + 1;
      bfound = block_min_i(bfound, rs);
      if (bfound == INT_MAX) {
        // fewer than kKbig elements in the window: keep the window, and all
        // of the chunk when nothing lies below it
        athr = (static_cast<int>(tot) >= nallow_c) ? INT_MIN : babs_m - (kNB - 1);
      } else {
        athr = babs_m - bfound;
      }
    }
    // ---- P3: candidate keys into the workspace ----
    uint64_t* cdst = ws.cands + (static_cast<int64_t>(row) * ws.smax + chunk) * kCapC;
    for (int gb = warp * 32; gb < ngroups; gb += kCT) {
      const int g = gb + lane;
      float v[G];
      bool anyt = false;
      if (g < ngroups) {
        sl.load(g, v);
#pragma unroll
        for (int k = 0; k < G; ++k) {
          const bool t = thr_path ? (v[k] >= tau) : (v[k] > RL_NEG_INF && babs(v[k], rt) >= athr);
          anyt |= t && (v[k] > RL_NEG_INF);
        }
      }
      if (!__any_sync(0xffffffffu, anyt)) continue;
#pragma unroll
      for (int k = 0; k < G; ++k) {
        bool take = false;
        if (anyt) {
          const float x = v[k];
          take = x > RL_NEG_INF && (thr_path ? (x >= tau) : (babs(x, rt) >= athr));
        }
        const uint32_t bal = __ballot_sync(0xffffffffu, take);
        if (bal) {
          int base = 0;
          if (lane == 0) base = atomicAdd(&ctrl->ncand, __popc(bal));
          base = __shfl_sync(0xffffffffu, base, 0);
          if (take) {
            const int idx = base + __popc(bal & ((1u << lane) - 1u));
            if (idx < kCapC) cdst[idx] = cand_key(v[k], static_cast<uint32_t>(start + g * G + k));
          }
        }
      }
    }
    if (hist_path) {
      uint32_t* gc = ws.hcnt + (static_cast<int64_t>(row) * ws.smax + chunk) * kNB;
      unsigned long long* gm = ws.hmass + (static_cast<int64_t>(row) * ws.smax + chunk) * kNB;
      for (int b = tid; b < kNB; b += kCT) {
        gc[b] = cnt[b];
        gm[b] = mass[b];
      }
    }
  }
  __syncthreads();
  if (tid == 0) {
    ChunkSum s;
    s.m = m_c;
    s.argmax = argmax_c;
    s.nallow = nallow_c;
    s.flags = bad_c | (timed_out ? 2 : 0) | (ctrl->ncand > kCapC ? 4 : 0);
    s.z = z_c;
    s.ncand = min(ctrl->ncand, kCapC);
    s.babs_m = babs_m;
    s.athr = athr;
    s.tau = tau;
    ws.sums[static_cast<int64_t>(row) * ws.smax + chunk] = s;
    __threadfence();
    const int prev = atomicAdd(&ws.row_done[row], 1);
    ctrl->is_last = prev == S - 1;
  }
  __syncthreads();
  if (timed_out) {
    // never leave with a copy still landing in this CTA's shared memory
    for (int p = 0; p < kNPiece; ++p) mbar_wait(&mbar[p], 0, kWaitBudget);
  }
  if (!ctrl->is_last) return;

  // =====================================================================
  // Finisher: the last CTA of the row
  // =====================================================================
  __threadfence();
  if (tid < S) {
    const ChunkSum* src_s = ws.sums + static_cast<int64_t>(row) * ws.smax + tid;
    ChunkSum s;
    s.m = __ldcg(&src_s->m);
    s.argmax = __ldcg(&src_s->argmax);
    s.nallow = __ldcg(&src_s->nallow);
    s.flags = __ldcg(&src_s->flags);
    s.z = __ldcg(&src_s->z);
    s.ncand = __ldcg(&src_s->ncand);
    s.babs_m = __ldcg(&src_s->babs_m);
    s.athr = __ldcg(&src_s->athr);
    s.tau = __ldcg(&src_s->tau);
    sums_s[tid] = s;
  }
  __syncthreads();
  float m = RL_NEG_INF;
  int gargmax = INT_MAX, gallow = 0, gflags = 0;
  int athr_max = INT_MIN;
  for (int c = 0; c < S; ++c) {
    const ChunkSum& s = sums_s[c];
    gallow += s.nallow;
    gflags |= s.flags;
    athr_max = max(athr_max, s.athr);
    if (s.m > m) {
      m = s.m;
      gargmax = s.argmax;
    } else if (s.m == m) {
      gargmax = min(gargmax, s.argmax);
    }
  }
  int row_st = 0;
  if (gflags & 2) row_st = RL_ERR_TIMEOUT;
  else if ((gflags & 1) || gallow == 0 || !(fabsf(T) < RL_POS_INF)) row_st = RL_ERR_NONFINITE;
  else if (gflags & 4) row_st = RL_ERR_UNSUPPORTED;

  auto finish = [&](int status, int token, float prob) {
    if (tid == 0) {
      const bool ok = status == 0;
      a.out_tok[row] = ok ? token + a.vocab_offset : -1;
      if (a.out_prob) a.out_prob[row] = ok ? prob : 0.0f;
      if (a.row_status) a.row_status[row] = status;
      ws.row_done[row] = 0;  // ready for the next launch
    }
  };

  if (row_st != 0 || greedy) {
    finish(row_st, gargmax, 1.0f);
    if (a.list_len && tid == 0) {
      const bool ok = row_st == 0;
      a.list_len[row] = (ok && a.list_cap > 0) ? 1 : 0;
      if (ok && a.list_cap > 0) {
        a.list_ids[static_cast<int64_t>(row) * a.list_cap] = gargmax + a.vocab_offset;
        a.list_probs[static_cast<int64_t>(row) * a.list_cap] = 1.0f;
      }
    }
    return;
  }

  // Z = sum_c z_c * 2^((m_c - m) log2(e) / T)
  double zpart = 0.0;
  if (tid < S && sums_s[tid].nallow > 0)
    zpart = sums_s[tid].z * exp2((static_cast<double>(sums_s[tid].m) - static_cast<double>(m)) *
                                 (kLog2e / static_cast<double>(T)));
  const double Z = block_sum_d(zpart, rs);
  const float u = a.uniforms[row];
  const int K = (prm.top_k > 0 && prm.top_k < gallow) ? prm.top_k : gallow;
  const bool mass_mode = prm.top_p < 1.0f;
  uint64_t* keys = reinterpret_cast<uint64_t*>(data);  // the chunk is no longer needed
  if (tid == 0) {
    Walk& w = *wk;
    w.phase = 0;
    w.K = K;
    w.mass_mode = mass_mode;
    w.cut_in_seg = 0;
    w.cut_idx = -1;
    w.status = 0;
    w.token = -1;
    w.prob = 0.0f;
    w.count_before = 0;
    w.mass_before = 0.0;
    w.Z = Z;
    w.t2 = static_cast<double>(prm.top_p) * Z;
    w.S = 0.0;
    w.t3 = 0.0;
  }
  __syncthreads();

  if (thr_path) {
    // ---- merge the candidate lists, sort, exact top-k / top-p / draw ----
    int off = 0;
    for (int c = 0; c < S; ++c) {
      const int n = sums_s[c].ncand;
      const uint64_t* srcc = ws.cands + (static_cast<int64_t>(row) * ws.smax + c) * kCapC;
      for (int i = tid; i < n && off + i < kMergeCap; i += kCT) keys[off + i] = __ldcg(srcc + i);
      off += n;
    }
    if (off > kMergeCap) {
      finish(RL_ERR_UNSUPPORTED, -1, 0.0f);
      return;
    }
    const int P = pow2_ceil(off);
    for (int i = off + tid; i < P; i += kCT) keys[i] = 0ull;
    __syncthreads();
    block_sort_desc(keys, P);
    const int nlist = min(K, off);
    double cum_at = 0.0;
    const int f = sweep(keys, nlist, *wk, m, rt, 0, rs, &cum_at);
    const int cut = (f == INT_MAX) ? nlist - 1 : f;
    if (f == INT_MAX) {
      // cumulative mass never reached top_p inside the list (rounding): the
      // list end is the cutoff; recompute its cumulative mass
      double tot = 0.0;
      for (int c0 = 0; c0 < nlist; c0 += kCT) {
        const int j = c0 + tid;
        double t;
        block_scan_d(j < nlist ? static_cast<double>(exact_e(key_val(keys[j]), m, rt)) : 0.0, rs, &t);
        tot += t;
      }
      cum_at = tot;
    }
    if (tid == 0) {
      wk->S = cum_at;
      wk->t3 = static_cast<double>(u) * cum_at;
    }
    __syncthreads();
    const int d = sweep(keys, cut + 1, *wk, m, rt, 1, rs, &cum_at);
    const int j = (d == INT_MAX) ? cut : d;
    if (a.list_len) {
      const int nl = min(nlist, a.list_cap);
      for (int i = tid; i < nl; i += kCT) {
        a.list_ids[static_cast<int64_t>(row) * a.list_cap + i] = static_cast<int>(key_id(keys[i])) + a.vocab_offset;
        a.list_probs[static_cast<int64_t>(row) * a.list_cap + i] =
            static_cast<float>(static_cast<double>(exact_e(key_val(keys[i]), m, rt)) / Z);
      }
      if (tid == 0) a.list_len[row] = nl;
    }
    const float ej = exact_e(key_val(keys[j]), m, rt);
    finish(0, static_cast<int>(key_id(keys[j])), static_cast<float>(static_cast<double>(ej) / wk->S));
    return;
  }

  // ---- histogram path: merge the chunk histograms on the row's grid ----
  const int Bmax = babs(m, rt);
  double* gcnt = reinterpret_cast<double*>(smem + kOffCnt);
  double* gmass = reinterpret_cast<double*>(smem + kOffMass);
  {
    double c2[2] = {0.0, 0.0}, m2[2] = {0.0, 0.0};
    for (int c = 0; c < S; ++c) {
      const ChunkSum& s = sums_s[c];
      if (s.nallow == 0) continue;
      const int shift = Bmax - s.babs_m;
      const double f = exp2((static_cast<double>(s.m) - static_cast<double>(m)) * (kLog2e / static_cast<double>(T))) /
                       kMassScale;
      const uint32_t* gc = ws.hcnt + (static_cast<int64_t>(row) * ws.smax + c) * kNB;
      const unsigned long long* gm = ws.hmass + (static_cast<int64_t>(row) * ws.smax + c) * kNB;
#pragma unroll
      for (int q = 0; q < 2; ++q) {
        const int i = 2 * tid + q - shift;
        if (i >= 0 && i < kNB) {
          c2[q] += static_cast<double>(__ldcg(gc + i));
          m2[q] += static_cast<double>(__ldcg(gm + i)) * f;
        }
      }
    }
    double tc, tm;
    const double ci = block_scan_d(c2[0] + c2[1], rs, &tc);
    const double mi = block_scan_d(m2[0] + m2[1], rs, &tm);
    gcnt[2 * tid] = ci - c2[1];
    gcnt[2 * tid + 1] = ci;
    gmass[2 * tid] = mi - m2[1];
    gmass[2 * tid + 1] = mi;
    __syncthreads();
  }
  // gcnt / gmass: inclusive cumulative counts / masses per row bin j (absolute bin Bmax - j)
  const bool need_q1 = K < gallow;
  auto first_bin = [&](int kind, double target) -> int {
    // kind 0: count >= target; 1: mass >= target; 2: mass > target
    int b = INT_MAX;
    for (int j = tid; j < kNB; j += kCT) {
      const double cur = kind == 0 ? gcnt[j] : gmass[j];
      const double prev = j ? (kind == 0 ? gcnt[j - 1] : gmass[j - 1]) : 0.0;
      const bool hit = kind == 2 ? (cur > target && !(prev > target)) : (cur >= target && !(prev >= target));
      if (hit) b = j;
    }
    return block_min_i(b, rs);
  };
  int bin;
  if (!need_q1 && !mass_mode) {
    // the list is every allowed id: cutoff at its end, S = Z
    if (tid == 0) {
      wk->phase = 1;
      wk->S = Z;
      wk->t3 = static_cast<double>(u) * Z;
    }
    __syncthreads();
    bin = first_bin(2, wk->t3);
  } else {
    const int b1 = need_q1 ? first_bin(0, static_cast<double>(K)) : INT_MAX;
    const int b2 = mass_mode ? first_bin(1, wk->t2) : INT_MAX;
    bin = min(b1, b2);
  }
  // ---- bin-by-bin walk ----
  int32_t* hid = reinterpret_cast<int32_t*>(smem + kOffHist);  // finisher history table (sorted)
  float* hval = reinterpret_cast<float*>(smem + kOffPen);
  uint64_t* bkeys = keys;                                       // keys of one bin (<= kMergeCap)
  int nh = -1;  // history table built on first re-read
  for (int round = 0; round < kMaxRounds; ++round) {
    if (bin >= kNB) {
      if (tid == 0) wk->status = RL_ERR_UNSUPPORTED;  // beyond the 64-nat window
      break;
    }
    const int A = Bmax - bin;
    bool covered = true;
    for (int c = 0; c < S; ++c)
      if (sums_s[c].nallow > 0 && sums_s[c].athr > A) covered = false;
    if (tid == 0) ctrl->nbin = 0;
    __syncthreads();
    if (covered) {
      for (int c = 0; c < S; ++c) {
        const int n = sums_s[c].ncand;
        const uint64_t* srcc = ws.cands + (static_cast<int64_t>(row) * ws.smax + c) * kCapC;
        for (int i = tid; i < n; i += kCT) {
          const uint64_t key = __ldcg(srcc + i);
          if (babs(key_val(key), rt) == A) {
            const int idx = atomicAdd(&ctrl->nbin, 1);
            if (idx < kMergeCap) bkeys[idx] = key;
          }
        }
      }
    } else {
      // re-read the row (L2-resident) for the elements of bin A
      if (nh < 0) {
        // sorted, de-duplicated history ids with their penalised values
        int hlr = a.hist ? a.hist_len[row] : 0;
        hlr = max(0, min(hlr, min(a.hist_stride, kHmax)));
        const int P = pow2_ceil(max(hlr, 1));
        for (int j = tid; j < P; j += kCT) {
          uint64_t h = ~0ull;
          if (j < hlr) {
            const int hv = a.hist[static_cast<int64_t>(row) * a.hist_stride + j] - a.vocab_offset;
            if (hv >= 0 && hv < V) h = static_cast<uint64_t>(hv);
          }
          bkeys[j] = h;
        }
        __syncthreads();
        block_sort_desc(bkeys, P);  // descending; position j ascending is P-1-j
        const E* xr0 = reinterpret_cast<const E*>(a.logits) + static_cast<int64_t>(row) * a.ld;
        // each thread owns ascending positions tid and tid + kCT (P <= kHmax <= 2 kCT)
        int fl[2] = {0, 0};
        uint64_t idv[2] = {~0ull, ~0ull};
        int cntv[2] = {0, 0};
#pragma unroll
        for (int q = 0; q < 2; ++q) {
          const int j = tid + q * kCT;
          if (j < P) {
            const uint64_t h = bkeys[P - 1 - j];
            if (h != ~0ull && (j == 0 || bkeys[P - j] != h)) {
              fl[q] = 1;
              idv[q] = h;
              int c = 0;
              for (int t = j; t < P && bkeys[P - 1 - t] == h; ++t) ++c;
              cntv[q] = c;
            }
          }
        }
        // output positions in ascending order: positions 0..kCT-1, then kCT..P-1
        {
          double t0;
          const double i0 = block_scan_d(static_cast<double>(fl[0]), rs, &t0);
          double t1;
          const double i1 = block_scan_d(static_cast<double>(fl[1]), rs, &t1);
          const int p0 = static_cast<int>(i0) - fl[0];
          const int p1 = static_cast<int>(t0) + static_cast<int>(i1) - fl[1];
          auto pen = [&](int id, int c) {
            float v;
            if constexpr (sizeof(E) == 4) {
              v = __ldcg(xr0 + id);
            } else {
              v = bf16_bits_to_f32(__ldcg(reinterpret_cast<const unsigned short*>(xr0) + id));
            }
            const float x1 = (v < 0.0f) ? mul_rn(v, prm.repeat_penalty) : div_rn(v, prm.repeat_penalty);
            return sub_rn(sub_rn(x1, mul_rn(static_cast<float>(c), prm.frequency_penalty)), prm.presence_penalty);
          };
          if (fl[0]) {
            hid[p0] = static_cast<int32_t>(idv[0]);
            hval[p0] = pen(static_cast<int>(idv[0]), cntv[0]);
          }
          if (fl[1]) {
            hid[p1] = static_cast<int32_t>(idv[1]);
            hval[p1] = pen(static_cast<int>(idv[1]), cntv[1]);
          }
          nh = static_cast<int>(t0 + t1);
        }
        if (tid == 0) ctrl->nbin = 0;
        __syncthreads();
      }
      const E* xr = reinterpret_cast<const E*>(a.logits) + static_cast<int64_t>(row) * a.ld;
      for (int i = tid; i < V; i += kCT) {
        float x;
        if constexpr (sizeof(E) == 4) {
          x = __ldcg(xr + i);
        } else {
          x = bf16_bits_to_f32(__ldcg(reinterpret_cast<const unsigned short*>(xr) + i));
        }
        if (nh > 0) x = hist_value(x, i, hid, hval, nh);
        if (mask_on && !((mrow[i >> 5] >> (i & 31)) & 1u)) continue;
        if (!(x > RL_NEG_INF)) continue;
        if (babs(x, rt) == A) {
          const int idx = atomicAdd(&ctrl->nbin, 1);
          if (idx < kMergeCap) bkeys[idx] = cand_key(x, static_cast<uint32_t>(i));
        }
      }
    }
    __syncthreads();
    const int nb = ctrl->nbin;
    if (nb > kMergeCap) {
      if (tid == 0) wk->status = RL_ERR_UNSUPPORTED;
      break;
    }
    const int P = pow2_ceil(max(nb, 1));
    for (int i = nb + tid; i < P; i += kCT) bkeys[i] = 0ull;
    __syncthreads();
    block_sort_desc(bkeys, P);
    if (tid == 0) {
      wk->count_before = bin ? static_cast<long long>(gcnt[bin - 1]) : 0;
      wk->mass_before = bin ? gmass[bin - 1] : 0.0;
    }
    __syncthreads();
    int next = INT_MAX;
    double cum_at = 0.0;
    if (wk->phase == 0) {
      const int f = sweep(bkeys, nb, *wk, m, rt, 0, rs, &cum_at);
      if (f != INT_MAX) {
        if (tid == 0) {
          wk->cut_in_seg = 1;
          wk->cut_idx = f;
          wk->S = cum_at;
          wk->t3 = static_cast<double>(u) * cum_at;
          wk->phase = 1;
        }
      } else {
        next = bin + 1;
      }
    } else if (tid == 0) {
      wk->cut_in_seg = 0;
    }
    __syncthreads();
    if (wk->phase == 1 && next == INT_MAX) {
      if (wk->t3 < wk->mass_before) {
        const int b3 = first_bin(2, wk->t3);
        next = (b3 < bin) ? b3 : max(0, bin - 1);
      } else {
        const int d = sweep(bkeys, nb, *wk, m, rt, 1, rs, &cum_at);
        if (tid == 0) {
          int j = -1;
          if (d != INT_MAX && (!wk->cut_in_seg || d <= wk->cut_idx)) j = d;
          else if (wk->cut_in_seg) j = wk->cut_idx;
          if (j >= 0) {
            const uint64_t key = bkeys[j];
            wk->token = static_cast<int>(key_id(key));
            wk->prob = static_cast<float>(static_cast<double>(exact_e(key_val(key), m, rt)) / wk->S);
            wk->phase = 2;
          }
        }
        __syncthreads();
        if (wk->phase != 2) next = bin + 1;
      }
    }
    __syncthreads();
    if (wk->phase == 2) break;
    bin = next;
  }
  __syncthreads();
  if (a.list_len && tid == 0) a.list_len[row] = -1;  // lists are reported on the threshold path only
  const Walk& w = *wk;
  if (w.phase == 2 && w.status == 0) finish(0, w.token, w.prob);
  else finish(w.status ? w.status : RL_ERR_UNSUPPORTED, -1, 0.0f);
}

// ---------------------------------------------------------------------------
// Host launcher
// ---------------------------------------------------------------------------
template <typename E>
static cudaError_t launch_typed(const SpecArgs& a, int S, int smem, cudaStream_t stream) {
  auto k = spec_chunk_kernel<E>;
  cudaError_t err = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  if (err != cudaSuccess) return err;
  k<<<dim3(S, a.B, 1), dim3(kCT, 1, 1), smem, stream>>>(a);
  return cudaGetLastError();
}

cudaError_t launch_spec(const SpecArgs& args_in, int dtype, cudaStream_t stream) {
  SpecArgs a = args_in;
  const int es = dtype == RL_BF16 ? 2 : 4;
  a.chunk_elems = kChunkBytes / es;
  const int S = spec_chunks(a.V, es);
  const int smem = spec_smem_bytes(es);
  if (dtype == RL_BF16) return launch_typed<uint16_t>(a, S, smem, stream);
  return launch_typed<float>(a, S, smem, stream);
}

}  // namespace rl
