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
// Design (B200, sm_100a). One launch, grid (chunks, rows), three CTAs per SM.
// Every CTA streams one 48 KB chunk (12288 logits) of one row into shared
// memory with bulk async copies (cp.async.bulk + mbarrier) -- the only HBM
// read of those logits -- applies the row's penalties and mask in place, and
// reduces the chunk to a summary in the handle's workspace. Each pass keeps
// its 32 values per thread in registers (8 unrolled 16-byte loads):
//   P1  chunk max, allowed count, non-finite check, per-thread maxima
//   P2  Z partial: sum of 2^((x - m_c) * log2(e)/T) (split constant, ex2)
//       histogram rows also bin every logit on an absolute grid (16 bins per
//       nat) and add its bin-relative mass (u32 fixed point; u32 atomics)
//   P3  candidate keys (value desc, id asc) of every logit that can be in the
//       row's top-k: x >= tau, tau from the per-thread maxima (top_k <= 128),
//       or the chunk's top 512 by the histogram.
// The last CTA of a row to arrive (arrival counter) finishes the row: global
// max and Z, the exact top-k list (tightened threshold + rank sort, exact
// exp), the inclusive top-p cutoff and the draw. Rows without a small top_k
// walk the merged histogram bin by bin; a bin not covered by the candidate
// lists is re-read from the row (L2-resident by then).
#include <climits>

#include "common.cuh"
#include "spec_kernel.cuh"

namespace rl {

constexpr uint16_t kBf16NegInf = 0xff80;
constexpr double kLog2e = 1.4426950408889634074;
constexpr int kBinsPT = (kNB + kCT - 1) / kCT;  // histogram bins per thread in scans (3)

// ---------------------------------------------------------------------------
// Row arithmetic
// ---------------------------------------------------------------------------
struct RowT {
  float T, rT;       // temperature, RN(1/T)
  bool fast_div;     // Markstein division valid for T
  float c_hi, c_lo;  // log2(e)/T split in two floats
  float cb;          // absolute bins per logit unit: kRbin / T
  float dlt;         // log2(e) / kRbin: log2 width of one bin
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
  r.dlt = static_cast<float>(kLog2e / static_cast<double>(kRbin));
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
__device__ __forceinline__ int babs(float x, const RowT& r) { return __float2int_rd(__fmul_rn(x, r.cb)); }

// ---------------------------------------------------------------------------
// Chunk access: 4 consecutive logits per 16-byte (f32) / 8-byte (bf16) load.
// ---------------------------------------------------------------------------
template <typename E>
__device__ __forceinline__ void load4(const E* data, int g, float (&v)[4]);
template <>
__device__ __forceinline__ void load4<float>(const float* data, int g, float (&v)[4]) {
  const float4 q = reinterpret_cast<const float4*>(data)[g];
  v[0] = q.x;
  v[1] = q.y;
  v[2] = q.z;
  v[3] = q.w;
}
template <>
__device__ __forceinline__ void load4<uint16_t>(const uint16_t* data, int g, float (&v)[4]) {
  const uint2 q = reinterpret_cast<const uint2*>(data)[g];
  v[0] = __uint_as_float(q.x << 16);
  v[1] = __uint_as_float(q.x & 0xffff0000u);
  v[2] = __uint_as_float(q.y << 16);
  v[3] = __uint_as_float(q.y & 0xffff0000u);
}
// all kGPT groups of this thread (group g = tid + k * kCT)
template <typename E>
__device__ __forceinline__ void load_all(const E* data, float (&v)[kGPT][4]) {
#pragma unroll
  for (int k = 0; k < kGPT; ++k) load4<E>(data, threadIdx.x + k * kCT, v[k]);
}

// ---------------------------------------------------------------------------
// Block / warp helpers (kCT threads)
// ---------------------------------------------------------------------------
struct RedScratch {
  double d[kCW];
  float f[kCW];
  int i[kCW];
  int j[kCW];
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

// Descending sort of one float per lane across a warp (bitonic, shuffles).
__device__ __forceinline__ float warp_sort_desc(float v) {
  const int lane = threadIdx.x & 31;
#pragma unroll
  for (int k = 2; k <= 32; k <<= 1) {
#pragma unroll
    for (int j = k >> 1; j > 0; j >>= 1) {
      const float o = __shfl_xor_sync(0xffffffffu, v, j);
      const bool desc = (lane & k) == 0 || k == 32;
      const bool lower = (lane & j) == 0;
      v = (desc == lower) ? fmaxf(v, o) : fminf(v, o);
    }
  }
  return v;
}

// Lower bound of the k-th largest of the values held one per thread: every
// warp holds at least ceil(k / kCW) values >= the result, so at least k
// values are. -inf if some warp holds fewer finite values.
__device__ __forceinline__ float block_kth_lower_bound(float v, int k, RedScratch* rs) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int j = min((k + kCW - 1) / kCW, 32);
  const float s = warp_sort_desc(v);
  const float wj = __shfl_sync(0xffffffffu, s, j - 1);
  __syncthreads();
  if (lane == 0) rs->f[warp] = wj;
  __syncthreads();
  float t = RL_POS_INF;
  for (int w = 0; w < kCW; ++w) t = fminf(t, rs->f[w]);
  return t;
}

// out[rank] = key for every key of rank < keep (keys unique; rank = number of
// larger keys): the top `keep` keys in descending order.
__device__ void rank_sort(const uint64_t* in, int n, uint64_t* out, int keep) {
  for (int i = threadIdx.x; i < n; i += kCT) {
    const uint64_t k = in[i];
    int r = 0;
    for (int j = 0; j < n; ++j) r += in[j] > k;
    if (r < keep) out[r] = k;
  }
  __syncthreads();
}

// ---------------------------------------------------------------------------
// Shared-memory layout
// ---------------------------------------------------------------------------
struct Ctrl {
  int n_local;  // history entries inside the chunk
  int ncand;    // candidate keys written
  int is_last;
  int nsel;     // finisher: keys selected
  int nbin;     // finisher: keys gathered for the current bin
  int pad[3];
};

// Finisher walk state (masses relative to the row max, e-units).
struct Walk {
  int phase;       // 0: find the cutoff, 1: find the draw, 2: done
  int K;           // list length
  int mass_mode;   // top_p < 1
  int cut_in_seg;  // the cutoff element is in the current segment
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
constexpr int kOffCnt = 1024;                  // kNB u32 counts
constexpr int kOffMass = kOffCnt + kNB * 4;    // kNB u32 masses
constexpr int kOffHist = kOffMass + kNB * 4;   // kHmax ints (finisher: sorted history ids)
constexpr int kOffPen = kOffHist + kHmax * 4;  // kHmax floats (finisher: their values)
constexpr int kOffSums = kOffPen + kHmax * 4;  // kSmax ChunkSum (finisher)
constexpr int kOffData = ((kOffSums + kSmax * static_cast<int>(sizeof(ChunkSum)) + 127) / 128) * 128;
constexpr int kDataBytes = kCE * 4;            // f32 chunk; finisher: keys + merged histograms
static_assert(kMergeCap * 8 + kNB * 16 <= kDataBytes, "finisher region");
static_assert(sizeof(Walk) <= 128, "walk");
static_assert(kOffRed + sizeof(RedScratch) <= kOffCnt, "smem header");

int spec_smem_bytes(int /*es*/) { return kOffData + kDataBytes; }
int spec_chunks(int V) { return (V + kCE - 1) / kCE; }

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

// Penalised value of id from the finisher's sorted history table, or x.
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
__global__ void __launch_bounds__(kCT, 3) spec_chunk_kernel(const SpecArgs a) {
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
  uint32_t* cnt = reinterpret_cast<uint32_t*>(smem + kOffCnt);
  uint32_t* mass = reinterpret_cast<uint32_t*>(smem + kOffMass);
  int32_t* hist_local = reinterpret_cast<int32_t*>(smem + kOffHist);
  float* pen_val = reinterpret_cast<float*>(smem + kOffPen);
  ChunkSum* sums_s = reinterpret_cast<ChunkSum*>(smem + kOffSums);
  E* data = reinterpret_cast<E*>(smem + kOffData);

  const int V = a.V;
  const int start = chunk * kCE;
  const int len = max(0, min(kCE, V - start));
  constexpr int es = static_cast<int>(sizeof(E));
  const Workspace& ws = a.ws;

  const rl_row_params prm = a.params[row];
  const float T = prm.temperature;
  const bool greedy = !(T > 0.0f);  // NaN is reported as non-finite by the finisher
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
  }
  if (hist_path)
    for (int b = tid; b < kNB; b += kCT) {
      cnt[b] = 0u;
      mass[b] = 0u;
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
    for (int i = len + tid; i < kCE; i += kCT) data[i] = neg;
  }
  __syncthreads();

  // ---- penalties: one warp per history entry (count + first occurrence) ----
  const int n_local = min(ctrl->n_local, kHmax);
  for (int t = warp; t < n_local; t += kCW) {
    const int h = hist_local[t];
    int c = 0;
    bool first = true;
    for (int j0 = 0; j0 < n_local; j0 += 32) {
      const int j = j0 + lane;
      const bool eq = j < n_local && hist_local[j] == h;
      const uint32_t bal = __ballot_sync(0xffffffffu, eq);
      c += __popc(bal);
      if (eq && j < t) first = false;
    }
    first = __all_sync(0xffffffffu, first);
    if (lane == 0) {
      if (first) {
        float v;
        if constexpr (sizeof(E) == 4) {
          v = data[h];
        } else {
          v = bf16_bits_to_f32(data[h]);
        }
        const float x1 = (v < 0.0f) ? mul_rn(v, prm.repeat_penalty) : div_rn(v, prm.repeat_penalty);
        pen_val[t] = sub_rn(sub_rn(x1, mul_rn(static_cast<float>(c), prm.frequency_penalty)), prm.presence_penalty);
      } else {
        pen_val[t] = __int_as_float(0x7fffffff);  // duplicate entry: no-op
      }
    }
  }
  __syncthreads();
  const bool dup_free = true;
  (void)dup_free;
  // f32: write the penalised values in place; bf16 chunks cannot hold them,
  // so they are patched into the registers after every load (few slots).
  if constexpr (sizeof(E) == 4) {
    for (int t = tid; t < n_local; t += kCT)
      if (!(pen_val[t] != pen_val[t])) data[hist_local[t]] = pen_val[t];
    __syncthreads();
  }
  // masked ids -> -inf in place
  if (mask_on) {
    for (int g = tid; g < kCE / 4; g += kCT) {
      const int id0 = start + g * 4;
      const uint32_t bits = id0 < V ? (mrow[id0 >> 5] >> (id0 & 31)) : 0u;
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        if (!((bits >> k) & 1u)) {
          if constexpr (sizeof(E) == 4) {
            data[g * 4 + k] = RL_NEG_INF;
          } else {
            data[g * 4 + k] = kBf16NegInf;
          }
        }
      }
    }
    __syncthreads();
  }
  // bf16: patch the penalised slots this thread owns (masked slots stay -inf)
  auto patch = [&](float (&v)[kGPT][4]) {
    if constexpr (sizeof(E) == 2) {
      for (int t = 0; t < n_local; ++t) {
        const float pv = pen_val[t];
        if (pv != pv) continue;  // duplicate entry
        const int h = hist_local[t];
        const int g = h >> 2;
        if ((g % kCT) != static_cast<int>(threadIdx.x)) continue;
        const int q0 = g / kCT;
#pragma unroll
        for (int q = 0; q < kGPT; ++q)
#pragma unroll
          for (int k = 0; k < 4; ++k)
            if (q == q0 && k == (h & 3) && v[q][k] > RL_NEG_INF) v[q][k] = pv;
      }
    }
  };

  // ---- P1: chunk max / allowed count / non-finite; per-thread max ----
  float mx = RL_NEG_INF;
  int nallow = 0;
  int bad = 0;
  int amx = INT_MAX;
  {
    float v[kGPT][4];
    load_all<E>(data, v);
    patch(v);
#pragma unroll
    for (int q = 0; q < kGPT; ++q) {
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        const float x = v[q][k];
        nallow += (x > RL_NEG_INF) ? 1 : 0;
        bad |= (x != x) || (x == RL_POS_INF);
        mx = fmaxf(mx, x);
      }
    }
    if (greedy) {
#pragma unroll
      for (int q = 0; q < kGPT; ++q)
#pragma unroll
        for (int k = 0; k < 4; ++k)
          if (v[q][k] == mx) amx = min(amx, (static_cast<int>(threadIdx.x) + q * kCT) * 4 + k);
    }
  }
  float m_c;
  int argmax_c, nallow_c, bad_c;
  {
    const float wm = warp_max(mx);
    int wa = (mx == wm) ? amx : INT_MAX;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) wa = min(wa, __shfl_xor_sync(0xffffffffu, wa, o));
    const int wn = warp_sum_i(nallow);
    const int wb = __any_sync(0xffffffffu, bad);
    __syncthreads();
    if (lane == 0) {
      rs->f[warp] = wm;
      rs->i[warp] = wa;
      rs->j[warp] = wn | (wb << 30);
    }
    __syncthreads();
    float bm = RL_NEG_INF;
    int ba = INT_MAX, bn = 0, bb = 0;
    for (int w = 0; w < kCW; ++w) {
      bn += rs->j[w] & 0x3fffffff;
      bb |= rs->j[w] >> 30;
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
  int binovf = 0;
  const RowT rt = make_rowt(greedy ? 1.0f : T);
  if (!greedy && nallow_c > 0 && !bad_c) {
    babs_m = babs(m_c, rt);
    float v[kGPT][4];
    load_all<E>(data, v);
    patch(v);
    // ---- P2: Z partial (+ histograms) ----
    float z4[4] = {0.0f, 0.0f, 0.0f, 0.0f};
#pragma unroll
    for (int q = 0; q < kGPT; ++q) {
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        const float x = v[q][k];
        z4[k] += fast_e(x, m_c, rt);  // -inf contributes 0
        if (hist_path && x > RL_NEG_INF) {
          const float y = __fmul_rn(x, rt.cb);
          const float af = floorf(y);
          const int b = babs_m - static_cast<int>(af);
          if (b < kNB) {
            const float eb = ex2_approx((y - af - 1.0f) * rt.dlt);  // mass relative to the bin top
            atomicAdd(&cnt[b], 1u);
            atomicAdd(&mass[b], __float2uint_rn(eb * kMassQ));
          }
        }
      }
    }
    z_c = block_sum_d(static_cast<double>((z4[0] + z4[1]) + (z4[2] + z4[3])), rs);
    // ---- collection threshold ----
    if (thr_path) {
      tau = block_kth_lower_bound(mx, prm.top_k, rs);
      if (!(tau > RL_NEG_INF)) tau = -3.402823466e38f;  // too few values: keep all
    } else {
      // first bin whose cumulative count reaches kKbig
      uint32_t c[kBinsPT];
      uint32_t csum = 0;
#pragma unroll
      for (int q = 0; q < kBinsPT; ++q) {
        const int b = static_cast<int>(threadIdx.x) * kBinsPT + q;
        c[q] = b < kNB ? cnt[b] : 0u;
        csum += c[q];
        if (c[q] > static_cast<uint32_t>(kBinCntSafe)) binovf = 1;
      }
      double tot;
      const double incl = block_scan_d(static_cast<double>(csum), rs, &tot);
      double run = incl - static_cast<double>(csum);
      int bfound = INT_MAX;
#pragma unroll
      for (int q = 0; q < kBinsPT; ++q) {
        if (run < kKbig && run + c[q] >= kKbig && bfound == INT_MAX)
          bfound = static_cast<int>(threadIdx.x) * kBinsPT + q;
        run += c[q];
      }
      bfound = block_min_i(bfound, rs);
      binovf = block_or_i(binovf, rs);
      if (bfound == INT_MAX) {
        // fewer than kKbig logits in the window: keep the window, and all of
        // the chunk when nothing lies below it
        athr = (static_cast<int>(tot) >= nallow_c) ? INT_MIN : babs_m - (kNB - 1);
      } else {
        athr = babs_m - bfound;
      }
    }
    // ---- P3: candidate keys into the workspace ----
    uint64_t* cdst = ws.cands + (static_cast<int64_t>(row) * ws.smax + chunk) * kCapC;
#pragma unroll
    for (int q = 0; q < kGPT; ++q) {
      bool take[4];
      bool anyt = false;
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        const float x = v[q][k];
        take[k] = x > RL_NEG_INF && (thr_path ? (x >= tau) : (babs(x, rt) >= athr));
        anyt |= take[k];
      }
      if (!__any_sync(0xffffffffu, anyt)) continue;
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        const uint32_t bal = __ballot_sync(0xffffffffu, take[k]);
        if (bal) {
          int base = 0;
          if (lane == 0) base = atomicAdd(&ctrl->ncand, __popc(bal));
          base = __shfl_sync(0xffffffffu, base, 0);
          if (take[k]) {
            const int idx = base + __popc(bal & ((1u << lane) - 1u));
            if (idx < kCapC)
              cdst[idx] = cand_key(v[q][k], static_cast<uint32_t>(start + (static_cast<int>(threadIdx.x) + q * kCT) * 4 + k));
          }
        }
      }
    }
    if (hist_path) {
      uint32_t* gc = ws.hcnt + (static_cast<int64_t>(row) * ws.smax + chunk) * kNB;
      uint32_t* gm = ws.hmass + (static_cast<int64_t>(row) * ws.smax + chunk) * kNB;
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
    s.flags = bad_c | (timed_out ? 2 : 0) | (ctrl->ncand > kCapC ? 4 : 0) | (binovf ? 8 : 0);
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
  float tau_max = RL_NEG_INF;
  for (int c = 0; c < S; ++c) {
    const ChunkSum& s = sums_s[c];
    gallow += s.nallow;
    gflags |= s.flags;
    if (s.nallow > 0) tau_max = fmaxf(tau_max, s.tau);
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
  else if (gflags & 12) row_st = RL_ERR_UNSUPPORTED;

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
  uint64_t* keys = reinterpret_cast<uint64_t*>(data);         // kMergeCap / 2 keys
  uint64_t* keys2 = keys + kMergeCap / 2;                     // kMergeCap / 2 keys
  double* gcnt = reinterpret_cast<double*>(keys + kMergeCap);  // kNB (histogram path)
  double* gmass = gcnt + kNB;                                  // kNB
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
    ctrl->nsel = 0;
  }
  __syncthreads();

  if (thr_path) {
    // ---- the row's top-k: candidates >= the largest chunk threshold ----
    // (the row's k-th value >= every chunk's k-th value >= that chunk's tau)
    for (int c = 0; c < S; ++c) {
      const int n = sums_s[c].ncand;
      const uint64_t* srcc = ws.cands + (static_cast<int64_t>(row) * ws.smax + c) * kCapC;
      for (int i = tid; i < n; i += kCT) {
        const uint64_t key = __ldcg(srcc + i);
        if (key_val(key) >= tau_max) {
          const int idx = atomicAdd(&ctrl->nsel, 1);
          if (idx < kMergeCap / 2) keys[idx] = key;
        }
      }
    }
    __syncthreads();
    int n = ctrl->nsel;
    if (n > kMergeCap / 2) {
      finish(RL_ERR_UNSUPPORTED, -1, 0.0f);
      return;
    }
    // tighten once more on the merged keys, then rank-sort the survivors
    {
      float tm = RL_NEG_INF;
      for (int i = tid; i < n; i += kCT) tm = fmaxf(tm, key_val(keys[i]));
      float t2 = block_kth_lower_bound(tm, K, rs);
      if (!(t2 > RL_NEG_INF)) t2 = -3.402823466e38f;
      if (tid == 0) ctrl->nsel = 0;
      __syncthreads();
      for (int i = tid; i < n; i += kCT) {
        const uint64_t key = keys[i];
        if (key_val(key) >= t2) keys2[atomicAdd(&ctrl->nsel, 1)] = key;
      }
      __syncthreads();
      n = ctrl->nsel;
    }
    const int nlist = min(K, n);
    rank_sort(keys2, n, keys, nlist);  // keys[0..nlist): the top-k, descending
    double cum_at = 0.0;
    const int f = sweep(keys, nlist, *wk, m, rt, 0, rs, &cum_at);
    const int cut = (f == INT_MAX) ? nlist - 1 : f;
    if (f == INT_MAX) {
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
  // Row bin j holds absolute bin A = Bmax - j. A logit of bin A has mass
  // e = e_bin * 2^(((A + 1)/cb - m) * log2(e)/T), e_bin its bin-relative mass.
  const int Bmax = babs(m, rt);
  {
    const double cl = kLog2e / static_cast<double>(T);
    const double cbd = static_cast<double>(rt.cb);
    double cq[kBinsPT], mq[kBinsPT];
    double csum = 0.0, msum = 0.0;
#pragma unroll
    for (int q = 0; q < kBinsPT; ++q) {
      const int j = static_cast<int>(threadIdx.x) * kBinsPT + q;
      double cc = 0.0, mm = 0.0;
      if (j < kNB) {
        const int A = Bmax - j;
        for (int c = 0; c < S; ++c) {
          const ChunkSum& s = sums_s[c];
          if (s.nallow == 0) continue;
          const int i = s.babs_m - A;
          if (i >= 0 && i < kNB) {
            const int64_t base = (static_cast<int64_t>(row) * ws.smax + c) * kNB + i;
            cc += static_cast<double>(__ldcg(ws.hcnt + base));
            mm += static_cast<double>(__ldcg(ws.hmass + base));
          }
        }
        mm *= exp2(((static_cast<double>(A) + 1.0) / cbd - static_cast<double>(m)) * cl) / static_cast<double>(kMassQ);
      }
      cq[q] = cc;
      mq[q] = mm;
      csum += cc;
      msum += mm;
    }
    double tc, tm;
    double ci = block_scan_d(csum, rs, &tc) - csum;
    double mi = block_scan_d(msum, rs, &tm) - msum;
#pragma unroll
    for (int q = 0; q < kBinsPT; ++q) {
      const int j = static_cast<int>(threadIdx.x) * kBinsPT + q;
      ci += cq[q];
      mi += mq[q];
      if (j < kNB) {
        gcnt[j] = ci;
        gmass[j] = mi;
      }
    }
    __syncthreads();
  }
  // gcnt / gmass: inclusive cumulative counts / masses per row bin
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
  uint64_t* bkeys = keys;   // keys of one bin (<= kMergeCap / 2)
  uint64_t* skeys = keys2;  // the same, sorted
  int nh = -1;              // history table built on the first re-read
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
            if (idx < kMergeCap / 2) bkeys[idx] = key;
          }
        }
      }
    } else {
      // re-read the row (L2-resident) for the logits of bin A
      if (nh < 0) {
        // sorted, de-duplicated history ids with their penalised values
        int hlr = a.hist ? a.hist_len[row] : 0;
        hlr = max(0, min(hlr, min(a.hist_stride, kHmax)));
        if (tid == 0) ctrl->nsel = 0;
        __syncthreads();
        for (int j = tid; j < hlr; j += kCT) {
          const int hv = a.hist[static_cast<int64_t>(row) * a.hist_stride + j] - a.vocab_offset;
          if (hv >= 0 && hv < V) bkeys[atomicAdd(&ctrl->nsel, 1)] = (static_cast<uint64_t>(hv) << 32) | j;
        }
        __syncthreads();
        const int nrows = ctrl->nsel;
        rank_sort(bkeys, nrows, skeys, nrows);  // descending (id, position)
        const E* xr0 = reinterpret_cast<const E*>(a.logits) + static_cast<int64_t>(row) * a.ld;
        if (tid == 0) ctrl->nsel = 0;
        __syncthreads();
        // ascending position p is skeys[nrows - 1 - p]; the first of each id run applies
        for (int p = tid; p < nrows; p += kCT) {
          const int id = static_cast<int>(skeys[nrows - 1 - p] >> 32);
          if (p > 0 && static_cast<int>(skeys[nrows - p] >> 32) == id) continue;
          int c = 0;
          for (int q = p; q < nrows && static_cast<int>(skeys[nrows - 1 - q] >> 32) == id; ++q) ++c;
          float v;
          if constexpr (sizeof(E) == 4) {
            v = __ldcg(xr0 + id);
          } else {
            v = bf16_bits_to_f32(__ldcg(reinterpret_cast<const unsigned short*>(xr0) + id));
          }
          const float x1 = (v < 0.0f) ? mul_rn(v, prm.repeat_penalty) : div_rn(v, prm.repeat_penalty);
          const float pv = sub_rn(sub_rn(x1, mul_rn(static_cast<float>(c), prm.frequency_penalty)), prm.presence_penalty);
          bkeys[atomicAdd(&ctrl->nsel, 1)] = (static_cast<uint64_t>(static_cast<uint32_t>(id)) << 32) | __float_as_uint(pv);
        }
        __syncthreads();
        nh = ctrl->nsel;
        rank_sort(bkeys, nh, skeys, nh);  // descending id
        for (int j = tid; j < nh; j += kCT) {
          const uint64_t kv = skeys[nh - 1 - j];  // ascending id
          hid[j] = static_cast<int32_t>(kv >> 32);
          hval[j] = __uint_as_float(static_cast<uint32_t>(kv & 0xffffffffu));
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
          if (idx < kMergeCap / 2) bkeys[idx] = cand_key(x, static_cast<uint32_t>(i));
        }
      }
    }
    __syncthreads();
    const int nb = ctrl->nbin;
    if (nb > kMergeCap / 2) {
      if (tid == 0) wk->status = RL_ERR_UNSUPPORTED;
      break;
    }
    rank_sort(bkeys, nb, skeys, nb);
    if (tid == 0) {
      wk->count_before = bin ? static_cast<long long>(gcnt[bin - 1]) : 0;
      wk->mass_before = bin ? gmass[bin - 1] : 0.0;
    }
    __syncthreads();
    int next = INT_MAX;
    double cum_at = 0.0;
    if (wk->phase == 0) {
      const int f = sweep(skeys, nb, *wk, m, rt, 0, rs, &cum_at);
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
        const int d = sweep(skeys, nb, *wk, m, rt, 1, rs, &cum_at);
        if (tid == 0) {
          int j = -1;
          if (d != INT_MAX && (!wk->cut_in_seg || d <= wk->cut_idx)) j = d;
          else if (wk->cut_in_seg) j = wk->cut_idx;
          if (j >= 0) {
            const uint64_t key = skeys[j];
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
  if (a.list_len && tid == 0) a.list_len[row] = -1;  // lists are reported on the threshold path
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

cudaError_t launch_spec(const SpecArgs& a, int dtype, cudaStream_t stream) {
  const int S = spec_chunks(a.V);
  const int smem = spec_smem_bytes(dtype == RL_BF16 ? 2 : 4);
  if (dtype == RL_BF16) return launch_typed<uint16_t>(a, S, smem, stream);
  return launch_typed<float>(a, S, smem, stream);
}

}  // namespace rl
