// Batched spec sampling: penalties -> mask -> temperature -> softmax ->
// top-k -> top-p -> draw, one thread-block cluster per row.
//
// Reference behaviour (chenyusolar/rust-llm, src/decoder.rs):
//   temperature softmax        Decoder::sample_with_params   decoder.rs:44-55
//   repetition penalty rule    Decoder::apply_repeat_penalty decoder.rs:102-110
//   top-k order                Decoder::top_k_logits         decoder.rs:112-122
//   inclusive top-p cutoff     Decoder::sample_top_p         decoder.rs:124-144
//   strict '<' draw            Decoder::sample_multinomial   decoder.rs:146-158
//   empty allowed set -> all   Sampler::sample_with_grammar  decoder.rs:362-364
//
// Design (B200, sm_100a): the row is split over the C CTAs of a cluster; each
// CTA pulls its slice into shared memory with bulk async copies
// (cp.async.bulk + mbarrier): one HBM read per logit. Every later pass runs
// out of shared memory. Cross-CTA reductions go through distributed shared
// memory and cluster barriers; rank 0 plans and finishes:
//   B0  mask popcount exchange (overlaps the copy)
//   P1  max / argmax / allowed count                         -> R1 exchange
//   P2  exact l = (x - m)/T, e = exp(l), Z partials, count and
//       mass histograms over l (16 bins per nat, 64 nats)    -> R2, rank 0 merges
//   P3  collect the elements of the bins rank 0 asks for into its buffer
//       (one round in the common case, a few for very large nuclei)
//   rank 0 sorts the collected keys (value desc, id asc), runs exact
//   cumulative sums from the histogram prefix, finds the cutoff and the draw.
// No global scratch memory is used.
#include <climits>

#include "common.cuh"
#include "spec_kernel.cuh"

namespace rl {

// bf16 slices cannot hold a penalised f32 value in place: the slot gets this
// NaN pattern and the value lives in a side table.
constexpr uint16_t kBf16Marker = 0x7fc1;
constexpr uint16_t kBf16NegInf = 0xff80;

struct RowCtx {
  float m;        // max allowed (penalised) logit
  float T, rT;    // temperature and RN(1/T)
  bool fast_div;  // Markstein division is valid for this T
};

__device__ __forceinline__ float temp_div(float d, const RowCtx& c) {
  if (c.fast_div && (d == 0.0f || fabsf(d) >= 8.077935669e-28f /* 2^-90 */))
    return div_fixed(d, c.T, c.rT);
  return div_rn(d, c.T);
}
// l = (x - m) / T exactly as the CPU restatement computes it.
__device__ __forceinline__ float row_l(float x, const RowCtx& c) { return temp_div(sub_rn(x, c.m), c); }
__device__ __forceinline__ int bin_of(float l) {
  const float s = -l * kRbin;  // exact: kRbin is a power of two
  return s < static_cast<float>(kNB) ? static_cast<int>(s) : kNB;
}

// ---------------------------------------------------------------------------
// Slice access: values of G consecutive elements per 16-byte shared load.
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
  const int32_t* pen_id;  // local ids of the penalised entries (-1: duplicate)
  const float* pen_val;   // their penalised values
  int n_pen;
  __device__ __noinline__ float lookup(int local) const {
    for (int t = 0; t < n_pen; ++t)
      if (pen_id[t] == local) return pen_val[t];
    return __int_as_float(0x7fffffff);  // a NaN input stays NaN
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
// Block helpers (kNT threads)
// ---------------------------------------------------------------------------
struct RedScratch {
  double d[kNWarp];
  float f[kNWarp];
  int i[kNWarp];
  int j[kNWarp];
  int k[kNWarp];
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
    double t = lane < kNWarp ? rs->d[lane] : 0.0;
    t = warp_sum_d(t);
    if (lane == 0) rs->bcast_d = t;
  }
  __syncthreads();
  return rs->bcast_d;
}

__device__ __forceinline__ int block_sum_i(int v, RedScratch* rs) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  v = warp_sum_i(v);
  __syncthreads();
  if (lane == 0) rs->i[warp] = v;
  __syncthreads();
  if (warp == 0) {
    int t = lane < kNWarp ? rs->i[lane] : 0;
    t = warp_sum_i(t);
    if (lane == 0) rs->bcast_i = t;
  }
  __syncthreads();
  return rs->bcast_i;
}

__device__ __forceinline__ int block_min_i(int v, RedScratch* rs) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = min(v, __shfl_xor_sync(0xffffffffu, v, o));
  __syncthreads();
  if (lane == 0) rs->i[warp] = v;
  __syncthreads();
  if (warp == 0) {
    int t = lane < kNWarp ? rs->i[lane] : INT_MAX;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) t = min(t, __shfl_xor_sync(0xffffffffu, t, o));
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
    double t = lane < kNWarp ? rs->d[lane] : 0.0;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const double n = __shfl_up_sync(0xffffffffu, t, o);
      if (lane >= o) t += n;
    }
    if (lane < kNWarp) rs->d[lane] = t;
  }
  __syncthreads();
  const double off = warp > 0 ? rs->d[warp - 1] : 0.0;
  *total = rs->d[kNWarp - 1];
  return v + off;
}

// Descending bitonic sort of P (power of two, <= kCap) 64-bit keys.
__device__ void block_sort_desc(uint64_t* s, int P) {
  for (int k = 2; k <= P; k <<= 1) {
    for (int j = k >> 1; j > 0; j >>= 1) {
      for (int i = threadIdx.x; i < P; i += kNT) {
        const int ixj = i ^ j;
        if (ixj > i) {
          const uint64_t a = s[i], b = s[ixj];
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

__device__ __forceinline__ void cluster_arrive_relaxed() {
  asm volatile("barrier.cluster.arrive.relaxed.aligned;" ::: "memory");
}
__device__ __forceinline__ void cluster_wait() {
  asm volatile("barrier.cluster.wait.aligned;" ::: "memory");
}

// ---------------------------------------------------------------------------
// Shared-memory layout
// ---------------------------------------------------------------------------
struct Xch {
  float max;
  int argmax;
  int nallow;
  int bad;
  int pop;
  int pad;
  double z;
};

enum PlanOp : int { kPlanDone = 0, kPlanCollect = 1 };

struct Plan {
  int op;
  int lo, hi;  // inclusive bin range
  float x_lo, x_hi;
};

struct Ctrl {
  int n_local;
  int cand_count;
  int timeout;
  int pad;
};

// Rank-0 state of the walk down the ordered list.
struct Walk {
  int phase;        // 0: find the cutoff, 1: find the draw, 2: done
  int K;            // list length
  int mass_mode;    // top_p < 1
  int fast;         // the collected segment starts at the top of the list
  int seg_lo, seg_hi;
  int cut_in_seg;   // the cutoff element is in the current segment
  int cut_idx;      // its index in the sorted segment
  long long count_before;
  double mass_before;  // e-units above the segment
  double Z;
  double t2;           // top_p * Z
  double S;            // mass through the cutoff element
  double t3;           // u * S
  int token;
  float prob;
  int status;
  int list_done;
};

constexpr int kOffMbar = 0;
constexpr int kOffXch = 128;
constexpr int kOffPlan = kOffXch + kCmax * static_cast<int>(sizeof(Xch));
constexpr int kOffCtrl = kOffPlan + 64;
constexpr int kOffWalk = kOffCtrl + 64;
constexpr int kOffRed = kOffWalk + 256;
constexpr int kOffCnt = 2048;
constexpr int kOffMass = kOffCnt + kNB * 4;
constexpr int kOffCand = kOffMass + kNB * 8;
constexpr int kOffHist = kOffCand + kCap * 8;
constexpr int kOffPen = kOffHist + kHmax * 4;
constexpr int kOffData = kOffPen + kHmax * 4;
static_assert(sizeof(Walk) <= 256, "walk state");
static_assert(kOffRed + sizeof(RedScratch) <= kOffCnt, "smem header overflow");
static_assert(kOffData % 128 == 0, "data alignment");

int spec_smem_bytes(int L, int es) { return kOffData + L * es; }

// Conservative x-range of the bins [lo, hi]; the exact bin test follows.
__device__ __forceinline__ void plan_bounds(Plan& p, float m, float T) {
  p.x_lo = m - T * (static_cast<float>(p.hi + 1) / kRbin) * 1.001f - 1e-30f;
  p.x_hi = p.lo == 0 ? RL_POS_INF : m - T * (static_cast<float>(p.lo) / kRbin) * 0.999f + 1e-30f;
}

// First nonempty bin after `b` (cumulative counts in cnt), kNB if none.
__device__ __forceinline__ int next_nonempty(const uint32_t* cnt, int b) {
  for (int q = b + 1; q < kNB; ++q)
    if (cnt[q] > cnt[q - 1]) return q;
  return kNB;
}

// Sweep over the sorted segment: first index j whose running cumulative mass
// (mass_before + e_0 + ... + e_j) satisfies the condition. mode 0: cutoff
// (list position K-1, or cum >= t2 when mass_mode); mode 1: cum > t3.
// Returns INT_MAX if none; *cum_at receives the cumulative mass at j.
__device__ int sweep_segment(const uint64_t* cand, int n, const Walk& w, const RowCtx& rc,
                             int mode, RedScratch* rs, double* cum_at) {
  double run = w.mass_before;
  for (int c0 = 0; c0 < n; c0 += kNT) {
    const int j = c0 + threadIdx.x;
    const bool valid = j < n;
    float e = 0.0f;
    if (valid) e = expf(row_l(key_val(cand[j]), rc));
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

// ---------------------------------------------------------------------------
// The kernel
// ---------------------------------------------------------------------------
template <typename E>
__global__ void __launch_bounds__(kNT, 2) spec_sample_kernel(const SpecArgs a) {
  extern __shared__ __align__(128) unsigned char smem[];
  cg::cluster_group cluster = cg::this_cluster();
  cluster_arrive_relaxed();  // matched by cluster_wait() before the first DSMEM access
  const int rank = static_cast<int>(cluster.block_rank());
  const int C = static_cast<int>(cluster.num_blocks());
  const int row = blockIdx.y;
  const int tid = threadIdx.x;
  const int lane = tid & 31;
  const int warp = tid >> 5;

  uint64_t* mbar = reinterpret_cast<uint64_t*>(smem + kOffMbar);
  Xch* xch = reinterpret_cast<Xch*>(smem + kOffXch);
  Plan* plan = reinterpret_cast<Plan*>(smem + kOffPlan);
  Ctrl* ctrl = reinterpret_cast<Ctrl*>(smem + kOffCtrl);
  Walk* wk = reinterpret_cast<Walk*>(smem + kOffWalk);
  RedScratch* rs = reinterpret_cast<RedScratch*>(smem + kOffRed);
  uint32_t* cnt = reinterpret_cast<uint32_t*>(smem + kOffCnt);
  unsigned long long* mass = reinterpret_cast<unsigned long long*>(smem + kOffMass);
  uint64_t* cand = reinterpret_cast<uint64_t*>(smem + kOffCand);
  int32_t* hist_local = reinterpret_cast<int32_t*>(smem + kOffHist);
  float* pen_val = reinterpret_cast<float*>(smem + kOffPen);
  E* data = reinterpret_cast<E*>(smem + kOffData);

  const int L = a.L;
  const int V = a.V;
  const int start = rank * L;
  const int len = max(0, min(L, V - start));
  constexpr int es = static_cast<int>(sizeof(E));
  constexpr int G = Slice<E>::G;
  const int ngroups = L / G;

  const rl_row_params prm = a.params[row];
  const float u = a.uniforms[row];

  // ---- prologue: mbarriers, bulk copy of the slice ----
  const E* src = reinterpret_cast<const E*>(a.logits) + static_cast<int64_t>(row) * a.ld + start;
  const uint32_t bulk_bytes = static_cast<uint32_t>(len * es) & ~15u;
  const bool use_bulk = ((reinterpret_cast<uintptr_t>(src) & 15u) == 0) && bulk_bytes > 0;
  if (tid == 0) {
    for (int p = 0; p < kNPiece; ++p) mbar_init(&mbar[p], 1);
    fence_mbar_init();
    ctrl->n_local = 0;
    ctrl->cand_count = 0;
    ctrl->timeout = 0;
  }
  for (int b = tid; b < kNB; b += kNT) {
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

  // history ids inside this slice (local index), overlapping the copy
  const int vstart = a.vocab_offset + start;
  int hl = a.hist ? a.hist_len[row] : 0;
  hl = max(0, min(hl, min(a.hist_stride, kHmax)));
  for (int j = tid; j < hl; j += kNT) {
    const int h = a.hist[static_cast<int64_t>(row) * a.hist_stride + j];
    const int loc = h - vstart;
    if (h >= a.vocab_offset && loc >= 0 && loc < len) {
      const int idx = atomicAdd(&ctrl->n_local, 1);
      hist_local[idx] = loc;
    }
  }
  // mask popcount over this slice (ids < V only)
  int pop = 0;
  const uint32_t* mrow = a.mask ? a.mask + static_cast<int64_t>(row) * a.mask_stride : nullptr;
  if (mrow) {
    const int w0 = start >> 5;
    const int nw = (len + 31) >> 5;
    for (int w = tid; w < nw; w += kNT) {
      uint32_t bits = mrow[w0 + w];
      const int rem = len - w * 32;
      if (rem < 32) bits &= (1u << rem) - 1u;
      pop += __popc(bits);
    }
  }
  pop = block_sum_i(pop, rs);
  cluster_wait();  // every CTA of the cluster has started
  if (tid < C) cluster.map_shared_rank(&xch[rank], tid)->pop = pop;
  cluster.sync();  // B0
  bool mask_on = false;
  if (mrow) {
    int tot = 0;
    for (int r = 0; r < C; ++r) tot += xch[r].pop;
    mask_on = tot > 0;
  }

  // ---- wait for the slice; unaligned remainder; pad the tail ----
  if (use_bulk) {
    bool ok = true;
    for (int p = 0; p < kNPiece; ++p) ok &= mbar_wait(&mbar[p], 0, kWaitBudget);
    if (!ok) ctrl->timeout = 1;
  }
  {
    const int first_plain = use_bulk ? static_cast<int>(bulk_bytes / es) : 0;
    for (int i = first_plain + tid; i < len; i += kNT) data[i] = src[i];
    E neg;
    if constexpr (sizeof(E) == 4) {
      neg = RL_NEG_INF;
    } else {
      neg = kBf16NegInf;
    }
    for (int i = len + tid; i < L; i += kNT) data[i] = neg;
  }
  __syncthreads();

  // ---- penalties on this slice's history ids (first occurrence applies) ----
  const int n_local = min(ctrl->n_local, kHmax);
  for (int t = tid; t < n_local; t += kNT) {
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
      const float x2 = sub_rn(x1, mul_rn(static_cast<float>(c), prm.frequency_penalty));
      const float x3 = sub_rn(x2, prm.presence_penalty);
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
    for (int t = tid; t < n_local; t += kNT) {
      const int h = hist_local[t];
      bool first = true;
      for (int j = 0; j < t; ++j)
        if (hist_local[j] == h) first = false;
      if (first) data[h] = kBf16Marker;
    }
    __syncthreads();
    for (int t = tid; t < n_local; t += kNT) {
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

  // ---- P1: max / lowest argmax / allowed count / non-finite ----
  float mx = RL_NEG_INF;
  int amx = INT_MAX;
  int nallow = 0;
  int bad = 0;
  for (int g = tid; g < ngroups; g += kNT) {
    float v[G];
    sl.load(g, v);
    uint32_t bits = 0xffffffffu;
    if (mask_on) bits = (start + g * G < V) ? (mrow[(start + g * G) >> 5] >> ((g * G) & 31)) : 0u;
#pragma unroll
    for (int k = 0; k < G; ++k) {
      const float x = v[k];
      const bool on = (bits >> k) & 1u;
      if (on && x > RL_NEG_INF) {
        if (!(x < RL_POS_INF)) bad = 1;
        ++nallow;
        if (x > mx) {
          mx = x;
          amx = g * G + k;
        }
      } else if (on && x != x) {
        bad = 1;
      }
    }
  }
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
    if (tid == 0) {
      float bm = RL_NEG_INF;
      int ba = INT_MAX, bn = 0, bb = 0;
      for (int w = 0; w < kNWarp; ++w) {
        bn += rs->j[w];
        bb |= rs->k[w] ? 1 : 0;
        if (rs->f[w] > bm) {
          bm = rs->f[w];
          ba = rs->i[w];
        } else if (rs->f[w] == bm) {
          ba = min(ba, rs->i[w]);
        }
      }
      rs->f[0] = bm;
      rs->i[0] = ba == INT_MAX ? INT_MAX : ba + start;
      rs->j[0] = bn;
      rs->k[0] = bb | (ctrl->timeout ? 2 : 0);
    }
    __syncthreads();
    if (tid < C) {
      Xch* dst = cluster.map_shared_rank(&xch[rank], tid);
      dst->max = rs->f[0];
      dst->argmax = rs->i[0];
      dst->nallow = rs->j[0];
      dst->bad = rs->k[0];
    }
  }
  cluster.sync();  // R1
  float m = RL_NEG_INF;
  int gargmax = INT_MAX;
  int gallow = 0;
  int gbad = 0;
  for (int r = 0; r < C; ++r) {
    const Xch& s = xch[r];
    gallow += s.nallow;
    gbad |= s.bad;
    if (s.max > m) {
      m = s.max;
      gargmax = s.argmax;
    } else if (s.max == m) {
      gargmax = min(gargmax, s.argmax);
    }
  }
  const float T = prm.temperature;
  int row_st = 0;
  if (gbad & 2)
    row_st = RL_ERR_TIMEOUT;
  else if (gbad || gallow == 0 || !(fabsf(T) < RL_POS_INF))
    row_st = RL_ERR_NONFINITE;
  if (row_st != 0 || T <= 0.0f) {
    // greedy row (T <= 0) or invalid row: decided identically in every CTA
    if (rank == 0 && tid == 0) {
      const bool ok = row_st == 0;
      a.out_tok[row] = ok ? gargmax + a.vocab_offset : -1;
      if (a.out_prob) a.out_prob[row] = ok ? 1.0f : 0.0f;
      if (a.row_status) a.row_status[row] = row_st;
      if (a.list_len) {
        a.list_len[row] = (ok && a.list_cap > 0) ? 1 : 0;
        if (ok && a.list_cap > 0) {
          a.list_ids[static_cast<int64_t>(row) * a.list_cap] = gargmax + a.vocab_offset;
          a.list_probs[static_cast<int64_t>(row) * a.list_cap] = 1.0f;
        }
      }
    }
    return;
  }

  // masked ids -> -inf in place, so that the later passes need no mask
  if (mask_on) {
    for (int g = tid; g < ngroups; g += kNT) {
      const uint32_t bits =
          (start + g * G < V) ? (mrow[(start + g * G) >> 5] >> ((g * G) & 31)) : 0u;
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

  RowCtx rc;
  rc.m = m;
  rc.T = T;
  rc.rT = __frcp_rn(T);
  rc.fast_div = (T >= 9.5367431640625e-07f) && (T <= 1048576.0f);
  const int Klist = (prm.top_k > 0 && prm.top_k < gallow) ? prm.top_k : gallow;
  const bool need_q1 = Klist < gallow;
  const bool mass_mode = prm.top_p < 1.0f;
  const bool want_mass = mass_mode || !need_q1;

  // ---- P2: Z partials, count and mass histograms over l ----
  float zsum = 0.0f;
  for (int g = tid; g < ngroups; g += kNT) {
    float v[G];
    sl.load(g, v);
#pragma unroll
    for (int k = 0; k < G; ++k) {
      const float x = v[k];
      if (x > RL_NEG_INF) {
        const float l = row_l(x, rc);
        const float e = expf(l);
        zsum += e;
        const int b = bin_of(l);
        if (b < kNB) {
          atomicAdd(&cnt[b], 1u);
          if (want_mass) atomicAdd(&mass[b], __float2ull_rn(e * kMassScaleF));
        }
      }
    }
  }
  {
    const double zb = block_sum_d(static_cast<double>(zsum), rs);
    if (tid == 0) cluster.map_shared_rank(&xch[rank], 0)->z = zb;
  }
  cluster.sync();  // R2

  // ---- rank 0: merge histograms, first plan ----
  if (rank == 0) {
    double Z = 0.0;
    for (int r = 0; r < C; ++r) Z += xch[r].z;
    for (int b = tid; b < kNB; b += kNT) {
      uint32_t c = cnt[b];
      unsigned long long ms = mass[b];
      for (int r = 1; r < C; ++r) {
        c += *cluster.map_shared_rank(&cnt[b], r);
        if (want_mass) ms += *cluster.map_shared_rank(&mass[b], r);
      }
      cnt[b] = c;
      mass[b] = ms;
    }
    __syncthreads();
    // inclusive prefix sums over the bins (kPer consecutive bins per thread)
    constexpr int kPer = kNB / kNT;
    uint32_t cc[kPer];
    unsigned long long mm[kPer];
    uint32_t csum = 0;
    unsigned long long msum = 0;
#pragma unroll
    for (int q = 0; q < kPer; ++q) {
      csum += cnt[tid * kPer + q];
      msum += mass[tid * kPer + q];
      cc[q] = csum;
      mm[q] = msum;
    }
    double ctot, mtot;
    // doubles hold these integers exactly (counts < 2^31, masses < 2^53)
    const double cpre = block_scan_d(static_cast<double>(csum), rs, &ctot) - static_cast<double>(csum);
    const double mpre = block_scan_d(static_cast<double>(msum), rs, &mtot) - static_cast<double>(msum);
#pragma unroll
    for (int q = 0; q < kPer; ++q) {
      cnt[tid * kPer + q] = cc[q] + static_cast<uint32_t>(cpre);
      mass[tid * kPer + q] = mm[q] + static_cast<unsigned long long>(mpre);
    }
    __syncthreads();
    // cnt / mass now hold inclusive cumulative counts / masses.
    const double t2 = static_cast<double>(prm.top_p) * Z;
    const double t2q = t2 * kMassScale;
    const double t3z = static_cast<double>(u) * Z;  // draw target when the list is everything
    const double t3zq = t3z * kMassScale;
    int b1 = kNB, b2 = kNB, b3 = kNB;
    for (int b = tid; b < kNB; b += kNT) {
      const uint32_t pc = b ? cnt[b - 1] : 0u;
      if (cnt[b] >= static_cast<uint32_t>(Klist) && pc < static_cast<uint32_t>(Klist)) b1 = b;
      const double pm = b ? static_cast<double>(mass[b - 1]) : 0.0;
      const double cm = static_cast<double>(mass[b]);
      if (mass_mode && cm >= t2q && pm < t2q) b2 = b;
      if (cm > t3zq && pm <= t3zq) b3 = b;
    }
    b1 = block_min_i(b1, rs);
    b2 = block_min_i(b2, rs);
    b3 = block_min_i(b3, rs);
    if (tid == 0) {
      Walk& w = *wk;
      w.K = Klist;
      w.mass_mode = mass_mode;
      w.Z = Z;
      w.t2 = t2;
      w.S = 0.0;
      w.t3 = 0.0;
      w.status = 0;
      w.token = -1;
      w.prob = 0.0f;
      w.cut_in_seg = 0;
      w.cut_idx = -1;
      w.list_done = 0;
      Plan p;
      p.op = kPlanCollect;
      if (!need_q1 && !mass_mode) {
        // the list is every allowed id: the cutoff is its end, S = Z
        w.phase = 1;
        w.S = Z;
        w.t3 = t3z;
        if (b3 >= kNB) {
          w.status = RL_ERR_UNSUPPORTED;  // draw beyond the 64-nat window
          p.op = kPlanDone;
        } else if (cnt[b3] <= static_cast<uint32_t>(kCap)) {
          p.lo = 0;
          p.hi = b3;
        } else {
          p.lo = b3;
          p.hi = b3;
        }
      } else {
        w.phase = 0;
        const int bA = min(b1, b2);
        if (bA >= kNB) {
          w.status = RL_ERR_UNSUPPORTED;  // cutoff beyond the 64-nat window
          p.op = kPlanDone;
        } else {
          int bF = (mass_mode && b2 <= b1) ? min(bA + 1, min(b1, kNB - 1)) : bA;
          if (a.list_len) {
            // debug: also collect the first min(K, list_cap) list entries
            const uint32_t want = static_cast<uint32_t>(min(Klist, a.list_cap));
            int bL = bF;
            while (bL < kNB - 1 && cnt[bL] < want) ++bL;
            if (cnt[bL] <= static_cast<uint32_t>(kCap)) bF = max(bF, bL);
          }
          if (cnt[bF] <= static_cast<uint32_t>(kCap)) {
            p.lo = 0;
            p.hi = bF;
          } else {
            p.lo = bA;
            p.hi = bA;
          }
        }
      }
      if (p.op == kPlanCollect) {
        const uint32_t pop_lo = cnt[p.hi] - (p.lo ? cnt[p.lo - 1] : 0u);
        if (pop_lo > static_cast<uint32_t>(kCap)) {
          w.status = RL_ERR_UNSUPPORTED;  // one bin holds more than the buffer
          p.op = kPlanDone;
        }
      }
      w.fast = p.lo == 0;
      w.seg_lo = p.lo;
      w.seg_hi = p.hi;
      w.count_before = p.lo ? cnt[p.lo - 1] : 0;
      w.mass_before = p.lo ? static_cast<double>(mass[p.lo - 1]) / kMassScale : 0.0;
      plan_bounds(p, m, T);
      ctrl->cand_count = 0;
      for (int r = 0; r < C; ++r) *cluster.map_shared_rank(plan, r) = p;
    }
  }

  // ---- collection rounds (uniform across the cluster) ----
  for (int round = 0;; ++round) {
    cluster.sync();  // plan visible everywhere
    const Plan p = *plan;
    if (p.op == kPlanDone) break;
    int* rcount = cluster.map_shared_rank(&ctrl->cand_count, 0);
    uint64_t* rcand = cluster.map_shared_rank(cand, 0);
    for (int gb = warp * 32; gb < ngroups; gb += kNT) {
      const int g = gb + lane;
      float v[G];
      if (g < ngroups) {
        sl.load(g, v);
      } else {
#pragma unroll
        for (int k = 0; k < G; ++k) v[k] = RL_NEG_INF;
      }
#pragma unroll
      for (int k = 0; k < G; ++k) {
        const float x = v[k];
        bool take = false;
        if (x >= p.x_lo && x <= p.x_hi && x > RL_NEG_INF) {
          const int b = bin_of(row_l(x, rc));
          take = b >= p.lo && b <= p.hi;
        }
        const uint32_t bal = __ballot_sync(0xffffffffu, take);
        if (bal) {
          int base = 0;
          if (lane == 0) base = atomicAdd(rcount, __popc(bal));
          base = __shfl_sync(0xffffffffu, base, 0);
          if (take) {
            const int idx = base + __popc(bal & ((1u << lane) - 1u));
            if (idx < kCap) rcand[idx] = cand_key(x, static_cast<uint32_t>(start + g * G + k));
          }
        }
      }
    }
    cluster.sync();  // collected
    if (rank != 0) continue;

    // ---- rank 0: sort and walk the collected segment ----
    Walk& w = *wk;
    const int ncol = ctrl->cand_count;
    int next_lo = -1;  // >= 0: collect this single bin next
    if (ncol > kCap) {
      if (tid == 0) w.status = RL_ERR_UNSUPPORTED;
    } else if (ncol > 0) {
      int P = 1;
      while (P < ncol) P <<= 1;
      for (int i = ncol + tid; i < P; i += kNT) cand[i] = 0ull;
      __syncthreads();
      block_sort_desc(cand, P);
      double cum_at = 0.0;
      if (w.phase == 0) {
        const int f = sweep_segment(cand, ncol, w, rc, 0, rs, &cum_at);
        if (f != INT_MAX) {
          if (tid == 0) {
            w.cut_in_seg = 1;
            w.cut_idx = f;
            w.S = cum_at;
            w.t3 = static_cast<double>(u) * cum_at;
            w.phase = 1;
          }
          __syncthreads();
          if (a.list_len && w.fast && tid == 0) w.list_done = 1;
          if (a.list_len && w.fast) {
            // the ordered list from its top through the cutoff (or the K-th)
            const int nl = min(min(w.K, ncol), a.list_cap);
            for (int j = tid; j < nl; j += kNT) {
              const uint64_t key = cand[j];
              a.list_ids[static_cast<int64_t>(row) * a.list_cap + j] =
                  static_cast<int>(key_id(key)) + a.vocab_offset;
              a.list_probs[static_cast<int64_t>(row) * a.list_cap + j] =
                  static_cast<float>(static_cast<double>(expf(row_l(key_val(key), rc))) / w.Z);
            }
            if (tid == 0) a.list_len[row] = (nl == min(w.K, a.list_cap)) ? nl : -1;
          }
        } else {
          next_lo = next_nonempty(cnt, w.seg_hi);
        }
      } else if (tid == 0) {
        w.cut_in_seg = 0;
      }
      __syncthreads();
      if (w.phase == 1 && next_lo < 0) {
        if (w.t3 < w.mass_before) {
          // the draw lies above this segment: locate its bin
          const double t3q = w.t3 * kMassScale;
          int b3 = kNB;
          for (int b = tid; b < kNB; b += kNT) {
            const double pm = b ? static_cast<double>(mass[b - 1]) : 0.0;
            if (static_cast<double>(mass[b]) > t3q && pm <= t3q) b3 = b;
          }
          b3 = block_min_i(b3, rs);
          next_lo = (b3 < w.seg_lo) ? b3 : max(0, w.seg_lo - 1);
          if (tid == 0) w.cut_in_seg = 0;
        } else {
          const int f = sweep_segment(cand, ncol, w, rc, 1, rs, &cum_at);
          if (tid == 0) {
            int j = -1;
            if (f != INT_MAX && (!w.cut_in_seg || f <= w.cut_idx)) j = f;
            else if (w.cut_in_seg) j = w.cut_idx;  // u*S reached nowhere before the cutoff
            if (j >= 0) {
              const uint64_t key = cand[j];
              const float e = expf(row_l(key_val(key), rc));
              w.token = static_cast<int>(key_id(key));
              w.prob = static_cast<float>(static_cast<double>(e) / w.S);
              w.phase = 2;
            }
          }
          __syncthreads();
          if (w.phase != 2) next_lo = next_nonempty(cnt, w.seg_hi);
        }
      }
    } else {
      // empty segment: move on
      next_lo = next_nonempty(cnt, w.seg_hi);
    }
    __syncthreads();
    if (tid == 0) {
      Plan np;
      np.op = kPlanDone;
      if (w.status == 0 && w.phase != 2) {
        if (next_lo < 0 || next_lo >= kNB || round + 1 >= kMaxRounds) {
          w.status = RL_ERR_UNSUPPORTED;
        } else {
          const uint32_t popb = cnt[next_lo] - (next_lo ? cnt[next_lo - 1] : 0u);
          if (popb > static_cast<uint32_t>(kCap)) {
            w.status = RL_ERR_UNSUPPORTED;
          } else {
            np.op = kPlanCollect;
            np.lo = next_lo;
            np.hi = next_lo;
            plan_bounds(np, m, T);
            w.fast = next_lo == 0;
            w.seg_lo = next_lo;
            w.seg_hi = next_lo;
            w.count_before = next_lo ? cnt[next_lo - 1] : 0;
            w.mass_before = next_lo ? static_cast<double>(mass[next_lo - 1]) / kMassScale : 0.0;
          }
        }
      }
      ctrl->cand_count = 0;
      for (int r = 0; r < C; ++r) *cluster.map_shared_rank(plan, r) = np;
    }
  }

  if (rank == 0 && tid == 0) {
    const Walk& w = *wk;
    const bool ok = w.status == 0 && w.phase == 2;
    const int st = ok ? 0 : (w.status ? w.status : RL_ERR_UNSUPPORTED);
    a.out_tok[row] = ok ? w.token + a.vocab_offset : -1;
    if (a.out_prob) a.out_prob[row] = ok ? w.prob : 0.0f;
    if (a.row_status) a.row_status[row] = st;
    if (a.list_len && !w.list_done) a.list_len[row] = -1;
  }
}

// ---------------------------------------------------------------------------
// Host launcher
// ---------------------------------------------------------------------------
int spec_pick_cluster(int B, int V, int es, int num_sms) {
  // smallest power of two keeping each slice <= 64 KB (two CTAs per SM)...
  int C = 1;
  while (C < kCmax && static_cast<int64_t>(V) * es > static_cast<int64_t>(C) * 65536) C <<= 1;
  // ...then widen small batches so that one row spreads over more SMs
  while (C < 8 && static_cast<int64_t>(B) * C * 2 <= num_sms) C <<= 1;
  return C;
}

template <typename E>
static cudaError_t launch_typed(const SpecArgs& a, int C, int smem, cudaStream_t stream) {
  auto k = spec_sample_kernel<E>;
  cudaError_t err = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  if (err == cudaSuccess && C > 8)
    err = cudaFuncSetAttribute(k, cudaFuncAttributeNonPortableClusterSizeAllowed, 1);
  if (err != cudaSuccess) return err;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(C, a.B, 1);
  cfg.blockDim = dim3(kNT, 1, 1);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = C;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, k, a);
}

cudaError_t launch_spec(const SpecArgs& args_in, int dtype, int num_sms, cudaStream_t stream) {
  SpecArgs a = args_in;
  const int es = dtype == RL_BF16 ? 2 : 4;
  const int C = spec_pick_cluster(a.B, a.V, es, num_sms);
  const int per = (a.V + C - 1) / C;
  a.L = ((per + 127) / 128) * 128;
  const int smem = spec_smem_bytes(a.L, es);
  if (dtype == RL_BF16) return launch_typed<uint16_t>(a, C, smem, stream);
  return launch_typed<float>(a, C, smem, stream);
}

}  // namespace rl
