// CPU oracle for the logits -> token sampling path of chenyusolar/rust-llm.
//
// TEST INFRASTRUCTURE ONLY. This file is the oracle the CUDA sampler is tested against:
// only tests/, __graft_entry__.smoke() and bench.py's cpu_baseline / reference
// legs may load it. The product library never links or calls it.
//
// PARITY UNPINNED: the reference (src/decoder.rs, scalar Rust) cannot be
// built here (no cargo/rustc) and its own test suite holds no golden vectors
// for this path (its only tests are src/utils.rs:246-263, unrelated). This
// restatement is cross-checked against an independent pure-Python restatement
// (tests/golden/make_golden.py) and against hand-derived known-answer cases,
// not against outputs of the reference itself.
//
// Two profiles:
//
//  ref_exact  -- a literal restatement of the live reference path:
//     Decoder::sample_with_params   src/decoder.rs:35-100   (orc_decoder_sample)
//     Decoder::greedy_sample        src/decoder.rs:160-167  (orc_greedy)
//     Sampler::sample_with_grammar  src/decoder.rs:359-376  (orc_grammar_greedy)
//     BeamSearch::search, one step  src/decoder.rs:217-276  (orc_beam_step, raw logits)
//     SpeculativeDecoder::sample, softmax_at, verify_and_accept
//                                   src/inference.rs:335-429 (orc_specdec_*)
//     Model::matmul_vec (the LM head) src/model.rs:246-261   (orc_matmul_vec)
//     with rand_secure() (src/decoder.rs:170-188) replaced by an injected
//     uniform. All arithmetic is f32, sums are sequential left-to-right,
//     exp is the platform libm expf (what Rust's f32::exp lowers to on Linux),
//     sorts are stable descending (slice::sort_by is a stable merge sort).
//
//  spec       -- the batched pipeline the CUDA sampler implements, assembled
//     from the reference's building blocks:
//       repetition penalty sign rule   apply_repeat_penalty  decoder.rs:102-110
//                                      (applied to history ids only)
//       presence / frequency penalty   (no reference code; OpenAI convention)
//       temperature                    sample_with_params    decoder.rs:44-49
//                                      (subtract max, divide by T, exp)
//       top-k order                    top_k_logits          decoder.rs:112-122
//       top-p inclusive cutoff         sample_top_p          decoder.rs:124-144
//       draw with strict '<'           sample_multinomial    decoder.rs:146-158
//     Probability sums and cumulative sums are carried in double so that a
//     parallel device reduction can agree with them to ~1e-9; the per-element
//     arithmetic (penalty, max-subtract, IEEE divide by T) is bit-identical
//     on both sides, only exp() differs (libm vs CUDA, ~1 ulp).
//
// Build: g++ -O2 -std=c++17 -ffp-contract=off -fno-fast-math -fPIC -shared
// (-ffp-contract=off: no a*b+c contraction, so every f32 op rounds like Rust's.)

#include <algorithm>
#include <cmath>
#include <cstdint>
#include <cstring>
#include <cfloat>
#include <thread>
#include <vector>
#include <limits>

namespace {

// f32::max semantics: if one argument is NaN the other is returned.
inline float rust_max(float a, float b) { return std::fmax(a, b); }

// partial_cmp(..).unwrap_or(Equal) for a descending sort: "a before b" iff a > b.
inline bool desc_before(float a, float b) { return a > b; }

struct IdVal {
  int32_t id;
  float v;
};

inline float bf16_to_f32(uint16_t h) {
  uint32_t u = static_cast<uint32_t>(h) << 16;
  float f;
  std::memcpy(&f, &u, 4);
  return f;
}

inline bool mask_bit(const uint32_t* mask_row, int i) {
  return (mask_row[i >> 5] >> (i & 31)) & 1u;
}

}  // namespace

extern "C" {

// Row parameters, laid out exactly like rl_row_params in include/rl_sampler.h.
struct orc_row_params {
  float temperature;
  float top_p;
  int32_t top_k;
  float repeat_penalty;
  float presence_penalty;
  float frequency_penalty;
};

// ---------------------------------------------------------------------------
// ref_exact: Decoder::sample_with_params (src/decoder.rs:35-100)
// ---------------------------------------------------------------------------
// Returns the token. out_prob (nullable) receives the final probability
// array entry of the returned id (after the top-p renormalisation), which is
// what the reference's logits[i] holds when it returns i.
// out_cutoff (nullable) receives the top-p cutoff position (-1 if top_p >= 1).
// out_draw_margin (nullable) receives min |r - cumsum| over the two cumsum
// values bracketing the draw (how close the draw was to a CDF boundary).
// out_cut_margin (nullable) receives min |top_p - cumsum| over the two sorted
// cumsum values bracketing the cutoff.
int32_t orc_decoder_sample(const float* logits_in, int V, float temperature, float top_p,
                           float r, float* out_prob, int32_t* out_cutoff,
                           double* out_draw_margin, double* out_cut_margin) {
  std::vector<float> logits(logits_in, logits_in + V);  // decoder.rs:42 to_vec

  if (temperature > 0.0f) {  // decoder.rs:44-55
    float max_logit = -FLT_MAX;  // f32::MIN
    for (int i = 0; i < V; ++i) max_logit = rust_max(max_logit, logits[i]);
    for (int i = 0; i < V; ++i) logits[i] = (logits[i] - max_logit) / temperature;
    for (int i = 0; i < V; ++i) logits[i] = std::exp(logits[i]);  // expf
    float sum = 0.0f;
    for (int i = 0; i < V; ++i) sum += logits[i];
    if (sum > 0.0f)
      for (int i = 0; i < V; ++i) logits[i] /= sum;
  }

  int32_t cutoff_out = -1;
  double cut_margin = INFINITY;
  if (top_p < 1.0f) {  // decoder.rs:57-81
    std::vector<IdVal> sorted(V);
    for (int i = 0; i < V; ++i) sorted[i] = {i, logits[i]};
    std::stable_sort(sorted.begin(), sorted.end(),
                     [](const IdVal& a, const IdVal& b) { return desc_before(a.v, b.v); });
    float cumsum = 0.0f;
    int cutoff = V;  // unwrap_or(sorted.len())
    float prev = 0.0f;
    for (int i = 0; i < V; ++i) {
      prev = cumsum;
      cumsum += sorted[i].v;
      if (cumsum >= top_p) {
        cutoff = i;
        break;
      }
    }
    if (cutoff < V) {
      cut_margin = std::min(std::fabs((double)cumsum - (double)top_p),
                            std::fabs((double)prev - (double)top_p));
    } else {
      cut_margin = std::fabs((double)cumsum - (double)top_p);
    }
    cutoff_out = cutoff;
    // decoder.rs:71-75: zeroes logits[i] for ORIGINAL id i > cutoff.
    for (int i = 0; i < V; ++i)
      if (i > cutoff) logits[i] = 0.0f;
    float sum = 0.0f;
    for (int i = 0; i < V; ++i) sum += logits[i];
    if (sum > 0.0f)
      for (int i = 0; i < V; ++i) logits[i] /= sum;
  }

  // decoder.rs:83-90: id-order CDF, non-strict comparison.
  float cumsum = 0.0f;
  int32_t tok = -1;
  double draw_margin = INFINITY;
  for (int i = 0; i < V; ++i) {
    float prev = cumsum;
    cumsum += logits[i];
    if (r <= cumsum) {
      tok = i;
      draw_margin = std::min(std::fabs((double)cumsum - (double)r),
                             std::fabs((double)r - (double)prev));
      break;
    }
  }
  if (tok < 0) {
    // decoder.rs:92-97: max_by returns the LAST maximum.
    int best = 0;
    for (int i = 1; i < V; ++i)
      if (!(logits[i] < logits[best])) best = i;  // ties and NaN-Equal move to later
    tok = V > 0 ? best : 0;
    draw_margin = std::fabs((double)cumsum - (double)r);
  }
  if (out_prob) *out_prob = (tok >= 0 && tok < V) ? logits[tok] : 0.0f;
  if (out_cutoff) *out_cutoff = cutoff_out;
  if (out_draw_margin) *out_draw_margin = draw_margin;
  if (out_cut_margin) *out_cut_margin = cut_margin;
  return tok;
}

// Model::matmul_vec (src/model.rs:246-261), the LM head of Model::forward
// (:236-241): logits[i] = sum over j < min(hidden, len / vocab) of
// input[j] * weight[i * hidden + j], left to right in f32, terms whose index
// passes the weight's length left out. Rows of a batch (rows > 1) are
// independent calls of the same loop; rows are split over nthreads threads.
void orc_matmul_vec(const float* input, const float* weight, int64_t weight_len, int hidden, int vocab, int rows,
                    float* out, int nthreads) {
  const int64_t kmax = std::min<int64_t>(hidden, weight_len / std::max(vocab, 1));
  auto run = [&](int r0, int r1) {
    for (int r = r0; r < r1; ++r) {
      const float* x = input + static_cast<int64_t>(r) * hidden;
      float* o = out + static_cast<int64_t>(r) * vocab;
      for (int i = 0; i < vocab; ++i) {
        float sum = 0.0f;
        for (int64_t j = 0; j < kmax; ++j) {
          const int64_t idx = static_cast<int64_t>(i) * hidden + j;
          if (idx < weight_len) sum += x[j] * weight[idx];
        }
        o[i] = sum;
      }
    }
  };
  nthreads = std::max(1, std::min(nthreads, rows));
  if (nthreads == 1) {
    run(0, rows);
    return;
  }
  std::vector<std::thread> ts;
  for (int t = 0; t < nthreads; ++t) ts.emplace_back(run, rows * t / nthreads, rows * (t + 1) / nthreads);
  for (auto& t : ts) t.join();
}

// Decoder::greedy_sample (src/decoder.rs:160-167): argmax, last maximum wins.
int32_t orc_greedy(const float* logits, int V) {
  if (V <= 0) return 0;  // unwrap_or(0)
  int best = 0;
  for (int i = 1; i < V; ++i)
    if (!(logits[i] < logits[best])) best = i;
  return best;
}

// Sampler::sample_with_grammar (src/decoder.rs:359-376) with the allowed set
// given as a bit-packed mask (bit i&31 of word i>>5, LSB first). An empty
// allowed set means every id is allowed (decoder.rs:362-364). Stable
// descending sort of the allowed (id, logit) pairs, take the first: the
// lowest allowed id among the maxima.
int32_t orc_grammar_greedy(const float* logits, int V, const uint32_t* mask_row) {
  int best = -1;
  bool any = false;
  for (int i = 0; i < V; ++i) any |= mask_bit(mask_row, i);
  for (int i = 0; i < V; ++i) {
    if (any && !mask_bit(mask_row, i)) continue;
    if (best < 0 || logits[i] > logits[best]) best = i;
  }
  return best < 0 ? 0 : best;
}

// ---------------------------------------------------------------------------
// spec profile, one row
// ---------------------------------------------------------------------------
// Steps (per row):
//  1. penalties on history ids (unique id i with count c): x1 = x<0 ? x*rp : x/rp;
//     x2 = x1 - (float)c*freq; x3 = x2 - pres. History ids outside [0, V) ignored.
//  2. mask: bit clear -> id excluded. A row whose mask allows nothing allows all.
//     Ids whose logit is -inf after the penalties are excluded as well.
//  3. T <= 0: greedy over allowed x3, ties -> lowest id, prob 1.
//  4. m = max allowed x3; l_i = (x3_i - m) / T (f32, IEEE); e_i = expf(l_i);
//     Z = sum(double e_i); p_i = e_i / Z (double).
//  5. K = top_k > 0 ? min(top_k, n_allowed) : n_allowed; order (x3 desc, id asc).
//  6. top_p < 1: cum_j = sum_{i<=j} p (double); cutoff = first j with cum_j >= top_p,
//     else K; cutoff = min(cutoff, K-1). top_p >= 1: cutoff = K-1.
//  7. S = cum_cutoff; draw j = first j <= cutoff with cum_j > u*S (else cutoff).
//     token = L[j], prob = (float)(p_j / S).
// Return value: 0 ok, 1 non-finite input (NaN or +inf on an allowed id, no
// finite allowed logit, or non-finite T).
struct orc_spec_out {
  int32_t token;
  float prob;
  int32_t K;         // size of the top-k list
  int32_t cutoff;    // index into the ordered list of the last kept entry
  double draw_margin;  // min |cum - uS| / S over the cumsums bracketing the draw
  double cut_margin;   // min |cum - top_p| over the cumsums bracketing the cutoff
  double Z;
  float max_x;       // m (after penalties)
  int32_t cut_id;    // id of the last kept entry (ids[cutoff])
};

int orc_spec_sample_row(const float* x_in, int V, const int32_t* hist, int hlen,
                        const uint32_t* mask_row, const orc_row_params* prm, float u,
                        orc_spec_out* out, int32_t* out_list_ids, float* out_list_p,
                        int list_cap) {
  std::vector<float> x(x_in, x_in + V);
  // 1. penalties
  if (hlen > 0) {
    std::vector<int32_t> h;
    h.reserve(hlen);
    for (int j = 0; j < hlen; ++j)
      if (hist[j] >= 0 && hist[j] < V) h.push_back(hist[j]);
    std::sort(h.begin(), h.end());
    for (size_t j = 0; j < h.size();) {
      size_t k = j;
      while (k < h.size() && h[k] == h[j]) ++k;
      int id = h[j];
      int c = static_cast<int>(k - j);
      float v = x[id];
      float x1 = (v < 0.0f) ? v * prm->repeat_penalty : v / prm->repeat_penalty;
      float cf = static_cast<float>(c) * prm->frequency_penalty;
      float x2 = x1 - cf;
      float x3 = x2 - prm->presence_penalty;
      x[id] = x3;
      j = k;
    }
  }
  // 2. mask
  std::vector<uint8_t> allowed(V, 1);
  int n_allowed = V;
  if (mask_row) {
    int cnt = 0;
    for (int i = 0; i < V; ++i) cnt += mask_bit(mask_row, i);
    if (cnt > 0) {
      for (int i = 0; i < V; ++i) allowed[i] = mask_bit(mask_row, i);
      n_allowed = cnt;
    }
  }
  out->draw_margin = INFINITY;
  out->cut_margin = INFINITY;
  // validity; a -inf logit (after penalties) has zero probability and is
  // excluded from the list like a masked id
  float m = -INFINITY;
  int argmax = -1;
  for (int i = 0; i < V; ++i) {
    if (!allowed[i]) continue;
    if (std::isnan(x[i]) || x[i] == INFINITY) return 1;
    if (x[i] == -INFINITY) {
      allowed[i] = 0;
      --n_allowed;
      continue;
    }
    if (argmax < 0 || x[i] > m) {
      m = x[i];
      argmax = i;
    }
  }
  if (n_allowed == 0) return 1;
  out->max_x = m;
  const float T = prm->temperature;
  if (!std::isfinite(T)) return 1;
  // 3. greedy
  if (T <= 0.0f) {
    out->token = argmax;
    out->prob = 1.0f;
    out->K = 1;
    out->cutoff = 0;
    out->cut_id = argmax;
    out->Z = 1.0;
    if (out_list_ids && list_cap > 0) {
      out_list_ids[0] = argmax;
      if (out_list_p) out_list_p[0] = 1.0f;
    }
    return 0;
  }
  // 4. softmax
  std::vector<float> e(V, 0.0f);
  double Z = 0.0;
  for (int i = 0; i < V; ++i) {
    if (!allowed[i]) continue;
    float d = x[i] - m;
    float l = d / T;
    e[i] = std::exp(l);
    Z += static_cast<double>(e[i]);
  }
  out->Z = Z;
  // 5. ordered list
  std::vector<int32_t> ids;
  ids.reserve(n_allowed);
  for (int i = 0; i < V; ++i)
    if (allowed[i]) ids.push_back(i);
  int K = (prm->top_k > 0) ? std::min(prm->top_k, n_allowed) : n_allowed;
  auto cmp = [&](int32_t a, int32_t b) {
    if (x[a] != x[b]) return x[a] > x[b];
    return a < b;
  };
  if (K < n_allowed) {
    std::partial_sort(ids.begin(), ids.begin() + K, ids.end(), cmp);
  } else {
    std::sort(ids.begin(), ids.end(), cmp);
  }
  ids.resize(K);
  // 6. top-p cutoff
  std::vector<double> cum(K);
  double c = 0.0;
  for (int j = 0; j < K; ++j) {
    c += static_cast<double>(e[ids[j]]) / Z;
    cum[j] = c;
  }
  int cutoff = K - 1;
  if (prm->top_p < 1.0f) {
    const double tp = static_cast<double>(prm->top_p);
    int cpos = K;
    for (int j = 0; j < K; ++j)
      if (cum[j] >= tp) {
        cpos = j;
        break;
      }
    cutoff = std::min(cpos, K - 1);
    double mg = std::fabs(cum[cutoff] - tp);
    if (cutoff > 0) mg = std::min(mg, std::fabs(cum[cutoff - 1] - tp));
    out->cut_margin = mg;
  }
  // 7. draw
  const double S = cum[cutoff];
  const double target = static_cast<double>(u) * S;
  int j = cutoff;
  for (int t = 0; t <= cutoff; ++t)
    if (cum[t] > target) {
      j = t;
      break;
    }
  double dm = std::fabs(cum[j] - target);
  if (j > 0) dm = std::min(dm, std::fabs(target - cum[j - 1]));
  out->draw_margin = dm / S;
  out->token = ids[j];
  out->prob = static_cast<float>((static_cast<double>(e[ids[j]]) / Z) / S);
  out->K = K;
  out->cutoff = cutoff;
  out->cut_id = ids[cutoff];
  if (out_list_ids) {
    for (int t = 0; t < K && t < list_cap; ++t) {
      out_list_ids[t] = ids[t];
      if (out_list_p) out_list_p[t] = static_cast<float>(static_cast<double>(e[ids[t]]) / Z);
    }
  }
  return 0;
}

// Batched spec sampling over B rows with an optional thread pool (CPU baseline).
// dtype 0 = f32 logits, 1 = bf16 logits (row stride ld elements).
// hist: B x hist_stride int32, hist_len[B]; mask: B x mask_stride uint32 or null.
// Returns the number of rows whose status was non-zero.
int orc_spec_sample_batch(const void* logits, int dtype, int B, int V, int64_t ld,
                          const int32_t* hist, const int32_t* hist_len, int hist_stride,
                          const uint32_t* mask, int64_t mask_stride,
                          const orc_row_params* params, const float* uniforms,
                          int32_t* out_tok, float* out_prob, int nthreads) {
  if (nthreads < 1) nthreads = 1;
  std::vector<int> bad(nthreads, 0);
  auto work = [&](int t) {
    std::vector<float> row;
    for (int b = t; b < B; b += nthreads) {
      const float* xr;
      if (dtype == 1) {
        row.resize(V);
        const uint16_t* src = static_cast<const uint16_t*>(logits) + ld * b;
        for (int i = 0; i < V; ++i) row[i] = bf16_to_f32(src[i]);
        xr = row.data();
      } else {
        xr = static_cast<const float*>(logits) + ld * b;
      }
      orc_spec_out o{};
      int st = orc_spec_sample_row(xr, V, hist ? hist + (int64_t)hist_stride * b : nullptr,
                                   hist_len ? hist_len[b] : 0,
                                   mask ? mask + mask_stride * b : nullptr, &params[b],
                                   uniforms[b], &o, nullptr, nullptr, 0);
      if (st) {
        bad[t]++;
        out_tok[b] = -1;
        if (out_prob) out_prob[b] = 0.0f;
      } else {
        out_tok[b] = o.token;
        if (out_prob) out_prob[b] = o.prob;
      }
    }
  };
  if (nthreads == 1) {
    work(0);
  } else {
    std::vector<std::thread> th;
    for (int t = 0; t < nthreads; ++t) th.emplace_back(work, t);
    for (auto& x : th) x.join();
  }
  int nb = 0;
  for (int v : bad) nb += v;
  return nb;
}

// Batched ref_exact sampling (Decoder::sample_with_params per row).
void orc_decoder_sample_batch(const float* logits, int B, int V, int64_t ld,
                              const float* temperature, const float* top_p,
                              const float* uniforms, int32_t* out_tok, float* out_prob,
                              int nthreads) {
  if (nthreads < 1) nthreads = 1;
  auto work = [&](int t) {
    for (int b = t; b < B; b += nthreads)
      out_tok[b] = orc_decoder_sample(logits + ld * b, V, temperature[b], top_p[b], uniforms[b],
                                      out_prob ? out_prob + b : nullptr, nullptr, nullptr,
                                      nullptr);
  };
  if (nthreads == 1) {
    work(0);
  } else {
    std::vector<std::thread> th;
    for (int t = 0; t < nthreads; ++t) th.emplace_back(work, t);
    for (auto& x : th) x.join();
  }
}

// ---------------------------------------------------------------------------
// Beam step (BeamSearch::search inner loop, src/decoder.rs:227-270)
// ---------------------------------------------------------------------------
// items x beams hypotheses; logits row (item*beams + b) with stride ld.
// scores[item*beams+b] cumulative score; done[...] completion flag;
// lens[...] current token count of the hypothesis.
// log_softmax = 0: ref_exact (raw logits, decoder.rs:236-256);
// log_softmax = 1: spec (x - lse, lse = m + log(sum exp(x - m))).
// For each item the candidates are: a completed beam carries itself over
// (decoder.rs:231-234, token -1); a live beam contributes its top 2*beams ids
// by (value desc, id asc) with score (s + v) / lp(len + 1) (decoder.rs:249-255,
// lp = 1 if alpha == 1 else ((len+6)/6)^alpha, decoder.rs:278-284) and done
// = (id == eos). All candidates are stable-sorted by score descending
// (decoder.rs:260-264): ties keep push order, i.e. beam ascending, then value
// descending, then id ascending. The first n_out are written per item.
void orc_beam_step(const float* logits, int items, int beams, int V, int64_t ld,
                   const float* scores, const uint8_t* done, const int32_t* lens,
                   float alpha, int eos, int log_softmax, int n_out, int32_t* out_beam,
                   int32_t* out_tok, float* out_score, uint8_t* out_done) {
  struct Cand {
    float score;
    int32_t beam;
    int32_t tok;
    uint8_t done;
  };
  const int topk = 2 * beams;
  std::vector<int32_t> ids(V);
  for (int it = 0; it < items; ++it) {
    std::vector<Cand> all;
    for (int b = 0; b < beams; ++b) {
      const int row = it * beams + b;
      if (done[row]) {
        all.push_back({scores[row], b, -1, 1});
        continue;
      }
      const float* x = logits + ld * row;
      float lse = 0.0f;
      if (log_softmax) {
        float m = -INFINITY;
        for (int i = 0; i < V; ++i) m = std::max(m, x[i]);
        double Z = 0.0;
        for (int i = 0; i < V; ++i) Z += static_cast<double>(std::exp(x[i] - m));
        lse = static_cast<float>(static_cast<double>(m) + std::log(Z));
      }
      for (int i = 0; i < V; ++i) ids[i] = i;
      const int k = std::min(topk, V);
      std::partial_sort(ids.begin(), ids.begin() + k, ids.end(), [&](int32_t a, int32_t c) {
        if (x[a] != x[c]) return x[a] > x[c];
        return a < c;
      });
      float lp = 1.0f;
      if (alpha != 1.0f) {
        float len = static_cast<float>(lens[row] + 1);
        lp = std::pow((len + 6.0f) / 6.0f, alpha);
      }
      for (int j = 0; j < k; ++j) {
        const int32_t id = ids[j];
        const float v = log_softmax ? (x[id] - lse) : x[id];
        const float ns = scores[row] + v;
        all.push_back({ns / lp, b, id, static_cast<uint8_t>(id == eos)});
      }
    }
    std::stable_sort(all.begin(), all.end(),
                     [](const Cand& a, const Cand& c) { return a.score > c.score; });
    for (int j = 0; j < n_out; ++j) {
      const int o = it * n_out + j;
      if (j < static_cast<int>(all.size())) {
        out_beam[o] = all[j].beam;
        out_tok[o] = all[j].tok;
        out_score[o] = all[j].score;
        out_done[o] = all[j].done;
      } else {
        out_beam[o] = -1;
        out_tok[o] = -1;
        out_score[o] = -INFINITY;
        out_done[o] = 0;
      }
    }
  }
}

// ---------------------------------------------------------------------------
// SpeculativeDecoder (src/inference.rs:238-438), with rand_simple()
// (src/inference.rs:432-438) replaced by injected uniforms.
// ---------------------------------------------------------------------------

// SpeculativeDecoder::sample (src/inference.rs:376-414): ids below `offset`
// are skipped (.skip(offset)); the token id includes the offset.
int32_t orc_specdec_sample(const float* logits, int V, float temperature, int offset, float r) {
  if (offset < 0) return -1;  // a usize in the reference
  if (temperature <= 0.0f) {  // :379-387 argmax, max_by: the LAST maximum
    int best = -1;
    float bv = 0.0f;
    for (int i = offset; i < V; ++i) {
      if (logits[i] != logits[i]) return -1;  // partial_cmp(..).unwrap() panics on NaN
      if (best < 0 || !(logits[i] < bv)) {
        best = i;
        bv = logits[i];
      }
    }
    return best < 0 ? 0 : best;  // unwrap_or(0)
  }
  std::vector<float> adjusted;  // :389-395 v / temperature
  for (int i = offset; i < V; ++i) adjusted.push_back(logits[i] / temperature);
  float max_val = -FLT_MAX;  // :397 fold(f32::MIN, max)
  for (float v : adjusted) max_val = rust_max(max_val, v);
  for (float& v : adjusted) v = std::exp(v - max_val);  // :398
  float sum = 0.0f;  // :400 sequential f32 sum
  for (float v : adjusted) sum += v;
  if (sum > 0.0f)
    for (float& v : adjusted) v /= sum;
  float cumsum = 0.0f;  // :405-411 id-order draw, r <= cumsum
  for (size_t i = 0; i < adjusted.size(); ++i) {
    cumsum += adjusted[i];
    if (r <= cumsum) return static_cast<int32_t>(i) + offset;
  }
  return V - 1;  // :413
}

// SpeculativeDecoder::softmax_at (src/inference.rs:416-429).
float orc_specdec_softmax_at(const float* logits, int V, int64_t idx) {
  if (idx < 0 || idx >= V) return 0.0f;  // a negative Token cast to usize is out of range
  float max_logit = -FLT_MAX;
  for (int i = 0; i < V; ++i) max_logit = rust_max(max_logit, logits[i]);
  float exp_sum = 0.0f;
  for (int i = 0; i < V; ++i) exp_sum += std::exp(logits[i] - max_logit);
  return exp_sum > 0.0f ? std::exp(logits[idx] - max_logit) / exp_sum : 0.0f;
}

// SpeculativeDecoder::verify_and_accept (src/inference.rs:335-374) for one
// request: returns the accepted count; *out_token is the token the caller
// appends after the accepted drafts (the bonus token when every draft is
// accepted and room > 0, the fallback sample of generate (:293-300) when
// none is), or -1. draw_u is the uniform of that one draw.
int32_t orc_specdec_verify(const float* logits, int V, const int32_t* drafts, int D, const float* accept_u,
                           int room, float draw_u, int32_t* out_token) {
  int accepted = 0;
  for (int i = 0; i < D; ++i) {
    const float draft_prob = orc_specdec_softmax_at(logits, V, drafts[i]);
    const float target_prob = orc_specdec_softmax_at(logits, V, drafts[i]);
    const float acceptance = draft_prob > 0.0f ? std::fmin(target_prob / draft_prob, 1.0f) : 0.0f;
    if (accept_u[i] < acceptance) {
      accepted = i + 1;
    } else {
      break;
    }
  }
  int32_t tok = -1;
  if (accepted == D && room > 0) {  // :363-369 the bonus token
    const int32_t bonus = orc_specdec_sample(logits, V, 1.0f, D, draw_u);
    if (bonus > 0 && bonus != (D > 0 ? drafts[D - 1] : 0)) tok = bonus;
  } else if (accepted == 0) {  // generate :293-300 the fallback token
    const int32_t t = orc_specdec_sample(logits, V, 1.0f, D, draw_u);
    if (t > 0) tok = t;
  }
  *out_token = tok;
  return accepted;
}

}  // extern "C"
