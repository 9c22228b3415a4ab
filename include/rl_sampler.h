/*
 * rl_sampler.h -- C ABI of the B200 (sm_100a) logits -> token sampler.
 *
 * Drop-in device backend for the sampling path of chenyusolar/rust-llm
 * (src/decoder.rs). Plain pointers and sizes only; every entry point returns
 * an rl_status and never aborts, throws or traps (the reference's release
 * profile is panic = "abort", Cargo.toml:40-43, so errors must come back as
 * values). The last error message of the calling thread is rl_last_error().
 *
 * Device pointers: every logits / history / mask / params / uniforms / output
 * pointer passed to an entry point without a _host suffix is a device pointer
 * on the handle's device. Work is enqueued on `stream` (a cudaStream_t passed
 * as void*, NULL = legacy default stream) and is asynchronous unless stated.
 *
 * Layouts:
 *  - logits: row-major [B, V] with row stride `ld` elements (ld >= V).
 *  - history: row-major [B, hist_stride] int32 token ids; hist_len[b] of them
 *    are valid. Ids outside [0, V) are ignored.
 *  - mask: row-major [B, mask_stride] uint32 words; bit (i & 31) of word
 *    (i >> 5) set <=> token id i is allowed (LSB first). A row with no bit set
 *    allows every id (src/decoder.rs:362-364).
 *  - uniforms: one float in [0, 1) per row; it replaces rand_secure()
 *    (src/decoder.rs:170-188), which cannot be seeded.
 */
#ifndef RL_SAMPLER_H
#define RL_SAMPLER_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef enum {
  RL_OK = 0,
  RL_ERR_INVALID_ARG = 1, /* null pointer, bad enum, negative size           */
  RL_ERR_SHAPE = 2,       /* size beyond the handle's limits or the kernel's */
  RL_ERR_OOM = 3,         /* device allocation failed (create only)          */
  RL_ERR_CUDA = 4,        /* a CUDA runtime call failed                      */
  RL_ERR_NCCL = 5,        /* an NCCL call failed (sharded sampling)          */
  RL_ERR_TIMEOUT = 6,     /* a bounded device-side wait expired              */
  RL_ERR_UNSUPPORTED = 7, /* feature not built into this library             */
  RL_ERR_NONFINITE = 8    /* a row's inputs were not finite (see row_status) */
} rl_status;

typedef enum { RL_F32 = 0, RL_BF16 = 1 } rl_dtype;

/* Per-row sampling parameters (24 bytes). SamplingParams, src/decoder.rs:294-316,
 * plus presence/frequency penalties (absent from the reference). */
typedef struct {
  float temperature;       /* <= 0: greedy (argmax, lowest id on ties)        */
  float top_p;             /* >= 1: no nucleus cut                            */
  int32_t top_k;           /* <= 0: off (k = number of allowed ids)           */
  float repeat_penalty;    /* history ids: x<0 ? x*rp : x/rp (decoder.rs:102) */
  float presence_penalty;  /* history ids: x -= pres                          */
  float frequency_penalty; /* history ids: x -= count*freq                    */
} rl_row_params;

typedef struct rl_sampler rl_sampler;

/* Creates a sampler on `device`. The handle owns a small device workspace
 * sized by the limits (allocated here, never in a sampling call).
 * Replaces the per-call construction of Decoder / Sampler
 * (src/decoder.rs:19-29, :325-331). flags: 0, or RL_CREATE_SHARDED to also
 * allocate the exchange buffers of rl_sample_sharded (1056 B per row for this
 * rank and 16 x that for the gathered records). */
#define RL_CREATE_SHARDED 1u
rl_status rl_sampler_create(rl_sampler** out, int device, int max_batch, int max_vocab,
                            int max_history, uint32_t flags);
rl_status rl_sampler_destroy(rl_sampler* h);

/* Thread-local message of the last failing call on this thread ("" if none). */
const char* rl_last_error(void);

/* Library version string. */
const char* rl_version(void);

/*
 * Debug switches of a handle (diagnostics; flags = 0 turns them off). No
 * counterpart in the reference: they exercise this library's failure path.
 * RL_DEBUG_EXPIRE_WAIT: every item of the spec sampler's streaming kernel
 * first waits, with a budget of about two thousand cycles, on a device
 * barrier that nothing completes; the wait runs out and every row of the call
 * reports RL_ERR_TIMEOUT in row_status (token -1), as a device wait that ran
 * out of its budget would, without a fault or a hang. Later calls with the
 * switch off sample normally on the same handle.
 */
#define RL_DEBUG_EXPIRE_WAIT 1u
/* RL_DEBUG_TIMING: each spec sampling call (rl_sample_batch and the entries
 * built on it) records CUDA events around each of its kernels on the call's
 * stream; rl_sampler_kernel_times returns the last call's per-kernel device
 * times in launch order: for rows of more than 45056 logits the streaming
 * kernel, then the finish kernel; for shorter rows without a mask the one
 * short-row kernel.
 * The events between the two kernels keep the finish kernel from starting
 * early, so a timed step can run a little longer than an untimed one. */
#define RL_DEBUG_TIMING 2u
rl_status rl_sampler_set_debug(rl_sampler* h, uint32_t flags);
/* Waits for the last timed call and writes up to cap kernel times (ms) to
 * ms[]; *n gets their count (0 when no call was timed). */
rl_status rl_sampler_kernel_times(rl_sampler* h, float* ms, int cap, int* n);

/*
 * Self-check of the fixed-divisor division that the spec sampler uses for
 * every logit / temperature (no counterpart in the reference). For each T[j]
 * (device array, nT <= 65535) counts the a[i] (device array) whose quotient
 * differs in any bit from IEEE division (__fdiv_rn) into mismatch[j], and sets
 * fast[j] = 1 when the fixed-divisor path is in use for T[j] (device arrays
 * [nT]). Asynchronous on `stream`.
 */
rl_status rl_selfcheck_div(const float* a, int n, const float* T, int nT, uint32_t* mismatch, uint32_t* fast,
                           void* stream);

/*
 * Batched spec sampling: penalties -> mask -> temperature -> softmax ->
 * top-k -> top-p -> draw, one token per row.
 * Replaces the serial per-sequence loop of ContinuousBatchingEngine::step
 * (src/inference.rs:112-138) calling Model::sample_with_params
 * (src/model.rs:484-486 -> src/decoder.rs:35-100), extended with the
 * reference's top_k_logits / sample_top_p / sample_multinomial helpers
 * (src/decoder.rs:112-158) and history penalties.
 *  out_tok[B]   sampled ids (device)
 *  out_prob[B]  probability of the sampled id after the top-p renormalisation
 *               (device, nullable)
 *  row_status[B] per-row status, 0 ok / RL_ERR_NONFINITE (device, nullable)
 */
rl_status rl_sample_batch(rl_sampler* h, const void* logits, rl_dtype dtype, int B, int V,
                          int64_t ld, const int32_t* hist, const int32_t* hist_len,
                          int hist_stride, const uint32_t* mask, int64_t mask_stride,
                          const rl_row_params* params, const float* uniforms, int32_t* out_tok,
                          float* out_prob, int32_t* row_status, void* stream);

/*
 * Same as rl_sample_batch, and also writes, for inspection, what the
 * reference's top_k_logits / sample_top_p (src/decoder.rs:112-144) would
 * hold for each row, in (logit desc, id asc) order:
 *  list_ids / list_probs [B, list_cap]: the top-k list (ids, full-vocabulary
 *      probabilities); list_len[B] = min(K, list_cap) when the kernel holds
 *      the whole list (K <= 128), else -1. K = top_k, or the allowed count
 *      when top_k is off.
 *  out_cut [B, 3] (nullable): K; the position in that order of the last
 *      entry the top-k / top-p cutoff keeps; that entry's id (-2 when the
 *      kernel does not resolve it: rows without a cutoff whose list is
 *      longer than the kernel materialises). Together they fix the kept set
 *      (every key at or above the last kept one). Debug launches also count
 *      logits per histogram bin, so they run slower than rl_sample_batch.
 */
rl_status rl_sample_batch_debug(rl_sampler* h, const void* logits, rl_dtype dtype, int B,
                                int V, int64_t ld, const int32_t* hist, const int32_t* hist_len,
                                int hist_stride, const uint32_t* mask, int64_t mask_stride,
                                const rl_row_params* params, const float* uniforms,
                                int32_t* out_tok, float* out_prob, int32_t* row_status,
                                int32_t* list_ids, float* list_probs, int32_t* list_len,
                                int list_cap, int32_t* out_cut, void* stream);

/*
 * Host-buffer convenience wrapper of rl_sample_batch (f32 logits): copies the
 * inputs to the handle's device staging buffers, samples, copies the outputs
 * back and synchronises. Backs the &[f32] Rust signatures
 * (Decoder::sample_with_params, src/decoder.rs:35). hist/hist_len/mask/out_prob
 * may be NULL.
 */
rl_status rl_sample_host(rl_sampler* h, const float* logits, int B, int V, const int32_t* hist,
                         const int32_t* hist_len, int hist_stride, const uint32_t* mask,
                         int64_t mask_stride, const rl_row_params* params, const float* uniforms,
                         int32_t* out_tok, float* out_prob);

/*
 * rl_sample_batch without a handle and without any allocation. No
 * counterpart in the reference: it serves callers that cannot allocate where
 * they sample (inside CUDA-graph capture, allocator-free decode loops, FFI
 * callers with no place to keep a handle). Same arguments and results as
 * rl_sample_batch, on the current device; every buffer must be device memory
 * of that device (else RL_ERR_INVALID_ARG). Its scratch is a fixed device
 * array of the library (9.7 MB, the candidate overflow of at most 296 CTAs);
 * sizes beyond V <= 2093056, hist_stride <= 1024, B <= 65535 return
 * RL_ERR_SHAPE. The first call on a device reads the SM count and configures
 * the kernels of both dtypes (no allocation); it must come before any stream
 * capture (inside one it returns RL_ERR_UNSUPPORTED). The scratch's device
 * address is looked up on every call made outside a capture, so a reset
 * device (cudaDeviceReset, which reloads the module) is picked up there;
 * calls inside a capture reuse the last address, so capture after a reset
 * only once an uncaptured call has run. Nothing in the scratch must start at
 * zero. Calls that overlap in time on one device share the scratch and race:
 * serialise them.
 */
rl_status rl_sample_batch_static(const void* logits, rl_dtype dtype, int B, int V, int64_t ld,
                                 const int32_t* hist, const int32_t* hist_len, int hist_stride,
                                 const uint32_t* mask, int64_t mask_stride,
                                 const rl_row_params* params, const float* uniforms,
                                 int32_t* out_tok, float* out_prob, int32_t* row_status,
                                 void* stream);

/*
 * ref_exact profile: Decoder::sample_with_params (src/decoder.rs:35-100)
 * reproduced quirk for quirk, per row: temperature softmax; if top_p < 1 a
 * stable descending sort, cumsum >= top_p cutoff, zeroing of ORIGINAL ids
 * greater than the cutoff position (decoder.rs:71-75), renormalisation; then
 * the id-order draw r <= cumsum and the last-max argmax fallback.
 * Decoder::sample (decoder.rs:31-33) is temperature = 1, top_p = 0.9.
 *  temperature[B], top_p[B], uniforms[B]: device arrays.
 *  out_prob[B]: the returned id's entry of the final probability array (nullable).
 * Every sum is the reference's left-to-right f32 accumulation, reproduced bit
 * for bit; exp is the correctly rounded f32 exponential. A row holding NaN or
 * +-inf gets token -1 and probability 0 (the reference's result there depends
 * on NaN ordering). B <= max_batch, V <= max_vocab. A row is worked on in one
 * CTA's shared memory when it fits (V <= 53248 on a B200), else in the
 * handle's staging buffer (which rl_sample_host and rl_decoder_sample_host
 * also use: one call at a time per handle).
 */
rl_status rl_decoder_sample(rl_sampler* h, const float* logits, int B, int V, int64_t ld,
                            const float* temperature, const float* top_p, const float* uniforms,
                            int32_t* out_tok, float* out_prob, void* stream);

/*
 * rl_decoder_sample on host buffers (synchronous): logits [B, V] row-major
 * f32, temperature[B], top_p[B], uniforms[B] in host memory; out_tok[B] and
 * out_prob[B] (nullable) written in host memory. Backs the &[f32] Rust
 * signatures of Decoder::sample / Decoder::sample_with_params
 * (src/decoder.rs:31-100) with the reference's own semantics.
 */
rl_status rl_decoder_sample_host(rl_sampler* h, const float* logits, int B, int V, const float* temperature,
                                 const float* top_p, const float* uniforms, int32_t* out_tok, float* out_prob);

/* Decoder::greedy_sample (src/decoder.rs:160-167): argmax, LAST maximum on ties. */
rl_status rl_greedy(rl_sampler* h, const float* logits, int B, int V, int64_t ld,
                    int32_t* out_tok, void* stream);

/* Sampler::sample_with_grammar (src/decoder.rs:359-376): argmax over the
 * allowed ids of the bit-packed mask, LOWEST allowed id on ties; an all-zero
 * mask row allows every id. */
rl_status rl_grammar_greedy(rl_sampler* h, const float* logits, int B, int V, int64_t ld,
                            const uint32_t* mask, int64_t mask_stride, int32_t* out_tok,
                            void* stream);

/* rl_greedy and rl_grammar_greedy on host buffers (synchronous): logits
 * [B, V] row-major f32 and mask [B, mask_stride] u32 in host memory, out_tok[B]
 * written in host memory. They back the &[f32] signatures of
 * Sampler::sample_with_grammar (src/decoder.rs:359-376) and the error
 * fallback of the infallible (-> Token) wrappers. B <= max_batch and
 * V <= max_vocab of the handle. */
rl_status rl_greedy_host(rl_sampler* h, const float* logits, int B, int V, int32_t* out_tok);
rl_status rl_grammar_greedy_host(rl_sampler* h, const float* logits, int B, int V, const uint32_t* mask,
                                 int64_t mask_stride, int32_t* out_tok);

/*
 * Speculative decoding (SpeculativeDecoder, src/inference.rs:238-438): its
 * sampling arithmetic on device buffers, bit-exact with the reference for the
 * same uniforms (the reference draws them with rand_simple(), :432-438). One
 * CTA per row; logits [B, V] f32 at row stride ld.
 *
 * rl_specdec_sample -- SpeculativeDecoder::sample (:376-414) per row:
 * temperature[b] <= 0 takes the argmax of the ids >= offset[b] (the LAST
 * maximum; 0 when offset >= V); otherwise v / T, max from f32::MIN,
 * exp(v - max), a left-to-right f32 sum divided out when > 0, and the id-order
 * draw with uniforms[b] (first id with r <= cumsum, else V - 1). Token ids
 * include the offset. The draft model's draws are (T 0.8, offset 1), the
 * target's (T 1.0, offset = the number of drafts).
 *
 * rl_specdec_verify -- SpeculativeDecoder::verify_and_accept (:335-374) per
 * request b: drafts[b, 0 .. n_draft[b]) (row stride draft_stride, 1 <=
 * n_draft[b] <= draft_stride) against the target row. out_accepted[b] = the
 * number of leading drafts whose softmax_at probability (:416-429) p > 0 has
 * accept_u[b, i] < min(p / p, 1) (accept_u at row stride draft_stride). Then
 * one draw of sample(target, 1.0, n_draft) with draw_u[b]: when every draft
 * was accepted and room[b] > 0 (generated.len() < max_tokens) it is the bonus
 * token, kept when > 0 and not the last draft; when none was accepted it is
 * generate's fallback token (:293-300), kept when > 0. out_tok[b] = the kept
 * token, else -1.
 *
 * Deviation: a row holding NaN or +inf gives out_tok -1 (and out_accepted -1);
 * the reference panics or walks NaN sums there. n_draft outside [1,
 * draft_stride] gives -1 / -1 (the reference never verifies an empty draft).
 */
rl_status rl_specdec_sample(rl_sampler* h, const float* logits, int B, int V, int64_t ld, const float* temperature,
                            const int32_t* offset, const float* uniforms, int32_t* out_tok, void* stream);
rl_status rl_specdec_verify(rl_sampler* h, const float* logits, int B, int V, int64_t ld, const int32_t* drafts,
                            int draft_stride, const int32_t* n_draft, const float* accept_u, const int32_t* room,
                            const float* draw_u, int32_t* out_accepted, int32_t* out_tok, void* stream);

/*
 * Grammar-constrained decoding with a real GBNF grammar: the step after the
 * reference's toy Grammar (src/decoder.rs:378-557), whose get_allowed_tokens
 * (:466-529) matches single tokens against rule variants. A grammar in GBNF
 * notation ("literal", [class], [^class], ., rule names, ( ... ), * + ?
 * {m,n}; '#' comments; \xHH \uHHHH \UHHHHHHHH escapes; classes and '.' are
 * over Unicode characters) is compiled against the vocabulary (each token's
 * text as UTF-8 bytes; a character may span tokens) into a stack automaton
 * over bytes and a byte trie of the tokens. Per
 * sequence a state; per step rl_gbnf_mask writes the bit-packed allowed row
 * that rl_sample_batch (mask argument) and rl_grammar_greedy take, and
 * rl_gbnf_accept advances the state by the sampled token. Host functions:
 * no device work, no handle; a grammar is read-only after create and may be
 * shared between threads, a state belongs to one thread at a time.
 *
 * rl_gbnf_create: text (NUL-terminated), the start rule's name, V tokens
 *   (tokens[t], token_len[t] bytes; a token of length 0 never matches) and the
 *   end-of-sequence id (-1: none), which is allowed exactly when the start rule
 *   is complete. RL_ERR_INVALID_ARG on a syntax error or an undefined rule,
 *   RL_ERR_UNSUPPORTED on left recursion (the message names the rule).
 * rl_gbnf_mask: row[words >= ceil(V/32)] := the allowed tokens; *n_allowed
 *   (nullable) their count. A row of zeros means none (after the end token);
 *   the samplers read an all-zero row as "every id", so stop such a sequence.
 * rl_gbnf_mask_batch: the same for B states into mask[B, mask_stride], rows
 *   spread over nthreads host threads.
 * rl_gbnf_accept: advances the state by one token; RL_ERR_INVALID_ARG (state
 *   unchanged) if the grammar does not allow it.
 * States grow with the grammar's ambiguity; beyond 4096 stacks or 1024 frames
 * a call returns RL_ERR_SHAPE.
 */
typedef struct rl_gbnf rl_gbnf;
typedef struct rl_gbnf_state rl_gbnf_state;
rl_status rl_gbnf_create(const char* text, const char* root, int V, const char* const* tokens,
                         const int32_t* token_len, int32_t eos_id, rl_gbnf** out);
void rl_gbnf_destroy(rl_gbnf* g);
rl_status rl_gbnf_state_create(const rl_gbnf* g, rl_gbnf_state** out);
void rl_gbnf_state_destroy(rl_gbnf_state* s);
rl_status rl_gbnf_state_copy(const rl_gbnf_state* src, rl_gbnf_state* dst);
int rl_gbnf_accepting(const rl_gbnf_state* s);
rl_status rl_gbnf_accept(const rl_gbnf* g, rl_gbnf_state* s, int32_t token);
rl_status rl_gbnf_mask(const rl_gbnf* g, const rl_gbnf_state* s, uint32_t* mask_row, int64_t words,
                       int32_t* n_allowed);
/* rl_gbnf_accept for B states and their tokens, rows spread over host
 * threads; row_status[B] (nullable) gets each row's status (a refused row's
 * state is unchanged); the call returns the first failing row's status. */
rl_status rl_gbnf_accept_batch(const rl_gbnf* g, rl_gbnf_state* const* states, const int32_t* tokens, int B,
                               int32_t* row_status, int nthreads);
rl_status rl_gbnf_mask_batch(const rl_gbnf* g, const rl_gbnf_state* const* states, int B, uint32_t* mask,
                             int64_t mask_stride, int32_t* n_allowed, int nthreads);

/*
 * LM head feeding the sampler (src/model.rs:236-262: the final projection of
 * Model::forward, matmul_vec's logits[i] = sum_j hidden[j] * W[i * H + j]),
 * batched, on the tensor cores: logits[b, v] = sum_h hidden[b, h] * W[v, h].
 * hidden [B, ldh] and weight [V, ldw] are bf16 (raw uint16 bits), K-major,
 * 16-byte aligned, ldh and ldw multiples of 8; H a multiple of 64; the sums
 * are f32 (products of bf16 values are exact in f32; the order of the
 * additions is the tensor cores', not the reference's left-to-right loop).
 * Any B (rows beyond 256 run as further launches that stream the weight
 * again); B <= max_batch of the handle.
 *
 * rl_lmhead_logits: the logits into out_logits [B, ldo] (RL_F32 or RL_BF16,
 *   rounded to nearest even).
 * rl_lmhead_greedy: Decoder::greedy_sample (src/decoder.rs:160-167) of those
 *   logits, LAST maximum on ties, fused into the GEMM's epilogue: out_tok[B]
 *   and row_status[B] (nullable; RL_ERR_TIMEOUT with token -1 when a device
 *   wait ran out). out_logits (f32, nullable) also receives the logits; when
 *   it is NULL the logits are never written to memory.
 * rl_lmhead_sample: the logits (f32) into the handle's staging buffer, then
 *   rl_sample_batch on them (no mask); V <= max_vocab of the handle.
 */
rl_status rl_lmhead_logits(rl_sampler* h, const uint16_t* hidden, int64_t ldh, const uint16_t* weight, int64_t ldw,
                           int B, int H, int V, void* out_logits, rl_dtype out_dtype, int64_t ldo, void* stream);
rl_status rl_lmhead_greedy(rl_sampler* h, const uint16_t* hidden, int64_t ldh, const uint16_t* weight, int64_t ldw,
                           int B, int H, int V, int32_t* out_tok, int32_t* row_status, float* out_logits, int64_t ldo,
                           void* stream);
rl_status rl_lmhead_sample(rl_sampler* h, const uint16_t* hidden, int64_t ldh, const uint16_t* weight, int64_t ldw,
                           int B, int H, int V, const int32_t* hist, const int32_t* hist_len, int hist_stride,
                           const rl_row_params* params, const float* uniforms, int32_t* out_tok, float* out_prob,
                           int32_t* row_status, void* stream);

/*
 * Vocabulary-sharded sampling (a row's logits split by vocabulary across
 * devices). No single reference function: it splits the spec pipeline above
 * so that each device streams only its columns and the devices exchange 4 KB
 * per row. Per step:
 *   1. every shard g calls rl_sample_partial on its columns [off_g, off_g+V_g);
 *   2. the callers all-gather the keys and stats (e.g. NCCL) into [G, B, ...];
 *   3. rl_sample_merge draws each row's token from the G partial results.
 * The result equals rl_sample_batch on the whole row (up to the order in
 * which the softmax sums are added). Rows with temperature <= 0 take the
 * argmax; sampled rows need 1 <= top_k <= 128 (RL_ERR_UNSUPPORTED in
 * row_status otherwise).
 */
typedef struct {
  float m;        /* max over the shard's allowed finite logits (-inf if none) */
  int32_t argmax; /* lowest global id at m, -1 if none                      */
  int32_t nallow; /* allowed finite logits of the shard                      */
  int32_t flags;  /* 1: non-finite input, 2: a device wait ran out            */
  double z;       /* sum of exp((x - m) / T) over the shard                  */
  int32_t n;      /* keys in the shard's list                                */
  int32_t pad;
} rl_part_stats;  /* 32 bytes */

#define RL_PART_KEYS 128 /* keys per row of a partial list */

/*
 * One shard's partial result: penalties (history ids are global; ids outside
 * the shard are skipped), mask (bit i <-> the shard's column i), temperature
 * and the row's sorted top-min(top_k, 128) list.
 *  out_keys  [B, RL_PART_KEYS] uint64 keys, descending: bits 63..32 the
 *            penalised logit as an order-preserving uint32, bits 31..0 the
 *            bitwise NOT of the global id (equal logits: lower id first).
 *  out_stats [B] rl_part_stats.
 */
rl_status rl_sample_partial(rl_sampler* h, const void* logits, rl_dtype dtype, int B, int V,
                            int64_t ld, int vocab_offset, const int32_t* hist,
                            const int32_t* hist_len, int hist_stride, const uint32_t* mask,
                            int64_t mask_stride, const rl_row_params* params, uint64_t* out_keys,
                            rl_part_stats* out_stats, void* stream);

/*
 * Merge of G <= 16 partial results per row: keys [G, B, RL_PART_KEYS],
 * stats [G, B] (shard-major, as an all-gather lays them out). Outputs as
 * rl_sample_batch.
 */
rl_status rl_sample_merge(rl_sampler* h, int G, int B, const uint64_t* keys,
                          const rl_part_stats* stats, const rl_row_params* params,
                          const float* uniforms, int32_t* out_tok, float* out_prob,
                          int32_t* row_status, void* stream);

/*
 * Vocabulary-sharded sampling in one call per rank, with the exchange over
 * NCCL. No single reference function: it replaces sampling whole rows on one
 * thread (ContinuousBatchingEngine::step, src/inference.rs:112-138 ->
 * Model::sample_with_params) when a row's vocabulary is split across the G
 * devices of an NCCL communicator (one rank per device, G <= 16). Every rank
 * calls it with its own columns [vocab_offset, vocab_offset + V_local) of the
 * same rows, in the same order; the rank streams them (rl_sample_partial),
 * the ranks' packed records (the sorted top-min(top_k, 128) list and the
 * softmax summary, 1056 bytes per row) are all-gathered with one
 * ncclAllGather on `stream`, and every rank merges them (rl_sample_merge) into
 * the same tokens. History ids are global; mask_shard bit i is the rank's
 * column i. Rows with temperature <= 0 take the argmax; sampled rows need
 * 1 <= top_k <= 128 (RL_ERR_UNSUPPORTED in row_status otherwise).
 *  comm: an ncclComm_t (void*) of this device, e.g. from rl_nccl_comm_init.
 *  The handle needs RL_CREATE_SHARDED. NCCL errors return RL_ERR_NCCL.
 */
rl_status rl_sample_sharded(rl_sampler* h, void* comm, const void* logits, rl_dtype dtype, int B, int V_local,
                            int64_t ld, int vocab_offset, int V_global, const int32_t* hist,
                            const int32_t* hist_len, int hist_stride, const uint32_t* mask_shard,
                            int64_t mask_stride, const rl_row_params* params, const float* uniforms,
                            int32_t* out_tok, float* out_prob, int32_t* row_status, void* stream);

/*
 * NCCL communicators for rl_sample_sharded (NCCL is loaded at run time: the
 * one already in the process, else libnccl.so.2, or the file named by the
 * RL_NCCL_LIBRARY environment variable; RL_ERR_UNSUPPORTED without it).
 * Rank 0 makes an id (RL_NCCL_ID_BYTES bytes), the caller hands it to every
 * rank by its own means, and each rank creates its communicator with its
 * device current (ncclGetUniqueId / ncclCommInitRank / ncclCommDestroy).
 */
#define RL_NCCL_ID_BYTES 128
rl_status rl_nccl_unique_id(void* id_out);
rl_status rl_nccl_comm_init(void** comm_out, int nranks, const void* id, int rank);
rl_status rl_nccl_comm_destroy(void* comm);

/*
 * One beam-search step for `items` independent searches of `beams` beams
 * (BeamSearch::search, src/decoder.rs:227-270, batched over items and beams).
 *  logits      [items*beams, V] (row = item*beams + beam), stride ld
 *  beam_scores [items*beams] cumulative scores
 *  beam_done   [items*beams] 1 if the hypothesis is complete (carried over)
 *  beam_len    [items*beams] current token count (used when alpha != 1)
 * Candidates: a completed beam carries itself (token -1); a live beam offers
 * its top 2*beams ids with score (s + v) / lp(len+1), v = x - logsumexp(x)
 * when log_softmax != 0 (spec) or the raw logit x when 0 (the reference's
 * decoder.rs:249), lp = 1 if alpha == 1 else ((len+7)/6)^alpha
 * (decoder.rs:278-284); done = (id == eos). Output per item: the best n_out
 * candidates ordered by score desc, then beam asc, then logit desc, then id asc
 * (the reference's stable-sort order), n_out <= 2*beams:
 *  out_beam/out_tok/out_score/out_done [items, n_out]; an item with fewer
 *  candidates than n_out pads with beam = tok = -1, score = -inf.
 * 1 <= beams <= 16; items * beams <= max_batch; V <= max_vocab.
 */
rl_status rl_beam_step(rl_sampler* h, const float* logits, int items, int beams, int V,
                       int64_t ld, const float* beam_scores, const uint8_t* beam_done,
                       const int32_t* beam_len, float alpha, int eos, int log_softmax, int n_out,
                       int32_t* out_beam, int32_t* out_tok, float* out_score, uint8_t* out_done,
                       void* stream);

#ifdef __cplusplus
}
#endif

#endif /* RL_SAMPLER_H */
