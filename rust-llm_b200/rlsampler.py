"""ctypes front end of librl_sampler.so (include/rl_sampler.h).

Device buffers are torch tensors (torch is used only for device memory and
streams); every call goes through the C ABI. There is no fallback: if the
shared library is missing or fails to load, import of the sampler fails.
"""
from __future__ import annotations

import ctypes
import os
import re

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
LIB_PATH = os.path.join(HERE, "librl_sampler.so")
HEADER = os.path.join(ROOT, "include", "rl_sampler.h")

RL_OK = 0
RL_ERR_INVALID_ARG = 1
RL_ERR_SHAPE = 2
RL_ERR_OOM = 3
RL_ERR_CUDA = 4
RL_ERR_NCCL = 5
RL_ERR_TIMEOUT = 6
RL_ERR_UNSUPPORTED = 7
RL_ERR_NONFINITE = 8
RL_F32 = 0
RL_BF16 = 1
RL_DEBUG_EXPIRE_WAIT = 1
RL_DEBUG_TIMING = 2
RL_CREATE_SHARDED = 1
NCCL_ID_BYTES = 128  # RL_NCCL_ID_BYTES

PART_KEYS = 128  # RL_PART_KEYS
PART_REC = PART_KEYS + 4  # u64 words of a packed partial record (keys, then rl_part_stats)
PART_STATS_DTYPE = np.dtype(
    [
        ("m", np.float32),
        ("argmax", np.int32),
        ("nallow", np.int32),
        ("flags", np.int32),
        ("z", np.float64),
        ("n", np.int32),
        ("pad", np.int32),
    ]
)

STATUS_NAMES = {0: "OK", 1: "INVALID_ARG", 2: "SHAPE", 3: "OOM", 4: "CUDA", 5: "NCCL",
                6: "TIMEOUT", 7: "UNSUPPORTED", 8: "NONFINITE"}

ROW_PARAMS_DTYPE = np.dtype(
    [
        ("temperature", np.float32),
        ("top_p", np.float32),
        ("top_k", np.int32),
        ("repeat_penalty", np.float32),
        ("presence_penalty", np.float32),
        ("frequency_penalty", np.float32),
    ]
)


class RLError(RuntimeError):
    def __init__(self, status, msg):
        super().__init__(f"{STATUS_NAMES.get(status, status)}: {msg}")
        self.status = status


_lib = None


def declared_symbols():
    """Entry points declared in include/rl_sampler.h."""
    txt = open(HEADER).read()
    return sorted(set(re.findall(r"^\s*(?:rl_status|const char\*)\s+(rl_\w+)\s*\(", txt, re.M)))


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise RLError(RL_ERR_UNSUPPORTED, f"{LIB_PATH} is missing: run rust-llm_b200/build.py")
        L = ctypes.CDLL(LIB_PATH)
        P = ctypes.c_void_p
        I = ctypes.c_int
        I64 = ctypes.c_int64
        F = ctypes.c_float
        L.rl_last_error.restype = ctypes.c_char_p
        L.rl_last_error.argtypes = []
        L.rl_version.restype = ctypes.c_char_p
        L.rl_version.argtypes = []
        L.rl_sampler_create.restype = I
        L.rl_sampler_create.argtypes = [ctypes.POINTER(P), I, I, I, I, ctypes.c_uint32]
        L.rl_sampler_destroy.restype = I
        L.rl_sampler_destroy.argtypes = [P]
        L.rl_sample_batch.restype = I
        L.rl_sample_batch.argtypes = [P, P, I, I, I, I64, P, P, I, P, I64, P, P, P, P, P, P]
        L.rl_sample_batch_debug.restype = I
        L.rl_sample_batch_debug.argtypes = [P, P, I, I, I, I64, P, P, I, P, I64, P, P, P, P, P, P,
                                            P, P, I, P, P]
        L.rl_sample_batch_static.restype = I
        L.rl_sample_batch_static.argtypes = [P, I, I, I, I64, P, P, I, P, I64, P, P, P, P, P, P]
        L.rl_sample_host.restype = I
        L.rl_sample_host.argtypes = [P, P, I, I, P, P, I, P, I64, P, P, P, P]
        L.rl_decoder_sample.restype = I
        L.rl_decoder_sample.argtypes = [P, P, I, I, I64, P, P, P, P, P, P]
        L.rl_decoder_sample_host.restype = I
        L.rl_decoder_sample_host.argtypes = [P, P, I, I, P, P, P, P, P]
        L.rl_greedy.restype = I
        L.rl_greedy.argtypes = [P, P, I, I, I64, P, P]
        L.rl_grammar_greedy.restype = I
        L.rl_grammar_greedy.argtypes = [P, P, I, I, I64, P, I64, P, P]
        L.rl_specdec_sample.restype = I
        L.rl_specdec_sample.argtypes = [P, P, I, I, I64, P, P, P, P, P]
        L.rl_specdec_verify.restype = I
        L.rl_specdec_verify.argtypes = [P, P, I, I, I64, P, I, P, P, P, P, P, P, P]
        L.rl_greedy_host.restype = I
        L.rl_greedy_host.argtypes = [P, P, I, I, P]
        L.rl_grammar_greedy_host.restype = I
        L.rl_grammar_greedy_host.argtypes = [P, P, I, I, P, I64, P]
        L.rl_beam_step.restype = I
        L.rl_beam_step.argtypes = [P, P, I, I, I, I64, P, P, P, F, I, I, I, P, P, P, P, P]
        L.rl_sample_partial.restype = I
        L.rl_sample_partial.argtypes = [P, P, I, I, I, I64, I, P, P, I, P, I64, P, P, P, P]
        L.rl_sample_merge.restype = I
        L.rl_sample_merge.argtypes = [P, I, I, P, P, P, P, P, P, P, P]
        L.rl_sample_sharded.restype = I
        L.rl_sample_sharded.argtypes = [P, P, P, I, I, I, I64, I, I, P, P, I, P, I64, P, P, P, P, P, P]
        L.rl_nccl_unique_id.restype = I
        L.rl_nccl_unique_id.argtypes = [P]
        L.rl_nccl_comm_init.restype = I
        L.rl_nccl_comm_init.argtypes = [ctypes.POINTER(P), I, P, I]
        L.rl_nccl_comm_destroy.restype = I
        L.rl_nccl_comm_destroy.argtypes = [P]
        L.rl_sampler_kernel_times.restype = I
        L.rl_sampler_kernel_times.argtypes = [P, P, I, P]
        L.rl_sampler_set_debug.restype = I
        L.rl_sampler_set_debug.argtypes = [P, ctypes.c_uint32]
        L.rl_selfcheck_div.restype = I
        L.rl_selfcheck_div.argtypes = [P, I, P, I, P, P, P]
        L.rl_gbnf_create.restype = I
        L.rl_gbnf_create.argtypes = [ctypes.c_char_p, ctypes.c_char_p, I, P, P, ctypes.c_int32, ctypes.POINTER(P)]
        L.rl_gbnf_destroy.restype = None
        L.rl_gbnf_destroy.argtypes = [P]
        L.rl_gbnf_state_create.restype = I
        L.rl_gbnf_state_create.argtypes = [P, ctypes.POINTER(P)]
        L.rl_gbnf_state_destroy.restype = None
        L.rl_gbnf_state_destroy.argtypes = [P]
        L.rl_gbnf_state_copy.restype = I
        L.rl_gbnf_state_copy.argtypes = [P, P]
        L.rl_gbnf_accepting.restype = I
        L.rl_gbnf_accepting.argtypes = [P]
        L.rl_gbnf_accept.restype = I
        L.rl_gbnf_accept.argtypes = [P, P, ctypes.c_int32]
        L.rl_gbnf_mask.restype = I
        L.rl_gbnf_mask.argtypes = [P, P, P, I64, P]
        L.rl_gbnf_accept_batch.restype = I
        L.rl_gbnf_accept_batch.argtypes = [P, P, P, I, P, I]
        L.rl_gbnf_mask_batch.restype = I
        L.rl_gbnf_mask_batch.argtypes = [P, P, I, P, I64, P, I]
        L.rl_lmhead_logits.restype = I
        L.rl_lmhead_logits.argtypes = [P, P, I64, P, I64, I, I, I, P, I, I64, P]
        L.rl_lmhead_greedy.restype = I
        L.rl_lmhead_greedy.argtypes = [P, P, I64, P, I64, I, I, I, P, P, P, I64, P]
        L.rl_lmhead_sample.restype = I
        L.rl_lmhead_sample.argtypes = [P, P, I64, P, I64, I, I, I, P, P, I, P, P, P, P, P, P]
        _lib = L
    return _lib


def last_error() -> str:
    return lib().rl_last_error().decode()


def check(st, what=""):
    if st != RL_OK:
        raise RLError(st, f"{what}: {last_error()}")


def _ptr(t):
    """Device (or host numpy) pointer of a tensor/array, None for None."""
    if t is None:
        return None
    if isinstance(t, np.ndarray):
        return t.ctypes.data_as(ctypes.c_void_p)
    return ctypes.c_void_p(t.data_ptr())


def _stream(stream):
    if stream is None:
        import torch

        stream = torch.cuda.current_stream()
    return ctypes.c_void_p(stream.cuda_stream)


class Sampler:
    """Owns an rl_sampler handle on one device."""

    def __init__(self, device=0, max_batch=256, max_vocab=131072, max_history=1024, flags=0):
        h = ctypes.c_void_p()
        check(lib().rl_sampler_create(ctypes.byref(h), device, max_batch, max_vocab, max_history, flags),
              "rl_sampler_create")
        self.h = h
        self.device = device

    def set_debug(self, flags):
        """rl_sampler_set_debug: RL_DEBUG_* switches (0 = off)."""
        check(lib().rl_sampler_set_debug(self.h, int(flags)), "rl_sampler_set_debug")

    def kernel_times(self):
        """rl_sampler_kernel_times: the last timed call's kernel times (ms)."""
        buf = (ctypes.c_float * 4)()
        n = ctypes.c_int()
        check(lib().rl_sampler_kernel_times(self.h, buf, 4, ctypes.byref(n)), "rl_sampler_kernel_times")
        return [buf[i] for i in range(n.value)]

    def close(self):
        if self.h:
            lib().rl_sampler_destroy(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    # -- spec profile ---------------------------------------------------------
    def sample(self, logits, params, uniforms, hist=None, hist_len=None, mask=None, out_tok=None,
               out_prob=None, row_status=None, stream=None):
        """logits [B, V] f32/bf16 (cuda), params: torch uint8 view of rl_row_params[B] (cuda)."""
        import torch

        B, V = logits.shape
        dtype = RL_BF16 if logits.dtype == torch.bfloat16 else RL_F32
        dev = logits.device
        if out_tok is None:
            out_tok = torch.empty(B, dtype=torch.int32, device=dev)
        if out_prob is None:
            out_prob = torch.empty(B, dtype=torch.float32, device=dev)
        if row_status is None:
            row_status = torch.empty(B, dtype=torch.int32, device=dev)
        hs = hist.shape[1] if hist is not None else 0
        ms = mask.shape[1] if mask is not None else 0
        check(lib().rl_sample_batch(self.h, _ptr(logits), dtype, B, V, logits.stride(0), _ptr(hist),
                                    _ptr(hist_len), hs, _ptr(mask), ms, _ptr(params), _ptr(uniforms),
                                    _ptr(out_tok), _ptr(out_prob), _ptr(row_status), _stream(stream)),
              "rl_sample_batch")
        return out_tok, out_prob, row_status

    def sample_debug(self, logits, params, uniforms, hist=None, hist_len=None, mask=None, list_cap=1024,
                     stream=None):
        import torch

        B, V = logits.shape
        dtype = RL_BF16 if logits.dtype == torch.bfloat16 else RL_F32
        dev = logits.device
        out_tok = torch.empty(B, dtype=torch.int32, device=dev)
        out_prob = torch.empty(B, dtype=torch.float32, device=dev)
        row_status = torch.empty(B, dtype=torch.int32, device=dev)
        list_ids = torch.full((B, list_cap), -1, dtype=torch.int32, device=dev)
        list_probs = torch.zeros((B, list_cap), dtype=torch.float32, device=dev)
        list_len = torch.zeros(B, dtype=torch.int32, device=dev)
        cut = torch.full((B, 3), -3, dtype=torch.int32, device=dev)
        hs = hist.shape[1] if hist is not None else 0
        ms = mask.shape[1] if mask is not None else 0
        check(lib().rl_sample_batch_debug(self.h, _ptr(logits), dtype, B, V, logits.stride(0), _ptr(hist),
                                          _ptr(hist_len), hs, _ptr(mask), ms, _ptr(params), _ptr(uniforms),
                                          _ptr(out_tok), _ptr(out_prob), _ptr(row_status), _ptr(list_ids),
                                          _ptr(list_probs), _ptr(list_len), list_cap, _ptr(cut), _stream(stream)),
              "rl_sample_batch_debug")
        return out_tok, out_prob, row_status, list_ids, list_probs, list_len, cut

    # -- vocabulary shards -------------------------------------------------------
    def sample_partial(self, logits, vocab_offset, params, hist=None, hist_len=None, mask=None, out_keys=None,
                       out_stats=None, stream=None):
        """One shard's partial result (rl_sample_partial): keys [B, PART_KEYS]
        int64 (the uint64 key bits) and stats [B, 32] uint8 (rl_part_stats)."""
        import torch

        B, V = logits.shape
        dtype = RL_BF16 if logits.dtype == torch.bfloat16 else RL_F32
        dev = logits.device
        if out_keys is None:
            out_keys = torch.empty((B, PART_KEYS), dtype=torch.int64, device=dev)
        if out_stats is None:
            out_stats = torch.empty((B, PART_STATS_DTYPE.itemsize), dtype=torch.uint8, device=dev)
        hs = hist.shape[1] if hist is not None else 0
        ms = mask.shape[1] if mask is not None else 0
        check(lib().rl_sample_partial(self.h, _ptr(logits), dtype, B, V, logits.stride(0), int(vocab_offset),
                                      _ptr(hist), _ptr(hist_len), hs, _ptr(mask), ms, _ptr(params),
                                      _ptr(out_keys), _ptr(out_stats), _stream(stream)),
              "rl_sample_partial")
        return out_keys, out_stats

    def sample_merge(self, keys, stats, params, uniforms, out_tok=None, out_prob=None, row_status=None,
                     stream=None):
        """rl_sample_merge over keys [G, B, PART_KEYS] and stats [G, B, 32]."""
        import torch

        G, B = keys.shape[0], keys.shape[1]
        dev = keys.device
        if out_tok is None:
            out_tok = torch.empty(B, dtype=torch.int32, device=dev)
        if out_prob is None:
            out_prob = torch.empty(B, dtype=torch.float32, device=dev)
        if row_status is None:
            row_status = torch.empty(B, dtype=torch.int32, device=dev)
        check(lib().rl_sample_merge(self.h, G, B, _ptr(keys.contiguous()), _ptr(stats.contiguous()), _ptr(params),
                                    _ptr(uniforms), _ptr(out_tok), _ptr(out_prob), _ptr(row_status),
                                    _stream(stream)),
              "rl_sample_merge")
        return out_tok, out_prob, row_status

    def sample_sharded(self, comm, logits_shard, vocab_offset, V_global, params, uniforms, hist=None, hist_len=None,
                       mask_shard=None, out_tok=None, out_prob=None, row_status=None, stream=None):
        """rl_sample_sharded: this rank's columns [vocab_offset, + width) of
        the rows, one NCCL all-gather on `comm`, the merged draw (global ids).
        The handle needs flags=RL_CREATE_SHARDED."""
        import torch

        B, W = logits_shard.shape
        dtype = RL_BF16 if logits_shard.dtype == torch.bfloat16 else RL_F32
        dev = logits_shard.device
        if out_tok is None:
            out_tok = torch.empty(B, dtype=torch.int32, device=dev)
        if out_prob is None:
            out_prob = torch.empty(B, dtype=torch.float32, device=dev)
        if row_status is None:
            row_status = torch.empty(B, dtype=torch.int32, device=dev)
        hs = hist.shape[1] if hist is not None else 0
        ms = mask_shard.shape[1] if mask_shard is not None else 0
        check(lib().rl_sample_sharded(self.h, ctypes.c_void_p(comm), _ptr(logits_shard), dtype, B, W,
                                      logits_shard.stride(0), int(vocab_offset), int(V_global), _ptr(hist),
                                      _ptr(hist_len), hs, _ptr(mask_shard), ms, _ptr(params), _ptr(uniforms),
                                      _ptr(out_tok), _ptr(out_prob), _ptr(row_status), _stream(stream)),
              "rl_sample_sharded")
        return out_tok, out_prob, row_status

    # -- beam search ----------------------------------------------------------------
    def beam_step(self, logits, items, beams, scores, done, lens=None, alpha=1.0, eos=2, log_softmax=1,
                  n_out=None, stream=None):
        """One BeamSearch::search step for items x beams rows of f32 logits
        (row = item * beams + beam). Returns (beam, tok, score, done), each
        [items, n_out]."""
        import torch

        R, V = logits.shape
        assert R == items * beams
        n_out = 2 * beams if n_out is None else n_out
        dev = logits.device
        ob = torch.empty((items, n_out), dtype=torch.int32, device=dev)
        ot = torch.empty((items, n_out), dtype=torch.int32, device=dev)
        osc = torch.empty((items, n_out), dtype=torch.float32, device=dev)
        od = torch.empty((items, n_out), dtype=torch.uint8, device=dev)
        check(lib().rl_beam_step(self.h, _ptr(logits), items, beams, V, logits.stride(0), _ptr(scores), _ptr(done),
                                 _ptr(lens), float(alpha), int(eos), int(log_softmax), n_out, _ptr(ob), _ptr(ot),
                                 _ptr(osc), _ptr(od), _stream(stream)),
              "rl_beam_step")
        return ob, ot, osc, od

    def sample_host(self, logits, params, uniforms, hist=None, hist_len=None, mask=None):
        """Host numpy buffers in and out (synchronous)."""
        B, V = logits.shape
        out_tok = np.empty(B, np.int32)
        out_prob = np.empty(B, np.float32)
        hs = hist.shape[1] if hist is not None else 0
        ms = mask.shape[1] if mask is not None else 0
        check(lib().rl_sample_host(self.h, _ptr(np.ascontiguousarray(logits, np.float32)), B, V, _ptr(hist),
                                   _ptr(hist_len), hs, _ptr(mask), ms, _ptr(params), _ptr(uniforms),
                                   _ptr(out_tok), _ptr(out_prob)),
              "rl_sample_host")
        return out_tok, out_prob

    def decoder_sample(self, logits, temperature, top_p, uniforms, out_tok=None, out_prob=None, stream=None):
        """rl_decoder_sample: Decoder::sample_with_params semantics on device rows
        [B, V] f32; temperature / top_p / uniforms are [B] f32 device tensors."""
        import torch

        B, V = logits.shape
        dev = logits.device
        if out_tok is None:
            out_tok = torch.empty(B, dtype=torch.int32, device=dev)
        if out_prob is None:
            out_prob = torch.empty(B, dtype=torch.float32, device=dev)
        check(lib().rl_decoder_sample(self.h, _ptr(logits), B, V, logits.stride(0), _ptr(temperature), _ptr(top_p),
                                      _ptr(uniforms), _ptr(out_tok), _ptr(out_prob), _stream(stream)),
              "rl_decoder_sample")
        return out_tok, out_prob

    def decoder_sample_host(self, logits, temperature, top_p, uniforms):
        """rl_decoder_sample_host: Decoder::sample_with_params semantics on host
        rows [B, V] f32 with per-row temperature / top_p / uniform; returns
        (tokens, probs) as numpy arrays."""
        lg = np.ascontiguousarray(logits, np.float32)
        if lg.ndim == 1:
            lg = lg[None, :]
        B, V = lg.shape
        t = np.ascontiguousarray(np.broadcast_to(np.asarray(temperature, np.float32), (B,)))
        p = np.ascontiguousarray(np.broadcast_to(np.asarray(top_p, np.float32), (B,)))
        u = np.ascontiguousarray(np.broadcast_to(np.asarray(uniforms, np.float32), (B,)))
        tok = np.empty(B, np.int32)
        prob = np.empty(B, np.float32)
        check(lib().rl_decoder_sample_host(self.h, _ptr(lg), B, V, _ptr(t), _ptr(p), _ptr(u), _ptr(tok), _ptr(prob)),
              "rl_decoder_sample_host")
        return tok, prob

    def greedy_host(self, logits):
        """rl_greedy_host: argmax (last maximum on ties) of host rows."""
        lg = np.ascontiguousarray(logits, np.float32)
        if lg.ndim == 1:
            lg = lg[None, :]
        tok = np.empty(lg.shape[0], np.int32)
        check(lib().rl_greedy_host(self.h, _ptr(lg), lg.shape[0], lg.shape[1], _ptr(tok)), "rl_greedy_host")
        return tok

    def grammar_greedy_host(self, logits, mask):
        """rl_grammar_greedy_host: argmax over the allowed ids of the bit-packed
        mask rows (lowest id on ties; an all-zero row allows every id)."""
        lg = np.ascontiguousarray(logits, np.float32)
        m = np.ascontiguousarray(mask, np.uint32)
        if lg.ndim == 1:
            lg, m = lg[None, :], m[None, :]
        tok = np.empty(lg.shape[0], np.int32)
        check(lib().rl_grammar_greedy_host(self.h, _ptr(lg), lg.shape[0], lg.shape[1], _ptr(m), m.shape[1], _ptr(tok)),
              "rl_grammar_greedy_host")
        return tok

    # -- speculative decoding ---------------------------------------------------
    def specdec_sample(self, logits, temperature, offset, uniforms, stream=None):
        """rl_specdec_sample: SpeculativeDecoder::sample per row of device
        logits [B, V] f32; temperature / offset / uniforms are [B] device tensors."""
        import torch

        B, V = logits.shape
        out = torch.empty(B, dtype=torch.int32, device=logits.device)
        check(lib().rl_specdec_sample(self.h, _ptr(logits), B, V, logits.stride(0), _ptr(temperature), _ptr(offset),
                                      _ptr(uniforms), _ptr(out), _stream(stream)),
              "rl_specdec_sample")
        return out

    def specdec_verify(self, logits, drafts, n_draft, accept_u, room, draw_u, stream=None):
        """rl_specdec_verify: SpeculativeDecoder::verify_and_accept per request;
        drafts / accept_u [B, Dmax] (same row stride), n_draft / room / draw_u
        [B] (device). Returns (accepted [B], token [B]) device tensors."""
        import torch

        B, V = logits.shape
        if accept_u.stride(0) != drafts.stride(0):
            raise ValueError("specdec_verify: drafts and accept_u need the same row stride")
        dev = logits.device
        acc = torch.empty(B, dtype=torch.int32, device=dev)
        tok = torch.empty(B, dtype=torch.int32, device=dev)
        check(lib().rl_specdec_verify(self.h, _ptr(logits), B, V, logits.stride(0), _ptr(drafts), drafts.stride(0),
                                      _ptr(n_draft), _ptr(accept_u), _ptr(room), _ptr(draw_u), _ptr(acc), _ptr(tok),
                                      _stream(stream)),
              "rl_specdec_verify")
        return acc, tok

    # -- LM head ------------------------------------------------------------
    @staticmethod
    def _lm_operands(hidden, weight):
        import torch

        if hidden.dtype != torch.bfloat16 or weight.dtype != torch.bfloat16:
            raise ValueError("lmhead: hidden and weight must be bf16")
        if hidden.stride(1) != 1 or weight.stride(1) != 1:
            raise ValueError("lmhead: hidden and weight must be row-major (unit inner stride)")
        B, H = hidden.shape
        V, H2 = weight.shape
        if H != H2:
            raise ValueError(f"lmhead: hidden has {H} columns, weight {H2}")
        return B, H, V

    def lmhead_logits(self, hidden, weight, out=None, out_dtype=None, stream=None):
        """rl_lmhead_logits: hidden [B, H] @ weight[V, H]^T on the tensor
        cores (bf16 operands, f32 sums) into out [B, V] (f32 or bf16)."""
        import torch

        B, H, V = self._lm_operands(hidden, weight)
        if out is None:
            out = torch.empty(B, V, dtype=out_dtype or torch.float32, device=hidden.device)
        dt = RL_BF16 if out.dtype == torch.bfloat16 else RL_F32
        check(lib().rl_lmhead_logits(self.h, _ptr(hidden), hidden.stride(0), _ptr(weight), weight.stride(0), B, H, V,
                                     _ptr(out), dt, out.stride(0), _stream(stream)),
              "rl_lmhead_logits")
        return out

    def lmhead_greedy(self, hidden, weight, out_logits=None, stream=None):
        """rl_lmhead_greedy: the last-maximum argmax of each row's logits,
        fused into the GEMM. Returns (tokens [B], row_status [B]); out_logits
        (f32 [B, V], optional) also receives the logits."""
        import torch

        B, H, V = self._lm_operands(hidden, weight)
        tok = torch.empty(B, dtype=torch.int32, device=hidden.device)
        st = torch.empty(B, dtype=torch.int32, device=hidden.device)
        ldo = out_logits.stride(0) if out_logits is not None else V
        check(lib().rl_lmhead_greedy(self.h, _ptr(hidden), hidden.stride(0), _ptr(weight), weight.stride(0), B, H, V,
                                     _ptr(tok), _ptr(st), _ptr(out_logits), ldo, _stream(stream)),
              "rl_lmhead_greedy")
        return tok, st

    def lmhead_sample(self, hidden, weight, params, uniforms, hist=None, hist_len=None, out_tok=None, out_prob=None,
                      row_status=None, stream=None):
        """rl_lmhead_sample: the LM head's logits sampled by the batched
        sampler (same params / uniforms / history as sample())."""
        import torch

        B, H, V = self._lm_operands(hidden, weight)
        dev = hidden.device
        out_tok = out_tok if out_tok is not None else torch.empty(B, dtype=torch.int32, device=dev)
        out_prob = out_prob if out_prob is not None else torch.empty(B, dtype=torch.float32, device=dev)
        row_status = row_status if row_status is not None else torch.empty(B, dtype=torch.int32, device=dev)
        hs = hist.shape[1] if hist is not None else 0
        check(lib().rl_lmhead_sample(self.h, _ptr(hidden), hidden.stride(0), _ptr(weight), weight.stride(0), B, H, V,
                                     _ptr(hist), _ptr(hist_len), hs, _ptr(params), _ptr(uniforms), _ptr(out_tok),
                                     _ptr(out_prob), _ptr(row_status), _stream(stream)),
              "rl_lmhead_sample")
        return out_tok, out_prob, row_status

    def sample_host_ptrs(self, logits_p, B, V, params_p, u_p, tok_p, prob_p, hist_p=None, hist_len_p=None,
                         hist_stride=0, mask_p=None, mask_stride=0):
        """Host-pointer variant (pinned buffers) used by the end-to-end benchmark."""
        check(lib().rl_sample_host(self.h, logits_p, B, V, hist_p, hist_len_p, hist_stride, mask_p,
                                   mask_stride, params_p, u_p, tok_p, prob_p),
              "rl_sample_host")


def params_tensor(p: np.ndarray, device):
    """rl_row_params[B] (numpy structured) -> cuda uint8 tensor holding the same bytes."""
    import torch

    return torch.from_numpy(np.ascontiguousarray(p).view(np.uint8).copy()).to(device)


def sample_static(logits, params, uniforms, hist=None, hist_len=None, mask=None, out_tok=None, out_prob=None,
                  row_status=None, stream=None):
    """rl_sample_batch_static: spec sampling on the current device with no
    handle and no allocation inside the call (outputs are allocated here when
    not given). Same arguments and results as Sampler.sample."""
    import torch

    B, V = logits.shape
    dtype = RL_BF16 if logits.dtype == torch.bfloat16 else RL_F32
    dev = logits.device
    if out_tok is None:
        out_tok = torch.empty(B, dtype=torch.int32, device=dev)
    if out_prob is None:
        out_prob = torch.empty(B, dtype=torch.float32, device=dev)
    if row_status is None:
        row_status = torch.empty(B, dtype=torch.int32, device=dev)
    hs = hist.shape[1] if hist is not None else 0
    ms = mask.shape[1] if mask is not None else 0
    # the entry point runs on the current device with that device's scratch:
    # make the tensors' device current, and use its stream
    with torch.cuda.device(dev):
        if stream is None:
            stream = torch.cuda.current_stream(dev)
        _call_static(logits, dtype, B, V, hist, hist_len, hs, mask, ms, params, uniforms, out_tok, out_prob,
                     row_status, stream)
    return out_tok, out_prob, row_status


def _call_static(logits, dtype, B, V, hist, hist_len, hs, mask, ms, params, uniforms, out_tok, out_prob, row_status,
                 stream):
    check(lib().rl_sample_batch_static(_ptr(logits), dtype, B, V, logits.stride(0), _ptr(hist), _ptr(hist_len), hs,
                                       _ptr(mask), ms, _ptr(params), _ptr(uniforms), _ptr(out_tok), _ptr(out_prob),
                                       _ptr(row_status), _stream(stream)),
          "rl_sample_batch_static")


def selfcheck_div(a, T, stream=None):
    """rl_selfcheck_div over device float32 tensors a [n] and T [nT]: per T the
    count of quotients that differ in any bit from IEEE division, and whether
    the fixed-divisor path is in use for it. Returns two cpu numpy arrays."""
    import torch

    nT = T.numel()
    mism = torch.zeros(nT, dtype=torch.int32, device=a.device)
    fast = torch.zeros(nT, dtype=torch.int32, device=a.device)
    check(lib().rl_selfcheck_div(_ptr(a), a.numel(), _ptr(T), nT, _ptr(mism), _ptr(fast), _stream(stream)),
          "rl_selfcheck_div")
    torch.cuda.synchronize(a.device)
    return mism.cpu().numpy().astype(np.uint32), fast.cpu().numpy()


def nccl_unique_id() -> bytes:
    """rl_nccl_unique_id: a new NCCL communicator id (made on one rank)."""
    buf = ctypes.create_string_buffer(NCCL_ID_BYTES)
    check(lib().rl_nccl_unique_id(ctypes.cast(buf, ctypes.c_void_p)), "rl_nccl_unique_id")
    return buf.raw


def nccl_comm_init(nranks: int, id_bytes: bytes, rank: int) -> int:
    """rl_nccl_comm_init on the current device: returns the ncclComm_t as an int."""
    if len(id_bytes) != NCCL_ID_BYTES:
        raise ValueError("an NCCL id has 128 bytes")
    buf = ctypes.create_string_buffer(bytes(id_bytes), NCCL_ID_BYTES)
    c = ctypes.c_void_p()
    check(lib().rl_nccl_comm_init(ctypes.byref(c), int(nranks), ctypes.cast(buf, ctypes.c_void_p), int(rank)),
          "rl_nccl_comm_init")
    return c.value


def nccl_comm_destroy(comm: int) -> None:
    check(lib().rl_nccl_comm_destroy(ctypes.c_void_p(comm)), "rl_nccl_comm_destroy")
