"""ctypes front end of the CPU oracle (oracle/oracle.cpp).

Test infrastructure only: imported by tests/, __graft_entry__.smoke() and
bench.py's cpu_baseline / reference legs, never by the product library.
Parity is unpinned against the reference itself (see oracle.cpp's header).
"""
from __future__ import annotations

import ctypes
import os
import subprocess
from dataclasses import dataclass

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB_PATH = os.path.join(_HERE, "build", "liboracle.so")
_lib = None


class RowParams(ctypes.Structure):
    _fields_ = [
        ("temperature", ctypes.c_float),
        ("top_p", ctypes.c_float),
        ("top_k", ctypes.c_int32),
        ("repeat_penalty", ctypes.c_float),
        ("presence_penalty", ctypes.c_float),
        ("frequency_penalty", ctypes.c_float),
    ]


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


class SpecOut(ctypes.Structure):
    _fields_ = [
        ("token", ctypes.c_int32),
        ("prob", ctypes.c_float),
        ("K", ctypes.c_int32),
        ("cutoff", ctypes.c_int32),
        ("draw_margin", ctypes.c_double),
        ("cut_margin", ctypes.c_double),
        ("Z", ctypes.c_double),
        ("max_x", ctypes.c_float),
        ("cut_id", ctypes.c_int32),
    ]


def build() -> str:
    """Compile liboracle.so with the committed Makefile (idempotent)."""
    subprocess.run(["make", "-s", "-C", _HERE], check=True)
    return _LIB_PATH


def lib():
    global _lib
    if _lib is None:
        src = os.path.join(_HERE, "oracle.cpp")
        if (not os.path.exists(_LIB_PATH)) or os.path.getmtime(_LIB_PATH) < os.path.getmtime(src):
            build()
        L = ctypes.CDLL(_LIB_PATH)
        P = ctypes.c_void_p
        L.orc_decoder_sample.restype = ctypes.c_int32
        L.orc_decoder_sample.argtypes = [P, ctypes.c_int, ctypes.c_float, ctypes.c_float,
                                         ctypes.c_float, P, P, P, P]
        L.orc_greedy.restype = ctypes.c_int32
        L.orc_greedy.argtypes = [P, ctypes.c_int]
        L.orc_grammar_greedy.restype = ctypes.c_int32
        L.orc_grammar_greedy.argtypes = [P, ctypes.c_int, P]
        L.orc_spec_sample_row.restype = ctypes.c_int
        L.orc_spec_sample_row.argtypes = [P, ctypes.c_int, P, ctypes.c_int, P, P, ctypes.c_float,
                                          P, P, P, ctypes.c_int]
        L.orc_spec_sample_batch.restype = ctypes.c_int
        L.orc_spec_sample_batch.argtypes = [P, ctypes.c_int, ctypes.c_int, ctypes.c_int,
                                            ctypes.c_int64, P, P, ctypes.c_int, P, ctypes.c_int64,
                                            P, P, P, P, ctypes.c_int]
        L.orc_decoder_sample_batch.restype = None
        L.orc_decoder_sample_batch.argtypes = [P, ctypes.c_int, ctypes.c_int, ctypes.c_int64, P,
                                               P, P, P, P, ctypes.c_int]
        L.orc_beam_step.restype = None
        L.orc_beam_step.argtypes = [P, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int64,
                                    P, P, P, ctypes.c_float, ctypes.c_int, ctypes.c_int,
                                    ctypes.c_int, P, P, P, P]
        L.orc_specdec_sample.restype = ctypes.c_int32
        L.orc_specdec_sample.argtypes = [P, ctypes.c_int, ctypes.c_float, ctypes.c_int, ctypes.c_float]
        L.orc_specdec_softmax_at.restype = ctypes.c_float
        L.orc_specdec_softmax_at.argtypes = [P, ctypes.c_int, ctypes.c_int64]
        L.orc_specdec_verify.restype = ctypes.c_int32
        L.orc_specdec_verify.argtypes = [P, ctypes.c_int, P, ctypes.c_int, P, ctypes.c_int, ctypes.c_float, P]
        L.orc_matmul_vec.restype = None
        L.orc_matmul_vec.argtypes = [P, P, ctypes.c_int64, ctypes.c_int, ctypes.c_int, ctypes.c_int, P, ctypes.c_int]
        _lib = L
    return _lib


def _p(a):
    return None if a is None else a.ctypes.data_as(ctypes.c_void_p)


def decoder_sample(logits, temperature, top_p, r):
    """ref_exact Decoder::sample_with_params on one f32 row -> dict."""
    x = np.ascontiguousarray(logits, dtype=np.float32)
    prob = np.zeros(1, np.float32)
    cut = np.zeros(1, np.int32)
    dm = np.zeros(1, np.float64)
    cm = np.zeros(1, np.float64)
    tok = lib().orc_decoder_sample(_p(x), x.size, float(temperature), float(top_p), float(r),
                                   _p(prob), _p(cut), _p(dm), _p(cm))
    return dict(token=int(tok), prob=float(prob[0]), cutoff=int(cut[0]),
                draw_margin=float(dm[0]), cut_margin=float(cm[0]))


def matmul_vec(hidden, weight, nthreads=1):
    """Model::matmul_vec (src/model.rs:246-261) per row of hidden [rows, H]
    (f32) against weight [V, H] (f32): sequential f32 sums."""
    x = np.ascontiguousarray(hidden, np.float32)
    if x.ndim == 1:
        x = x[None, :]
    w = np.ascontiguousarray(weight, np.float32)
    V, H = w.shape
    out = np.empty((x.shape[0], V), np.float32)
    lib().orc_matmul_vec(_p(x), _p(w), ctypes.c_int64(w.size), H, V, x.shape[0], _p(out), nthreads)
    return out


def greedy(logits):
    x = np.ascontiguousarray(logits, dtype=np.float32)
    return int(lib().orc_greedy(_p(x), x.size))


def grammar_greedy(logits, mask_row):
    x = np.ascontiguousarray(logits, dtype=np.float32)
    m = np.ascontiguousarray(mask_row, dtype=np.uint32)
    return int(lib().orc_grammar_greedy(_p(x), x.size, _p(m)))


@dataclass
class SpecResult:
    status: int
    token: int
    prob: float
    K: int
    cutoff: int
    draw_margin: float
    cut_margin: float
    Z: float
    max_x: float
    list_ids: np.ndarray
    list_p: np.ndarray
    cut_id: int = -1


def spec_sample_row(logits, hist, mask_row, params, u, list_cap=0) -> SpecResult:
    """spec profile on one row (f32 values; bf16 callers convert first)."""
    x = np.ascontiguousarray(logits, dtype=np.float32)
    h = np.ascontiguousarray(hist if hist is not None else np.zeros(0), dtype=np.int32)
    m = None if mask_row is None else np.ascontiguousarray(mask_row, dtype=np.uint32)
    prm = RowParams(*[params[k] for k in ("temperature", "top_p", "top_k", "repeat_penalty",
                                          "presence_penalty", "frequency_penalty")])
    out = SpecOut()
    ids = np.zeros(max(list_cap, 1), np.int32)
    ps = np.zeros(max(list_cap, 1), np.float32)
    st = lib().orc_spec_sample_row(_p(x), x.size, _p(h), h.size, _p(m), ctypes.byref(prm),
                                   float(u), ctypes.byref(out), _p(ids), _p(ps), list_cap)
    n = min(out.K, list_cap) if st == 0 else 0
    return SpecResult(st, out.token, out.prob, out.K, out.cutoff, out.draw_margin, out.cut_margin,
                      out.Z, out.max_x, ids[:n].copy(), ps[:n].copy(), out.cut_id)


def spec_sample_batch(logits, hist, hist_len, mask, params, uniforms, nthreads=1, dtype=0):
    """Batched spec sampling (threads over rows) -> (tokens, probs, n_bad)."""
    B, V = logits.shape
    lg = np.ascontiguousarray(logits)
    tok = np.zeros(B, np.int32)
    prob = np.zeros(B, np.float32)
    hs = hist.shape[1] if hist is not None else 0
    ms = mask.shape[1] if mask is not None else 0
    bad = lib().orc_spec_sample_batch(_p(lg), dtype, B, V, V, _p(hist), _p(hist_len), hs,
                                      _p(mask), ms, _p(params), _p(uniforms), _p(tok), _p(prob),
                                      nthreads)
    return tok, prob, bad


def decoder_sample_batch(logits, temperature, top_p, uniforms, nthreads=1):
    B, V = logits.shape
    lg = np.ascontiguousarray(logits, dtype=np.float32)
    tok = np.zeros(B, np.int32)
    prob = np.zeros(B, np.float32)
    t = np.ascontiguousarray(temperature, np.float32)
    p = np.ascontiguousarray(top_p, np.float32)
    u = np.ascontiguousarray(uniforms, np.float32)
    lib().orc_decoder_sample_batch(_p(lg), B, V, V, _p(t), _p(p), _p(u), _p(tok), _p(prob),
                                   nthreads)
    return tok, prob


def beam_step(logits, items, beams, scores, done, lens, alpha, eos, log_softmax, n_out):
    lg = np.ascontiguousarray(logits, dtype=np.float32)
    V = lg.shape[1]
    sc = np.ascontiguousarray(scores, np.float32)
    dn = np.ascontiguousarray(done, np.uint8)
    ln = np.ascontiguousarray(lens, np.int32)
    ob = np.zeros((items, n_out), np.int32)
    ot = np.zeros((items, n_out), np.int32)
    os_ = np.zeros((items, n_out), np.float32)
    od = np.zeros((items, n_out), np.uint8)
    lib().orc_beam_step(_p(lg), items, beams, V, V, _p(sc), _p(dn), _p(ln), float(alpha),
                        int(eos), int(log_softmax), n_out, _p(ob), _p(ot), _p(os_), _p(od))
    return ob, ot, os_, od


def specdec_sample(logits, temperature, offset, r):
    """SpeculativeDecoder::sample (src/inference.rs:376-414) on one f32 row."""
    x = np.ascontiguousarray(logits, dtype=np.float32)
    return int(lib().orc_specdec_sample(_p(x), x.size, float(temperature), int(offset), float(r)))


def specdec_softmax_at(logits, idx):
    """SpeculativeDecoder::softmax_at (src/inference.rs:416-429)."""
    x = np.ascontiguousarray(logits, dtype=np.float32)
    return float(lib().orc_specdec_softmax_at(_p(x), x.size, int(idx)))


def specdec_verify(logits, drafts, accept_u, room, draw_u):
    """SpeculativeDecoder::verify_and_accept (src/inference.rs:335-374) for one
    request -> (accepted count, appended token or -1)."""
    x = np.ascontiguousarray(logits, dtype=np.float32)
    d = np.ascontiguousarray(drafts, dtype=np.int32)
    a = np.ascontiguousarray(accept_u, dtype=np.float32)
    tok = np.zeros(1, np.int32)
    acc = lib().orc_specdec_verify(_p(x), x.size, _p(d), d.size, _p(a), int(room), float(draw_u), _p(tok))
    return int(acc), int(tok[0])
