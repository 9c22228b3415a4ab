"""Seeded synthetic sampling workloads (the five benchmark configurations).

The reference publishes no benchmark data; these generators produce inputs
with the shapes and value distributions of each configuration. numpy PCG64
seeded with 1000*config + step for the data and seed + 7_000_000 for the
per-row uniform draws, so that the CPU oracle and the device see the same bytes.
"""
from __future__ import annotations

from dataclasses import dataclass

import numpy as np

from rlsampler import ROW_PARAMS_DTYPE

CONFIGS = {
    1: dict(name="single_seq_cli_defaults", B=1, V=32000),
    2: dict(name="hetero_batch_b256_v128256_f32", B=256, V=128256),
    3: dict(name="grammar_b64_v32000", B=64, V=32000),
    4: dict(name="beam_16x8_v151936", items=16, beams=8, V=151936),
    5: dict(name="vocab_shard_b1024_v256000_bf16", B=1024, V=256000),
}


@dataclass
class SampleBatch:
    logits: np.ndarray          # [B, V] float32 (bf16 configs: the bf16 values as float32)
    params: np.ndarray          # [B] ROW_PARAMS_DTYPE
    uniforms: np.ndarray        # [B] float32
    hist: np.ndarray | None     # [B, H] int32
    hist_len: np.ndarray | None  # [B] int32
    mask: np.ndarray | None     # [B, ceil(V/32)] uint32
    bf16_bits: np.ndarray | None = None  # [B, V] uint16 for bf16 configs


def _rng(config, step, salt=0):
    return np.random.Generator(np.random.PCG64(1000 * config + step + salt))


def uniforms(config, step, B):
    r = _rng(config, step, 7_000_000)
    return r.random(B, dtype=np.float64).astype(np.float32) * np.float32(1.0 - 2 ** -24)


def f32_to_bf16_bits(x: np.ndarray) -> np.ndarray:
    """Round-to-nearest-even f32 -> bf16 bit patterns."""
    u = x.astype(np.float32).view(np.uint32)
    r = ((u >> 16) & 1) + np.uint32(0x7FFF)
    return ((u + r) >> 16).astype(np.uint16)


def bf16_bits_to_f32(b: np.ndarray) -> np.ndarray:
    return (b.astype(np.uint32) << 16).view(np.float32)


def config1(step, B=1, V=32000):
    r = _rng(1, step)
    x = r.normal(0.0, 3.0, (B, V)).astype(np.float32)
    for b in range(B):
        x[b, r.choice(V, 5, replace=False)] += np.float32(8.0)
    p = np.zeros(B, ROW_PARAMS_DTYPE)
    p["temperature"] = 1.0
    p["top_p"] = 0.9
    p["top_k"] = 40
    p["repeat_penalty"] = 1.1
    hist = r.integers(0, V, (B, 64)).astype(np.int32)
    return SampleBatch(x, p, uniforms(1, step, B), hist, np.full(B, 64, np.int32), None)


def config2(step, B=256, V=128256, rows=None):
    """Heterogeneous continuous batch. `rows` selects a subset of the B rows
    (same values as the full batch) for quick parity checks."""
    r = _rng(2, step)
    prior = (-1.1 * np.log(np.arange(V, dtype=np.float64) + 1.0)).astype(np.float32)
    p = np.zeros(B, ROW_PARAMS_DTYPE)
    p["temperature"] = r.uniform(0.5, 1.5, B)
    p["top_k"] = r.choice(np.array([0, 20, 50, 100]), B)
    p["top_p"] = r.uniform(0.8, 1.0, B)
    p["repeat_penalty"] = r.uniform(1.0, 1.3, B)
    p["presence_penalty"] = r.uniform(0.0, 0.5, B)
    p["frequency_penalty"] = r.uniform(0.0, 0.5, B)
    hist = r.integers(0, V, (B, 512)).astype(np.int32)
    idx = np.arange(B) if rows is None else np.asarray(rows)
    x = np.empty((len(idx), V), np.float32)
    for n, b in enumerate(idx):
        rb = _rng(2, step, 100_000 + 131 * int(b))
        x[n] = rb.normal(0.0, 4.0, V).astype(np.float32) + prior
    u = uniforms(2, step, B)
    return SampleBatch(x, p[idx], u[idx], hist[idx], np.full(len(idx), 512, np.int32), None)


def config3(step, B=64, V=32000):
    r = _rng(3, step)
    x = r.normal(0.0, 3.0, (B, V)).astype(np.float32)
    W = (V + 31) // 32
    mask = np.zeros((B, W), np.uint32)
    for b in range(B):
        dens = r.uniform(0.02, 0.30)
        bits = r.random(V) < dens
        if not bits.any():
            bits[r.integers(0, V)] = True
        packed = np.zeros(W * 32, np.uint64)
        packed[:V] = bits
        mask[b] = (packed.reshape(W, 32) << np.arange(32, dtype=np.uint64)).sum(axis=1).astype(np.uint32)
    p = np.zeros(B, ROW_PARAMS_DTYPE)
    p["temperature"] = 0.7
    p["top_k"] = 50
    p["top_p"] = 0.95
    p["repeat_penalty"] = 1.0
    return SampleBatch(x, p, uniforms(3, step, B), None, None, mask)


@dataclass
class BeamBatch:
    logits: np.ndarray  # [items * beams, V] float32, row = item * beams + beam
    items: int
    beams: int
    scores: np.ndarray  # [items * beams] float32 cumulative beam scores
    done: np.ndarray    # [items * beams] uint8
    lens: np.ndarray    # [items * beams] int32
    alpha: float = 1.0
    eos: int = 2


def config4(step, items=16, beams=8, V=151936, done_frac=0.0):
    """Beam-search step: logits ~ N(0, 3^2), scores ~ U[-20, 0], length
    penalty 1.0, EOS id 2. `done_frac` marks a share of the beams complete
    (the benchmark configuration has none)."""
    r = _rng(4, step)
    R = items * beams
    x = r.normal(0.0, 3.0, (R, V)).astype(np.float32)
    scores = r.uniform(-20.0, 0.0, R).astype(np.float32)
    done = (r.random(R) < done_frac).astype(np.uint8)
    lens = r.integers(1, 64, R).astype(np.int32)
    return BeamBatch(x, items, beams, scores, done, lens)


def config5_rows(step, B=1024, V=256000, rows=None):
    r = _rng(5, step)
    hist = r.integers(0, V, (B, 256)).astype(np.int32)
    idx = np.arange(B) if rows is None else np.asarray(rows)
    bits = np.empty((len(idx), V), np.uint16)
    for n, b in enumerate(idx):
        rb = _rng(5, step, 100_000 + 131 * int(b))
        bits[n] = f32_to_bf16_bits(rb.normal(0.0, 4.0, V).astype(np.float32))
    p = np.zeros(len(idx), ROW_PARAMS_DTYPE)
    p["temperature"] = 0.8
    p["top_k"] = 64
    p["top_p"] = 0.95
    p["repeat_penalty"] = 1.2
    u = uniforms(5, step, B)[idx]
    return SampleBatch(bf16_bits_to_f32(bits), p, u, hist[idx], np.full(len(idx), 256, np.int32), None,
                       bf16_bits=bits)


def mask_from_allowed(V, allowed_rows):
    W = (V + 31) // 32
    m = np.zeros((len(allowed_rows), W), np.uint32)
    for b, ids in enumerate(allowed_rows):
        for i in ids:
            m[b, i >> 5] |= np.uint32(1 << (i & 31))
    return m


# ---------------------------------------------------------------------------
# Grammar-constrained decoding: a JSON grammar in GBNF notation and a seeded
# synthetic byte-level vocabulary (no tokenizer files are available offline)
# ---------------------------------------------------------------------------
GBNF_JSON = r'''
root   ::= ws value ws
value  ::= object | array | string | number | "true" | "false" | "null"
object ::= "{" ws ( member ( ws "," ws member )* )? ws "}"
member ::= string ws ":" ws value
array  ::= "[" ws ( value ( ws "," ws value )* )? ws "]"
string ::= "\"" ( [^"\\\x00-\x1f] | "\\" ( ["\\/bfnrt] | "u" [0-9a-fA-F]{4} ) )* "\""
number ::= "-"? ( "0" | [1-9] [0-9]* ) ( "." [0-9]+ )? ( [eE] [-+]? [0-9]+ )?
ws     ::= [ \t\n]*
'''


def json_vocab(V=32000, seed=31):
    """V tokens: the 256 single bytes, a few JSON pieces, random 2-6 byte
    strings over a JSON-like alphabet; the last id is the end token (no
    bytes)."""
    rng = np.random.default_rng(seed)
    toks = [bytes([c]) for c in range(256)]
    toks += [b'{"', b'":', b'",', b'"}', b"true", b"false", b"null", b"[]", b"{}", b", ", b": "]
    alpha = list(b'abcdekxyz"{}[]:,0123456789.- ')
    seen = set(toks)
    while len(toks) < V - 1:
        t = bytes(rng.choice(alpha, int(rng.integers(2, 7))).tolist())
        if t not in seen:
            seen.add(t)
            toks.append(t)
    return toks + [b""]
