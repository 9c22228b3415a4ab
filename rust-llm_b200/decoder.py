"""The reference's single-sequence sampling interface (src/decoder.rs), on
the B200 library.

Same names, fields, defaults, argument meaning and results as the Rust
types they mirror; every token comes from the device through the C ABI
(include/rl_sampler.h), never from a host computation:

  SamplingParams  src/decoder.rs:294-316 (with Default), plus the two
                  penalties of the batched spec path (0.0 = absent)
  Decoder         src/decoder.rs:8-168: sample / sample_with_params are the
                  reference's own semantics (rl_decoder_sample_host: the
                  i > cutoff index quirk, the id-order CDF draw with `<=`,
                  the last-maximum fallback); greedy_sample is rl_greedy_host
  Sampler         src/decoder.rs:318-376: the 64-token prev_tokens ring, the
                  grammar path (rl_grammar_greedy_host over a bit-packed mask)
                  and, without a grammar, Decoder::sample at temperature 1.0
                  and top_p 0.9 (the reference ignores the params there)

The reference draws with rand_secure() (src/decoder.rs:170-188); here the
uniform comes from `uniform` (a callable returning a float in [0, 1)), by
default a numpy PCG64 stream, so that runs can be replayed.

Errors: the Rust signatures are infallible (-> Token). A failed sampling
call is logged and answered by the device argmax (rl_greedy_host, the
reference's greedy_sample); when that fails too, RLError is raised. Without
the library (not built, or no GPU) every call raises.
"""
from __future__ import annotations

import logging
import threading
from dataclasses import dataclass

import numpy as np

import rlsampler

log = logging.getLogger("rl_sampler")

PREV_TOKENS = 64  # Sampler::prev_tokens capacity (src/decoder.rs:321, 350-354)

_local = threading.local()


def _handle(device: int, vocab: int) -> rlsampler.Sampler:
    """A per-thread, per-device rl_sampler handle for single-row host calls
    (handles are not shared between threads); grown when a longer row comes."""
    cache = getattr(_local, "handles", None)
    if cache is None:
        cache = _local.handles = {}
    h = cache.get(device)
    if h is None or h.max_vocab < vocab:
        if h is not None:
            h.close()
        cap = max(vocab, 32000)
        h = rlsampler.Sampler(device, max_batch=1, max_vocab=cap, max_history=0)
        h.max_vocab = cap
        cache[device] = h
    return h


def _default_uniform(seed=None):
    rng = np.random.Generator(np.random.PCG64(seed))
    return lambda: float(np.float32(rng.random()) * np.float32(1.0 - 2.0 ** -24))


@dataclass
class SamplingParams:
    """src/decoder.rs:294-316. The mirostat fields are carried as in the
    reference, which reads them nowhere (no mirostat sampler exists there)."""

    temperature: float = 1.0
    top_p: float = 0.9
    top_k: int = 40
    repeat_penalty: float = 1.1
    mirostat: bool = False
    mirostat_tau: float = 5.0
    mirostat_eta: float = 0.1
    # the batched spec path's additions (rl_row_params); 0.0 leaves them out
    presence_penalty: float = 0.0
    frequency_penalty: float = 0.0

    def row(self) -> np.ndarray:
        """This row's rl_row_params for the batched spec entry points."""
        p = np.zeros(1, rlsampler.ROW_PARAMS_DTYPE)
        p["temperature"] = self.temperature
        p["top_p"] = self.top_p
        p["top_k"] = self.top_k
        p["repeat_penalty"] = self.repeat_penalty
        p["presence_penalty"] = self.presence_penalty
        p["frequency_penalty"] = self.frequency_penalty
        return p


class Decoder:
    """src/decoder.rs:8-29 (fields and Decoder::new defaults)."""

    def __init__(self, vocab_size: int, hidden_size: int = 0, device: int = 0, uniform=None):
        self.vocab_size = vocab_size
        self.hidden_size = hidden_size
        self.temperature = 1.0
        self.top_p = 0.9
        self.top_k = 40
        self.repeat_penalty = 1.1
        self.last_n_tokens = 64
        self.device = device
        self.uniform = uniform or _default_uniform()

    def sample(self, logits, _tokenizer=None) -> int:
        """Decoder::sample (src/decoder.rs:31-33): temperature 1.0, top_p 0.9,
        whatever the fields say."""
        return self.sample_with_params(logits, _tokenizer, 1.0, 0.9)

    def sample_with_params(self, logits, _tokenizer, temperature: float, top_p: float) -> int:
        """Decoder::sample_with_params (src/decoder.rs:35-100) on the device."""
        x = np.ascontiguousarray(logits, np.float32).reshape(-1)
        h = _handle(self.device, x.size)
        try:
            tok, _ = h.decoder_sample_host(x, temperature, top_p, self.uniform())
            return int(tok[0])
        except rlsampler.RLError as err:
            log.warning("rl_decoder_sample_host failed (%s); answering with the device argmax", err)
            return int(h.greedy_host(x)[0])

    def greedy_sample(self, logits) -> int:
        """Decoder::greedy_sample (src/decoder.rs:160-167): last maximum on ties."""
        x = np.ascontiguousarray(logits, np.float32).reshape(-1)
        return int(_handle(self.device, x.size).greedy_host(x)[0])


def allowed_mask(allowed, V: int) -> np.ndarray:
    """Allowed ids -> one bit-packed mask row (bit j of word w is id 32w + j);
    an empty set gives the all-zero row, which allows every id as the
    reference does (src/decoder.rs:362-364)."""
    m = np.zeros((V + 31) // 32, np.uint32)
    ids = np.asarray([i for i in allowed if 0 <= i < V], np.int64)
    if ids.size:
        np.bitwise_or.at(m, ids >> 5, (np.uint32(1) << (ids & 31).astype(np.uint32)))
    return m


class Sampler:
    """src/decoder.rs:318-357: a sequence's sampler and its last 64 tokens."""

    def __init__(self, params: SamplingParams | None = None, device: int = 0, uniform=None):
        self.params = params or SamplingParams()
        self.grammar = None
        self.prev_tokens: list[int] = []
        self.device = device
        self.uniform = uniform or _default_uniform()

    def with_grammar(self, grammar) -> "Sampler":
        """Sampler::with_grammar: `grammar` has get_allowed_tokens(prev_tokens)
        -> iterable of ids -- grammar.Grammar, the reference's Grammar
        (src/decoder.rs:378-557), or any object with that method."""
        self.grammar = grammar
        return self

    def sample(self, logits) -> int:
        x = np.ascontiguousarray(logits, np.float32).reshape(-1)
        if self.grammar is not None:
            token = self.sample_with_grammar(x, self.grammar)
        else:
            d = Decoder(x.size, 0, self.device, self.uniform)
            d.temperature = self.params.temperature
            d.top_p = self.params.top_p
            d.top_k = self.params.top_k
            d.repeat_penalty = self.params.repeat_penalty
            token = d.sample(x)
        if len(self.prev_tokens) >= PREV_TOKENS:
            self.prev_tokens.pop(0)
        self.prev_tokens.append(token)
        return token

    def sample_with_grammar(self, logits, grammar) -> int:
        """Sampler::sample_with_grammar (src/decoder.rs:359-376): the allowed
        id with the largest logit, the lowest such id on ties."""
        x = np.ascontiguousarray(logits, np.float32).reshape(-1)
        m = allowed_mask(grammar.get_allowed_tokens(list(self.prev_tokens)), x.size)
        return int(_handle(self.device, x.size).grammar_greedy_host(x, m)[0])
