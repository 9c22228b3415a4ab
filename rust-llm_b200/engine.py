"""The sampling part of ContinuousBatchingEngine::step (src/inference.rs:
103-141), one device call per step for the whole batch.

The reference loops over the running sequences, and for each one runs the
model, calls Model::sample_with_params(logits, state.temperature,
state.top_p) (src/model.rs:484-486 -> src/decoder.rs:35-100), pushes the
token and updates the sequence's counters. BatchStep does the same updates
for every live sequence at once, given the step's logits already on the
device (one row per live sequence, in the order `live()` returns):

  semantics "ref_exact" (default): rl_decoder_sample, the reference's own
      sample_with_params per row -- the same tokens as the reference's loop
      for the same uniforms;
  semantics "spec": rl_sample_batch with each sequence's optional top_k and
      penalties over its last HISTORY tokens (the batched pipeline).

SequenceState mirrors src/inference.rs:31-40 and carries the optional
sampler fields the batched path adds (all off by default).
"""
from __future__ import annotations

from dataclasses import dataclass, field

import numpy as np

import rlsampler

HISTORY = 64  # tokens of a sequence's history the penalties see (Sampler::prev_tokens)


@dataclass
class SequenceState:
    """src/inference.rs:31-40, plus the batched path's optional fields."""

    seq_id: int
    tokens: list = field(default_factory=list)
    position: int = 0
    finished: bool = False
    generated_tokens: int = 0
    max_tokens: int = 0
    temperature: float = 1.0
    top_p: float = 0.9
    # batched path only (0 / 1.0 = off)
    top_k: int = 0
    repeat_penalty: float = 1.0
    presence_penalty: float = 0.0
    frequency_penalty: float = 0.0

    def live(self) -> bool:
        """The reference's skip test (src/inference.rs:117-119), negated."""
        return not self.finished and self.generated_tokens < self.max_tokens


def live(states):
    """The sequences a step samples, in order."""
    return [s for s in states if s.live()]


def params_of(states) -> np.ndarray:
    p = np.zeros(len(states), rlsampler.ROW_PARAMS_DTYPE)
    for i, s in enumerate(states):
        p[i] = (s.temperature, s.top_p, s.top_k, s.repeat_penalty, s.presence_penalty, s.frequency_penalty)
    return p


def history_of(states, width=HISTORY):
    """[B, width] int32 ids (each sequence's last `width` tokens) and [B] lengths."""
    h = np.zeros((len(states), width), np.int32)
    n = np.zeros(len(states), np.int32)
    for i, s in enumerate(states):
        t = s.tokens[-width:]
        h[i, : len(t)] = t
        n[i] = len(t)
    return h, n


def apply(states, tokens) -> dict:
    """The reference's per-sequence updates (src/inference.rs:128-138) for the
    sampled tokens; returns {seq_id: token}."""
    out = {}
    for s, t in zip(states, tokens):
        t = int(t)
        s.tokens.append(t)
        s.generated_tokens += 1
        s.position += 1
        out[s.seq_id] = t
        if t == 0 or s.generated_tokens >= s.max_tokens:
            s.finished = True
    return out


class BatchStep:
    """One device sampling call per engine step (see the module docstring)."""

    def __init__(self, vocab: int, max_batch: int, device: int = 0, semantics: str = "ref_exact", uniform=None):
        if semantics not in ("ref_exact", "spec"):
            raise ValueError(f"semantics {semantics!r}")
        self.V = vocab
        self.semantics = semantics
        self.device = device
        self.sampler = rlsampler.Sampler(device, max_batch=max_batch, max_vocab=vocab, max_history=HISTORY)
        rng = np.random.Generator(np.random.PCG64())
        self.uniform = uniform or (lambda n: (rng.random(n) * (1.0 - 2.0 ** -24)).astype(np.float32))

    def sample(self, states, logits, uniforms=None):
        """Tokens for `states` (the live sequences, in order) from device logits
        [len(states), V] f32; the states are not changed."""
        import torch

        B = len(states)
        if logits.shape[0] != B or logits.shape[1] != self.V:
            raise ValueError(f"logits {tuple(logits.shape)} for {B} sequences of vocabulary {self.V}")
        dev = logits.device
        u = np.ascontiguousarray(self.uniform(B) if uniforms is None else uniforms, np.float32)
        du = torch.from_numpy(u).to(dev)
        if self.semantics == "ref_exact":
            T = torch.tensor([s.temperature for s in states], dtype=torch.float32, device=dev)
            P = torch.tensor([s.top_p for s in states], dtype=torch.float32, device=dev)
            tok, _ = self.sampler.decoder_sample(logits, T, P, du)
            return tok.cpu().numpy()
        h, n = history_of(states)
        tok, _, st = self.sampler.sample(logits, rlsampler.params_tensor(params_of(states), dev), du,
                                         torch.from_numpy(h).to(dev), torch.from_numpy(n).to(dev))
        st = st.cpu().numpy()
        if (st != 0).any():
            bad = int(np.flatnonzero(st)[0])
            raise rlsampler.RLError(int(st[bad]), f"sequence {states[bad].seq_id}: row status {int(st[bad])}")
        return tok.cpu().numpy()

    def step(self, states, logits, uniforms=None) -> dict:
        """Samples the live sequences (logits: one row per live sequence, in
        order) and applies the reference's updates; returns {seq_id: token}."""
        act = live(states)
        if not act:
            return {}
        return apply(act, self.sample(act, logits, uniforms))

    def close(self):
        self.sampler.close()
