"""The decoder.rs mirror (rust-llm_b200/decoder.py) on the device, token for
token against the oracle's restatement of the reference:

- Sampler::sample without a grammar over config-1 rows: Decoder::sample at
  temperature 1.0 / top_p 0.9 (src/decoder.rs:338-347 -> :31-100), the
  uniforms replayed into orc_decoder_sample; the 64-token ring at the end;
- Decoder::sample_with_params on config-1 and long rows, per-call T/top_p;
- Sampler::sample_with_grammar over config-3 rows and masks
  (src/decoder.rs:359-376) against orc_grammar_greedy;
- Decoder::greedy_sample against orc_greedy (last maximum on ties).
"""
import numpy as np
import pytest

import decoder
import oracle
import workloads

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu


class Replay:
    """A uniform source whose draws are kept for the oracle."""

    def __init__(self, seed):
        self.r = np.random.Generator(np.random.PCG64(seed))
        self.drawn = []

    def __call__(self):
        u = float(np.float32(self.r.random()) * np.float32(1.0 - 2.0 ** -24))
        self.drawn.append(u)
        return u


def test_sampler_without_grammar_is_decoder_sample():
    u = Replay(11)
    s = decoder.Sampler(decoder.SamplingParams(temperature=0.3, top_p=0.5, top_k=5), uniform=u)
    want = []
    for step in range(80):
        x = workloads.config1(step).logits[0]
        got = s.sample(x)
        want.append(oracle.decoder_sample(x, 1.0, 0.9, u.drawn[-1])["token"])
        assert got == want[-1], f"step {step}"
    assert s.prev_tokens == want[-64:]


@pytest.mark.parametrize("V", [32000, 128256])
def test_sample_with_params_matches_oracle(V):
    u = Replay(12)
    d = decoder.Decoder(V, uniform=u)
    r = np.random.Generator(np.random.PCG64(V))
    for step in range(20):
        x = (r.normal(0.0, 3.0, V) - 1.1 * np.log1p(np.arange(V))).astype(np.float32)
        T = float(r.uniform(0.5, 1.5))
        p = float(r.choice([0.5, 0.9, 0.95, 1.0]))
        got = d.sample_with_params(x, None, T, p)
        assert got == oracle.decoder_sample(x, T, p, u.drawn[-1])["token"], f"V={V} step {step}"


def test_grammar_sampler_matches_oracle():
    class Table:
        def __init__(self, rows):
            self.rows = rows
            self.i = 0

        def get_allowed_tokens(self, prev):
            ids = self.rows[self.i]
            self.i += 1
            return ids

    b = workloads.config3(0)
    V = b.logits.shape[1]
    rows = []
    for r in range(b.mask.shape[0]):
        bits = np.unpackbits(b.mask[r].view(np.uint8), bitorder="little")[:V]
        rows.append(np.flatnonzero(bits).tolist())
    rows[5] = []  # an empty allowed set: every id
    s = decoder.Sampler().with_grammar(Table(rows))
    for r in range(len(rows)):
        got = s.sample(b.logits[r])
        assert got == oracle.grammar_greedy(b.logits[r], decoder.allowed_mask(rows[r], V)), f"row {r}"
    assert len(s.prev_tokens) == decoder.PREV_TOKENS


def test_greedy_sample_last_maximum():
    d = decoder.Decoder(1000)
    x = np.zeros(1000, np.float32)
    x[[7, 300, 999]] = 5.0
    assert d.greedy_sample(x) == 999 == oracle.greedy(x)
    y = workloads.config1(3).logits[0]
    assert d.greedy_sample(y) == oracle.greedy(y)


def test_sampler_with_the_reference_grammar():
    """Sampler.with_grammar over grammar.Grammar (the reference's parser and
    state machine): each step's mask comes from the last ten tokens."""
    import grammar

    g = grammar.Grammar.from_ggnf('a ::= "xy" | [5, 7, 9]\nb ::= a | "z"\nc ::= b | "{" | [0, 1, 2]\n')
    V = 256
    rng = np.random.default_rng(21)
    s = decoder.Sampler().with_grammar(g)
    for step in range(40):
        x = rng.normal(0.0, 2.0, V).astype(np.float32)
        m = g.mask(s.prev_tokens, V)
        want = oracle.grammar_greedy(x, m)
        assert s.sample(x) == want, f"step {step}"
