"""Host logic of the decoder.rs mirror (rust-llm_b200/decoder.py), without a
GPU: the SamplingParams defaults, the 64-token prev_tokens ring, the
grammar's allowed-id mask, which parameters reach the device call, and the
error fallback. The device calls are replaced by a recording fake; the
tokens themselves are checked on the GPU in test_decoder_mirror_gpu.py.
"""
import numpy as np
import pytest

import decoder
import oracle
import rlsampler


class FakeHandle:
    """Stands in for the rl_sampler handle: records the calls, answers with
    fixed tokens, and fails on request."""

    def __init__(self, fail_sample=False):
        self.calls = []
        self.fail_sample = fail_sample
        self.next_token = 0

    def decoder_sample_host(self, x, t, p, u):
        self.calls.append(("decoder", x.size, float(t), float(p), float(u)))
        if self.fail_sample:
            raise rlsampler.RLError(rlsampler.RL_ERR_CUDA, "injected")
        self.next_token += 1
        return np.array([self.next_token], np.int32), np.array([0.5], np.float32)

    def greedy_host(self, x):
        self.calls.append(("greedy", x.size))
        return np.array([int(np.flatnonzero(x == x.max())[-1])], np.int32)

    def grammar_greedy_host(self, x, m):
        self.calls.append(("grammar", x.size, m.copy()))
        return np.array([oracle.grammar_greedy(x, m)], np.int32)


@pytest.fixture
def fake(monkeypatch):
    h = FakeHandle()
    monkeypatch.setattr(decoder, "_handle", lambda device, vocab: h)
    return h


def test_sampling_params_default_matches_reference():
    p = decoder.SamplingParams()
    assert (p.temperature, p.top_p, p.top_k, p.repeat_penalty) == (1.0, 0.9, 40, 1.1)
    assert (p.mirostat, p.mirostat_tau, p.mirostat_eta) == (False, 5.0, 0.1)
    assert (p.presence_penalty, p.frequency_penalty) == (0.0, 0.0)
    r = p.row()
    assert r.dtype == rlsampler.ROW_PARAMS_DTYPE and r["top_k"][0] == 40
    assert np.isclose(r["repeat_penalty"][0], 1.1)


def test_decoder_new_defaults():
    d = decoder.Decoder(32000, 4096)
    assert (d.vocab_size, d.hidden_size) == (32000, 4096)
    assert (d.temperature, d.top_p, d.top_k, d.repeat_penalty, d.last_n_tokens) == (1.0, 0.9, 40, 1.1, 64)


def test_decoder_sample_uses_fixed_temperature_and_top_p(fake):
    d = decoder.Decoder(100, uniform=lambda: 0.25)
    d.temperature, d.top_p = 0.3, 0.5  # Decoder::sample ignores the fields
    d.sample(np.zeros(100, np.float32), object())
    d.sample_with_params(np.zeros(100, np.float32), None, 0.7, 0.95)
    assert fake.calls[0] == ("decoder", 100, 1.0, pytest.approx(0.9), 0.25)
    assert fake.calls[1] == ("decoder", 100, pytest.approx(0.7), pytest.approx(0.95), 0.25)


def test_sampler_ring_keeps_last_64_tokens(fake):
    s = decoder.Sampler(decoder.SamplingParams(temperature=0.2, top_p=0.5), uniform=lambda: 0.5)
    got = [s.sample(np.zeros(50, np.float32)) for _ in range(100)]
    assert got == list(range(1, 101))
    assert s.prev_tokens == list(range(37, 101)) and len(s.prev_tokens) == decoder.PREV_TOKENS
    # no grammar: Decoder::sample, so T = 1.0 and top_p = 0.9 whatever the params say
    assert all(c[2] == 1.0 and c[3] == pytest.approx(0.9) for c in fake.calls)


def test_failed_sample_falls_back_to_device_argmax(fake):
    fake.fail_sample = True
    x = np.array([1.0, 3.0, 2.0, 3.0], np.float32)
    s = decoder.Sampler()
    assert s.sample(x) == 3  # greedy_sample: last maximum on ties
    assert [c[0] for c in fake.calls] == ["decoder", "greedy"]
    assert s.prev_tokens == [3]


class ToyGrammar:
    def __init__(self, table):
        self.table = table
        self.seen = []

    def get_allowed_tokens(self, prev):
        self.seen.append(list(prev))
        return self.table.get(len(prev), [])


def test_grammar_path_masks_and_records(fake):
    V = 70
    x = np.linspace(0.0, 1.0, V).astype(np.float32)
    g = ToyGrammar({0: [3, 5, 64], 1: [], 2: [69, 2, 2]})
    s = decoder.Sampler().with_grammar(g)
    assert s.sample(x) == 64
    assert s.sample(x) == V - 1  # empty allowed set: every id
    assert s.sample(x) == 69
    assert g.seen == [[], [64], [64, 69]]
    m0 = fake.calls[0][2]
    assert m0.shape == ((V + 31) // 32,) and m0[0] == (1 << 3) | (1 << 5) and m0[2] == 1
    assert not fake.calls[1][2].any()


def test_allowed_mask_drops_out_of_range_ids():
    m = decoder.allowed_mask([0, 31, 32, 99, -1, 100], 100)
    assert m.tolist() == [1 | (1 << 31), 1, 0, 1 << 3]
