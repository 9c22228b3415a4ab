"""rl_greedy (Decoder::greedy_sample, last maximum) and rl_grammar_greedy
(Sampler::sample_with_grammar, lowest allowed id among the maxima, empty
allowed set = all ids) against the oracle, bit-exact."""
import numpy as np
import pytest

import oracle
import rlsampler
import workloads

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def sampler():
    s = rlsampler.Sampler(0, max_batch=512, max_vocab=262144, max_history=16)
    yield s
    s.close()


def _run(s, x, mask=None):
    L = rlsampler.lib()
    dev = "cuda:0"
    xt = torch.from_numpy(x).to(dev)
    out = torch.empty(x.shape[0], dtype=torch.int32, device=dev)
    st = torch.cuda.current_stream().cuda_stream
    if mask is None:
        rlsampler.check(L.rl_greedy(s.h, rlsampler._ptr(xt), x.shape[0], x.shape[1], x.shape[1],
                                    rlsampler._ptr(out), st), "rl_greedy")
    else:
        mt = torch.from_numpy(mask.view(np.int32)).to(dev)
        rlsampler.check(L.rl_grammar_greedy(s.h, rlsampler._ptr(xt), x.shape[0], x.shape[1], x.shape[1],
                                            rlsampler._ptr(mt), mask.shape[1], rlsampler._ptr(out), st),
                        "rl_grammar_greedy")
    torch.cuda.synchronize()
    return out.cpu().numpy()


@pytest.mark.parametrize("V", [1, 3, 31, 32, 33, 1000, 32000, 151936])
def test_greedy_last_max(sampler, V):
    rng = np.random.default_rng(V)
    x = rng.integers(-5, 6, (16, V)).astype(np.float32)  # many ties
    got = _run(sampler, x)
    want = [oracle.greedy(x[b]) for b in range(16)]
    assert list(got) == want


@pytest.mark.parametrize("V", [5, 64, 1000, 32000])
def test_grammar_greedy_lowest_allowed(sampler, V):
    rng = np.random.default_rng(V + 1)
    B = 16
    x = rng.integers(-5, 6, (B, V)).astype(np.float32)
    allowed = [np.nonzero(rng.random(V) < d)[0] for d in np.linspace(0.0, 0.6, B)]
    allowed[0] = np.array([], np.int64)  # empty -> all ids
    mask = workloads.mask_from_allowed(V, allowed)
    got = _run(sampler, x, mask)
    want = [oracle.grammar_greedy(x[b], mask[b]) for b in range(B)]
    assert list(got) == want


def test_grammar_greedy_config3(sampler):
    b = workloads.config3(0)
    got = _run(sampler, b.logits, b.mask)
    want = [oracle.grammar_greedy(b.logits[i], b.mask[i]) for i in range(b.logits.shape[0])]
    assert list(got) == want


def test_signed_zero_ties(sampler):
    """-0.0 and +0.0 tie (Rust's partial_cmp); greedy keeps the last of them,
    the grammar path the lowest allowed id."""
    V = 4099
    rng = np.random.default_rng(99)
    x = -np.abs(rng.normal(1.0, 1.0, (8, V))).astype(np.float32) - np.float32(0.5)
    for b in range(8):
        pos = rng.choice(V, 6, replace=False)
        x[b, pos[:3]] = np.float32(0.0)
        x[b, pos[3:]] = np.float32(-0.0)
    got = _run(sampler, x)
    assert list(got) == [oracle.greedy(x[b]) for b in range(8)]
    mask = workloads.mask_from_allowed(V, [np.arange(V)] * 8)
    got = _run(sampler, x, mask)
    assert list(got) == [oracle.grammar_greedy(x[b], mask[b]) for b in range(8)]
