"""Speculative decoding on the device (rl_specdec_sample, rl_specdec_verify)
against the oracle's restatement of SpeculativeDecoder (src/inference.rs:
335-429), token for token on the same uniforms.

Rows: seeded N(0, 3^2) logits with the shapes of the sampler workloads, plus
the edge cases the reference's code has: ties (rounded logits), -inf
entries, all -inf rows, offsets at and past the end, temperatures <= 0 and
NaN, uniforms 0 and just below 1, drafts with probability 0 (exp underflow),
out-of-range and negative draft ids, no room for a bonus token.
"""
import numpy as np
import pytest

import oracle
import rlsampler

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

DEV = "cuda:0"


def _rows(rng, B, V):
    x = rng.normal(0.0, 3.0, (B, V)).astype(np.float32)
    x[1] = np.round(x[1])  # many ties
    x[2, rng.choice(V, V // 3, replace=False)] = -np.inf
    x[3] = -np.inf  # every adjusted value -inf
    x[4] = np.round(x[4] * 4) / 4
    return x


@pytest.fixture(scope="module")
def sampler():
    s = rlsampler.Sampler(0, max_batch=256, max_vocab=1 << 18, max_history=0)
    yield s
    s.close()


@pytest.mark.parametrize("V", [7, 32000, 151936])
def test_specdec_sample_matches_oracle(sampler, V):
    rng = np.random.default_rng(V)
    B = 64
    x = _rows(rng, B, V)
    T = rng.choice(np.array([0.8, 1.0, 1.0, 0.5, 2.0, 0.0, -1.0], np.float32), B)
    T[5] = np.nan
    off = rng.choice(np.array([0, 1, 1, 4, 5], np.int32), B)
    off[6], off[7], off[8] = V - 1, V, V + 3
    T[7] = 0.0
    u = (rng.random(B) * (1 - 2 ** -24)).astype(np.float32)
    u[9], u[10] = 0.0, np.nextafter(np.float32(1), np.float32(0))
    got = sampler.specdec_sample(torch.from_numpy(x).to(DEV), torch.from_numpy(T).to(DEV),
                                 torch.from_numpy(off).to(DEV), torch.from_numpy(u).to(DEV)).cpu().numpy()
    for b in range(B):
        want = oracle.specdec_sample(x[b], T[b], off[b], u[b])
        assert got[b] == want, f"V={V} row {b}: T={T[b]} offset={off[b]} u={u[b]}: {got[b]} vs {want}"


def test_specdec_sample_draft_and_target_settings(sampler):
    """The reference's own calls: draft draws (T 0.8, offset 1) and target
    draws (T 1.0, offset = drafts) over many rows and uniforms."""
    rng = np.random.default_rng(3)
    B, V = 256, 32000
    x = (rng.normal(0.0, 3.0, (B, V)) - 1.1 * np.log1p(np.arange(V))).astype(np.float32)
    xd = torch.from_numpy(x).to(DEV)
    for T, off in ((0.8, 1), (1.0, 4)):
        u = (rng.random(B) * (1 - 2 ** -24)).astype(np.float32)
        got = sampler.specdec_sample(xd, torch.full((B,), T, device=DEV), torch.full((B,), off, dtype=torch.int32,
                                                                                   device=DEV),
                                     torch.from_numpy(u).to(DEV)).cpu().numpy()
        want = np.array([oracle.specdec_sample(x[b], T, off, u[b]) for b in range(B)])
        assert np.array_equal(got, want), np.flatnonzero(got != want)


def test_specdec_sample_nonfinite_rows_report_minus_one(sampler):
    x = np.zeros((2, 100), np.float32)
    x[0, 5] = np.nan
    x[1, 7] = np.inf
    got = sampler.specdec_sample(torch.from_numpy(x).to(DEV), torch.ones(2, device=DEV),
                                 torch.zeros(2, dtype=torch.int32, device=DEV), torch.full((2,), 0.5, device=DEV))
    assert got.cpu().tolist() == [-1, -1]


@pytest.mark.parametrize("V", [32000, 128256])
def test_specdec_verify_matches_oracle(sampler, V):
    rng = np.random.default_rng(100 + V)
    B, Dmax = 96, 8
    x = _rows(rng, B, V)
    drafts = np.zeros((B, Dmax), np.int32)
    nd = rng.integers(1, Dmax + 1, B).astype(np.int32)
    for b in range(B):
        order = np.argsort(-x[b], kind="stable")
        drafts[b] = order[rng.integers(0, 50, Dmax)]  # likely tokens
        if b % 5 == 1:  # a draft of probability 0 (exp underflows)
            j = rng.integers(0, nd[b])
            x[b, drafts[b, j]] = -1e30
        if b % 7 == 2:
            drafts[b, rng.integers(0, nd[b])] = V + 5  # outside the row
        if b % 11 == 3:
            drafts[b, 0] = -3
    x[3] = -np.inf
    x[3, 17] = 0.0  # one finite logit
    acc_u = (rng.random((B, Dmax)) * (1 - 2 ** -24)).astype(np.float32)
    acc_u[0] = np.nextafter(np.float32(1), np.float32(0))
    room = rng.integers(0, 2, B).astype(np.int32)
    draw_u = (rng.random(B) * (1 - 2 ** -24)).astype(np.float32)
    acc, tok = sampler.specdec_verify(torch.from_numpy(x).to(DEV), torch.from_numpy(drafts).to(DEV),
                                      torch.from_numpy(nd).to(DEV), torch.from_numpy(acc_u).to(DEV),
                                      torch.from_numpy(room).to(DEV), torch.from_numpy(draw_u).to(DEV))
    acc, tok = acc.cpu().numpy(), tok.cpu().numpy()
    kinds = {"all": 0, "none": 0, "partial": 0, "token": 0}
    for b in range(B):
        wa, wt = oracle.specdec_verify(x[b], drafts[b, : nd[b]], acc_u[b, : nd[b]], room[b], draw_u[b])
        assert (acc[b], tok[b]) == (wa, wt), f"V={V} request {b}: ({acc[b]}, {tok[b]}) vs ({wa}, {wt})"
        kinds["all" if wa == nd[b] else "none" if wa == 0 else "partial"] += 1
        kinds["token"] += wt >= 0
    # the cases the reference distinguishes all occur
    assert min(kinds.values()) > 0, kinds


def test_specdec_verify_bad_requests(sampler):
    x = np.zeros((3, 50), np.float32)
    x[1, 3] = np.nan
    drafts = np.ones((3, 4), np.int32)
    nd = np.array([0, 2, 5], np.int32)  # empty draft; NaN row; more drafts than the stride
    z = torch.zeros((3, 4), device=DEV)
    acc, tok = sampler.specdec_verify(torch.from_numpy(x).to(DEV), torch.from_numpy(drafts).to(DEV),
                                      torch.from_numpy(nd).to(DEV), z, torch.ones(3, dtype=torch.int32, device=DEV),
                                      torch.zeros(3, device=DEV))
    assert acc.cpu().tolist() == [-1, -1, -1] and tok.cpu().tolist() == [-1, -1, -1]
