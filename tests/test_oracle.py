"""The CPU oracle against the golden vectors (hand-derived known answers and
an independent pure-Python restatement of src/decoder.rs)."""
import json
import os

import numpy as np
import pytest

import oracle

GOLD = json.load(open(os.path.join(os.path.dirname(__file__), "golden", "golden.json")))


def _mask_from_allowed(V, allowed):
    m = np.zeros((V + 31) // 32, np.uint32)
    for i in allowed:
        m[i >> 5] |= np.uint32(1 << (i & 31))
    return m


@pytest.mark.parametrize("case", GOLD["decoder"], ids=lambda c: c["name"])
def test_decoder_sample_golden(case):
    r = oracle.decoder_sample(np.array(case["logits"], np.float32), case["T"], case["top_p"], case["r"])
    assert r["token"] == case["token"]
    assert r["prob"] == np.float32(case["prob"])
    assert r["cutoff"] == case["cutoff"]


@pytest.mark.parametrize("case", GOLD["greedy"], ids=lambda c: c["name"])
def test_greedy_golden(case):
    assert oracle.greedy(np.array(case["logits"], np.float32)) == case["token"]


@pytest.mark.parametrize("case", GOLD["grammar"], ids=lambda c: c["name"])
def test_grammar_golden(case):
    x = np.array(case["logits"], np.float32)
    assert oracle.grammar_greedy(x, _mask_from_allowed(x.size, case["allowed"])) == case["token"]


@pytest.mark.parametrize("case", GOLD["spec"], ids=lambda c: c["name"])
def test_spec_golden(case):
    x = np.array(case["logits"], np.float32)
    mask = _mask_from_allowed(x.size, case["allowed"]) if case["allowed"] else None
    prm = dict(temperature=case["T"], top_p=case["top_p"], top_k=case["top_k"],
               repeat_penalty=case["rp"], presence_penalty=case["pres"],
               frequency_penalty=case["freq"])
    r = oracle.spec_sample_row(x, np.array(case["hist"], np.int32), mask, prm, case["u"], list_cap=4096)
    assert r.status == 0
    assert r.token == case["token"]
    assert r.prob == np.float32(case["prob"])
    assert list(r.list_ids) == case["list"]


@pytest.mark.parametrize("case", GOLD["beam"], ids=lambda c: c["name"])
def test_beam_golden(case):
    beams = case["beams"]
    rows = np.array(case["rows"], np.float32)
    n_out = len(case["out"])
    ob, ot, os_, od = oracle.beam_step(rows, 1, beams, case["scores"], case["done"], case["lens"],
                                       case["alpha"], case["eos"], case["log_softmax"], n_out)
    got = [[float(os_[0, j]), int(ob[0, j]), int(ot[0, j]), int(od[0, j])] for j in range(n_out)]
    assert got == [[float(np.float32(c[0])), c[1], c[2], c[3]] for c in case["out"]]


def test_spec_batch_matches_rows():
    rng = np.random.default_rng(3)
    B, V = 6, 500
    x = rng.normal(0, 4, (B, V)).astype(np.float32)
    hist = rng.integers(0, V, (B, 16)).astype(np.int32)
    hl = np.full(B, 16, np.int32)
    prm = np.zeros(B, oracle.ROW_PARAMS_DTYPE)
    prm["temperature"] = 0.9
    prm["top_p"] = 0.9
    prm["top_k"] = [0, 5, 50, 0, 1, 10]
    prm["repeat_penalty"] = 1.2
    prm["presence_penalty"] = 0.1
    prm["frequency_penalty"] = 0.2
    u = rng.random(B).astype(np.float32)
    tok, prob, bad = oracle.spec_sample_batch(x, hist, hl, None, prm, u, nthreads=3)
    assert bad == 0
    for b in range(B):
        r = oracle.spec_sample_row(x[b], hist[b], None, {k: prm[b][k].item() for k in prm.dtype.names}, u[b])
        assert r.token == tok[b] and r.prob == prob[b]


def test_spec_nonfinite_rejected():
    x = np.array([0.0, np.nan, 1.0], np.float32)
    prm = dict(temperature=1.0, top_p=1.0, top_k=0, repeat_penalty=1.0, presence_penalty=0.0,
               frequency_penalty=0.0)
    assert oracle.spec_sample_row(x, None, None, prm, 0.5).status == 1
    x = np.full(3, -np.inf, np.float32)
    assert oracle.spec_sample_row(x, None, None, prm, 0.5).status == 1
