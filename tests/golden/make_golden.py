"""Generates tests/golden/golden.json: small known-answer vectors for the
sampling path of chenyusolar/rust-llm (src/decoder.rs).

The reference cannot be built in this environment (no cargo/rustc) and its
tests hold no vectors for this path, so the expected outputs come from
  (a) hand-derived known answers for each documented quirk, asserted below, and
  (b) an independent pure-Python restatement of decoder.rs written with
      float32 scalars (every op rounded to f32, exp through libm's expf,
      the function Rust's f32::exp lowers to on Linux).
The C++ oracle (oracle/oracle.cpp) is checked against this file by
tests/test_oracle.py. Run:  python tests/golden/make_golden.py
"""
from __future__ import annotations

import ctypes
import ctypes.util
import json
import math
import os

import numpy as np

f32 = np.float32
_libm = ctypes.CDLL(ctypes.util.find_library("m") or "libm.so.6")
_libm.expf.restype = ctypes.c_float
_libm.expf.argtypes = [ctypes.c_float]
FLT_MIN_RUST = f32(-3.4028234663852886e38)  # f32::MIN


def expf(x):
    return f32(_libm.expf(float(x)))


def stable_sort_desc(pairs):
    # slice::sort_by is stable; key: value descending (NaN never used here).
    return sorted(pairs, key=lambda iv: -float(iv[1]))


# ---- restatement of Decoder::sample_with_params, src/decoder.rs:35-100 ----
def ref_decoder_sample(logits, temperature, top_p, r):
    l = [f32(v) for v in logits]
    T = f32(temperature)
    if T > f32(0.0):
        m = FLT_MIN_RUST
        for v in l:
            m = v if v > m else m
        l = [f32(f32(v - m) / T) for v in l]
        l = [expf(v) for v in l]
        s = f32(0.0)
        for v in l:
            s = f32(s + v)
        if s > f32(0.0):
            l = [f32(v / s) for v in l]
    cutoff = -1
    if f32(top_p) < f32(1.0):
        srt = stable_sort_desc(list(enumerate(l)))
        c = f32(0.0)
        cutoff = len(srt)
        for i, (_, p) in enumerate(srt):
            c = f32(c + p)
            if c >= f32(top_p):
                cutoff = i
                break
        l = [f32(0.0) if i > cutoff else v for i, v in enumerate(l)]
        s = f32(0.0)
        for v in l:
            s = f32(s + v)
        if s > f32(0.0):
            l = [f32(v / s) for v in l]
    c = f32(0.0)
    for i, p in enumerate(l):
        c = f32(c + p)
        if f32(r) <= c:
            return i, float(l[i]), cutoff
    best = 0
    for i in range(1, len(l)):
        if not (l[i] < l[best]):
            best = i
    return best, float(l[best]), cutoff


# ---- Decoder::greedy_sample, src/decoder.rs:160-167 (last max) ----
def ref_greedy(logits):
    best = 0
    for i in range(1, len(logits)):
        if not (f32(logits[i]) < f32(logits[best])):
            best = i
    return best


# ---- Sampler::sample_with_grammar, src/decoder.rs:359-376 ----
def ref_grammar_greedy(logits, allowed_ids):
    allowed = sorted(set(allowed_ids))
    if not allowed:
        allowed = list(range(len(logits)))
    srt = stable_sort_desc([(i, f32(logits[i])) for i in allowed])
    return srt[0][0]


# ---- spec profile (see oracle.cpp for the step list) ----
def spec_sample(logits, hist, allowed_ids, T, top_k, top_p, rp, pres, freq, u):
    x = [f32(v) for v in logits]
    V = len(x)
    counts = {}
    for h in hist:
        if 0 <= h < V:
            counts[h] = counts.get(h, 0) + 1
    for i, c in counts.items():
        v = x[i]
        x1 = f32(v * f32(rp)) if v < f32(0.0) else f32(v / f32(rp))
        x2 = f32(x1 - f32(f32(c) * f32(freq)))
        x[i] = f32(x2 - f32(pres))
    allowed = sorted(set(allowed_ids)) if allowed_ids else list(range(V))
    order = sorted(allowed, key=lambda i: (-float(x[i]), i))
    if f32(T) <= f32(0.0):
        return dict(token=order[0], prob=1.0, list=[order[0]])
    m = x[order[0]]
    e = {i: expf(f32(f32(x[i] - m) / f32(T))) for i in allowed}
    Z = math.fsum([0.0])  # keep the same left-to-right double sum as the oracle
    Z = 0.0
    for i in allowed:
        Z += float(e[i])
    K = min(top_k, len(allowed)) if top_k > 0 else len(allowed)
    L = order[:K]
    cum = []
    c = 0.0
    for i in L:
        c += float(e[i]) / Z
        cum.append(c)
    cutoff = K - 1
    if f32(top_p) < f32(1.0):
        pos = K
        for j, cv in enumerate(cum):
            if cv >= float(f32(top_p)):
                pos = j
                break
        cutoff = min(pos, K - 1)
    S = cum[cutoff]
    target = float(f32(u)) * S
    j = cutoff
    for t in range(cutoff + 1):
        if cum[t] > target:
            j = t
            break
    prob = float(f32((float(e[L[j]]) / Z) / S))
    return dict(token=L[j], prob=prob, list=L, cutoff=cutoff)


def ref_beam_step(rows, scores, done, lens, beams, alpha, eos, log_softmax):
    """One BeamSearch::search iteration (src/decoder.rs:227-265) for one item."""
    allc = []
    for b in range(beams):
        if done[b]:
            allc.append((float(f32(scores[b])), b, -1, 1))
            continue
        x = [f32(v) for v in rows[b]]
        lse = f32(0.0)
        if log_softmax:
            m = max(x)
            Z = 0.0
            for v in x:
                Z += float(expf(f32(v - m)))
            lse = f32(float(m) + math.log(Z))
        srt = sorted(range(len(x)), key=lambda i: (-float(x[i]), i))[: 2 * beams]
        lp = f32(1.0)
        if f32(alpha) != f32(1.0):
            ln = f32(lens[b] + 1)
            lp = f32(math.pow(float(f32(f32(ln + f32(6.0)) / f32(6.0))), float(alpha)))
        for i in srt:
            v = f32(x[i] - lse) if log_softmax else x[i]
            ns = f32(f32(scores[b]) + v)
            allc.append((float(f32(ns / lp)), b, i, int(i == eos)))
    allc.sort(key=lambda c: -c[0])  # stable
    return allc


def main():
    rng = np.random.default_rng(20261201)
    cases = {"decoder": [], "greedy": [], "grammar": [], "spec": [], "beam": []}

    # ---------------- hand-derived known answers ----------------
    # K1 decoder.rs:71-75 quirk: the dominant id 3 puts the sorted cutoff at
    # position 0, so every ORIGINAL id > 0 is zeroed and id 0 is returned for any r.
    t, p, cut = ref_decoder_sample([0.0, 0.0, 0.0, 10.0], 1.0, 0.9, 0.5)
    assert (t, cut, p) == (0, 0, 1.0), (t, cut, p)
    cases["decoder"].append(dict(name="cutoff_quirk_zeroes_original_ids", logits=[0.0, 0.0, 0.0, 10.0],
                                 T=1.0, top_p=0.9, r=0.5, token=0, prob=1.0, cutoff=0))
    # K2 decoder.rs:87 '<=': r = 0 returns id 0 although p_0 == 0 (expf(-200) == 0).
    t, p, cut = ref_decoder_sample([-200.0, 0.0, 0.0], 1.0, 1.0, 0.0)
    assert (t, p) == (0, 0.0)
    cases["decoder"].append(dict(name="draw_le_returns_zero_prob_id", logits=[-200.0, 0.0, 0.0],
                                 T=1.0, top_p=1.0, r=0.0, token=0, prob=0.0, cutoff=-1))
    # K3 temperature <= 0 skips the softmax: raw logits are the weights
    # (decoder.rs:44); cumsum of [0.25, 0.5, 0.25] crosses r = 0.6 at id 1.
    t, p, cut = ref_decoder_sample([0.25, 0.5, 0.25], 0.0, 1.0, 0.6)
    assert (t, p) == (1, 0.5)
    cases["decoder"].append(dict(name="nonpositive_temperature_raw_weights", logits=[0.25, 0.5, 0.25],
                                 T=0.0, top_p=1.0, r=0.6, token=1, prob=0.5, cutoff=-1))
    # K4 r beyond the total mass falls back to the LAST maximum (decoder.rs:92-97).
    t, p, cut = ref_decoder_sample([0.25, 0.25, 0.25], 0.0, 1.0, 0.9)
    assert t == 2
    cases["decoder"].append(dict(name="fallback_last_max", logits=[0.25, 0.25, 0.25], T=0.0,
                                 top_p=1.0, r=0.9, token=2, prob=0.25, cutoff=-1))
    # K5 greedy_sample keeps the LAST maximum.
    assert ref_greedy([1.0, 3.0, 3.0, 2.0]) == 2
    cases["greedy"].append(dict(name="last_max", logits=[1.0, 3.0, 3.0, 2.0], token=2))
    # K6 grammar greedy: lowest allowed id among maxima; empty set -> all ids.
    assert ref_grammar_greedy([1.0, 3.0, 3.0, 2.0], []) == 1
    cases["grammar"].append(dict(name="empty_allowed_means_all", logits=[1.0, 3.0, 3.0, 2.0],
                                 allowed=[], token=1))
    assert ref_grammar_greedy([1.0, 3.0, 3.0, 9.0], [0, 2]) == 2
    cases["grammar"].append(dict(name="masked_max_ignored", logits=[1.0, 3.0, 3.0, 9.0],
                                 allowed=[0, 2], token=2))
    # K7 spec: top_p >= 1 keeps the whole top-k list; u = 0 draws the first entry.
    r = spec_sample([1.0, 2.0, 3.0, 4.0], [], [], 1.0, 2, 1.0, 1.0, 0.0, 0.0, 0.0)
    assert r["token"] == 3 and r["cutoff"] == 1
    cases["spec"].append(dict(name="top_p_one_keeps_all_u0_first", logits=[1.0, 2.0, 3.0, 4.0], hist=[],
                              allowed=[], T=1.0, top_k=2, top_p=1.0, rp=1.0, pres=0.0, freq=0.0,
                              u=0.0, token=3, prob=r["prob"], list=[3, 2]))
    # K8 spec: repetition penalty sign rule (decoder.rs:102-110) on history ids only:
    # x=4 -> 4/2 = 2 (ties id 1's 2.0, lower id wins the order), x=-1 -> -2.
    r = spec_sample([-1.0, 2.0, 0.5, 4.0], [3, 0], [], 0.0, 0, 1.0, 2.0, 0.0, 0.0, 0.0)
    assert r["token"] == 1
    cases["spec"].append(dict(name="repeat_penalty_sign_rule_greedy", logits=[-1.0, 2.0, 0.5, 4.0],
                              hist=[3, 0], allowed=[], T=0.0, top_k=0, top_p=1.0, rp=2.0, pres=0.0,
                              freq=0.0, u=0.0, token=1, prob=1.0, list=[1]))
    # K9 spec: frequency counts repeats, presence applies once: id 2 seen 3x.
    r = spec_sample([0.0, 1.0, 3.0], [2, 2, 2], [], 0.0, 0, 1.0, 1.0, 0.5, 0.5, 0.0)
    assert r["token"] == 1  # 3 - 3*0.5 - 0.5 = 1.0 ties id 1 -> lower id 1
    cases["spec"].append(dict(name="frequency_and_presence", logits=[0.0, 1.0, 3.0], hist=[2, 2, 2],
                              allowed=[], T=0.0, top_k=0, top_p=1.0, rp=1.0, pres=0.5, freq=0.5,
                              u=0.0, token=1, prob=1.0, list=[1]))
    # K10 spec: the inclusive cutoff of sample_top_p (decoder.rs:134-136) keeps
    # the element that crosses top_p: p = [0.5, 0.3, 0.2] (top_p 0.6 keeps 2).
    lg = [math.log(0.5), math.log(0.3), math.log(0.2)]
    r = spec_sample(lg, [], [], 1.0, 0, 0.6, 1.0, 0.0, 0.0, 0.99)
    assert r["cutoff"] == 1 and r["token"] == 1
    cases["spec"].append(dict(name="inclusive_top_p_cutoff", logits=lg, hist=[], allowed=[], T=1.0,
                              top_k=0, top_p=0.6, rp=1.0, pres=0.0, freq=0.0, u=0.99, token=1,
                              prob=r["prob"], list=[0, 1, 2]))
    # K11 beam: a completed beam is carried over unchanged (decoder.rs:231-234).
    allc = ref_beam_step([[0.0] * 4, [5.0, 1.0, 0.0, 0.0]], [-0.1, -3.0], [1, 0], [3, 3], 2, 1.0, 2, 0)
    assert allc[0] == (float(f32(5.0 - 3.0)), 1, 0, 0) and allc[1] == (float(f32(-0.1)), 0, -1, 1)
    cases["beam"].append(dict(name="completed_beam_carried", rows=[[0.0] * 4, [5.0, 1.0, 0.0, 0.0]],
                              scores=[-0.1, -3.0], done=[1, 0], lens=[3, 3], beams=2, alpha=1.0,
                              eos=2, log_softmax=0, out=[list(c) for c in allc[:4]]))

    # ---------------- random vectors from the restatement ----------------
    for n in range(24):
        V = int(rng.integers(1, 70))
        x = (rng.normal(0, 3, V)).astype(np.float32)
        T = float(f32(rng.choice([0.0, 0.5, 1.0, 1.7])))
        tp = float(f32(rng.choice([0.5, 0.9, 1.0])))
        r = float(f32(rng.integers(0, 1000000) / 1e6))  # rand_secure's grid
        t, p, cut = ref_decoder_sample(x, T, tp, r)
        cases["decoder"].append(dict(name=f"rand{n}", logits=[float(v) for v in x], T=T, top_p=tp, r=r,
                                     token=t, prob=p, cutoff=cut))
    for n in range(12):
        V = int(rng.integers(1, 40))
        x = rng.integers(-3, 4, V).astype(np.float32)  # many ties
        cases["greedy"].append(dict(name=f"rand{n}", logits=[float(v) for v in x], token=ref_greedy(x)))
        allowed = [int(i) for i in np.nonzero(rng.random(V) < 0.4)[0]]
        cases["grammar"].append(dict(name=f"rand{n}", logits=[float(v) for v in x], allowed=allowed,
                                     token=ref_grammar_greedy(x, allowed)))
    for n in range(40):
        V = int(rng.integers(1, 300))
        x = (rng.normal(0, 4, V)).astype(np.float32)
        if n % 5 == 0:
            x = np.round(x).astype(np.float32)  # ties
        hist = [int(v) for v in rng.integers(-2, V + 2, int(rng.integers(0, 20)))]
        allowed = [int(i) for i in np.nonzero(rng.random(V) < 0.3)[0]] if n % 3 == 0 else []
        T = float(f32(rng.choice([0.0, 0.7, 1.0, 1.3])))
        tk = int(rng.choice([0, 1, 5, 20, 1000]))
        tp = float(f32(rng.choice([0.8, 0.95, 1.0])))
        rp = float(f32(rng.uniform(1.0, 1.3)))
        pres = float(f32(rng.uniform(0, 0.5)))
        freq = float(f32(rng.uniform(0, 0.5)))
        u = float(f32(rng.random()))
        res = spec_sample(x, hist, allowed, T, tk, tp, rp, pres, freq, u)
        cases["spec"].append(dict(name=f"rand{n}", logits=[float(v) for v in x], hist=hist,
                                  allowed=allowed, T=T, top_k=tk, top_p=tp, rp=rp, pres=pres,
                                  freq=freq, u=u, token=res["token"], prob=res["prob"],
                                  list=[int(i) for i in res["list"]]))
    for n in range(8):
        beams = int(rng.integers(1, 5))
        V = int(rng.integers(2 * beams, 40))
        rows = rng.normal(0, 3, (beams, V)).astype(np.float32)
        scores = rng.uniform(-20, 0, beams).astype(np.float32)
        done = (rng.random(beams) < 0.3).astype(int)
        lens = rng.integers(1, 10, beams)
        alpha = float(rng.choice([1.0, 0.8]))
        lsm = int(n % 2)
        allc = ref_beam_step(rows, scores, done, lens, beams, alpha, 2, lsm)
        cases["beam"].append(dict(name=f"rand{n}", rows=rows.tolist(), scores=scores.tolist(),
                                  done=done.tolist(), lens=lens.tolist(), beams=beams, alpha=alpha,
                                  eos=2, log_softmax=lsm, out=[list(c) for c in allc[: 2 * beams]]))

    out = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden.json")
    with open(out, "w") as f:
        json.dump(cases, f, indent=0)
    print("wrote", out, {k: len(v) for k, v in cases.items()})


if __name__ == "__main__":
    main()
