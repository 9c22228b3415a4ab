"""Grammar-constrained generation on the device: the GBNF masks
(rl_gbnf_mask_batch) fed to the batched sampler (rl_sample_batch), over a
32,000-token synthetic vocabulary and the JSON grammar.

Every step: each sampled token is one the grammar allows (its bit is set in
the row the sampler was given), the device tokens equal the oracle's masked
spec sampler on the same logits, masks and uniforms, and the token is then
accepted into the row's state. Sequences that reach the end token parse as
JSON.
"""
import json

import numpy as np
import pytest

import grammar
import oracle
import rlsampler
import workloads

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu


def test_json_generation_through_the_device_sampler():
    rng = np.random.default_rng(31)
    toks = workloads.json_vocab(32000)
    V = len(toks)
    eos = V - 1
    g = grammar.Gbnf(workloads.GBNF_JSON, toks, eos_id=eos)
    B, steps = 16, 40
    states = [g.new_state() for _ in range(B)]
    text = [b"" for _ in range(B)]
    done = [False] * B
    dev = "cuda:0"
    s = rlsampler.Sampler(0, max_batch=B, max_vocab=V, max_history=1)
    p = np.zeros(B, rlsampler.ROW_PARAMS_DTYPE)
    p["temperature"] = 0.8
    p["top_k"] = 50
    p["top_p"] = 0.95
    p["repeat_penalty"] = 1.0
    pd = rlsampler.params_tensor(p, dev)
    finished = 0
    for step in range(steps):
        rows, n = g.mask_batch(states)
        live = [b for b in range(B) if not done[b]]
        if not live:
            break
        assert all(n[b] > 0 for b in live)
        x = rng.normal(0.0, 3.0, (B, V)).astype(np.float32)
        x[:, eos] += 10.0 if step > 20 else 0.0  # let the complete documents end
        u = rng.random(B).astype(np.float32)
        tok, prob, st = s.sample(torch.from_numpy(x).to(dev), pd, torch.from_numpy(u).to(dev),
                                 mask=torch.from_numpy(rows.view(np.int32)).to(dev))
        tok = tok.cpu().numpy()
        assert (st.cpu().numpy() == 0).all()
        otok, _, bad = oracle.spec_sample_batch(x, None, None, rows, p, u, nthreads=8)
        assert bad == 0
        for b in live:
            t = int(tok[b])
            assert (rows[b, t >> 5] >> (t & 31)) & 1, (step, b, t)
            assert t == otok[b], (step, b, t, otok[b])
            g.accept(states[b], t)
            if t == eos:
                done[b] = True
                finished += 1
                json.loads(text[b].decode("latin-1"))  # any byte is a character of a string
            else:
                text[b] += toks[t]
    assert finished > 0
