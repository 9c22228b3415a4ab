"""The batched engine step (rust-llm_b200/engine.py) on the device, over many
steps of a changing set of sequences, against the reference's per-sequence
loop (src/inference.rs:112-138) run with the oracle on the same logits and
uniforms: the ref_exact step token for token, the spec step within the
boundary tolerance."""
import numpy as np
import pytest

import engine
import oracle

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

V = 32000


def make_states(rng, n):
    out = []
    for i in range(n):
        out.append(engine.SequenceState(seq_id=100 + i, tokens=[int(t) for t in rng.integers(1, V, 3)],
                                        max_tokens=int(rng.integers(1, 12)),
                                        temperature=float(rng.choice([0.0, 0.7, 1.0, 1.3])),
                                        top_p=float(rng.choice([0.5, 0.9, 1.0])),
                                        top_k=int(rng.choice([0, 40])), repeat_penalty=1.1,
                                        presence_penalty=0.1, frequency_penalty=0.2))
    return out


def run(semantics):
    rng = np.random.default_rng(5 if semantics == "ref_exact" else 6)
    ours = make_states(rng, 24)
    ref = [engine.SequenceState(**vars(s)) for s in ours]
    for s in ref:
        s.tokens = list(s.tokens)
    eng = engine.BatchStep(V, max_batch=64, semantics=semantics)
    steps = boundary = 0
    try:
        while engine.live(ours):
            act = engine.live(ours)
            x = (rng.normal(0.0, 3.0, (len(act), V)) - 1.1 * np.log1p(np.arange(V))).astype(np.float32)
            x[:, 0] -= 30.0  # token 0 (end of sequence) is rare
            u = (rng.random(len(act)) * (1 - 2 ** -24)).astype(np.float32)
            got = eng.step(ours, torch.from_numpy(x).to("cuda:0"), uniforms=u)
            ract = engine.live(ref)
            want = []
            for i, s in enumerate(ract):
                if semantics == "ref_exact":
                    want.append(oracle.decoder_sample(x[i], s.temperature, s.top_p, u[i])["token"])
                else:
                    prm = {k: v for k, v in zip(("temperature", "top_p", "top_k", "repeat_penalty",
                                                 "presence_penalty", "frequency_penalty"),
                                                engine.params_of([s])[0].tolist())}
                    r = oracle.spec_sample_row(x[i], np.array(s.tokens[-engine.HISTORY:], np.int32), None, prm, u[i])
                    if got[s.seq_id] != r.token:
                        assert min(r.draw_margin, r.cut_margin) < 1e-6, f"seq {s.seq_id}"
                        boundary += 1
                        want.append(got[s.seq_id])  # keep both histories equal
                        continue
                    want.append(r.token)
            engine.apply(ract, np.array(want, np.int32))
            assert got == {s.seq_id: s.tokens[-1] for s in ract}
            steps += 1
        assert all(a.tokens == b.tokens and a.finished == b.finished for a, b in zip(ours, ref))
        assert steps > 3
    finally:
        eng.close()
    return boundary


def test_engine_step_ref_exact_matches_the_reference_loop():
    assert run("ref_exact") == 0


def test_engine_step_spec_matches_the_oracle():
    assert run("spec") <= 2
