"""Host logic of the batched engine step (rust-llm_b200/engine.py) without a
GPU: which sequences a step samples, the per-sequence updates of
ContinuousBatchingEngine::step (src/inference.rs:117-138), and the rows of
parameters and history the batched path builds."""
import numpy as np

import engine
import rlsampler


def seqs():
    return [
        engine.SequenceState(seq_id=1, tokens=[5, 6], max_tokens=3, temperature=0.7, top_p=0.8),
        engine.SequenceState(seq_id=2, tokens=[1], max_tokens=0),                    # nothing to generate
        engine.SequenceState(seq_id=3, tokens=list(range(100)), max_tokens=5, top_k=40,
                             repeat_penalty=1.1, presence_penalty=0.2, frequency_penalty=0.3),
        engine.SequenceState(seq_id=4, tokens=[9], max_tokens=9, finished=True),
    ]


def test_live_skips_finished_and_exhausted():
    assert [s.seq_id for s in engine.live(seqs())] == [1, 3]


def test_apply_follows_the_reference_updates():
    s = seqs()
    act = engine.live(s)
    out = engine.apply(act, np.array([7, 0], np.int32))
    assert out == {1: 7, 3: 0}
    a, b = act
    assert a.tokens == [5, 6, 7] and a.generated_tokens == 1 and a.position == 1 and not a.finished
    assert b.finished and b.tokens[-1] == 0  # token 0 ends a sequence
    out = engine.apply([a, a], np.array([8, 9], np.int32))
    assert a.generated_tokens == 3 and a.finished  # max_tokens reached
    assert engine.live(s) == []


def test_rows_of_params_and_history():
    act = engine.live(seqs())
    p = engine.params_of(act)
    assert p.dtype == rlsampler.ROW_PARAMS_DTYPE
    assert p["top_k"].tolist() == [0, 40]
    assert np.allclose(p["temperature"], [0.7, 1.0]) and np.allclose(p["top_p"], [0.8, 0.9])
    assert np.allclose(p["repeat_penalty"], [1.0, 1.1]) and np.allclose(p["frequency_penalty"], [0.0, 0.3])
    h, n = engine.history_of(act)
    assert h.shape == (2, engine.HISTORY) and n.tolist() == [2, 64]
    assert h[0, :2].tolist() == [5, 6] and h[1].tolist() == list(range(36, 100))
