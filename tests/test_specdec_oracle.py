"""Known answers for the oracle's restatement of SpeculativeDecoder's sampling
(src/inference.rs:335-429), derived by hand from the reference's code; they
pin the restatement that the device kernels are compared with."""
import numpy as np

import oracle


def f32(*v):
    return np.array(v, np.float32)


def test_sample_argmax_branch():
    # temperature <= 0: Iterator::max_by over the ids >= offset, the LAST maximum
    assert oracle.specdec_sample(f32(0, 1, 2, 3), 0.0, 0, 0.5) == 3
    assert oracle.specdec_sample(f32(1, 5, 5, 2), 0.0, 0, 0.5) == 2
    assert oracle.specdec_sample(f32(1, 5, 5, 2), -1.0, 3, 0.5) == 3
    assert oracle.specdec_sample(f32(0.0, -0.0), 0.0, 0, 0.5) == 1  # -0 == +0: the later one
    assert oracle.specdec_sample(f32(1, 2), 0.0, 2, 0.5) == 0  # nothing left: unwrap_or(0)
    assert oracle.specdec_sample(f32(1, np.nan), 0.0, 0, 0.5) == -1  # partial_cmp(..).unwrap() panics


def test_sample_draw_branch():
    # T = 1 over two equal logits: p = [0.5, 0.5]; the first id with r <= cumsum
    x = f32(0, 0)
    assert oracle.specdec_sample(x, 1.0, 0, 0.0) == 0
    assert oracle.specdec_sample(x, 1.0, 0, 0.5) == 0
    assert oracle.specdec_sample(x, 1.0, 0, float(np.nextafter(np.float32(0.5), np.float32(1)))) == 1
    assert oracle.specdec_sample(x, 1.0, 0, 1.0) == 1
    # the offset skips ids and is added back; an empty range falls to V - 1
    assert oracle.specdec_sample(f32(9, 0, 0), 1.0, 1, 0.0) == 1
    assert oracle.specdec_sample(f32(9, 0, 0), 1.0, 3, 0.0) == 2
    # a row whose adjusted values are all -inf: sum 0, not divided; r = 0 takes the first id
    ninf = -np.inf
    assert oracle.specdec_sample(f32(ninf, ninf), 1.0, 0, 0.0) == 0
    assert oracle.specdec_sample(f32(ninf, ninf), 1.0, 0, 0.25) == 1  # falls through to V - 1


def test_softmax_at():
    assert oracle.specdec_softmax_at(f32(0, 0, 0), 1) == np.float32(1.0) / np.float32(3.0)
    assert oracle.specdec_softmax_at(f32(0, 0, 0), 3) == 0.0  # outside the row
    assert oracle.specdec_softmax_at(f32(0, 0, 0), -1) == 0.0  # a negative Token as usize
    assert oracle.specdec_softmax_at(f32(0, -200), 1) == 0.0  # exp(-200) underflows in f32


def test_verify_and_accept():
    x = f32(0, -200, 5, 0)
    # draft 1 has probability 0: one accepted, no draw
    assert oracle.specdec_verify(x, [2, 1], [0.0, 0.0], 1, 0.5) == (1, -1)
    # none accepted: generate's fallback draw sample(x, 1.0, 1) over [-200, 5, 0] -> id 2
    assert oracle.specdec_verify(x, [1], [0.0], 1, 0.5) == (0, 2)
    assert oracle.specdec_verify(x, [-1], [0.0], 0, 0.5) == (0, 2)
    assert oracle.specdec_verify(x, [4], [0.0], 0, 0.5) == (0, 2)
    # all accepted, room left: the bonus draw sample(x, 1.0, 2) over [5, 0] -> id 2
    assert oracle.specdec_verify(x, [2, 3], [0.9999, 0.5], 1, 0.1) == (2, 2)
    # ... not kept when it repeats the last draft, nor without room
    assert oracle.specdec_verify(x, [3, 2], [0.0, 0.0], 1, 0.1) == (2, -1)
    assert oracle.specdec_verify(x, [2, 3], [0.0, 0.0], 0, 0.1) == (2, -1)
    # a drawn token 0 is not kept (token > 0 only): V = 1, the bonus draw has
    # no ids past the offset and falls to V - 1 = 0
    assert oracle.specdec_verify(f32(7), [0], [0.0], 1, 0.5) == (1, -1)
    # a rejected first draft whose fallback draw lands past it
    assert oracle.specdec_verify(f32(7, -300), [1], [0.0], 1, 0.5) == (0, 1)
