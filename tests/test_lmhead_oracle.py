"""orc_matmul_vec, the oracle's restatement of Model::matmul_vec
(src/model.rs:246-261), against known answers and a float64 product:
sequential f32 sums, the weight-length guard and the min(hidden, len/vocab)
bound of the reference's loop."""
import numpy as np

import oracle


def test_known_answers():
    x = np.array([1.0, 2.0, 3.0], np.float32)
    w = np.array([[1, 0, 0], [0, 1, 0], [1, 1, 1], [0.5, -0.5, 2.0]], np.float32)
    assert oracle.matmul_vec(x, w)[0].tolist() == [1.0, 2.0, 6.0, 5.5]


def test_sequential_f32_sum_order():
    # 1e8 + 1 - 1e8 in f32, left to right: the 1 is lost at the first add
    x = np.array([1.0, 1.0, 1.0], np.float32)
    w = np.array([[1e8, 1.0, -1e8]], np.float32)
    assert oracle.matmul_vec(x, w)[0, 0] == 0.0


def test_close_to_float64_and_threads_agree():
    r = np.random.default_rng(3)
    x = r.normal(size=(6, 256)).astype(np.float32)
    w = r.normal(size=(500, 256)).astype(np.float32) / 16
    a = oracle.matmul_vec(x, w, nthreads=1)
    b = oracle.matmul_vec(x, w, nthreads=4)
    assert np.array_equal(a, b)
    ref = x.astype(np.float64) @ w.astype(np.float64).T
    bound = 256 * 2.0 ** -24 * (np.abs(x).astype(np.float64) @ np.abs(w).astype(np.float64).T)
    assert (np.abs(a - ref) <= bound).all()
