"""Parity of the CUDA spec sampler (rl_sample_batch_debug, through the C ABI)
with the CPU oracle on identical seeded inputs.

Bar: status equal; top-k id lists bit-exact; the kept set of every row bit
exact (the list size K, the position of the last kept entry in (logit desc,
id asc) order and that entry's id); probabilities within 1e-5 relative;
sampled tokens identical except where the oracle reports the draw (or the
top-p cutoff) within 1e-6 of a CDF boundary -- those are counted (see
conftest.PARITY) and reported, not failed.
"""
import concurrent.futures as cf
import os

import numpy as np
import pytest

import oracle
import rlsampler
import workloads
from conftest import parity_add

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

PROB_RTOL = 1e-5
BOUNDARY = 1e-6
NTHREADS = max(1, min(32, os.cpu_count() or 1))
PARITY_STEPS = int(os.environ.get("RL_PARITY_STEPS", "20"))


@pytest.fixture(scope="module")
def sampler():
    s = rlsampler.Sampler(0, max_batch=1024, max_vocab=262144, max_history=1024)
    yield s
    s.close()


def run_gpu(s, batch, list_cap=1024, bf16=False):
    dev = "cuda:0"
    if bf16:
        lg = torch.from_numpy(batch.bf16_bits.view(np.int16)).to(dev).view(torch.bfloat16)
    else:
        lg = torch.from_numpy(batch.logits).to(dev)
    p = rlsampler.params_tensor(batch.params, dev)
    u = torch.from_numpy(batch.uniforms).to(dev)
    hist = torch.from_numpy(batch.hist).to(dev) if batch.hist is not None else None
    hl = torch.from_numpy(batch.hist_len).to(dev) if batch.hist_len is not None else None
    mask = torch.from_numpy(batch.mask.view(np.int32)).to(dev) if batch.mask is not None else None
    out = s.sample_debug(lg, p, u, hist, hl, mask, list_cap=list_cap)
    torch.cuda.synchronize()
    return [t.cpu().numpy() for t in out]


def oracle_rows(batch, list_cap):
    """The oracle on every row, rows spread over host threads (the ctypes
    call releases the GIL)."""
    B = batch.logits.shape[0]

    def one(b):
        prm = {k: batch.params[b][k].item() for k in batch.params.dtype.names}
        h = batch.hist[b][: batch.hist_len[b]] if batch.hist is not None else None
        m = batch.mask[b] if batch.mask is not None else None
        return oracle.spec_sample_row(batch.logits[b], h, m, prm, batch.uniforms[b], list_cap=list_cap)

    with cf.ThreadPoolExecutor(NTHREADS) as ex:
        return list(ex.map(one, range(B)))


def compare(batch, gpu, list_cap=1024, label="", key=None):
    tok, prob, st, lids, lps, llen, cut = gpu
    refs = oracle_rows(batch, list_cap)
    n = dict(rows=0, tokens_equal=0, boundary=0, kept_set_checked=0, cut_boundary=0, lists_checked=0,
             prob_on_cut_boundary=0)
    for b, r in enumerate(refs):
        exp_st = 0 if r.status == 0 else rlsampler.RL_ERR_NONFINITE
        assert st[b] == exp_st, f"{label} row {b}: status {st[b]} vs {exp_st}"
        n["rows"] += 1
        if r.status:
            continue
        # the kept set: K, the last kept position and its id
        assert cut[b, 0] == r.K, f"{label} row {b}: K {cut[b, 0]} vs {r.K}"
        if r.cut_margin < BOUNDARY:
            n["cut_boundary"] += 1
        else:
            assert cut[b, 1] == r.cutoff, f"{label} row {b}: cutoff position {cut[b, 1]} vs {r.cutoff}"
            if cut[b, 2] != -2:
                assert cut[b, 2] == r.cut_id, f"{label} row {b}: cutoff id {cut[b, 2]} vs {r.cut_id}"
            n["kept_set_checked"] += 1
        m = llen[b]
        if m >= 0:
            want = min(r.K, list_cap)
            assert m == want, f"{label} row {b}: list length {m} vs {want}"
            assert np.array_equal(lids[b, :m], r.list_ids[:m]), f"{label} row {b}: top-k ids differ"
            np.testing.assert_allclose(lps[b, :m], r.list_p[:m], rtol=PROB_RTOL, atol=1e-30,
                                       err_msg=f"{label} row {b}: list probabilities")
            n["lists_checked"] += 1
        if tok[b] != r.token:
            near = min(r.draw_margin, r.cut_margin) < BOUNDARY
            assert near, (f"{label} row {b}: token {tok[b]} vs oracle {r.token} "
                          f"(draw margin {r.draw_margin:.3g}, cut margin {r.cut_margin:.3g})")
            n["boundary"] += 1
            continue
        n["tokens_equal"] += 1
        if r.cut_margin < BOUNDARY and abs(prob[b] - r.prob) > PROB_RTOL * abs(r.prob):
            # same token, but the cutoff (and so the renormalising mass) sits
            # on a CDF boundary
            n["prob_on_cut_boundary"] = n.get("prob_on_cut_boundary", 0) + 1
            continue
        np.testing.assert_allclose(prob[b], r.prob, rtol=PROB_RTOL, err_msg=f"{label} row {b}: prob")
    parity_add(key or label, **n)
    return n["boundary"]


def make_batch(rng, B, V, T, top_k, top_p, hist_len=0, mask_density=None, rp=1.1, pres=0.2, freq=0.3,
               scale=3.0, ties=False):
    x = rng.normal(0, scale, (B, V)).astype(np.float32)
    if ties:
        x = np.round(x).astype(np.float32)
    p = np.zeros(B, rlsampler.ROW_PARAMS_DTYPE)
    p["temperature"] = T
    p["top_k"] = top_k
    p["top_p"] = top_p
    p["repeat_penalty"] = rp
    p["presence_penalty"] = pres
    p["frequency_penalty"] = freq
    u = rng.random(B).astype(np.float32)
    hist = hl = None
    if hist_len:
        hist = rng.integers(-3, V + 3, (B, hist_len)).astype(np.int32)
        hist[:, : hist_len // 4] = rng.integers(0, min(V, 8), (B, hist_len // 4))  # repeats
        hl = rng.integers(0, hist_len + 1, B).astype(np.int32)
    mask = None
    if mask_density is not None:
        allowed = [np.nonzero(rng.random(V) < mask_density)[0] for _ in range(B)]
        mask = workloads.mask_from_allowed(V, allowed)
    return workloads.SampleBatch(x, p, u, hist, hl, mask)


SMALL = [
    # B, V, T, top_k, top_p, hist, mask_density, ties
    (4, 1, 1.0, 0, 1.0, 0, None, False),
    (4, 2, 0.7, 0, 0.9, 3, None, False),
    (8, 7, 1.0, 3, 0.5, 4, None, True),
    (8, 100, 0.5, 0, 0.95, 16, 0.3, False),
    (8, 1000, 1.3, 50, 0.9, 64, None, False),
    (8, 1000, 0.0, 0, 1.0, 64, None, True),      # greedy, ties -> lowest id
    (8, 5000, 1.0, 1, 0.9, 32, None, False),
    (8, 5000, 1.0, 6000, 1.0, 32, 0.05, False),  # k > V
    (6, 32000, 1.0, 40, 0.9, 64, None, False),
    (6, 32000, 0.7, 0, 0.95, 0, 0.1, False),
    (6, 32000, 1.5, 0, 1.0, 0, None, False),      # full-vocabulary draw
    (4, 32001, 0.9, 100, 0.8, 128, 0.5, False),   # V not a multiple of 4
    (4, 2048, 1.0, 20, 0.99, 0, None, True),
]


@pytest.mark.parametrize("case", SMALL, ids=lambda c: f"B{c[0]}_V{c[1]}_T{c[2]}_k{c[3]}_p{c[4]}")
def test_small_shapes(sampler, case):
    B, V, T, k, tp, hl, md, ties = case
    rng = np.random.default_rng(hash(case) & 0xFFFFFFFF)
    batch = make_batch(rng, B, V, T, k, tp, hl, md, ties=ties)
    compare(batch, run_gpu(sampler, batch), label=str(case), key="small_shapes")


BIG_K = [
    # B, V, T, top_k, top_p, hist, mask_density: top-k lists longer than the
    # kernel's 128-key list (kept set compared through the cutoff export),
    # and masked rows whose allowed set exceeds 128 with top_k off
    (4, 32000, 1.0, 129, 1.0, 64, None),
    (4, 32000, 0.8, 500, 1.0, 64, None),
    (4, 128256, 1.2, 1000, 1.0, 256, None),
    (4, 32000, 1.1, 300, 0.97, 0, None),
    (4, 32000, 0.9, 0, 1.0, 0, 0.02),
    (4, 32000, 1.3, 0, 0.95, 64, 0.05),
    (4, 32000, 1.0, 200, 0.9, 0, 0.2),
]


@pytest.mark.parametrize("case", BIG_K, ids=lambda c: f"B{c[0]}_V{c[1]}_k{c[3]}_p{c[4]}_m{c[6]}")
def test_big_k_and_masked_sets(sampler, case):
    B, V, T, k, tp, hl, md = case
    rng = np.random.default_rng(hash(case) & 0xFFFFFFFF)
    batch = make_batch(rng, B, V, T, k, tp, hl, md)
    compare(batch, run_gpu(sampler, batch), label=str(case), key="big_k_and_masked")


DEEP = [
    # B, V, T, top_k, top_p, hist, scale, ties: full-vocabulary rows whose
    # top-p cutoff lies far below the top-128 list (streamed histogram, one
    # bin re-read with the draw bin predicted), a 1024-id history whose
    # repeats overflow an id range of the counting sort, and rounded logits
    # whose bins overflow the collect (exact radix walk)
    (4, 128256, 1.3, 0, 0.9, 1024, 2.0, False),
    (4, 128256, 0.8, 0, 0.97, 256, 3.0, False),
    (3, 128256, 1.0, 0, 0.9, 64, 1.0, True),
    (3, 128256, 1.0, 0, 1.0, 0, 2.0, False),
    # flat rows (Gaussian logits, no prior, high temperature): the cutoff and
    # draw bins overflow the collect buffer together but not alone (T 1.5),
    # or a bin alone overflows it and is split into sub-ranges by one more
    # re-read (T 2 and 3; with top_k beyond the list, counts too)
    (4, 128256, 1.5, 0, 0.95, 0, 3.0, False),
    (4, 128256, 2.0, 0, 0.9, 64, 3.0, False),
    (4, 128256, 3.0, 0, 0.5, 0, 3.0, False),
    (3, 128256, 3.0, 0, 0.99, 256, 3.0, False),
    (3, 128256, 2.5, 2000, 0.95, 0, 3.0, False),
]


@pytest.mark.parametrize("case", DEEP, ids=lambda c: f"B{c[0]}_V{c[1]}_T{c[2]}_p{c[4]}_h{c[5]}_ties{int(c[7])}")
def test_deep_top_p_rows(sampler, case):
    B, V, T, k, tp, hl, scale, ties = case
    rng = np.random.default_rng(hash(case) & 0xFFFFFFFF)
    batch = make_batch(rng, B, V, T, k, tp, hl, None, scale=scale, ties=ties)
    compare(batch, run_gpu(sampler, batch), label=str(case), key="deep_top_p")


def test_config2_full_batches(sampler):
    """Every row of the heterogeneous batch (B=256 x V=128256) over
    PARITY_STEPS regenerated steps."""
    total = 0
    for step in range(PARITY_STEPS):
        batch = workloads.config2(step)
        total += compare(batch, run_gpu(sampler, batch), label=f"config2 step {step}", key="config2")
    print(f"config2: {total} boundary cases over {PARITY_STEPS} steps")


def test_config3_full(sampler):
    for step in range(PARITY_STEPS):
        batch = workloads.config3(step)
        compare(batch, run_gpu(sampler, batch), label=f"config3 step {step}", key="config3")


def test_config1_spec(sampler):
    for step in range(PARITY_STEPS):
        batch = workloads.config1(step)
        compare(batch, run_gpu(sampler, batch), label=f"config1 step {step}", key="config1_spec")


def test_config5_rows_bf16(sampler):
    rows = list(range(0, 1024, 8))
    for step in range(max(1, PARITY_STEPS // 5)):
        batch = workloads.config5_rows(step, rows=rows)
        compare(batch, run_gpu(sampler, batch, bf16=True), label=f"config5 bf16 step {step}", key="config5_one_piece")


def test_nonfinite_rows_flagged(sampler):
    rng = np.random.default_rng(7)
    batch = make_batch(rng, 4, 300, 1.0, 0, 0.9)
    batch.logits[1, 17] = np.nan
    batch.logits[2, :] = -np.inf
    batch.logits[3, 5] = np.inf
    tok, prob, st, *_ = run_gpu(sampler, batch)
    assert list(st) == [0, rlsampler.RL_ERR_NONFINITE, rlsampler.RL_ERR_NONFINITE, rlsampler.RL_ERR_NONFINITE]
    assert list(tok[1:]) == [-1, -1, -1]


def test_full_size_config2_properties(sampler):
    """Full B=256 x V=128256 through the production entry (rl_sample_batch):
    every row OK, deterministic across runs, equal to the debug launch, and
    top-k rows draw from their list."""
    batch = workloads.config2(0)
    dev = "cuda:0"
    lg = torch.from_numpy(batch.logits).to(dev)
    p = rlsampler.params_tensor(batch.params, dev)
    u = torch.from_numpy(batch.uniforms).to(dev)
    hist = torch.from_numpy(batch.hist).to(dev)
    hl = torch.from_numpy(batch.hist_len).to(dev)
    runs = []
    for _ in range(3):
        t, pr, st = sampler.sample(lg, p, u, hist, hl)
        torch.cuda.synchronize()
        runs.append((t.cpu().numpy(), pr.cpu().numpy(), st.cpu().numpy()))
    for t, pr, st in runs:
        assert (st == 0).all()
        assert np.array_equal(t, runs[0][0]) and np.array_equal(pr, runs[0][1])
    g = run_gpu(sampler, batch)
    assert np.array_equal(g[0], runs[0][0]) and np.array_equal(g[1], runs[0][1])
    assert ((g[0] >= 0) & (g[0] < 128256)).all()
    for b in range(256):
        k = batch.params[b]["top_k"]
        if k > 0 and g[5][b] >= 0:
            assert g[0][b] in set(g[3][b, : g[5][b]].tolist())


def run_plain(s, batch, bf16=False):
    """rl_sample_batch itself (no inspection outputs): for rows of at most
    45056 logits without a mask this is the short-row kernel."""
    dev = "cuda:0"
    if bf16:
        lg = torch.from_numpy(batch.bf16_bits.view(np.int16)).to(dev).view(torch.bfloat16)
    else:
        lg = torch.from_numpy(batch.logits).to(dev)
    p = rlsampler.params_tensor(batch.params, dev)
    u = torch.from_numpy(batch.uniforms).to(dev)
    hist = torch.from_numpy(batch.hist).to(dev) if batch.hist is not None else None
    hl = torch.from_numpy(batch.hist_len).to(dev) if batch.hist_len is not None else None
    mask = torch.from_numpy(batch.mask.view(np.int32)).to(dev) if batch.mask is not None else None
    tok, prob, st = s.sample(lg, p, u, hist, hl, mask)
    torch.cuda.synchronize()
    return tok.cpu().numpy(), prob.cpu().numpy(), st.cpu().numpy()


def compare_plain(batch, got, label, key):
    tok, prob, st = got
    refs = oracle_rows(batch, 0)
    n = dict(rows=0, tokens_equal=0, boundary=0, prob_on_cut_boundary=0)
    for b, r in enumerate(refs):
        exp_st = 0 if r.status == 0 else rlsampler.RL_ERR_NONFINITE
        assert st[b] == exp_st, f"{label} row {b}: status {st[b]} vs {exp_st}"
        n["rows"] += 1
        if r.status:
            continue
        if tok[b] != r.token:
            assert min(r.draw_margin, r.cut_margin) < BOUNDARY, (
                f"{label} row {b}: token {tok[b]} vs oracle {r.token} "
                f"(draw margin {r.draw_margin:.3g}, cut margin {r.cut_margin:.3g})")
            n["boundary"] += 1
            continue
        n["tokens_equal"] += 1
        if r.cut_margin < BOUNDARY and abs(prob[b] - r.prob) > PROB_RTOL * abs(r.prob):
            n["prob_on_cut_boundary"] += 1
            continue
        np.testing.assert_allclose(prob[b], r.prob, rtol=PROB_RTOL, err_msg=f"{label} row {b}: prob")
    parity_add(key, **n)


SHORT = [c for c in SMALL if c[6] is None] + [
    # B, V, T, top_k, top_p, hist, mask_density, ties: short unmasked rows
    # whose ordered list spans several 1024-key batches, or a whole row
    (4, 32000, 1.0, 129, 1.0, 64, None, False),
    (4, 32000, 0.8, 500, 1.0, 64, None, False),
    (4, 32000, 1.1, 3000, 0.97, 0, None, False),
    (4, 45056, 1.3, 0, 0.999, 512, None, False),
    (4, 20000, 1.0, 0, 0.9, 1024, None, True),
    (64, 32000, 0.7, 50, 0.95, 0, None, False),
]


@pytest.mark.parametrize("case", SHORT, ids=lambda c: f"B{c[0]}_V{c[1]}_T{c[2]}_k{c[3]}_p{c[4]}_h{c[5]}")
def test_short_rows_plain_entry(sampler, case):
    B, V, T, k, tp, hl, md, ties = case
    rng = np.random.default_rng((hash(case) + 1) & 0xFFFFFFFF)
    batch = make_batch(rng, B, V, T, k, tp, hl, md, ties=ties)
    compare_plain(batch, run_plain(sampler, batch), str(case), "short_rows_plain")


def test_short_rows_config1_and_bf16(sampler):
    for step in range(PARITY_STEPS):
        batch = workloads.config1(step)
        compare_plain(batch, run_plain(sampler, batch), f"config1 plain step {step}", "config1_plain")
    rng = np.random.default_rng(99)
    batch = make_batch(rng, 16, 32000, 0.9, 64, 0.95, 256, None)
    bits = workloads.f32_to_bf16_bits(batch.logits)
    batch.logits = workloads.bf16_bits_to_f32(bits)
    batch.bf16_bits = bits
    compare_plain(batch, run_plain(sampler, batch, bf16=True), "bf16 short rows", "short_rows_bf16")


def test_short_rows_nonfinite(sampler):
    rng = np.random.default_rng(8)
    batch = make_batch(rng, 4, 300, 1.0, 0, 0.9)
    batch.logits[1, 17] = np.nan
    batch.logits[2, :] = -np.inf
    batch.logits[3, 5] = np.inf
    tok, prob, st = run_plain(sampler, batch)
    assert list(st) == [0, rlsampler.RL_ERR_NONFINITE, rlsampler.RL_ERR_NONFINITE, rlsampler.RL_ERR_NONFINITE]
    assert list(tok[1:]) == [-1, -1, -1]
