"""Parity of the beam step (rl_beam_step) and of vocabulary-sharded sampling
(rl_sample_partial + rl_sample_merge) with the CPU oracle, through the C ABI.

Beam step: beams, tokens and done flags equal to the oracle's
(BeamSearch::search order: score desc, beam asc, logit desc, id asc);
scores within 2e-5 absolute (the device's log-sum-exp is a parallel double
sum, the oracle's a sequential one, so lse can differ in its last f32 bit).
A swap of two neighbours whose oracle scores lie within that tolerance is
counted, not failed.

Shards: G partial results of column slices of the same rows, merged on the
device, give the one-piece sampler's token and probability (within 1e-5
relative), except where the oracle puts the draw or the top-p cutoff within
1e-6 of a CDF boundary.
"""
import numpy as np
import pytest

import oracle
import rlsampler
import sharded
import workloads

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

SCORE_ATOL = 2e-5
PROB_RTOL = 1e-5
BOUNDARY = 1e-6


@pytest.fixture(scope="module")
def sampler():
    s = rlsampler.Sampler(0, max_batch=256, max_vocab=262144, max_history=1024)
    yield s
    s.close()


def _beam_gpu(s, bb, n_out, log_softmax=1):
    dev = "cuda:0"
    lg = torch.from_numpy(bb.logits).to(dev)
    sc = torch.from_numpy(bb.scores).to(dev)
    dn = torch.from_numpy(bb.done).to(dev)
    ln = torch.from_numpy(bb.lens).to(dev)
    out = s.beam_step(lg, bb.items, bb.beams, sc, dn, ln, bb.alpha, bb.eos, log_softmax, n_out)
    return [t.cpu().numpy() for t in out]


def _beam_agree(got, ref):
    gb, gt, gs, gd = got
    rb, rt, rs, rd = ref
    items, n = rb.shape
    swaps = 0
    for it in range(items):
        np.testing.assert_allclose(gs[it], rs[it], rtol=0, atol=SCORE_ATOL, err_msg=f"item {it}: scores")
        for j in range(n):
            if gb[it, j] == rb[it, j] and gt[it, j] == rt[it, j]:
                assert gd[it, j] == rd[it, j], f"item {it} pos {j}: done flag"
                continue
            near = [abs(float(rs[it, j]) - float(rs[it, jj])) < SCORE_ATOL
                    for jj in (j - 1, j + 1) if 0 <= jj < n]
            assert any(near) or j == n - 1, \
                f"item {it} pos {j}: ({gb[it, j]},{gt[it, j]}) vs oracle ({rb[it, j]},{rt[it, j]})"
            swaps += 1
    return swaps


def test_beam_config4_full(sampler):
    bb = workloads.config4(0)
    n_out = 2 * bb.beams
    got = _beam_gpu(sampler, bb, n_out)
    ref = oracle.beam_step(bb.logits, bb.items, bb.beams, bb.scores, bb.done, bb.lens, bb.alpha, bb.eos, 1, n_out)
    swaps = _beam_agree(got, ref)
    assert swaps <= 1, f"{swaps} near-tie swaps"
    assert (got[0] >= 0).all() and (got[0] < bb.beams).all()


@pytest.mark.parametrize("case", [
    # items, beams, V, done_frac, alpha, log_softmax, n_out
    (4, 4, 5000, 0.3, 0.6, 0, 6),
    (3, 8, 151936, 0.25, 1.0, 1, 16),
    (2, 16, 32000, 0.0, 1.2, 1, 32),
    (5, 4, 7, 0.0, 1.0, 1, 8),
], ids=lambda c: f"i{c[0]}_b{c[1]}_V{c[2]}_d{c[3]}_a{c[4]}_ls{c[5]}_n{c[6]}")
def test_beam_variants(sampler, case):
    items, beams, V, dfrac, alpha, ls, n_out = case
    bb = workloads.config4(1, items=items, beams=beams, V=V, done_frac=dfrac)
    bb.alpha = alpha
    if V > 2:
        bb.logits[0, 2] = bb.logits[0].max() + 1.0  # EOS on top of beam 0 of item 0
    got = _beam_gpu(sampler, bb, n_out, ls)
    ref = oracle.beam_step(bb.logits, items, beams, bb.scores, bb.done, bb.lens, alpha, bb.eos, ls, n_out)
    _beam_agree(got, ref)


def test_beam_all_done_item_pads(sampler):
    bb = workloads.config4(2, items=2, beams=4, V=3000)
    bb.done[:4] = 1  # item 0: every beam complete -> 4 candidates, n_out 8
    got = _beam_gpu(sampler, bb, 8)
    ref = oracle.beam_step(bb.logits, 2, 4, bb.scores, bb.done, bb.lens, bb.alpha, bb.eos, 1, 8)
    _beam_agree(got, ref)
    assert (got[0][0, 4:] == -1).all() and np.isneginf(got[2][0, 4:]).all()
    assert (got[1][0, :4] == -1).all() and (got[3][0, :4] == 1).all()


def _shard_inputs(rows, greedy_row=None):
    batch = workloads.config5_rows(2, rows=rows)
    if greedy_row is not None:
        batch.params["temperature"][greedy_row] = 0.0
    dev = "cuda:0"
    lg = torch.from_numpy(batch.bf16_bits.view(np.int16)).to(dev).view(torch.bfloat16)
    p = rlsampler.params_tensor(batch.params, dev)
    u = torch.from_numpy(batch.uniforms).to(dev)
    hist = torch.from_numpy(batch.hist).to(dev)
    hl = torch.from_numpy(batch.hist_len).to(dev)
    return batch, lg, p, u, hist, hl


@pytest.mark.parametrize("G", [2, 3, 4, 8])
def test_shard_merge_matches_one_piece(sampler, G):
    rows = list(range(0, 1024, 64))
    batch, lg, p, u, hist, hl = _shard_inputs(rows, greedy_row=3)
    V = lg.shape[1]
    keys, stats = [], []
    for off, w in sharded.shard_bounds(V, G):
        k, s = sampler.sample_partial(lg[:, off:off + w], off, p, hist, hl)
        keys.append(k)
        stats.append(s)
        kh = k.cpu().numpy().view(np.uint64)
        sh = sharded.stats_view(s)
        assert (sh["flags"] == 0).all() and (sh["nallow"] == w).all()
        for b in range(len(rows)):
            n = int(sh["n"][b])
            if batch.params["temperature"][b] > 0:
                assert n == min(64, w)
            ids = np.uint64(0xFFFFFFFF) - (kh[b, :n] & np.uint64(0xFFFFFFFF))
            assert ((ids >= off) & (ids < off + w)).all()
            assert (kh[b, :n][:-1] > kh[b, :n][1:]).all()
    tok, prob, st = [t.cpu().numpy() for t in sampler.sample_merge(torch.stack(keys), torch.stack(stats), p, u)]
    ref_tok, ref_prob, ref_st = [t.cpu().numpy() for t in sampler.sample(lg, p, u, hist, hl)]
    assert (st == 0).all() and (ref_st == 0).all()
    assert tok[3] == ref_tok[3]  # greedy row: the global argmax
    boundary = 0
    for b in range(len(rows)):
        if tok[b] == ref_tok[b]:
            np.testing.assert_allclose(prob[b], ref_prob[b], rtol=PROB_RTOL, err_msg=f"row {b}: prob")
            continue
        prm = {k: batch.params[b][k].item() for k in batch.params.dtype.names}
        r = oracle.spec_sample_row(batch.logits[b], batch.hist[b], None, prm, batch.uniforms[b])
        assert min(r.draw_margin, r.cut_margin) < BOUNDARY, f"row {b}: merged {tok[b]} vs one-piece {ref_tok[b]}"
        boundary += 1
    assert boundary <= 1


def test_shard_merge_vs_oracle(sampler):
    rows = [5, 77, 300, 901]
    batch, lg, p, u, hist, hl = _shard_inputs(rows)
    V = lg.shape[1]
    keys, stats = [], []
    for off, w in sharded.shard_bounds(V, 4):
        k, s = sampler.sample_partial(lg[:, off:off + w], off, p, hist, hl)
        keys.append(k)
        stats.append(s)
    tok, prob, st = [t.cpu().numpy() for t in sampler.sample_merge(torch.stack(keys), torch.stack(stats), p, u)]
    for b in range(len(rows)):
        prm = {k: batch.params[b][k].item() for k in batch.params.dtype.names}
        r = oracle.spec_sample_row(batch.logits[b], batch.hist[b], None, prm, batch.uniforms[b])
        assert st[b] == r.status == 0
        if tok[b] != r.token:
            assert min(r.draw_margin, r.cut_margin) < BOUNDARY
        else:
            np.testing.assert_allclose(prob[b], r.prob, rtol=PROB_RTOL)


def test_shard_merge_rejects_unsupported_rows(sampler):
    rows = [0, 1]
    batch, lg, p, u, hist, hl = _shard_inputs(rows)
    batch.params["top_k"][1] = 0  # top-k off: not mergeable from 128-key lists
    p = rlsampler.params_tensor(batch.params, "cuda:0")
    V = lg.shape[1]
    keys, stats = [], []
    for off, w in sharded.shard_bounds(V, 2):
        k, s = sampler.sample_partial(lg[:, off:off + w], off, p, hist, hl)
        keys.append(k)
        stats.append(s)
    tok, prob, st = [t.cpu().numpy() for t in sampler.sample_merge(torch.stack(keys), torch.stack(stats), p, u)]
    assert st[0] == 0 and st[1] == rlsampler.RL_ERR_UNSUPPORTED and tok[1] == -1


def test_beam_config4_steps(sampler):
    """Config 4 over 10 seeded steps (16 items x 8 beams x V 151936), against
    the oracle; near-tie swaps counted into the parity record."""
    from conftest import parity_add

    steps = 10
    swaps = 0
    for step in range(steps):
        bb = workloads.config4(step)
        n_out = 2 * bb.beams
        got = _beam_gpu(sampler, bb, n_out)
        ref = oracle.beam_step(bb.logits, bb.items, bb.beams, bb.scores, bb.done, bb.lens, bb.alpha, bb.eos, 1,
                               n_out)
        swaps += _beam_agree(got, ref)
    assert swaps <= steps
    parity_add("config4_beam", steps=steps, candidates=steps * 16 * 16, near_tie_swaps=swaps)


def test_shard_config5_steps(sampler):
    """Config 5 (vocabulary shards, bf16, top_k 64, top_p 0.95) over 20
    seeded steps with G = 8 shards merged on one device, 64 rows a step,
    against the oracle on the whole row."""
    from conftest import parity_add

    steps = 20
    G = 8
    dev = "cuda:0"
    n = dict(rows=0, tokens_equal=0, boundary=0, prob_on_cut_boundary=0)
    for step in range(steps):
        rows = list(range(step % 16, 1024, 16))
        batch = workloads.config5_rows(step, rows=rows)
        lg = torch.from_numpy(batch.bf16_bits.view(np.int16)).to(dev).view(torch.bfloat16)
        p = rlsampler.params_tensor(batch.params, dev)
        u = torch.from_numpy(batch.uniforms).to(dev)
        hist = torch.from_numpy(batch.hist).to(dev)
        hl = torch.from_numpy(batch.hist_len).to(dev)
        V = lg.shape[1]
        keys, stats = [], []
        for off, w in sharded.shard_bounds(V, G):
            k, s = sampler.sample_partial(lg[:, off:off + w], off, p, hist, hl)
            keys.append(k)
            stats.append(s)
        tok, prob, st = [t.cpu().numpy() for t in sampler.sample_merge(torch.stack(keys), torch.stack(stats), p, u)]
        for b in range(len(rows)):
            prm = {k: batch.params[b][k].item() for k in batch.params.dtype.names}
            r = oracle.spec_sample_row(batch.logits[b], batch.hist[b], None, prm, batch.uniforms[b])
            assert st[b] == r.status == 0
            n["rows"] += 1
            if tok[b] != r.token:
                assert min(r.draw_margin, r.cut_margin) < BOUNDARY, f"step {step} row {rows[b]}"
                n["boundary"] += 1
                continue
            n["tokens_equal"] += 1
            if r.cut_margin < BOUNDARY and abs(prob[b] - r.prob) > PROB_RTOL * abs(r.prob):
                # same token, but the cutoff (and so the renormalising mass)
                # sits on a CDF boundary
                n["prob_on_cut_boundary"] = n.get("prob_on_cut_boundary", 0) + 1
                continue
            np.testing.assert_allclose(prob[b], r.prob, rtol=PROB_RTOL)
    parity_add("config5_sharded_G8", **n)
