"""rl_sample_batch_static (no handle, no allocation in the call) against the
handle-based rl_sample_batch on the same inputs, over two calls in a row.

Both run the same kernel; the static entry always streams a row as one
segment, the handle-based one splits small batches into segments, so the
softmax sums are added in a different order. Tokens must agree except where
the oracle puts the draw or the top-p cutoff within 1e-6 of a CDF boundary;
probabilities within 1e-5 relative.
"""
import numpy as np
import pytest

import oracle
import rlsampler
import workloads

PROB_RTOL = 1e-5
BOUNDARY = 1e-6


def test_static_rejects_bad_sizes_without_gpu():
    lib = rlsampler.lib()
    P = None
    # B < 0 and V beyond the kernel's id range are rejected before any device call
    assert lib.rl_sample_batch_static(P, 0, -1, 100, 100, P, P, 0, P, 0, P, P, P, P, P, P) == \
        rlsampler.RL_ERR_INVALID_ARG
    big = (1 << 21)
    st = lib.rl_sample_batch_static(1, 0, 1, big, big, P, P, 0, P, 0, 1, 1, 1, P, P, P)
    assert st == rlsampler.RL_ERR_SHAPE
    assert b"V" in lib.rl_last_error()


@pytest.mark.gpu
def test_static_matches_handle_path_twice():
    import torch

    dev = "cuda:0"
    rows = list(range(0, 256, 8))  # 32 rows of the config-2 batch, full vocabulary
    batch = workloads.config2(3, rows=rows)
    lg = torch.from_numpy(batch.logits).to(dev)
    p = rlsampler.params_tensor(batch.params, dev)
    u = torch.from_numpy(batch.uniforms).to(dev)
    hist = torch.from_numpy(batch.hist).to(dev)
    hl = torch.from_numpy(batch.hist_len).to(dev)

    s = rlsampler.Sampler(0, max_batch=64, max_vocab=batch.logits.shape[1], max_history=512)
    try:
        ref_tok, ref_prob, ref_st = [t.cpu().numpy() for t in s.sample(lg, p, u, hist, hl)]
    finally:
        s.close()
    assert (ref_st == 0).all()

    outs = []
    for _ in range(2):
        tok, prob, st = rlsampler.sample_static(lg, p, u, hist, hl)
        torch.cuda.synchronize()
        outs.append((tok.cpu().numpy(), prob.cpu().numpy(), st.cpu().numpy()))
    # two calls in a row give the same results
    assert np.array_equal(outs[0][0], outs[1][0]) and np.array_equal(outs[0][1], outs[1][1])

    tok, prob, st = outs[0]
    assert (st == 0).all()
    _agree(batch, (tok, prob, st), (ref_tok, ref_prob, ref_st))


def _agree(batch, got, ref):
    tok, prob, st = got
    ref_tok, ref_prob, ref_st = ref
    assert np.array_equal(st, ref_st)
    for b in range(len(tok)):
        if st[b] != 0:
            continue
        if tok[b] == ref_tok[b]:
            np.testing.assert_allclose(prob[b], ref_prob[b], rtol=PROB_RTOL, err_msg=f"row {b}: prob")
            continue
        prm = {k: batch.params[b][k].item() for k in batch.params.dtype.names}
        r = oracle.spec_sample_row(batch.logits[b], batch.hist[b][: batch.hist_len[b]], None, prm,
                                   batch.uniforms[b])
        assert min(r.draw_margin, r.cut_margin) < BOUNDARY, \
            f"row {b}: static token {tok[b]} vs handle token {ref_tok[b]} away from a CDF boundary"


@pytest.mark.gpu
def test_static_bf16_and_greedy_rows():
    import torch

    dev = "cuda:0"
    batch = workloads.config5_rows(1, rows=list(range(0, 1024, 256)))
    lg = torch.from_numpy(batch.bf16_bits.view(np.int16)).to(dev).view(torch.bfloat16)
    batch.params["temperature"][0] = 0.0  # one greedy row
    p = rlsampler.params_tensor(batch.params, dev)
    u = torch.from_numpy(batch.uniforms).to(dev)
    hist = torch.from_numpy(batch.hist).to(dev)
    hl = torch.from_numpy(batch.hist_len).to(dev)
    s = rlsampler.Sampler(0, max_batch=8, max_vocab=batch.logits.shape[1], max_history=512)
    try:
        ref = [t.cpu().numpy() for t in s.sample(lg, p, u, hist, hl)]
    finally:
        s.close()
    for _ in range(2):
        got = [t.cpu().numpy() for t in rlsampler.sample_static(lg, p, u, hist, hl)]
        assert got[0][0] == ref[0][0]  # greedy row: argmax
        _agree(batch, got, ref)


@pytest.mark.gpu
def test_static_masked_rows_match_handle_path():
    """Grammar masks through the entry that allocates nothing (config 3)."""
    import torch

    dev = "cuda:0"
    batch = workloads.config3(4)
    lg = torch.from_numpy(batch.logits).to(dev)
    p = rlsampler.params_tensor(batch.params, dev)
    u = torch.from_numpy(batch.uniforms).to(dev)
    mask = torch.from_numpy(batch.mask.view(np.int32)).to(dev)
    s = rlsampler.Sampler(0, max_batch=64, max_vocab=batch.logits.shape[1], max_history=0)
    try:
        ref = [t.cpu().numpy() for t in s.sample(lg, p, u, mask=mask)]
    finally:
        s.close()
    for _ in range(2):
        got = [t.cpu().numpy() for t in rlsampler.sample_static(lg, p, u, mask=mask)]
        _agree(batch, got, ref)


@pytest.mark.gpu
def test_static_allocates_nothing_and_replays_in_a_graph():
    """No device memory is taken by a call (free memory unchanged), and a
    call captured into a CUDA graph after a warm call replays to the eager
    results, twice."""
    import torch

    dev = "cuda:0"
    batch = workloads.config2(5, rows=list(range(0, 256, 16)))
    lg = torch.from_numpy(batch.logits).to(dev)
    p = rlsampler.params_tensor(batch.params, dev)
    u = torch.from_numpy(batch.uniforms).to(dev)
    hist = torch.from_numpy(batch.hist).to(dev)
    hl = torch.from_numpy(batch.hist_len).to(dev)
    B = lg.shape[0]
    tok = torch.empty(B, dtype=torch.int32, device=dev)
    prob = torch.empty(B, dtype=torch.float32, device=dev)
    st = torch.empty(B, dtype=torch.int32, device=dev)
    rlsampler.sample_static(lg, p, u, hist, hl, out_tok=tok, out_prob=prob, row_status=st)  # warm
    torch.cuda.synchronize()
    eager = (tok.cpu().numpy().copy(), prob.cpu().numpy().copy(), st.cpu().numpy().copy())
    free0, _ = torch.cuda.mem_get_info()
    rlsampler.sample_static(lg, p, u, hist, hl, out_tok=tok, out_prob=prob, row_status=st)
    torch.cuda.synchronize()
    free1, _ = torch.cuda.mem_get_info()
    assert free1 == free0

    g = torch.cuda.CUDAGraph()
    side = torch.cuda.Stream()
    with torch.cuda.stream(side):
        with torch.cuda.graph(g, stream=side):
            rlsampler.sample_static(lg, p, u, hist, hl, out_tok=tok, out_prob=prob, row_status=st)
    for _ in range(2):
        tok.fill_(-7)
        g.replay()
        torch.cuda.synchronize()
        assert np.array_equal(tok.cpu().numpy(), eager[0])
        assert np.array_equal(prob.cpu().numpy(), eager[1])
        assert np.array_equal(st.cpu().numpy(), eager[2])
    del g


@pytest.mark.gpu
def test_static_rejects_host_buffers():
    """Buffers that are not device memory of the current device are refused
    before any launch."""
    import torch

    dev = "cuda:0"
    lg = torch.zeros((2, 64), device=dev)
    p = rlsampler.params_tensor(np.zeros(2, rlsampler.ROW_PARAMS_DTYPE), dev)
    u = torch.zeros(2, device=dev)
    host_tok = torch.empty(2, dtype=torch.int32, pin_memory=True)
    with pytest.raises(rlsampler.RLError) as e:
        rlsampler.sample_static(lg, p, u, out_tok=host_tok)
    assert e.value.status == rlsampler.RL_ERR_INVALID_ARG
