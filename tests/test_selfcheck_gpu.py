"""The library's device self-checks and failure path.

- rl_selfcheck_div: the fixed-divisor division the spec sampler applies to
  every logit (logit - max) / T must equal IEEE division bit for bit; bit-exact
  top-k sets rest on it. Checked over numerators spanning every binade the
  sampler can meet and temperatures spanning the fixed-divisor range, its
  edges and the benchmark workloads' values.
- RL_DEBUG_EXPIRE_WAIT: a bounded device wait that runs out reports
  RL_ERR_TIMEOUT in row_status (no fault, no hang), and the same handle
  samples correctly afterwards.
"""
import numpy as np
import pytest

import oracle
import rlsampler

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu


def _numerators(rng, n):
    # sign * 2^e * (1 + f): e over the binades of the fast path and beyond
    # it (|a| >= 2^-90 takes the fixed-divisor path), plus exact values
    e = rng.integers(-100, 128, n)
    f = rng.random(n)
    a = (np.where(rng.random(n) < 0.5, -1.0, 1.0) * np.ldexp(1.0 + f, e)).astype(np.float32)
    special = np.array([0.0, -0.0, 1.0, -1.0, 2.0 ** -90, -(2.0 ** -90), 2.0 ** -91, 8.077935669e-28,
                        np.nextafter(np.float32(8.077935669e-28), np.float32(0)), 3.0e38, -3.0e38,
                        1.0000001, 0.99999994, 16.0, -0.5, 7.0, 1e-30, -1e-35], np.float32)
    return np.concatenate([special, a[np.isfinite(a)]]).astype(np.float32)


def _temperatures(rng):
    lo, hi = 2.0 ** -20, 2.0 ** 20
    edges = [lo, hi, np.nextafter(np.float32(lo), np.float32(0)), np.nextafter(np.float32(hi), np.float32(np.inf)),
             np.nextafter(np.float32(lo), np.float32(1)), np.nextafter(np.float32(hi), np.float32(0)),
             1.0, 0.5, 1.5, 0.7, 0.8, 1.3, 0.1, 3.0, 1e-3, 1e3]
    logu = np.exp(rng.uniform(np.log(lo), np.log(hi), 200))
    bench = rng.uniform(0.5, 1.5, 100)
    return np.concatenate([np.array(edges), logu, bench]).astype(np.float32)


def test_fixed_divisor_division_is_ieee_exact():
    rng = np.random.default_rng(20)
    a = _numerators(rng, 1 << 20)
    T = _temperatures(rng)
    dev = "cuda:0"
    mism, fast = rlsampler.selfcheck_div(torch.from_numpy(a).to(dev), torch.from_numpy(T).to(dev))
    # the fixed-divisor path is taken exactly on [2^-20, 2^20]
    want_fast = (T >= np.float32(2.0 ** -20)) & (T <= np.float32(2.0 ** 20))
    assert np.array_equal(fast.astype(bool), want_fast)
    assert want_fast.sum() > 300
    bad = {float(T[j]): int(mism[j]) for j in range(T.size) if mism[j]}
    assert not bad, f"quotients differing from IEEE division: {bad}"


def _batch(rng, B=6, V=5000):
    x = rng.normal(0, 3, (B, V)).astype(np.float32)
    p = np.zeros(B, rlsampler.ROW_PARAMS_DTYPE)
    p["temperature"] = [1.0, 0.7, 0.0, 1.2, 0.9, 1.0]
    p["top_k"] = [0, 40, 0, 200, 1, 0]
    p["top_p"] = [0.9, 0.95, 1.0, 0.9, 1.0, 1.0]
    p["repeat_penalty"] = 1.1
    u = rng.random(B).astype(np.float32)
    return x, p, u


def test_expired_wait_reports_timeout_then_recovers():
    s = rlsampler.Sampler(0, max_batch=16, max_vocab=8192, max_history=64)
    try:
        rng = np.random.default_rng(5)
        x, p, u = _batch(rng)
        dev = "cuda:0"
        xt, pt, ut = torch.from_numpy(x).to(dev), rlsampler.params_tensor(p, dev), torch.from_numpy(u).to(dev)
        s.set_debug(rlsampler.RL_DEBUG_EXPIRE_WAIT)
        tok, prob, st = s.sample(xt, pt, ut)
        torch.cuda.synchronize()
        assert (st.cpu().numpy() == rlsampler.RL_ERR_TIMEOUT).all()
        assert (tok.cpu().numpy() == -1).all()
        s.set_debug(0)
        tok, prob, st = s.sample(xt, pt, ut)
        torch.cuda.synchronize()
        tok, prob, st = tok.cpu().numpy(), prob.cpu().numpy(), st.cpu().numpy()
        assert (st == 0).all()
        for b in range(x.shape[0]):
            prm = {k: p[b][k].item() for k in p.dtype.names}
            r = oracle.spec_sample_row(x[b], None, None, prm, u[b])
            if tok[b] != r.token:
                assert min(r.draw_margin, r.cut_margin) < 1e-6
            else:
                assert abs(prob[b] - r.prob) <= 1e-5 * abs(r.prob)
    finally:
        s.close()


def test_debug_flags_rejected_when_unknown():
    s = rlsampler.Sampler(0, max_batch=4, max_vocab=1024, max_history=0)
    try:
        with pytest.raises(rlsampler.RLError):
            s.set_debug(0x80)
    finally:
        s.close()


def test_kernel_times_after_a_timed_call():
    """RL_DEBUG_TIMING: rl_sampler_kernel_times returns the device times of the
    last call's kernels -- one for short unmasked rows (the short-row kernel),
    two otherwise (the streaming and finish kernels); off again, none."""
    import workloads

    dev = torch.device("cuda", 0)
    s = rlsampler.Sampler(0, max_batch=64, max_vocab=128256, max_history=512)
    try:
        assert s.kernel_times() == []
        b = workloads.config3(0)
        lg = torch.from_numpy(b.logits).to(dev)
        mask = torch.from_numpy(b.mask.view(np.int32)).to(dev)
        prm = rlsampler.params_tensor(b.params, dev)
        u = torch.from_numpy(b.uniforms).to(dev)
        s.set_debug(rlsampler.RL_DEBUG_TIMING)
        tok, _, st = s.sample(lg, prm, u, mask=mask)
        t = s.kernel_times()
        assert len(t) == 2 and all(0.0 < x < 1000.0 for x in t)
        ref, _, _ = oracle.spec_sample_batch(b.logits, None, None, b.mask, b.params, b.uniforms)
        assert (st.cpu().numpy() == 0).all()
        assert (tok.cpu().numpy() == ref).mean() > 0.98
        b2 = workloads.config2(0, rows=list(range(8)))
        s.sample(torch.from_numpy(b2.logits).to(dev), rlsampler.params_tensor(b2.params, dev),
                 torch.from_numpy(b2.uniforms).to(dev), torch.from_numpy(b2.hist).to(dev),
                 torch.from_numpy(b2.hist_len).to(dev))
        t = s.kernel_times()
        assert len(t) == 2 and all(0.0 < x < 1000.0 for x in t)
        b1 = workloads.config1(0)
        s.sample(torch.from_numpy(b1.logits).to(dev), rlsampler.params_tensor(b1.params, dev),
                 torch.from_numpy(b1.uniforms).to(dev), torch.from_numpy(b1.hist).to(dev),
                 torch.from_numpy(b1.hist_len).to(dev))
        t = s.kernel_times()
        assert len(t) == 1 and 0.0 < t[0] < 1000.0
        s.set_debug(0)
        s.sample(lg, prm, u, mask=mask)
        assert s.kernel_times() == []
    finally:
        s.close()
