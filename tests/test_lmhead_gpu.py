"""The LM head feeding the sampler (src/model.rs:236-262: logits = hidden @
W^T, matmul_vec) on the tensor cores, rl_lmhead_*:

- logits against a float64 product of the same bf16 operands, within the
  error bound of an f32 sum of H exact products (H * 2^-22 * sum |products|),
  and against the oracle's matmul_vec (the reference's sequential f32 loop);
- bf16 logits equal the f32 logits rounded to nearest even, bit for bit;
- the fused greedy token equals the last-maximum argmax (the oracle's
  greedy_sample) of the kernel's own f32 logits, with and without writing
  them, ties included;
- rl_lmhead_sample equals rl_sample_batch on the kernel's own logits, and the
  oracle's spec sampler on them;
- shapes: B not a multiple of 16, B > 256 (two launches), V not a multiple of
  128, V < 128, H = 64; argument errors.
"""
import numpy as np
import pytest

import oracle
import rlsampler
import workloads

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def smp():
    s = rlsampler.Sampler(0, max_batch=320, max_vocab=40000, max_history=64)
    yield s
    s.close()


def operands(B, H, V, seed):
    g = torch.Generator(device="cuda").manual_seed(seed)
    hidden = torch.randn(B, H, generator=g, device="cuda").to(torch.bfloat16)
    weight = (torch.randn(V, H, generator=g, device="cuda") * H ** -0.5 * 3.0).to(torch.bfloat16)
    return hidden, weight


def check_logits(hidden, weight, got):
    h64, w64 = hidden.double(), weight.double()
    ref = h64 @ w64.T
    bound = hidden.shape[1] * 2.0 ** -22 * (h64.abs() @ w64.abs().T) + 1e-30
    err = (got.double() - ref).abs()
    assert bool((err <= bound).all()), f"max err {err.max().item():.3e}, bound {bound.max().item():.3e}"


SHAPES = [(1, 64, 1), (1, 128, 200), (3, 256, 1000), (16, 512, 4096), (17, 1024, 5000), (64, 2048, 32000),
          (256, 256, 3000), (300, 128, 700), (200, 4096, 32000)]


@pytest.mark.parametrize("B,H,V", SHAPES)
def test_logits_f32(smp, B, H, V):
    hidden, weight = operands(B, H, V, B * 7 + V)
    got = smp.lmhead_logits(hidden, weight)
    torch.cuda.synchronize()
    check_logits(hidden, weight, got)


@pytest.mark.parametrize("B,H,V", [(1, 64, 300), (5, 512, 2000), (17, 1024, 5000)])
def test_logits_against_the_oracle_matmul_vec(smp, B, H, V):
    """orc_matmul_vec (src/model.rs:246-261: sequential f32 sums) on the
    same bf16 values: the two f32 sums differ only in the order of the
    additions, so they agree within twice the bound of one."""
    hidden, weight = operands(B, H, V, 40 + B)
    got = smp.lmhead_logits(hidden, weight)
    torch.cuda.synchronize()
    x, w = hidden.float().cpu().numpy(), weight.float().cpu().numpy()
    ref = oracle.matmul_vec(x, w, nthreads=4)
    bound = H * 2.0 ** -21 * (np.abs(x).astype(np.float64) @ np.abs(w).astype(np.float64).T) + 1e-30
    err = np.abs(got.cpu().numpy().astype(np.float64) - ref.astype(np.float64))
    assert (err <= bound).all(), float(err.max())


def test_logits_bf16_is_rounded_f32(smp):
    hidden, weight = operands(40, 512, 3000, 5)
    f = smp.lmhead_logits(hidden, weight)
    b = smp.lmhead_logits(hidden, weight, out_dtype=torch.bfloat16)
    torch.cuda.synchronize()
    assert torch.equal(b.view(torch.int16), f.to(torch.bfloat16).view(torch.int16))


def test_logits_strided_out(smp):
    hidden, weight = operands(5, 256, 1000, 6)
    buf = torch.full((5, 1040), 7.0, device="cuda")
    smp.lmhead_logits(hidden, weight, out=buf[:, :1000])
    torch.cuda.synchronize()
    check_logits(hidden, weight, buf[:, :1000])
    assert bool((buf[:, 1000:] == 7.0).all())


@pytest.mark.parametrize("B,H,V", [(1, 64, 1), (3, 256, 1000), (17, 1024, 5000), (256, 512, 32000),
                                   (300, 128, 700)])
def test_greedy_matches_own_logits(smp, B, H, V):
    hidden, weight = operands(B, H, V, 3 * B + V)
    lg = torch.empty(B, V, device="cuda")
    tok, st = smp.lmhead_greedy(hidden, weight, out_logits=lg)
    tok2, st2 = smp.lmhead_greedy(hidden, weight)
    torch.cuda.synchronize()
    check_logits(hidden, weight, lg)
    x = lg.cpu().numpy()
    want = np.array([oracle.greedy(x[b]) for b in range(B)], np.int32)
    assert (st.cpu().numpy() == 0).all() and (st2.cpu().numpy() == 0).all()
    assert np.array_equal(tok.cpu().numpy(), want)
    assert np.array_equal(tok2.cpu().numpy(), want)


def test_greedy_ties_take_the_last_maximum(smp):
    B, H, V = 4, 128, 1000
    hidden, weight = operands(B, H, V, 9)
    hidden = hidden.abs()
    w = weight.clone()
    w[[5, 77, 300, 611]] = 1.0  # four identical rows, the largest logits of every row
    tok, st = smp.lmhead_greedy(hidden, w)
    torch.cuda.synchronize()
    assert tok.cpu().tolist() == [611] * B
    assert st.cpu().tolist() == [0] * B


def test_sample_equals_sampler_on_own_logits(smp):
    B, H, V = 64, 1024, 32000
    hidden, weight = operands(B, H, V, 11)
    r = np.random.default_rng(11)
    p = np.zeros(B, rlsampler.ROW_PARAMS_DTYPE)
    p["temperature"] = r.uniform(0.5, 1.5, B)
    p["top_k"] = r.choice([0, 1, 20, 50], B)
    p["top_p"] = r.uniform(0.8, 1.0, B)
    p["repeat_penalty"] = r.uniform(1.0, 1.3, B)
    hist = r.integers(0, V, (B, 64)).astype(np.int32)
    hl = r.integers(0, 65, B).astype(np.int32)
    u = workloads.uniforms(9, 0, B)
    pd = rlsampler.params_tensor(p, "cuda")
    ud = torch.from_numpy(u).cuda()
    hd = torch.from_numpy(hist).cuda()
    hld = torch.from_numpy(hl).cuda()
    tok, prob, st = smp.lmhead_sample(hidden, weight, pd, ud, hd, hld)
    lg = smp.lmhead_logits(hidden, weight)
    tok2, prob2, st2 = smp.sample(lg, pd, ud, hd, hld)
    torch.cuda.synchronize()
    assert (st.cpu().numpy() == 0).all()
    assert torch.equal(tok, tok2) and torch.equal(prob, prob2) and torch.equal(st, st2)
    x = lg.cpu().numpy()
    otok, oprob, bad = oracle.spec_sample_batch(x, hist, hl, None, p, u, nthreads=8)
    assert bad == 0
    assert np.array_equal(tok.cpu().numpy(), otok)
    np.testing.assert_allclose(prob.cpu().numpy(), oprob, rtol=1e-5, atol=1e-7)


def test_argument_errors(smp):
    hidden, weight = operands(4, 128, 300, 1)
    with pytest.raises(rlsampler.RLError) as e:
        smp.lmhead_logits(hidden[:, :100], weight[:, :100])  # H not a multiple of 64
    assert e.value.status == rlsampler.RL_ERR_UNSUPPORTED
    h2 = torch.empty(4, 136, dtype=torch.bfloat16, device="cuda")
    with pytest.raises(rlsampler.RLError) as e:
        smp.lmhead_logits(h2[:, 1:129], weight)  # 2-byte offset: not 16-byte aligned
    assert e.value.status == rlsampler.RL_ERR_INVALID_ARG
    big = torch.empty(321, 128, dtype=torch.bfloat16, device="cuda")
    with pytest.raises(rlsampler.RLError) as e:
        smp.lmhead_greedy(big, weight)  # beyond max_batch
    assert e.value.status == rlsampler.RL_ERR_SHAPE
