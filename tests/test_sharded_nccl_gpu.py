"""rl_sample_sharded: vocabulary shards exchanged over NCCL inside the
library (one packed record per row and rank, one ncclAllGather), against the
one-piece sampler and the oracle.

On one GPU the communicator has a single rank (the all-gather copies the
rank's own records). With two or more GPUs the test also runs two ranks as
child processes, one per GPU, each holding half of the vocabulary.
"""
import datetime
import os
import socket

import numpy as np
import pytest

import oracle
import rlsampler
import sharded
import workloads

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

PROB_RTOL = 1e-5
BOUNDARY = 1e-6


def _inputs(step, rows, dev):
    batch = workloads.config5_rows(step, rows=rows)
    lg = torch.from_numpy(batch.bf16_bits.view(np.int16)).to(dev).view(torch.bfloat16)
    p = rlsampler.params_tensor(batch.params, dev)
    u = torch.from_numpy(batch.uniforms).to(dev)
    hist = torch.from_numpy(batch.hist).to(dev)
    hl = torch.from_numpy(batch.hist_len).to(dev)
    return batch, lg, p, u, hist, hl


def _agree(batch, got, ref, label):
    tok, prob, st = got
    rtok, rprob, rst = ref
    assert (st == 0).all() and (rst == 0).all(), label
    for b in range(len(tok)):
        if tok[b] == rtok[b]:
            np.testing.assert_allclose(prob[b], rprob[b], rtol=PROB_RTOL, err_msg=f"{label} row {b}")
            continue
        prm = {k: batch.params[b][k].item() for k in batch.params.dtype.names}
        r = oracle.spec_sample_row(batch.logits[b], batch.hist[b], None, prm, batch.uniforms[b])
        assert min(r.draw_margin, r.cut_margin) < BOUNDARY, f"{label} row {b}: {tok[b]} vs {rtok[b]}"


def test_one_rank_communicator_matches_one_piece():
    dev = "cuda:0"
    torch.cuda.set_device(0)
    uid = rlsampler.nccl_unique_id()
    comm = rlsampler.nccl_comm_init(1, uid, 0)
    s = rlsampler.Sampler(0, max_batch=128, max_vocab=256000, max_history=256, flags=rlsampler.RL_CREATE_SHARDED)
    try:
        batch, lg, p, u, hist, hl = _inputs(6, list(range(0, 1024, 16)), dev)
        V = lg.shape[1]
        got = [t.cpu().numpy() for t in s.sample_sharded(comm, lg, 0, V, p, u, hist, hl)]
        ref = [t.cpu().numpy() for t in s.sample(lg, p, u, hist, hl)]
        _agree(batch, got, ref, "G=1")
        # a handle without the exchange buffers refuses
        s2 = rlsampler.Sampler(0, max_batch=8, max_vocab=1024, max_history=0)
        try:
            with pytest.raises(rlsampler.RLError) as e:
                s2.sample_sharded(comm, lg[:2, :1024], 0, V, p[: 2 * 24], u[:2])
            assert e.value.status == rlsampler.RL_ERR_UNSUPPORTED
        finally:
            s2.close()
    finally:
        s.close()
        rlsampler.nccl_comm_destroy(comm)


def _free_port():
    with socket.socket() as sk:
        sk.bind(("127.0.0.1", 0))
        return sk.getsockname()[1]


def _rank(rank, world, port, out_dir):
    import torch.distributed as dist

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dev = f"cuda:{rank}"
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=120))
    try:
        rows = list(range(3, 1024, 32))
        batch, lg, p, u, hist, hl = _inputs(7, rows, dev)
        V = lg.shape[1]
        ss = sharded.ShardedSampler(V, max_batch=64, device=dev, max_history=256)
        try:
            off, w = ss.offset, ss.width
            for _ in range(2):  # two calls in a row
                tok, prob, st = [t.cpu().numpy() for t in ss.sample(lg[:, off:off + w].contiguous(), p, u, hist, hl)]
            np.save(os.path.join(out_dir, f"tok{rank}.npy"), tok)
            np.save(os.path.join(out_dir, f"prob{rank}.npy"), prob)
            np.save(os.path.join(out_dir, f"st{rank}.npy"), st)
            if rank == 0:
                one = rlsampler.Sampler(0, max_batch=64, max_vocab=V, max_history=256)
                try:
                    ref = [t.cpu().numpy() for t in one.sample(lg, p, u, hist, hl)]
                finally:
                    one.close()
                for name, arr in zip(("rtok", "rprob", "rst"), ref):
                    np.save(os.path.join(out_dir, f"{name}.npy"), arr)
        finally:
            ss.close()
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_two_ranks_over_nccl(tmp_path):
    import torch.multiprocessing as mp

    world = 2
    mp.start_processes(_rank, args=(world, _free_port(), str(tmp_path)), nprocs=world, start_method="spawn")
    t0, t1 = np.load(tmp_path / "tok0.npy"), np.load(tmp_path / "tok1.npy")
    assert np.array_equal(t0, t1)  # every rank draws the same tokens
    assert np.array_equal(np.load(tmp_path / "prob0.npy"), np.load(tmp_path / "prob1.npy"))
    batch = workloads.config5_rows(7, rows=list(range(3, 1024, 32)))
    got = (t0, np.load(tmp_path / "prob0.npy"), np.load(tmp_path / "st0.npy"))
    ref = (np.load(tmp_path / "rtok.npy"), np.load(tmp_path / "rprob.npy"), np.load(tmp_path / "rst.npy"))
    _agree(batch, got, ref, "G=2")
