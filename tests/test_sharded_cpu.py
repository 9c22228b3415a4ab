"""Host side of vocabulary-sharded sampling, on CPU: the shard split, the
packed records and their single all-gather over two gloo ranks (the layout
rl_sample_sharded's NCCL all-gather produces), the communicator-id exchange
of ShardedSampler, and the merge identity (the G partial results determine
the one-piece result) checked against the oracle.

The partial results here are computed with numpy from each rank's columns,
in the layout rl_sample_partial writes (sorted uint64 keys, rl_part_stats).
"""
import os
import socket

import numpy as np
import pytest

import oracle
import rlsampler
import sharded
import workloads

torch = pytest.importorskip("torch")

BOUNDARY = 1e-6


def test_shard_bounds_cover_and_align():
    for V in (32000, 151936, 256000, 1000, 8 * 17 + 3):
        for G in (1, 2, 3, 4, 8):
            try:
                b = sharded.shard_bounds(V, G)
            except ValueError:
                step = -(-(-(-V // G)) // sharded.SHARD_ALIGN) * sharded.SHARD_ALIGN
                assert (G - 1) * step >= V  # a rank would get no columns
                continue
            assert b[0][0] == 0 and sum(w for _, w in b) == V
            for (o1, w1), (o2, _) in zip(b, b[1:]):
                assert o1 + w1 == o2 and o2 % sharded.SHARD_ALIGN == 0
    with pytest.raises(ValueError):
        sharded.shard_bounds(16, 4)


def _ord_key(x):
    u = x.astype(np.float32).view(np.uint32).astype(np.uint64)
    neg = (u >> np.uint64(31)) == 1
    return np.where(neg, np.uint64(0xFFFFFFFF) - u, u | np.uint64(0x80000000))


def _penalised(x, hist, rp):
    y = x.astype(np.float32).copy()
    for i in np.unique(hist):
        v = y[i]
        y[i] = v * np.float32(rp) if v < 0 else v / np.float32(rp)
    return y


def numpy_partial(y_shard, off, T, top_k):
    """One shard's rl_part_stats record and key list (numpy)."""
    st = np.zeros(1, rlsampler.PART_STATS_DTYPE)
    keys = np.zeros(rlsampler.PART_KEYS, np.uint64)
    M = y_shard.max()
    st["m"] = M
    st["argmax"] = off + int(np.argmax(y_shard))
    st["nallow"] = y_shard.size
    e = np.exp(((y_shard - M) / np.float32(T)).astype(np.float32))
    st["z"] = e.astype(np.float64).sum()
    k = (_ord_key(y_shard) << np.uint64(32)) | (np.uint64(0xFFFFFFFF) - (np.arange(y_shard.size) + off).astype(np.uint64))
    k = np.sort(k)[::-1][: min(top_k, y_shard.size)]
    keys[: k.size] = k
    st["n"] = k.size
    return keys, st


def numpy_merge(keys, stats, T, top_k, top_p, u):
    """The device merge restated: keys [G, 128] uint64, stats [G]."""
    M = stats["m"].max()
    Z = float((stats["z"] * np.exp((stats["m"].astype(np.float64) - float(M)) / float(T))).sum())
    allk = np.concatenate([keys[g, : stats["n"][g]] for g in range(len(stats))])
    K = min(top_k, int(stats["nallow"].sum()))
    top = np.sort(allk)[::-1][:K]
    hi = (top >> np.uint64(32)).astype(np.uint64)
    neg = hi < np.uint64(0x80000000)
    bits = np.where(neg, np.uint64(0xFFFFFFFF) - hi, hi & np.uint64(0x7FFFFFFF)).astype(np.uint32)
    x = bits.view(np.float32)
    ids = (np.uint64(0xFFFFFFFF) - (top & np.uint64(0xFFFFFFFF))).astype(np.int64)
    e = np.exp(((x - M) / np.float32(T)).astype(np.float32)).astype(np.float64)
    cum = np.cumsum(e / Z)
    cut = K - 1
    if top_p < 1.0:
        hit = np.nonzero(cum >= top_p)[0]
        if hit.size:
            cut = min(cut, int(hit[0]))
    S = cum[cut]
    d = np.nonzero(cum[: cut + 1] > u * S)[0]
    d = int(d[0]) if d.size else cut
    return int(ids[d]), float(e[d] / Z / S)


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank, world, port, V, B, out_dir):
    import torch.distributed as dist

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=__import__("datetime").timedelta(seconds=60))
    try:
        batch = workloads.config5_rows(4, B=B, V=V)
        off, w = sharded.shard_bounds(V, world)[rank]
        keys = np.zeros((B, rlsampler.PART_KEYS), np.uint64)
        stats = np.zeros(B, rlsampler.PART_STATS_DTYPE)
        for b in range(B):
            y = _penalised(batch.logits[b], batch.hist[b], batch.params["repeat_penalty"][b])
            k, st = numpy_partial(y[off:off + w], off, batch.params["temperature"][b], batch.params["top_k"][b])
            keys[b], stats[b] = k, st[0]
        kt = torch.from_numpy(keys.view(np.int64).copy())
        stt = torch.from_numpy(stats.view(np.uint8).reshape(B, -1).copy())
        rec = sharded.pack_records(kt, stt)
        assert tuple(rec.shape) == (B, rlsampler.PART_REC)
        gathered = sharded.gather_records(rec)  # one collective for keys and stats
        assert tuple(gathered.shape) == (world, B, rlsampler.PART_REC)
        kall, sall = sharded.unpack_records(gathered)
        assert tuple(kall.shape) == (world, B, rlsampler.PART_KEYS)
        assert tuple(sall.shape) == (world, B, rlsampler.PART_STATS_DTYPE.itemsize)
        np.save(os.path.join(out_dir, f"k{rank}.npy"), kall.numpy())
        np.save(os.path.join(out_dir, f"s{rank}.npy"), sall.numpy())
        np.save(os.path.join(out_dir, f"own{rank}.npy"), keys.view(np.int64))
        # the communicator id made on rank 0 reaches every rank
        uid = sharded.exchange_id(make_id=lambda: bytes(range(128)))
        np.save(os.path.join(out_dir, f"id{rank}.npy"), np.frombuffer(uid, np.uint8))
    finally:
        dist.destroy_process_group()


def test_gather_layout_and_merge_identity_two_gloo_ranks(tmp_path):
    import torch.multiprocessing as mp

    V, B, world = 4096, 6, 2
    mp.start_processes(_rank_main, args=(world, _free_port(), V, B, str(tmp_path)), nprocs=world,
                       start_method="spawn")
    k0, k1 = np.load(tmp_path / "k0.npy"), np.load(tmp_path / "k1.npy")
    assert np.array_equal(k0, k1)  # every rank holds the same gathered results
    for g in range(world):
        assert np.array_equal(np.load(tmp_path / f"id{g}.npy"), np.arange(128, dtype=np.uint8))
    for g in range(world):
        assert np.array_equal(k0[g], np.load(tmp_path / f"own{g}.npy"))  # rank g's result at index g
    stats = sharded.stats_view(np.load(tmp_path / "s0.npy"))
    keys = k0.view(np.uint64)
    batch = workloads.config5_rows(4, B=B, V=V)
    boundary = 0
    for b in range(B):
        prm = {k: batch.params[b][k].item() for k in batch.params.dtype.names}
        tok, prob = numpy_merge(keys[:, b], stats[:, b], prm["temperature"], prm["top_k"], prm["top_p"],
                                float(batch.uniforms[b]))
        r = oracle.spec_sample_row(batch.logits[b], batch.hist[b], None, prm, batch.uniforms[b])
        assert r.status == 0
        if tok != r.token:
            assert min(r.draw_margin, r.cut_margin) < BOUNDARY
            boundary += 1
        else:
            np.testing.assert_allclose(prob, r.prob, rtol=1e-5)
    assert boundary <= 1


def test_packed_records_round_trip():
    """The packed record keeps the keys and the 32-byte summary of a row."""
    B = 3
    keys = torch.arange(B * rlsampler.PART_KEYS, dtype=torch.int64).view(B, -1) * 7919
    st = np.zeros(B, rlsampler.PART_STATS_DTYPE)
    st["m"] = [1.5, -2.0, 3.25]
    st["argmax"] = [4, 5, 6]
    st["z"] = [0.5, 1.25, 9.0]
    st["n"] = [128, 3, 0]
    stats = torch.from_numpy(st.view(np.uint8).reshape(B, -1).copy())
    rec = sharded.pack_records(keys, stats)
    k2, s2 = sharded.unpack_records(rec)
    assert torch.equal(k2, keys) and torch.equal(s2, stats)
    back = sharded.stats_view(s2)
    assert np.array_equal(back, st)
