"""Vocabulary-sharded sampling over ranks (one process per GPU).

A row's logits are split by vocabulary across the ranks of a process group:
rank g holds columns [offset_g, offset_g + width_g). Each step every rank
calls rl_sample_sharded, which

  1. streams only the rank's columns (penalties, mask, temperature, the
     shard's sorted top-min(top_k, 128) list and its softmax sum relative to
     the shard's max) into one packed record per row (1056 bytes),
  2. all-gathers the records of every rank with a single ncclAllGather on
     the library's own NCCL communicator,
  3. merges the G records into the row's token.

Every rank then holds the same tokens, equal to sampling the whole row in
one piece up to the order in which the softmax sums are added. The
all-gather is the only collective on the path. The communicator is made
with rl_nccl_comm_init from an id that rank 0 makes and the process group
broadcasts (any torch.distributed backend carries the 128 bytes).

gather_records is the same exchange done by torch.distributed (one
all_gather_into_tensor of the packed records): the layout rl_sample_sharded
hands to its merge, usable with any backend -- the CPU tests run it on gloo.
"""
from __future__ import annotations

import numpy as np

import rlsampler

# columns per shard boundary: 8 bf16 / 4 f32 logits keep each shard's row
# start on a 16-byte boundary when the full row is
SHARD_ALIGN = 8


def shard_bounds(V: int, world: int, align: int = SHARD_ALIGN):
    """Contiguous split of V columns into `world` shards whose offsets are
    multiples of `align`; returns [(offset, width)] per rank."""
    if world < 1 or V < 1:
        raise ValueError(f"shard_bounds: V={V} world={world}")
    step = -(-V // world)
    step = -(-step // align) * align
    out = []
    for g in range(world):
        lo = min(g * step, V)
        hi = min(lo + step, V)
        if hi <= lo:
            raise ValueError(f"shard_bounds: V={V} leaves rank {g} of {world} without columns")
        out.append((lo, hi - lo))
    return out


def pack_records(keys, stats):
    """keys [B, 128] int64 and stats [B, 32] uint8 (one rank's partial
    results) -> packed records [B, 132] int64: the 128 keys, then the 32-byte
    rl_part_stats, as rl_sample_sharded lays a row out."""
    import torch

    B = keys.shape[0]
    rec = torch.empty((B, rlsampler.PART_REC), dtype=torch.int64, device=keys.device)
    rec[:, : rlsampler.PART_KEYS] = keys
    rec[:, rlsampler.PART_KEYS:] = stats.contiguous().view(torch.int64).view(B, 4)
    return rec


def unpack_records(rec):
    """Packed records [..., 132] int64 -> (keys [..., 128] int64, stats [..., 32] uint8)."""
    import torch

    keys = rec[..., : rlsampler.PART_KEYS]
    stats = rec[..., rlsampler.PART_KEYS:].contiguous().view(torch.uint8)
    return keys, stats


def gather_records(rec, group=None):
    """One all-gather of every rank's packed records [B, 132] into the
    shard-major [G, B, 132] layout (rank g's records at index g)."""
    import torch
    import torch.distributed as dist

    G = dist.get_world_size(group)
    B = rec.shape[0]
    out = torch.empty((G * B, rec.shape[1]), dtype=rec.dtype, device=rec.device)
    dist.all_gather_into_tensor(out, rec.contiguous(), group=group)
    return out.view(G, B, rec.shape[1])


def exchange_id(group=None, make_id=None) -> bytes:
    """Rank 0 makes a communicator id (rl_nccl_unique_id unless make_id is
    given) and the group broadcasts it; every rank returns the same bytes."""
    import torch.distributed as dist

    make = make_id or rlsampler.nccl_unique_id
    box = [make() if dist.get_rank(group) == 0 else None]
    src = 0 if group is None else dist.get_global_rank(group, 0)
    dist.broadcast_object_list(box, src=src, group=group)
    return bytes(box[0])


class ShardedSampler:
    """Samples rows whose vocabulary is split across the ranks of `group`
    (one rank per GPU), through rl_sample_sharded and an NCCL communicator of
    its own."""

    def __init__(self, V: int, max_batch: int, group=None, device=None, max_history: int = 1024):
        import torch
        import torch.distributed as dist

        self.group = group
        self.rank = dist.get_rank(group)
        self.world = dist.get_world_size(group)
        if self.world > 16:
            raise ValueError("rl_sample_sharded takes at most 16 ranks")
        self.V = V
        self.bounds = shard_bounds(V, self.world)
        self.offset, self.width = self.bounds[self.rank]
        dev = torch.device("cuda", torch.cuda.current_device()) if device is None else torch.device(device)
        self.device = dev
        self.sampler = rlsampler.Sampler(dev.index or 0, max_batch=max_batch, max_vocab=self.width,
                                         max_history=max_history, flags=rlsampler.RL_CREATE_SHARDED)
        uid = exchange_id(group)
        with torch.cuda.device(dev):
            self.comm = rlsampler.nccl_comm_init(self.world, uid, self.rank)

    def sample(self, logits_shard, params, uniforms, hist=None, hist_len=None, mask_shard=None, out_tok=None,
               out_prob=None, row_status=None, stream=None):
        """logits_shard [B, width] (this rank's columns, f32 or bf16);
        params / uniforms / hist as rlsampler.Sampler.sample (history ids
        global). Returns (tokens, probs, row_status) with global ids, the
        same on every rank."""
        if logits_shard.shape[1] != self.width:
            raise ValueError(f"rank {self.rank}: shard has {logits_shard.shape[1]} columns, expected {self.width}")
        return self.sampler.sample_sharded(self.comm, logits_shard, self.offset, self.V, params, uniforms, hist,
                                           hist_len, mask_shard, out_tok, out_prob, row_status, stream)

    def close(self):
        if self.comm:
            rlsampler.nccl_comm_destroy(self.comm)
            self.comm = 0
        self.sampler.close()


def stats_view(stats) -> np.ndarray:
    """Host view of gathered stats bytes [..., 32] as rl_part_stats records."""
    a = np.ascontiguousarray(stats.cpu().numpy() if hasattr(stats, "cpu") else stats)
    return a.view(rlsampler.PART_STATS_DTYPE).reshape(a.shape[:-1])
