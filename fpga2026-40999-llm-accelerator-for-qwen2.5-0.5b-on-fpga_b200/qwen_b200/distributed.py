"""Host logic of the multi-GPU decode: one process per GPU, each rank holding a
full replica and its own requests (no data-path collective), plus the
optional vocab-sharded LM head whose per-rank (value, index) candidates are
combined with one all-gather. The reference has no multi-device path; the
argmax rule (highest index on ties) is model_backend.py:113-114.

Collectives go through torch.distributed with whatever backend the process
group was created with: NCCL over NVLink on the GPU box (tensors on the
current CUDA device), gloo on CPU in the tests.
"""
import numpy as np


def shard_requests(n_requests, world, rank):
    """Contiguous block of request ids owned by `rank`: the first
    n_requests % world ranks hold one extra request."""
    if world < 1 or not 0 <= rank < world or n_requests < 0:
        raise ValueError('bad shard request')
    base, extra = divmod(n_requests, world)
    start = rank * base + min(rank, extra)
    return range(start, start + base + (1 if rank < extra else 0))


def vocab_shard(vocab, world, rank):
    """[begin, end) of the LM-head rows rank `rank` computes; every shard but
    possibly the last is a multiple of 128 rows (whole tensor-core tiles)."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError('bad shard request')
    per = -(-vocab // world)
    per = -(-per // 128) * 128
    begin = min(vocab, rank * per)
    return begin, min(vocab, begin + per)


def _device(group=None):
    import torch
    import torch.distributed as dist
    backend = dist.get_backend(group)
    return torch.device('cuda', torch.cuda.current_device()) if backend == 'nccl' else torch.device('cpu')


def reduce_over_ranks(value, op='max', group=None):
    """max or sum of a host scalar over all ranks (float64)."""
    import torch
    import torch.distributed as dist
    if not dist.is_initialized() or dist.get_world_size(group) == 1:
        return float(value)
    t = torch.tensor([float(value)], dtype=torch.float64, device=_device(group))
    dist.all_reduce(t, op=dist.ReduceOp.MAX if op == 'max' else dist.ReduceOp.SUM, group=group)
    return float(t.item())


def better(v, i, bv, bi):
    """(v, i) beats (bv, bi): larger value, or equal value and larger index."""
    return v > bv or (v == bv and i > bi)


def combine_candidates(values, indices):
    """values, indices [ranks][rows] -> best index per row over the ranks
    (largest value, highest index on ties)."""
    values = np.asarray(values, dtype=np.float32)
    indices = np.asarray(indices, dtype=np.int64)
    out = np.empty(values.shape[1], dtype=np.int64)
    for r in range(values.shape[1]):
        bv, bi = values[0, r], indices[0, r]
        for k in range(1, values.shape[0]):
            if better(values[k, r], indices[k, r], bv, bi):
                bv, bi = values[k, r], indices[k, r]
        out[r] = bi
    return out


def allgather_argmax(local_values, local_indices, group=None):
    """Every rank contributes its rows' best (value, global index) over its
    vocab shard; returns the best index per row over all shards, the same on
    every rank."""
    import torch
    import torch.distributed as dist
    dev = _device(group)
    world = dist.get_world_size(group)
    v = torch.as_tensor(np.asarray(local_values, dtype=np.float32), device=dev)
    i = torch.as_tensor(np.asarray(local_indices, dtype=np.int64), device=dev)
    vs = [torch.empty_like(v) for _ in range(world)]
    is_ = [torch.empty_like(i) for _ in range(world)]
    dist.all_gather(vs, v, group=group)
    dist.all_gather(is_, i, group=group)
    return combine_candidates(np.stack([t.cpu().numpy() for t in vs]), np.stack([t.cpu().numpy() for t in is_]))
