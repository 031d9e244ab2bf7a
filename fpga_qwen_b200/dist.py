"""Host-side multi-GPU logic: KV-head shards, communicator set-up, request balancing.

One process per GPU (torchrun). ``torch.distributed`` is used only to share the NCCL unique
id and for host barriers; the data path (all-gather of head-sharded outputs, KV handoff)
runs inside libqattn.so (``qa_gather_heads``, ``qa_kv_send``/``qa_kv_recv``).

* KV-head sharding: rank r of W holds KV heads [r*8/W, (r+1)*8/W) and their GQA query
  heads; the gathered output has heads in global order.
* Request sharding: independent sequences are spread over ranks by estimated cost (causal
  prefill work + decode KV reads), longest first, no collective on the data path.
* Disaggregated serving: prefill ranks hand finished KV blocks to decode ranks.
"""
from __future__ import annotations

import heapq
from datetime import timedelta

import numpy as np

N_KV_HEADS = 8
GROUP = 2
D = 128


def head_shard(rank: int, world: int, n_kv_heads: int = N_KV_HEADS):
    """(kv_head_begin, kv_head_count) held by `rank`."""
    if n_kv_heads % world:
        raise ValueError(f"{n_kv_heads} KV heads do not split over {world} ranks")
    count = n_kv_heads // world
    return rank * count, count


def gather_reference(locals_by_rank):
    """NumPy statement of qa_gather_heads: rank r's [L][n][hq_local][128] -> [L][n][W*hq_local][128]."""
    return np.concatenate(list(locals_by_rank), axis=2)


def share_unique_id(make_id, group=None) -> bytes:
    """Rank 0 creates the NCCL unique id with make_id(); every rank returns the same bytes."""
    import torch.distributed as dist
    obj = [make_id() if dist.get_rank(group) == 0 else None]
    dist.broadcast_object_list(obj, src=0, group=group)
    return obj[0]


def init_comm(ctx, group=None):
    """Joins every rank's context to one NCCL communicator."""
    import torch.distributed as dist
    from .qattn import comm_unique_id
    uid = share_unique_id(comm_unique_id, group)
    ctx.comm_init(dist.get_world_size(group), dist.get_rank(group), uid)


def request_cost(length: int, decode_steps: int) -> float:
    """Relative cost of one request: causal prefill key visits + decode key reads."""
    return length * (length + 1) / 2 + decode_steps * (length + decode_steps / 2)


def balance_requests(lengths, world: int, decode_steps: int = 128):
    """Longest-processing-time assignment of requests to ranks; returns one index list per rank."""
    heap = [(0.0, r) for r in range(world)]
    out = [[] for _ in range(world)]
    for i in sorted(range(len(lengths)), key=lambda i: -request_cost(lengths[i], decode_steps)):
        load, r = heapq.heappop(heap)
        out[r].append(i)
        heapq.heappush(heap, (load + request_cost(lengths[i], decode_steps), r))
    return [sorted(x) for x in out]


def config5_lengths(n: int = 64, lo: int = 85, hi: int = 3968, seed: int = 5):
    """Prompt lengths of the 64-request workload: n draws from U[lo, hi] with a fixed seed."""
    rng = np.random.default_rng(seed)
    return [int(x) for x in rng.integers(lo, hi + 1, n)]


def short_timeout(seconds: float = 60.0):
    return timedelta(seconds=seconds)
