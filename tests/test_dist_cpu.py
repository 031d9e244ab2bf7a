"""Multi-process host logic on CPU (gloo, world size 2): head shards, the gather layout,
request balancing, and failure detection of a rank that never joins. No GPU."""
import os
import socket
import time

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from fpga_qwen_b200 import dist as qd


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _init(rank, world, port, timeout=30):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=qd.short_timeout(timeout))


def _gather_worker(rank, world, port, out_dir):
    _init(rank, world, port)
    L, n = 3, 5
    begin, count = qd.head_shard(rank, world)
    hq_local = qd.GROUP * count
    # local output of this rank: value encodes (layer, row, global q head, channel)
    local = np.zeros((L, n, hq_local, qd.D), np.float32)
    for h in range(hq_local):
        gh = qd.GROUP * begin + h
        local[:, :, h, :] = gh * 1000 + np.arange(L)[:, None, None] * 100 + np.arange(n)[None, :, None] + \
            np.arange(qd.D)[None, None, :] * 1e-3
    parts = [torch.empty_like(torch.from_numpy(local)) for _ in range(world)]
    dist.all_gather(parts, torch.from_numpy(local))
    full = qd.gather_reference([p.numpy() for p in parts])
    np.save(os.path.join(out_dir, f"full{rank}.npy"), full)
    # the NCCL unique-id sharing path, with a stand-in id maker
    uid = qd.share_unique_id(lambda: bytes(range(128)))
    assert uid == bytes(range(128))
    dist.barrier()
    dist.destroy_process_group()


def test_head_shards_and_gather_layout(tmp_path):
    world = 2
    port = _free_port()
    mp.start_processes(_gather_worker, args=(world, port, str(tmp_path)), nprocs=world, start_method="spawn")
    for rank in range(world):
        full = np.load(tmp_path / f"full{rank}.npy")
        assert full.shape == (3, 5, 16, 128)
        for gh in range(16):
            expect = gh * 1000 + np.arange(3)[:, None, None] * 100 + np.arange(5)[None, :, None] + \
                np.arange(128)[None, None, :] * 1e-3
            assert np.allclose(full[:, :, gh, :], expect)


@pytest.mark.parametrize("world", [1, 2, 4, 8])
def test_head_shard_partition(world):
    heads = []
    for r in range(world):
        b, c = qd.head_shard(r, world)
        heads += list(range(b, b + c))
    assert heads == list(range(8))
    with pytest.raises(ValueError):
        qd.head_shard(0, 3)


def test_request_balancing_config5():
    lengths = qd.config5_lengths()
    assert len(lengths) == 64 and min(lengths) >= 85 and max(lengths) <= 3968
    assert lengths == qd.config5_lengths()                     # seeded
    for world in (1, 2, 4, 8):
        parts = qd.balance_requests(lengths, world)
        assert sorted(i for p in parts for i in p) == list(range(64))
        loads = [sum(qd.request_cost(lengths[i], 128) for i in p) for p in parts]
        assert max(loads) / (sum(loads) / world) < 1.10        # within 10% of perfect balance


def _dead_peer_worker(rank, world, port, out_dir):
    if rank == 1:
        return                                                  # this rank never joins
    t0 = time.time()
    try:
        _init(rank, world, port, timeout=5)
        dist.barrier()
        ok = False
    except Exception:
        ok = True
    with open(os.path.join(out_dir, "rank0.txt"), "w") as f:
        f.write(f"{ok} {time.time() - t0:.1f}")


def test_rank_that_never_joins_is_detected(tmp_path):
    """A peer that dies before joining surfaces as an error on the host within the short
    process-group timeout, not as a hang."""
    world = 2
    port = _free_port()
    mp.start_processes(_dead_peer_worker, args=(world, port, str(tmp_path)), nprocs=world, start_method="spawn")
    ok, secs = (tmp_path / "rank0.txt").read_text().split()
    assert ok == "True" and float(secs) < 60
