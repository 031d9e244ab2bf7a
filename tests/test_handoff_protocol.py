"""The prefill -> decode KV handoff's staging and ordering protocol, restated on CPU.

qa_kv_send / qa_kv_recv (kv_transfer in csrc/qattn.cu) pipeline consecutive handoffs over two
staging buffers, used alternately (b = request index mod 2), with two streams per rank:
  sender    context stream: wait kv_comm_done[b] (the previous send from buffer b finished),
            pack the sequence's rows into buffer b, record kv_packed;
            comm stream: wait kv_packed, ncclSend(buffer b), record kv_comm_done[b];
  receiver  comm stream: wait kv_unpacked[b] (the previous unpack from buffer b finished),
            ncclRecv(buffer b), record kv_comm_done[b];
            context stream: wait kv_comm_done[b], unpack buffer b into the slot, record
            kv_unpacked[b].
Here two processes stand in for the GPUs (gloo point-to-point for NCCL), a thread per stream
runs its operations in order, and events follow CUDA's rule: a wait covers the last record
issued before the wait was issued. Random pauses interleave everything. Every received slot
must hold exactly its request's rows. Each planted variant leaves one wait out (a mistake in
this model, not in the library) and makes the operation it guards slow, so that the overwrite
it allows always happens: the check catches both.
"""
import datetime
import os
import queue
import random
import socket
import threading
import time

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

REQUESTS = 6
ROWS = [300, 17, 256, 129, 400, 64]       # rows per request (the buffers hold the largest)
WIDTH = 32                                 # values per row


def payload(i):
    n = ROWS[i]
    return (np.arange(n * WIDTH, dtype=np.int64) + 1_000_000 * (i + 1)).reshape(n, WIDTH)


class Event:
    """cudaEvent_t: record on a stream, wait from another; a wait covers the last record issued
    before it."""

    def __init__(self):
        self.issued = 0
        self.done = 0
        self.cv = threading.Condition()

    def issue_record(self):
        self.issued += 1
        return self.issued

    def complete(self, version):
        with self.cv:
            self.done = max(self.done, version)
            self.cv.notify_all()

    def wait_for(self, version):
        with self.cv:
            ok = self.cv.wait_for(lambda: self.done >= version, timeout=30)
            assert ok, "event never completed"


class Stream:
    """A stream: one thread running its operations in issue order."""

    def __init__(self, rnd):
        self.q = queue.Queue()
        self.rnd = rnd
        self.error = None
        self.t = threading.Thread(target=self._run, daemon=True)
        self.t.start()

    def _run(self):
        while True:
            op = self.q.get()
            if op is None:
                return
            try:
                op()
            except Exception as e:           # noqa: BLE001 - reported by join()
                self.error = e
                return

    def run(self, fn):
        self.q.put(fn)

    def record(self, ev):
        v = ev.issue_record()
        self.q.put(lambda: ev.complete(v))

    def wait(self, ev):
        v = ev.issued
        self.q.put(lambda: ev.wait_for(v))

    def join(self):
        self.q.put(None)
        self.t.join(timeout=60)
        if self.error:
            raise self.error


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _rank(rank, port, variant, out_dir, seed):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=2, timeout=datetime.timedelta(seconds=60))
    rnd = random.Random(seed * 7 + rank)

    def pause(scale=0.003):
        if rnd.random() < 0.5:
            time.sleep(rnd.random() * scale)

    ctx, comm = Stream(rnd), Stream(rnd)
    cap = max(ROWS) * WIDTH
    bufs = [torch.zeros(cap, dtype=torch.int64), torch.zeros(cap, dtype=torch.int64)]
    comm_done, unpacked, packed = [Event(), Event()], [Event(), Event()], Event()
    slots = {}
    for i in range(REQUESTS):
        b = i % 2
        n = ROWS[i] * WIDTH
        if rank == 0:
            if variant != "sender_no_wait":
                ctx.wait(comm_done[b])

            def pack(i=i, b=b, n=n):
                src = payload(i).reshape(-1)
                half = n // 2
                bufs[b][:half] = torch.from_numpy(src[:half])
                pause()
                bufs[b][half:n] = torch.from_numpy(src[half:])
            ctx.run(pack)
            ctx.record(packed)
            comm.wait(packed)

            def send(i=i, b=b, n=n):
                # the planted variant's transfer is slow, so the next pack into b lands first
                time.sleep(0.08 if variant == "sender_no_wait" and i == 0 else rnd.random() * 0.003)
                dist.send(bufs[b][:n].clone(), dst=1)
            comm.run(send)
            comm.record(comm_done[b])
        else:
            if variant != "receiver_no_wait":
                comm.wait(unpacked[b])

            def recv(b=b, n=n):
                pause()
                t = torch.empty(n, dtype=torch.int64)
                dist.recv(t, src=0)
                bufs[b][:n] = t
            comm.run(recv)
            comm.record(comm_done[b])
            ctx.wait(comm_done[b])

            def unpack(i=i, b=b, n=n):
                half = n // 2
                first = bufs[b][:half].clone()
                # the planted variant's unpack is slow, so the next receive into b lands first
                time.sleep(0.08 if variant == "receiver_no_wait" and i == 0 else rnd.random() * 0.003)
                slots[i] = torch.cat([first, bufs[b][half:n].clone()]).numpy().reshape(ROWS[i], WIDTH)
            ctx.run(unpack)
            ctx.record(unpacked[b])
    ctx.join()
    comm.join()
    if rank == 1:
        ok = [bool(np.array_equal(slots[i], payload(i))) for i in range(REQUESTS)]
        np.save(os.path.join(out_dir, f"{variant}_{seed}.npy"), np.array(ok))
    dist.barrier()
    dist.destroy_process_group()


def _run(tmp_path, variant, seed):
    mp.start_processes(_rank, args=(_free_port(), variant, str(tmp_path), seed), nprocs=2, start_method="spawn")
    return np.load(tmp_path / f"{variant}_{seed}.npy")


@pytest.mark.parametrize("seed", [1, 2, 3])
def test_pipelined_handoffs_deliver_every_request_intact(tmp_path, seed):
    assert _run(tmp_path, "protocol", seed).all()


@pytest.mark.parametrize("variant", ["sender_no_wait", "receiver_no_wait"])
def test_a_missing_wait_is_caught(tmp_path, variant):
    ok = _run(tmp_path, variant, 1)
    assert not ok.all(), "the planted overwrite went unnoticed"
