"""The prefill head-gather flag protocol, restated on CPU with processes standing in for GPUs.

qa_attn_prefill_gather (csrc/qattn.cu) runs, per call k, on every rank r:
  gate        prefill_gate_kernel: mark "r copied call k-1 out of its landing buffer" in every
              peer's flag array (PF_ACK + r), then wait until every peer marked the same;
  compute     the prefill kernels store r's output rows into r's own output and into every
              peer's landing buffer (peer stores);
  signal      prefill_signal_kernel: mark "r's rows of call k are stored" (PF_READY + r) in
              every peer's flag array;
  wait/copy   prefill_wait_copy_kernel: wait for every peer's ready mark of call k, then copy
              the peers' rows from r's landing buffer into r's output.
Here shared arrays stand in for the peer-mapped flag arrays and landing buffers, and random
pauses interleave the ranks. Every copy must read the rows of its own call: a landing buffer
may not be rewritten before its owner has copied it. The planted variant without the gate
(a mistake in this model, not in the library) shows the check catches that overwrite.
"""
import multiprocessing as mp
import random
import time

import pytest

PF_READY, PF_ACK, WORDS = 16, 32, 64
ROWS = 64                  # rows each rank contributes per call


def value(call, rank, i):
    return call * 1_000_000 + rank * 1_000 + i


def _wait(flags, rank, base, nranks, target, deadline):
    for p in range(nranks):
        if p == rank:
            continue
        while flags[rank * WORDS + base + p] < target:
            if time.monotonic() > deadline:
                return False
            time.sleep(0.0002)
    return True


def _rank(rank, nranks, calls, gate, slow_copy_rank, flags, landing, errors, seed):
    rnd = random.Random(seed * 101 + rank)
    deadline = time.monotonic() + 60
    out = [0] * (nranks * ROWS)
    for k in range(1, calls + 1):
        if gate:
            for p in range(nranks):
                if p != rank:
                    flags[p * WORDS + PF_ACK + rank] = k - 1
            if not _wait(flags, rank, PF_ACK, nranks, k - 1, deadline):
                errors[rank] = -52
                return
        for i in range(ROWS):                                  # compute: local and peer stores
            v = value(k, rank, i)
            out[rank * ROWS + i] = v
            for p in range(nranks):
                if p != rank:
                    landing[p * nranks * ROWS + rank * ROWS + i] = v
            if rnd.random() < 0.05:
                time.sleep(rnd.random() * 0.002)
        for p in range(nranks):                                # signal
            if p != rank:
                flags[p * WORDS + PF_READY + rank] = k
        if not _wait(flags, rank, PF_READY, nranks, k, deadline):
            errors[rank] = -53
            return
        for p in range(nranks):                                # copy the peers' rows
            if p == rank:
                continue
            for i in range(ROWS):
                if rank == slow_copy_rank and i == ROWS // 2:
                    time.sleep(0.05)                           # a slow copy: peers run ahead
                out[p * ROWS + i] = landing[rank * nranks * ROWS + p * ROWS + i]
        for p in range(nranks):
            for i in range(ROWS):
                if out[p * ROWS + i] != value(k, p, i):
                    errors[rank] += 1


def run_protocol(nranks, calls, gate=True, slow_copy_rank=-1, seed=0):
    ctx = mp.get_context("spawn")
    flags = ctx.Array("q", nranks * WORDS, lock=False)
    landing = ctx.Array("q", nranks * nranks * ROWS, lock=False)
    errors = ctx.Array("q", nranks, lock=False)
    procs = [ctx.Process(target=_rank, args=(r, nranks, calls, gate, slow_copy_rank, flags, landing, errors, seed))
             for r in range(nranks)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(120)
        assert p.exitcode == 0
    return list(errors)


@pytest.mark.parametrize("nranks", [2, 4])
def test_every_copy_reads_its_own_call(nranks):
    assert run_protocol(nranks, calls=12, seed=nranks) == [0] * nranks


def test_slow_copy_holds_back_the_peers():
    assert run_protocol(2, calls=4, slow_copy_rank=1) == [0, 0]


def test_planted_missing_gate_is_caught():
    errors = run_protocol(2, calls=4, gate=False, slow_copy_rank=1)
    assert errors[1] > 0          # rank 0 rewrote rank 1's landing buffer during its copy
