"""The head-gather flag protocols, restated on CPU with processes standing in for GPUs.

qa_attn_prefill_gather (csrc/qattn.cu) runs, per call k, on every rank r:
  gate        prefill_gate_kernel: mark "r copied call k-1 out of its landing buffer" in every
              peer's flag array (PF_ACK + r), then wait until every peer marked the same;
  compute     the prefill kernels store r's output rows into r's own output and into every
              peer's landing buffer (peer stores);
  signal      prefill_signal_kernel: mark "r's rows of call k are stored" (PF_READY + r) in
              every peer's flag array;
  wait/copy   prefill_wait_copy_kernel: wait for every peer's ready mark of call k, then copy
              the peers' rows from r's landing buffer into r's output.
qa_decode_step_gather has no acknowledgement: its landing buffers alternate by step, the
decode kernel's last CTA marks "r finished step s" (word r) in every rank's flag array after all
of r's stores, and gather_wait_copy_kernel waits for every rank's mark, then copies.
Here shared arrays stand in for the peer-mapped flag arrays and landing buffers, and random
pauses interleave the ranks. Every copy must read the rows of its own call: a landing buffer
may not be rewritten before its owner has copied it. The planted variant without the gate
(a mistake in this model, not in the library) shows the check catches that overwrite; so
does the decode variant with a single landing buffer.
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


@pytest.mark.parametrize("nranks", [2, 4, 8])
def test_every_copy_reads_its_own_call(nranks):
    assert run_protocol(nranks, calls=12, seed=nranks) == [0] * nranks


def test_slow_copy_holds_back_the_peers():
    assert run_protocol(2, calls=4, slow_copy_rank=1) == [0, 0]


def test_planted_missing_gate_is_caught():
    errors = run_protocol(2, calls=4, gate=False, slow_copy_rank=1)
    assert errors[1] > 0          # rank 0 rewrote rank 1's landing buffer during its copy


def _rank_decode(rank, nranks, steps, buffers, slow_copy_rank, flags, landing, errors, seed):
    rnd = random.Random(seed * 103 + rank)
    deadline = time.monotonic() + 60
    size = nranks * ROWS
    out = [0] * size
    for st in range(1, steps + 1):
        base = (st % buffers) * nranks * size                  # landing buffer of this step
        for i in range(ROWS):                                  # the decode kernel's stores, every rank
            v = value(st, rank, i)
            for p in range(nranks):
                landing[base + p * size + rank * ROWS + i] = v
            if rnd.random() < 0.05:
                time.sleep(rnd.random() * 0.002)
        for p in range(nranks):                                # the last CTA's marks
            flags[p * WORDS + rank] = st
        if not _wait(flags, rank, 0, nranks, st, deadline) or flags[rank * WORDS + rank] < st:
            errors[rank] = -51
            return
        for i in range(size):                                  # gather_wait_copy_kernel
            if rank == slow_copy_rank and i == 0:
                time.sleep(0.05)                               # a slow copy: peers run ahead
            out[i] = landing[base + rank * size + i]
        for p in range(nranks):
            for i in range(ROWS):
                if out[p * ROWS + i] != value(st, p, i):
                    errors[rank] += 1


def run_decode_protocol(nranks, steps, buffers=2, slow_copy_rank=-1, seed=0):
    ctx = mp.get_context("spawn")
    flags = ctx.Array("q", nranks * WORDS, lock=False)
    landing = ctx.Array("q", buffers * nranks * nranks * ROWS, lock=False)
    errors = ctx.Array("q", nranks, lock=False)
    procs = [ctx.Process(target=_rank_decode,
                         args=(r, nranks, steps, buffers, slow_copy_rank, flags, landing, errors, seed))
             for r in range(nranks)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(120)
        assert p.exitcode == 0
    return list(errors)


@pytest.mark.parametrize("nranks", [2, 4, 8])
def test_decode_gather_alternating_buffers(nranks):
    assert run_decode_protocol(nranks, steps=16, seed=nranks) == [0] * nranks
    assert run_decode_protocol(nranks, steps=4, slow_copy_rank=nranks - 1) == [0] * nranks


def test_planted_single_decode_buffer_is_caught():
    errors = run_decode_protocol(2, steps=4, buffers=1, slow_copy_rank=1)
    assert errors[1] > 0          # rank 0's next step rewrote the buffer rank 1 was copying
