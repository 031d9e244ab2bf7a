"""Two-GPU tests of the multi-GPU entry points (run on a box with >= 2 GPUs; skipped otherwise).

* KV-head sharding: each rank holds 4 of the 8 KV heads; prefill + decode outputs gathered
  with qa_gather_heads equal a single-GPU context holding all heads (within the attention
  tolerance), and each rank's KV bytes equal the matching heads of the single-GPU store.
* Prefill -> decode handoff: rank 0 appends three sequences and ships their KV rows to
  rank 1 back to back with qa_kv_send/qa_kv_recv (double-buffered staging, so the third
  transfer reuses the first buffer); rank 1's KV bytes equal the same sequences appended
  locally, bit for bit, and its positions are the sent row counts.
* Fused decode step with the head gather done by the kernel (qa_decode_step_gather: peer
  stores over NVLink, or NCCL where peer mapping is unavailable) equals a full-head
  context's fused decode step on every rank.
NVLS is switched off (NCCL_NVLS_ENABLE=0) and ranks leave only between steps.
"""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from tests import helpers as H

pytestmark = [pytest.mark.gpu,
              pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2,
                                 reason="needs two GPUs")]


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _worker(rank, world, port, out_dir):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    from fpga_qwen_b200 import dist as qd
    from fpga_qwen_b200 import qattn
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=qd.short_timeout(120))
    L, n, steps = 4, 300, 3
    begin, count = qd.head_shard(rank, world)
    stream = torch.cuda.current_stream().cuda_stream
    shard = qattn.Context(n_layers=L, context=1024, max_seqs=2, kv_head_begin=begin, kv_head_count=count,
                          device=rank)
    shard.set_stream(stream)
    full = qattn.Context(n_layers=L, context=1024, max_seqs=2, device=rank)
    full.set_stream(stream)
    qd.init_comm(shard)
    qw, kw = H.norms(77, L)
    H.set_norms(shard, qw, kw)
    H.set_norms(full, qw, kw)
    # all-head inputs, and this rank's slice of them
    q, k, v = H.inputs(77, L, 0, n + steps)
    hq = 2 * count
    qs, ks, vs = (q[:, :, 2 * begin:2 * begin + hq].contiguous(), k[:, :, begin:begin + count].contiguous(),
                  v[:, :, begin:begin + count].contiguous())
    report = {}
    keep = []

    def run(ctx, qq, kk, vv, gather):
        outs = []
        qn = torch.empty_like(qq[:, :n])
        # keep the contiguous copies alive until the queued kernels have read them
        qp, kp, vp = qq[:, :n].contiguous(), kk[:, :n].contiguous(), vv[:, :n].contiguous()
        keep.extend((qp, kp, vp))
        ctx.append(0, 0, L, 0, n, qp.data_ptr(), kp.data_ptr(), vp.data_ptr(), qn.data_ptr())
        out = torch.empty_like(qn)
        ctx.attn_prefill(0, 0, L, 0, n, qn.data_ptr(), out.data_ptr())
        ctx.commit(0, n)
        outs.append(out)
        for s in range(steps):
            p = n + s
            qn1 = torch.empty_like(qq[:, p:p + 1])
            q1, k1, v1 = qq[:, p:p + 1].contiguous(), kk[:, p:p + 1].contiguous(), vv[:, p:p + 1].contiguous()
            keep.extend((q1, k1, v1))
            ctx.append(0, 0, L, p, 1, q1.data_ptr(), k1.data_ptr(), v1.data_ptr(), qn1.data_ptr())
            o = torch.empty_like(qn1)
            ctx.attn_decode(0, 0, L, p, 1, qn1.data_ptr(), o.data_ptr())
            ctx.commit(0, 1)
            outs.append(o)
        local = torch.cat(outs, dim=1).contiguous()
        report["local_" + ("shard" if gather else "full")] = local.cpu().numpy()
        if not gather:
            return local
        g = torch.empty((L, n + steps, 16, 128), dtype=torch.float32, device="cuda")
        ctx.gather_heads(L, n + steps, local.data_ptr(), g.data_ptr())
        # the same gather in layer groups on the communication stream (groups of 1 and 3 layers),
        # with other work queued on the context stream meanwhile: the same bits
        ga = torch.full_like(g, float("nan"))
        t = n + steps
        # filler: the next (uncommitted) row appended again and attended, twice
        ctx.append(0, 0, L, t, 1, q1.data_ptr(), k1.data_ptr(), v1.data_ptr(), qn1.data_ptr())
        for l0, nl in ((0, 1), (1, 3)):
            ctx.gather_heads_async(nl, t, local[l0:].data_ptr(), ga[l0:].data_ptr())
            scratch = torch.empty_like(qn1)
            keep.append(scratch)
            ctx.attn_decode(0, 0, L, t, 1, qn1.data_ptr(), scratch.data_ptr())
        ctx.comm_join()
        torch.cuda.synchronize()
        report["async_gather_equal"] = bool(torch.equal(ga, g))
        # prefill with the head gather inside the kernels (peer stores): the same bits as
        # qa_attn_prefill + qa_gather_heads, for a whole prefill twice in a row (the second
        # call reuses the landing buffers) and a chunk starting at position 128
        ctx.reset(1)
        qn_b = torch.empty_like(qn)
        keep.append(qn_b)
        ctx.append(1, 0, L, 0, n, qp.data_ptr(), kp.data_ptr(), vp.data_ptr(), qn_b.data_ptr())
        pf_equal = True
        for pos0, cnt, reps in ((0, n, 2), (128, n - 128, 1)):
            if pos0:
                ctx.commit(1, pos0)
            qrows = qn_b[:, pos0:pos0 + cnt].contiguous()
            loc = torch.empty((L, cnt, hq, 128), dtype=torch.float32, device="cuda")
            ref = torch.empty((L, cnt, 16, 128), dtype=torch.float32, device="cuda")
            keep.extend((qrows, loc, ref))
            ctx.attn_prefill(1, 0, L, pos0, cnt, qrows.data_ptr(), loc.data_ptr())
            ctx.gather_heads(L, cnt, loc.data_ptr(), ref.data_ptr())
            for _ in range(reps):
                got = torch.full_like(ref, float("nan"))
                ctx.attn_prefill_gather(1, 0, L, pos0, cnt, qrows.data_ptr(), got.data_ptr())
                ctx.sync()
                pf_equal &= bool(torch.equal(got, ref))
        report["prefill_gather_equal"] = pf_equal
        return g

    gathered = run(shard, qs, ks, vs, gather=True)
    reference = run(full, q, k, v, gather=False)
    torch.cuda.synchronize()
    mx, rms = H.err_stats(gathered.cpu().numpy(), reference.cpu().numpy())
    report["gather_max"], report["gather_rms"] = mx, rms
    lmx, lrms = H.err_stats(report.pop("local_shard"), report.pop("local_full")[:, :, 2 * begin:2 * begin + hq])
    report["local_max"], report["local_rms"] = lmx, lrms
    kv_equal = True
    for layer in range(L):
        for h in range(count):
            for kvsel in (0, 1):
                a = H.read_plane(shard, 0, layer, kvsel, h, 0, n + steps)
                b = H.read_plane(full, 0, layer, kvsel, begin + h, 0, n + steps)
                kv_equal &= bool(np.array_equal(a, b))
    report["kv_equal"] = kv_equal

    # prefill -> decode handoff of three sequences back to back (the third reuses the first
    # staging buffer): rank 0 sends its slots 0, 1, 2, rank 1 receives them into slots 1, 2, 3
    # and compares every plane with the same sequences appended locally
    dist.barrier()
    lens = (n, 150, 257)
    full_comm = qattn.Context(n_layers=L, context=1024, max_seqs=4, device=rank)
    full_comm.set_stream(stream)
    H.set_norms(full_comm, qw, kw)
    qd.init_comm(full_comm)
    local_ref = qattn.Context(n_layers=L, context=1024, max_seqs=3, device=rank)
    local_ref.set_stream(stream)
    H.set_norms(local_ref, qw, kw)
    for i, ln in enumerate(lens):
        qi, ki, vi = H.inputs(300 + i, L, 0, ln)
        keep.extend((qi, ki, vi))
        dst = full_comm if rank == 0 else local_ref
        qn_i = torch.empty_like(qi)
        keep.append(qn_i)
        dst.append(i, 0, L, 0, ln, qi.data_ptr(), ki.data_ptr(), vi.data_ptr(), qn_i.data_ptr())
        dst.commit(i, ln)
    for i, ln in enumerate(lens):
        if rank == 0:
            full_comm.kv_send(i, ln, 1)
        else:
            full_comm.kv_recv(i + 1, ln, 0)
    full_comm.sync()
    local_ref.sync()
    if rank == 1:
        same = True
        for i, ln in enumerate(lens):
            for layer in range(L):
                for h in range(8):
                    for kvsel in (0, 1):
                        same &= bool(np.array_equal(H.read_plane(full_comm, i + 1, layer, kvsel, h, 0, ln),
                                                    H.read_plane(local_ref, i, layer, kvsel, h, 0, ln)))
        report["handoff_equal"] = same
        report["handoff_pos"] = [full_comm.position(i + 1) for i in range(3)]
    # fused decode step with the head gather done over peer memory (qa_decode_step_gather)
    # against the full-head context's fused decode step
    dist.barrier()
    P, gsteps = 300, 3                        # the inputs hold rows [0, 303)
    g_shard = qattn.Context(n_layers=L, context=1024, max_seqs=1, kv_head_begin=begin, kv_head_count=count,
                            device=rank)
    g_full = qattn.Context(n_layers=L, context=1024, max_seqs=1, device=rank)
    for c in (g_shard, g_full):
        c.set_stream(stream)
        H.set_norms(c, qw, kw)
    qd.init_comm(g_shard)
    g_shard.set_step_overlap(True)                 # steps and gather waits chained by dependent launch
    report["peer_mapped"] = g_shard.comm_info()[2]
    hist_s = [t[:, :P].contiguous() for t in (qs, ks, vs)]
    hist_f = [t[:, :P].contiguous() for t in (q, k, v)]
    keep.extend(hist_s + hist_f)
    for c, hh in ((g_shard, hist_s), (g_full, hist_f)):
        qn_h = torch.empty_like(hh[0])
        keep.append(qn_h)
        c.append(0, 0, L, 0, P, hh[0].data_ptr(), hh[1].data_ptr(), hh[2].data_ptr(), qn_h.data_ptr())
        c.commit(0, P)
    gmax = 0.0
    for st in range(gsteps):
        p = P + st
        s1 = [t[:, p:p + 1].contiguous() for t in (qs, ks, vs)]
        f1 = [t[:, p:p + 1].contiguous() for t in (q, k, v)]
        keep.extend(s1 + f1)
        got = torch.full((L, 1, 16, 128), float("nan"), device="cuda")
        ref = torch.empty((L, 1, 16, 128), device="cuda")
        g_shard.decode_step_gather(0, 0, L, p, s1[0].data_ptr(), s1[1].data_ptr(), s1[2].data_ptr(), 0, got.data_ptr())
        g_full.decode_step(0, 0, L, p, f1[0].data_ptr(), f1[1].data_ptr(), f1[2].data_ptr(), 0, ref.data_ptr())
        g_shard.commit(0, 1)
        g_full.commit(0, 1)
        torch.cuda.synchronize()
        gmax = max(gmax, H.err_stats(got.cpu().numpy(), ref.cpu().numpy())[0])
    g_shard.sync()
    report["peer_gather_max"] = gmax
    dist.barrier()
    g_shard.comm_destroy()
    full_comm.comm_destroy()
    shard.comm_destroy()
    np.save(os.path.join(out_dir, f"report{rank}.npy"), report, allow_pickle=True)
    dist.destroy_process_group()


def test_head_sharded_gather_and_kv_handoff(tmp_path):
    world = 2
    mp.start_processes(_worker, args=(world, _free_port(), str(tmp_path)), nprocs=world, start_method="spawn")
    for rank in range(world):
        rep = np.load(tmp_path / f"report{rank}.npy", allow_pickle=True).item()
        assert rep["kv_equal"], rep
        assert rep["async_gather_equal"], rep
        assert rep["prefill_gather_equal"], rep
        assert rep["gather_max"] < H.MAX_ABS and rep["gather_rms"] < H.RMS, rep
        assert rep["peer_gather_max"] < 1e-5, rep             # same heads, different key split
        if rank == 1:
            assert rep["handoff_equal"] and rep["handoff_pos"] == [300, 150, 257], rep


def _skip_worker(rank, world, port, out_dir):
    """Rank 1 leaves one gathering call out (between steps, nothing of its own in flight); rank
    0's bounded wait for rank 1's mark runs out after the lowered limit and its qa_sync reports
    QA_ERR_TIMEOUT, after which rank 0's context keeps working. Done once for the decode step's
    gather (error code 51: the wait for the peers' "step done" marks) and once for the
    prefill's (code 52: the gate's wait for the peers' "landing buffer free" marks)."""
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    from fpga_qwen_b200 import dist as qd
    from fpga_qwen_b200 import qattn
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=qd.short_timeout(120))
    L, P = 2, 200
    begin, count = qd.head_shard(rank, world)
    stream = torch.cuda.current_stream().cuda_stream
    q, k, v = H.inputs(81, L, 0, P + 2)
    qs, ks, vs = (q[:, :, 2 * begin:2 * begin + 2 * count].contiguous(), k[:, :, begin:begin + count].contiguous(),
                  v[:, :, begin:begin + count].contiguous())
    report = {}
    for kind in ("decode", "prefill"):
        ctx = qattn.Context(n_layers=L, context=512, max_seqs=1, kv_head_begin=begin, kv_head_count=count,
                            device=rank)
        ctx.set_stream(stream)
        qd.init_comm(ctx)
        mapped = ctx.comm_info()[2]
        flags = [None, None]
        dist.all_gather_object(flags, mapped)
        report[kind + "_mapped"] = all(flags)
        if not all(flags):          # the NCCL fallback has no bounded wait to exercise: skip
            ctx.comm_destroy()
            ctx.close()
            continue
        ctx.set_wait_limit(200000)                      # 200 ms
        hist = [t[:, :P].contiguous() for t in (qs, ks, vs)]
        qn = torch.empty_like(hist[0])
        ctx.append(0, 0, L, 0, P, hist[0].data_ptr(), hist[1].data_ptr(), hist[2].data_ptr(), qn.data_ptr())
        full = torch.empty((L, P, 16, 128), device="cuda")
        if kind == "prefill":
            # both ranks once, then rank 1 leaves the second call out
            ctx.attn_prefill_gather(0, 0, L, 0, P, qn.data_ptr(), full.data_ptr())
            ctx.sync()
            dist.barrier()
            if rank == 0:
                ctx.attn_prefill_gather(0, 0, L, 0, P, qn.data_ptr(), full.data_ptr())
        else:
            ctx.commit(0, P)
            row = [t[:, P:P + 1].contiguous() for t in (qs, ks, vs)]
            out = torch.empty((L, 1, 16, 128), device="cuda")
            ctx.decode_step_gather(0, 0, L, P, row[0].data_ptr(), row[1].data_ptr(), row[2].data_ptr(), 0,
                                   out.data_ptr())
            ctx.commit(0, 1)
            ctx.sync()
            dist.barrier()
            row2 = [t[:, P + 1:P + 2].contiguous() for t in (qs, ks, vs)]
            if rank == 0:
                ctx.decode_step_gather(0, 0, L, P + 1, row2[0].data_ptr(), row2[1].data_ptr(), row2[2].data_ptr(),
                                       0, out.data_ptr())
        status = 0
        try:
            ctx.sync()
        except qattn.QAttnError as e:
            status = e.status
            report[kind + "_message"] = str(e)
        report[kind + "_status"] = status
        if rank == 0:
            ctx.sync()                                   # reported once, then cleared
            # the context keeps working: a local decode of its heads on a fresh sequence
            ctx.reset(0)
            ctx.append(0, 0, L, 0, P, hist[0].data_ptr(), hist[1].data_ptr(), hist[2].data_ptr(), qn.data_ptr())
            ctx.commit(0, P - 1)
            o = torch.empty_like(qn[:, P - 1:P])
            q1 = qn[:, P - 1:P].contiguous()
            ctx.attn_decode(0, 0, L, P - 1, 1, q1.data_ptr(), o.data_ptr())
            ctx.sync()
            report[kind + "_after_finite"] = bool(torch.isfinite(o).all())
        dist.barrier()                                   # nobody's kernels are in flight now
        ctx.comm_destroy()
        ctx.close()
    np.save(os.path.join(out_dir, f"skip{rank}.npy"), report, allow_pickle=True)
    dist.destroy_process_group()


def test_peer_that_skips_a_gather_makes_the_wait_expire(tmp_path):
    world = 2
    mp.start_processes(_skip_worker, args=(world, _free_port(), str(tmp_path)), nprocs=world, start_method="spawn")
    r0 = np.load(tmp_path / "skip0.npy", allow_pickle=True).item()
    r1 = np.load(tmp_path / "skip1.npy", allow_pickle=True).item()
    for kind, code in (("decode", 51), ("prefill", 52)):
        if not r0[kind + "_mapped"]:
            pytest.skip("no peer mapping between the GPUs: the gathers run on NCCL")
        assert r0[kind + "_status"] == 6 and f"code {code}" in r0[kind + "_message"], r0
        assert r0[kind + "_after_finite"], r0
        assert r1[kind + "_status"] == 0, r1
