"""Failure detection on one GPU without a fault: a bounded device-side wait that runs out.

The waits that can expire in service are the ones on other GPUs' flags (the head gathers of
qa_attn_prefill_gather and qa_decode_step_gather): a peer that stops answering must not hold
this GPU. qa_selftest_timeout launches that wait kernel on a flag word nothing sets, with the
limit lowered by qa_set_wait_limit, so the expiry path runs on one GPU: the kernel gives up
after the limit (it never traps), the error reaches the host through qa_sync or through the
next host-buffer call (which then resets its sequence), is cleared once reported, and the
context keeps working.
"""
import time

import numpy as np
import pytest
import torch

from fpga_qwen_b200 import qattn
from oracle import oracle as O
from tests import helpers as H

pytestmark = pytest.mark.gpu

LIMIT_US = 20000          # 20 ms


def _ctx(**kw):
    ctx = qattn.Context(**kw)
    if not kw.get("io_host"):
        ctx.set_stream(torch.cuda.current_stream().cuda_stream)
    return ctx


def test_expired_wait_is_reported_by_sync_then_cleared():
    L, n = 2, 40
    ctx = _ctx(n_layers=L, context=256)
    qw, kw = H.norms(61, L)
    H.set_norms(ctx, qw, kw)
    ctx.set_wait_limit(LIMIT_US)
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    ctx.selftest_timeout()
    with pytest.raises(qattn.QAttnError) as err:
        ctx.sync()
    waited = time.perf_counter() - t0
    assert err.value.status == qattn.QA_ERR_TIMEOUT
    assert "code 51" in str(err.value)
    assert waited >= LIMIT_US * 1e-6                 # the kernel returned only after the limit
    ctx.sync()                                       # reported once, then cleared
    # the context keeps working: an append + prefill that matches the oracle
    q, k, v = H.inputs(61, L, 0, n)
    qn, out = torch.empty_like(q), torch.empty_like(q)
    ctx.append(0, 0, L, 0, n, q.data_ptr(), k.data_ptr(), v.data_ptr(), qn.data_ptr())
    ctx.attn_prefill(0, 0, L, 0, n, qn.data_ptr(), out.data_ptr())
    ctx.commit(0, n)
    ctx.sync()
    tables = O.rope_tables(256)
    for layer in range(L):
        kv = O.LayerKV(8, 256)
        qref = O.append(kv, 0, q[layer].cpu().numpy(), k[layer].cpu().numpy(), v[layer].cpu().numpy(),
                        qw[layer], kw[layer], tables)
        H.check("after an expired wait", out[layer].cpu().numpy(), O.attention(kv, 0, qref, threads=4))
    # the default limit comes back with 0
    ctx.set_wait_limit(0)
    ctx.close()


def test_host_buffer_call_reports_the_timeout_and_resets_its_sequence():
    L, n = 2, 40
    dev = _ctx(n_layers=L, context=256)
    host = _ctx(n_layers=L, context=256, io_host=1)
    qw, kw = H.norms(62, L)
    for c in (dev, host):
        H.set_norms(c, qw, kw)
    q, k, v = H.inputs(62, L, 0, n + 1)
    qh, kh, vh = (np.ascontiguousarray(t.cpu().numpy()) for t in (q, k, v))
    hist = [np.ascontiguousarray(t[:, :n]) for t in (qh, kh, vh)]
    row = [np.ascontiguousarray(t[:, n:n + 1]) for t in (qh, kh, vh)]
    qo = np.empty_like(hist[0])
    host.append(0, 0, L, 0, n, hist[0].ctypes.data, hist[1].ctypes.data, hist[2].ctypes.data, qo.ctypes.data)
    host.commit(0, n)
    host.set_wait_limit(LIMIT_US)
    host.selftest_timeout()
    out_h = np.empty_like(row[0])
    with pytest.raises(qattn.QAttnError) as err:
        host.decode_step(0, 0, L, n, row[0].ctypes.data, row[1].ctypes.data, row[2].ctypes.data, 0, out_h.ctypes.data)
    assert err.value.status == qattn.QA_ERR_TIMEOUT
    assert host.position(0) == 0                     # the sequence was reset, as after a CUDA error
    host.sync()                                      # already reported: nothing pending
    # the next calls succeed and give the device-pointer context's results
    host.append(0, 0, L, 0, n, hist[0].ctypes.data, hist[1].ctypes.data, hist[2].ctypes.data, qo.ctypes.data)
    host.commit(0, n)
    host.decode_step(0, 0, L, n, row[0].ctypes.data, row[1].ctypes.data, row[2].ctypes.data, 0, out_h.ctypes.data)
    host.commit(0, 1)
    qn = torch.empty_like(q[:, :n])
    hq, hk, hv = (t[:, :n].contiguous() for t in (q, k, v))
    dev.append(0, 0, L, 0, n, hq.data_ptr(), hk.data_ptr(), hv.data_ptr(), qn.data_ptr())
    dev.commit(0, n)
    r1 = [t[:, n:n + 1].contiguous() for t in (q, k, v)]
    out_d = torch.empty_like(r1[0])
    dev.decode_step(0, 0, L, n, r1[0].data_ptr(), r1[1].data_ptr(), r1[2].data_ptr(), 0, out_d.data_ptr())
    dev.commit(0, 1)
    dev.sync()
    assert np.array_equal(out_h, out_d.cpu().numpy())
    assert host.position(0) == n + 1
    dev.close()
    host.close()
