"""qa_attn_decode_noalloc: decode attention for callers that may not allocate device memory.

Hosts that reserve all HBM for their own arena (or give this library a fixed budget) cannot
let it call cudaMalloc. This entry point keeps its scratch in a fixed device array inside
the library and works on caller-owned memory only. The test builds a KV history with the
regular context, then calls the no-allocation entry point twice in a row (different row
counts and positions, so the second call meets the first call's leftovers in the shared
array) and checks each result against qa_attn_decode on the same inputs, within the
attention tolerance used by every parity test (max-abs 1e-3, RMS 1e-4).

It also checks the property the entry point exists for: device free memory does not change
across a call, and, in a fresh process with lazy module loading (the CUDA default, which
defers loading a kernel's module and its device arrays to first use), not even across the
first call after qa_create, which loads the fixed array and the kernel up front.

The file sorts last so that a run stopping at the first failure has run everything else.
"""
import os
import subprocess
import sys
from pathlib import Path

import numpy as np
import pytest
import torch

from fpga_qwen_b200 import qattn
from tests import helpers as H

pytestmark = pytest.mark.gpu


def _regular_decode(ctx, pos0, qn):
    out = torch.empty_like(qn)
    ctx.attn_decode(0, 0, qn.shape[0], pos0, qn.shape[1], qn.data_ptr(), out.data_ptr())
    return out


def test_noalloc_decode_matches_the_regular_entry_point_on_two_calls():
    L, P = 28, 3000
    ctx = qattn.Context(n_layers=L, context=4096)
    stream = torch.cuda.current_stream().cuda_stream
    ctx.set_stream(stream)
    qw, kw = H.norms(31, L)
    H.set_norms(ctx, qw, kw)
    q, k, v = H.inputs(31, L, 0, P + 2)
    qn_p = torch.empty_like(q[:, :P])
    # the contiguous copies stay referenced until the queued kernels have read them
    qp, kp, vp = q[:, :P].contiguous(), k[:, :P].contiguous(), v[:, :P].contiguous()
    ctx.append(0, 0, L, 0, P, qp.data_ptr(), kp.data_ptr(), vp.data_ptr(), qn_p.data_ptr())
    ctx.commit(0, P)
    qn = torch.empty_like(q[:, P:])
    qt, kt, vt = q[:, P:].contiguous(), k[:, P:].contiguous(), v[:, P:].contiguous()
    ctx.append(0, 0, L, P, 2, qt.data_ptr(), kt.data_ptr(), vt.data_ptr(), qn.data_ptr())
    kv_slot = ctx.kv_pointer(0, 0, 0, 0)

    # call 1: two rows (B2 verify shape), all 28 layers
    out1 = torch.full_like(qn, float("nan"))
    st = qattn.attn_decode_noalloc(kv_slot, L, 8, 4096, 0, L, P, 2, qn.data_ptr(), out1.data_ptr(), stream)
    assert st == qattn.QA_OK
    # call 2: one row over a layer sub-range, reusing the array the first call left behind
    q1 = qn[3:20, :1].contiguous()
    out2 = torch.full_like(q1, float("nan"))
    torch.cuda.synchronize()
    free_before = torch.cuda.mem_get_info()[0]
    st = qattn.attn_decode_noalloc(kv_slot, L, 8, 4096, 3, 17, P, 1, q1.data_ptr(), out2.data_ptr(), stream)
    assert st == qattn.QA_OK
    torch.cuda.synchronize()
    assert torch.cuda.mem_get_info()[0] == free_before          # the call took no device memory

    ref1 = _regular_decode(ctx, P, qn)
    ref2 = torch.empty_like(q1)
    ctx.attn_decode(0, 3, 17, P, 1, q1.data_ptr(), ref2.data_ptr())
    torch.cuda.synchronize()
    ctx.sync()
    for got, ref in ((out1, ref1), (out2, ref2)):
        g, r = got.cpu().numpy(), ref.cpu().numpy()
        assert np.isfinite(g).all()
        mx, rms = H.err_stats(g, r)
        assert mx < H.MAX_ABS and rms < H.RMS, (mx, rms)
    ctx.close()


def test_noalloc_decode_rejects_requests_beyond_its_fixed_array():
    # 64 layers x 4 rows x 16 KV heads needs more records than the 4 MiB array holds; the
    # call is refused before anything runs (the pointers are never dereferenced).
    buf = torch.empty(1024, dtype=torch.float32, device="cuda")
    p = buf.data_ptr()
    st = qattn.attn_decode_noalloc(p, 64, 16, 4096, 0, 64, 100, 4, p, p, 0)
    assert st == qattn.QA_ERR_CAPACITY
    assert qattn.attn_decode_noalloc(p, 28, 8, 4096, 0, 28, 4095, 2, p, p, 0) == qattn.QA_ERR_CAPACITY
    assert qattn.attn_decode_noalloc(p, 28, 8, 4096, 0, 28, 10, 5, p, p, 0) == qattn.QA_ERR_INVALID
    assert qattn.attn_decode_noalloc(0, 28, 8, 4096, 0, 28, 10, 1, p, p, 0) == qattn.QA_ERR_INVALID


_LAZY_SCRIPT = r"""
import sys, torch
sys.path.insert(0, sys.argv[1])
from fpga_qwen_b200 import qattn
from tests import helpers as H
L, P = 4, 500
ctx = qattn.Context(n_layers=L, context=1024)
stream = torch.cuda.current_stream().cuda_stream
ctx.set_stream(stream)
q, k, v = H.inputs(33, L, 0, P + 1)
qn = torch.empty_like(q)
ctx.append(0, 0, L, 0, P + 1, q.data_ptr(), k.data_ptr(), v.data_ptr(), qn.data_ptr())
ctx.commit(0, P)
q1 = qn[:, P:].contiguous()
out = torch.empty_like(q1)
ref = torch.empty_like(q1)
torch.cuda.synchronize()
free0 = torch.cuda.mem_get_info()[0]
for _ in range(2):
    st = qattn.attn_decode_noalloc(ctx.kv_pointer(0, 0, 0, 0), L, 8, 1024, 0, L, P, 1, q1.data_ptr(),
                                   out.data_ptr(), stream)
    assert st == 0, st
torch.cuda.synchronize()
free1 = torch.cuda.mem_get_info()[0]
ctx.attn_decode(0, 0, L, P, 1, q1.data_ptr(), ref.data_ptr())
ctx.sync()
mx, rms = H.err_stats(out.cpu().numpy(), ref.cpu().numpy())
print(free0, free1, mx, rms)
assert free1 == free0, (free0, free1)
assert mx < H.MAX_ABS and rms < H.RMS, (mx, rms)
"""


def test_first_call_after_create_allocates_nothing_under_lazy_loading():
    root = Path(__file__).resolve().parents[1]
    env = dict(os.environ, CUDA_MODULE_LOADING="LAZY")
    res = subprocess.run([sys.executable, "-c", _LAZY_SCRIPT, str(root)], env=env, capture_output=True, text=True,
                         timeout=300)
    assert res.returncode == 0, res.stdout[-2000:] + res.stderr[-4000:]
