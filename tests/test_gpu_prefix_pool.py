"""GPU: the prefix block pool (qa_block_pool / qa_block_save / qa_block_load) under the
cross-session cache. A request served from the pool holds the same KV rows, bit for bit, as
a fresh prefill, after the slot that computed the prefix was reused by another request."""
import numpy as np
import pytest
import torch

from fpga_qwen_b200 import qattn
from fpga_qwen_b200.prefix import BlockPrefixCache
from tests import helpers as H

pytestmark = pytest.mark.gpu


def _ctx(L, slots, context):
    ctx = qattn.Context(n_layers=L, max_seqs=slots, context=context)
    ctx.set_stream(torch.cuda.current_stream().cuda_stream)
    return ctx


def _append(ctx, seq, pos0, q, k, v):
    qn = torch.empty_like(q)
    ctx.append(seq, 0, q.shape[0], pos0, q.shape[1], q.data_ptr(), k.data_ptr(), v.data_ptr(), qn.data_ptr())
    return qn


def test_pool_serves_prefix_after_its_slot_was_reused():
    L, ctxlen = 4, 2048
    ctx = _ctx(L, 3, ctxlen)
    qw, kw = H.norms(8, L)
    H.set_norms(ctx, qw, kw)
    cache = BlockPrefixCache(ctx, 4)
    ids_a = [int(x) for x in np.random.default_rng(1).integers(0, 151_936, 1100)]
    ids_b = ids_a[:1024] + [int(x) for x in np.random.default_rng(2).integers(0, 151_936, 200)]
    # request A prefills 1100 rows in slot 0; its two canonical chunks go to the pool
    qa, ka, va = H.inputs(1234, L, 0, 1100)
    ctx.reset(0)
    _append(ctx, 0, 0, qa, ka, va)
    ctx.commit(0, 1100)
    assert cache.save(0, ids_a) == 2
    # slot 0 is reused by an unrelated request
    qo, ko, vo = H.inputs(99, L, 0, 600)
    assert cache.load(0, [7] * 600) == 0
    _append(ctx, 0, 0, qo, ko, vo)
    ctx.commit(0, 600)
    # request B shares A's first 1024 tokens: served from the pool into slot 1, tail recomputed
    qt, kt, vt = H.inputs(5678, L, 1024, 200)
    assert cache.load(1, ids_b) == 1024
    assert ctx.position(1) == 1024
    qn_b = _append(ctx, 1, 1024, qt, kt, vt)
    out_b = torch.empty_like(qn_b)
    ctx.attn_prefill(1, 0, L, 1024, 200, qn_b.data_ptr(), out_b.data_ptr())
    ctx.commit(1, 200)
    # B fresh in slot 2: A's first 1024 rows regenerated from A's seed, then the same tail
    qf, kf, vf = H.inputs(1234, L, 0, 1024)
    _append(ctx, 2, 0, qf, kf, vf)
    ctx.commit(2, 1024)
    qn_f = _append(ctx, 2, 1024, qt, kt, vt)
    out_f = torch.empty_like(qn_f)
    ctx.attn_prefill(2, 0, L, 1024, 200, qn_f.data_ptr(), out_f.data_ptr())
    ctx.commit(2, 200)
    torch.cuda.synchronize()
    for layer in range(L):
        for kvsel in (0, 1):
            for h in range(8):
                assert np.array_equal(H.read_plane(ctx, 1, layer, kvsel, h, 0, 1224),
                                      H.read_plane(ctx, 2, layer, kvsel, h, 0, 1224))
    assert torch.equal(out_b, out_f)
    ctx.close()


def test_pool_validation_leaves_state_unchanged():
    L = 2
    ctx = _ctx(L, 2, 2048)
    qa, ka, va = H.inputs(3, L, 0, 700)
    _append(ctx, 0, 0, qa, ka, va)
    ctx.commit(0, 700)
    with pytest.raises(qattn.QAttnError):
        ctx.block_save(0, 0, 0)                     # no pool yet
    ctx.block_pool(2)
    ctx.block_save(0, 0, 1)
    bad = [
        lambda: ctx.block_save(0, 1, 0),            # chunk 1 is not committed (700 rows)
        lambda: ctx.block_save(0, 0, 2),            # block outside the pool
        lambda: ctx.block_save(0, 4, 0),            # chunk outside the context
        lambda: ctx.block_load(1, 0, 0),            # block 0 is empty
        lambda: ctx.block_load(0, 0, 1),            # slot 0 is at 700, not at chunk 0's start
        lambda: ctx.block_load(1, 1, 1),            # block 1 holds chunk 0
        lambda: ctx.block_pool(-1),
    ]
    for call in bad:
        with pytest.raises(qattn.QAttnError):
            call()
        assert ctx.position(0) == 700 and ctx.position(1) == 0
    ctx.block_load(1, 0, 1)
    assert ctx.position(1) == 512
    torch.cuda.synchronize()
    for layer in range(L):
        assert np.array_equal(H.read_plane(ctx, 1, layer, 0, 3, 0, 512), H.read_plane(ctx, 0, layer, 0, 3, 0, 512))
        assert np.array_equal(H.read_plane(ctx, 1, layer, 1, 5, 0, 512), H.read_plane(ctx, 0, layer, 1, 5, 0, 512))
    ctx.close()
