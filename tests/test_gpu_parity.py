"""GPU parity tests: the CUDA library against the CPU restatement of the reference.

Bar: KV contents and prefix copies bit-exact; attention outputs within max-abs 1e-3 and
RMS 1e-4 of the oracle (tampajohn/fpga-qwen engine/core.cpp arithmetic) on the same
seeded inputs. All calls go through the C ABI (libqattn.so).
"""
import numpy as np
import pytest
import torch

from fpga_qwen_b200 import qattn
from oracle import oracle as O
from tests import helpers as H

pytestmark = pytest.mark.gpu

TABLES = None


def tables():
    global TABLES
    if TABLES is None:
        TABLES = O.rope_tables(4096)
    return TABLES


def make_ctx(layers=28, max_seqs=1, context=4096, **kw):
    ctx = qattn.Context(n_layers=layers, max_seqs=max_seqs, context=context, **kw)
    ctx.set_stream(torch.cuda.current_stream().cuda_stream)
    return ctx


def gpu_append(ctx, seq, pos0, q, k, v):
    L, n = q.shape[0], q.shape[1]
    qn = torch.empty_like(q)
    ctx.append(seq, 0, L, pos0, n, q.data_ptr(), k.data_ptr(), v.data_ptr(), qn.data_ptr())
    return qn


def gpu_attend(ctx, seq, pos0, qn, decode=False):
    L, n = qn.shape[0], qn.shape[1]
    out = torch.empty_like(qn)
    fn = ctx.attn_decode if decode else ctx.attn_prefill
    fn(seq, 0, L, pos0, n, qn.data_ptr(), out.data_ptr())
    return out


def oracle_layer(q, k, v, qw, kw, pos0, ctx_len=4096, kv=None):
    """Oracle append (+ attention) of one layer given host arrays [n][h][128]."""
    kv = kv or O.LayerKV(k.shape[1], ctx_len)
    qn = O.append(kv, pos0, q, k, v, qw, kw, tables())
    return kv, qn


# ---------------------------------------------------------------------------------------------
def test_append_bit_exact_all_layers():
    """Config-1 shape: 85-row prefill append over all 28 layers, bit-exact K, V and q_out."""
    L, n = 28, 85
    ctx = make_ctx(L)
    qw, kw = H.norms(11, L)
    H.set_norms(ctx, qw, kw)
    q, k, v = H.inputs(11, L, 0, n)
    qn = gpu_append(ctx, 0, 0, q, k, v)
    torch.cuda.synchronize()
    qh, kh, vh, qnh = q.cpu().numpy(), k.cpu().numpy(), v.cpu().numpy(), qn.cpu().numpy()
    for layer in range(L):
        kv, qref = oracle_layer(qh[layer], kh[layer], vh[layer], qw[layer], kw[layer], 0, ctx_len=128)
        assert np.array_equal(qnh[layer].view(np.uint32), qref.view(np.uint32)), f"q_out layer {layer}"
        for h in range(8):
            assert np.array_equal(H.read_plane(ctx, 0, layer, 0, h, 0, n), kv.k[h, :n]), f"K layer {layer} head {h}"
            assert np.array_equal(H.read_plane(ctx, 0, layer, 1, h, 0, n), kv.v[h, :n]), f"V layer {layer} head {h}"
    ctx.close()


def test_golden_fixture_through_the_gpu(golden):
    """Reference NumPy-oracle inputs: GPU K/V/q bit-exact with the restatement, V bit-exact
    with the reference oracle, attention within tolerance of the reference oracle."""
    T = 40
    ctx = make_ctx(1, context=64)
    for layer in golden["layers"]:
        ctx.reset(0)
        H.set_norms(ctx, golden[f"L{layer}_q_norm"][None], golden[f"L{layer}_k_norm"][None])
        q = torch.from_numpy(golden[f"L{layer}_q_pre"][None].copy()).cuda()
        k = torch.from_numpy(golden[f"L{layer}_k_pre"][None].copy()).cuda()
        v = torch.from_numpy(golden[f"L{layer}_v_pre"][None].copy()).cuda()
        qn = gpu_append(ctx, 0, 0, q, k, v)
        out = gpu_attend(ctx, 0, 0, qn)
        torch.cuda.synchronize()
        kv, qref = oracle_layer(golden[f"L{layer}_q_pre"], golden[f"L{layer}_k_pre"], golden[f"L{layer}_v_pre"],
                                golden[f"L{layer}_q_norm"], golden[f"L{layer}_k_norm"], 0, ctx_len=64)
        assert np.array_equal(qn.cpu().numpy()[0], qref)
        for h in range(8):
            gk = H.read_plane(ctx, 0, 0, 0, h, 0, T)
            gv = H.read_plane(ctx, 0, 0, 1, h, 0, T)
            assert np.array_equal(gk, kv.k[h, :T]) and np.array_equal(gv, kv.v[h, :T])
            assert np.array_equal(gv.view(np.float16).astype(np.float32), golden[f"L{layer}_v16"][:, h])
        mx, rms = H.err_stats(out.cpu().numpy()[0], golden[f"L{layer}_out"])
        assert mx < H.MAX_ABS and rms < H.RMS, (mx, rms)
    ctx.close()


@pytest.mark.parametrize("pos0,n", [(0, 1), (0, 2), (0, 31), (0, 32), (0, 33), (0, 85), (0, 127), (0, 128),
                                    (0, 129), (0, 452), (17, 64), (512, 512), (1000, 129)])
def test_prefill_attention_parity(pos0, n):
    """Causal prefill attention vs the oracle on edge lengths (31/32/33, 127/128/129, odd
    final rows, a 512 tail at P=512) over 2 layers."""
    L = 2
    ctx = make_ctx(L, context=2048)
    qw, kw = H.norms(5, L)
    H.set_norms(ctx, qw, kw)
    seed = 100 + n + pos0
    if pos0:
        q0, k0, v0 = H.inputs(seed, L, 0, pos0)
        gpu_append(ctx, 0, 0, q0, k0, v0)
        ctx.commit(0, pos0)
    q, k, v = H.inputs(seed, L, pos0, n)
    qn = gpu_append(ctx, 0, pos0, q, k, v)
    out = gpu_attend(ctx, 0, pos0, qn)
    torch.cuda.synchronize()
    outh, qnh = out.cpu().numpy(), qn.cpu().numpy()
    for layer in range(L):
        kv = H.read_layer_kv(ctx, 0, layer, pos0 + n, 2048)
        ref = O.attention(kv, pos0, qnh[layer], threads=8)
        mx, rms = H.err_stats(outh[layer], ref)
        assert mx < H.MAX_ABS and rms < H.RMS, (layer, mx, rms)
    ctx.close()


@pytest.mark.parametrize("chunks", [[(p, 512) for p in range(0, 3584, 512)] + [(3584, 384)], [(0, 3000), (3000, 700)]])
def test_chunked_prefill_one_layer_calls(chunks):
    """The engine's prefill pattern: a prompt in chunks (512 rows like core.cpp:712, or an
    unaligned offset), each chunk appended for both layers and then attended one layer per
    call. These launches hold fewer work items than SMs, so each item's key tiles are split
    over several CTAs and merged; every chunk's rows are compared with the oracle."""
    L = 2
    ctx = make_ctx(L, context=4096)
    qw, kw = H.norms(7, L)
    H.set_norms(ctx, qw, kw)
    for ci, (pos0, n) in enumerate(chunks):
        q, k, v = H.inputs(300 + ci, L, pos0, n)
        qn = gpu_append(ctx, 0, pos0, q, k, v)
        out = torch.empty_like(qn)
        for layer in range(L):
            ctx.attn_prefill(0, layer, 1, pos0, n, qn[layer].data_ptr(), out[layer].data_ptr())
        torch.cuda.synchronize()
        outh, qnh = out.cpu().numpy(), qn.cpu().numpy()
        for layer in range(L):
            kv = H.read_layer_kv(ctx, 0, layer, pos0 + n, 4096)
            ref = O.attention(kv, pos0, qnh[layer], threads=8)
            mx, rms = H.err_stats(outh[layer], ref)
            H.record("chunked prefill, one-layer calls (split key ranges)", mx, rms, n)
            assert mx < H.MAX_ABS and rms < H.RMS, (pos0, n, layer, mx, rms)
        ctx.commit(0, n)
    ctx.close()


def test_config1_prefill_then_32_decode_steps():
    """85-row prefill + 32 decode steps (the odd final row), 28 layers, vs the oracle."""
    L, n, steps = 28, 85, 32
    ctx = make_ctx(L, context=256)
    qw, kw = H.norms(1, L)
    H.set_norms(ctx, qw, kw)
    q, k, v = H.inputs(1, L, 0, n + steps)
    qh, kh, vh = q.cpu().numpy(), k.cpu().numpy(), v.cpu().numpy()
    qn = gpu_append(ctx, 0, 0, q[:, :n].contiguous(), k[:, :n].contiguous(), v[:, :n].contiguous())
    outs = [gpu_attend(ctx, 0, 0, qn)]
    ctx.commit(0, n)
    for s in range(steps):
        p = n + s
        qs = gpu_append(ctx, 0, p, q[:, p:p + 1].contiguous(), k[:, p:p + 1].contiguous(), v[:, p:p + 1].contiguous())
        outs.append(gpu_attend(ctx, 0, p, qs, decode=True))
        ctx.commit(0, 1)
    torch.cuda.synchronize()
    got = np.concatenate([o.cpu().numpy() for o in outs], axis=1)
    worst = 0.0
    for layer in range(L):
        kv, qref = oracle_layer(qh[layer], kh[layer], vh[layer], qw[layer], kw[layer], 0, ctx_len=256)
        ref = O.attention(kv, 0, qref, threads=8)
        mx, rms = H.err_stats(got[layer], ref)
        worst = max(worst, mx)
        assert mx < H.MAX_ABS and rms < H.RMS, (layer, mx, rms)
        gk = np.stack([H.read_plane(ctx, 0, layer, 0, h, 0, n + steps) for h in range(8)])
        assert np.array_equal(gk, kv.k[:, :n + steps])
    ctx.close()


def test_decode_rows_and_verify_two():
    """Two-row verify (B2) and single-row decode at a long context equal the oracle; split
    count does not change results beyond tolerance."""
    L, P = 4, 3000
    ctx = make_ctx(L, context=4096)
    qw, kw = H.norms(9, L)
    H.set_norms(ctx, qw, kw)
    q, k, v = H.inputs(9, L, 0, P + 2)
    gpu_append(ctx, 0, 0, q[:, :P].contiguous(), k[:, :P].contiguous(), v[:, :P].contiguous())
    ctx.commit(0, P)
    qn = gpu_append(ctx, 0, P, q[:, P:].contiguous(), k[:, P:].contiguous(), v[:, P:].contiguous())
    out2 = gpu_attend(ctx, 0, P, qn, decode=True)
    out1 = gpu_attend(ctx, 0, P, qn[:, :1].contiguous(), decode=True)
    torch.cuda.synchronize()
    for layer in range(L):
        kv = H.read_layer_kv(ctx, 0, layer, P + 2, 4096)
        ref = O.attention(kv, P, qn.cpu().numpy()[layer], threads=8)
        mx, rms = H.err_stats(out2.cpu().numpy()[layer], ref)
        assert mx < H.MAX_ABS and rms < H.RMS
        mx1, _ = H.err_stats(out1.cpu().numpy()[layer, 0], ref[0])
        assert mx1 < H.MAX_ABS
    ctx.close()


def test_prefix_copy_bit_exact_config3():
    """Canonical prefix reuse: A prefills 1024 rows; B copies A's 512-row canonical prefix, then
    prefills its own 512-row tail and decodes. B's KV equals a fresh prefill of B, bit for bit."""
    L = 28
    ctx = make_ctx(L, max_seqs=3, context=1280)
    qw, kw = H.norms(3, L)
    H.set_norms(ctx, qw, kw)
    qa, ka, va = H.inputs(1234, L, 0, 1024)           # request A
    gpu_append(ctx, 0, 0, qa, ka, va)
    ctx.commit(0, 1024)
    qt, kt, vt = H.inputs(5678, L, 512, 512)          # B's tail: new seed, positions 512..1023
    # B via reuse: block copy of A's first 512 rows, then tail recompute
    ctx.copy_prefix(0, 1, 512)
    qn_b = gpu_append(ctx, 1, 512, qt, kt, vt)
    out_b = gpu_attend(ctx, 1, 512, qn_b)
    ctx.commit(1, 512)
    # B fresh: regenerate positions 0..511 from A's seed, then the same tail
    qf, kf, vf = H.inputs(1234, L, 0, 512)
    gpu_append(ctx, 2, 0, qf, kf, vf)
    ctx.commit(2, 512)
    qn_f = gpu_append(ctx, 2, 512, qt, kt, vt)
    out_f = gpu_attend(ctx, 2, 512, qn_f)
    ctx.commit(2, 512)
    torch.cuda.synchronize()
    assert ctx.position(1) == ctx.position(2) == 1024
    for layer in range(L):
        for kvsel in (0, 1):
            for h in range(8):
                assert np.array_equal(H.read_plane(ctx, 1, layer, kvsel, h, 0, 1024),
                                      H.read_plane(ctx, 2, layer, kvsel, h, 0, 1024))
    assert torch.equal(out_b, out_f)
    ctx.close()


def test_validation_leaves_state_unchanged():
    ctx = make_ctx(2, max_seqs=2, context=64)
    q, k, v = H.inputs(2, 2, 0, 8)
    qn = torch.empty_like(q)
    gpu_append(ctx, 0, 0, q, k, v)
    ctx.commit(0, 8)
    cases = [
        lambda: ctx.append(0, 0, 2, 7, 8, q.data_ptr(), k.data_ptr(), v.data_ptr(), qn.data_ptr()),   # wrong pos0
        lambda: ctx.append(0, 0, 2, 8, 57, q.data_ptr(), k.data_ptr(), v.data_ptr(), qn.data_ptr()),  # capacity
        lambda: ctx.append(2, 0, 2, 0, 8, q.data_ptr(), k.data_ptr(), v.data_ptr(), qn.data_ptr()),   # bad seq
        lambda: ctx.append(0, 1, 2, 8, 8, q.data_ptr(), k.data_ptr(), v.data_ptr(), qn.data_ptr()),   # layers
        lambda: ctx.append(0, 0, 2, 8, 0, q.data_ptr(), k.data_ptr(), v.data_ptr(), qn.data_ptr()),   # empty
        lambda: ctx.attn_prefill(0, 0, 2, 8, 1, qn.data_ptr(), qn.data_ptr()),                        # not appended
        lambda: ctx.attn_decode(0, 0, 2, 8, 5, qn.data_ptr(), qn.data_ptr()),                         # too many rows
        lambda: ctx.truncate(0, 9),
        lambda: ctx.commit(0, 1),                                                                      # not appended
        lambda: ctx.copy_prefix(0, 1, 512),                                                            # too short
        lambda: ctx.decode_step(0, 0, 2, 7, q.data_ptr(), k.data_ptr(), v.data_ptr(), 0, qn.data_ptr()),  # wrong pos
        lambda: ctx.decode_step(0, 0, 2, 8, 0, k.data_ptr(), v.data_ptr(), 0, qn.data_ptr()),            # null input
        lambda: ctx.decode_step_batch([0, 0], 0, 2, q.data_ptr(), k.data_ptr(), v.data_ptr(), 0,
                                      qn.data_ptr()),                                                  # duplicate seq
    ]
    for case in cases:
        with pytest.raises(qattn.QAttnError):
            case()
        assert ctx.position(0) == 8 and ctx.position(1) == 0
    ctx.truncate(0, 3)
    assert ctx.position(0) == 3
    ctx.close()


def test_engine_mirror_state_machine():
    """The Model-API mirror: prefill/step/verify_two/commit_verified/truncate semantics."""
    from fpga_qwen_b200.engine import AttentionModel
    L = 28
    ctx = make_ctx(L, context=128)
    m = AttentionModel(ctx)
    q, k, v = H.inputs(4, L, 0, 20)
    out = m.prefill(q[:, :10].contiguous(), k[:, :10].contiguous(), v[:, :10].contiguous())
    assert m.position == 10
    o1 = m.step(q[:, 10:11].contiguous(), k[:, 10:11].contiguous(), v[:, 10:11].contiguous())
    assert m.position == 11
    ov = m.verify_two(q[:, 11:13].contiguous(), k[:, 11:13].contiguous(), v[:, 11:13].contiguous())
    assert m.position == 11
    with pytest.raises(qattn.QAttnError):
        m.step(q[:, 11:12].contiguous(), k[:, 11:12].contiguous(), v[:, 11:12].contiguous())
    m.commit_verified(1)
    assert m.position == 12
    # sequential-step equivalence of the verified first row
    m.truncate(11)
    o2 = m.step(q[:, 11:12].contiguous(), k[:, 11:12].contiguous(), v[:, 11:12].contiguous())
    torch.cuda.synchronize()
    assert torch.allclose(ov[:, :1], o2, atol=1e-6, rtol=0)
    assert out.shape == (L, 10, 16, 128) and o1.shape == (L, 1, 16, 128)
    ctx.close()


def test_config4_full_size_sampled_rows():
    """The 3968 + 128 workload at full size on one GPU: 3968-row prefill over 28 layers, then 4
    decode steps. KV bytes of sampled layers are bit-exact with the oracle's append; sampled
    rows (tile edges, the position-128 boundary between the FP32 and tensor-core paths,
    random rows) and the decode outputs are within tolerance of the oracle."""
    L, n, steps = 28, 3968, 4
    ctx = make_ctx(L, context=4096)
    qw, kw = H.norms(21, L)
    H.set_norms(ctx, qw, kw)
    q, k, v = H.inputs(21, L, 0, n + steps)
    qn = gpu_append(ctx, 0, 0, q[:, :n].contiguous(), k[:, :n].contiguous(), v[:, :n].contiguous())
    out = gpu_attend(ctx, 0, 0, qn)
    ctx.commit(0, n)
    dec = []
    for s in range(steps):
        p = n + s
        qs = gpu_append(ctx, 0, p, q[:, p:p + 1].contiguous(), k[:, p:p + 1].contiguous(), v[:, p:p + 1].contiguous())
        dec.append(gpu_attend(ctx, 0, p, qs, decode=True))
        ctx.commit(0, 1)
    torch.cuda.synchronize()
    rng = np.random.default_rng(0)
    rows = sorted(set([0, 1, 2, 63, 126, 127, 128, 129, 130, 255, 256, 257, 1000, 2047, 2048, 3839, 3840, 3967]
                      + rng.integers(0, n, 24).tolist()))
    outh = out.cpu().numpy()
    dech = np.concatenate([d.cpu().numpy() for d in dec], axis=1)
    for layer in (0, 13, 27):
        qh, kh, vh = (t[layer].cpu().numpy() for t in (q, k, v))
        kv, qref = oracle_layer(qh, kh, vh, qw[layer], kw[layer], 0, ctx_len=4096)
        gk = np.stack([H.read_plane(ctx, 0, layer, 0, h, 0, n + steps) for h in range(8)])
        gv = np.stack([H.read_plane(ctx, 0, layer, 1, h, 0, n + steps) for h in range(8)])
        assert np.array_equal(gk, kv.k[:, :n + steps]) and np.array_equal(gv, kv.v[:, :n + steps])
        ref = np.stack([O.attention(kv, r, qref[r:r + 1], threads=8)[0] for r in rows])
        mx, rms = H.err_stats(outh[layer][rows], ref)
        assert mx < H.MAX_ABS and rms < H.RMS, (layer, mx, rms)
        refd = np.stack([O.attention(kv, n + s, qref[n + s:n + s + 1], threads=8)[0] for s in range(steps)])
        mx, rms = H.err_stats(dech[layer], refd)
        assert mx < H.MAX_ABS and rms < H.RMS, (layer, mx, rms)
    ctx.close()


def test_prefill_is_deterministic_and_matches_single_layer_calls():
    """Layer-batched and per-layer calls give identical bits; repeated calls are deterministic."""
    L, n = 3, 700
    ctx = make_ctx(L, max_seqs=2, context=1024)
    q, k, v = H.inputs(8, L, 0, n)
    qn = gpu_append(ctx, 0, 0, q, k, v)
    out_all = gpu_attend(ctx, 0, 0, qn)
    out_again = gpu_attend(ctx, 0, 0, qn)
    per_layer = torch.empty_like(qn)
    for layer in range(L):
        qn1 = torch.empty_like(q[layer:layer + 1])
        ctx.append(1, layer, 1, 0, n, q[layer].data_ptr(), k[layer].data_ptr(), v[layer].data_ptr(), qn1.data_ptr())
        ctx.attn_prefill(1, layer, 1, 0, n, qn1.data_ptr(), per_layer[layer].data_ptr())
    torch.cuda.synchronize()
    ctx.sync()
    assert torch.equal(out_all, out_again)
    assert torch.equal(out_all, per_layer)
    ctx.close()


@pytest.mark.parametrize("layers,pos0,n", [(28, 0, 1), (28, 0, 4), (3, 63, 1), (1, 4094, 2), (28, 3000, 3),
                                           (5, 129, 4), (2, 1, 1), (28, 4092, 4)])
def test_decode_partitions(layers, pos0, n):
    """Decode / verify rows over the even key partition: ranges that split units, ranges that
    hold several whole units, 1..4 rows, tiny and full contexts — all within tolerance of the
    oracle, and repeat calls are bitwise deterministic."""
    ctx = make_ctx(layers, context=4096)
    qw, kw = H.norms(40 + n, layers)
    H.set_norms(ctx, qw, kw)
    q, k, v = H.inputs(40 + pos0, layers, 0, pos0 + n)
    if pos0:
        gpu_append(ctx, 0, 0, q[:, :pos0].contiguous(), k[:, :pos0].contiguous(), v[:, :pos0].contiguous())
        ctx.commit(0, pos0)
    qn = gpu_append(ctx, 0, pos0, q[:, pos0:].contiguous(), k[:, pos0:].contiguous(), v[:, pos0:].contiguous())
    out = gpu_attend(ctx, 0, pos0, qn, decode=True)
    again = gpu_attend(ctx, 0, pos0, qn, decode=True)
    torch.cuda.synchronize()
    ctx.sync()
    assert torch.equal(out, again)
    outh, qnh = out.cpu().numpy(), qn.cpu().numpy()
    for layer in sorted({0, layers // 2, layers - 1}):
        kv = H.read_layer_kv(ctx, 0, layer, pos0 + n, 4096)
        ref = O.attention(kv, pos0, qnh[layer], threads=8)
        mx, rms = H.err_stats(outh[layer], ref)
        assert mx < H.MAX_ABS and rms < H.RMS, (layer, mx, rms)
    ctx.close()


@pytest.mark.parametrize("begin,count", [(4, 4), (6, 2), (3, 1)])
def test_head_sharded_context_single_gpu(begin, count):
    """A context holding KV heads [begin, begin+count) (one GPU's shard) computes exactly the
    slice of a full context: KV bytes equal, attention within tolerance of the oracle."""
    L, n, steps = 3, 260, 2
    ctx = make_ctx(L, context=512, kv_head_begin=begin, kv_head_count=count)
    qw, kw = H.norms(61, L)
    H.set_norms(ctx, qw, kw)
    q, k, v = H.inputs(61, L, 0, n + steps, hkv=count, head0=begin)
    qn = gpu_append(ctx, 0, 0, q[:, :n].contiguous(), k[:, :n].contiguous(), v[:, :n].contiguous())
    out = gpu_attend(ctx, 0, 0, qn)
    ctx.commit(0, n)
    qd = gpu_append(ctx, 0, n, q[:, n:].contiguous(), k[:, n:].contiguous(), v[:, n:].contiguous())
    outd = gpu_attend(ctx, 0, n, qd, decode=True)
    torch.cuda.synchronize()
    got = np.concatenate([out.cpu().numpy(), outd.cpu().numpy()], axis=1)
    qh, kh, vh = q.cpu().numpy(), k.cpu().numpy(), v.cpu().numpy()
    for layer in range(L):
        kv, qref = oracle_layer(qh[layer], kh[layer], vh[layer], qw[layer], kw[layer], 0, ctx_len=512)
        gk = np.stack([H.read_plane(ctx, 0, layer, 0, h, 0, n + steps) for h in range(count)])
        assert np.array_equal(gk, kv.k[:, :n + steps])
        ref = O.attention(kv, 0, qref, threads=8)
        mx, rms = H.err_stats(got[layer], ref)
        assert mx < H.MAX_ABS and rms < H.RMS, (layer, mx, rms)
    ctx.close()


def test_batched_decode_over_sequences():
    """Config-5 style serving: six sequences of different lengths decode together through
    qa_append_batch / qa_attn_decode_batch / qa_commit_batch; every sequence's KV rows are
    bit-exact and its outputs within tolerance of the oracle, and a batch equals the same
    rows decoded one sequence at a time."""
    L, steps = 2, 3
    lengths = [5, 130, 700, 1500, 3000, 4000]
    S = len(lengths)
    ctx = make_ctx(L, max_seqs=S, context=4096)
    qw, kw = H.norms(90, L)
    H.set_norms(ctx, qw, kw)
    data = []
    for s_, n in enumerate(lengths):
        q, k, v = H.inputs(900 + s_, L, 0, n + steps)
        data.append((q, k, v))
        gpu_append(ctx, s_, 0, q[:, :n].contiguous(), k[:, :n].contiguous(), v[:, :n].contiguous())
        ctx.commit(s_, n)
    seqs = list(range(S))
    outs = []
    for st in range(steps):
        qb = torch.stack([data[s_][0][:, lengths[s_] + st] for s_ in seqs], dim=1).contiguous()   # [L][S][16][128]
        kb = torch.stack([data[s_][1][:, lengths[s_] + st] for s_ in seqs], dim=1).contiguous()
        vb = torch.stack([data[s_][2][:, lengths[s_] + st] for s_ in seqs], dim=1).contiguous()
        qn = torch.empty_like(qb)
        ctx.append_batch(seqs, 0, L, qb.data_ptr(), kb.data_ptr(), vb.data_ptr(), qn.data_ptr())
        out = torch.empty_like(qn)
        ctx.attn_decode_batch(seqs, 0, L, qn.data_ptr(), out.data_ptr())
        # the same rows one sequence at a time (positions not yet committed)
        single = torch.empty_like(qn)
        for s_ in seqs:
            q1 = qn[:, s_:s_ + 1].contiguous()
            o1 = torch.empty_like(q1)
            ctx.attn_decode(s_, 0, L, lengths[s_] + st, 1, q1.data_ptr(), o1.data_ptr())
            single[:, s_:s_ + 1] = o1
        ctx.commit_batch(seqs)
        torch.cuda.synchronize()
        mx, _ = H.err_stats(out.cpu().numpy(), single.cpu().numpy())
        assert mx < 1e-5, mx
        outs.append(out.cpu().numpy())
    for s_ in seqs:
        n = lengths[s_]
        assert ctx.position(s_) == n + steps
        q, k, v = (t.cpu().numpy() for t in data[s_])
        for layer in range(L):
            kv, qref = oracle_layer(q[layer], k[layer], v[layer], qw[layer], kw[layer], 0, ctx_len=4096)
            gk = np.stack([H.read_plane(ctx, s_, layer, 0, h, 0, n + steps) for h in range(8)])
            assert np.array_equal(gk, kv.k[:, :n + steps])
            for st in range(steps):
                ref = O.attention(kv, n + st, qref[n + st:n + st + 1], threads=8)[0]
                mx, rms = H.err_stats(outs[st][layer, s_], ref)
                assert mx < H.MAX_ABS and rms < H.RMS, (s_, layer, st, mx, rms)
    ctx.close()


def test_batched_decode_64_requests_many_segments_per_cta():
    """The multi-request shape: 64 sequences with the seeded U[85, 3968] prompt lengths decode
    in one batched launch. Each CTA's key range then spans several (layer, sequence, head)
    units, so the copy ring runs across segment boundaries and the score buffer is sized by
    the longest unit rather than by the range. The batch equals the same rows decoded one
    sequence at a time, and sampled sequences (shortest, longest, two others) agree with the
    oracle on the GPU's own KV planes."""
    from fpga_qwen_b200 import dist as qd
    L, steps = 2, 2
    lengths = qd.config5_lengths()
    S = len(lengths)
    ctx = make_ctx(L, max_seqs=S, context=4096)
    qw, kw = H.norms(91, L)
    H.set_norms(ctx, qw, kw)
    for s_, n in enumerate(lengths):
        q, k, v = H.inputs(2000 + s_, L, 0, n)
        gpu_append(ctx, s_, 0, q, k, v)
        ctx.commit(s_, n)
        torch.cuda.synchronize()
        del q, k, v
    seqs = list(range(S))
    check = sorted({int(np.argmin(lengths)), int(np.argmax(lengths)), 7, 40})
    for st in range(steps):
        rows = [H.inputs(2000 + s_, L, lengths[s_] + st, 1) for s_ in seqs]
        qb, kb, vb = (torch.cat([r[i] for r in rows], dim=1).contiguous() for i in range(3))   # [L][S][h][128]
        qn = torch.empty_like(qb)
        ctx.append_batch(seqs, 0, L, qb.data_ptr(), kb.data_ptr(), vb.data_ptr(), qn.data_ptr())
        out = torch.full_like(qn, float("nan"))
        ctx.attn_decode_batch(seqs, 0, L, qn.data_ptr(), out.data_ptr())
        single = torch.empty_like(qn)
        for s_ in seqs:
            q1 = qn[:, s_:s_ + 1].contiguous()
            o1 = torch.empty_like(q1)
            ctx.attn_decode(s_, 0, L, lengths[s_] + st, 1, q1.data_ptr(), o1.data_ptr())
            single[:, s_:s_ + 1] = o1
        torch.cuda.synchronize()
        got = out.cpu().numpy()
        assert np.isfinite(got).all()
        mx, _ = H.err_stats(got, single.cpu().numpy())
        assert mx < 1e-5, mx
        qh = qn.cpu().numpy()
        for s_ in check:
            pos = lengths[s_] + st
            for layer in range(L):
                kv = H.read_layer_kv(ctx, s_, layer, pos + 1, 4096)
                ref = O.attention(kv, pos, qh[layer, s_:s_ + 1], threads=8)[0]
                mx, rms = H.err_stats(got[layer, s_], ref)
                assert mx < H.MAX_ABS and rms < H.RMS, (s_, layer, st, mx, rms)
        ctx.commit_batch(seqs)
    assert all(ctx.position(s_) == lengths[s_] + steps for s_ in seqs)
    ctx.close()


def _decode_ref_and_fused(L, P, steps, seed, q_out_too=True):
    """Two contexts with the same P-row history: one decodes with qa_append + qa_attn_decode,
    the other with the fused qa_decode_step. Returns per-step (ref, fused) outputs and the
    contexts."""
    ref, fus = make_ctx(L, context=4096), make_ctx(L, context=4096)
    qw, kw = H.norms(seed, L)
    for c in (ref, fus):
        H.set_norms(c, qw, kw)
    q, k, v = H.inputs(seed, L, 0, P + steps)
    if P:
        hist = [t[:, :P].contiguous() for t in (q, k, v)]
        for c in (ref, fus):
            gpu_append(c, 0, 0, *hist)
            c.commit(0, P)
    res = []
    for st in range(steps):
        p = P + st
        q1, k1, v1 = (t[:, p:p + 1].contiguous() for t in (q, k, v))
        qn_r, out_r = torch.empty_like(q1), torch.empty_like(q1)
        ref.append(0, 0, L, p, 1, q1.data_ptr(), k1.data_ptr(), v1.data_ptr(), qn_r.data_ptr())
        ref.attn_decode(0, 0, L, p, 1, qn_r.data_ptr(), out_r.data_ptr())
        ref.commit(0, 1)
        qn_f = torch.full_like(q1, float("nan"))
        out_f = torch.full_like(q1, float("nan"))
        fus.decode_step(0, 0, L, p, q1.data_ptr(), k1.data_ptr(), v1.data_ptr(),
                        qn_f.data_ptr() if q_out_too else 0, out_f.data_ptr())
        fus.commit(0, 1)
        torch.cuda.synchronize()
        res.append((qn_r, out_r, qn_f, out_f, (q1, k1, v1)))
    return ref, fus, res, (qw, kw)


@pytest.mark.parametrize("P", [0, 5, 40, 3000])
def test_fused_decode_step_is_bit_identical_to_append_then_decode(P):
    """qa_decode_step writes the same K/V bits and q_out as qa_append and returns the same
    attention output bits as qa_attn_decode: the first token (P = 0, the new row is the only
    key), P = 5, P = 40 (one CTA range spans three units) and a 3000-row history. The short
    contexts (P = 0, 5) take the entry point's append + decode fallback; the others run the
    single fused kernel."""
    L, steps = 28, 3
    ref, fus, res, _ = _decode_ref_and_fused(L, P, steps, 70 + P)
    for qn_r, out_r, qn_f, out_f, _ in res:
        assert torch.equal(qn_r, qn_f)
        assert torch.equal(out_r, out_f)
    for layer in (0, 13, 27):
        for h in range(8):
            for kvsel in (0, 1):
                assert np.array_equal(H.read_plane(ref, 0, layer, kvsel, h, 0, P + steps),
                                      H.read_plane(fus, 0, layer, kvsel, h, 0, P + steps))
    assert fus.position(0) == P + steps
    ref.close(); fus.close()


def test_fused_decode_step_without_q_out_and_against_the_oracle():
    L, P, steps = 2, 140, 2
    ref, fus, res, (qw, kw) = _decode_ref_and_fused(L, P, steps, 81, q_out_too=False)
    for qn_r, out_r, qn_f, out_f, _ in res:
        assert torch.equal(out_r, out_f)
        assert torch.isnan(qn_f).all()            # q_out = NULL: nothing written
    q, k, v = H.inputs(81, L, 0, P + steps)
    qh, kh, vh = (t.cpu().numpy() for t in (q, k, v))
    for layer in range(L):
        kv, qref = oracle_layer(qh[layer], kh[layer], vh[layer], qw[layer], kw[layer], 0, ctx_len=4096)
        for st in range(steps):
            o = O.attention(kv, P + st, qref[P + st:P + st + 1], threads=8)[0]
            mx, rms = H.err_stats(res[st][3][layer, 0].cpu().numpy(), o)
            assert mx < H.MAX_ABS and rms < H.RMS, (layer, st, mx, rms)
    ref.close(); fus.close()


def test_fused_decode_step_batch_64_requests():
    """qa_decode_step_batch over the 64 config-5 sequences equals qa_append_batch +
    qa_attn_decode_batch bit for bit (outputs, q_out and the new K/V rows)."""
    from fpga_qwen_b200 import dist as qd
    L = 2
    lengths = qd.config5_lengths()
    S = len(lengths)
    ctxs = [make_ctx(L, max_seqs=S, context=4096) for _ in range(2)]
    qw, kw = H.norms(92, L)
    for c in ctxs:
        H.set_norms(c, qw, kw)
    for s_, n in enumerate(lengths):
        q, k, v = H.inputs(3000 + s_, L, 0, n)
        for c in ctxs:
            gpu_append(c, s_, 0, q, k, v)
            c.commit(s_, n)
        torch.cuda.synchronize()
        del q, k, v
    seqs = list(range(S))
    for st in range(2):
        rows = [H.inputs(3000 + s_, L, lengths[s_] + st, 1) for s_ in seqs]
        qb, kb, vb = (torch.cat([r[i] for r in rows], dim=1).contiguous() for i in range(3))
        qn_r, out_r = torch.empty_like(qb), torch.empty_like(qb)
        ctxs[0].append_batch(seqs, 0, L, qb.data_ptr(), kb.data_ptr(), vb.data_ptr(), qn_r.data_ptr())
        ctxs[0].attn_decode_batch(seqs, 0, L, qn_r.data_ptr(), out_r.data_ptr())
        qn_f, out_f = torch.full_like(qb, float("nan")), torch.full_like(qb, float("nan"))
        ctxs[1].decode_step_batch(seqs, 0, L, qb.data_ptr(), kb.data_ptr(), vb.data_ptr(), qn_f.data_ptr(),
                                  out_f.data_ptr())
        for c in ctxs:
            c.commit_batch(seqs)
        torch.cuda.synchronize()
        assert torch.equal(qn_r, qn_f)
        assert torch.equal(out_r, out_f)
    for s_ in (0, 7, 40, 63):
        n = lengths[s_] + 2
        for kvsel in (0, 1):
            assert np.array_equal(H.read_plane(ctxs[0], s_, 1, kvsel, 3, n - 3, 3),
                                  H.read_plane(ctxs[1], s_, 1, kvsel, 3, n - 3, 3))
    for c in ctxs:
        c.close()


def test_fused_decode_step_host_buffers():
    """The io_host form of qa_decode_step (host input/output arrays, copies inside the call)
    gives the device form's results."""
    L, P = 4, 200
    dev = make_ctx(L, context=1024)
    host = qattn.Context(n_layers=L, context=1024, io_host=1)
    qw, kw = H.norms(93, L)
    q, k, v = H.inputs(93, L, 0, P + 1)
    for c in (dev, host):
        H.set_norms(c, qw, kw)
    gpu_append(dev, 0, 0, *(t[:, :P].contiguous() for t in (q, k, v)))
    dev.commit(0, P)
    qh, kh, vh = (np.ascontiguousarray(t[:, :P].cpu().numpy()) for t in (q, k, v))
    qo = np.empty_like(qh)
    host.append(0, 0, L, 0, P, qh.ctypes.data, kh.ctypes.data, vh.ctypes.data, qo.ctypes.data)
    host.commit(0, P)
    q1, k1, v1 = (t[:, P:P + 1].contiguous() for t in (q, k, v))
    qn_d, out_d = torch.empty_like(q1), torch.empty_like(q1)
    dev.decode_step(0, 0, L, P, q1.data_ptr(), k1.data_ptr(), v1.data_ptr(), qn_d.data_ptr(), out_d.data_ptr())
    torch.cuda.synchronize()
    qh1, kh1, vh1 = (np.ascontiguousarray(t.cpu().numpy()) for t in (q1, k1, v1))
    qn_h, out_h = np.empty_like(qh1), np.empty_like(qh1)
    host.decode_step(0, 0, L, P, qh1.ctypes.data, kh1.ctypes.data, vh1.ctypes.data, qn_h.ctypes.data, out_h.ctypes.data)
    assert np.array_equal(qn_h, qn_d.cpu().numpy())
    assert np.array_equal(out_h, out_d.cpu().numpy())
    dev.close(); host.close()


def test_pinned_host_buffers_go_direct():
    """io_host calls whose host buffers are all pinned (here torch's pin_memory) let the kernels
    read inputs and write outputs over PCIe with no staging copy: fused decode steps with and
    without q_out, an attention-only decode and a one-row append give the device-pointer
    context's results bit for bit; a misaligned pinned buffer falls back to the staging copies
    with the same results."""
    L, P = 28, 300
    dev = make_ctx(L, context=1024)
    host = qattn.Context(n_layers=L, context=1024, io_host=1)
    qw, kw = H.norms(94, L)
    q, k, v = H.inputs(94, L, 0, P + 4)
    for c in (dev, host):
        H.set_norms(c, qw, kw)
    gpu_append(dev, 0, 0, *(t[:, :P].contiguous() for t in (q, k, v)))
    dev.commit(0, P)
    qh, kh, vh = (np.ascontiguousarray(t[:, :P].cpu().numpy()) for t in (q, k, v))
    qo = np.empty_like(qh)
    host.append(0, 0, L, 0, P, qh.ctypes.data, kh.ctypes.data, vh.ctypes.data, qo.ctypes.data)
    host.commit(0, P)

    def pinned(t):
        return t.cpu().pin_memory()

    for s, with_q in ((0, True), (1, False)):
        q1, k1, v1 = (t[:, P + s:P + s + 1].contiguous() for t in (q, k, v))
        qn_d, out_d = torch.empty_like(q1), torch.empty_like(q1)
        dev.decode_step(0, 0, L, P + s, q1.data_ptr(), k1.data_ptr(), v1.data_ptr(), qn_d.data_ptr(), out_d.data_ptr())
        dev.commit(0, 1)
        torch.cuda.synchronize()
        qp, kp, vp = (pinned(t) for t in (q1, k1, v1))
        qn_h, out_h = torch.full_like(qp, float("nan")).pin_memory(), torch.full_like(qp, float("nan")).pin_memory()
        host.decode_step(0, 0, L, P + s, qp.data_ptr(), kp.data_ptr(), vp.data_ptr(),
                         qn_h.data_ptr() if with_q else 0, out_h.data_ptr())
        host.commit(0, 1)
        assert torch.equal(out_h, out_d.cpu())
        if with_q:
            assert torch.equal(qn_h, qn_d.cpu())
    # one layer per call, as an engine that runs its projections between the layers calls it:
    # each unit is split over many CTAs, so the pinned buffers go through the staging copies
    q1, k1, v1 = (t[:, P + 2:P + 3].contiguous() for t in (q, k, v))
    qp, kp, vp = (pinned(t) for t in (q1, k1, v1))
    out_d = torch.empty_like(q1)
    out_h = torch.full_like(qp, float("nan")).pin_memory()
    for layer in range(L):
        dev.decode_step(0, layer, 1, P + 2, q1[layer].data_ptr(), k1[layer].data_ptr(), v1[layer].data_ptr(), 0,
                        out_d[layer].data_ptr())
        host.decode_step(0, layer, 1, P + 2, qp[layer].data_ptr(), kp[layer].data_ptr(), vp[layer].data_ptr(), 0,
                         out_h[layer].data_ptr())
    dev.commit(0, 1)
    host.commit(0, 1)
    torch.cuda.synchronize()
    assert torch.equal(out_h, out_d.cpu())
    # attention-only decode of the committed rows at P + 3 after a one-row append, both pinned
    q1, k1, v1 = (t[:, P + 3:P + 4].contiguous() for t in (q, k, v))
    qn_d = gpu_append(dev, 0, P + 3, q1, k1, v1)
    out_d = gpu_attend(dev, 0, P + 3, qn_d, decode=True)
    torch.cuda.synchronize()
    qp, kp, vp = (pinned(t) for t in (q1, k1, v1))
    qn_h = torch.empty_like(qp).pin_memory()
    host.append(0, 0, L, P + 3, 1, qp.data_ptr(), kp.data_ptr(), vp.data_ptr(), qn_h.data_ptr())
    assert torch.equal(qn_h, qn_d.cpu())
    out_h = torch.empty_like(qp).pin_memory()
    host.attn_decode(0, 0, L, P + 3, 1, qn_h.data_ptr(), out_h.data_ptr())
    assert torch.equal(out_h, out_d.cpu())
    # a pinned buffer 4 bytes off a 16-byte boundary takes the staging copies
    big = torch.empty(qn_h.numel() + 4).pin_memory()
    shifted = big[1:1 + qn_h.numel()].view_as(qn_h)
    shifted.copy_(qn_h)
    out_s = torch.empty(out_h.numel() + 4).pin_memory()[1:1 + out_h.numel()].view_as(out_h)
    host.attn_decode(0, 0, L, P + 3, 1, shifted.data_ptr(), out_s.data_ptr())
    assert torch.equal(out_s, out_d.cpu())
    dev.close(); host.close()


def test_host_buffer_calls_in_layer_chunks_and_per_layer():
    """io_host calls whose rows x layers exceed the staging made at creation (one layer of the
    context's rows) run in layer chunks; per-layer decode steps, the shape an engine that
    interleaves its projections makes, go through the packed one-copy-each-way path. Both give
    the device-pointer context's results bit for bit."""
    L, P, steps = 6, 1000, 3
    dev = make_ctx(L, context=1024)
    host = qattn.Context(n_layers=L, context=1024, io_host=1)
    qw, kw = H.norms(96, L)
    for c in (dev, host):
        H.set_norms(c, qw, kw)
    q, k, v = H.inputs(96, L, 0, P + steps)
    qd, kd, vd = (t[:, :P].contiguous() for t in (q, k, v))
    qn_d = gpu_append(dev, 0, 0, qd, kd, vd)
    out_d = gpu_attend(dev, 0, 0, qn_d)
    dev.commit(0, P)
    qh, kh, vh = (np.ascontiguousarray(t[:, :P].cpu().numpy()) for t in (q, k, v))
    qn_h, out_h = np.empty_like(qh), np.empty_like(qh)
    host.append(0, 0, L, 0, P, qh.ctypes.data, kh.ctypes.data, vh.ctypes.data, qn_h.ctypes.data)
    host.attn_prefill(0, 0, L, 0, P, qn_h.ctypes.data, out_h.ctypes.data)
    host.commit(0, P)
    torch.cuda.synchronize()
    assert np.array_equal(qn_h, qn_d.cpu().numpy())
    assert np.array_equal(out_h, out_d.cpu().numpy())
    keep = []
    for st in range(steps):
        p = P + st
        for layer in range(L):
            r = [t[layer:layer + 1, p:p + 1].contiguous() for t in (q, k, v)]
            keep.extend(r)
            qo_d, o_d = torch.empty_like(r[0]), torch.empty_like(r[0])
            dev.decode_step(0, layer, 1, p, r[0].data_ptr(), r[1].data_ptr(), r[2].data_ptr(), qo_d.data_ptr(),
                            o_d.data_ptr())
            rh = [np.ascontiguousarray(t.cpu().numpy()) for t in r]
            qo_h, o_h = np.empty_like(rh[0]), np.empty_like(rh[0])
            host.decode_step(0, layer, 1, p, rh[0].ctypes.data, rh[1].ctypes.data, rh[2].ctypes.data,
                             qo_h.ctypes.data, o_h.ctypes.data)
            torch.cuda.synchronize()
            assert np.array_equal(qo_h, qo_d.cpu().numpy()) and np.array_equal(o_h, o_d.cpu().numpy())
        dev.commit(0, 1)
        host.commit(0, 1)
    for layer in (0, L - 1):
        for kvsel in (0, 1):
            assert np.array_equal(H.read_plane(dev, 0, layer, kvsel, 2, 0, P + steps),
                                  H.read_plane(host, 0, layer, kvsel, 2, 0, P + steps))
    dev.close(); host.close()


def test_fused_decode_step_batch_long_sequences():
    """A batch whose CTA ranges stay within four units (three sequences of 3000-4000 rows,
    28 layers) runs the fused kernel; it equals qa_append_batch + qa_attn_decode_batch."""
    L, lengths = 28, [3000, 3500, 4000]
    S = len(lengths)
    ctxs = [make_ctx(L, max_seqs=S, context=4096) for _ in range(2)]
    qw, kw = H.norms(94, L)
    for c in ctxs:
        H.set_norms(c, qw, kw)
    for s_, n in enumerate(lengths):
        q, k, v = H.inputs(4000 + s_, L, 0, n - 1)
        for c in ctxs:
            gpu_append(c, s_, 0, q, k, v)
            c.commit(s_, n - 1)
        torch.cuda.synchronize()
        del q, k, v
    seqs = list(range(S))
    rows = [H.inputs(4000 + s_, L, lengths[s_] - 1, 1) for s_ in seqs]
    qb, kb, vb = (torch.cat([r[i] for r in rows], dim=1).contiguous() for i in range(3))
    qn_r, out_r = torch.empty_like(qb), torch.empty_like(qb)
    ctxs[0].append_batch(seqs, 0, L, qb.data_ptr(), kb.data_ptr(), vb.data_ptr(), qn_r.data_ptr())
    ctxs[0].attn_decode_batch(seqs, 0, L, qn_r.data_ptr(), out_r.data_ptr())
    qn_f, out_f = torch.full_like(qb, float("nan")), torch.full_like(qb, float("nan"))
    ctxs[1].decode_step_batch(seqs, 0, L, qb.data_ptr(), kb.data_ptr(), vb.data_ptr(), qn_f.data_ptr(),
                              out_f.data_ptr())
    torch.cuda.synchronize()
    ctxs[1].sync()
    assert torch.equal(qn_r, qn_f)
    assert torch.equal(out_r, out_f)
    for s_, n in enumerate(lengths):
        for kvsel in (0, 1):
            assert np.array_equal(H.read_plane(ctxs[0], s_, 27, kvsel, 5, n - 1, 1),
                                  H.read_plane(ctxs[1], s_, 27, kvsel, 5, n - 1, 1))
    for c in ctxs:
        c.close()


def test_overlapped_decode_steps_match_serial_steps():
    """With qa_set_step_overlap on, 24 fused decode steps issued back to back (each starting
    while the previous one finishes) write the same K/V rows and outputs as the same steps
    with the overlap off; a prefix copy issued in between ends the overlap for one step."""
    L, P, steps = 28, 3000, 24
    ctxs = [make_ctx(L, max_seqs=2, context=4096) for _ in range(2)]
    qw, kw = H.norms(95, L)
    q, k, v = H.inputs(95, L, 0, P + steps)
    hist = [t[:, :P].contiguous() for t in (q, k, v)]
    rows = [[t[:, p:p + 1].contiguous() for t in (q, k, v)] for p in range(P, P + steps)]
    outs = []
    for idx, c in enumerate(ctxs):
        H.set_norms(c, qw, kw)
        gpu_append(c, 0, 0, *hist)
        c.commit(0, P)
        c.set_step_overlap(idx == 1)
        o = torch.empty((steps, L, 1, 16, 128), device="cuda")
        for st in range(steps):
            if st == 12:
                c.copy_prefix(0, 1, 512)           # another kernel between two steps
            q1, k1, v1 = rows[st]
            c.decode_step(0, 0, L, P + st, q1.data_ptr(), k1.data_ptr(), v1.data_ptr(), 0, o[st].data_ptr())
            c.commit(0, 1)
        outs.append(o)
    torch.cuda.synchronize()
    for c in ctxs:
        c.sync()
    assert torch.equal(outs[0], outs[1])
    for layer in (0, 27):
        for kvsel in (0, 1):
            assert np.array_equal(H.read_plane(ctxs[0], 0, layer, kvsel, 6, P - 2, steps + 2),
                                  H.read_plane(ctxs[1], 0, layer, kvsel, 6, P - 2, steps + 2))
    for c in ctxs:
        c.close()
