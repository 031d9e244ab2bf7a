"""The north_star workloads end to end on the GPU, checked in full against the oracle.

Each test runs one workload at its stated shape through the C ABI and compares every row of
every layer with the CPU restatement of engine/core.cpp: KV bytes and normalised queries
bit-exact, attention outputs within max-abs 1e-3 / RMS 1e-4 (north_star tolerance):

* 452-row prefill + 32 decode steps (the multi-tile causal prefill; fused decode steps);
* canonical prefix reuse: request A prefills 1024 rows as two 512-row chunks (core.cpp:712);
  request B copies A's 512-row prefix, prefills its own 512-row tail and decodes 128 steps;
  B equals a fresh prefill of the same rows bit for bit, and the oracle within tolerance;
* 3968-row prefill + 128 decode steps (overlapped fused decode steps, as the benchmark runs);
* 64 requests with the seeded U[85, 3968] prompt lengths, each prefilled, then 128 batched
  fused decode steps over all of them;
* the reference's own NumPy oracle on 200 tokens (tests/golden/numpyqwen_t200.npz), whose
  rows at positions >= 128 run on the tensor-core kernel.

The worst error per case is printed in pytest's terminal summary.
"""
import os

import numpy as np
import pytest
import torch

from fpga_qwen_b200 import qattn
from oracle import oracle as O
from tests import helpers as H

pytestmark = pytest.mark.gpu

THREADS = os.cpu_count() or 4
_TABLES = {}


def tables(n=4096):
    if n not in _TABLES:
        _TABLES[n] = O.rope_tables(n)
    return _TABLES[n]


def make_ctx(layers=28, max_seqs=1, context=4096, **kw):
    ctx = qattn.Context(n_layers=layers, max_seqs=max_seqs, context=context, **kw)
    ctx.set_stream(torch.cuda.current_stream().cuda_stream)
    return ctx


class Inputs:
    """Keeps every tensor handed to the library alive until the stream has consumed it."""

    def __init__(self):
        self.keep = []

    def __call__(self, t):
        t = t.contiguous()
        self.keep.append(t)
        return t


def prefill(ctx, seq, pos0, q, k, v, keep):
    L, n = q.shape[0], q.shape[1]
    qn, out = torch.empty_like(q), torch.empty_like(q)
    ctx.append(seq, 0, L, pos0, n, keep(q).data_ptr(), keep(k).data_ptr(), keep(v).data_ptr(), qn.data_ptr())
    ctx.attn_prefill(seq, 0, L, pos0, n, qn.data_ptr(), out.data_ptr())
    ctx.commit(seq, n)
    return qn, out


def oracle_rows(q, k, v, qw, kw, ctx_len):
    """Oracle append of rows 0..n-1 of one layer into planes of ctx_len rows; returns
    (LayerKV, normalised query rows)."""
    kv = O.LayerKV(k.shape[1], ctx_len)
    return kv, O.append(kv, 0, q, k, v, qw, kw, tables())


def assert_kv(ctx, seq, layer, kv, n):
    for h in range(kv.hkv):
        assert np.array_equal(H.read_plane(ctx, seq, layer, 0, h, 0, n), kv.k[h, :n]), ("K", layer, h)
        assert np.array_equal(H.read_plane(ctx, seq, layer, 1, h, 0, n), kv.v[h, :n]), ("V", layer, h)


# ---------------------------------------------------------------------------------------------
def test_golden200_through_the_gpu(golden200):
    """The reference NumpyQwen's 200-token inputs: one 200-row prefill, and the same rows as a
    127-row prefill followed by a 73-row chunk at position 127 (row 127 on FP32 cores, rows
    from 128 on the tensor cores). K/V and queries bit-exact with the restatement; outputs of
    rows 96..199 within tolerance of the reference oracle's own outputs and of the restatement."""
    rows = golden200["rows"]
    T = golden200["L27_q_pre"].shape[0]
    for layer in golden200["layers"]:
        g = {name: golden200[f"L{layer}_{name}"] for name in ("q_pre", "k_pre", "v_pre", "q_norm", "k_norm", "out")}
        kv, qref = oracle_rows(g["q_pre"], g["k_pre"], g["v_pre"], g["q_norm"], g["k_norm"], 256)
        ref = O.attention(kv, int(rows[0]), qref[rows], threads=THREADS)
        for split in (None, 127):
            ctx = make_ctx(1, context=256)
            H.set_norms(ctx, g["q_norm"][None], g["k_norm"][None])
            keep = Inputs()
            q, k, v = (torch.from_numpy(g[x][None].copy()).cuda() for x in ("q_pre", "k_pre", "v_pre"))
            if split is None:
                qn, out = prefill(ctx, 0, 0, q, k, v, keep)
            else:
                qa, oa = prefill(ctx, 0, 0, q[:, :split], k[:, :split], v[:, :split], keep)
                qb, ob = prefill(ctx, 0, split, q[:, split:], k[:, split:], v[:, split:], keep)
                qn, out = torch.cat([qa, qb], 1), torch.cat([oa, ob], 1)
            torch.cuda.synchronize()
            assert np.array_equal(qn.cpu().numpy()[0], qref)
            assert_kv(ctx, 0, 0, kv, T)
            got = out.cpu().numpy()[0][rows]
            H.check("golden200 vs reference NumpyQwen", got, g["out"])
            H.check("golden200 vs restatement", got, ref)
            ctx.close()


def test_config2_prefill_452_then_32_decode_steps():
    """452-row prefill + 32 fused decode steps over 28 layers: every row of every layer."""
    L, n, steps = 28, 452, 32
    ctx = make_ctx(L, context=512)
    qw, kw = H.norms(2, L)
    H.set_norms(ctx, qw, kw)
    q, k, v = H.inputs(2, L, 0, n + steps)
    keep = Inputs()
    qn, out = prefill(ctx, 0, 0, q[:, :n], k[:, :n], v[:, :n], keep)
    dq, dout = [], []
    for s in range(steps):
        p = n + s
        qo, o = torch.empty_like(q[:, p:p + 1]), torch.empty_like(q[:, p:p + 1])
        ctx.decode_step(0, 0, L, p, keep(q[:, p:p + 1]).data_ptr(), keep(k[:, p:p + 1]).data_ptr(),
                        keep(v[:, p:p + 1]).data_ptr(), qo.data_ptr(), o.data_ptr())
        ctx.commit(0, 1)
        dq.append(qo)
        dout.append(o)
    torch.cuda.synchronize()
    ctx.sync()
    qs = torch.cat([qn] + dq, 1).cpu().numpy()
    outs = torch.cat([out] + dout, 1).cpu().numpy()
    qh, kh, vh = q.cpu().numpy(), k.cpu().numpy(), v.cpu().numpy()
    for layer in range(L):
        kv, qref = oracle_rows(qh[layer], kh[layer], vh[layer], qw[layer], kw[layer], 512)
        assert np.array_equal(qs[layer], qref)
        assert_kv(ctx, 0, layer, kv, n + steps)
        ref = O.attention(kv, 0, qref, threads=THREADS)
        H.check("config2 prefill 452", outs[layer, :n], ref[:n])
        H.check("config2 decode 32 steps", outs[layer, n:], ref[n:])
    ctx.close()


def test_config3_prefix_reuse_then_128_decode_steps():
    """Request A prefills 1024 rows as two 512-row chunks. Request B copies A's canonical
    512-row prefix, prefills its own 512-row tail (new seed) at position 512 and decodes 128
    steps. B's KV rows and outputs equal a fresh prefill of the same rows (slot 2) bit for
    bit, and B's tail and decode outputs, like A's outputs, agree with the oracle."""
    L, steps = 28, 128
    ctx = make_ctx(L, max_seqs=3, context=1280)
    qw, kw = H.norms(3, L)
    H.set_norms(ctx, qw, kw)
    keep = Inputs()
    qa, ka, va = H.inputs(1234, L, 0, 1024)                       # request A
    _, a0 = prefill(ctx, 0, 0, qa[:, :512], ka[:, :512], va[:, :512], keep)
    _, a1 = prefill(ctx, 0, 512, qa[:, 512:], ka[:, 512:], va[:, 512:], keep)
    qt, kt, vt = H.inputs(5678, L, 512, 512 + steps)              # B's tail and decode rows
    outs = {}
    for seq in (1, 2):
        if seq == 1:
            ctx.copy_prefix(0, 1, 512)                            # reuse A's canonical block
        else:
            prefill(ctx, 2, 0, qa[:, :512], ka[:, :512], va[:, :512], keep)   # fresh: regenerate it
        _, tail = prefill(ctx, seq, 512, qt[:, :512], kt[:, :512], vt[:, :512], keep)
        dec = []
        for s in range(steps):
            p = 1024 + s
            r = slice(512 + s, 513 + s)
            qn1 = torch.empty_like(qt[:, r])
            ctx.append(seq, 0, L, p, 1, keep(qt[:, r]).data_ptr(), keep(kt[:, r]).data_ptr(),
                       keep(vt[:, r]).data_ptr(), qn1.data_ptr())
            o = torch.empty_like(qn1)
            ctx.attn_decode(seq, 0, L, p, 1, qn1.data_ptr(), o.data_ptr())
            ctx.commit(seq, 1)
            dec.append(o)
        outs[seq] = torch.cat([tail] + dec, 1)
    torch.cuda.synchronize()
    ctx.sync()
    assert ctx.position(1) == ctx.position(2) == 1024 + steps
    assert torch.equal(outs[1], outs[2])
    n_b = 1024 + steps
    a_out = torch.cat([a0, a1], 1).cpu().numpy()
    b_out = outs[1].cpu().numpy()
    qah, kah, vah = qa.cpu().numpy(), ka.cpu().numpy(), va.cpu().numpy()
    qth, kth, vth = qt.cpu().numpy(), kt.cpu().numpy(), vt.cpu().numpy()
    for layer in range(L):
        for kvsel in (0, 1):
            for h in range(8):
                assert np.array_equal(H.read_plane(ctx, 1, layer, kvsel, h, 0, n_b),
                                      H.read_plane(ctx, 2, layer, kvsel, h, 0, n_b))
        kv_a, q_a = oracle_rows(qah[layer], kah[layer], vah[layer], qw[layer], kw[layer], 1280)
        H.check("config3 request A prefill 2x512", a_out[layer], O.attention(kv_a, 0, q_a, threads=THREADS))
        qb = np.concatenate([qah[layer, :512], qth[layer]])
        kb = np.concatenate([kah[layer, :512], kth[layer]])
        vb = np.concatenate([vah[layer, :512], vth[layer]])
        kv_b, q_b = oracle_rows(qb, kb, vb, qw[layer], kw[layer], 1280)
        assert_kv(ctx, 1, layer, kv_b, n_b)
        ref = O.attention(kv_b, 512, q_b[512:], threads=THREADS)
        H.check("config3 request B tail 512 @ P=512", b_out[layer, :512], ref[:512])
        H.check("config3 request B decode 128 steps", b_out[layer, 512:], ref[512:])
    ctx.close()


def test_config4_prefill_3968_then_128_decode_steps():
    """3968-row prefill + 128 overlapped fused decode steps over 28 layers on one GPU, the
    benchmark's step: every row of every layer against the oracle, every KV byte exact."""
    L, n, steps = 28, 3968, 128
    ctx = make_ctx(L, context=4096)
    ctx.set_step_overlap(True)
    qw, kw = H.norms(21, L)
    H.set_norms(ctx, qw, kw)
    q, k, v = H.inputs(21, L, 0, n + steps)
    keep = Inputs()
    qn, out = prefill(ctx, 0, 0, q[:, :n], k[:, :n], v[:, :n], keep)
    dec = torch.empty((steps, L, 1, 16, 128), device="cuda")
    for s in range(steps):
        p = n + s
        ctx.decode_step(0, 0, L, p, keep(q[:, p:p + 1]).data_ptr(), keep(k[:, p:p + 1]).data_ptr(),
                        keep(v[:, p:p + 1]).data_ptr(), 0, dec[s].data_ptr())
        ctx.commit(0, 1)
    torch.cuda.synchronize()
    ctx.sync()
    for layer in range(L):
        qh, kh, vh = (t[layer].cpu().numpy() for t in (q, k, v))
        kv, qref = oracle_rows(qh, kh, vh, qw[layer], kw[layer], 4096)
        assert np.array_equal(qn[layer].cpu().numpy(), qref[:n])
        assert_kv(ctx, 0, layer, kv, n + steps)
        ref = O.attention(kv, 0, qref, threads=THREADS)
        H.check("config4 prefill 3968", out[layer].cpu().numpy(), ref[:n])
        H.check("config4 decode 128 steps", dec[:, layer, 0].cpu().numpy(), ref[n:])
    ctx.close()


def test_config5_64_requests_prefill_then_128_batched_decode_steps():
    """64 requests with the seeded U[85, 3968] prompt lengths: each prefilled over 28 layers,
    then 128 fused decode steps batched over all 64 sequences. Layers 0 and 27 are checked in
    full for every request (every prefill row, KV bytes, decode steps 0, 63 and 127); at step
    127 the batched outputs of every layer equal single-sequence decode steps."""
    from fpga_qwen_b200 import dist as qd
    L, steps = 28, 128
    lengths = qd.config5_lengths()
    S = len(lengths)
    check_layers, check_steps = (0, 27), (0, 63, 127)
    ctx = make_ctx(L, max_seqs=S, context=4096)
    qw, kw = H.norms(5, L)
    H.set_norms(ctx, qw, kw)
    ref_state = {}                    # (request, layer) -> oracle planes and decode query rows
    for s_, n in enumerate(lengths):
        q, k, v = H.inputs(5000 + s_, L, 0, n + steps)
        keep = Inputs()
        _, out = prefill(ctx, s_, 0, q[:, :n], k[:, :n], v[:, :n], keep)
        torch.cuda.synchronize()
        for layer in check_layers:
            qh, kh, vh = (t[layer].cpu().numpy() for t in (q, k, v))
            kv, qref = oracle_rows(qh, kh, vh, qw[layer], kw[layer], n + steps)
            H.check("config5 prefill (64 lengths)", out[layer].cpu().numpy(),
                    O.attention(kv, 0, qref[:n], threads=THREADS))
            ref_state[s_, layer] = (kv, qref[n:])
        del q, k, v, out, keep
    seqs = list(range(S))
    dec = {}
    single = None
    for st in range(steps):
        rows = [H.inputs(5000 + s_, L, lengths[s_] + st, 1) for s_ in seqs]
        qb, kb, vb = (torch.cat([r[i] for r in rows], dim=1).contiguous() for i in range(3))   # [L][S][h][128]
        if st == steps - 1:
            # the last step also as append + one decode per sequence (positions not yet committed)
            qn = torch.empty_like(qb)
            ctx.append_batch(seqs, 0, L, qb.data_ptr(), kb.data_ptr(), vb.data_ptr(), qn.data_ptr())
            single = torch.empty_like(qb)
            for s_ in seqs:
                q1 = qn[:, s_:s_ + 1].contiguous()
                o1 = torch.empty_like(q1)
                ctx.attn_decode(s_, 0, L, lengths[s_] + st, 1, q1.data_ptr(), o1.data_ptr())
                single[:, s_:s_ + 1] = o1
        out = torch.empty_like(qb)
        ctx.decode_step_batch(seqs, 0, L, qb.data_ptr(), kb.data_ptr(), vb.data_ptr(), 0, out.data_ptr())
        ctx.commit_batch(seqs)
        if st in check_steps:
            torch.cuda.synchronize()
            dec[st] = out.cpu().numpy()
    torch.cuda.synchronize()
    ctx.sync()
    mx, _ = H.err_stats(dec[steps - 1], single.cpu().numpy())
    assert mx < 1e-5, mx
    assert all(ctx.position(s_) == lengths[s_] + steps for s_ in seqs)
    for (s_, layer), (kv, qdec) in ref_state.items():
        n = lengths[s_]
        assert_kv(ctx, s_, layer, kv, n + steps)
        refd = np.stack([O.attention(kv, n + st, qdec[st:st + 1], threads=THREADS)[0] for st in check_steps])
        gotd = np.stack([dec[st][layer, s_] for st in check_steps])
        H.check("config5 batched decode (64 seqs)", gotd, refd)
    ctx.close()
