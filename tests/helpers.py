"""Shared helpers of the GPU parity tests: seeded inputs on the device, oracle replay."""
from __future__ import annotations

import numpy as np
import torch

from fpga_qwen_b200 import qattn
from oracle import oracle as O

D = 128
KIND_Q, KIND_K, KIND_V, KIND_QN, KIND_KN = range(5)


def synth(seed, kind, layer0, n_layers, pos0, n, head0, heads, mean=0.0, std=1.0):
    t = torch.empty((n_layers, n, heads, D), dtype=torch.float32, device="cuda")
    qattn.synth_fill(t.data_ptr(), seed, kind, layer0, n_layers, pos0, n, head0, heads, mean, std,
                     torch.cuda.current_stream().cuda_stream)
    return t


def inputs(seed, layers, pos0, n, hkv=8, head0=0, layer0=0):
    """Pre-norm q [L][n][2*hkv][128], k, v [L][n][hkv][128] on the GPU (N(0,1))."""
    q = synth(seed, KIND_Q, layer0, layers, pos0, n, 2 * head0, 2 * hkv)
    k = synth(seed, KIND_K, layer0, layers, pos0, n, head0, hkv)
    v = synth(seed, KIND_V, layer0, layers, pos0, n, head0, hkv)
    return q, k, v


def norms(seed, layers):
    """Per-layer q_norm, k_norm weights [L][128] ~ N(1, 0.05) (host numpy)."""
    qn = synth(seed, KIND_QN, 0, layers, 0, 1, 0, 1, 1.0, 0.05).reshape(layers, D)
    kn = synth(seed, KIND_KN, 0, layers, 0, 1, 0, 1, 1.0, 0.05).reshape(layers, D)
    return qn.cpu().numpy(), kn.cpu().numpy()


def set_norms(ctx, qn, kn):
    for layer in range(qn.shape[0]):
        a, b = np.ascontiguousarray(qn[layer]), np.ascontiguousarray(kn[layer])
        ctx.set_norms(layer, a.ctypes.data, b.ctypes.data)


def read_plane(ctx, seq, layer, kv, head, pos0, n):
    out = np.empty((n, D), np.uint16)
    ctx.read_kv(seq, layer, kv, head, pos0, n, out.ctypes.data)
    return out


def read_layer_kv(ctx, seq, layer, ntok, oracle_ctx):
    """The GPU's FP16 planes of one layer, as an oracle LayerKV with context oracle_ctx."""
    kv = O.LayerKV(ctx.hkv, oracle_ctx)
    for h in range(ctx.hkv):
        kv.k[h, :ntok] = read_plane(ctx, seq, layer, 0, h, 0, ntok)
        kv.v[h, :ntok] = read_plane(ctx, seq, layer, 1, h, 0, ntok)
    return kv


def err_stats(out, ref):
    d = np.abs(np.asarray(out, np.float64) - np.asarray(ref, np.float64))
    return float(d.max()), float(np.sqrt((d * d).mean()))


MAX_ABS = 1e-3   # north_star tolerance on attention outputs
RMS = 1e-4


# Worst attention error seen per named case in this session, printed in pytest's terminal
# summary (tests/conftest.py) so that a GPU run's log carries the parity figures.
PARITY = {}


def record(name, mx, rms, rows):
    """Keeps the worst max-abs and RMS of `name` over the calls; `rows` counts compared rows."""
    old = PARITY.get(name)
    if old is None:
        PARITY[name] = [mx, rms, rows]
    else:
        old[0], old[1], old[2] = max(old[0], mx), max(old[1], rms), old[2] + rows


def check(name, got, ref):
    """Attention outputs within the north_star tolerance (max-abs 1e-3, RMS 1e-4); recorded."""
    mx, rms = err_stats(got, ref)
    record(name, mx, rms, int(np.prod(np.shape(got)[:-2])) if np.ndim(got) >= 2 else 1)
    assert mx < MAX_ABS and rms < RMS, (name, mx, rms)
    return mx, rms
