"""NumPy/ctypes front end of the C++ CPU restatement (``qattn_oracle.cpp``).

TEST INFRASTRUCTURE ONLY: imported by tests/, ``__graft_entry__.smoke()`` and the
CPU-baseline / reference arm of ``bench.py`` as the checker. The product library never
imports it.

Every function mirrors one piece of tampajohn/fpga-qwen ``engine/core.cpp``; the C++
file's header lists the line ranges. Parity of this restatement is pinned against the
reference's own NumPy oracle (``tests/test_full_model.py:44-71``) through the fixtures
in ``tests/golden/`` and against known-answer cases in ``tests/test_oracle.py``.
"""
from __future__ import annotations

import ctypes
import os
import subprocess
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
LIB_PATH = HERE / "liboracle_qattn.so"
D = 128

_lib = None


def build() -> Path:
    """Compile the restatement with its Makefile (idempotent)."""
    subprocess.run(["make", "-s", "-C", str(HERE)], check=True)
    return LIB_PATH


def lib() -> ctypes.CDLL:
    global _lib
    if _lib is None:
        if not LIB_PATH.exists():
            build()
        _lib = ctypes.CDLL(str(LIB_PATH))
        f32p = np.ctypeslib.ndpointer(np.float32, flags="C_CONTIGUOUS")
        u16p = np.ctypeslib.ndpointer(np.uint16, flags="C_CONTIGUOUS")
        i = ctypes.c_int
        _lib.qo_rope_tables.argtypes = [i, f32p, f32p]
        _lib.qo_norm.argtypes = [f32p, f32p, f32p, i]
        _lib.qo_rope.argtypes = [f32p, f32p, f32p]
        _lib.qo_f32_to_f16.argtypes = [f32p, u16p, ctypes.c_size_t]
        _lib.qo_f16_to_f32.argtypes = [u16p, f32p, ctypes.c_size_t]
        _lib.qo_append.argtypes = [i, i, i, i, i, f32p, f32p, f32p, f32p, f32p, f32p, f32p,
                                   f32p, u16p, u16p]
        _lib.qo_attention.argtypes = [i, i, i, i, i, f32p, u16p, u16p, f32p, i]
        _lib.qo_project.argtypes = [f32p, u16p, i, i, i, i, f32p, i]
        _lib.qo_mlp_gate.argtypes = [f32p, f32p, ctypes.c_size_t]
        for name in ("qo_rope_tables", "qo_norm", "qo_rope", "qo_f32_to_f16", "qo_f16_to_f32",
                     "qo_append", "qo_attention", "qo_release_pool", "qo_project", "qo_mlp_gate"):
            getattr(_lib, name).restype = None
    return _lib


def _f32(a):
    return np.ascontiguousarray(a, dtype=np.float32)


def rope_tables(context: int):
    """``[context][64]`` cos and sin tables (core.cpp:287-288)."""
    c = np.empty((context, 64), np.float32)
    s = np.empty((context, 64), np.float32)
    lib().qo_rope_tables(context, c, s)
    return c, s


def norm(x, w):
    """Per-row RMSNorm of core.cpp:207-215 (rows of length w.size)."""
    x = _f32(x)
    out = np.empty_like(x)
    n = w.size
    flat_in, flat_out = x.reshape(-1, n), out.reshape(-1, n)
    for r in range(flat_in.shape[0]):
        row = np.empty(n, np.float32)
        lib().qo_norm(np.ascontiguousarray(flat_in[r]), _f32(w), row, n)
        flat_out[r] = row
    return out


def f32_to_f16_bits(x):
    x = _f32(x)
    out = np.empty(x.shape, np.uint16)
    lib().qo_f32_to_f16(x.reshape(-1), out.reshape(-1), x.size)
    return out


class LayerKV:
    """One layer's KV planes in the reference's per-layer layout ``[hkv][ctx][128]`` FP16."""

    def __init__(self, hkv: int, ctx: int):
        self.hkv, self.ctx = hkv, ctx
        self.k = np.zeros((hkv, ctx, D), np.uint16)
        self.v = np.zeros((hkv, ctx, D), np.uint16)


def append(kv: LayerKV, pos0: int, q_pre, k_pre, v_pre, qw, kw, tables):
    """Norm + RoPE + FP16 KV write for rows at positions ``pos0..pos0+n-1`` (core.cpp:395-406).

    Returns the normed and roped query ``[n][hq][128]`` FP32.
    """
    q_pre, k_pre, v_pre = _f32(q_pre), _f32(k_pre), _f32(v_pre)
    n, hq = q_pre.shape[0], q_pre.shape[1]
    q_out = np.empty_like(q_pre)
    cos, sin = tables
    lib().qo_append(hq, kv.hkv, kv.ctx, pos0, n, q_pre, k_pre, v_pre, _f32(qw), _f32(kw),
                    cos, sin, q_out, kv.k, kv.v)
    return q_out


def attention(kv: LayerKV, pos0: int, q, threads: int = 1):
    """Causal GQA attention of rows at positions ``pos0..pos0+n-1`` (core.cpp:407-624)."""
    q = _f32(q)
    n, hq = q.shape[0], q.shape[1]
    out = np.empty_like(q)
    lib().qo_attention(hq, kv.hkv, kv.ctx, pos0, n, q, kv.k, kv.v, out, int(threads))
    return out


def project(x, w_f16, sgemm: bool = False, threads: int = 1):
    """core.cpp:292-301: x [batch][cols] FP32 through w [rows][cols] FP16 bits -> [batch][rows].
    sgemm=False: the eight-lane dot per output (one row, or the FP16-only vocabulary matrix);
    sgemm=True: ascending-column FP32 sum standing in for cblas_sgemm (parity by tolerance)."""
    x = _f32(np.atleast_2d(x))
    w = np.ascontiguousarray(w_f16, dtype=np.uint16)
    rows, cols = w.shape
    if cols % 8 or x.shape[1] != cols:
        raise ValueError("columns must match and be a multiple of 8")
    y = np.empty((x.shape[0], rows), np.float32)
    lib().qo_project(x, w, rows, cols, x.shape[0], int(sgemm), y, threads)
    return y


def mlp_gate(gate, up):
    """core.cpp:636-639: gate * (0.5 + 0.5*tanh(gate*0.5)) * up (glibc tanhf for vvtanhf)."""
    g = _f32(gate).copy()
    lib().qo_mlp_gate(g, _f32(up), g.size)
    return g
