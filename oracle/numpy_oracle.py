"""Second, independent formula check: a NumPy restatement of the reference's NumPy oracle.

TEST INFRASTRUCTURE ONLY (tests/ import it as a checker).

It restates the attention math of tampajohn/fpga-qwen ``tests/test_full_model.py:44-71``
(``NumpyQwen.token``), generalised to a batch of causal rows:

* ``norm``: ``x / sqrt(mean(x*x) + 1e-6) * w`` in FP32 (:44-45) — note the reference's
  NumPy oracle uses an FP32 mean, not the C++ engine's FP64 sum, so it agrees with the C++
  restatement to a few ulp, not bit for bit.
* ``rope``: split halves, ``left*cos - right*sin``, ``right*cos + left*sin`` (:46-50).
* current K and V rounded to FP16 before attention (:60-63).
* ``np.repeat(…, 2, axis=1)`` GQA (:67); scores ``einsum / float32(sqrt(128))``; max-subtract,
  ``exp``, normalise, ``einsum`` with V (:68-71).
"""
from __future__ import annotations

import numpy as np


def rope_tables(context: int):
    pos = np.arange(context, dtype=np.float64)[:, None]
    angle = pos / (1000000.0 ** (np.arange(64, dtype=np.float64) * 2 / 128))
    return np.cos(angle).astype(np.float32), np.sin(angle).astype(np.float32)


def norm(x, weight):
    x = x.astype(np.float32)
    return x / np.sqrt(np.mean(x * x, axis=-1, keepdims=True) + np.float32(1e-6)) * weight


def rope(x, cos, sin):
    left, right = np.split(x, 2, axis=-1)
    return np.concatenate((left * cos - right * sin, right * cos + left * sin), axis=-1)


def append(q_pre, k_pre, v_pre, qw, kw, positions):
    """Returns (q, k16, v16): normed+roped q FP32 and FP16-rounded k, v (as float32)."""
    cos, sin = rope_tables(int(positions.max()) + 1)
    c, s = cos[positions][:, None, :], sin[positions][:, None, :]
    q = rope(norm(q_pre, qw), c, s).astype(np.float32)
    k = rope(norm(k_pre, kw), c, s).astype(np.float16).astype(np.float32)
    v = v_pre.astype(np.float16).astype(np.float32)
    return q, k, v


def attention(q, keys, vals, pos0):
    """q ``[n][hq][128]``; keys/vals ``[t][hkv][128]`` (FP16 values as float32) holding at
    least ``pos0+n`` positions. Row b sees keys ``[0, pos0+b]``."""
    n, hq, _ = q.shape
    group = hq // keys.shape[1]
    out = np.empty_like(q)
    for b in range(n):
        t = pos0 + b + 1
        kk = np.repeat(keys[:t], group, axis=1)
        vv = np.repeat(vals[:t], group, axis=1)
        scores = np.einsum('hd,thd->ht', q[b], kk) / np.float32(np.sqrt(128))
        probs = np.exp(scores - scores.max(axis=-1, keepdims=True))
        probs /= probs.sum(axis=-1, keepdims=True)
        out[b] = np.einsum('ht,thd->hd', probs, vv)
    return out
