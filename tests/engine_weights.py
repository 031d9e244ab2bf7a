"""The synthetic checkpoint of tests/golden/numpyqwen_engine.npz, regenerated without the
reference: make_golden.checkpoint_tensors with the fixture's seed, BF16-rounded as NumpyQwen
reads them, matrices rounded to FP16 (weight_precision='f16')."""
from __future__ import annotations

import sys
from pathlib import Path

import numpy as np

GOLDEN = Path(__file__).resolve().parent / "golden"


def engine_weights():
    sys.path.insert(0, str(GOLDEN))
    import make_golden as G
    rng = np.random.default_rng(G.ENGINE_SEED)
    out = {}
    for name, value in G.checkpoint_tensors(rng).items():
        v = G.bf16_values(value)
        if v.ndim == 2:
            v = v.astype(np.float16).astype(np.float32)
        out[name] = v
    return out, G.H, G.F, G.V
