"""The oracle's projection restatement (core.cpp:292-301, :636-639), pinned against the
reference's own NumPy model.

tests/golden/numpyqwen_proj_t3.npz (tests/golden/make_golden.py --projections) records, at
layer 0 of a synthetic checkpoint run through NumpyQwen with FP16-rounded matrices, the
input and output of every matrix product, the MLP activation, the final normalised hidden
state and the logits. NumPy sums in its BLAS order, the engine in its eight-lane order
(or Accelerate's, for batched products), so the bar is a relative tolerance; the known-answer
and invariance cases below are exact.
"""
from pathlib import Path

import numpy as np
import pytest

from oracle import oracle as O

FIX = np.load(Path(__file__).parent / "golden" / "numpyqwen_proj_t3.npz")
REL = 2e-6         # |y - ref| <= REL * sum_j |x_j w_j| (FP32 sums of one row, any order)


def bound(x, w16):
    w = w16.view(np.float16).astype(np.float64)
    return np.abs(x.astype(np.float64)) @ np.abs(w).T


@pytest.mark.parametrize("kind", ["q", "k", "v", "o", "gate", "up", "down"])
@pytest.mark.parametrize("sgemm", [False, True])
def test_projection_matches_numpyqwen(kind, sgemm):
    x, w, ref = FIX[f"{kind}_in"], FIX[f"w_{kind}"], FIX[f"{kind}_out"]
    y = O.project(x, w, sgemm=sgemm)
    err = np.abs(y.astype(np.float64) - ref)
    assert np.all(err <= REL * bound(x, w) + 1e-30), (kind, err.max())


def test_mlp_activation_matches_numpyqwen():
    act = O.mlp_gate(FIX["gate_out"], FIX["up_out"])
    np.testing.assert_allclose(act, FIX["down_in"], rtol=2e-6, atol=1e-9)


def test_vocabulary_head_matches_numpyqwen():
    # the embedding matrix has no FP32 copy (core.cpp:267): the eight-lane dot per logit
    logits = O.project(FIX["final_hidden"], FIX["embed"])[0]
    err = np.abs(logits.astype(np.float64) - FIX["logits"])
    assert np.all(err <= REL * bound(FIX["final_hidden"][None], FIX["embed"])[0])


def test_one_hot_rows_select_a_column_exactly():
    rng = np.random.default_rng(3)
    w = rng.standard_normal((40, 96)).astype(np.float16)
    for j in (0, 5, 95):
        x = np.zeros(96, np.float32)
        x[j] = 1.0
        for sgemm in (False, True):
            assert np.array_equal(O.project(x, w.view(np.uint16), sgemm=sgemm)[0], w[:, j].astype(np.float32))


def test_rows_do_not_depend_on_batch_or_threads():
    rng = np.random.default_rng(4)
    w = rng.standard_normal((70, 1024)).astype(np.float16).view(np.uint16)
    x = rng.standard_normal((5, 1024)).astype(np.float32)
    for sgemm in (False, True):
        whole = O.project(x, w, sgemm=sgemm, threads=4)
        for b in range(5):
            assert np.array_equal(O.project(x[b], w, sgemm=sgemm)[0], whole[b])


def test_eight_lane_order_differs_from_a_sequential_sum():
    # the two paths are distinct restatements: on long rows they round differently somewhere
    rng = np.random.default_rng(5)
    w = rng.standard_normal((256, 1024)).astype(np.float16).view(np.uint16)
    x = rng.standard_normal((1, 1024)).astype(np.float32)
    assert not np.array_equal(O.project(x, w), O.project(x, w, sgemm=True))
