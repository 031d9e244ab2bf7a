"""CPU tests of the oracle: pinned against the reference's own NumPy oracle and known answers.

The fixture ``tests/golden/numpyqwen_t40.npz`` was produced by running tampajohn/fpga-qwen's
``NumpyQwen`` (tests/test_full_model.py:14-80) unchanged; see ``tests/golden/make_golden.py``.
"""
import numpy as np
import pytest

from oracle import numpy_oracle as N
from oracle import oracle as O

T = 40


@pytest.fixture(scope="module")
def tables():
    return O.rope_tables(4096)


def _oracle_layer(golden, layer, tables):
    kv = O.LayerKV(8, 64)
    q = O.append(kv, 0, golden[f"L{layer}_q_pre"], golden[f"L{layer}_k_pre"], golden[f"L{layer}_v_pre"],
                 golden[f"L{layer}_q_norm"], golden[f"L{layer}_k_norm"], tables)
    return kv, q


def _as_tokens(plane):
    return plane[:, :T].view(np.float16).astype(np.float32).transpose(1, 0, 2)


def test_rope_tables_bit_exact_with_reference_formula(tables):
    # core.cpp:287-288 and test_full_model.py:46 compute the same FP64 angle, cos/sin -> FP32.
    c, s = N.rope_tables(4096)
    assert np.array_equal(tables[0], c) and np.array_equal(tables[1], s)


def test_fp16_rounding_matches_numpy_rne():
    rng = np.random.default_rng(3)
    special = np.array([0.0, -0.0, 1.0, 65504.0, 65519.0, 65520.0, 1e9, -1e9, np.inf, -np.inf,
                        2.0 ** -24, 2.0 ** -25, 3 * 2.0 ** -26, 2.0 ** -14, 2.0 ** -15 + 2.0 ** -26,
                        1 + 2.0 ** -11, 1 + 3 * 2.0 ** -11, 6.1e-5, 5.96e-8], np.float32)
    x = np.concatenate([special, rng.standard_normal(100000).astype(np.float32) * 4,
                        (rng.standard_normal(20000) * 1e-5).astype(np.float32),
                        rng.uniform(-70000, 70000, 20000).astype(np.float32)])
    assert np.array_equal(O.f32_to_f16_bits(x), x.astype(np.float16).view(np.uint16))


def test_v_rows_bit_exact_with_reference_oracle(golden, tables):
    for layer in golden["layers"]:
        kv, _ = _oracle_layer(golden, layer, tables)
        assert np.array_equal(_as_tokens(kv.v), golden[f"L{layer}_v16"])


def test_k_rows_within_one_fp16_ulp_of_reference_oracle(golden, tables):
    # The NumPy oracle normalises with an FP32 mean and a division (test_full_model.py:44-45);
    # the C++ engine sums squares in FP64 and multiplies by a reciprocal (core.cpp:207-215).
    # The two agree to a few FP32 ulp, which can move an FP16 rounding by one step.
    for layer in golden["layers"]:
        kv, _ = _oracle_layer(golden, layer, tables)
        mine = kv.k[:, :T].transpose(1, 0, 2).astype(np.int32)
        ref = golden[f"L{layer}_k16"].astype(np.float16).view(np.uint16).astype(np.int32)
        diff = np.abs(mine - ref)
        assert diff.max() <= 1
        assert (diff != 0).mean() < 1e-3


def test_rotated_query_matches_reference_oracle(golden, tables):
    for layer in golden["layers"]:
        _, q = _oracle_layer(golden, layer, tables)
        ref = golden[f"L{layer}_q_rot"]
        assert np.abs(q - ref).max() <= 4e-6 * max(1.0, np.abs(ref).max())


def test_attention_on_identical_inputs_matches_reference_oracle(golden):
    for layer in golden["layers"]:
        kv = O.LayerKV(8, 64)
        kv.k[:, :T] = golden[f"L{layer}_k16"].astype(np.float16).view(np.uint16).transpose(1, 0, 2)
        kv.v[:, :T] = golden[f"L{layer}_v16"].astype(np.float16).view(np.uint16).transpose(1, 0, 2)
        out = O.attention(kv, 0, golden[f"L{layer}_q_rot"], threads=2)
        assert np.abs(out - golden[f"L{layer}_out"]).max() < 5e-6
        # the NumPy restatement reproduces the reference oracle bit for bit
        nout = N.attention(golden[f"L{layer}_q_rot"], golden[f"L{layer}_k16"], golden[f"L{layer}_v16"], 0)
        assert np.array_equal(nout, golden[f"L{layer}_out"])


def test_full_append_then_attention_tracks_reference_oracle(golden, tables):
    for layer in golden["layers"]:
        kv, q = _oracle_layer(golden, layer, tables)
        out = O.attention(kv, 0, q, threads=3)
        assert np.abs(out - golden[f"L{layer}_out"]).max() < 1e-3


def test_batched_rows_equal_single_token_steps_bitwise(golden, tables):
    # core.cpp:128-130/148-149/548-550: batched prefill keeps each output's arithmetic.
    kv, q = _oracle_layer(golden, 0, tables)
    batched = O.attention(kv, 0, q, threads=4)
    steps = np.concatenate([O.attention(kv, t, q[t:t + 1], threads=5) for t in range(T)])
    assert np.array_equal(batched, steps)


@pytest.mark.parametrize("threads", [1, 2, 3, 6, 12])
def test_thread_count_invariance(golden, tables, threads):
    kv, q = _oracle_layer(golden, 27, tables)
    base = O.attention(kv, 0, q, threads=1)
    assert np.array_equal(base, O.attention(kv, 0, q, threads=threads))


def test_known_answers(tables):
    rng = np.random.default_rng(0)
    # RoPE at position 0 is the identity.
    x = rng.standard_normal(128).astype(np.float32)
    y = x.copy()
    O.lib().qo_rope(y, np.ascontiguousarray(tables[0][0]), np.ascontiguousarray(tables[1][0]))
    assert np.array_equal(x, y)
    # Norm of a constant vector with unit weights is sign(c) (up to the 1e-6 epsilon).
    out = O.norm(np.full(128, 3.0, np.float32), np.ones(128, np.float32))
    assert np.allclose(out, 1.0, atol=1e-6)
    # n = 1: the only probability is exactly 1, so the output is V_0 exactly.
    kv = O.LayerKV(8, 16)
    kv.v[:] = rng.standard_normal(kv.v.shape).astype(np.float16).view(np.uint16)
    kv.k[:] = rng.standard_normal(kv.k.shape).astype(np.float16).view(np.uint16)
    q = rng.standard_normal((1, 16, 128)).astype(np.float32)
    out = O.attention(kv, 0, q)
    for h in range(16):
        assert np.array_equal(out[0, h], kv.v[h // 2, 0].view(np.float16).astype(np.float32))
    # Identical keys: uniform probabilities, output is the mean of the values.
    kv.k[:] = kv.k[:, :1]
    out = O.attention(kv, 7, rng.standard_normal((1, 16, 128)).astype(np.float32))
    mean = kv.v[:, :8].view(np.float16).astype(np.float64).mean(axis=1)
    for h in range(16):
        assert np.allclose(out[0, h], mean[h // 2], atol=2e-6)


# ---- the 200-token fixture: rows at positions >= 128 (the library's tensor-core rows) ----------
def _oracle_layer200(g, layer, tables):
    kv = O.LayerKV(8, 256)
    q = O.append(kv, 0, g[f"L{layer}_q_pre"], g[f"L{layer}_k_pre"], g[f"L{layer}_v_pre"],
                 g[f"L{layer}_q_norm"], g[f"L{layer}_k_norm"], tables)
    return kv, q


def test_long_fixture_kv_rows_match_reference_oracle(golden200, tables):
    T = golden200[f"L27_q_pre"].shape[0]
    for layer in golden200["layers"]:
        kv, _ = _oracle_layer200(golden200, layer, tables)
        v_ref = golden200[f"L{layer}_v16"].astype(np.float16).view(np.uint16)
        assert np.array_equal(kv.v[:, :T].transpose(1, 0, 2), v_ref)
        # Within one FP16 ulp, as for the 40-token fixture, except where RoPE cancels to a small
        # value: there the few-FP32-ulp difference of the two norms is a larger share of the
        # result, and the bound is absolute (2.5e-7, two FP16 ulps at 1.2e-4).
        mine = kv.k[:, :T].transpose(1, 0, 2)
        k_ref = golden200[f"L{layer}_k16"].astype(np.float16)
        diff = np.abs(mine.astype(np.int32) - k_ref.view(np.uint16).astype(np.int32))
        absdiff = np.abs(mine.view(np.float16).astype(np.float64) - k_ref.astype(np.float64))
        assert ((diff <= 1) | (absdiff <= 2.5e-7)).all()
        assert (diff != 0).mean() < 1e-3


def test_long_fixture_attention_past_row_128_matches_reference_oracle(golden200, tables):
    rows = golden200["rows"]
    T = int(rows[-1]) + 1
    for layer in golden200["layers"]:
        # identical inputs: the reference oracle's FP16 K/V and rotated query
        kv = O.LayerKV(8, 256)
        kv.k[:, :T] = golden200[f"L{layer}_k16"].astype(np.float16).view(np.uint16).transpose(1, 0, 2)
        kv.v[:, :T] = golden200[f"L{layer}_v16"].astype(np.float16).view(np.uint16).transpose(1, 0, 2)
        out = O.attention(kv, int(rows[0]), golden200[f"L{layer}_q_rot"], threads=4)
        assert np.abs(out - golden200[f"L{layer}_out"]).max() < 5e-6
        # the whole path from the pre-norm inputs
        kv2, q = _oracle_layer200(golden200, layer, tables)
        assert np.abs(q[rows] - golden200[f"L{layer}_q_rot"]).max() <= 4e-6 * max(1.0, np.abs(q).max())
        out2 = O.attention(kv2, int(rows[0]), q[rows], threads=4)
        assert np.abs(out2 - golden200[f"L{layer}_out"]).max() < 1e-3
