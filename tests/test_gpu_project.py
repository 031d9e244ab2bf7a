"""GPU projections (qa_project / qa_project_group) against the oracle's eight-lane dot.

The reference computes every decode-time projection (one row), every verification projection
(two rows) and the FP16-only vocabulary head with its eight-lane dot (engine/core.cpp:119-147,
:182-206, :292-349, :705, :713); the library must reproduce it bit for bit. The oracle
restatement (oracle.project, sgemm=False) is pinned to the reference's NumpyQwen through
tests/golden/numpyqwen_proj_t3.npz (tests/test_oracle_projection.py).
"""
import os
from pathlib import Path

import numpy as np
import pytest
import torch

from fpga_qwen_b200 import qattn
from oracle import oracle as O

pytestmark = pytest.mark.gpu

THREADS = os.cpu_count() or 4
SHAPES = {"q": (2048, 1024), "k": (1024, 1024), "v": (1024, 1024), "o": (1024, 2048),
          "gate": (3072, 1024), "up": (3072, 1024), "down": (1024, 3072)}


def _ctx(**kw):
    ctx = qattn.Context(n_layers=1, context=256, **kw)
    if not kw.get("io_host"):
        ctx.set_stream(torch.cuda.current_stream().cuda_stream)
    return ctx


def _matrix(rng, rows, cols, scale=None):
    scale = scale or 1.0 / np.sqrt(cols)
    return (rng.standard_normal((rows, cols)) * scale).astype(np.float16).view(np.uint16)


def _gpu_project(ctx, w16, x, batch):
    w = torch.from_numpy(w16.view(np.int16)).cuda()
    xd = torch.from_numpy(np.ascontiguousarray(x, np.float32)).cuda()
    y = torch.full((batch, w16.shape[0]), float("nan"), device="cuda")
    ctx.project(w.data_ptr(), w16.shape[0], w16.shape[1], xd.data_ptr(), batch, y.data_ptr())
    torch.cuda.synchronize()
    ctx.sync()
    return y.cpu().numpy()


@pytest.mark.parametrize("name", list(SHAPES))
@pytest.mark.parametrize("batch", [1, 2])
def test_layer_projections_bit_exact(name, batch):
    rng = np.random.default_rng(10 * list(SHAPES).index(name) + batch)
    rows, cols = SHAPES[name]
    w = _matrix(rng, rows, cols)
    x = rng.standard_normal((batch, cols)).astype(np.float32)
    ctx = _ctx()
    got = _gpu_project(ctx, w, x, batch)
    assert np.array_equal(got, O.project(x, w, threads=THREADS)), name
    ctx.close()


def test_vocabulary_head_bit_exact():
    rng = np.random.default_rng(7)
    w = _matrix(rng, 151936, 1024, scale=0.05)
    x = rng.standard_normal((1, 1024)).astype(np.float32)
    ctx = _ctx()
    got = _gpu_project(ctx, w, x, 1)
    assert np.array_equal(got, O.project(x, w, threads=THREADS))
    ctx.close()


def test_group_ragged_shapes_and_batches_bit_exact():
    """q/k/v as one launch; rows that are not a multiple of the 16-row tile, a width that is not
    a multiple of the 128-column chunk, and batches that need several passes (the persistent
    kernel); at batch 1 and 2 the same shapes take the small-launch kernel, whose row slices
    cross matrix boundaries, and a 4096-column case whose slice is too large for it. The
    small-launch kernel gives each row 8, 4 or 2 threads by the rows a slice holds: q/k/v
    (28 rows per SM) takes 8, gate/up (42) takes 4 and a 10,000-row group (68) takes 2."""
    rng = np.random.default_rng(8)
    ctx = _ctx()
    for rows, cols, batch in (((2048, 1024, 1024), 1024, 1), ((2048, 1024, 1024), 1024, 2),
                              ((37, 5, 300), 776, 3), ((37, 5, 300), 776, 2), ((37, 5, 300), 776, 1),
                              ((16, 17), 8, 5), ((16, 17), 8, 1), ((3000, 3000), 4096, 2),
                              ((1,), 3072, 2), ((3072, 3072), 1024, 1), ((3072, 3072), 1024, 2),
                              ((5000, 5000), 520, 1), ((5000, 4999), 512, 2)):
        ws = [_matrix(rng, r, cols) for r in rows]
        x = rng.standard_normal((batch, cols)).astype(np.float32)
        wd = [torch.from_numpy(w.view(np.int16)).cuda() for w in ws]
        xd = torch.from_numpy(x).cuda()
        ys = [torch.full((batch, r), float("nan"), device="cuda") for r in rows]
        ctx.project_group([t.data_ptr() for t in wd], list(rows), cols, xd.data_ptr(), batch,
                          [t.data_ptr() for t in ys])
        torch.cuda.synchronize()
        for w, y in zip(ws, ys):
            assert np.array_equal(y.cpu().numpy(), O.project(x, w, threads=THREADS)), (rows, cols, batch)
    ctx.close()


def test_reference_fixture_through_the_gpu():
    """The matrices and inputs NumpyQwen recorded: the GPU equals the restatement bit for bit
    (and so lies within the restatement's pinned tolerance of the reference)."""
    fix = np.load(Path(__file__).parent / "golden" / "numpyqwen_proj_t3.npz")
    ctx = _ctx()
    for kind in ("q", "k", "v", "o", "gate", "up", "down"):
        x, w = fix[f"{kind}_in"], np.ascontiguousarray(fix[f"w_{kind}"])
        got = _gpu_project(ctx, w, x, x.shape[0])
        assert np.array_equal(got, O.project(x, w)), kind
    logits = _gpu_project(ctx, np.ascontiguousarray(fix["embed"]), fix["final_hidden"][None], 1)
    assert np.array_equal(logits, O.project(fix["final_hidden"][None], fix["embed"]))
    ctx.close()


def test_host_buffers_and_validation():
    rng = np.random.default_rng(9)
    rows, cols = 3072, 1024
    w = _matrix(rng, rows, cols)
    x = rng.standard_normal((2, cols)).astype(np.float32)
    wd = torch.from_numpy(w.view(np.int16)).cuda()
    host = _ctx(io_host=1)
    y = np.full((2, rows), np.nan, np.float32)
    host.project(wd.data_ptr(), rows, cols, x.ctypes.data, 2, y.ctypes.data)
    assert np.array_equal(y, O.project(x, w, threads=THREADS))
    with pytest.raises(qattn.QAttnError) as e:
        host.project(wd.data_ptr(), rows, 1020, x.ctypes.data, 1, y.ctypes.data)
    assert e.value.status == qattn.QA_ERR_INVALID
    with pytest.raises(qattn.QAttnError) as e:
        host.project(wd.data_ptr() + 2, rows, cols, x.ctypes.data, 1, y.ctypes.data)     # not 16-byte aligned
    assert e.value.status == qattn.QA_ERR_INVALID
    host.close()


def _gemm_check(got, x, ws):
    """Each matrix's batched product within FP32 accumulation rounding of the exact product: the
    split FP16 input keeps 22 bits, the sums run in FP32 (as sgemm's, in another order)."""
    for y, w in zip(got, ws):
        exact = x.astype(np.float64) @ w.view(np.float16).astype(np.float64).T
        scale = np.abs(x).astype(np.float64) @ np.abs(w.view(np.float16).astype(np.float64)).T
        err = np.abs(y.astype(np.float64) - exact)
        assert (err <= 1e-5 * scale + 1e-30).all(), (err / np.maximum(scale, 1e-30)).max()


@pytest.mark.parametrize("rows,cols,batch", [((2048, 1024, 1024), 1024, 512), ((3072, 3072), 1024, 129),
                                             ((1024,), 3072, 37), ((1024,), 2048, 600), ((37, 5, 300), 776, 3),
                                             ((3000,), 8200, 5)])
def test_gemm_batched_prompt_rows(rows, cols, batch):
    """qa_project_group_gemm (tensor cores; batches over one or several 512-row chunks, ragged
    rows, widths that are not a multiple of the 64-column K step, and a width beyond the tensor
    path's 8192 that runs on the CUDA cores) against the exact product, and against the CPU
    restatement of the reference's batched sgemm form."""
    rng = np.random.default_rng(sum(rows) + cols + batch)
    ws = [_matrix(rng, r, cols) for r in rows]
    x = rng.standard_normal((batch, cols)).astype(np.float32)
    ctx = _ctx()
    wd = [torch.from_numpy(w.view(np.int16)).cuda() for w in ws]
    xd = torch.from_numpy(x).cuda()
    ys = [torch.full((batch, r), float("nan"), device="cuda") for r in rows]
    ctx.project_group_gemm([t.data_ptr() for t in wd], list(rows), cols, xd.data_ptr(), batch, [t.data_ptr() for t in ys])
    torch.cuda.synchronize()
    ctx.sync()
    got = [y.cpu().numpy() for y in ys]
    _gemm_check(got, x, ws)
    if batch <= 129:
        for y, w in zip(got, ws):
            ref = O.project(x, w, sgemm=True, threads=THREADS)
            assert np.abs(y - ref).max() <= 1e-5 * max(1.0, float(np.abs(ref).max()))
    ctx.close()


def test_gemm_rows_of_extreme_magnitude_and_host_buffers():
    """Input rows scaled by 1e-20 and 1e20 keep full relative precision (each row is brought to a
    fixed range by an exact power of two before the FP16 split); a row of FP32 subnormals (whose
    power of two would overflow) stays finite; the host-buffer form gives the device form's
    results."""
    rng = np.random.default_rng(12)
    w = _matrix(rng, 1024, 1024)
    x = rng.standard_normal((40, 1024)).astype(np.float32)
    x[3] *= 1e-20
    x[7] *= 1e20
    x[11] = 0.0
    x[15] *= np.float32(1e-39)
    wd = torch.from_numpy(w.view(np.int16)).cuda()
    dev = _ctx()
    y = torch.empty((40, 1024), device="cuda")
    dev.project_gemm(wd.data_ptr(), 1024, 1024, torch.from_numpy(x).cuda().data_ptr(), 40, y.data_ptr())
    torch.cuda.synchronize()
    got = y.cpu().numpy()
    _gemm_check([got], x, [w])
    assert (got[11] == 0).all() and np.isfinite(got).all()
    host = _ctx(io_host=1)
    yh = np.full((40, 1024), np.nan, np.float32)
    host.project_gemm(wd.data_ptr(), 1024, 1024, x.ctypes.data, 40, yh.ctypes.data)
    assert np.array_equal(yh, got)
    dev.close(); host.close()
