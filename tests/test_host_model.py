"""The C++ host mirror of qwen_cpu::Model (fpga_qwen_b200/host/attention_model.hpp).

CPU: the header compiles against include/qattn.h, links libqattn.so, and turns a failed
qa_create into std::runtime_error. GPU: a C++ run with host buffers (prefill, steps,
verify_two / commit_verified, truncate, and the reference's refusals) gives the same outputs,
bit for bit, as the same calls through the library's device-pointer API, and the same
positions and messages as engine/core.cpp:707-752.
"""
import shutil
import subprocess
from pathlib import Path

import numpy as np
import pytest
import torch

ROOT = Path(__file__).resolve().parents[1]
L, HQ, HKV, D = 4, 16, 8, 128


def build(tmp: Path) -> Path:
    if shutil.which("g++") is None:
        pytest.skip("g++ not available")
    lib = ROOT / "fpga_qwen_b200" / "libqattn.so"
    if not lib.exists():
        pytest.fail("libqattn.so is not built")
    exe = tmp / "host_model_main"
    subprocess.run(["g++", "-std=c++17", "-O1", "-Wall", "-Werror", f"-I{ROOT / 'include'}",
                    f"-I{ROOT / 'fpga_qwen_b200' / 'host'}", str(ROOT / "tests" / "host_model_main.cpp"),
                    f"-L{lib.parent}", "-lqattn", f"-Wl,-rpath,{lib.parent}", "-o", str(exe)],
                   check=True, capture_output=True, text=True)
    return exe


def test_header_builds_and_reports_create_failure(tmp_path):
    if torch.cuda.is_available():
        pytest.skip("a GPU is present: the no-device error path is not reachable")
    exe = build(tmp_path)
    res = subprocess.run([str(exe), "nogpu"], capture_output=True, text=True, timeout=60)
    assert res.returncode == 0, res.stdout + res.stderr
    assert res.stdout.startswith("caught: qa_create:"), res.stdout


def _parse(path: Path):
    a = np.fromfile(path, dtype=np.float32)
    off = 0

    def take(*shape):
        nonlocal off
        n = int(np.prod(shape))
        x = a[off:off + n].reshape(shape)
        off += n
        return x

    norms = [(take(D).copy(), take(D).copy()) for _ in range(L)]

    def call(n):
        return take(L, n, HQ, D), take(L, n, HKV, D), take(L, n, HKV, D), take(L, n, HQ, D)

    calls = {"prefill": call(85), "steps": [call(1) for _ in range(3)], "verify": call(2), "last": call(1)}
    assert off == a.size
    return norms, calls


@pytest.mark.gpu
def test_host_model_matches_library(tmp_path):
    from fpga_qwen_b200 import qattn

    exe = build(tmp_path)
    out_file = tmp_path / "run.bin"
    res = subprocess.run([str(exe), "gpu", str(out_file)], capture_output=True, text=True, timeout=300)
    assert res.returncode == 0, res.stdout + res.stderr
    lines = dict(line.split(" ", 1) for line in res.stdout.strip().splitlines())
    assert lines["base"].split() == ["88", "pending_pos", "88", "commit_pos", "89", "final_pos", "51"]
    assert lines["pending_msg"] == "Commit or discard pending verification before inference"
    assert lines["rewind_msg"] == "Rewind position out of range"

    norms, calls = _parse(out_file)
    ctx = qattn.Context(n_layers=L, context=512, max_seqs=1)
    ctx.set_stream(torch.cuda.current_stream().cuda_stream)
    for layer, (qw, kw) in enumerate(norms):
        ctx.set_norms(layer, qw.ctypes.data, kw.ctypes.data)
    keep = []

    def dev(x):
        t = torch.from_numpy(np.ascontiguousarray(x)).cuda()
        keep.append(t)
        return t

    q, k, v, want = (dev(x) for x in calls["prefill"])
    qn, out = torch.empty_like(q), torch.empty_like(q)
    ctx.append(0, 0, L, 0, 85, q.data_ptr(), k.data_ptr(), v.data_ptr(), qn.data_ptr())
    ctx.attn_prefill(0, 0, L, 0, 85, qn.data_ptr(), out.data_ptr())
    ctx.commit(0, 85)
    assert torch.equal(out, want)
    for s, rows in enumerate(calls["steps"]):
        q, k, v, want = (dev(x) for x in rows)
        out = torch.empty_like(q)
        ctx.decode_step(0, 0, L, 85 + s, q.data_ptr(), k.data_ptr(), v.data_ptr(), 0, out.data_ptr())
        ctx.commit(0, 1)
        assert torch.equal(out, want), s
    q, k, v, want = (dev(x) for x in calls["verify"])
    qn, out = torch.empty_like(q), torch.empty_like(q)
    ctx.append(0, 0, L, 88, 2, q.data_ptr(), k.data_ptr(), v.data_ptr(), qn.data_ptr())
    ctx.attn_decode(0, 0, L, 88, 2, qn.data_ptr(), out.data_ptr())
    assert torch.equal(out, want)
    ctx.commit(0, 1)
    ctx.truncate(0, 50)
    q, k, v, want = (dev(x) for x in calls["last"])
    out = torch.empty_like(q)
    ctx.decode_step(0, 0, L, 50, q.data_ptr(), k.data_ptr(), v.data_ptr(), 0, out.data_ptr())
    ctx.commit(0, 1)
    torch.cuda.synchronize()
    assert torch.equal(out, want)
    assert ctx.position(0) == 51
    ctx.close()


@pytest.mark.gpu
def test_engine_loop_layer_by_layer(tmp_path):
    """The engine's own loop through the layer-by-layer form (begin_rows / layer_rows /
    end_rows), host buffers: each layer's q, k, v come from a residual that the previous
    layer's attention output updated (a stand-in for o_proj and the MLP), so the library must
    serve layer l before layer l+1's inputs exist. The recorded inputs follow from the
    recorded outputs exactly; every layer's outputs agree with the oracle replaying the same
    rows; positions and refusals follow engine/core.cpp (the position advances after the last
    layer; verification rows wait for commit_verified)."""
    from oracle import oracle as O
    from tests import helpers as H

    exe = build(tmp_path)
    out_file = tmp_path / "engine.bin"
    res = subprocess.run([str(exe), "engine", str(out_file)], capture_output=True, text=True, timeout=300)
    assert res.returncode == 0, res.stdout + res.stderr
    lines = dict(line.split(" ", 1) for line in res.stdout.strip().splitlines())
    assert lines["positions"].split() == ["85", "88", "1", "89"]
    assert lines["order_msg"] == "Layers must run in order"
    assert lines["open_msg"] == "A layer pass is already open"

    a = np.fromfile(out_file, dtype=np.float32)
    off = 0

    def take(*shape):
        nonlocal off
        n = int(np.prod(shape))
        x = a[off:off + n].reshape(shape)
        off += n
        return x

    norms = [(take(D).copy(), take(D).copy()) for _ in range(L)]
    passes = []                      # (pos0, n, [per layer (q, k, v, out)])
    pos = 0
    for n in (85, 1, 1, 1, 2):
        r = take(n, HQ * D).copy()
        layers = []
        for layer in range(L):
            q, k, v, out = take(n, HQ, D), take(n, HKV, D), take(n, HKV, D), take(n, HQ, D)
            # the stand-in projection of this layer's residual, in the same FP32 operations
            sa = np.float32(1.0) + np.float32(0.01) * np.float32(layer)
            sb = np.float32(0.001) * np.float32(layer)
            assert np.array_equal(q.reshape(n, -1), r * sa + sb)
            assert np.array_equal(k.reshape(n, -1), r[:, :HKV * D] * np.float32(0.9))
            assert np.array_equal(v.reshape(n, -1), r[:, HKV * D:] * np.float32(1.1))
            layers.append((q, k, v, out))
            r = r + np.float32(0.5) * out.reshape(n, -1)
        passes.append((pos, n, layers))
        pos += n
    assert off == a.size
    tables = O.rope_tables(512)
    for layer in range(L):
        kv = O.LayerKV(HKV, 512)
        for pos0, n, layers in passes:
            q, k, v, out = layers[layer]
            qn = O.append(kv, pos0, q, k, v, norms[layer][0], norms[layer][1], tables)
            H.check("engine loop layer by layer (host buffers)", out, O.attention(kv, pos0, qn, threads=4))
