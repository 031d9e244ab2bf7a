"""The reference engine's forward pass with attention and projections on the GPU.

fpga_qwen_b200/host/qwen_forward.hpp is an x86 host build of Model::Impl's forward pass
(engine/core.cpp:353-714): the host keeps the engine's glue (embedding lookup, RMSNorm,
residual adds, MLP gate) and calls the library, layer by layer, for every projection and for
the attention of each layer, with the activations in host vectors as in the engine. It runs
prefill, decode steps, a B2 verification with commit_verified and a rewind over the token ids
of tests/golden/numpyqwen_engine.npz, whose logits the reference's own NumpyQwen produced on
the same synthetic checkpoint (28 layers, 16/8 heads x 128, hidden 64, FP16 matrices and KV).
The bar is the reference's own gate for full logits against NumpyQwen with a checkpoint
(max-abs 0.01, RMS 0.002) and the same top token.
"""
import shutil
import subprocess
from pathlib import Path

import numpy as np
import pytest

from tests.engine_weights import engine_weights

ROOT = Path(__file__).resolve().parents[1]
FIX = np.load(ROOT / "tests" / "golden" / "numpyqwen_engine.npz")
# (row of the fixture, its logits' source) in the order the scenario produces them
SCENARIO_ROWS = [7, 8, 9, 10, 11, 12, 8, 9]
MAX_ABS, RMS = 0.01, 0.002


def check_logits(got, rows):
    ref = FIX["logits"][rows]
    d = np.abs(np.asarray(got, np.float64) - ref)
    assert d.max() < MAX_ABS and np.sqrt((d * d).mean()) < RMS, (d.max(), np.sqrt((d * d).mean()))
    assert (np.argmax(got, axis=-1) == np.argmax(ref, axis=-1)).all()
    return d.max()


def oracle_scenario():
    from oracle.engine_oracle import EngineOracle
    w, *_ = engine_weights()
    ids = [int(t) for t in FIX["ids"]]
    e = EngineOracle(w, context=64)
    out = [e.chunk(ids[0:8]), e.chunk(ids[8:9]), e.chunk(ids[9:10])]
    out.append(e.chunk(ids[10:12], verify=True))
    e.commit(2)
    out.append(e.chunk(ids[12:13]))
    e.truncate(5)
    out += [e.chunk(ids[5:9]), e.chunk(ids[9:10])]
    return np.concatenate(out), e.pos


def test_engine_oracle_matches_numpyqwen():
    """The CPU restatement of the engine's forward pass (oracle/engine_oracle.py) against the
    reference's NumpyQwen: pins the glue the GPU engine test relies on."""
    got, pos = oracle_scenario()
    assert pos == 10
    check_logits(got, SCENARIO_ROWS)


def _write_inputs(tmp: Path):
    w, H, F, V = engine_weights()
    f16 = lambda a: np.ascontiguousarray(a, np.float32).astype(np.float16).tobytes()
    f32 = lambda a: np.ascontiguousarray(a, np.float32).tobytes()
    with open(tmp / "weights.bin", "wb") as f:
        f.write(np.array([28, H, F, V], np.int32).tobytes())
        f.write(f16(w["model.embed_tokens.weight"]))
        f.write(f32(w["model.norm.weight"]))
        for layer in range(28):
            p = f"model.layers.{layer}."
            for name in ("input_layernorm", "post_attention_layernorm", "self_attn.q_norm", "self_attn.k_norm"):
                f.write(f32(w[p + name + ".weight"]))
            for name in ("self_attn.q_proj", "self_attn.k_proj", "self_attn.v_proj", "self_attn.o_proj",
                         "mlp.gate_proj", "mlp.up_proj", "mlp.down_proj"):
                f.write(f16(w[p + name + ".weight"]))
    (tmp / "ids.bin").write_bytes(np.asarray(FIX["ids"], np.int32).tobytes())
    return V


@pytest.mark.gpu
def test_gpu_engine_forward_matches_numpyqwen(tmp_path):
    from tests import helpers as H
    if shutil.which("g++") is None:
        pytest.skip("g++ not available")
    lib = ROOT / "fpga_qwen_b200" / "libqattn.so"
    exe = tmp_path / "engine_main"
    subprocess.run(["g++", "-std=c++17", "-O1", "-Wall", "-Werror", f"-I{ROOT / 'include'}",
                    f"-I{ROOT / 'fpga_qwen_b200' / 'host'}", "-I/usr/local/cuda/include",
                    str(ROOT / "tests" / "engine_main.cpp"), f"-L{lib.parent}", "-lqattn", "-L/usr/local/cuda/lib64",
                    "-lcudart", f"-Wl,-rpath,{lib.parent}", "-o", str(exe)], check=True, capture_output=True, text=True)
    V = _write_inputs(tmp_path)
    res = subprocess.run([str(exe), str(tmp_path / "weights.bin"), str(tmp_path / "ids.bin"), str(tmp_path / "out.bin")],
                         capture_output=True, text=True, timeout=300)
    assert res.returncode == 0, res.stdout + res.stderr
    assert res.stdout.split() == ["position", "10"]
    got = np.fromfile(tmp_path / "out.bin", dtype=np.float32).reshape(-1, V)
    assert got.shape[0] == len(SCENARIO_ROWS)
    mx = check_logits(got, SCENARIO_ROWS)
    ref, _ = oracle_scenario()
    d = np.abs(got.astype(np.float64) - ref)
    H.record("engine forward logits vs NumpyQwen", mx, 0.0, len(SCENARIO_ROWS))
    assert d.max() < 0.01, d.max()


@pytest.mark.gpu
def test_gpu_engine_long_prompt_chunk_on_tensor_cores(tmp_path):
    """A 150-token prompt in one chunk: its projections run batched on the tensor cores
    (qa_project_gemm, where the reference uses cblas_sgemm, engine/core.cpp:294), then one
    decode step on the eight-lane GEMVs. Both rows' logits against the CPU restatement of the
    forward pass (which sums the batched products in FP32, as sgemm does) within the
    reference's full-logit gate, with the same top token."""
    from oracle.engine_oracle import EngineOracle
    from tests import helpers as H
    if shutil.which("g++") is None:
        pytest.skip("g++ not available")
    lib = ROOT / "fpga_qwen_b200" / "libqattn.so"
    exe = tmp_path / "engine_main"
    subprocess.run(["g++", "-std=c++17", "-O1", "-Wall", "-Werror", f"-I{ROOT / 'include'}",
                    f"-I{ROOT / 'fpga_qwen_b200' / 'host'}", "-I/usr/local/cuda/include",
                    str(ROOT / "tests" / "engine_main.cpp"), f"-L{lib.parent}", "-lqattn", "-L/usr/local/cuda/lib64",
                    "-lcudart", f"-Wl,-rpath,{lib.parent}", "-o", str(exe)], check=True, capture_output=True, text=True)
    V = _write_inputs(tmp_path)
    ids = np.random.default_rng(150).integers(0, V, 150).astype(np.int32)
    (tmp_path / "long_ids.bin").write_bytes(ids.tobytes())
    res = subprocess.run([str(exe), str(tmp_path / "weights.bin"), str(tmp_path / "long_ids.bin"),
                          str(tmp_path / "long_out.bin"), "long"], capture_output=True, text=True, timeout=300)
    assert res.returncode == 0, res.stdout + res.stderr
    assert res.stdout.split() == ["position", "150"]
    got = np.fromfile(tmp_path / "long_out.bin", dtype=np.float32).reshape(2, V)
    w, *_ = engine_weights()
    e = EngineOracle(w, context=256)
    ref = np.concatenate([e.chunk([int(t) for t in ids[:-1]]), e.chunk([int(ids[-1])])]).astype(np.float64)
    d = np.abs(got.astype(np.float64) - ref)
    H.record("engine 150-token prompt (tensor-core projections)", float(d.max()), float(np.sqrt((d * d).mean())), 2)
    assert d.max() < MAX_ABS and np.sqrt((d * d).mean()) < RMS, (d.max(), np.sqrt((d * d).mean()))
    assert (np.argmax(got, axis=-1) == np.argmax(ref, axis=-1)).all()
