"""CPU tests of the C-ABI boundary: the library loads and exports what the headers declare.

No compute is launched here (no GPU in the build container)."""
import re
from pathlib import Path

import pytest

from fpga_qwen_b200 import qattn

ROOT = Path(__file__).resolve().parents[1]


def declared_functions():
    names = set()
    for header in sorted((ROOT / "include").glob("*.h")):
        text = re.sub(r"/\*.*?\*/", "", header.read_text(), flags=re.S)
        names.update(re.findall(r"\b(qa_\w+)\s*\(", text))
    return sorted(names)


def test_library_exports_every_declared_function():
    lib = qattn.lib()
    declared = declared_functions()
    assert len(declared) >= 20
    for name in declared:
        assert hasattr(lib, name), name
    assert set(declared) == set(qattn.EXPORTS)


def test_defaults_match_the_reference_model_shape():
    cfg = qattn.default_config()
    # engine/core.cpp:28 (D=128, Q=16, K=8, L=28), :237 (context <= 4096), :288 (theta 1e6), :213 (eps)
    assert (cfg.n_layers, cfg.n_q_heads, cfg.n_kv_heads, cfg.head_dim, cfg.context) == (28, 16, 8, 128, 4096)
    assert cfg.rope_theta == 1e6 and abs(cfg.norm_eps - 1e-6) < 1e-12
    assert cfg.kv_head_begin == 0 and cfg.kv_head_count == 0 and cfg.io_host == 0


def test_status_strings_and_version():
    lib = qattn.lib()
    assert lib.qa_status_string(0) == b"ok"
    assert lib.qa_status_string(2) == b"context capacity exceeded"
    assert b"sm_100a" in lib.qa_version()


def test_library_is_built_for_sm100a_only():
    """The build recipe targets sm_100a alone, and every kernel the compiler reported (the
    ptxas -v log of each source, written next to its object) was compiled for sm_100a."""
    from fpga_qwen_b200 import build
    gencodes = [build.NVCC_FLAGS[i + 1] for i, f in enumerate(build.NVCC_FLAGS) if f == "-gencode"]
    assert gencodes == ["arch=compute_100a,code=sm_100a"]
    logs = sorted(build.BUILD.glob("*.ptxas.txt"))
    if not logs:
        pytest.skip("library not built here")
    arches = set()
    for log in logs:
        arches |= set(re.findall(r"for 'sm_(\d+a?)'", log.read_text()))
    assert arches == {"100a"}, arches


def test_create_rejects_unsupported_shapes_before_touching_the_device():
    lib = qattn.lib()
    import ctypes
    for bad in (dict(head_dim=64), dict(n_q_heads=24), dict(context=4097), dict(context=0),
                dict(max_seqs=0), dict(kv_head_begin=7, kv_head_count=2)):
        cfg = qattn.default_config(**bad)
        h = ctypes.c_void_p()
        assert lib.qa_create(ctypes.byref(cfg), ctypes.byref(h)) in (qattn.QA_ERR_INVALID, qattn.QA_ERR_UNSUPPORTED)
        assert not h.value


def test_decode_loop_bench_builds(tmp_path):
    """bench.py builds the C++ decode-loop timing tool against the library on the GPU box; it
    must compile here too (no run: that needs a GPU)."""
    import shutil
    import subprocess
    if not shutil.which("g++") or not qattn.LIB_PATH.exists():
        pytest.skip("g++ or the library missing")
    root = qattn.LIB_PATH.parent.parent
    exe = tmp_path / "decode_loop_bench"
    res = subprocess.run(["g++", "-O2", "-std=c++17", f"-I{root / 'include'}",
                          str(root / "fpga_qwen_b200" / "host" / "decode_loop_bench.cpp"),
                          f"-L{qattn.LIB_PATH.parent}", "-lqattn", f"-Wl,-rpath,{qattn.LIB_PATH.parent}",
                          "-o", str(exe)], capture_output=True, text=True)
    assert res.returncode == 0, res.stderr[-2000:]
