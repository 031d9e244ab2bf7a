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
    import subprocess
    out = subprocess.run(["cuobjdump", "--list-elf", str(qattn.LIB_PATH)], capture_output=True, text=True)
    if out.returncode != 0:
        pytest.skip("cuobjdump unavailable")
    arches = set(re.findall(r"sm_(\d+a?)", out.stdout))
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
