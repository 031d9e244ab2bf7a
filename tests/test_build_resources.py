"""Compile-time resources of the CUDA kernels (ptxas reports written by fpga_qwen_b200.build).

The launches rely on them: the tensor-core prefill moves registers between warpgroups with
setmaxnreg and refuses to launch unless it was built with exactly 168 registers per thread;
the decode kernels run two 128-thread CTAs per SM (65,536 registers / 256 threads: at most 255
per thread, the architectural limit) and the FP32 head-rows kernel one 512-thread CTA (at most
128); and no kernel may spill to local memory.
"""
import re

import pytest

from fpga_qwen_b200 import build


def kernels():
    build.build()
    out = {}
    for log in sorted(build.BUILD.glob("*.ptxas.txt")):
        entry, spills = None, None
        for line in log.read_text().splitlines():
            m = re.search(r"Compiling entry function '([^']+)'", line)
            if m:
                entry = m.group(1)
                continue
            m = re.search(r"(\d+) bytes spill stores, (\d+) bytes spill loads", line)
            if m and entry:
                spills = int(m.group(1)) + int(m.group(2))
            m = re.search(r"Used (\d+) registers", line)
            if m and entry:
                out[entry] = (int(m.group(1)), spills)
                entry = None
    return out


@pytest.fixture(scope="module")
def resources():
    res = kernels()
    assert res, "no ptxas reports found"
    return res


def _pick(resources, name):
    found = {k: v for k, v in resources.items() if name in k}
    assert found, name
    return found


def test_no_kernel_spills(resources):
    assert {k: v for k, v in resources.items() if v[1]} == {}


def test_prefill_register_split_is_consistent(resources):
    found = _pick(resources, "attn_prefill_sm100_kernel")
    assert len(found) == 3                          # single-GPU, key-segment split and peer-store instantiations
    assert all(regs == 168 for regs, _ in found.values()), found


@pytest.mark.parametrize("name,budget", [("attn_decode_sm100_kernel", 255), ("attn_head_rows_kernel", 128)])
def test_occupancy_register_budgets(resources, name, budget):
    found = _pick(resources, name)
    assert all(regs <= budget for regs, _ in found.values()), found
