"""Generate golden attention/KV fixtures by running the reference's own NumPy oracle.

Run where a checkout of tampajohn/fpga-qwen is available, with its directory in
``FPGA_QWEN_REF``::

    FPGA_QWEN_REF=<checkout> python tests/golden/make_golden.py                 # 40 tokens
    FPGA_QWEN_REF=<checkout> python tests/golden/make_golden.py --tokens 200    # 200 tokens
    FPGA_QWEN_REF=<checkout> python tests/golden/make_golden.py --projections   # projections
    FPGA_QWEN_REF=<checkout> python tests/golden/make_golden.py --engine        # engine logits

It imports ``NumpyQwen`` from the reference's ``tests/test_full_model.py`` (lines 14-80)
unchanged and runs ``NumpyQwen.token`` on a synthetic checkpoint written in the
safetensors layout its constructor reads (:20-34): BF16 tensors, the real 28 layers,
16 query heads, 8 KV heads and head_dim 128, with a small hidden size (64), MLP width (8)
and vocabulary (16), since only the attention inputs matter here and no Qwen3-0.6B
checkpoint is available. ``kv_precision='f16'`` selects the FP16 current-K/V rounding of
:60-63.

While it runs, two probes record what the reference computes:

* an ``ndarray`` subclass on the q/k/v projection weights records each projection
  result, i.e. the pre-norm q ``[16,128]`` and k, v ``[8,128]`` of every (token, layer);
* a wrapper on ``np.einsum`` records the normed+roped query (first operand of the
  ``'hd,thd->ht'`` call) and the attention output (result of ``'ht,thd->hd'``).

The FP16 K/V rows come from the oracle's own cache payload. The recorded arrays for a few
layers are written to ``tests/golden/numpyqwen_t{T}.npz``; the tests feed the pre-norm
inputs to the C++ restatement and to the CUDA library and compare.

``--tokens 200`` writes ``numpyqwen_t200.npz``: layer 27 only, with the rotated query and the
attention output kept for rows 96..199 (key ``rows``), so that the rows at positions >= 128,
which the library computes on the tensor cores, and the 127/128/129 boundary are pinned to the
reference; the FP16 K/V rows are stored as float16. The pre-norm inputs cover every row.
"""
from __future__ import annotations

import json
import os
import struct
import sys
import tempfile
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
TOKENS = 40                 # covers causal lengths 1..40, incl. the 31/32/33 edges
KEEP_LAYERS = (0, 27)       # layers written to the fixture
LONG_TOKENS, LONG_LAYERS, LONG_FIRST_ROW = 200, (27,), 96    # the --tokens 200 fixture
H, F, V = 64, 8, 16
SEED = 20261201


def bf16_bits(x: np.ndarray) -> np.ndarray:
    """float32 -> bfloat16 bits, round to nearest even."""
    u = x.astype(np.float32).view(np.uint32).astype(np.uint64)
    u = (u + 0x7FFF + ((u >> 16) & 1)) >> 16
    return u.astype(np.uint16)


def checkpoint_tensors(rng: np.random.Generator) -> dict:
    """The synthetic checkpoint's tensors (float64, before BF16 rounding), in writing order."""
    tensors = {}
    tensors["model.embed_tokens.weight"] = rng.standard_normal((V, H))
    tensors["model.norm.weight"] = np.ones(H)
    for layer in range(28):
        p = f"model.layers.{layer}."
        tensors[p + "input_layernorm.weight"] = np.ones(H)
        tensors[p + "post_attention_layernorm.weight"] = np.ones(H)
        tensors[p + "self_attn.q_norm.weight"] = rng.normal(1.0, 0.05, 128)
        tensors[p + "self_attn.k_norm.weight"] = rng.normal(1.0, 0.05, 128)
        # rows ~ N(0, 1/H) so that projections of the unit-RMS hidden state are ~N(0,1)
        tensors[p + "self_attn.q_proj.weight"] = rng.standard_normal((2048, H)) / np.sqrt(H)
        tensors[p + "self_attn.k_proj.weight"] = rng.standard_normal((1024, H)) / np.sqrt(H)
        tensors[p + "self_attn.v_proj.weight"] = rng.standard_normal((1024, H)) / np.sqrt(H)
        tensors[p + "self_attn.o_proj.weight"] = rng.standard_normal((H, 2048)) * 0.02
        tensors[p + "mlp.gate_proj.weight"] = rng.standard_normal((F, H)) * 0.1
        tensors[p + "mlp.up_proj.weight"] = rng.standard_normal((F, H)) * 0.1
        tensors[p + "mlp.down_proj.weight"] = rng.standard_normal((H, F)) * 0.1
    return tensors


def bf16_values(x: np.ndarray) -> np.ndarray:
    """float -> the float32 value of its BF16 rounding (what NumpyQwen reads from the file)."""
    return (bf16_bits(np.asarray(x, np.float32)).astype(np.uint32) << 16).view(np.float32)


def write_checkpoint(path: Path, rng: np.random.Generator) -> None:
    tensors = checkpoint_tensors(rng)
    header, blobs, offset = {}, [], 0
    for name, value in tensors.items():
        raw = bf16_bits(np.asarray(value, np.float32)).tobytes()
        header[name] = {"dtype": "BF16", "shape": list(np.shape(value)),
                        "data_offsets": [offset, offset + len(raw)]}
        blobs.append(raw)
        offset += len(raw)
    head = json.dumps(header).encode()
    head += b" " * (-len(head) % 8)
    with path.open("wb") as f:
        f.write(struct.pack("<Q", len(head)))
        f.write(head)
        for raw in blobs:
            f.write(raw)


def reference_dir() -> Path:
    ref = os.environ.get("FPGA_QWEN_REF")
    if not ref:
        raise SystemExit("set FPGA_QWEN_REF to a checkout of tampajohn/fpga-qwen")
    return Path(ref)


def main(tokens: int = TOKENS) -> None:
    sys.path.insert(0, str(reference_dir()))
    from tests.test_full_model import NumpyQwen  # the reference's oracle, unchanged

    long_form = tokens != TOKENS
    keep_layers = LONG_LAYERS if long_form else KEEP_LAYERS
    rows = np.arange(LONG_FIRST_ROW if long_form else 0, tokens)

    rng = np.random.default_rng(SEED)
    with tempfile.TemporaryDirectory() as tmp:
        model = Path(tmp)
        write_checkpoint(model / "model.safetensors", rng)
        oracle = NumpyQwen(model, weight_precision="bf16", kv_precision="f16")

    log = {}
    current = {"token": -1}

    class Recorded(np.ndarray):
        def __array_ufunc__(self, ufunc, method, *inputs, **kwargs):
            args = [np.asarray(a) if isinstance(a, Recorded) else a for a in inputs]
            out = getattr(ufunc, method)(*args, **kwargs)
            if ufunc is np.matmul:
                log[(current["token"], self.layer, self.kind)] = np.array(out, np.float32)
            return out

    for layer in range(28):
        for kind in ("q", "k", "v"):
            name = f"model.layers.{layer}.self_attn.{kind}_proj.weight"
            w = oracle.weights[name].view(Recorded)
            w.layer, w.kind = layer, kind
            oracle.weights[name] = w

    real_einsum = np.einsum
    einsum_layer = {"qk": 0, "pv": 0}

    def einsum(subscripts, *operands, **kwargs):
        out = real_einsum(subscripts, *operands, **kwargs)
        if subscripts == "hd,thd->ht":
            log[(current["token"], einsum_layer["qk"], "q_rot")] = np.array(operands[0], np.float32)
            einsum_layer["qk"] += 1
        elif subscripts == "ht,thd->hd":
            log[(current["token"], einsum_layer["pv"], "out")] = np.array(out, np.float32)
            einsum_layer["pv"] += 1
        return out

    np.einsum = einsum
    try:
        ids = rng.integers(0, V, tokens)
        for t, token in enumerate(ids):
            current["token"] = t
            einsum_layer["qk"] = einsum_layer["pv"] = 0
            oracle.token(int(token), logits=False)
    finally:
        np.einsum = real_einsum

    kv_type = np.float16 if long_form else np.float32
    arrays = {"layers": np.array(keep_layers, np.int32)}
    if long_form:
        arrays["rows"] = rows.astype(np.int32)
    for layer in keep_layers:
        p = f"model.layers.{layer}.self_attn."
        arrays[f"L{layer}_q_pre"] = np.stack([log[(t, layer, "q")].reshape(16, 128) for t in range(tokens)])
        arrays[f"L{layer}_k_pre"] = np.stack([log[(t, layer, "k")].reshape(8, 128) for t in range(tokens)])
        arrays[f"L{layer}_v_pre"] = np.stack([log[(t, layer, "v")].reshape(8, 128) for t in range(tokens)])
        arrays[f"L{layer}_q_rot"] = np.stack([log[(t, layer, "q_rot")] for t in rows])
        arrays[f"L{layer}_k16"] = np.stack([oracle.cache[t][layer][0] for t in range(tokens)]).astype(kv_type)
        arrays[f"L{layer}_v16"] = np.stack([oracle.cache[t][layer][1] for t in range(tokens)]).astype(kv_type)
        arrays[f"L{layer}_out"] = np.stack([log[(t, layer, "out")] for t in rows])
        arrays[f"L{layer}_q_norm"] = np.asarray(oracle.weights[p + "q_norm.weight"], np.float32)
        arrays[f"L{layer}_k_norm"] = np.asarray(oracle.weights[p + "k_norm.weight"], np.float32)
    out = HERE / f"numpyqwen_t{tokens}.npz"
    np.savez_compressed(out, **arrays)
    print(f"wrote {out} ({out.stat().st_size} bytes)")


PROJ_TOKENS = 3             # projection fixture: tokens, all recorded at layer 0
PROJ_SEED = 20261202


def projections() -> None:
    """Projection fixture (numpyqwen_proj_t3.npz) for the oracle's projection restatement.

    Runs NumpyQwen with ``weight_precision='f16'`` (matrices rounded to FP16 and widened, as
    the engine stores them) on a second synthetic checkpoint, and records at layer 0 the
    input and output of every matrix product (q/k/v/o, gate/up/down) per token, the MLP
    activation, and for the last token the final normalised hidden state and the logits.
    """
    sys.path.insert(0, str(reference_dir()))
    from tests.test_full_model import NumpyQwen  # the reference's oracle, unchanged

    rng = np.random.default_rng(PROJ_SEED)
    with tempfile.TemporaryDirectory() as tmp:
        model = Path(tmp)
        write_checkpoint(model / "model.safetensors", rng)
        oracle = NumpyQwen(model, weight_precision="f16", kv_precision="f16")

    log = {}
    current = {"token": -1}

    class Recorded(np.ndarray):
        def __array_ufunc__(self, ufunc, method, *inputs, **kwargs):
            args = [np.asarray(a) if isinstance(a, Recorded) else a for a in inputs]
            out = getattr(ufunc, method)(*args, **kwargs)
            if ufunc is np.matmul:
                log[(current["token"], self.kind, "in")] = np.array(args[1], np.float32)
                log[(current["token"], self.kind, "out")] = np.array(out, np.float32)
            elif ufunc is np.multiply and self.kind == "final_norm":
                log[(current["token"], "final_norm", "out")] = np.array(out, np.float32)
            return out

    kinds = {"self_attn.q_proj": "q", "self_attn.k_proj": "k", "self_attn.v_proj": "v",
             "self_attn.o_proj": "o", "mlp.gate_proj": "gate", "mlp.up_proj": "up", "mlp.down_proj": "down"}
    weights = {}
    for suffix, kind in kinds.items():
        name = f"model.layers.0.{suffix}.weight"
        weights[kind] = np.asarray(oracle.weights[name], np.float32)
        w = oracle.weights[name].view(Recorded)
        w.kind = kind
        oracle.weights[name] = w
    fn = oracle.weights["model.norm.weight"].view(Recorded)
    fn.kind = "final_norm"
    oracle.weights["model.norm.weight"] = fn

    ids = rng.integers(0, V, PROJ_TOKENS)
    logits = None
    for t, token in enumerate(ids):
        current["token"] = t
        logits = oracle.token(int(token), logits=(t == PROJ_TOKENS - 1))

    arrays = {}
    for kind, w in weights.items():
        arrays[f"w_{kind}"] = w.astype(np.float16).view(np.uint16)       # exact: already FP16 values
        arrays[f"{kind}_in"] = np.stack([log[(t, kind, "in")] for t in range(PROJ_TOKENS)])
        arrays[f"{kind}_out"] = np.stack([log[(t, kind, "out")] for t in range(PROJ_TOKENS)])
    arrays["embed"] = np.asarray(oracle.weights["model.embed_tokens.weight"], np.float32).astype(np.float16).view(np.uint16)
    arrays["final_hidden"] = log[(PROJ_TOKENS - 1, "final_norm", "out")]
    arrays["logits"] = np.asarray(logits, np.float32)
    out = HERE / f"numpyqwen_proj_t{PROJ_TOKENS}.npz"
    np.savez_compressed(out, **arrays)
    print(f"wrote {out} ({out.stat().st_size} bytes)")


ENGINE_SEED = 20261203
ENGINE_TOKENS = 13


def engine() -> None:
    """Engine fixture (numpyqwen_engine.npz): NumpyQwen with FP16 matrices and FP16 KV (the
    engine's precision, weight_precision='f16', kv_precision='f16') on a third synthetic
    checkpoint (seed ENGINE_SEED, regenerated by the test from checkpoint_tensors), fed
    ENGINE_TOKENS token ids one at a time; records the logits after every token. A host engine
    that prefills, decodes, verifies and rewinds over the same ids must reproduce the logits of
    each prefix."""
    sys.path.insert(0, str(reference_dir()))
    from tests.test_full_model import NumpyQwen  # the reference's oracle, unchanged

    rng = np.random.default_rng(ENGINE_SEED)
    with tempfile.TemporaryDirectory() as tmp:
        model = Path(tmp)
        write_checkpoint(model / "model.safetensors", rng)
        oracle = NumpyQwen(model, weight_precision="f16", kv_precision="f16")
    ids = rng.integers(0, V, ENGINE_TOKENS)
    logits = np.stack([np.asarray(oracle.token(int(t)), np.float32) for t in ids])
    out = HERE / "numpyqwen_engine.npz"
    np.savez_compressed(out, ids=ids.astype(np.int32), logits=logits)
    print(f"wrote {out} ({out.stat().st_size} bytes)")


if __name__ == "__main__":
    if "--engine" in sys.argv:
        engine()
    elif "--projections" in sys.argv:
        projections()
    elif "--tokens" in sys.argv:
        main(int(sys.argv[sys.argv.index("--tokens") + 1]))
    else:
        main()
