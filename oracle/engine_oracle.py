"""CPU restatement of the reference engine's forward pass around attention.

TEST INFRASTRUCTURE ONLY: the checker of the host engine test (tests/test_engine.py). The
product library never imports it.

Model::Impl::chunk (tampajohn/fpga-qwen engine/core.cpp:353-646) for `batch` new tokens:
  x = embedding rows of the ids (:382-383)
  per layer: h = norm(x) (:385-386); q, k, v = projections of h (:387-394); per row and head
  norm + RoPE of q and k and the FP16 K/V store (:395-406); causal attention (:407-624);
  x += o_proj(attended) (:625-626); h = norm(x) (:627); gate, up = projections of h
  (:628-632); gate = gate * (0.5 + 0.5 tanh(gate/2)) * up (:636-639); x += down_proj(gate)
  (:640-641)
  pos += batch (:643); the last row's hidden state = norm(x_last, model.norm) (:645)
and Model::Impl::append's logits = embedding matrix . last hidden (:713); the B2
verify_chunk (:647-706) is the same per row for two rows, with both rows' logits.
Projections of one row use the eight-lane dot (project / project_group, :292-320); batched
rows over a layer matrix use cblas_sgemm (:294), restated as an FP32 sum in column order; the
FP16-only embedding matrix always uses the eight-lane dot. The pieces are the oracle's own
restatements (oracle.py): norm, project, append, attention, mlp_gate.
"""
from __future__ import annotations

import numpy as np

from . import oracle as O

Q_HEADS, KV_HEADS, D = 16, 8, 128


class EngineOracle:
    """weights: name -> float32 array (matrices already rounded to FP16 values), as NumpyQwen
    reads them with weight_precision='f16'."""

    def __init__(self, weights, layers=28, context=256, threads=4):
        self.w = weights
        self.layers, self.context, self.threads = layers, context, threads
        self.f16 = {k: v.astype(np.float16).view(np.uint16) for k, v in weights.items() if v.ndim == 2}
        self.kv = [O.LayerKV(KV_HEADS, context) for _ in range(layers)]
        self.tables = O.rope_tables(context)
        self.pos = 0

    def _w(self, layer, suffix):
        return self.w[f"model.layers.{layer}.{suffix}.weight"]

    def _m(self, layer, suffix):
        return self.f16[f"model.layers.{layer}.{suffix}.weight"]

    def _project(self, name16, x, batched):
        return O.project(x, name16, sgemm=batched, threads=self.threads)

    def chunk(self, ids, verify=False):
        """Runs len(ids) new tokens at the current position; returns the logits of the last
        row (or of both rows with verify=True). verify leaves the position unchanged."""
        ids = list(ids)
        n = len(ids)
        batched = n > 1 and not verify          # verification keeps the one-row dot (:182-206)
        x = self.f16["model.embed_tokens.weight"][ids].view(np.float16).astype(np.float32)
        for layer in range(self.layers):
            h = O.norm(x, self._w(layer, "input_layernorm"))
            q = self._project(self._m(layer, "self_attn.q_proj"), h, batched).reshape(n, Q_HEADS, D)
            k = self._project(self._m(layer, "self_attn.k_proj"), h, batched).reshape(n, KV_HEADS, D)
            v = self._project(self._m(layer, "self_attn.v_proj"), h, batched).reshape(n, KV_HEADS, D)
            qn = O.append(self.kv[layer], self.pos, q, k, v, self._w(layer, "self_attn.q_norm"),
                          self._w(layer, "self_attn.k_norm"), self.tables)
            att = O.attention(self.kv[layer], self.pos, qn, threads=self.threads).reshape(n, -1)
            x = x + self._project(self._m(layer, "self_attn.o_proj"), att, batched)
            h = O.norm(x, self._w(layer, "post_attention_layernorm"))
            gate = self._project(self._m(layer, "mlp.gate_proj"), h, batched)
            up = self._project(self._m(layer, "mlp.up_proj"), h, batched)
            x = x + self._project(self._m(layer, "mlp.down_proj"), O.mlp_gate(gate, up), batched)
        rows = x if verify else x[-1:]
        hidden = O.norm(rows, self.w["model.norm.weight"])
        logits = O.project(hidden, self.f16["model.embed_tokens.weight"], threads=self.threads)
        if not verify:
            self.pos += n
        return logits

    def commit(self, count):
        """Model::commit_verified: the first `count` verified rows join the history (:745-750)."""
        self.pos += count

    def truncate(self, pos):
        self.pos = pos
