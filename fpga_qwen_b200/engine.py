"""Host-side mirror of the reference's model API, restricted to the attention/KV path.

``AttentionModel`` keeps the state machine of tampajohn/fpga-qwen ``qwen_cpu::Model``
(engine/core.hpp:25-56, engine/core.cpp:707-752) for one sequence slot of a
:class:`~fpga_qwen_b200.qattn.Context`:

* ``prefill`` / ``step`` append rows and return attention outputs (core.cpp:707-714,
  727-728); prefill walks 512-row chunks like ``Impl::append`` (core.cpp:712);
* ``verify_two`` evaluates two rows without advancing the position, and blocks further
  inference until ``commit_verified``, ``reset`` or ``truncate`` (core.cpp:729-752,
  core.hpp:38-45);
* ``truncate`` / ``reset`` are O(1) logical operations (core.cpp:718-726);
* a validation failure leaves state unchanged; an execution failure resets the sequence
  (core.hpp:41).

Instead of token IDs it takes the attention inputs directly — pre-norm ``q [L][n][hq][128]``,
``k, v [L][n][hkv][128]`` FP32 CUDA tensors — because projections are outside this path.
"""
from __future__ import annotations

import torch

from .qattn import Context, PREFIX_CHUNK, QAttnError, QA_ERR_STATE, QA_ERR_CAPACITY, QA_ERR_INVALID


class AttentionModel:
    def __init__(self, ctx: Context, seq: int = 0):
        self.ctx, self.seq = ctx, seq
        self.verification_pending = False
        self.layers = ctx.config.n_layers

    # -- state -------------------------------------------------------------------------------
    @property
    def position(self) -> int:
        return self.ctx.position(self.seq)

    def reset(self):
        self.ctx.reset(self.seq)
        self.verification_pending = False

    def truncate(self, position: int):
        self.ctx.truncate(self.seq, position)
        self.verification_pending = False

    # -- inference ---------------------------------------------------------------------------
    def _check_inputs(self, q, k, v):
        for name, t, heads in (("q", q, self.ctx.hq), ("k", k, self.ctx.hkv), ("v", v, self.ctx.hkv)):
            if not (isinstance(t, torch.Tensor) and t.is_cuda and t.dtype == torch.float32 and t.is_contiguous()):
                raise QAttnError(QA_ERR_INVALID, f"{name} must be a contiguous float32 CUDA tensor")
            if t.dim() != 4 or t.shape[0] != self.layers or t.shape[2] != heads or t.shape[3] != 128:
                raise QAttnError(QA_ERR_INVALID, f"{name} has shape {tuple(t.shape)}")
        if not (q.shape[1] == k.shape[1] == v.shape[1]) or q.shape[1] < 1:
            raise QAttnError(QA_ERR_INVALID, "Empty token input")

    def _run(self, q, k, v, decode: bool, commit: bool):
        n = q.shape[1]
        pos = self.position
        self.ctx.set_stream(torch.cuda.current_stream(q.device).cuda_stream)
        qn = torch.empty_like(q)
        out = torch.empty_like(q)
        try:
            for b0 in range(0, n, PREFIX_CHUNK):
                b1 = min(n, b0 + PREFIX_CHUNK)
                rows = b1 - b0
                for layer in range(self.layers):
                    self.ctx.append(self.seq, layer, 1, pos + b0, rows, q[layer, b0:b1].data_ptr(),
                                    k[layer, b0:b1].data_ptr(), v[layer, b0:b1].data_ptr(),
                                    qn[layer, b0:b1].data_ptr())
                    fn = self.ctx.attn_decode if decode else self.ctx.attn_prefill
                    fn(self.seq, layer, 1, pos + b0, rows, qn[layer, b0:b1].data_ptr(), out[layer, b0:b1].data_ptr())
                if commit:
                    self.ctx.commit(self.seq, rows)
        except QAttnError as e:
            if e.status not in (QA_ERR_INVALID, QA_ERR_CAPACITY, QA_ERR_STATE):
                self.reset()
            raise
        return out

    def prefill(self, q, k, v):
        if self.verification_pending:
            raise QAttnError(QA_ERR_STATE, "Commit or discard pending verification before inference")
        self._check_inputs(q, k, v)
        if q.shape[1] > self.ctx.config.context - self.position:
            raise QAttnError(QA_ERR_CAPACITY, "Context capacity exceeded")
        return self._run(q, k, v, decode=q.shape[1] <= 1, commit=True)

    def step(self, q, k, v):
        self._check_inputs(q, k, v)
        if q.shape[1] != 1:
            raise QAttnError(QA_ERR_INVALID, "step takes one row")
        return self.prefill(q, k, v)

    def verify_two(self, q, k, v):
        if self.verification_pending:
            raise QAttnError(QA_ERR_STATE, "Verification already pending")
        self._check_inputs(q, k, v)
        if q.shape[1] != 2:
            raise QAttnError(QA_ERR_INVALID, "verify_two takes two rows")
        if self.position > self.ctx.config.context - 2:
            raise QAttnError(QA_ERR_CAPACITY, "Context capacity exceeded")
        out = self._run(q, k, v, decode=True, commit=False)
        self.verification_pending = True
        return out

    def commit_verified(self, count: int):
        if not self.verification_pending:
            raise QAttnError(QA_ERR_STATE, "No verification pending")
        if count not in (1, 2):
            raise QAttnError(QA_ERR_INVALID, "Commit count must be one or two")
        self.ctx.commit(self.seq, count)
        self.verification_pending = False
