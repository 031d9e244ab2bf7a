"""ctypes binding of libqattn.so (the C ABI in include/qattn.h).

This is a thin, 1:1 binding: every function returns the C status and raises ``QAttnError``
with ``qa_last_error`` on failure. Tensor arguments are raw addresses (``int``): device
addresses for contexts created with ``io_host=0`` (e.g. ``torch.Tensor.data_ptr()``), host
addresses for ``io_host=1`` (e.g. ``numpy.ndarray.ctypes.data``).

The library must exist: there is no fallback. Build it with ``python -m fpga_qwen_b200.build``.
"""
from __future__ import annotations

import ctypes
import os
from pathlib import Path

LIB_PATH = Path(__file__).resolve().parent / "libqattn.so"

QA_OK = 0
STATUS = {1: "invalid argument", 2: "context capacity exceeded", 3: "invalid state", 4: "CUDA error",
          5: "NCCL error", 6: "device wait timed out", 7: "out of device memory", 8: "unsupported"}
QA_ERR_INVALID, QA_ERR_CAPACITY, QA_ERR_STATE, QA_ERR_CUDA = 1, 2, 3, 4
QA_ERR_NCCL, QA_ERR_TIMEOUT, QA_ERR_OOM, QA_ERR_UNSUPPORTED = 5, 6, 7, 8
PREFIX_CHUNK = 512
MAX_DECODE_ROWS = 4
MAX_BATCH = 64
HEAD_DIM = 128


class QAttnError(RuntimeError):
    """A non-zero status from the C ABI (the C++ engine maps these to std::runtime_error)."""

    def __init__(self, status: int, message: str):
        super().__init__(f"{STATUS.get(status, 'error')} ({status}): {message}")
        self.status = status


class Config(ctypes.Structure):
    _fields_ = [("n_layers", ctypes.c_int), ("n_q_heads", ctypes.c_int), ("n_kv_heads", ctypes.c_int),
                ("head_dim", ctypes.c_int), ("context", ctypes.c_int), ("max_seqs", ctypes.c_int),
                ("kv_head_begin", ctypes.c_int), ("kv_head_count", ctypes.c_int),
                ("rope_theta", ctypes.c_double), ("norm_eps", ctypes.c_float), ("device", ctypes.c_int),
                ("io_host", ctypes.c_int)]


_lib = None

_SIGNATURES = {
    "qa_default_config": (None, [ctypes.POINTER(Config)]),
    "qa_create": (ctypes.c_int, [ctypes.POINTER(Config), ctypes.POINTER(ctypes.c_void_p)]),
    "qa_destroy": (None, [ctypes.c_void_p]),
    "qa_last_error": (ctypes.c_char_p, [ctypes.c_void_p]),
    "qa_status_string": (ctypes.c_char_p, [ctypes.c_int]),
    "qa_version": (ctypes.c_char_p, []),
    "qa_set_stream": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_void_p]),
    "qa_sync": (ctypes.c_int, [ctypes.c_void_p]),
    "qa_set_wait_limit": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_int]),
    "qa_selftest_timeout": (ctypes.c_int, [ctypes.c_void_p]),
    "qa_set_norms": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_int, ctypes.c_void_p, ctypes.c_void_p]),
    "qa_position": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_int, ctypes.POINTER(ctypes.c_int)]),
    "qa_reset": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_int]),
    "qa_truncate": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_int, ctypes.c_int]),
    "qa_commit": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_int, ctypes.c_int]),
    "qa_append": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int,
                                 ctypes.c_int, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p,
                                 ctypes.c_void_p]),
    "qa_attn_prefill": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int,
                                       ctypes.c_int, ctypes.c_void_p, ctypes.c_void_p]),
    "qa_attn_decode": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int,
                                      ctypes.c_int, ctypes.c_void_p, ctypes.c_void_p]),
    "qa_copy_prefix": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_int, ctypes.c_int, ctypes.c_int]),
    "qa_read_kv": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int,
                                  ctypes.c_int, ctypes.c_int, ctypes.c_void_p]),
    "qa_kv_pointer": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int,
                                     ctypes.POINTER(ctypes.c_void_p)]),
    "qa_kv_slot_bytes": (ctypes.c_int, [ctypes.c_void_p, ctypes.POINTER(ctypes.c_size_t)]),
    "qa_append_batch": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int, ctypes.c_int, ctypes.c_int,
                                       ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p]),
    "qa_attn_decode_batch": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int, ctypes.c_int,
                                            ctypes.c_int, ctypes.c_void_p, ctypes.c_void_p]),
    "qa_commit_batch": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int]),
    "qa_comm_unique_id": (ctypes.c_int, [ctypes.c_char_p]),
    "qa_comm_init": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_int, ctypes.c_int, ctypes.c_char_p]),
    "qa_comm_destroy": (ctypes.c_int, [ctypes.c_void_p]),
    "qa_gather_heads": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_int, ctypes.c_int, ctypes.c_void_p, ctypes.c_void_p]),
    "qa_kv_send": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_int, ctypes.c_int, ctypes.c_int]),
    "qa_kv_recv": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_int, ctypes.c_int, ctypes.c_int]),
    "qa_comm_join": (ctypes.c_int, [ctypes.c_void_p]),
    "qa_block_pool": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_int]),
    "qa_block_save": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_int, ctypes.c_int, ctypes.c_int]),
    "qa_block_load": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_int, ctypes.c_int, ctypes.c_int]),
    "qa_gather_heads_async": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_int, ctypes.c_int, ctypes.c_void_p,
                                             ctypes.c_void_p]),
    "qa_attn_prefill_gather": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int,
                                              ctypes.c_int, ctypes.c_void_p, ctypes.c_void_p]),
    "qa_set_step_overlap": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_int]),
    "qa_comm_info": (ctypes.c_int, [ctypes.c_void_p, ctypes.POINTER(ctypes.c_int), ctypes.POINTER(ctypes.c_int),
                                    ctypes.POINTER(ctypes.c_int)]),
    "qa_decode_step_gather": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int,
                                             ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p,
                                             ctypes.c_void_p]),
    "qa_decode_step": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int,
                                      ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p,
                                      ctypes.c_void_p]),
    "qa_decode_step_batch": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int, ctypes.c_int,
                                            ctypes.c_int, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p,
                                            ctypes.c_void_p, ctypes.c_void_p]),
    "qa_attn_decode_noalloc": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int,
                                              ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_void_p,
                                              ctypes.c_void_p, ctypes.c_void_p]),
    "qa_project": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int, ctypes.c_int, ctypes.c_void_p,
                                  ctypes.c_int, ctypes.c_void_p]),
    "qa_project_group": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_int, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int,
                                        ctypes.c_void_p, ctypes.c_int, ctypes.c_void_p]),
    "qa_project_gemm": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int, ctypes.c_int, ctypes.c_void_p,
                                       ctypes.c_int, ctypes.c_void_p]),
    "qa_project_group_gemm": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_int, ctypes.c_void_p, ctypes.c_void_p,
                                             ctypes.c_int, ctypes.c_void_p, ctypes.c_int, ctypes.c_void_p]),
    "qa_synth_fill": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_uint64, ctypes.c_int, ctypes.c_int, ctypes.c_int,
                                     ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_float,
                                     ctypes.c_float, ctypes.c_void_p]),
}

EXPORTS = tuple(_SIGNATURES)


def lib() -> ctypes.CDLL:
    """Loads libqattn.so (raises if it was not built: there is no fallback path)."""
    global _lib
    if _lib is None:
        path = Path(os.environ.get("QATTN_LIB", LIB_PATH))
        if not path.exists():
            raise RuntimeError(f"{path} is missing; build it with `python -m fpga_qwen_b200.build`")
        handle = ctypes.CDLL(str(path))
        for name, (res, args) in _SIGNATURES.items():
            fn = getattr(handle, name)
            fn.restype, fn.argtypes = res, args
        _lib = handle
    return _lib


def default_config(**overrides) -> Config:
    cfg = Config()
    lib().qa_default_config(ctypes.byref(cfg))
    for key, value in overrides.items():
        if not hasattr(cfg, key):
            raise TypeError(f"unknown config field {key}")
        setattr(cfg, key, value)
    return cfg


class Context:
    """Owns one ``qa_ctx``: the HBM KV store of ``max_seqs`` sequence slots and its state."""

    def __init__(self, **config):
        self.config = default_config(**config)
        handle = ctypes.c_void_p()
        st = lib().qa_create(ctypes.byref(self.config), ctypes.byref(handle))
        if st != QA_OK:
            raise QAttnError(st, "qa_create failed")
        self._h = handle
        heads = self.config.kv_head_count or self.config.n_kv_heads
        self.hkv = heads
        self.hq = heads * (self.config.n_q_heads // self.config.n_kv_heads)

    # -- helpers ---------------------------------------------------------------------------
    def _check(self, st: int):
        if st != QA_OK:
            raise QAttnError(st, lib().qa_last_error(self._h).decode())

    def close(self):
        if getattr(self, "_h", None):
            lib().qa_destroy(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()

    @property
    def handle(self):
        return self._h

    # -- ABI -------------------------------------------------------------------------------
    def set_stream(self, stream_ptr: int | None):
        """Run on a cudaStream_t. 0 is the legacy default stream (torch's default stream
        reports 0; it is passed as cudaStreamLegacy); None restores the context's own stream."""
        if stream_ptr == 0:
            stream_ptr = 1          # cudaStreamLegacy
        self._check(lib().qa_set_stream(self._h, stream_ptr))

    def sync(self):
        self._check(lib().qa_sync(self._h))

    def set_wait_limit(self, microseconds: int):
        """Limit of the bounded waits on other GPUs' flags (0: the default 2 s)."""
        self._check(lib().qa_set_wait_limit(self._h, microseconds))

    def selftest_timeout(self):
        """Launches a bounded wait on a flag nothing sets; the next sync() raises the timeout."""
        self._check(lib().qa_selftest_timeout(self._h))

    def set_norms(self, layer: int, q_norm_ptr: int, k_norm_ptr: int):
        self._check(lib().qa_set_norms(self._h, layer, q_norm_ptr, k_norm_ptr))

    def position(self, seq: int = 0) -> int:
        out = ctypes.c_int()
        st = lib().qa_position(self._h, seq, ctypes.byref(out))
        if st != QA_OK:
            raise QAttnError(st, "bad sequence")
        return out.value

    def reset(self, seq: int = 0):
        self._check(lib().qa_reset(self._h, seq))

    def truncate(self, seq: int, pos: int):
        self._check(lib().qa_truncate(self._h, seq, pos))

    def commit(self, seq: int, n: int):
        self._check(lib().qa_commit(self._h, seq, n))

    def append(self, seq, layer, n_layers, pos0, n, q_pre, k_pre, v, q_out):
        self._check(lib().qa_append(self._h, seq, layer, n_layers, pos0, n, q_pre, k_pre, v, q_out))

    def attn_prefill(self, seq, layer, n_layers, pos0, n, q, out):
        self._check(lib().qa_attn_prefill(self._h, seq, layer, n_layers, pos0, n, q, out))

    def attn_decode(self, seq, layer, n_layers, pos0, n, q, out):
        self._check(lib().qa_attn_decode(self._h, seq, layer, n_layers, pos0, n, q, out))

    def copy_prefix(self, src: int, dst: int, ntok: int):
        self._check(lib().qa_copy_prefix(self._h, src, dst, ntok))

    def block_pool(self, n_blocks: int):
        self._check(lib().qa_block_pool(self._h, n_blocks))

    def block_save(self, seq: int, chunk: int, block: int):
        self._check(lib().qa_block_save(self._h, seq, chunk, block))

    def block_load(self, seq: int, chunk: int, block: int):
        self._check(lib().qa_block_load(self._h, seq, chunk, block))

    def read_kv(self, seq, layer, kv, head, pos0, n, dst_ptr):
        self._check(lib().qa_read_kv(self._h, seq, layer, kv, head, pos0, n, dst_ptr))

    def kv_pointer(self, seq, layer, kv, head) -> int:
        out = ctypes.c_void_p()
        self._check(lib().qa_kv_pointer(self._h, seq, layer, kv, head, ctypes.byref(out)))
        return out.value

    # -- batched decode over sequences ------------------------------------------------------
    @staticmethod
    def _seq_array(seqs):
        arr = (ctypes.c_int * len(seqs))(*[int(x) for x in seqs])
        return arr, len(seqs)

    def append_batch(self, seqs, layer, n_layers, q_pre, k_pre, v, q_out):
        arr, n = self._seq_array(seqs)
        self._check(lib().qa_append_batch(self._h, arr, n, layer, n_layers, q_pre, k_pre, v, q_out))

    def attn_decode_batch(self, seqs, layer, n_layers, q, out):
        arr, n = self._seq_array(seqs)
        self._check(lib().qa_attn_decode_batch(self._h, arr, n, layer, n_layers, q, out))

    def decode_step(self, seq, layer, n_layers, pos, q_pre, k_pre, v, q_out, out):
        """Append of one new row + its decode attention in one launch (q_out may be 0)."""
        self._check(lib().qa_decode_step(self._h, seq, layer, n_layers, pos, q_pre, k_pre, v, q_out or None, out))

    def set_step_overlap(self, enable: bool):
        """Let consecutive fused decode steps overlap (programmatic dependent launch)."""
        self._check(lib().qa_set_step_overlap(self._h, 1 if enable else 0))

    def decode_step_batch(self, seqs, layer, n_layers, q_pre, k_pre, v, q_out, out):
        arr, n = self._seq_array(seqs)
        self._check(lib().qa_decode_step_batch(self._h, arr, n, layer, n_layers, q_pre, k_pre, v, q_out or None, out))

    def commit_batch(self, seqs):
        arr, n = self._seq_array(seqs)
        self._check(lib().qa_commit_batch(self._h, arr, n))

    # -- multi-GPU ------------------------------------------------------------------------
    def comm_init(self, nranks: int, rank: int, unique_id: bytes):
        if len(unique_id) != 128:
            raise ValueError("NCCL unique id must be 128 bytes")
        self._check(lib().qa_comm_init(self._h, nranks, rank, unique_id))

    def comm_destroy(self):
        self._check(lib().qa_comm_destroy(self._h))

    def gather_heads(self, n_layers: int, n: int, local_ptr: int, full_ptr: int):
        self._check(lib().qa_gather_heads(self._h, n_layers, n, local_ptr, full_ptr))

    def kv_send(self, seq: int, ntok: int, peer: int):
        self._check(lib().qa_kv_send(self._h, seq, ntok, peer))

    def kv_recv(self, seq: int, ntok: int, peer: int):
        self._check(lib().qa_kv_recv(self._h, seq, ntok, peer))

    def decode_step_gather(self, seq, layer, n_layers, pos, q_pre, k_pre, v, q_out, full):
        """Fused decode step on this rank's KV-head shard with the head gather over peer memory."""
        self._check(lib().qa_decode_step_gather(self._h, seq, layer, n_layers, pos, q_pre, k_pre, v, q_out or None,
                                                full))

    def comm_info(self):
        """(nranks, rank, peer_mapped) of the context's communicator."""
        n, r, pm = ctypes.c_int(), ctypes.c_int(), ctypes.c_int()
        self._check(lib().qa_comm_info(self._h, ctypes.byref(n), ctypes.byref(r), ctypes.byref(pm)))
        return n.value, r.value, bool(pm.value)

    def attn_prefill_gather(self, seq, layer, n_layers, pos0, n, q, full):
        """qa_attn_prefill on this rank's heads with the output rows of all ranks in `full`
        ([n_layers][n][all heads][128]); collective."""
        self._check(lib().qa_attn_prefill_gather(self._h, seq, layer, n_layers, pos0, n, q, full))

    def gather_heads_async(self, n_layers: int, n: int, local_ptr: int, full_ptr: int):
        """qa_gather_heads on the communication stream; complete after comm_join() or sync()."""
        self._check(lib().qa_gather_heads_async(self._h, n_layers, n, local_ptr, full_ptr))

    def comm_join(self):
        """Makes the context stream wait for the communication queued so far."""
        self._check(lib().qa_comm_join(self._h))

    def project(self, w_ptr: int, rows: int, cols: int, x_ptr: int, batch: int, y_ptr: int):
        """y [batch][rows] = eight-lane dot of x [batch][cols] with each row of the FP16 matrix w."""
        self._check(lib().qa_project(self._h, w_ptr, rows, cols, x_ptr, batch, y_ptr))

    def project_group(self, w_ptrs, rows, cols: int, x_ptr: int, batch: int, y_ptrs):
        """Several matrices sharing one input, one launch; y_ptrs[m] receives [batch][rows[m]]."""
        n = len(w_ptrs)
        ws = (ctypes.c_void_p * n)(*w_ptrs)
        rs = (ctypes.c_int * n)(*rows)
        ys = (ctypes.c_void_p * n)(*y_ptrs)
        self._check(lib().qa_project_group(self._h, n, ws, rs, cols, x_ptr, batch, ys))

    def project_gemm(self, w_ptr: int, rows: int, cols: int, x_ptr: int, batch: int, y_ptr: int):
        """Batched prompt rows on the tensor cores (FP32 products within accumulation rounding)."""
        self._check(lib().qa_project_gemm(self._h, w_ptr, rows, cols, x_ptr, batch, y_ptr))

    def project_group_gemm(self, w_ptrs, rows, cols: int, x_ptr: int, batch: int, y_ptrs):
        """project_group on the tensor cores; y_ptrs[m] receives [batch][rows[m]]."""
        n = len(w_ptrs)
        ws = (ctypes.c_void_p * n)(*w_ptrs)
        rs = (ctypes.c_int * n)(*rows)
        ys = (ctypes.c_void_p * n)(*y_ptrs)
        self._check(lib().qa_project_group_gemm(self._h, n, ws, rs, cols, x_ptr, batch, ys))

    def kv_slot_bytes(self) -> int:
        out = ctypes.c_size_t()
        self._check(lib().qa_kv_slot_bytes(self._h, ctypes.byref(out)))
        return out.value


def comm_unique_id() -> bytes:
    """A fresh NCCL unique id (128 bytes) for Context.comm_init."""
    buf = ctypes.create_string_buffer(128)
    st = lib().qa_comm_unique_id(buf)
    if st != QA_OK:
        raise QAttnError(st, "qa_comm_unique_id failed (is libnccl.so.2 available?)")
    return buf.raw


NOALLOC_SCRATCH_BYTES = 4 << 20


def attn_decode_noalloc(kv_slot_ptr: int, n_layers_total: int, n_kv_heads: int, context: int, layer: int,
                        n_layers: int, pos0: int, n: int, q_ptr: int, out_ptr: int, stream: int | None = None) -> int:
    """Split-context decode that allocates nothing (scratch in a fixed device array).
    Returns the C status; 0 is success. stream 0 means the legacy default stream."""
    if stream == 0:
        stream = 1          # cudaStreamLegacy
    return lib().qa_attn_decode_noalloc(kv_slot_ptr, n_layers_total, n_kv_heads, context, layer, n_layers, pos0, n,
                                        q_ptr, out_ptr, stream or None)


def synth_fill(dst_ptr: int, seed: int, kind: int, layer0: int, n_layers: int, pos0: int, n: int,
               head0: int, heads: int, mean: float = 0.0, std: float = 1.0, stream: int | None = None):
    st = lib().qa_synth_fill(dst_ptr, seed & 0xFFFFFFFFFFFFFFFF, kind, layer0, n_layers, pos0, n, head0, heads,
                             mean, std, stream or None)
    if st != QA_OK:
        raise QAttnError(st, "qa_synth_fill failed")
