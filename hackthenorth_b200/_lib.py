"""ctypes binding of ``libqb.so`` (declared in ``include/qb.h``).

There is no fallback: if the library is missing the engine refuses to run.
"""
from __future__ import annotations

import ctypes
import os

PKG = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(PKG, "libqb.so")

QB_OK = 0
QB_ERR_ARG = 1
QB_ERR_CAPACITY = 2
QB_ERR_CUDA = 3
QB_ERR_TIMEOUT = 4
QB_ERR_STATE = 5
QB_ERR_UNSUPPORTED = 6

c_int, c_float, c_void_p, c_size_t = ctypes.c_int, ctypes.c_float, ctypes.c_void_p, ctypes.c_size_t


class QbConfig(ctypes.Structure):
    _fields_ = [("hidden", c_int), ("n_heads", c_int), ("n_kv_heads", c_int), ("head_dim", c_int),
                ("ffn", c_int), ("n_layers", c_int), ("vocab", c_int), ("rms_eps", c_float)]


class QbLayerWeights(ctypes.Structure):
    _fields_ = [(n, c_void_p) for n in ("input_norm", "qkv", "q_norm", "k_norm", "o", "post_norm",
                                        "gate_up", "down")]


# name -> (restype, argtypes); every symbol include/qb.h declares.
SIGNATURES = {
    "qb_version": (ctypes.c_char_p, []),
    "qb_last_error": (ctypes.c_char_p, [c_void_p]),
    "qb_create": (c_int, [ctypes.POINTER(QbConfig), c_int, c_int, c_int, ctypes.POINTER(c_void_p)]),
    "qb_destroy": (c_int, [c_void_p]),
    "qb_nccl_unique_id": (c_int, [c_void_p, c_size_t]),
    "qb_tp_init": (c_int, [c_void_p, c_void_p]),
    "qb_bind_weights": (c_int, [c_void_p, ctypes.POINTER(QbLayerWeights), c_int, c_void_p, c_void_p, c_void_p]),
    "qb_workspace_bytes": (c_int, [c_void_p, ctypes.POINTER(c_size_t)]),
    "qb_bind_state": (c_int, [c_void_p, c_void_p, c_void_p, c_int, c_void_p, c_void_p, c_void_p, c_size_t]),
    "qb_decode_step": (c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_void_p]),
    "qb_set_batch": (c_int, [c_void_p, c_int]),
    "qb_prefill": (c_int, [c_void_p, c_void_p, c_int, c_void_p, c_void_p, c_void_p, c_void_p]),
    "qb_capture_decode": (c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_void_p]),
    "qb_replay_decode": (c_int, [c_void_p, c_void_p]),
    "qb_check": (c_int, [c_void_p, c_void_p]),
    "qb_set_trace": (c_int, [c_void_p, c_void_p, c_size_t]),
    "qb_trace_labels": (ctypes.c_char_p, [c_void_p]),
    "qb_prefill_scratch_bytes": (c_int, [c_void_p, c_int, c_void_p]),
    "qb_bind_prefill_weights": (c_int, [c_void_p, ctypes.POINTER(c_void_p), ctypes.POINTER(c_void_p), c_int]),
    "qb_prefill_batched": (c_int, [c_void_p, c_void_p, c_int, c_void_p, c_size_t, c_void_p, c_void_p, c_void_p,
                                   c_void_p]),
    "qb_gemm_bf16": (c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_int, c_int, c_int, c_int, c_void_p,
                             c_void_p]),
    "qb_verify": (c_int, [c_void_p, c_void_p, c_int, c_void_p, c_void_p, c_void_p, c_void_p]),
    "qb_capture_verify": (c_int, [c_void_p, c_void_p, c_int, c_void_p, c_void_p, c_void_p, c_void_p]),
    "qb_replay_verify": (c_int, [c_void_p, c_void_p]),
    "qb_norm_projection": (c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_int, c_int, c_float, c_int, c_void_p]),
    "qb_projection_residual": (c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_int, c_int, c_void_p]),
    "qb_projection_residual_peer": (c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_int, c_int,
                                            ctypes.POINTER(c_void_p), c_int, c_int, c_int, c_int, c_void_p,
                                            c_void_p, c_void_p]),
    "qb_op_scratch_bytes": (c_size_t, []),
    "qb_norm_greedy_head": (c_int, [c_void_p, c_void_p, c_void_p, c_int, c_int, c_float, c_void_p, c_void_p,
                                    c_void_p, c_size_t, c_void_p]),
    "qb_grouped_attention": (c_int, [c_void_p, c_void_p, c_void_p, c_int, c_int, c_int, c_int, c_void_p,
                                     c_void_p, c_void_p, c_size_t, c_void_p]),
    "qb_rope_attention": (c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_float, c_void_p, c_void_p,
                                  c_int, c_int, c_int, c_void_p, c_void_p, c_void_p, c_size_t, c_void_p]),
    "qb_op_check": (c_int, [c_void_p, c_void_p]),
    "qb_grouped_attention_noalloc": (c_int, [c_void_p, c_void_p, c_void_p, c_int, c_int, c_int, c_int, c_void_p,
                                             c_void_p, c_void_p, c_void_p]),
}

_lib = None


class QbError(RuntimeError):
    def __init__(self, code: int, msg: str):
        super().__init__(f"[qb {code}] {msg}")
        self.code = code


def load() -> ctypes.CDLL:
    """The loaded library; raises if it has not been built."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise RuntimeError(
                f"hackthenorth_b200: {LIB_PATH} is not built. Run `python -m hackthenorth_b200.build`. "
                "The engine has no CPU or PyTorch fallback.")
        lib = ctypes.CDLL(LIB_PATH)
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(lib, name)
            fn.restype = res
            fn.argtypes = args
        _lib = lib
    return _lib


def check(rc: int, ctx=None) -> None:
    if rc == QB_OK:
        return
    msg = load().qb_last_error(ctx).decode(errors="replace")
    if rc in (QB_ERR_ARG, QB_ERR_CAPACITY, QB_ERR_UNSUPPORTED):
        raise ValueError(f"[qb {rc}] {msg}")
    raise QbError(rc, msg)


def ptr(t) -> int:
    """Device address of a tensor (or None -> NULL)."""
    return None if t is None else t.data_ptr()


def stream_handle(stream=None):
    import torch

    s = torch.cuda.current_stream() if stream is None else stream
    return s.cuda_stream
