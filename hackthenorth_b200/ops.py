"""Op-level wrappers of the sm_100a kernels, mirroring the reference's kernel wrappers.

Like the reference (``dryft/engine/kernels/*.py``) each wrapper validates its
inputs (``ValueError`` on contract violations), allocates and returns new
outputs, never mutates inputs (except the KV cache written in place by
``rope_attention``), and launches on the current CUDA stream. Every call runs
the CUDA library; there is no PyTorch or CPU fallback.
"""
from __future__ import annotations

import torch

from . import _lib

BF16 = torch.bfloat16
_scratch = {}


def _op_scratch(device) -> torch.Tensor:
    """Zero-initialised per-device scratch for the split-KV and argmax partials.
    The kernels restore their counters to zero, so it is reused across calls
    (calls on different streams must not overlap)."""
    key = torch.device(device).index
    buf = _scratch.get(key)
    if buf is None:
        n = int(_lib.load().qb_op_scratch_bytes())
        buf = torch.zeros(n, dtype=torch.uint8, device=device)
        _scratch[key] = buf
    return buf


def _require(cond: bool, msg: str):
    if not cond:
        raise ValueError(msg)


def _bf16_cuda(*ts):
    for t in ts:
        if t is None:
            continue
        _require(t.is_cuda and t.dtype == BF16 and t.is_contiguous(),
                 "expected contiguous bf16 CUDA tensors")


def check_device_errors(device=None) -> None:
    """Synchronise and raise if an op-level kernel reported a device error."""
    buf = _op_scratch(device or torch.cuda.current_device())
    _lib.check(_lib.load().qb_op_check(buf.data_ptr(), _lib.stream_handle()))


def norm_projection(x, gain, weight, eps=1e-6, *, swiglu=False):
    """RMSNorm(x) (skipped when gain is None) fused with W.x; with ``swiglu`` the
    weight is ``[2N, K]`` gate/up-interleaved and the result is SwiGLU [N].
    ``dryft/engine/kernels/projection.py:36-53``."""
    _bf16_cuda(x, gain, weight)
    _require(x.numel() == x.shape[-1], "the batch-one path requires one hidden row")
    rows, k = weight.shape
    _require(x.shape[-1] == k and (gain is None or gain.numel() == k), "incompatible projection dimensions")
    if swiglu:
        _require(rows % 2 == 0, "packed gate/up width must be even")
    n = rows // 2 if swiglu else rows
    out = torch.empty((*x.shape[:-1], n), dtype=BF16, device=x.device)
    _lib.check(_lib.load().qb_norm_projection(x.data_ptr(), _lib.ptr(gain), weight.data_ptr(), out.data_ptr(),
                                              k, rows, float(eps), int(bool(swiglu)), _lib.stream_handle()))
    return out


def output_projection_residual(x, weight, residual):
    """bf16(bf16(W.x) + residual): ``dryft/engine/kernels/projection.py:70-83``."""
    _bf16_cuda(x, weight, residual)
    n, k = weight.shape
    _require(x.numel() == k and residual.numel() == n, "output projection requires one activation and residual row")
    out = torch.empty_like(residual)
    _lib.check(_lib.load().qb_projection_residual(x.data_ptr(), weight.data_ptr(), residual.data_ptr(),
                                                  out.data_ptr(), k, n, _lib.stream_handle()))
    return out


def projection_residual_peer(x, weight, residual, recv_words, rank, epoch, sublayer=0, parity=0):
    """One rank's share of a tensor-parallel o-proj / down projection with the
    cross-rank reduction in its epilogue: bf16(bf16(sum_r W_r.x_r) + residual),
    partials added in rank order (``dryft/engine/kernels/projection.py:70-83``
    with the sum spread over ranks). ``recv_words``: one uint64-viewable CUDA
    tensor (or raw device address) per rank, each ``[2, size, N]`` words;
    ``epoch``: CUDA int64 [1] (token base). Device-side wait timeouts surface
    through ``check_device_errors``."""
    _bf16_cuda(x, weight, residual)
    n, k = weight.shape
    _require(x.numel() == k and residual.numel() == n, "projection requires one activation and residual row")
    size = len(recv_words)
    _require(1 <= size <= 8 and 0 <= rank < size, "1..8 ranks, rank in range")
    _require(epoch.is_cuda and epoch.dtype == torch.int64 and epoch.numel() >= 1, "epoch must be CUDA int64")
    ptrs = []
    for t in recv_words:
        if isinstance(t, int):
            ptrs.append(t)
        else:
            _require(t.is_cuda and t.numel() * t.element_size() >= 2 * size * n * 8, "receive buffer too small")
            ptrs.append(t.data_ptr())
    arr = (_lib.c_void_p * size)(*ptrs)
    out = torch.empty_like(residual)
    scratch = _op_scratch(x.device)
    _lib.check(_lib.load().qb_projection_residual_peer(x.data_ptr(), weight.data_ptr(), residual.data_ptr(),
                                                       out.data_ptr(), k, n, arr, rank, size, sublayer, parity,
                                                       epoch.data_ptr(), scratch.data_ptr(), _lib.stream_handle()))
    return out


def down_residual(x, weight, residual):
    """Down projection + residual with one rounding before the add:
    ``dryft/engine/kernels/down.py:288-296``."""
    return output_projection_residual(x, weight, residual)


def greedy_token(x, weight, gain=None, eps=1e-6, return_logits=False):
    """(Optional final RMSNorm +) LM head + argmax of the bf16 logits with the
    lowest index on ties: ``dryft/engine/kernels/greedy.py:45-60``."""
    _bf16_cuda(x, weight, gain)
    _require(x.numel() == x.shape[-1], "the batch-one head takes one hidden row")
    v, k = weight.shape
    _require(x.shape[-1] == k, "incompatible head dimensions")
    token = torch.empty(1, dtype=torch.int64, device=x.device)
    logits = torch.empty(v, dtype=BF16, device=x.device) if return_logits else None
    scratch = _op_scratch(x.device)
    _lib.check(_lib.load().qb_norm_greedy_head(x.data_ptr(), _lib.ptr(gain), weight.data_ptr(), k, v, float(eps),
                                               _lib.ptr(logits), token.data_ptr(), scratch.data_ptr(),
                                               scratch.numel(), _lib.stream_handle()))
    return (token, logits) if return_logits else token


def grouped_attention(q, keys, values, positions):
    """Split-KV GQA attention. q ``[Q, Hq, D]`` (normalised, rotated), keys/values
    ``[Hkv, cap, D]``, positions int64 ``[Q]`` (consecutive) -> ``[Q, Hq, D]``.
    ``dryft/engine/kernels/attention.py:213-237`` (batch one)."""
    _bf16_cuda(q, keys, values)
    _require(q.dim() == 3 and keys.dim() == 3 and keys.shape == values.shape, "expected q [Q,Hq,D], kv [Hkv,cap,D]")
    Q, hq, d = q.shape
    hkv, cap, _ = keys.shape
    _require(d == 128 and keys.shape[2] == 128, "head_dim must be 128")
    _require(positions.is_cuda and positions.dtype == torch.int64 and positions.numel() == Q,
             "positions must be a CUDA int64 tensor with one entry per query")
    out = torch.empty_like(q)
    scratch = _op_scratch(q.device)
    _lib.check(_lib.load().qb_grouped_attention(q.data_ptr(), keys.data_ptr(), values.data_ptr(), hq, hkv, cap, Q,
                                                positions.data_ptr(), out.data_ptr(), scratch.data_ptr(),
                                                scratch.numel(), _lib.stream_handle()))
    return out


def rope_attention(qkv, q_norm, k_norm, cos, sin, keys, values, position, eps=1e-6, n_heads=None):
    """Decode attention with q/k RMSNorm + RoPE + KV append fused in.
    qkv packed ``[Hq*D + 2*Hkv*D]``; keys/values ``[Hkv, cap, D]`` updated at
    ``position`` (int64 [1] CUDA); cos/sin ``[cap, D]`` -> ``[Hq, D]``.
    ``dryft/engine/kernels/fused.py:153-165`` + ``attention.py:213-237``."""
    _bf16_cuda(qkv, q_norm, k_norm, cos, sin, keys, values)
    hkv, cap, d = keys.shape
    _require(d == 128, "head_dim must be 128")
    width = qkv.numel()
    hq = n_heads if n_heads is not None else width // d - 2 * hkv
    _require(width == (hq + 2 * hkv) * d, "packed qkv width does not match the cache heads")
    _require(cos.shape[0] >= cap and sin.shape[0] >= cap, "rope tables shorter than the cache")
    out = torch.empty((hq, d), dtype=BF16, device=qkv.device)
    scratch = _op_scratch(qkv.device)
    _lib.check(_lib.load().qb_rope_attention(qkv.data_ptr(), q_norm.data_ptr(), k_norm.data_ptr(), cos.data_ptr(),
                                             sin.data_ptr(), float(eps), keys.data_ptr(), values.data_ptr(), hq, hkv,
                                             cap, position.data_ptr(), out.data_ptr(), scratch.data_ptr(),
                                             scratch.numel(), _lib.stream_handle()))
    return out
