"""Torch-facing wrappers over the C ABI, including the reference's custom ops.

``torch.ops.pi05_infer.gate_up_geglu`` and ``torch.ops.pi05_infer.qkv_rope_kv``
keep the reference's names, schemas and semantics
(``pi05_infer/gemma/rlinf_fused_denoise.py:350-467``) so callers written against
the reference keep working; the dispatchers ``fused_gate_up_geglu`` /
``fused_qkv_rope_kv`` keep its contract of returning ``None`` when the fast path
does not apply (``rlinf_fused_denoise.py:489-562``).  The implementation is the
sm_100a library; there is no Triton and no eager fallback inside the ops.

The module also exports the rest of the reference module's public names
(``rlinf_fused_denoise.py:32-38``): ``HAVE_FUSED_DENOISE_OPS`` and the two
``fuse_*_enabled`` switches, so that the reference's own callers can import this
module in place of ``rlinf_fused_denoise`` (``modeling_gemma.py:54-60`` reads the
flag and keeps the module only when it is true).
"""

from __future__ import annotations

import os
from typing import Optional

import torch

from . import _lib

__all__ = [
    "HAVE_FUSED_DENOISE_OPS",
    "fuse_geglu_enabled",
    "fuse_qkv_rope_enabled",
    "fused_gate_up_geglu",
    "fused_qkv_rope_kv",
]


def _library_loads() -> bool:
    try:
        _lib.lib()
        return True
    except (RuntimeError, OSError):
        return False


# True when the sm_100a library is built and loads (the reference's flag is true
# when Triton imports, rlinf_fused_denoise.py:72-82).  Per call, the dispatchers
# still return None for CPU tensors, as the reference's do.
HAVE_FUSED_DENOISE_OPS = _library_loads()


def _env_int(name: str, default: int, legacy: Optional[str] = None) -> int:
    raw = os.environ.get(name) or (os.environ.get(legacy) if legacy else None)
    if not raw:
        return default
    try:
        return int(raw)
    except ValueError:
        return default


def fuse_geglu_enabled() -> bool:
    """True when the fused gate/up+GeGLU op should be used (kill switch
    ``RLINF_FUSE_GEGLU=0``, alias ``RLINF_FUSE_SWIGLU``; ``rlinf_fused_denoise.py:97-101``)."""
    return HAVE_FUSED_DENOISE_OPS and _env_int("RLINF_FUSE_GEGLU", 1, legacy="RLINF_FUSE_SWIGLU") != 0


def fuse_qkv_rope_enabled() -> bool:
    """True when the fused QKV+RoPE op should be used (kill switch
    ``RLINF_FUSE_QKV_ROPE=0``; ``rlinf_fused_denoise.py:104-106``)."""
    return HAVE_FUSED_DENOISE_OPS and _env_int("RLINF_FUSE_QKV_ROPE", 1) != 0

_WS = {}
_WS_TOKENS = 512
_WS_KV = 2048


def workspace(device: torch.device) -> torch.Tensor:
    """Per-device scratch for split-K / split-KV partials (zeroed once)."""
    device = torch.device(device)
    idx = device.index if device.index is not None else torch.cuda.current_device()
    ws = _WS.get(idx)
    if ws is None:
        nbytes = _lib.lib().pi05_workspace_bytes(_WS_TOKENS, _WS_KV)
        ws = torch.zeros(nbytes, dtype=torch.uint8, device=torch.device("cuda", idx))
        _WS[idx] = ws
    return ws


def _stream(device) -> int:
    return torch.cuda.current_stream(device).cuda_stream


def _p(t: Optional[torch.Tensor]) -> Optional[int]:
    return None if t is None else t.data_ptr()


def _check_bf16_cuda(*ts: torch.Tensor) -> None:
    for t in ts:
        if not t.is_cuda or t.dtype != torch.bfloat16 or not t.is_contiguous():
            raise ValueError("expected contiguous bf16 CUDA tensors")


def read_device_status(device=None) -> int:
    """Synchronise and read/clear the device status word (0 = no kernel timed out)."""
    ws = workspace(device or torch.device("cuda"))
    v = _lib.ctypes.c_int(0)
    rc = _lib.lib().pi05_read_device_status(_p(ws), _lib.ctypes.byref(v), _stream(ws.device))
    if rc not in (0, 7):
        raise _lib.Pi05Error("pi05_read_device_status", rc, _lib.last_error())
    return v.value


# ---------------------------------------------------------------------------
# raw ops (explicit outputs)
# ---------------------------------------------------------------------------


def linear(x: torch.Tensor, w: torch.Tensor, out: Optional[torch.Tensor] = None) -> torch.Tensor:
    _check_bf16_cuda(x, w)
    m, k = x.reshape(-1, x.shape[-1]).shape
    n = w.shape[0]
    if out is None:
        out = torch.empty(*x.shape[:-1], n, dtype=x.dtype, device=x.device)
    ws = workspace(x.device)
    _lib.call("pi05_linear", _p(x), _p(w), _p(out), m, n, k, _p(ws), ws.numel(), _stream(x.device))
    return out


def linear_gated_residual(
    x: torch.Tensor, w: torch.Tensor, resid: torch.Tensor, gate: Optional[torch.Tensor], out: Optional[torch.Tensor] = None
) -> torch.Tensor:
    """``resid + bf16(x @ w.T) * gate`` (gate fp32 ``[n]`` or None)."""
    _check_bf16_cuda(x, w, resid)
    m, k = x.reshape(-1, x.shape[-1]).shape
    n = w.shape[0]
    if gate is not None and (gate.dtype != torch.float32 or not gate.is_contiguous() or gate.numel() != n):
        raise ValueError("gate must be contiguous fp32 [n]")
    if out is None:
        out = torch.empty_like(resid)
    ws = workspace(x.device)
    _lib.call("pi05_linear_gated_residual", _p(x), _p(w), _p(resid), _p(gate), _p(out), m, n, k, _p(ws), ws.numel(),
              _stream(x.device))
    return out


def geglu(x: torch.Tensor, wg: torch.Tensor, wu: torch.Tensor, out: Optional[torch.Tensor] = None) -> torch.Tensor:
    _check_bf16_cuda(x, wg, wu)
    k = x.shape[-1]
    m = x.numel() // k
    n = wg.shape[0]
    if out is None:
        out = torch.empty(*x.shape[:-1], n, dtype=x.dtype, device=x.device)
    ws = workspace(x.device)
    _lib.call("pi05_gate_up_geglu", _p(x), _p(wg), _p(wu), _p(out), m, n, k, _p(ws), ws.numel(), _stream(x.device))
    return out


def qkv_rope(
    x: torch.Tensor, w: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor, q_out: torch.Tensor,
    k_cache: torch.Tensor, v_cache: torch.Tensor, krow0: int, n_q_heads: int, n_kv_heads: int, head_dim: int,
) -> torch.Tensor:
    _check_bf16_cuda(x, w, cos, sin, q_out, k_cache, v_cache)
    k = x.shape[-1]
    m = x.numel() // k
    kv_rows = k_cache.shape[-2]
    ws = workspace(x.device)
    _lib.call("pi05_qkv_rope_kv", _p(x), _p(w), _p(cos), _p(sin), _p(q_out), _p(k_cache), _p(v_cache), m, k, krow0,
              kv_rows, n_q_heads, n_kv_heads, head_dim, _p(ws), ws.numel(), _stream(x.device))
    return q_out


# ---------------------------------------------------------------------------
# the reference's custom ops (same namespace, names and schemas)
# ---------------------------------------------------------------------------


@torch.library.custom_op("pi05_infer::gate_up_geglu", mutates_args=())
def gate_up_geglu(x: torch.Tensor, wg: torch.Tensor, wu: torch.Tensor) -> torch.Tensor:
    """gelu_tanh(x @ wg.T) * (x @ wu.T) in one fused tcgen05 GEMM."""
    return geglu(x.contiguous(), wg, wu)


@gate_up_geglu.register_fake
def _(x, wg, wu):
    return x.new_empty((*x.shape[:-1], wg.shape[0]))


@torch.library.custom_op("pi05_infer::qkv_rope_kv", mutates_args={"k_cache", "v_cache"})
def qkv_rope_kv(
    x: torch.Tensor, w: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor, k_cache: torch.Tensor,
    v_cache: torch.Tensor, krow0: int, n_q_heads: int, n_kv_heads: int, head_dim: int,
) -> torch.Tensor:
    """Fused QKV projection + RoPE; q as ``[B, M, Hq, D]``, k/v into cache rows ``krow0:``."""
    b, m, _ = x.shape
    if b != 1:
        # one cache per observation: issue one launch per batch row
        q = torch.empty(b, m, n_q_heads, head_dim, dtype=x.dtype, device=x.device)
        for i in range(b):
            qkv_rope(x[i].contiguous(), w, cos.reshape(b, m, head_dim)[i].contiguous(),
                     sin.reshape(b, m, head_dim)[i].contiguous(), q[i], k_cache[i], v_cache[i], krow0, n_q_heads,
                     n_kv_heads, head_dim)
        return q
    q = torch.empty(b, m, n_q_heads, head_dim, dtype=x.dtype, device=x.device)
    qkv_rope(x.contiguous(), w, cos.reshape(m, head_dim).contiguous(), sin.reshape(m, head_dim).contiguous(), q,
             k_cache, v_cache, krow0, n_q_heads, n_kv_heads, head_dim)
    return q


@qkv_rope_kv.register_fake
def _(x, w, cos, sin, k_cache, v_cache, krow0, n_q_heads, n_kv_heads, head_dim):
    return x.new_empty((x.shape[0], x.shape[1], n_q_heads, head_dim))


def _rowmajor(w: torch.Tensor) -> bool:
    return w.dim() == 2 and w.stride(1) == 1 and w.stride(0) == w.shape[1]


def _needs_autograd(*ts: torch.Tensor) -> bool:
    return torch.is_grad_enabled() and any(t.requires_grad for t in ts)


def fused_gate_up_geglu(x: torch.Tensor, wg: torch.Tensor, wu: torch.Tensor) -> Optional[torch.Tensor]:
    """Dispatcher with the reference's guards (``rlinf_fused_denoise.py:489-517``): ``None`` = not applicable."""
    if not fuse_geglu_enabled() or _needs_autograd(x, wg, wu):
        return None
    if (
        not x.is_cuda
        or x.dtype != torch.bfloat16
        or wg.dtype is not x.dtype
        or wu.dtype is not x.dtype
        or wg.shape != wu.shape
        or not _rowmajor(wg)
        or not _rowmajor(wu)
        or x.stride(-1) != 1
        or x.shape[-1] % 64
        or wg.shape[0] % 64
    ):
        return None
    return torch.ops.pi05_infer.gate_up_geglu(x.contiguous(), wg, wu)


def fused_qkv_rope_kv(
    x: torch.Tensor, w: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor, k_cache: torch.Tensor,
    v_cache: torch.Tensor, krow0: int, n_q_heads: int, n_kv_heads: int, head_dim: int,
) -> Optional[torch.Tensor]:
    """Dispatcher with the reference's guards (``rlinf_fused_denoise.py:520-562``)."""
    if not fuse_qkv_rope_enabled() or _needs_autograd(x, w):
        return None
    if (
        not x.is_cuda
        or x.dim() != 3
        or x.dtype != torch.bfloat16
        or w.dtype is not x.dtype
        or not _rowmajor(w)
        or x.stride(-1) != 1
        or x.shape[-1] % 64
        or head_dim % 128
        or w.shape[0] != (n_q_heads + n_kv_heads * 2) * head_dim
        or cos.shape[-1] != head_dim
        or cos.dtype is not x.dtype
        or k_cache is None
        or v_cache is None
        or k_cache.dtype is not x.dtype
        or krow0 + x.shape[1] != k_cache.shape[2]
    ):
        return None
    return torch.ops.pi05_infer.qkv_rope_kv(x.contiguous(), w, cos, sin, k_cache, v_cache, krow0, n_q_heads,
                                            n_kv_heads, head_dim)
