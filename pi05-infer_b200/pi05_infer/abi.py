"""ctypes mirrors of the C structs in ``include/pi05_b200.h`` and typed wrappers
of the non-GEMM entry points."""

from __future__ import annotations

import ctypes

import torch

from . import _lib

_P = ctypes.c_void_p
_I = ctypes.c_int
_Z = ctypes.c_size_t
_F = ctypes.c_float


class Pi05ExpertLayer(ctypes.Structure):
    _fields_ = [
        ("w_qkv", _P), ("w_o", _P), ("w_gate", _P), ("w_up", _P), ("w_down", _P),
        ("k_cache", _P), ("v_cache", _P),
    ]


class Pi05ExpertFold(ctypes.Structure):
    _fields_ = [
        ("w_qkv", _P), ("w_gate", _P), ("w_up", _P), ("b_qkv", _P), ("b_gate", _P), ("b_up", _P),
    ]


class Pi05ExpertPlan(ctypes.Structure):
    _fields_ = [
        ("depth", _I), ("width", _I), ("mlp_dim", _I), ("n_q_heads", _I), ("n_kv_heads", _I), ("head_dim", _I),
        ("tokens", _I), ("action_dim", _I), ("prefix_len", _I), ("kv_rows", _I), ("eps", _F),
        ("layers", ctypes.POINTER(Pi05ExpertLayer)), ("num_steps", _I),
        ("host_timesteps", ctypes.POINTER(_F)), ("mod_table", _P),
        ("w_in", _P), ("b_in", _P), ("w_out", _P), ("b_out", _P),
        ("rope_cos", _P), ("rope_sin", _P), ("key_valid", _P),
        ("x_t", _P), ("v_t", _P), ("h", _P), ("xn", _P), ("q", _P), ("attn", _P), ("act", _P),
        ("workspace", _P), ("workspace_bytes", _Z), ("attn_splits", _I), ("trace", _P),
        ("fold", ctypes.POINTER(Pi05ExpertFold)),
        ("batch", _I), ("kv_stage", _P), ("host_step_coefs", ctypes.POINTER(_F)), ("step_noise", _P),
    ]


_EXTRA = {
    "pi05_rms_norm": (_I, [_P, _I, _P, _P, _P, _I, _I, _I, _F, _P]),
    "pi05_attention": (_I, [_P, _P, _P, _P, _P, _I, _I, _I, _F, _I, _P, _Z, _P]),
    "pi05_action_in": (_I, [_P, _P, _P, _P, _I, _I, _I, _P]),
    "pi05_final_euler": (_I, [_P, _P, _P, _P, _P, _P, _I, _I, _I, _F, _F, _F, _P]),
    "pi05_rope_table": (_I, [_P, _I, _I, _I, _P, _I, _P, _P, _P]),
    "pi05_adarms_table": (_I, [_P, _I, _I, _P, _P, _P, _P, _P, _P, _I, _P, _P, _Z, _P]),
    "pi05_denoise_step": (_I, [ctypes.POINTER(Pi05ExpertPlan), _I, _P]),
    "pi05_denoise_loop": (_I, [ctypes.POINTER(Pi05ExpertPlan), _P]),
    "pi05_fold_adarms": (_I, [_P, _I, _I, _P, _P, _P, _P, _P]),
    "pi05_preprocess_images": (_I, [_P, _I, _I, _I, _I, _P, _I, _P]),
    "pi05_normalize_rows": (_I, [_P, _I, _I, _P, _P, _I, _I, _P, _I, _P]),
    "pi05_unnormalize_rows": (_I, [_P, _I, _I, _P, _P, _I, _I, _P, _I, _P]),
}
_lib.SIGNATURES.update(_EXTRA)


def _bind():
    L = _lib.lib()
    for name, (res, args) in _EXTRA.items():
        f = getattr(L, name)
        f.restype = res
        f.argtypes = args
    return L


def ptr(t) -> int:
    return 0 if t is None else t.data_ptr()


def stream_of(device) -> int:
    return torch.cuda.current_stream(device).cuda_stream


def rms_norm(x, mod, weight, out, eps, stream=None):
    _bind()
    rows, d = x.shape[-2], x.shape[-1]
    rows = x.numel() // d
    _lib.call("pi05_rms_norm", ptr(x), d, ptr(mod), ptr(weight), ptr(out), d, rows, d, eps,
              stream if stream is not None else stream_of(x.device))
    return out


def attention(q, k, v, key_valid, out, scale, splits, ws, stream=None):
    _bind()
    d = q.shape[-1]
    rows = q.numel() // d
    _lib.call("pi05_attention", ptr(q), ptr(k), ptr(v), ptr(key_valid), ptr(out), rows, k.shape[-2], d, scale,
              splits, ptr(ws), ws.numel(), stream if stream is not None else stream_of(q.device))
    return out


def rope_table(valid, n_prefix, mode, rows, inv_freq, d, cos, sin, stream=None):
    _bind()
    _lib.call("pi05_rope_table", ptr(valid), n_prefix, mode, rows, ptr(inv_freq), d, ptr(cos), ptr(sin),
              stream if stream is not None else stream_of(cos.device))


def adarms_table(timesteps, width, w_tin, b_tin, w_tout, b_tout, w_dense, b_dense, n_norm, table, ws, stream=None):
    _bind()
    _lib.call("pi05_adarms_table", ptr(timesteps), timesteps.numel(), width, ptr(w_tin), ptr(b_tin), ptr(w_tout),
              ptr(b_tout), ptr(w_dense), ptr(b_dense), n_norm, ptr(table), ptr(ws), ws.numel(),
              stream if stream is not None else stream_of(table.device))


def fold_adarms(w, scale, shift, w_out, b_out, stream=None):
    """``w_out = bf16(w * (1 + scale))`` column-wise and ``b_out = w @ shift`` (fp32)."""
    _bind()
    rows, k = w.shape
    assert w_out.shape == w.shape and b_out.numel() == rows and scale.numel() == k and shift.numel() == k
    _lib.call("pi05_fold_adarms", ptr(w), rows, k, ptr(scale), ptr(shift), ptr(w_out), ptr(b_out),
              stream if stream is not None else stream_of(w.device))


def denoise_loop(plan: Pi05ExpertPlan, stream: int):
    _bind()
    _lib.call("pi05_denoise_loop", ctypes.byref(plan), stream)


def denoise_step(plan: Pi05ExpertPlan, step: int, stream: int):
    _bind()
    _lib.call("pi05_denoise_step", ctypes.byref(plan), step, stream)
