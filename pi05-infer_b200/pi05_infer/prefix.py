"""PaliGemma prefix LM (Gemma-2B) on the C ABI: fills the expert's static KV cache.

The reference runs the prefix through transformers' Gemma with a fused q|k|v
projection (``patches/prefix_qkv_fused.py``), then copies the DynamicCache into
the expert's static buffers (``prime_kv_static``).  Here the QKV epilogue writes
rotated K and raw V straight into those buffers.
"""

from __future__ import annotations

import ctypes
import os
from typing import Dict, List, Optional, Sequence

import torch

from . import _lib, abi, ops
from .config import GEMMA_2B, GemmaShape
from .expert import rope_inv_freq
from .synthetic import LM_PREFIX


class Pi05PrefixLayer(ctypes.Structure):
    _fields_ = [("w_qkv", ctypes.c_void_p), ("w_o", ctypes.c_void_p), ("w_gate", ctypes.c_void_p),
                ("w_up", ctypes.c_void_p), ("w_down", ctypes.c_void_p), ("ln1_w", ctypes.c_void_p),
                ("ln2_w", ctypes.c_void_p), ("k_cache", ctypes.c_void_p), ("v_cache", ctypes.c_void_p),
                ("wf_qkv", ctypes.c_void_p), ("wf_gate", ctypes.c_void_p), ("wf_up", ctypes.c_void_p)]


class Pi05PrefixPlan(ctypes.Structure):
    _fields_ = [
        ("depth", ctypes.c_int), ("width", ctypes.c_int), ("mlp_dim", ctypes.c_int), ("n_q_heads", ctypes.c_int),
        ("n_kv_heads", ctypes.c_int), ("head_dim", ctypes.c_int), ("tokens", ctypes.c_int), ("kv_rows", ctypes.c_int),
        ("eps", ctypes.c_float), ("layers", ctypes.POINTER(Pi05PrefixLayer)), ("key_valid", ctypes.c_void_p),
        ("inv_freq", ctypes.c_void_p), ("rope_cos", ctypes.c_void_p), ("rope_sin", ctypes.c_void_p),
        ("h", ctypes.c_void_p), ("xn", ctypes.c_void_p), ("q", ctypes.c_void_p), ("attn", ctypes.c_void_p),
        ("act", ctypes.c_void_p), ("workspace", ctypes.c_void_p), ("workspace_bytes", ctypes.c_size_t),
        ("kv_only_last_layer", ctypes.c_int), ("row_stats", ctypes.c_void_p),
    ]


_lib.SIGNATURES.update({
    "pi05_prefix_forward": (ctypes.c_int, [ctypes.POINTER(Pi05PrefixPlan), ctypes.c_void_p]),
    "pi05_embed_tokens": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_int, ctypes.c_void_p, ctypes.c_int, ctypes.c_int,
                                         ctypes.c_float, ctypes.c_void_p, ctypes.c_int, ctypes.c_void_p,
                                         ctypes.c_size_t, ctypes.c_void_p]),
})


def _bind():
    L = _lib.lib()
    for name in ("pi05_prefix_forward", "pi05_embed_tokens"):
        res, args = _lib.SIGNATURES[name]
        f = getattr(L, name)
        f.restype = res
        f.argtypes = args
    return L


class PrefixWeights:
    """Device copies of the prefix LM: bf16 GEMM weights, fp32 RMSNorm weights."""

    def __init__(self, sd: Dict[str, torch.Tensor], shape: GemmaShape = GEMMA_2B, device="cuda",
                 prefix: str = LM_PREFIX):
        self.shape = shape
        self.device = torch.device(device)
        self.prefix = prefix
        bf = dict(dtype=torch.bfloat16, device=self.device)
        f32 = dict(dtype=torch.float32, device=self.device)
        self.layers: List[Dict[str, torch.Tensor]] = []
        for _ in range(shape.depth):
            self.layers.append({
                "w_qkv": torch.empty((shape.qkv_dim, shape.width), **bf),
                "w_o": torch.empty((shape.width, shape.q_dim), **bf),
                "w_gate": torch.empty((shape.mlp_dim, shape.width), **bf),
                "w_up": torch.empty((shape.mlp_dim, shape.width), **bf),
                "w_down": torch.empty((shape.width, shape.mlp_dim), **bf),
                "ln1": torch.empty((shape.width,), **f32),
                "ln2": torch.empty((shape.width,), **f32),
            })
        # Folded copies (folded RMSNorms, PI05_FOLD_NORM=0 to run the norm kernels
        # instead): q|k|v with (1 + ln1) and gate / up with (1 + ln2) folded into their
        # columns; 2.7 GB at Gemma-2B.
        self.fold = os.environ.get("PI05_FOLD_NORM", "1") != "0"
        if self.fold:
            for L in self.layers:
                L["wf_qkv"] = torch.empty_like(L["w_qkv"])
                L["wf_gate"] = torch.empty_like(L["w_gate"])
                L["wf_up"] = torch.empty_like(L["w_up"])
        self.load(sd)

    def load(self, sd: Dict[str, torch.Tensor]) -> None:
        """(Re)pack in place (``refresh_fused_prefix_qkv``, ``prefix_qkv_fused.py:220-246``)."""
        for i, L in enumerate(self.layers):
            p = f"{self.prefix}layers.{i}."
            L["w_qkv"].copy_(torch.cat([sd[p + "self_attn.q_proj.weight"], sd[p + "self_attn.k_proj.weight"],
                                        sd[p + "self_attn.v_proj.weight"]], 0))
            L["w_o"].copy_(sd[p + "self_attn.o_proj.weight"])
            L["w_gate"].copy_(sd[p + "mlp.gate_proj.weight"])
            L["w_up"].copy_(sd[p + "mlp.up_proj.weight"])
            L["w_down"].copy_(sd[p + "mlp.down_proj.weight"])
            L["ln1"].copy_(sd[p + "input_layernorm.weight"])
            L["ln2"].copy_(sd[p + "post_attention_layernorm.weight"])
        if self.fold:
            self.build_fold()

    def build_fold(self) -> None:
        """Fold each layer's RMSNorm weights into its q|k|v and gate/up copies, in place."""
        s = self.shape
        zero = torch.zeros(s.width, dtype=torch.float32, device=self.device)
        bias = torch.empty(max(s.qkv_dim, s.mlp_dim), dtype=torch.float32, device=self.device)
        for L in self.layers:
            abi.fold_adarms(L["w_qkv"], L["ln1"], zero, L["wf_qkv"], bias[: s.qkv_dim])
            abi.fold_adarms(L["w_gate"], L["ln2"], zero, L["wf_gate"], bias[: s.mlp_dim])
            abi.fold_adarms(L["w_up"], L["ln2"], zero, L["wf_up"], bias[: s.mlp_dim])


class PrefixRunner:
    """Static buffers + C plan for the prefix forward of one observation."""

    def __init__(self, weights: PrefixWeights, tokens: int, k_cache: Sequence[torch.Tensor],
                 v_cache: Sequence[torch.Tensor], kv_only_last_layer: bool = True):
        s = weights.shape
        dev = weights.device
        self.w = weights
        self.tokens = tokens
        bf = dict(dtype=torch.bfloat16, device=dev)
        self.kv_rows = k_cache[0].shape[-2]
        self.key_valid = torch.ones(tokens, dtype=torch.uint8, device=dev)
        self.inv_freq = rope_inv_freq(s.head_dim, s.rope_base, dev)
        self.rope_cos = torch.empty((tokens, s.head_dim), **bf)
        self.rope_sin = torch.empty((tokens, s.head_dim), **bf)
        self.h = torch.zeros((tokens, s.width), **bf)
        self.xn = torch.zeros((tokens, s.width), **bf)
        self.q = torch.zeros((tokens, s.num_heads, s.head_dim), **bf)
        self.attn = torch.zeros((tokens, s.q_dim), **bf)
        self.act = torch.zeros((tokens, s.mlp_dim), **bf)
        self.ws = ops.workspace(dev)
        self._layers = (Pi05PrefixLayer * s.depth)()
        for i, L in enumerate(weights.layers):
            wf = [L[k].data_ptr() if weights.fold else None for k in ("wf_qkv", "wf_gate", "wf_up")]
            self._layers[i] = Pi05PrefixLayer(L["w_qkv"].data_ptr(), L["w_o"].data_ptr(), L["w_gate"].data_ptr(),
                                              L["w_up"].data_ptr(), L["w_down"].data_ptr(), L["ln1"].data_ptr(),
                                              L["ln2"].data_ptr(), k_cache[i].data_ptr(), v_cache[i].data_ptr(),
                                              *wf)
        # per-64-column sums of squares of h for the folded norms
        self.row_stats = torch.zeros((s.width // 64, tokens), dtype=torch.float32, device=dev)
        self.plan = Pi05PrefixPlan(
            depth=s.depth, width=s.width, mlp_dim=s.mlp_dim, n_q_heads=s.num_heads, n_kv_heads=s.num_kv_heads,
            head_dim=s.head_dim, tokens=tokens, kv_rows=self.kv_rows, eps=s.rms_eps,
            layers=ctypes.cast(self._layers, ctypes.POINTER(Pi05PrefixLayer)), key_valid=self.key_valid.data_ptr(),
            inv_freq=self.inv_freq.data_ptr(), rope_cos=self.rope_cos.data_ptr(), rope_sin=self.rope_sin.data_ptr(),
            h=self.h.data_ptr(), xn=self.xn.data_ptr(), q=self.q.data_ptr(), attn=self.attn.data_ptr(),
            act=self.act.data_ptr(), workspace=self.ws.data_ptr(), workspace_bytes=self.ws.numel(),
            kv_only_last_layer=1 if kv_only_last_layer else 0,
            row_stats=self.row_stats.data_ptr() if weights.fold else None)

    def target(self, k_cache: Sequence[torch.Tensor], v_cache: Sequence[torch.Tensor],
               key_valid: Optional[torch.Tensor] = None) -> None:
        """Point the plan at other KV caches ``[hkv, kv_rows, d]`` per layer (e.g.
        observation b's views of a batched denoise runner) and, optionally, another
        key mask (its first ``tokens`` entries are read).  The C call reads the plan
        when it is enqueued, so each enqueue (and a graph captured from it) keeps
        the targets it was enqueued with."""
        for i in range(len(self._layers)):
            self._layers[i].k_cache = k_cache[i].data_ptr()
            self._layers[i].v_cache = v_cache[i].data_ptr()
        self.plan.key_valid = (self.key_valid if key_valid is None else key_valid).data_ptr()

    def enqueue(self, stream: int) -> None:
        _bind()
        _lib.call("pi05_prefix_forward", ctypes.byref(self.plan), stream)

    def run(self, embs: torch.Tensor, valid: torch.Tensor) -> None:
        """Prefix forward over ``embs`` [P, width] with pad mask ``valid`` [P]."""
        self.h.copy_(embs.reshape(self.tokens, -1))
        self.key_valid.copy_(valid.reshape(-1).to(torch.uint8))
        self.enqueue(abi.stream_of(self.h.device))


def embed_tokens(table: torch.Tensor, ids: torch.Tensor, out: torch.Tensor, scale: float, ws: torch.Tensor,
                 stream: int) -> None:
    _bind()
    n = ids.numel()
    _lib.call("pi05_embed_tokens", table.data_ptr(), table.shape[0], ids.data_ptr(), n, table.shape[1], scale,
              out.data_ptr(), out.stride(0), ws.data_ptr(), ws.numel(), stream)
