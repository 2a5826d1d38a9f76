"""SigLIP So400m/14 + PaliGemma projector on the C ABI (``embed_image``).

Dtype policy follows the reference (``gemma_pytorch.py:84-104``): GEMM weights,
biases and LayerNorm parameters are the bf16 copies; the patch-embedding conv
and the position embedding stay fp32 in the reference -- here the conv runs as a
bf16 GEMM over im2col patches (fp32 accumulation) with the fp32 bias and
position embedding added before the single rounding.
"""

from __future__ import annotations

import ctypes
import os
from typing import Dict, List

import torch

from . import _lib, abi, ops
from .config import SIGLIP_SO400M, SiglipShape
from .synthetic import PROJECTOR_PREFIX, VISION_PREFIX

_P = ctypes.c_void_p


class Pi05SiglipLayer(ctypes.Structure):
    _fields_ = [(n, _P) for n in ("w_qkv", "b_qkv", "w_o", "b_o", "w_fc1", "b_fc1", "w_fc2", "b_fc2",
                                  "ln1_w", "ln1_b", "ln2_w", "ln2_b",
                                  "wf_qkv", "bf_qkv", "cs_qkv", "wf_fc1", "bf_fc1", "cs_fc1")]


class Pi05SiglipPlan(ctypes.Structure):
    _fields_ = [(n, ctypes.c_int) for n in ("depth", "width", "mlp_dim", "n_heads", "head_dim", "patch",
                                            "image_size", "num_views", "proj_dim")] + [
        ("eps", ctypes.c_float), ("layers", ctypes.POINTER(Pi05SiglipLayer)), ("w_patch", _P), ("b_patch", _P),
        ("pos_emb", _P), ("k_pad", ctypes.c_int), ("post_ln_w", _P), ("post_ln_b", _P), ("w_proj", _P),
        ("b_proj", _P), ("images", _P), ("cols", _P), ("h", _P), ("xn", _P), ("qkv", _P), ("attn", _P),
        ("act", _P), ("out", _P), ("ldo", ctypes.c_int), ("workspace", _P), ("workspace_bytes", ctypes.c_size_t),
        ("wf_proj", _P), ("bf_proj", _P), ("cs_proj", _P), ("row_stats", _P),
    ]


_lib.SIGNATURES.update({
    "pi05_siglip_forward": (ctypes.c_int, [ctypes.POINTER(Pi05SiglipPlan), _P]),
    "pi05_layer_norm": (ctypes.c_int, [_P, _P, _P, _P, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_float, _P]),
    "pi05_siglip_attention": (ctypes.c_int, [_P, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int,
                                             ctypes.c_int, _P, _P]),
})


def _bind():
    L = _lib.lib()
    for name in ("pi05_siglip_forward", "pi05_layer_norm", "pi05_siglip_attention"):
        res, args = _lib.SIGNATURES[name]
        f = getattr(L, name)
        f.restype = res
        f.argtypes = args
    return L


def _bf16_as_f32(t: torch.Tensor, device) -> torch.Tensor:
    """The reference holds these parameters in bf16; the kernels read them as fp32."""
    return t.to(device=device, dtype=torch.bfloat16).float().contiguous()


class SiglipWeights:
    def __init__(self, sd: Dict[str, torch.Tensor], shape: SiglipShape = SIGLIP_SO400M, device="cuda",
                 prefix: str = VISION_PREFIX, proj_prefix: str = PROJECTOR_PREFIX):
        self.shape = shape
        self.device = torch.device(device)
        self.prefix = prefix
        self.proj_prefix = proj_prefix
        kk = 3 * shape.patch * shape.patch
        self.k_pad = (kk + 63) // 64 * 64
        bf = dict(dtype=torch.bfloat16, device=self.device)
        f32 = dict(dtype=torch.float32, device=self.device)
        w = shape.width
        self.w_patch = torch.zeros((w, self.k_pad), **bf)
        self.b_patch = torch.empty((w,), **f32)
        self.pos = torch.empty((shape.num_patches, w), **f32)
        self.layers: List[Dict[str, torch.Tensor]] = []
        for _ in range(shape.depth):
            self.layers.append({
                "w_qkv": torch.empty((3 * w, w), **bf), "b_qkv": torch.empty((3 * w,), **f32),
                "w_o": torch.empty((w, w), **bf), "b_o": torch.empty((w,), **f32),
                "w_fc1": torch.empty((shape.mlp_dim, w), **bf), "b_fc1": torch.empty((shape.mlp_dim,), **f32),
                "w_fc2": torch.empty((w, shape.mlp_dim), **bf), "b_fc2": torch.empty((w,), **f32),
                "ln1_w": torch.empty((w,), **f32), "ln1_b": torch.empty((w,), **f32),
                "ln2_w": torch.empty((w,), **f32), "ln2_b": torch.empty((w,), **f32),
            })
        self.post_w = torch.empty((w,), **f32)
        self.post_b = torch.empty((w,), **f32)
        self.w_proj = torch.empty((shape.proj_dim, w), **bf)
        self.b_proj = torch.empty((shape.proj_dim,), **f32)
        # Folded LayerNorms (PI05_FOLD_NORM=0 runs the LayerNorm kernels instead):
        # q|k|v, fc1 and the projector with the preceding LayerNorm's gamma folded
        # into their columns, biases b + W . beta, and column sums of the folded
        # weights (the mean term of the normalisation).
        self.fold = os.environ.get("PI05_FOLD_NORM", "1") != "0"
        if self.fold:
            for L in self.layers:
                for n, rows in (("qkv", 3 * w), ("fc1", shape.mlp_dim)):
                    L["wf_" + n] = torch.empty((rows, w), **bf)
                    L["bf_" + n] = torch.empty((rows,), **f32)
                    L["cs_" + n] = torch.empty((rows,), **f32)
            self.wf_proj = torch.empty_like(self.w_proj)
            self.bf_proj = torch.empty_like(self.b_proj)
            self.cs_proj = torch.empty_like(self.b_proj)
        self.load(sd)

    def load(self, sd: Dict[str, torch.Tensor]) -> None:
        p, dev = self.prefix, self.device
        kk = 3 * self.shape.patch * self.shape.patch
        self.w_patch[:, :kk].copy_(sd[p + "embeddings.patch_embedding.weight"].reshape(self.shape.width, kk))
        self.b_patch.copy_(sd[p + "embeddings.patch_embedding.bias"])
        self.pos.copy_(sd[p + "embeddings.position_embedding.weight"])
        for i, L in enumerate(self.layers):
            q = f"{p}encoder.layers.{i}."
            L["w_qkv"].copy_(torch.cat([sd[q + f"self_attn.{n}_proj.weight"] for n in "qkv"], 0))
            L["b_qkv"].copy_(_bf16_as_f32(torch.cat([sd[q + f"self_attn.{n}_proj.bias"] for n in "qkv"], 0), dev))
            L["w_o"].copy_(sd[q + "self_attn.out_proj.weight"])
            L["b_o"].copy_(_bf16_as_f32(sd[q + "self_attn.out_proj.bias"], dev))
            L["w_fc1"].copy_(sd[q + "mlp.fc1.weight"])
            L["b_fc1"].copy_(_bf16_as_f32(sd[q + "mlp.fc1.bias"], dev))
            L["w_fc2"].copy_(sd[q + "mlp.fc2.weight"])
            L["b_fc2"].copy_(_bf16_as_f32(sd[q + "mlp.fc2.bias"], dev))
            for n in ("ln1", "ln2"):
                idx = n[-1]
                L[n + "_w"].copy_(_bf16_as_f32(sd[q + f"layer_norm{idx}.weight"], dev))
                L[n + "_b"].copy_(_bf16_as_f32(sd[q + f"layer_norm{idx}.bias"], dev))
        self.post_w.copy_(_bf16_as_f32(sd[p + "post_layernorm.weight"], dev))
        self.post_b.copy_(_bf16_as_f32(sd[p + "post_layernorm.bias"], dev))
        self.w_proj.copy_(sd[self.proj_prefix + "weight"])
        self.b_proj.copy_(_bf16_as_f32(sd[self.proj_prefix + "bias"], dev))
        if self.fold:
            self.build_fold()

    def build_fold(self) -> None:
        """LayerNorm(x) = (x - mean) * rstd * gamma + beta, so
        W . LayerNorm(x) + b = rstd * (W' . x - mean * colsum(W')) + (b + W . beta)
        with W' = bf16(W * gamma); the column sums are taken of the rounded W', so
        the mean term cancels its rounding exactly.  Built in place."""
        w = self.shape.width
        ones = torch.ones(w, dtype=torch.float32, device=self.device)
        zeros = torch.zeros(w, dtype=torch.float32, device=self.device)

        def fold(wt, gamma, beta, b, wf, bf, cs):
            abi.fold_adarms(wt, gamma - 1.0, beta, wf, bf)  # wf = bf16(W * gamma), bf = W . beta
            bf.add_(b)
            scratch = torch.empty_like(wf)
            abi.fold_adarms(wf, zeros, ones, scratch, cs)  # cs = sum_k wf[n, k]

        for L in self.layers:
            fold(L["w_qkv"], L["ln1_w"], L["ln1_b"], L["b_qkv"], L["wf_qkv"], L["bf_qkv"], L["cs_qkv"])
            fold(L["w_fc1"], L["ln2_w"], L["ln2_b"], L["b_fc1"], L["wf_fc1"], L["bf_fc1"], L["cs_fc1"])
        fold(self.w_proj, self.post_w, self.post_b, self.b_proj, self.wf_proj, self.bf_proj, self.cs_proj)


class SiglipRunner:
    """Static buffers + plan for ``num_views`` images per call."""

    def __init__(self, weights: SiglipWeights, num_views: int):
        s = weights.shape
        dev = weights.device
        self.w = weights
        self.num_views = num_views
        t = num_views * s.num_patches
        bf = dict(dtype=torch.bfloat16, device=dev)
        self.images = torch.zeros((num_views, 3, s.image_size, s.image_size), dtype=torch.float32, device=dev)
        self.cols = torch.zeros((t, weights.k_pad), **bf)
        self.h = torch.zeros((t, s.width), **bf)
        self.xn = torch.zeros((t, s.width), **bf)
        self.qkv = torch.zeros((t, 3 * s.width), **bf)
        self.attn = torch.zeros((t, s.width), **bf)
        self.act = torch.zeros((t, s.mlp_dim), **bf)
        self.ws = ops.workspace(dev)
        self._layers = (Pi05SiglipLayer * s.depth)()
        fk = ("wf_qkv", "bf_qkv", "cs_qkv", "wf_fc1", "bf_fc1", "cs_fc1")
        for i, L in enumerate(weights.layers):
            self._layers[i] = Pi05SiglipLayer(*[L[k].data_ptr() for k in (
                "w_qkv", "b_qkv", "w_o", "b_o", "w_fc1", "b_fc1", "w_fc2", "b_fc2", "ln1_w", "ln1_b", "ln2_w", "ln2_b")],
                *[L[k].data_ptr() if weights.fold else None for k in fk])
        # per-64-column sums and sums of squares of h for the folded LayerNorms
        self.row_stats = torch.zeros((2, s.width // 64, t), dtype=torch.float32, device=dev)
        self.use_fold = weights.fold  # False: the LayerNorm kernels (tests)
        self.plan = None

    def _plan(self, images: torch.Tensor, out: torch.Tensor) -> Pi05SiglipPlan:
        s, w = self.w.shape, self.w
        return Pi05SiglipPlan(
            depth=s.depth, width=s.width, mlp_dim=s.mlp_dim, n_heads=s.num_heads, head_dim=s.head_dim,
            patch=s.patch, image_size=s.image_size, num_views=self.num_views, proj_dim=s.proj_dim, eps=s.ln_eps,
            layers=ctypes.cast(self._layers, ctypes.POINTER(Pi05SiglipLayer)), w_patch=w.w_patch.data_ptr(),
            b_patch=w.b_patch.data_ptr(), pos_emb=w.pos.data_ptr(), k_pad=w.k_pad, post_ln_w=w.post_w.data_ptr(),
            post_ln_b=w.post_b.data_ptr(), w_proj=w.w_proj.data_ptr(), b_proj=w.b_proj.data_ptr(),
            images=images.data_ptr(), cols=self.cols.data_ptr(), h=self.h.data_ptr(), xn=self.xn.data_ptr(),
            qkv=self.qkv.data_ptr(), attn=self.attn.data_ptr(), act=self.act.data_ptr(), out=out.data_ptr(),
            ldo=out.stride(0), workspace=self.ws.data_ptr(), workspace_bytes=self.ws.numel(),
            wf_proj=w.wf_proj.data_ptr() if w.fold else None, bf_proj=w.bf_proj.data_ptr() if w.fold else None,
            cs_proj=w.cs_proj.data_ptr() if w.fold else None,
            row_stats=self.row_stats.data_ptr() if (w.fold and self.use_fold) else None)

    def enqueue(self, images: torch.Tensor, out: torch.Tensor, stream: int) -> None:
        """images [views, 3, H, W] fp32 (device), out rows [views*patches, proj] (bf16, row pitch any)."""
        _bind()
        if images.data_ptr() != self.images.data_ptr():
            self.images.copy_(images)
        self._keep = self._plan(self.images, out)
        _lib.call("pi05_siglip_forward", ctypes.byref(self._keep), stream)

    def run(self, images: torch.Tensor, out: torch.Tensor) -> torch.Tensor:
        self.enqueue(images.to(self.images.device, torch.float32), out, abi.stream_of(self.images.device))
        return out
