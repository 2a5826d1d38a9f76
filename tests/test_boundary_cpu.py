"""The drop-in boundary at the reference's own call site, on the CPU.

The reference's ``modeling_gemma.py:54-60`` imports ``rlinf_fused_denoise`` as
``_FUSED_OPS`` and keeps it only when ``HAVE_FUSED_DENOISE_OPS`` is true.  These
tests load the reference's unmodified ``modeling_gemma.py`` (installed under
``baseline/_ref``) with that import resolved to ``pi05_infer.ops`` and check that
the module is kept, that it exports the reference module's public names, and that
on CPU tensors its dispatchers decline (``None``) so the reference's eager path
runs and gives exactly the eager result.
"""

import pytest
import torch

from conftest import load_ref_loader

from pi05_infer import ops, synthetic
from pi05_infer.config import GemmaShape

import refglue

REF_PUBLIC = ["HAVE_FUSED_DENOISE_OPS", "fuse_geglu_enabled", "fuse_qkv_rope_enabled", "fused_gate_up_geglu",
              "fused_qkv_rope_kv"]


def test_ops_exports_reference_public_names():
    assert sorted(ops.__all__) == sorted(REF_PUBLIC)
    for n in REF_PUBLIC:
        assert hasattr(ops, n), n
    # the library is built in-tree, so the flag is true here as on the GPU box
    assert ops.HAVE_FUSED_DENOISE_OPS is True
    assert ops.fuse_geglu_enabled() and ops.fuse_qkv_rope_enabled()


def test_kill_switches(monkeypatch):
    monkeypatch.setenv("RLINF_FUSE_GEGLU", "0")
    assert not ops.fuse_geglu_enabled()
    monkeypatch.delenv("RLINF_FUSE_GEGLU")
    monkeypatch.setenv("RLINF_FUSE_SWIGLU", "0")  # legacy alias
    assert not ops.fuse_geglu_enabled()
    monkeypatch.setenv("RLINF_FUSE_QKV_ROPE", "0")
    assert not ops.fuse_qkv_rope_enabled()


def test_dispatchers_decline_cpu_tensors():
    x = torch.randn(1, 50, 1024, dtype=torch.bfloat16)
    w = torch.randn(4096, 1024, dtype=torch.bfloat16)
    assert ops.fused_gate_up_geglu(x, w, w) is None
    wq = torch.randn(2560, 1024, dtype=torch.bfloat16)
    cos = torch.randn(1, 50, 256, dtype=torch.bfloat16)
    kc = torch.zeros(1, 1, 100, 256, dtype=torch.bfloat16)
    assert ops.fused_qkv_rope_kv(x, wq, cos, cos, kc, kc.clone(), 50, 8, 1, 256) is None


def test_reference_keeps_substituted_module():
    rl = load_ref_loader()
    if rl is None:
        pytest.skip("reference not installed under baseline/_ref")
    mod = rl.load_modeling_gemma(fused_ops=ops, tag="cpu")
    assert mod._FUSED_OPS is ops


def test_reference_eager_path_unchanged_on_cpu(monkeypatch):
    """With pi05_infer.ops substituted, the reference expert on CPU tensors gives
    exactly its eager result (the dispatchers return None, as the reference's own
    do off-GPU), and both dispatchers were consulted."""
    rl = load_ref_loader()
    if rl is None:
        pytest.skip("reference not installed under baseline/_ref")
    calls = {"geglu": 0, "qkv": 0}
    real_g, real_q = ops.fused_gate_up_geglu, ops.fused_qkv_rope_kv

    def g(*a, **k):
        calls["geglu"] += 1
        return real_g(*a, **k)

    def q(*a, **k):
        calls["qkv"] += 1
        return real_q(*a, **k)

    monkeypatch.setattr(ops, "fused_gate_up_geglu", g)
    monkeypatch.setattr(ops, "fused_qkv_rope_kv", q)
    sub = rl.load_modeling_gemma(fused_ops=ops, tag="cpu2")
    eager = rl.load_modeling_gemma(fused_ops=None, tag="cpu2")
    assert eager._FUSED_OPS is None
    depth, p = 1, 24
    shape = GemmaShape(width=1024, depth=depth, mlp_dim=4096, num_heads=8, num_kv_heads=1, head_dim=256)
    w = synthetic.make_expert_weights(0, shape)
    kv = synthetic.make_prefix_kv(1, depth, p)
    x = synthetic.make_noise(2)
    pad = torch.ones(1, p, dtype=torch.bool)
    with torch.no_grad():
        m1 = refglue.build_expert(sub, rl, w, shape, depth, torch.float32)
        v1 = refglue.velocity(m1, w, x, 1.0, kv, pad, torch.float32, static_kv=True)
        m2 = refglue.build_expert(eager, rl, w, shape, depth, torch.float32)
        v2 = refglue.velocity(m2, w, x, 1.0, kv, pad, torch.float32, static_kv=True)
    assert calls["geglu"] == depth and calls["qkv"] == depth
    assert torch.equal(v1, v2)
