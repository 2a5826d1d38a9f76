"""Single-kernel workloads at the shapes of the pi0.5 hot path, for profilers.

``python kernel_cases.py CASE [--reps N]`` launches one
kernel family ``N`` times on ``cuda:0`` with seeded synthetic operands, so that an
``ncu`` capture (``-k`` on the kernel, ``-c`` a few launches) sees exactly the
launches of interest on a small device footprint:

  denoise_geglu  small-token GEMM + GeGLU, M=50, N=2x4096, K=1024 (Gemma-300M MLP),
                 one launch per layer over 18 layers of weights (302 MB > L2)
  denoise_down   small-token GEMM + gated residual, M=50, N=1024, K=4096
  prefix_geglu   many-token GEMM + GeGLU, M=968, N=2x16384, K=2048 (Gemma-2B MLP)
  prefix_down    many-token GEMM + residual, M=968, N=2048, K=16384
  prefix_qkv     many-token GEMM + RoPE into the KV cache, M=968, N=10x256, K=2048
  siglip_fc1     many-token GEMM + bias + GELU, M=768, N=4304, K=1152
  siglip_out     many-token GEMM + residual, M=768, N=1152, K=1152 (SigLIP out-proj)
  mqa_attention  denoise attention: 50 x 8 query rows over a 1018-key cache, d=256
  prefix_attention  prefix-LM attention: 968 x 8 query rows over 968 keys, d=256
                 (tcgen05 kernel, two key splits merged in-kernel)
  siglip_attention  SigLIP attention: 3 views x 16 heads, 256 x 256, head_dim 72,
                 one launch per layer over 27 layers of q|k|v (143 MB > L2)

``python kernel_cases.py duel`` runs the same-box comparison with the reference's
own Triton kernels (``_geglu_mm_kernel`` and ``_qkv_rope_kernel`` of
``pi05_infer/gemma/rlinf_fused_denoise.py``, loaded unmodified from
``baseline/_ref``) and prints one JSON line; ``bench.py`` adds the same record to
its output.
"""

import argparse
import math
import os
import sys

import torch

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(HERE, "pi05-infer_b200"))

from pi05_infer import abi, ops  # noqa: E402

CASES = ("denoise_geglu", "denoise_down", "prefix_geglu", "prefix_down", "prefix_qkv", "siglip_fc1", "siglip_out",
         "mqa_attention", "prefix_attention", "siglip_attention")


def _bf(t):
    return t.to(torch.bfloat16)


def build(case: str, dev="cuda"):
    """Operands for ``case``; returns (launch callable, algorithmic bytes, flops) per launch."""
    g = torch.Generator(device=dev).manual_seed(0)

    def rnd(*shape, s=1.0):
        return _bf(torch.randn(*shape, device=dev, generator=g) * s)

    if case == "denoise_geglu":
        x = rnd(50, 1024)
        ws = [(rnd(4096, 1024, s=0.02), rnd(4096, 1024, s=0.02)) for _ in range(18)]
        out = torch.empty(50, 4096, dtype=torch.bfloat16, device=dev)
        it = iter(range(1 << 60))

        def f():
            wg, wu = ws[next(it) % 18]
            ops.geglu(x, wg, wu, out=out)

        return f, 2 * 4096 * 1024 * 2 + 50 * 1024 * 2 + 50 * 4096 * 2, 2 * 50 * 8192 * 1024
    if case == "denoise_down":
        x = rnd(50, 4096)
        ws = [rnd(1024, 4096, s=0.02) for _ in range(18)]
        h = rnd(50, 1024)
        gate = torch.randn(1024, device=dev, generator=g)
        it = iter(range(1 << 60))

        def f():
            ops.linear_gated_residual(x, ws[next(it) % 18], h, gate, out=h)

        return f, 1024 * 4096 * 2 + 50 * 4096 * 2 + 2 * 50 * 1024 * 2, 2 * 50 * 1024 * 4096
    if case == "prefix_geglu":
        x = rnd(968, 2048)
        wg, wu = rnd(16384, 2048, s=0.02), rnd(16384, 2048, s=0.02)
        out = torch.empty(968, 16384, dtype=torch.bfloat16, device=dev)
        return (lambda: ops.geglu(x, wg, wu, out=out)), None, 2 * 968 * 32768 * 2048
    if case == "prefix_down":
        x = rnd(968, 16384)
        w = rnd(2048, 16384, s=0.02)
        h = rnd(968, 2048)
        return (lambda: ops.linear_gated_residual(x, w, h, None, out=h)), None, 2 * 968 * 2048 * 16384
    if case == "prefix_qkv":
        m, d = 968, 256
        x = rnd(m, 2048)
        w = rnd(10 * d, 2048, s=0.02)
        pos = torch.arange(m, device=dev).float()
        inv = 1.0 / (10000 ** (torch.arange(0, d, 2, device=dev).float() / d))
        emb = torch.cat([pos[:, None] * inv[None]] * 2, -1)
        cos, sin = _bf(emb.cos()), _bf(emb.sin())
        kc = torch.zeros(1, m + 50, d, dtype=torch.bfloat16, device=dev)
        vc = torch.zeros_like(kc)
        q = torch.empty(m, 8, d, dtype=torch.bfloat16, device=dev)
        return (lambda: ops.qkv_rope(x, w, cos, sin, q, kc, vc, 0, 8, 1, d)), None, 2 * m * 2560 * 2048
    if case == "siglip_fc1":
        x = rnd(768, 1152)
        w = rnd(4352, 1152, s=0.02)
        out = torch.empty(768, 4352, dtype=torch.bfloat16, device=dev)
        return (lambda: ops.linear(x, w, out=out)), None, 2 * 768 * 4352 * 1152
    if case == "siglip_out":
        x = rnd(768, 1152)
        ws = [rnd(1152, 1152, s=0.02) for _ in range(27)]
        h = rnd(768, 1152)
        it = iter(range(1 << 60))

        def f():
            ops.linear_gated_residual(x, ws[next(it) % 27], h, None, out=h)

        return f, None, 2 * 768 * 1152 * 1152
    if case == "prefix_attention":
        p, d = 968, 256
        q = rnd(p, 8, d)
        k = rnd(p, d)
        v = rnd(p, d)
        valid = torch.ones(p, dtype=torch.uint8, device=dev)
        out = torch.empty(p, 8 * d, dtype=torch.bfloat16, device=dev)
        wsp = ops.workspace(torch.device(dev))

        def f():
            abi.attention(q, k, v, valid, out, 1.0 / math.sqrt(d), 0, wsp)

        return f, p * d * 2 * 2 + 2 * p * 8 * d * 2, 4 * p * 8 * p * d
    if case == "mqa_attention":
        p, s, d = 968, 50, 256
        q = rnd(s, 8, d)
        k = rnd(p + s, d)
        v = rnd(p + s, d)
        valid = torch.ones(p + s, dtype=torch.uint8, device=dev)
        out = torch.empty(s, 8 * d, dtype=torch.bfloat16, device=dev)
        wsp = ops.workspace(torch.device(dev))

        def f():
            abi.attention(q, k, v, valid, out, 1.0 / math.sqrt(d), 0, wsp)

        return f, (p + s) * d * 2 * 2 + 2 * s * 8 * d * 2, 4 * s * 8 * (p + s) * d
    if case == "siglip_attention":
        import ctypes

        from pi05_infer import vision

        views, seq, width, heads, hd = 3, 256, 1152, 16, 72
        qkvs = [rnd(views * seq, 3 * width) for _ in range(27)]
        out = torch.empty(views * seq, width, dtype=torch.bfloat16, device=dev)
        fn = vision._bind().pi05_siglip_attention
        it = iter(range(1 << 60))

        def f():
            rc = fn(ctypes.c_void_p(qkvs[next(it) % 27].data_ptr()), views, seq, width, heads, hd,
                    ctypes.c_void_p(out.data_ptr()), ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
            if rc != 0:
                raise RuntimeError(f"pi05_siglip_attention: {rc}")

        return f, views * seq * 4 * width * 2, 4 * views * heads * seq * seq * hd
    raise ValueError(case)


def _graph_us(launches, reps: int) -> float:
    """Mean µs per launch of ``launches`` (one callable per layer), captured once in a
    CUDA graph and replayed ``reps`` times, timed with CUDA events on the replay stream."""
    for f in launches:
        f()
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        for f in launches:
            f()
    for _ in range(3):
        g.replay()
    torch.cuda.synchronize()
    st = torch.cuda.current_stream()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(st)
    for _ in range(reps):
        g.replay()
    e1.record(st)
    torch.cuda.synchronize()
    del g
    return e0.elapsed_time(e1) * 1e3 / (reps * len(launches))


def kernel_duel(reps: int = 20, dev: str = "cuda") -> dict:
    """The reference's Triton denoise kernels against this library's, same box, same
    timing: M=50 tokens, 18 layers of Gemma-300M weights (302 MB of gate/up and
    94 MB of q|k|v, both larger than L2), one launch per layer inside a CUDA graph.

    Loading the reference module registers its ``torch.ops.pi05_infer.*`` over this
    repository's registrations, so this runs last in its process; this library's
    kernels are called through ``ops.geglu`` / ``ops.qkv_rope`` (the C ABI), the
    reference's through the Python bodies of its custom ops (its Triton launches)."""
    import importlib.util

    spec = importlib.util.spec_from_file_location("pi05_ref_loader", os.path.join(HERE, "baseline", "ref_loader.py"))
    rl = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(rl)
    if not rl.available():
        return {"unavailable": "reference not installed under baseline/_ref"}
    refk = rl.load_fused_denoise()
    if not refk.HAVE_FUSED_DENOISE_OPS:
        return {"unavailable": "the reference's Triton kernels did not import"}
    ref_geglu = getattr(refk.gate_up_geglu, "_init_fn", refk.gate_up_geglu)
    ref_qkv = getattr(refk.qkv_rope_kv, "_init_fn", refk.qkv_rope_kv)
    g = torch.Generator(device=dev).manual_seed(0)

    def rnd(*shape, s=1.0):
        return _bf(torch.randn(*shape, device=dev, generator=g) * s)

    L, m, k, n, d, p = 18, 50, 1024, 4096, 256, 968
    x = rnd(1, m, k)
    wg = [rnd(n, k, s=0.02) for _ in range(L)]
    wu = [rnd(n, k, s=0.02) for _ in range(L)]
    wq = [rnd(10 * d, k, s=0.02) for _ in range(L)]
    pos = torch.arange(p, p + m, device=dev).float()
    inv = 1.0 / (10000 ** (torch.arange(0, d, 2, device=dev).float() / d))
    emb = torch.cat([pos[:, None] * inv[None]] * 2, -1)
    cos, sin = _bf(emb.cos())[None], _bf(emb.sin())[None]
    kc = [torch.zeros(1, 1, p + m, d, dtype=torch.bfloat16, device=dev) for _ in range(L)]
    vc = [torch.zeros(1, 1, p + m, d, dtype=torch.bfloat16, device=dev) for _ in range(L)]
    q_mine = torch.empty(m, 8, d, dtype=torch.bfloat16, device=dev)
    act_mine = torch.empty(m, n, dtype=torch.bfloat16, device=dev)
    outs = {}

    def rg(l):
        return lambda: outs.__setitem__("g", ref_geglu(x, wg[l], wu[l]))

    def rq(l):
        return lambda: outs.__setitem__("q", ref_qkv(x, wq[l], cos, sin, kc[l], vc[l], p, 8, 1, d))

    def mg(l):
        return lambda: ops.geglu(x[0], wg[l], wu[l], out=act_mine)

    def mq(l):
        return lambda: ops.qkv_rope(x[0], wq[l], cos[0], sin[0], q_mine, kc[l][0], vc[l][0], p, 8, 1, d)

    res = {}
    geglu_bytes = 2 * n * k * 2 + m * k * 2 + m * n * 2
    qkv_bytes = 10 * d * k * 2 + m * k * 2 + m * 8 * d * 2 + 2 * m * d * 2
    for name, nbytes, ref_f, mine_f in (("gate_up_geglu", geglu_bytes, rg, mg), ("qkv_rope_kv", qkv_bytes, rq, mq)):
        us_ref = _graph_us([ref_f(l) for l in range(L)], reps)
        us_mine = _graph_us([mine_f(l) for l in range(L)], reps)
        res[name] = {"ref_us": us_ref, "ours_us": us_mine, "speedup": us_ref / us_mine,
                     "ref_gbs": nbytes / (us_ref * 1e-6) / 1e9, "ours_gbs": nbytes / (us_mine * 1e-6) / 1e9,
                     "bytes_per_launch": nbytes}
    # both implementations compute the same thing (last layer's operands)
    ref_geglu(x, wg[-1], wu[-1])
    a_ref = ref_geglu(x, wg[-1], wu[-1])[0].float()
    ops.geglu(x[0], wg[-1], wu[-1], out=act_mine)
    q_ref = ref_qkv(x, wq[-1], cos, sin, kc[-1], vc[-1], p, 8, 1, d)[0].float()
    ops.qkv_rope(x[0], wq[-1], cos[0], sin[0], q_mine, kc[-1][0], vc[-1][0], p, 8, 1, d)
    torch.cuda.synchronize()
    res["gate_up_geglu"]["max_abs_diff"] = (act_mine.float() - a_ref).abs().max().item()
    res["qkv_rope_kv"]["max_abs_diff"] = (q_mine.float() - q_ref).abs().max().item()
    res["shapes"] = "M=50, K=1024; gate/up N=2x4096; q|k|v N=2560 with RoPE and KV rows 968..1017; 18 layers"
    res["status"] = ops.read_device_status()
    return res


def main(argv=None):
    ap = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    ap.add_argument("case", choices=CASES + ("duel",))
    ap.add_argument("--reps", type=int, default=3)
    args = ap.parse_args(argv)
    if args.case == "duel":
        import json

        res = kernel_duel(reps=max(args.reps, 5))
        print(json.dumps(res))
        return 0 if res.get("status", 0) == 0 else 1
    f, nbytes, flops = build(args.case)
    for _ in range(args.reps):
        f()
    torch.cuda.synchronize()
    status = ops.read_device_status()
    print(f"{args.case}: {args.reps} launches, bytes/launch {nbytes}, flop/launch {flops}, status {status}")
    return 0 if status == 0 else 1


if __name__ == "__main__":
    sys.exit(main())
