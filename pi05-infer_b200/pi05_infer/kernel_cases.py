"""Single-kernel workloads at the shapes of the pi0.5 hot path, for profilers.

``python pi05-infer_b200/pi05_infer/kernel_cases.py CASE [--reps N]`` launches one
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
  mqa_attention  denoise attention: 50 x 8 query rows over a 1018-key cache, d=256
  prefix_attention  prefix-LM attention: 968 x 8 query rows over 968 keys, d=256
                 (tcgen05 kernel, split-KV partials + combine)
"""

import argparse
import math
import os
import sys

import torch

if __package__ in (None, ""):
    sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))

from pi05_infer import abi, ops  # noqa: E402

CASES = ("denoise_geglu", "denoise_down", "prefix_geglu", "prefix_down", "prefix_qkv", "siglip_fc1",
         "mqa_attention", "prefix_attention")


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
    raise ValueError(case)


def main(argv=None):
    ap = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    ap.add_argument("case", choices=CASES)
    ap.add_argument("--reps", type=int, default=3)
    args = ap.parse_args(argv)
    f, nbytes, flops = build(args.case)
    for _ in range(args.reps):
        f()
    torch.cuda.synchronize()
    status = ops.read_device_status()
    print(f"{args.case}: {args.reps} launches, bytes/launch {nbytes}, flop/launch {flops}, status {status}")
    return 0 if status == 0 else 1


if __name__ == "__main__":
    sys.exit(main())
