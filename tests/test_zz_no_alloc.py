"""pi05_gate_up_geglu_noalloc: the GeGLU GEMM for hosts that may not allocate.

A robot control loop that forbids allocation while it runs, or a plugin whose
host framework owns all device memory, cannot pass the workspace that
pi05_gate_up_geglu needs.  The no-allocation entry point keeps its scratch in a
fixed array inside the library.  This test calls it through the C ABI twice in a
row per shape (the second call reuses the scratch the first one left behind) and
checks each result against an fp32 torch GeGLU on the same bf16 operands, with
the tolerance of the other GEMM tests.  The shapes reach each branch of the
split choice: two K splits that exactly fill the 4 MiB of partials (n=4096), a
split count reduced to one because the partials would not fit (n=4736: 74 tiles
x 2 splits = 4.6 MiB), and the size limits m=64 / n=16384, plus m=1.  After the
calls the sticky device status word reads zero.  The file is named so that
pytest collects it last.
"""

import ctypes

import pytest
import torch

from pi05_infer import _lib

pytestmark = pytest.mark.gpu


def gelu_tanh(x):
    return 0.5 * x * (1.0 + torch.tanh(0.7978845608028654 * (x + 0.044715 * x * x * x)))


def _close(got, ref, rtol=1.6e-2, atol=2e-3):
    err = (got.float() - ref).abs()
    bad = (err > atol + rtol * ref.abs()).sum().item()
    assert bad == 0, f"{bad} mismatches, max err {err.max().item():.3e}"


def _status(stream):
    v = ctypes.c_int(-1)
    rc = _lib.lib().pi05_gate_up_geglu_noalloc_status(ctypes.byref(v), stream)
    return rc, v.value


@pytest.mark.parametrize("m,n,k", [(50, 4096, 1024), (50, 4736, 1024), (64, 16384, 1024), (1, 4096, 1024)],
                         ids=["two-splits-fit", "splits-reduced", "limits", "m1"])
def test_noalloc_geglu_matches_fp32(m, n, k):
    f = _lib.lib().pi05_gate_up_geglu_noalloc
    g = torch.Generator(device="cuda").manual_seed(11)
    x = torch.randn(m, k, device="cuda", generator=g).bfloat16()
    wg = (torch.randn(n, k, device="cuda", generator=g) * 0.02).bfloat16()
    wu = (torch.randn(n, k, device="cuda", generator=g) * 0.02).bfloat16()
    gg = (x.float() @ wg.float().t()).bfloat16().float()
    ref = gelu_tanh(gg) * (x.float() @ wu.float().t())
    stream = torch.cuda.current_stream().cuda_stream
    for _ in range(2):
        out = torch.full((m, n), float("nan"), dtype=torch.bfloat16, device="cuda")
        rc = f(x.data_ptr(), wg.data_ptr(), wu.data_ptr(), out.data_ptr(), m, n, k, stream)
        assert rc == 0, _lib.last_error()
        torch.cuda.synchronize()
        _close(out, ref)
    assert _status(stream) == (0, 0)


def test_noalloc_geglu_limits():
    f = _lib.lib().pi05_gate_up_geglu_noalloc
    x = torch.zeros(65, 1024, dtype=torch.bfloat16, device="cuda")
    w = torch.zeros(16448, 1024, dtype=torch.bfloat16, device="cuda")
    out = torch.zeros(65, 16448, dtype=torch.bfloat16, device="cuda")
    stream = torch.cuda.current_stream().cuda_stream
    # sizes beyond the built-in scratch are refused with a message, before any launch
    for m, n, k in [(65, 4096, 1024), (50, 16448, 1024), (50, 4096, 16448)]:
        rc = f(x.data_ptr(), w.data_ptr(), w.data_ptr(), out.data_ptr(), m, n, k, stream)
        assert rc == 2 and "exceeds the built-in scratch" in _lib.last_error(), (m, n, k)
    rc = f(x.data_ptr(), w.data_ptr(), w.data_ptr(), out.data_ptr(), 50, 4100, 1024, stream)
    assert rc == 2  # n % 64
    assert _status(stream) == (0, 0)
