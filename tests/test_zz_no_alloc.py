"""pi05_gate_up_geglu_noalloc: the GeGLU GEMM for hosts that may not allocate.

A robot control loop that forbids allocation while it runs, or a plugin whose
host framework owns all device memory, cannot pass the workspace that
pi05_gate_up_geglu needs.  The no-allocation entry point keeps its scratch in a
fixed array inside the library.  This test calls it through the C ABI twice in a
row (the second call reuses the scratch the first one left behind) and checks
each result against the workspace entry point, with the tolerance of the other
GEMM tests.  The file is named so that pytest collects it last.
"""

import ctypes

import pytest
import torch

from pi05_infer import _lib, ops

pytestmark = pytest.mark.gpu


def _close(got, ref, rtol=1.6e-2, atol=2e-3):
    err = (got.float() - ref.float()).abs()
    bad = (err > atol + rtol * ref.float().abs()).sum().item()
    assert bad == 0, f"{bad} mismatches, max err {err.max().item():.3e}"


def test_noalloc_geglu_matches_workspace_entry_point():
    L = _lib.lib()
    f = L.pi05_gate_up_geglu_noalloc
    g = torch.Generator(device="cuda").manual_seed(11)
    m, n, k = 50, 4096, 1024
    x = torch.randn(m, k, device="cuda", generator=g).bfloat16()
    wg = (torch.randn(n, k, device="cuda", generator=g) * 0.02).bfloat16()
    wu = (torch.randn(n, k, device="cuda", generator=g) * 0.02).bfloat16()
    ref = ops.geglu(x, wg, wu)
    stream = torch.cuda.current_stream().cuda_stream
    for _ in range(2):
        out = torch.full_like(ref, float("nan"))
        rc = f(x.data_ptr(), wg.data_ptr(), wu.data_ptr(), out.data_ptr(), m, n, k, stream)
        assert rc == 0, _lib.last_error()
        torch.cuda.synchronize()
        _close(out, ref)
    # sizes beyond the built-in scratch are refused with a message, before any launch
    rc = f(x.data_ptr(), wg.data_ptr(), wu.data_ptr(), out.data_ptr(), 65, n, k, stream)
    assert rc == 2 and "exceeds the built-in scratch" in _lib.last_error()
