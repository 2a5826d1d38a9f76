"""Device-side failure detection, exercised without a GPU fault.

Every wait in the library's kernels is bounded.  These tests make one run out on
purpose through the test hook ``pi05_debug_set_fault``: in the global-memory
split-K path, split 1 of the first output tile leaves out its partial and its
arrival, so the other split's arrival wait (a counter that nothing will raise)
gives up after 50 ms.  The kernel must then return normally with the timeout bit
set in the device status word, the host must read it, and the next normal call
on the same context must give the right result.  Nothing faults, traps or hangs:
the wait is an ordinary bounded spin that ends.
"""

import ctypes

import pytest
import torch

from pi05_infer import _lib, ops

pytestmark = pytest.mark.gpu

TIMEOUT_EPILOGUE = 0x4


def gelu_tanh(x):
    return 0.5 * x * (1.0 + torch.tanh(0.7978845608028654 * (x + 0.044715 * x * x * x)))


def _operands(m=50, n=4096, k=1024):
    g = torch.Generator(device="cuda").manual_seed(5)
    x = torch.randn(m, k, device="cuda", generator=g).bfloat16()
    wg = (torch.randn(n, k, device="cuda", generator=g) * 0.02).bfloat16()
    wu = (torch.randn(n, k, device="cuda", generator=g) * 0.02).bfloat16()
    ref = gelu_tanh((x.float() @ wg.float().t()).bfloat16().float()) * (x.float() @ wu.float().t())
    return x, wg, wu, ref


def _close(got, ref, rtol=1.6e-2, atol=2e-3):
    err = (got.float() - ref).abs()
    bad = (err > atol + rtol * ref.abs()).sum().item()
    assert bad == 0, f"{bad} mismatches, max err {err.max().item():.3e}"


@pytest.fixture
def fault():
    L = _lib.lib()
    L.pi05_debug_set_splits(2)
    L.pi05_debug_set_fault(1, 50_000_000)  # 50 ms
    yield L
    L.pi05_debug_set_fault(-1, 0)
    L.pi05_debug_set_splits(0)


def test_split_k_wait_times_out_and_recovers(fault):
    L = fault
    x, wg, wu, ref = _operands()
    assert ops.read_device_status() == 0
    ws = ops.workspace(x.device)
    stream = torch.cuda.current_stream().cuda_stream
    out = ops.geglu(x, wg, wu)  # the launch itself succeeds
    torch.cuda.synchronize()
    L.pi05_debug_set_fault(-1, 0)
    v = ctypes.c_int(0)
    rc = L.pi05_read_device_status(ws.data_ptr(), ctypes.byref(v), stream)
    assert rc == 7 and v.value & TIMEOUT_EPILOGUE, (rc, v.value)
    assert "timed out" in _lib.last_error()
    # every other tile finished: output columns 64.. are right
    _close(out[:, 64:], ref[:, 64:])
    # the status was cleared by the read and the context is usable
    out2 = ops.geglu(x, wg, wu)
    torch.cuda.synchronize()
    _close(out2, ref)
    assert ops.read_device_status() == 0


def test_noalloc_status_reports_timeout(fault):
    L = fault
    x, wg, wu, ref = _operands()
    stream = torch.cuda.current_stream().cuda_stream
    out = torch.zeros(50, 4096, dtype=torch.bfloat16, device="cuda")
    rc = L.pi05_gate_up_geglu_noalloc(x.data_ptr(), wg.data_ptr(), wu.data_ptr(), out.data_ptr(), 50, 4096, 1024,
                                      stream)
    assert rc == 0, _lib.last_error()
    torch.cuda.synchronize()
    L.pi05_debug_set_fault(-1, 0)
    # a normal call does not clear the sticky status word
    rc = L.pi05_gate_up_geglu_noalloc(x.data_ptr(), wg.data_ptr(), wu.data_ptr(), out.data_ptr(), 50, 4096, 1024,
                                      stream)
    assert rc == 0, _lib.last_error()
    torch.cuda.synchronize()
    _close(out, ref)
    v = ctypes.c_int(0)
    rc = L.pi05_gate_up_geglu_noalloc_status(ctypes.byref(v), stream)
    assert rc == 7 and v.value & TIMEOUT_EPILOGUE, (rc, v.value)
    rc = L.pi05_gate_up_geglu_noalloc_status(ctypes.byref(v), stream)
    assert rc == 0 and v.value == 0
