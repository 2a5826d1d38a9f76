"""CPU tests: the C-ABI library exports every declared symbol, host-side validation
errors come back as status codes without touching a GPU, ctypes struct layouts
match the C header, replica sharding over gloo ranks."""

import ctypes
import os
import re
import subprocess
import tempfile

import pytest
import torch

from conftest import REPO

from pi05_infer import _lib, abi
from pi05_infer.prefix import Pi05PrefixLayer, Pi05PrefixPlan
from pi05_infer.replicas import max_over_ranks, serve, shard_range

HEADER = os.path.join(REPO, "include", "pi05_b200.h")


def declared_functions():
    src = open(HEADER).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    return sorted(set(re.findall(r"^\s*(?:const\s+)?[\w\s\*]+?\b(pi05_\w+)\s*\(", src, flags=re.M)))


def test_library_exports_every_declared_symbol():
    L = _lib.lib()
    names = declared_functions()
    assert len(names) >= 15
    missing = [n for n in names if not hasattr(L, n)]
    assert not missing, missing
    # and every declared function has a ctypes signature on the Python side
    import pi05_infer.prefix  # noqa: F401  (these modules register their signatures)
    import pi05_infer.vision  # noqa: F401
    assert not [n for n in names if n not in _lib.SIGNATURES], [n for n in names if n not in _lib.SIGNATURES]


def test_host_validation_without_gpu():
    L = _lib.lib()
    assert L.pi05_abi_version() == 2
    ws = L.pi05_workspace_bytes(50, 1018)
    assert ws > 40 << 20
    assert L.pi05_gate_up_geglu(None, None, None, None, 50, 4096, 1024, None, 0, None) == 1
    assert "null" in _lib.last_error()
    buf = (ctypes.c_char * 64)()
    # shape errors are reported before any device work
    assert L.pi05_linear(buf, buf, buf, 50, 1000, 1024, None, 0, None) == 2
    assert L.pi05_gate_up_geglu(buf, buf, buf, buf, 50, 4096, 1000, None, 0, None) == 2
    assert L.pi05_qkv_rope_kv(buf, buf, buf, buf, buf, buf, buf, 50, 1024, 1000, 1018, 8, 1, 256, None, 0,
                              None) == 2
    # missing workspace
    assert L.pi05_linear(buf, buf, buf, 50, 1024, 1024, None, 0, None) == 4
    with pytest.raises(_lib.Pi05Error, match="PI05_ERR_INVALID_ARG"):
        _lib.call("pi05_gate_up_geglu", None, None, None, None, 50, 4096, 1024, None, 0, None)
    # weight folding for the folded norms: argument checks before any launch
    from pi05_infer import abi  # noqa: F401  (binds the signature)
    f = L.pi05_fold_adarms
    f.argtypes = [ctypes.c_void_p, ctypes.c_int, ctypes.c_int] + [ctypes.c_void_p] * 5
    assert f(None, 8, 64, buf, buf, buf, buf, None) == 1 and "null" in _lib.last_error()
    assert f(buf, 8, 60, buf, buf, buf, buf, None) == 2 and "k % 8" in _lib.last_error()
    assert f(buf, 0, 64, buf, buf, buf, buf, None) == 2


STRUCT_PROBE = r"""
#include <stdio.h>
#include <stddef.h>
#include "pi05_b200.h"
#define P(T, f) printf(#T " " #f " %zu\n", offsetof(T, f));
int main(void) {
  P(Pi05ExpertLayer, w_qkv) P(Pi05ExpertLayer, v_cache)
  P(Pi05ExpertPlan, depth) P(Pi05ExpertPlan, eps) P(Pi05ExpertPlan, layers) P(Pi05ExpertPlan, num_steps)
  P(Pi05ExpertPlan, host_timesteps) P(Pi05ExpertPlan, mod_table) P(Pi05ExpertPlan, key_valid)
  P(Pi05ExpertPlan, x_t) P(Pi05ExpertPlan, act) P(Pi05ExpertPlan, workspace) P(Pi05ExpertPlan, workspace_bytes)
  P(Pi05ExpertPlan, attn_splits) P(Pi05ExpertPlan, trace) P(Pi05ExpertPlan, fold) P(Pi05ExpertPlan, batch)
  P(Pi05ExpertPlan, kv_stage) P(Pi05ExpertPlan, host_step_coefs) P(Pi05ExpertPlan, step_noise)
  P(Pi05PrefixLayer, ln1_w) P(Pi05PrefixLayer, v_cache)
  P(Pi05PrefixPlan, tokens) P(Pi05PrefixPlan, eps) P(Pi05PrefixPlan, layers) P(Pi05PrefixPlan, key_valid)
  P(Pi05PrefixPlan, act) P(Pi05PrefixPlan, workspace_bytes) P(Pi05PrefixPlan, kv_only_last_layer)
  printf("sizeof Pi05ExpertPlan %zu\nsizeof Pi05PrefixPlan %zu\n", sizeof(Pi05ExpertPlan), sizeof(Pi05PrefixPlan));
  return 0;
}
"""


def test_ctypes_struct_layout_matches_header():
    with tempfile.TemporaryDirectory() as d:
        c = os.path.join(d, "probe.c")
        exe = os.path.join(d, "probe")
        open(c, "w").write(STRUCT_PROBE)
        subprocess.run(["gcc", "-std=c99", "-I", os.path.dirname(HEADER), c, "-o", exe], check=True)
        out = subprocess.run([exe], check=True, capture_output=True, text=True).stdout
    types = {"Pi05ExpertLayer": abi.Pi05ExpertLayer, "Pi05ExpertPlan": abi.Pi05ExpertPlan,
             "Pi05PrefixLayer": Pi05PrefixLayer, "Pi05PrefixPlan": Pi05PrefixPlan}
    for line in out.splitlines():
        parts = line.split()
        if parts[0] == "sizeof":
            assert ctypes.sizeof(types[parts[1]]) == int(parts[2]), line
        else:
            t, f, off = parts
            assert getattr(types[t], f).offset == int(off), line


def test_shard_range_covers_batch():
    for n in (8, 32, 64, 7):
        for world in (1, 2, 4, 8):
            seen = []
            for r in range(world):
                seen += list(shard_range(n, world, r))
            assert seen == list(range(n))


def _replica_worker(rank, world, port, q):
    import torch.distributed as dist

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    out = serve(8, lambda i: torch.full((2,), float(i)), dist)
    t = max_over_ranks(float(rank + 1), dist)
    dist.barrier()
    dist.destroy_process_group()
    q.put((rank, [float(x[0]) for x in out], t))


def test_replicas_gloo_two_ranks():
    import socket

    import torch.multiprocessing as mp

    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_replica_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = [q.get(timeout=120) for _ in procs]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    for rank, outs, t in res:
        assert outs == [float(i) for i in range(8)]
        assert t == 2.0


def _failing_replica_worker(rank, world, port, q):
    """Rank 1's engine raises on its first observation (a replica failure made on
    the host); the survivors must see an error from the next collective within the
    process-group timeout instead of waiting for ever."""
    import datetime
    import time

    import torch.distributed as dist

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=15))

    def run_one(i):
        if rank == 1:
            raise RuntimeError("replica 1 failed")
        return torch.full((2,), float(i))

    t0 = time.monotonic()
    try:
        serve(8, run_one, dist)
        q.put((rank, "completed", time.monotonic() - t0))
    except Exception as e:  # noqa: BLE001 - any backend error is the detection
        q.put((rank, type(e).__name__, time.monotonic() - t0))
    # no destroy_process_group: the peer is gone


def test_replica_failure_detected_gloo():
    import socket

    import torch.multiprocessing as mp

    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_failing_replica_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = {}
    for _ in procs:
        rank, what, dt = q.get(timeout=120)
        res[rank] = (what, dt)
    for p in procs:
        p.join(timeout=60)
        if p.is_alive():
            p.kill()
    assert res[1][0] == "RuntimeError"  # the failing replica saw its own error
    assert res[0][0] != "completed"  # the survivor did not return a partial result
    assert res[0][1] < 60.0  # and learned of the failure within the bound


def test_sampler_coefficients_match_oracle():
    """The host-side per-step sampler weights (what the final Euler kernel applies)
    reproduce the oracle's flow_sde / flow_cps step and the flow_ode Euler update."""
    from conftest import load_oracle
    from pi05_infer.expert import sampler_coefs

    oracle = load_oracle()
    g = torch.Generator().manual_seed(0)
    x = torch.randn(50, 32, generator=g)
    v = torch.randn(50, 32, generator=g)
    n = torch.randn(50, 32, generator=g)
    ts = oracle.timesteps(10)
    for method in ("flow_ode", "flow_sde", "flow_cps"):
        c = sampler_coefs(10, method, 0.5)
        for s in range(10):
            t = float(ts[s])
            got = (x - v * t) * c[s, 0] + (x + v * (1 - t)) * c[s, 1] + n * c[s, 2]
            if method == "flow_ode":
                ref = oracle.euler(x, v, t, float(ts[s] - ts[s + 1]))
            else:
                ref = oracle.sampler_step(x, v, s, 10, method, 0.5, n)
            assert torch.allclose(got, ref, atol=1e-5), (method, s)
