"""GPU parity of the optional execution paths against the default one.

The switches are environment variables read once per process, so each variant runs
the 10-step denoise loop (config 2 shapes: Gemma-300M expert, 968-token prefix,
seeded synthetic weights / KV / noise) in a child process; the test compares the
final actions with the default path's under the denoise tolerance (max-abs <= 2e-2,
cosine >= 0.9999):

  PI05_FOLD_NORM=0    explicit adaRMS norm kernels instead of the default folded
                      norms (norm modulation folded into per-step q|k|v and
                      gate/up weights, rstd and bias applied to the accumulators)
  PI05_ATTN_WARPS=4   64-row attention CTAs instead of 32-row ones
  PI05_ATTN_PAIR=0    one warp per 16 query rows instead of a warp pair that splits
                      each key chunk (keys for S, head dims for P.V)
  PI05_PDL=0          launches without programmatic dependent launch
"""

import os
import subprocess
import sys

import pytest
import torch

from conftest import PKG_ROOT

pytestmark = pytest.mark.gpu

_SCRIPT = r"""
import sys
import torch
sys.path.insert(0, sys.argv[1])
from pi05_infer import ops, synthetic
from pi05_infer.config import GEMMA_300M
from pi05_infer.expert import DenoiseRunner, ExpertWeights

sd = synthetic.make_expert_weights(0)
kv = synthetic.make_prefix_kv(1, 18, 968)
kv = [(k[0, 0].bfloat16().cuda(), v[0, 0].bfloat16().cuda()) for k, v in kv]
noise = synthetic.make_noise(2)[0]
pad = torch.ones(968, dtype=torch.bool)
pad[-37:] = False
w = ExpertWeights(sd, GEMMA_300M, "cuda")
r = DenoiseRunner(w, prefix_len=968, num_steps=10)
r.set_prefix(kv, pad.cuda())
out = r.run(noise.cuda(), use_graph=True).float().cpu()
assert ops.read_device_status() == 0
torch.save(out, sys.argv[2])
"""


def _run(env_extra, path):
    env = dict(os.environ)
    for k in ("PI05_FOLD_NORM", "PI05_ATTN_WARPS", "PI05_ATTN_PAIR", "PI05_PDL"):
        env.pop(k, None)
    env.update(env_extra)
    subprocess.run([sys.executable, "-c", _SCRIPT, PKG_ROOT, path], env=env, check=True, timeout=600)
    return torch.load(path)


@pytest.fixture(scope="module")
def default_actions(tmp_path_factory):
    return _run({}, str(tmp_path_factory.mktemp("sw") / "default.pt"))


@pytest.mark.parametrize(
    "switch",
    [{"PI05_FOLD_NORM": "0"}, {"PI05_ATTN_WARPS": "4"}, {"PI05_ATTN_PAIR": "0"}, {"PI05_PDL": "0"}],
    ids=["norm_kernels", "attn_4warps", "attn_single_warps", "no_pdl"],
)
def test_switch_matches_default(default_actions, switch, tmp_path):
    got = _run(switch, str(tmp_path / "variant.pt"))
    ref = default_actions
    assert got.shape == ref.shape
    err = (got - ref).abs().max().item()
    cos = float((got.flatten().double() @ ref.flatten().double()) /
                (got.flatten().double().norm() * ref.flatten().double().norm()))
    assert err <= 2e-2, f"max-abs {err}"
    assert cos >= 0.9999, f"cosine {cos}"
