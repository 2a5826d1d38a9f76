#!/usr/bin/env python
"""Benchmark: pi0.5 sample_actions hot path on B200 (one JSON line on rank 0).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference] [--workload denoise|e2e]

Workloads:
  denoise : config 2 -- the 10-step Euler denoise loop of the Gemma-300M action
            expert at bs=1 over a 968-token prefix KV cache that a random-init
            Gemma-2B prefix LM fills from N(0,1) embeddings (one "step" = one full
            10-step loop = what sample_actions spends after the prefix).
  e2e     : config 3 -- sample_actions end to end (SigLIP + embeddings + prefix LM +
            denoise loop).
Synthetic seeded weights and inputs; no checkpoint or dataset.

Multi-GPU (torchrun): independent engine replicas, one observation each, no
collective on the data path; timing is the max over ranks.

--impl reference times the reference's math on the host CPU (the oracle port of
the reference path, all host threads) on bounded samples of the same workload.
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import time

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(HERE, "pi05-infer_b200"))

METRIC = "sample_actions ms @bs=1; denoise-step µs and HBM GB/s vs peak"
UNIT = "ms"
FALLBACK_HBM_GBS = 6650.0
FALLBACK_BF16_TFLOPS = 1590.0
PREFIX_LEN = 968


def _peaks():
    p = os.path.join(HERE, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as f:
            d = json.load(f)
        return float(d["hbm_gbs"]), float(d["bf16_tflops"]), float(d.get("bf16_tflops_sustained", d["bf16_tflops"])), "measured"
    return FALLBACK_HBM_GBS, FALLBACK_BF16_TFLOPS, 1400.0, "fallback"


def _traffic_from_profiles(kernel_key: str):
    """Per-launch DRAM bytes of `kernel_key` from the committed ncu summary, if any."""
    p = os.path.join(HERE, "profiles", "traffic.json")
    if not os.path.exists(p):
        return None
    try:
        with open(p) as f:
            return json.load(f).get(kernel_key)
    except Exception:
        return None


class ClockSampler:
    """nvidia-smi clocks / throttle reasons sampled during the timed region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.proc = None

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.gpu), f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "100"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except Exception:
            self.proc = None
        return self

    def __exit__(self, *a):
        self.lines = []
        if self.proc is not None:
            self.proc.terminate()
            try:
                out, _ = self.proc.communicate(timeout=5)
            except Exception:
                self.proc.kill()
                out = ""
            self.lines = [l for l in out.splitlines() if l.strip()]

    def sample_once(self):
        """One synchronous sample (for timed regions shorter than the polling period);
        call it while queued GPU work is still running."""
        try:
            out = subprocess.run(["nvidia-smi", "-i", str(self.gpu), f"--query-gpu={self.FIELDS}",
                                  "--format=csv,noheader,nounits"], capture_output=True, text=True, timeout=10).stdout
            self.extra = [l for l in out.splitlines() if l.strip()]
        except Exception:
            self.extra = []

    def summary(self):
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for l in getattr(self, "lines", []) + getattr(self, "extra", []):
            parts = [x.strip() for x in l.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                mx = float(parts[2])
            except ValueError:
                continue
            for n, v in zip(names, parts[5:9]):
                if v.lower().startswith("active"):
                    reasons.add(n)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": mx, "reasons": sorted(reasons),
                "samples": len(sm)}


def _dist():
    ws = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return ws, rank, local


def _load_oracle():
    import importlib.util

    spec = importlib.util.spec_from_file_location("pi05_oracle", os.path.join(HERE, "oracle", "pi05_oracle.py"))
    oracle = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(oracle)
    return oracle


class CpuSampler:
    """Bounded CPU samples of the reference path (oracle port, fp32, all host threads).

    One sample times one component of sample_actions on the host CPU: a SigLIP
    encoder layer over the 3 views (768 tokens), a Gemma-2B prefix layer over 968
    tokens, or one velocity evaluation of the 18-layer action expert (one Euler
    step).  The whole call is estimated as 27 x SigLIP layer + 18 x prefix layer +
    10 x velocity (config 3), or 10 x velocity (config 2).
    """

    def __init__(self, workload: str):
        import torch

        from pi05_infer import synthetic
        from pi05_infer.config import GemmaShape, SiglipShape

        torch.set_num_threads(os.cpu_count() or 1)
        self.torch = torch
        self.oracle = _load_oracle()
        self.workload = workload
        self.sd = synthetic.make_expert_weights(0)
        self.kv = [(k[0, 0], v[0, 0]) for k, v in synthetic.make_prefix_kv(1, 18, PREFIX_LEN)]
        self.noise = synthetic.make_noise(2)[0]
        self.pad = torch.ones(PREFIX_LEN, dtype=torch.bool)
        self.table = self.oracle.adarms_table(self.sd, 18, 10, synthetic.EXPERT_PREFIX)
        self.components = ["velocity"]
        if workload == "e2e":
            lm1 = GemmaShape(width=2048, depth=1, mlp_dim=16384, num_heads=8, num_kv_heads=1, head_dim=256)
            self.sd_lm = synthetic.make_prefix_lm_weights(10, lm1)
            self.embs = synthetic.make_prefix_embeddings(3, PREFIX_LEN, 2048)[0]
            self.sd_vis = synthetic.make_siglip_weights(20, SiglipShape(depth=1))
            self.imgs = synthetic.make_images(4, 3, 224)
            self.components = ["siglip_layer", "prefix_layer", "velocity"]
        self.times = {c: [] for c in self.components}

    def run(self, comp: str, record: bool = True) -> float:
        o = self.oracle
        t0 = time.perf_counter()
        if comp == "velocity":
            o.velocity(self.sd, self.noise, self.kv, self.table[0], self.pad, 18, "fp32")
        elif comp == "prefix_layer":
            self._prefix_layer()
        else:
            o.siglip_image_features(self.sd_vis, self.imgs, 1, "fp32")
        dt = time.perf_counter() - t0
        if record:
            self.times[comp].append(dt)
        return dt

    def _prefix_layer(self):
        """One full Gemma-2B decoder layer over the prefix (oracle math, fp32)."""
        o = self.oracle
        w, p = self.sd_lm, "paligemma_with_expert.paligemma.model.language_model.layers.0."
        h = self.embs
        xn = o.rms_norm(h, w[p + "input_layernorm.weight"], 1e-6, "fp32")
        q = (xn @ w[p + "self_attn.q_proj.weight"].t()).view(-1, 8, 256)
        k = xn @ w[p + "self_attn.k_proj.weight"].t()
        v = xn @ w[p + "self_attn.v_proj.weight"].t()
        a = o.attention(q, k, v, o.prefix_mask(self.pad), 1 / 16, "fp32")
        h = h + a @ w[p + "self_attn.o_proj.weight"].t()
        hn = o.rms_norm(h, w[p + "post_attention_layernorm.weight"], 1e-6, "fp32")
        act = o.gelu_tanh(hn @ w[p + "mlp.gate_proj.weight"].t()) * (hn @ w[p + "mlp.up_proj.weight"].t())
        return h + act @ w[p + "mlp.down_proj.weight"].t()

    def estimate_ms(self) -> float:
        mean = {c: statistics.mean(v) for c, v in self.times.items() if v}
        ms = 10 * mean["velocity"]
        if self.workload == "e2e":
            ms += 27 * mean["siglip_layer"] + 18 * mean["prefix_layer"]
        return ms * 1e3

    def describe(self) -> str:
        n = {c: len(v) for c, v in self.times.items()}
        if self.workload == "e2e":
            return (f"{n} timed component samples (fp32 torch CPU restatement of the reference path); "
                    "sample_actions estimated as 27 x SigLIP layer + 18 x Gemma-2B prefix layer + 10 x expert velocity")
        return f"{n['velocity']} expert velocity evaluations (fp32); loop = 10 x velocity"


def run_reference(args):
    """CPU reference arm: the oracle port of the reference path on the host cores."""
    ws, rank, _ = _dist()
    if rank != 0:
        return 0
    cs = CpuSampler(args.workload)
    for i in range(min(args.warmup, len(cs.components))):
        cs.run(cs.components[i % len(cs.components)], record=False)
    n = max(len(cs.components), min(args.steps, 60))
    for i in range(n):
        cs.run(cs.components[i % len(cs.components)])
    ms = cs.estimate_ms()
    line = {
        "impl": "reference", "metric": METRIC, "value": ms, "unit": UNIT, "n_gpus": ws, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": False, "scaling": "weak",
        "vs_baseline": None, "dtype": "f32", "data": "synthetic (seeded N(0,0.02) weights, N(0,1) inputs)",
        "config": _config(args, ws),
        "cpu_baseline": {"value": ms, "unit": UNIT, "cores": cs.torch.get_num_threads(), "kind": "port",
                         "sample": cs.describe() + f" (timed samples capped at 60 of --steps {args.steps})"},
        "e2e": {"value": ms, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)
    return 0


def _config(args, ws):
    if args.workload == "e2e":
        return {"workload": "config3: sample_actions end to end (SigLIP 3x224^2 + 200 tokens -> 968-token prefix LM -> 10-step denoise)",
                "global_batch": ws, "seq_len": PREFIX_LEN, "parallelism": f"replicas{ws}",
                "l2": "inputs larger than L2 (weights streamed every call)"}
    return {"workload": "config2: 10-step Euler denoise loop, Gemma-300M expert, bs=1, 968-token prefix KV from a random Gemma-2B prefix",
            "global_batch": ws, "seq_len": PREFIX_LEN + 50, "parallelism": f"replicas{ws}",
            "l2": "inputs larger than L2: 623 MB of bf16 expert weights streamed per Euler step (5x L2)"}


def run_ours(args):
    import torch

    ws, rank, local = _dist()
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    pg = None
    if ws > 1:
        import datetime

        import torch.distributed as dist

        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=dev)
        pg = dist

    from pi05_infer import _lib, synthetic
    from pi05_infer.config import GEMMA_2B, GEMMA_300M
    from pi05_infer.engine import OpenPi0Inference
    from pi05_infer.expert import DenoiseRunner, ExpertWeights

    hbm_peak, bf16_peak, bf16_sus, peak_src = _peaks()
    # Weights: same model on every replica; observation seeds differ per rank.
    engine = OpenPi0Inference.synthetic(device=dev, seed=0, with_vision=(args.workload == "e2e"))
    obs = engine.synthetic_observation(seed=100 + rank)
    noise = synthetic.make_noise(2 + rank).to(dev)
    engine.prepare(obs)  # prefix LM fills the KV cache (and SigLIP for e2e)

    launches0 = _lib.lib().pi05_launch_count()
    if args.workload == "e2e":
        step_fn = engine.capture_full(obs, noise)
    else:
        step_fn = engine.capture_denoise(noise)
    launches_per_step = _lib.lib().pi05_launch_count() - launches0

    def barrier():
        if pg is not None:
            pg.barrier()

    for _ in range(args.warmup):
        step_fn()
    torch.cuda.synchronize(dev)
    barrier()
    torch.cuda.synchronize(dev)
    stream = torch.cuda.current_stream(dev)
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    with ClockSampler(local) as clk:
        e0.record(stream)
        for _ in range(args.steps):
            step_fn()
        e1.record(stream)
        clk.sample_once()  # the replays queued above are still executing
        torch.cuda.synchronize(dev)
    barrier()
    ms = e0.elapsed_time(e1) / args.steps
    if pg is not None:
        t = torch.tensor([ms], device=dev)
        pg.all_reduce(t, op=pg.ReduceOp.MAX)
        ms = float(t.item())

    # Denoise-step sub-metric: the config-2 loop (10 Euler steps over the prefix
    # cache just filled) replayed alone as its own CUDA graph.
    den_fn = step_fn if args.workload == "denoise" else engine.capture_denoise(noise)
    den_ms = ms
    if args.workload != "denoise":
        for _ in range(3):
            den_fn()
        torch.cuda.synchronize(dev)
        e0.record(stream)
        n_den = max(10, args.steps // 2)
        for _ in range(n_den):
            den_fn()
        e1.record(stream)
        torch.cuda.synchronize(dev)
        den_ms = e0.elapsed_time(e1) / n_den
        if pg is not None:
            t = torch.tensor([den_ms], device=dev)
            pg.all_reduce(t, op=pg.ReduceOp.MAX)
            den_ms = float(t.item())

    # End to end through the public API: host noise (pinned) in, host actions out.
    noise_host = synthetic.make_noise(2 + rank).pin_memory()
    for _ in range(2):  # warm-up through the same API (graph capture on first use)
        if args.workload == "e2e":
            engine.sample_actions(obs, noise=noise_host)["actions"].cpu()
        else:
            engine.denoise(noise_host)["actions"].cpu()
    torch.cuda.synchronize(dev)
    barrier()
    e2e_n = max(10, args.steps // 4)
    t0 = time.perf_counter()
    for _ in range(e2e_n):
        if args.workload == "e2e":
            out = engine.sample_actions(obs, noise=noise_host)["actions"].cpu()
        else:
            out = engine.denoise(noise_host)["actions"].cpu()
    e2e_ms = (time.perf_counter() - t0) * 1e3 / e2e_n
    if pg is not None:
        t = torch.tensor([e2e_ms], device=dev)
        pg.all_reduce(t, op=pg.ReduceOp.MAX)
        e2e_ms = float(t.item())
    h2d = noise_host.numel() * 4 + (engine.observation_host_bytes(obs) if args.workload == "e2e" else 0)
    d2h = out.numel() * out.element_size()

    # Dominant kernel (largest share of the step in the ncu launch list): the
    # swap-AB tcgen05 GEMM with the gated-residual epilogue, here its down-projection
    # instance (8.4 MB of weights per launch), timed alone over all 18 layers.
    roof = engine.time_down_kernel(reps=20)
    achieved = roof["bytes"] / (roof["us"] * 1e-6) / 1e9
    traffic = _traffic_from_profiles("skinny_gemm_gated_resid_down")
    denoise_us = engine.last_denoise_step_us(den_ms)

    line = {
        "metric": METRIC, "value": ms, "unit": UNIT, "n_gpus": ws, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": ms, "higher_is_better": False, "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic (seeded random-init weights, N(0,1) prefix embeddings and noise)",
        "config": _config(args, ws),
        "throughput_obs_per_s": ws * 1000.0 / ms,
        "denoise_step": {"us": denoise_us, "algorithmic_bytes": engine.denoise_step_bytes(),
                         "hbm_gbs": engine.denoise_step_bytes() / (denoise_us * 1e-6) / 1e9 if denoise_us else None,
                         "frac_of_measured_hbm": (engine.denoise_step_bytes() / (denoise_us * 1e-6) / 1e9 / hbm_peak)
                         if denoise_us else None},
        "roofline": {"kernel": "skinny_gemm_kernel<GATED_RESID,64,3> (down_proj + gated residual, M=50, N=1024, "
                               "K=4096)",
                     "bound": "hbm", "achieved": achieved, "peak": hbm_peak, "unit": "GB/s",
                     "frac": achieved / hbm_peak, "traffic": traffic, "peak_source": peak_src,
                     "algorithmic_bytes_per_launch": roof["bytes"], "us_per_launch": roof["us"]},
        "e2e": {"value": e2e_ms, "unit": UNIT, "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h},
        "gpu_launches": launches_per_step * args.steps,
        "clocks": clk.summary(),
    }
    if ws == 1 and rank == 0 and not args.no_cpu_baseline:
        cs = CpuSampler(args.workload)
        for c in cs.components:
            cs.run(c, record=False)
        for _ in range(3):
            for c in cs.components:
                cs.run(c)
        line["cpu_baseline"] = {"value": cs.estimate_ms(), "unit": UNIT, "cores": cs.torch.get_num_threads(),
                                "kind": "port", "sample": cs.describe()}
    if rank == 0:
        print(json.dumps(line), flush=True)
    engine.release_graphs()
    if pg is not None:
        pg.barrier()
        pg.destroy_process_group()
    return 0


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=50)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--workload", choices=["denoise", "e2e"], default="e2e")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    if args.impl == "reference":
        return run_reference(args)
    return run_ours(args)


if __name__ == "__main__":
    sys.exit(main())
