#!/usr/bin/env python
"""GPT training steps/s on the rg CUDA device (B200), 1 to 8 GPUs, against rg's CPU interpreter.

Default workload: BASELINE config 5, the char-level GPT with vocab 96, context 256, d_model 512,
12 layers, 8 heads, GELU MLP 4x, pre-LayerNorm, AdamW(1e-3), global batch 512 split by batch over
the ranks (strong scaling: total work is fixed), Zipf(1.1) int32 tokens. A "step" is one
training step of the compiled plan: in-graph window sampling, forward, backward, the gradient
all-reduce when N > 1, and the AdamW update.

  python bench.py [--gpus N] [--steps K] [--warmup W] [--config NAME] [--impl ours|reference]

`value` is device time (CUDA events inside the run loop, state already in HBM); `e2e` is the
same run through the C-ABI run call from host buffers (state and data copied in, state and loss
history copied out, inside the timed region). `--impl reference` times rg's CPU interpreter (the
restatement under oracle/, rg itself cannot be built here) on a bounded sample of the workload.
"""
import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

CONFIGS = {
    # BASELINE config 5 (scaling config) and its one-GPU companion; config 4.
    "gpt-d512-l12": dict(vocab=96, block=256, d=512, heads=8, layers=12, batch=512, tokens="zipf"),
    "gpt-d256-l6": dict(vocab=96, block=256, d=256, heads=8, layers=6, batch=64, tokens="zipf"),
    "gpt-d128-l4": dict(vocab=96, block=128, d=128, heads=4, layers=4, batch=64, tokens="uniform"),
}
N_TOKENS = 200_000


def tokens_for(cfg):
    rng = np.random.default_rng(0)
    if cfg["tokens"] == "uniform":
        return rng.integers(0, cfg["vocab"], size=N_TOKENS, dtype="int32")
    p = (np.arange(cfg["vocab"]) + 1.0) ** -1.1
    return rng.choice(cfg["vocab"], size=N_TOKENS, p=p / p.sum()).astype("int32")


def train_flops(cfg, batch):
    """Matmul FLOPs of one training step (forward x3), full T x T attention, as the plan runs it."""
    d, t, L, v = cfg["d"], cfg["block"], cfg["layers"], cfg["vocab"]
    tokens = batch * t
    per_layer = 2 * tokens * d * (3 * d + d + 4 * d + 4 * d) + 2 * 2 * batch * t * t * d
    return 3 * (L * per_layer + 2 * tokens * d * v)


class Clocks:
    """Samples SM clocks and throttle reasons with nvidia-smi while the timed region runs."""

    def __init__(self, index):
        self.index, self.samples, self.stop = index, [], threading.Event()

    def __enter__(self):
        q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,clocks_event_reasons.hw_slowdown,"
             "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")
        try:
            self.proc = subprocess.Popen(["nvidia-smi", "-i", str(self.index), f"--query-gpu={q}", "--format=csv,noheader,nounits", "-lms", "200"],
                                         stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.reader = threading.Thread(target=self._read, daemon=True)
            self.reader.start()
        except OSError:
            self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            parts = [p.strip() for p in line.split(",")]
            if len(parts) >= 9:
                self.samples.append(parts)

    def __exit__(self, *exc):
        if self.proc:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self):
        if not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["no_samples"]}
        sm = [float(s[1]) for s in self.samples if s[1].replace(".", "").isdigit()]
        mx = [float(s[2]) for s in self.samples if s[2].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[k] for s in self.samples for k in range(4) if s[5 + k].lower() == "active"})
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(mx) if mx else None, "reasons": reasons, "samples": len(self.samples)}


def peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            p = json.load(f)
        return {"hbm_gbs": p["hbm_gbs"], "bf16_tflops": p["bf16_tflops"], "bf16_tflops_sustained": p["bf16_tflops_sustained"], "source": "measured"}
    except (OSError, KeyError, ValueError):
        return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0, "source": "fallback"}


def build_model(F, cfg, world, rank):
    model = F.gpt.GPT(vocab=cfg["vocab"], block=cfg["block"], d=cfg["d"], heads=cfg["heads"], layers=cfg["layers"])
    params = model.init(F.random.key(0))
    opt = F.optim.adamw(1e-3, weight_decay=0.01)
    state = {"params": params, "opt": opt.init(params), "key": F.random.key(1)}
    step = F.gpt.make_train_step(model, opt, cfg["batch"], world, rank)
    return step, state


def cpu_sample(cfg, seconds_budget=30.0):
    """rg's CPU interpreter (restated) on one-sequence batches of the same model: seconds per
    sequence, which scales linearly to the configured batch. Returns (seconds/step at the full
    batch, sample description, threads)."""
    sys.path.insert(0, os.path.join(ROOT, "oracle", "_build"))
    from rustautograd_b200 import build_ext
    build_ext.build_oracle()
    import _rg_oracle
    from rustautograd_b200 import frontend as F
    F.use(_rg_oracle, "cpu")
    sample = dict(cfg, batch=1)
    step, state = build_model(F, sample, 1, 0)
    tokens = F.tensor(tokens_for(cfg))
    c = F.compile(step, (state, tokens), validate="none", device="cpu")
    F.run(c, state, tokens, steps=1)  # first touch of the frame's pages
    t, n = 0.0, 0
    while n < 3 and t < seconds_budget:
        r = F.run(c, state, tokens, steps=1)
        t += r.elapsed
        n += 1
    per_seq = t / n
    return per_seq * cfg["batch"], f"{n} steps of batch 1 (T={cfg['block']}), scaled x{cfg['batch']} to the global batch", _rg_oracle.threads()


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--config", default="gpt-d512-l12", choices=sorted(CONFIGS))
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    args = ap.parse_args()
    cfg = CONFIGS[args.config]
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    metric = "GPT train steps/sec"
    workload = f"{args.config} global_batch={cfg['batch']} T={cfg['block']}"

    if args.impl == "reference":
        if rank != 0:
            return
        secs, sample, threads = cpu_sample(cfg)
        value = 1.0 / secs
        print(json.dumps({
            "impl": "reference", "metric": metric, "value": value, "unit": "steps/s", "n_gpus": args.gpus, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": secs * 1e3, "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
            "dtype": "f32", "data": "synthetic", "config": {"workload": workload},
            "cpu_baseline": {"value": value, "unit": "steps/s", "cores": threads, "kind": "port", "sample": sample},
            "e2e": {"value": value, "unit": "steps/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        }))
        return

    import torch
    torch.cuda.set_device(local)
    dist = None
    if world > 1:
        import datetime
        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300), device_id=torch.device("cuda", local))
    from rustautograd_b200 import _rg
    from rustautograd_b200 import frontend as F
    if not _rg.cuda_available():
        raise SystemExit("no usable sm_100 GPU: the CUDA device is unavailable")
    F.use(_rg, "cuda")
    if world > 1:
        uid = [_rg.dist_unique_id() if rank == 0 else None]
        dist.broadcast_object_list(uid, src=0)
        _rg.dist_init(rank, world, uid[0])

    step, state = build_model(F, cfg, world, rank)
    tokens = F.tensor(tokens_for(cfg))
    t0 = time.perf_counter()
    compiled = F.compile(step, (state, tokens), validate="none", device="cuda")
    compile_s = time.perf_counter() - t0
    n_state = len(F.flatten(state)[0])
    state_leaves = [F.tensor(l)._t for l in F.flatten(state)[0]]
    data = [tokens._t]
    state_map = [(k, k) for k in range(n_state)]
    hist = [n_state]

    def run(steps):
        return compiled._n.run(state_map, [n_state], hist, state_leaves, [data], steps)

    run(args.warmup)
    launches0 = compiled._n.launches()
    if dist:
        dist.barrier()
    torch.cuda.synchronize()
    with Clocks(local) as clocks:
        # The NVTX range marks the timed steps for profilers (ncu --nvtx --nvtx-include "timed/").
        torch.cuda.nvtx.range_push("timed")
        w0 = time.perf_counter()
        new_state, outputs, history, done, bad, device_s = run(args.steps)
        wall = time.perf_counter() - w0
        torch.cuda.nvtx.range_pop()
    torch.cuda.synchronize()
    if dist:
        dist.barrier()
    launches = compiled._n.launches() - launches0
    if dist:
        t = torch.tensor([device_s, wall], dtype=torch.float64, device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        device_s, wall = t.tolist()
    loss = history[0]
    state_bytes = sum(len(x.tobytes()) for x in state_leaves)
    data_bytes = len(tokens._t.tobytes())

    # Roofline of the dominant kernel class: per-step device times (CUDA events between plan
    # steps on the device's stream) over the same compiled plan and inputs. Every rank runs it:
    # the plan's all-reduce steps are collectives.
    secs = compiled._n.step_seconds(state_leaves + data, 2)
    out = None
    if rank == 0:
        value = done / device_s
        flops = train_flops(cfg, cfg["batch"]) / world
        pk = peaks()
        costs = compiled._n.step_costs()
        by_kind = {}
        for (kind, fl, by), s in zip(costs, secs):
            e = by_kind.setdefault(kind, [0.0, 0.0, 0.0, 0])
            e[0] += s
            e[1] += fl
            e[2] += by
            e[3] += 1
        total = sum(v[0] for v in by_kind.values())
        top = max(by_kind, key=lambda k: by_kind[k][0])
        t_s, fl, by, n = by_kind[top]
        if top == "matmul":
            achieved, peak, unit, bound = fl / t_s / 1e12, pk["bf16_tflops_sustained"], "TFLOP/s", "tensor"
        else:
            achieved, peak, unit, bound = by / t_s / 1e9, pk["hbm_gbs"], "GB/s", "hbm"
        fused = by_kind.get("fused", [1e-30, 0, 0, 0])
        roofline = {"bound": bound, "kernel": top, "achieved": achieved, "peak": peak, "unit": unit, "frac": achieved / peak,
                    "peak_source": pk["source"], "traffic": None, "launches_per_step": n, "share_of_step": t_s / total,
                    "fused_elementwise": {"achieved_gbs": fused[2] / fused[0] / 1e9, "frac_of_hbm": fused[2] / fused[0] / 1e9 / pk["hbm_gbs"],
                                          "share_of_step": fused[0] / total}}
        cpu = None
        if not args.no_cpu_baseline:
            secs_cpu, sample, threads = cpu_sample(cfg)
            cpu = {"value": 1.0 / secs_cpu, "unit": "steps/s", "cores": threads, "kind": "port", "sample": sample}
        out = {
            "metric": metric, "value": value, "unit": "steps/s", "n_gpus": world, "steps": done, "warmup": args.warmup,
            "ms_per_step": device_s / done * 1e3, "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
            "dtype": "f32", "data": "synthetic",
            "config": {"workload": workload, "global_batch": cfg["batch"], "per_rank_batch": cfg["batch"] // world, "seq_len": cfg["block"],
                       "d_model": cfg["d"], "layers": cfg["layers"], "heads": cfg["heads"], "vocab": cfg["vocab"],
                       "parallelism": f"dp{world}", "l2": "state (params + AdamW moments) larger than L2 is streamed every step"},
            "e2e": {"value": done / wall, "unit": "steps/s", "h2d_bytes_per_step": (state_bytes + data_bytes) / done,
                    "d2h_bytes_per_step": (state_bytes + 8 * done) / done},
            "gpu_launches": launches,
            "tflops_per_gpu": flops * done / device_s / 1e12,
            "roofline": roofline,
            "cpu_baseline": cpu,
            "clocks": clocks.summary(),
            "loss": {"first": loss[0], "last": loss[-1], "nonfinite_step": bad},
            "compile_seconds": compile_s,
        }
    if dist:
        dist.barrier()
        _rg.dist_finalize()
        dist.destroy_process_group()
    if out is not None:
        print(json.dumps(out))


if __name__ == "__main__":
    main()
