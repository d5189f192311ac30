#!/usr/bin/env python
"""Steps/s of rg plans on the CUDA device (B200), 1 to 8 GPUs, against rg's CPU interpreter.

Default workload: BASELINE config 5, the char-level GPT with vocab 96, context 256, d_model 512,
12 layers, 8 heads, GELU MLP 4x, pre-LayerNorm, AdamW(1e-3), global batch 512 split by batch over
the ranks (strong scaling: total work is fixed), Zipf(1.1) int32 tokens. A "step" is one
training step of the compiled plan: in-graph window sampling, forward, backward, the gradient
all-reduce when N > 1, and the AdamW update.

  python bench.py [--gpus N] [--steps K] [--warmup W] [--config NAME] [--impl ours|reference]

Other workloads (--config): gpt-d256-l6 (the 1-GPU companion of config 5), gpt-d128-l4
(config 4), adamw-c2 (config 2: the AdamW update of four large tensors, HBM-bound),
linreg-c1 (config 1), chain-c3 (config 3: matrix chains reordered by the e-graph search),
gemm-mlp (one 131072 x 512 x 2048 product of config 5, for profiling), gpt-d512-l1 (one layer of
the d512 model at batch 64, for profiling).

`value` is device time (CUDA events inside the run loop, state already in HBM); `e2e` is the
same run through the C-ABI run call from host buffers (state and data copied in, state and the
per-step history scalar copied out, inside the timed region). `--impl reference` times rg's CPU
interpreter (the restatement under oracle/; rg itself cannot be built here) on a bounded sample
of the workload.
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

N_TOKENS = 200_000


# ---------------------------------------------------------------------------------------------
# Workloads. Each builds (step function, state, data leaves) with the front end `F`, states the
# algorithmic work of one step, and times a bounded sample of itself on the CPU oracle.
# ---------------------------------------------------------------------------------------------

class Gpt:
    metric = "GPT train steps/sec"
    bound = "tensor"
    scalar_output = True

    def __init__(self, name, vocab, block, d, heads, layers, batch, tokens):
        self.name, self.vocab, self.block, self.d, self.heads, self.layers, self.batch, self.tokens = name, vocab, block, d, heads, layers, batch, tokens

    def tokens_array(self):
        rng = np.random.default_rng(0)
        if self.tokens == "uniform":
            return rng.integers(0, self.vocab, size=N_TOKENS, dtype="int32")
        p = (np.arange(self.vocab) + 1.0) ** -1.1
        return rng.choice(self.vocab, size=N_TOKENS, p=p / p.sum()).astype("int32")

    def build(self, F, world=1, rank=0, batch=None):
        batch = batch or self.batch
        model = F.gpt.GPT(vocab=self.vocab, block=self.block, d=self.d, heads=self.heads, layers=self.layers)
        params = model.init(F.random.key(0))
        opt = F.optim.adamw(1e-3, weight_decay=0.01)
        state = {"params": params, "opt": opt.init(params), "key": F.random.key(1)}
        return F.gpt.make_train_step(model, opt, batch, world, rank), state, [F.tensor(self.tokens_array())]

    def flops(self, batch=None):
        """Matmul FLOPs of one training step (forward x3), full T x T attention, as the plan runs it."""
        batch = batch or self.batch
        d, t, L, v = self.d, self.block, self.layers, self.vocab
        tokens = batch * t
        per_layer = 2 * tokens * d * (3 * d + d + 4 * d + 4 * d) + 2 * 2 * batch * t * t * d
        return 3 * (L * per_layer + 2 * tokens * d * v)

    def config(self, world):
        return {"workload": f"{self.name} global_batch={self.batch} T={self.block}", "global_batch": self.batch,
                "per_rank_batch": self.batch // world, "seq_len": self.block, "d_model": self.d, "layers": self.layers,
                "heads": self.heads, "vocab": self.vocab, "parallelism": f"dp{world}",
                "l2": "state (params + AdamW moments) larger than L2 is streamed every step"}

    def cpu_sample(self, F, oracle, full=False):
        """One step of the same model at batch 1 and, with `full`, one at batch 4. A full
        global-batch step is far beyond a bounded sample (hours at d512), so its time is
        extrapolated: with `full`, by the line through the two measured steps (the optimizer
        update and the other batch-independent work are its intercept); otherwise linearly from
        batch 1, which overstates the CPU step time (the interpreter goes parallel on more of a
        step's operations as the batch grows)."""
        batches = (1, 4) if full else (1,)
        secs = []
        for b in batches:
            step, state, data = self.build(F, batch=b)
            c = F.compile(step, (state, data[0]), validate="none", device="cpu")
            secs.append(F.run(c, state, data[0], steps=1).elapsed)
        if full:
            slope = (secs[1] - secs[0]) / (batches[1] - batches[0])
            est = secs[0] + slope * (self.batch - batches[0])
            method = f"line through the measured steps at batch {batches[0]} and {batches[1]}, evaluated at the global batch {self.batch}"
        else:
            est = secs[0] * self.batch
            method = f"the batch-1 step scaled x{self.batch} (linear from batch 1: an upper bound on the CPU step time)"
        return {"seconds_per_step": est, "sample_steps": len(batches), "sample_batches": list(batches), "sample_seconds": secs,
                "extrapolated": True, "method": method,
                "sample": f"{len(batches)} step(s) of T={self.block} windows at batch {', '.join(map(str, batches))}; {method}"}


class AdamW:
    """AdamW over four f32 tensors (25.17 M elements), grads as the data batch.
    Algorithmic traffic: read w, g, m, v and write w, m, v = 28 bytes per element per step."""
    metric = "AdamW steps/sec"
    bound = "hbm"
    scalar_output = True
    SHAPES = [(4096, 4096), (4096,), (1024, 4096), (4096, 1024)]

    def __init__(self, name):
        self.name = name
        self.n = sum(int(np.prod(s)) for s in self.SHAPES)

    def build(self, F, world=1, rank=0, scale=1):
        rng = np.random.default_rng(0)
        shapes = [tuple(max(1, x // scale) for x in s) for s in self.SHAPES]
        mk = lambda s: F.tensor((rng.normal(size=s) * 0.02).astype("float32"))
        params = [mk(s) for s in shapes]
        grads = [mk(s) for s in shapes]
        mu = [mk(s) for s in shapes]
        nu = [F.tensor(np.abs(mk(s).numpy())) for s in shapes]
        opt = F.optim.adamw(1e-3, 0.9, 0.999, 1e-8, 0.01)
        state = {"params": params, "opt": {"count": F.full((), 0, "float32"), "mu": mu, "nu": nu}}

        def step(state, g):
            p, o = opt.update(g, state["opt"], state["params"])
            return {"params": p, "opt": o}, o["count"]
        return step, state, grads

    def flops(self, batch=None):
        return 0.0

    def algorithmic_bytes(self):
        return 28.0 * self.n

    def config(self, world):
        return {"workload": f"{self.name} 4 tensors {self.n} elements", "elements": self.n, "parallelism": "replicas",
                "l2": "704 MB of state and gradients streamed every step (larger than L2)"}

    def cpu_sample(self, F, oracle, full=False):
        step, state, grads = self.build(F)
        c = F.compile(step, (state, grads), validate="none", device="cpu")
        n = 10 if full else 5
        t = F.run(c, state, grads, steps=n).elapsed
        return {"seconds_per_step": t / n, "sample_steps": n, "sample_seconds": [t], "extrapolated": False, "sample": f"{n} full steps in one run"}


class LinReg:
    """the README linear regression, 500 gradient steps per run."""
    metric = "linear-regression steps/sec"
    bound = "latency"
    scalar_output = True

    def __init__(self, name):
        self.name = name

    def build(self, F, world=1, rank=0):
        x = np.random.default_rng(0).normal(size=(256, 8)).astype("float32")
        y = x @ np.arange(8, dtype="float32")

        def step(w, batch):
            value, g = F.value_and_grad(lambda w, b: (((b[0] @ w) - b[1]) ** 2).mean())(w, batch)
            return w - 0.05 * g, value
        return step, F.zeros(8), [F.tensor(x), F.tensor(y)]

    def flops(self, batch=None):
        return 4.0 * 256 * 8

    def config(self, world):
        return {"workload": f"{self.name} x (256, 8) f32, lr 0.05", "parallelism": "replicas", "l2": "8 KB of data, L2-resident by design"}

    def cpu_sample(self, F, oracle, full=False):
        step, state, data = self.build(F)
        c = F.compile(step, (state, list(data)), validate="none", device="cpu")
        r = F.run(c, state, list(data), steps=500)
        return {"seconds_per_step": r.elapsed / 500, "sample_steps": 500, "sample_seconds": [r.elapsed], "extrapolated": False,
                "sample": "500 steps in one run"}


class Gemm:
    """One product of config 5's MLP (131072 tokens x 512 -> 2048), C as the state."""
    metric = "GEMM steps/sec"
    bound = "tensor"
    scalar_output = False

    def __init__(self, name, m, k, n):
        self.name, self.m, self.k, self.n = name, m, k, n

    def build(self, F, world=1, rank=0, m=None):
        m = m or self.m
        rng = np.random.default_rng(0)
        a = F.tensor(rng.normal(size=(m, self.k)).astype("float32"))
        b = F.tensor((rng.normal(size=(self.k, self.n)) * 0.05).astype("float32"))
        return (lambda c, ab: ab[0] @ ab[1]), F.zeros((m, self.n)), [a, b]

    def flops(self, batch=None):
        return 2.0 * self.m * self.k * self.n

    def config(self, world):
        return {"workload": f"{self.name} {self.m}x{self.k} @ {self.k}x{self.n} f32", "parallelism": "replicas",
                "l2": "operands and result (1.3 GB) larger than L2"}

    def cpu_sample(self, F, oracle, full=False):
        m = 1024
        step, state, data = self.build(F, m=m)
        c = F.compile(step, (state, list(data)), validate="none", device="cpu")
        t = F.run(c, state, list(data), steps=1).elapsed
        return {"seconds_per_step": t * self.m / m, "sample_steps": 1, "sample_seconds": [t], "extrapolated": True,
                "sample": f"one product with {m} of {self.m} rows, scaled x{self.m // m} (the product is linear in its rows)"}


class Chain:
    """value and gradients of sum(A@B@C@D) and sum(x@(U@V)@x^T), compiled with
    optimize="search-linear" (the e-graph reorders both chains). A step recomputes both losses
    and all seven gradients; the gradients are the state (replaced every step)."""
    metric = "matrix-chain steps/sec"
    bound = "tensor"
    scalar_output = True

    def __init__(self, name, scale=1):
        self.name, self.scale = name, scale

    def inputs(self, F, scale=None):
        s = scale or self.scale
        n = 4096 // s
        rng = np.random.default_rng(0)
        mk = lambda *shape: F.tensor(rng.normal(size=shape).astype("float32"))
        return [mk(n, 16), mk(16, n), mk(n, 16), mk(16, n), mk(1024 // s, n), mk(n, 32), mk(32, n)]

    @staticmethod
    def losses(F):
        f1 = lambda a, b, c, d: (a @ b @ c @ d).sum()
        f2 = lambda x, u, v: (x @ (u @ v) @ F.swapaxes(x, 0, 1)).sum()

        def step(grads, args):
            a, b, c, d, x, u, v = args
            l1, g1 = F.value_and_grad(f1, argnums=(0, 1, 2, 3))(a, b, c, d)
            l2, g2 = F.value_and_grad(f2, argnums=(0, 1, 2))(x, u, v)
            return list(g1) + list(g2), l1 + l2
        return step

    def build(self, F, world=1, rank=0, scale=None):
        args = self.inputs(F, scale)
        return self.losses(F), [F.zeros(a.shape) for a in args], args

    def compile_options(self):
        return {"optimize": "search-linear"}

    def flops(self, batch=None):
        return 0.0

    def config(self, world):
        return {"workload": f"{self.name} A(4096,16)@B@C@D and x(1024,4096)@(U@V)@x^T, values and gradients, search-linear",
                "parallelism": "replicas", "l2": "operands and products larger than L2 (the 4096x4096 output of the first chain)"}

    def cpu_sample(self, F, oracle, full=False):
        step, state, data = self.build(F, scale=4)
        c = F.compile(step, (state, data), validate="none", device="cpu", optimize="search-linear")
        t = F.run(c, state, data, steps=1).elapsed
        return {"seconds_per_step": t * 16, "sample_steps": 1, "sample_seconds": [t], "extrapolated": True,
                "sample": "one step at a quarter of every large dimension (16x fewer multiplications), scaled x16"}


WORKLOADS = {
    "gpt-d512-l12": Gpt("gpt-d512-l12", vocab=96, block=256, d=512, heads=8, layers=12, batch=512, tokens="zipf"),
    "gpt-d256-l6": Gpt("gpt-d256-l6", vocab=96, block=256, d=256, heads=8, layers=6, batch=64, tokens="zipf"),
    "gpt-d128-l4": Gpt("gpt-d128-l4", vocab=96, block=128, d=128, heads=4, layers=4, batch=64, tokens="uniform"),
    # One d512 layer at batch 64, for ncu captures of the kernels of the benchmarked step on a case
    # that holds a few GB (each (B, H, T, T) tensor is 134 MB, above L2).
    "gpt-d512-l1": Gpt("gpt-d512-l1", vocab=96, block=256, d=512, heads=8, layers=1, batch=64, tokens="zipf"),
    "adamw-c2": AdamW("adamw-c2"),
    "linreg-c1": LinReg("linreg-c1"),
    "gemm-mlp": Gemm("gemm-mlp", m=131072, k=512, n=2048),
    "chain-c3": Chain("chain-c3"),
}


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


def traffic_for(workload, kernel):
    """DRAM bytes per launch of the dominant kernel class and what launch they were measured on,
    from the committed ncu summaries (dram__bytes_read.sum + dram__bytes_write.sum)."""
    try:
        with open(os.path.join(ROOT, "profiles", "traffic.json")) as f:
            t = json.load(f).get(workload, {}).get(kernel)
        return (t["bytes"], t["of"]) if t else (None, None)
    except (OSError, ValueError, KeyError):
        return None, None


def cpu_baseline(w, full=False):
    """The CPU oracle (restated rg interpreter) on all host threads, on a bounded sample.
    Returns the sample's record (cpu_sample) with the thread count."""
    sys.path.insert(0, os.path.join(ROOT, "oracle", "_build"))
    from rustautograd_b200 import build_ext
    build_ext.build_oracle()
    import _rg_oracle
    from rustautograd_b200 import frontend as F
    F.use(_rg_oracle, "cpu")
    rec = w.cpu_sample(F, _rg_oracle, full=full)
    rec["cores"] = _rg_oracle.threads()
    return rec


def roofline(w, compiled, secs, pk):
    """The dominant kernel class of a step by device time (CUDA events between plan steps)."""
    costs = compiled._n.step_costs()
    by_kind = {}
    for (kind, fl, by), s in zip(costs, secs):
        if kind == "row_chain" and fl == 0 and by == 0:
            continue  # the other steps of a row chain, which runs as one kernel at its first step
        e = by_kind.setdefault(kind, [0.0, 0.0, 0.0, 0])
        e[0] += s
        e[1] += fl
        e[2] += by
        e[3] += 1
    total = sum(v[0] for v in by_kind.values()) or 1e-30
    top = max(by_kind, key=lambda k: by_kind[k][0])
    t_s, fl, by, n = by_kind[top]
    if top in ("matmul", "attention"):
        # Tensor-core classes: the products' FLOPs (2 m n k; for the fused attention its q k^T,
        # P v and backward products) per second against the measured bf16 peak.
        achieved, peak, unit, bound = fl / t_s / 1e12, pk["bf16_tflops_sustained"], "TFLOP/s", "tensor"
    else:
        achieved, peak, unit, bound = by / t_s / 1e9, pk["hbm_gbs"], "GB/s", "hbm"
    fused = by_kind.get("fused", [1e-30, 0, 0, 0])
    chains = by_kind.get("row_chain")
    attn = by_kind.get("attention")
    gemm = by_kind.get("matmul")
    traffic, traffic_of = traffic_for(w.name, top)
    return {"bound": bound, "kernel": top, "achieved": achieved, "peak": peak, "unit": unit, "frac": achieved / peak,
            "peak_source": pk["source"], "traffic": traffic, "traffic_of": traffic_of, "launches_per_step": n, "share_of_step": t_s / total,
            "algorithmic_per_launch": (fl if top == "matmul" else by) / max(n, 1),
            "fused_elementwise": {"achieved_gbs": fused[2] / fused[0] / 1e9, "frac_of_hbm": fused[2] / fused[0] / 1e9 / pk["hbm_gbs"],
                                  "share_of_step": fused[0] / total},
            "row_chains": None if chains is None else {"achieved_gbs": chains[2] / chains[0] / 1e9, "frac_of_hbm": chains[2] / chains[0] / 1e9 / pk["hbm_gbs"],
                                                       "share_of_step": chains[0] / total, "launches_per_step": chains[3]},
            "gemm": None if gemm is None else {"achieved_tflops": gemm[1] / gemm[0] / 1e12, "frac_of_bf16_sustained": gemm[1] / gemm[0] / 1e12 / pk["bf16_tflops_sustained"],
                                               # fp32-accurate products run as three TF32 products at half the bf16 rate:
                                               # their ceiling is 1/6 of the bf16 peak.
                                               "frac_of_3xtf32_ceiling": gemm[1] / gemm[0] / 1e12 / (pk["bf16_tflops_sustained"] / 6),
                                               "share_of_step": gemm[0] / total, "launches_per_step": gemm[3]},
            "attention": None if attn is None else {"achieved_tflops": attn[1] / attn[0] / 1e12, "share_of_step": attn[0] / total,
                                                    "frac_of_3xtf32_ceiling": attn[1] / attn[0] / 1e12 / (pk["bf16_tflops_sustained"] / 6),
                                                    "ops_per_step": attn[3]}}


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--config", default="gpt-d512-l12", choices=sorted(WORKLOADS))
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--full-cpu-baseline", action="store_true",
                    help="GPT workloads: fit the CPU step time through batches 1 and 4 (as --impl reference does) instead of scaling batch 1")
    args = ap.parse_args()
    w = WORKLOADS[args.config]
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))

    if args.impl == "reference":
        # rg's CPU interpreter (the restatement under oracle/; rg itself cannot be built here) on
        # every host thread. It runs a bounded sample, not --steps global-batch steps: "steps" and
        # "ms_per_step" describe the sample steps that actually ran, and "value" is the
        # workload's steps/s derived from them as "extrapolation" states.
        if rank != 0:
            return
        rec = cpu_baseline(w, full=True)
        value = 1.0 / rec["seconds_per_step"]
        ran = sum(rec["sample_seconds"])
        print(json.dumps({
            "impl": "reference", "metric": w.metric, "value": value, "unit": "steps/s", "n_gpus": args.gpus,
            "steps": rec["sample_steps"], "warmup": 0, "ms_per_step": ran / rec["sample_steps"] * 1e3,
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "f32", "data": "synthetic", "config": w.config(args.gpus),
            "extrapolation": {"extrapolated": rec["extrapolated"], "sample_batches": rec.get("sample_batches"),
                              "sample_seconds": rec["sample_seconds"], "seconds_per_workload_step": rec["seconds_per_step"],
                              "method": rec.get("method", rec["sample"])},
            "cpu_baseline": {"value": value, "unit": "steps/s", "cores": rec["cores"], "kind": "port", "sample": rec["sample"]},
            "e2e": {"value": value, "unit": "steps/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        }))
        return

    # Libraries write banners to stdout (NCCL prints its version at communicator set-up); they go
    # to stderr, so that rank 0's stdout is the one JSON line.
    json_out = os.fdopen(os.dup(1), "w")
    sys.stdout.flush()
    os.dup2(2, 1)
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
        if not isinstance(w, Gpt):
            raise SystemExit(f"{args.config} runs on one GPU (replicas only); the data-parallel path is the GPT step")
        uid = [_rg.dist_unique_id() if rank == 0 else None]
        dist.broadcast_object_list(uid, src=0)
        _rg.dist_init(rank, world, uid[0])

    step, state, data = w.build(F, world, rank)
    data_arg = data[0] if len(data) == 1 else list(data)
    t0 = time.perf_counter()
    options = w.compile_options() if hasattr(w, "compile_options") else {}
    compiled = F.compile(step, (state, data_arg), validate="none", device="cuda", **options)
    compile_s = time.perf_counter() - t0
    n_state = len(F.flatten(state)[0])
    state_leaves = [F.tensor(l)._t for l in F.flatten(state)[0]]
    data_leaves = [F.tensor(l)._t for l in F.flatten(data_arg)[0]]
    state_map = [(k, k) for k in range(n_state)]
    data_inputs = list(range(n_state, n_state + len(data_leaves)))
    hist = [n_state] if w.scalar_output else []  # the step's scalar output (loss, or the step count)

    def run(steps):
        return compiled._n.run(state_map, data_inputs, hist, state_leaves, [data_leaves], steps)

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
    hist0 = history[0] if history else [None]
    state_bytes = sum(len(x.tobytes()) for x in state_leaves)
    data_bytes = sum(len(x.tobytes()) for x in data_leaves)

    # Per-step device times for the roofline, on every rank: the plan's all-reduce steps are
    # collectives.
    secs = compiled._n.step_seconds(state_leaves + data_leaves, 2)
    out = None
    if rank == 0:
        value = done / device_s
        pk = peaks()
        rf = roofline(w, compiled, secs, pk)
        if w.bound == "hbm":
            # The whole step is one bandwidth-bound update: report it against HBM directly.
            gbs = w.algorithmic_bytes() / (device_s / done) / 1e9
            rf.update({"bound": "hbm", "kernel": "step", "achieved": gbs, "peak": pk["hbm_gbs"], "unit": "GB/s", "frac": gbs / pk["hbm_gbs"],
                       "algorithmic_per_launch": w.algorithmic_bytes() / max(rf["launches_per_step"], 1)})
        cpu = None
        if not args.no_cpu_baseline:
            rec = cpu_baseline(w, full=args.full_cpu_baseline)
            cpu = {"value": 1.0 / rec["seconds_per_step"], "unit": "steps/s", "cores": rec["cores"], "kind": "port", "sample": rec["sample"],
                   "sample_steps": rec["sample_steps"], "sample_seconds": rec["sample_seconds"], "extrapolated": rec["extrapolated"]}
        cfg = dict(w.config(world), frame_bytes=compiled._n.allocated_bytes(), row_chains=os.environ.get("RGC_ROW_CHAINS") != "0")
        out = {
            "metric": w.metric, "value": value, "unit": "steps/s", "n_gpus": world, "steps": done, "warmup": args.warmup,
            "ms_per_step": device_s / done * 1e3, "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
            "dtype": "f32", "data": "synthetic", "config": cfg,
            "e2e": {"value": done / wall, "unit": "steps/s", "h2d_bytes_per_step": (state_bytes + data_bytes) / done,
                    "d2h_bytes_per_step": (state_bytes + 8 * done) / done},
            "gpu_launches": launches,
            "tflops_per_gpu": w.flops() / world * done / device_s / 1e12,
            "roofline": rf,
            "cpu_baseline": cpu,
            "clocks": clocks.summary(),
            "history": {"first": hist0[0], "last": hist0[-1], "nonfinite_step": bad},
            "compile_seconds": compile_s,
        }
    if dist:
        dist.barrier()
        _rg.dist_finalize()
        dist.destroy_process_group()
    if out is not None:
        print(json.dumps(out), file=json_out, flush=True)


if __name__ == "__main__":
    main()
