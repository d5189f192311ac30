"""Data-parallel GPT step on two CPU ranks (gloo): the per-rank plans with their `all_reduce`
steps reproduce the single-process full-batch step. The same plans run on the CUDA device with
NCCL; here the oracle executes them and torch.distributed supplies the cross-rank sum."""
import os
import socket

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def gpt_step_outputs(F, world, rank, batch=4):
    model = F.gpt.GPT(vocab=13, block=8, d=16, heads=2, layers=2)
    params = F.tree_map(lambda v: v.cast("float64"), model.init(F.random.key(3)))
    opt = F.optim.adamw(1e-2, weight_decay=0.01)
    state = {"params": params, "opt": opt.init(params), "key": F.random.key(4)}
    tokens = F.tensor(np.random.default_rng(2).integers(0, 13, size=500, dtype="int32"))
    step = F.gpt.make_train_step(model, opt, batch, world, rank)
    c = F.compile(step, (state, tokens), validate="none", device="cpu")
    new_state, loss = c(state, tokens)
    return [x.numpy() for x in F.tree_leaves(new_state)], float(loss)


def _rank(rank, world, port, out_dir):
    import sys
    sys.path.insert(0, ROOT)
    sys.path.insert(0, os.path.join(ROOT, "oracle", "_build"))
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    import torch
    import torch.distributed as dist
    import datetime
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    import _rg_oracle
    from rustautograd_b200 import frontend as F

    def all_reduce(data, dtype):
        t = torch.frombuffer(bytearray(data), dtype={"float32": torch.float32, "float64": torch.float64}[dtype]).clone()
        dist.all_reduce(t)
        return t.numpy().tobytes()
    _rg_oracle.set_all_reduce(all_reduce)
    F.use(_rg_oracle, "cpu")
    leaves, loss = gpt_step_outputs(F, world, rank)
    np.savez(os.path.join(out_dir, f"rank{rank}.npz"), loss=loss, *leaves)
    _rg_oracle.set_all_reduce(None)
    dist.destroy_process_group()


def test_two_rank_step_equals_full_batch_step(oracle, tmp_path):
    mp = pytest.importorskip("torch.multiprocessing")
    from rustautograd_b200 import frontend as F
    F.use(oracle, "cpu")
    oracle.set_all_reduce(None)
    full, full_loss = gpt_step_outputs(F, 1, 0)
    port = free_port()
    mp.spawn(_rank, args=(2, port, str(tmp_path)), nprocs=2, join=True)
    ranks = [np.load(tmp_path / f"rank{r}.npz") for r in range(2)]
    for r in ranks:
        assert abs(float(r["loss"]) - full_loss) <= 1e-12 * abs(full_loss)
        for k, want in enumerate(full):
            got = r[f"arr_{k}"]
            if want.dtype.kind == "i":
                np.testing.assert_array_equal(got, want)
            else:
                np.testing.assert_allclose(got, want, rtol=1e-10, atol=1e-13)
    # Both ranks hold bit-identical replicated state after the all-reduced update.
    for k in range(len(full)):
        np.testing.assert_array_equal(ranks[0][f"arr_{k}"], ranks[1][f"arr_{k}"])


def test_device_plan_runs_the_all_reduces_after_the_backward(oracle):
    """For the device, the planner emits the all-reduces and what depends on them (the AdamW
    update, the reported loss) after every other step, so the all-reduces are consecutive steps
    (one staged NCCL operation on the GPU) instead of one between every pair of backward
    pieces. Plan order only: rg's CPU plan keeps its own order."""
    import json
    from rustautograd_b200 import frontend as F
    F.use(oracle, "cpu")
    model = F.gpt.GPT(vocab=13, block=8, d=16, heads=2, layers=2)
    params = model.init(F.random.key(3))
    opt = F.optim.adamw(1e-2, weight_decay=0.01)
    state = {"params": params, "opt": opt.init(params), "key": F.random.key(4)}
    tokens = F.tensor(np.random.default_rng(2).integers(0, 13, size=500, dtype="int32"))
    step = F.gpt.make_train_step(model, opt, 4, 2, 0)
    c = F.compile(step, (state, tokens), validate="none", device="cuda-plan")
    ops = [p.get("op") for p in json.loads(c._n.plan_summary()) if "op" in p or "fused" in p]
    at = [i for i, op in enumerate(ops) if op == "all_reduce"]
    assert len(at) == len(F.tree_leaves(params)) + 1  # every gradient and the loss
    assert at == list(range(at[0], at[0] + len(at))), "the all-reduces are consecutive steps"
