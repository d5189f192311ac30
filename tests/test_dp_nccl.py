"""Data parallelism on the CUDA device: two processes, one GPU each, NCCL all-reduce issued from
the plan. Needs two GPUs; with fewer the tests are skipped (the CPU gloo tests in
test_data_parallel.py cover the host-side logic everywhere)."""
import os
import socket

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _gpus():
    import torch
    return torch.cuda.device_count() if torch.cuda.is_available() else 0


def _model(F, world, rank, batch=8):
    model = F.gpt.GPT(vocab=40, block=16, d=32, heads=4, layers=2)
    params = model.init(F.random.key(0))
    opt = F.optim.adamw(1e-3, weight_decay=0.01)
    state = {"params": params, "opt": opt.init(params), "key": F.random.key(1)}
    tokens = F.tensor(np.random.default_rng(0).integers(0, 40, size=4000, dtype="int32"))
    return F.gpt.make_train_step(model, opt, batch, world, rank), state, tokens


def _rank(rank, world, port, out_dir, mode):
    import sys
    sys.path.insert(0, ROOT)
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0", RGC_COLLECTIVE_TIMEOUT_S="5",
                      RGC_TRACE_DIST="1")
    err = os.open(os.path.join(out_dir, f"rank{rank}.stderr"), os.O_WRONLY | os.O_CREAT | os.O_APPEND)
    os.dup2(err, 2)
    import datetime
    import faulthandler
    # Where each rank is blocked if it has not finished in time, for the failure message.
    trace = open(os.path.join(out_dir, f"rank{rank}.trace"), "w")
    faulthandler.dump_traceback_later(50, exit=False, file=trace)

    def progress(what):
        with open(os.path.join(out_dir, f"rank{rank}.progress"), "a") as f:
            f.write(what + "\n")
    import torch
    import torch.distributed as dist
    torch.cuda.set_device(rank)
    # gloo (CPU) only carries the NCCL id; the collectives are the plan's own.
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    from rustautograd_b200 import _rg
    from rustautograd_b200 import frontend as F
    F.use(_rg, "cuda")
    uid = [_rg.dist_unique_id() if rank == 0 else None]
    dist.broadcast_object_list(uid, src=0)
    _rg.dist_init(rank, world, uid[0])
    step, state, tokens = _model(F, world, rank)
    c = F.compile(step, (state, tokens), validate="none", device="cuda")
    dist.barrier()
    result = {}
    if mode == "train":
        r = F.run(c, state, tokens, steps=3)
        result = {"loss": np.array(r.history["aux"]), "leaves": [np.asarray(x.numpy()) for x in F.tree_leaves(r.state)]}
    elif mode == "stall":
        # One step together (the communicator's connections are up), then rank 1 leaves between
        # steps with nothing in flight; rank 0's next all-reduce has no partner and must end with
        # an error once the collective timeout has passed.
        F.run(c, state, tokens, steps=1)
        progress("first step done")
        dist.barrier()
        if rank == 1:
            np.save(os.path.join(out_dir, "rank1.npy"), np.array({}, dtype=object), allow_pickle=True)
            os._exit(0)
        try:
            F.run(c, state, tokens, steps=1)
            result = {"error": ""}
        except Exception as e:  # DiagnosticError from the device failure
            result = {"error": str(getattr(e, "diagnostic", e))}
        progress("second run returned: " + result["error"][:200])
    np.save(os.path.join(out_dir, f"rank{rank}.npy"), np.array(result, dtype=object), allow_pickle=True)
    _rg.dist_finalize()
    progress("finalized")
    faulthandler.cancel_dump_traceback_later()
    if mode != "stall":
        dist.destroy_process_group()


def _spawn(tmp_path, mode):
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    port = _free_port()
    procs = [ctx.Process(target=_rank, args=(r, 2, port, str(tmp_path), mode)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=150)
    for p in procs:
        if p.is_alive():
            p.kill()
    def read(name):
        path = os.path.join(tmp_path, name)
        return open(path).read() if os.path.exists(path) else ""
    if not all(p.exitcode == 0 for p in procs):
        pytest.fail(f"exit codes {[p.exitcode for p in procs]}\n" + "\n".join(
            f"--- rank{r}.{kind}\n{read(f'rank{r}.{kind}')[-4000:]}" for r in range(2) for kind in ("progress", "trace", "stderr")))
    return [np.load(os.path.join(tmp_path, f"rank{r}.npy"), allow_pickle=True).item() for r in range(2)]


@pytest.mark.skipif(_gpus() < 2, reason="needs two GPUs")
def test_two_gpu_training_matches_one_gpu(cuda, tmp_path):
    from rustautograd_b200 import frontend as F
    out = _spawn(tmp_path, "train")
    # Both ranks apply the same all-reduced update: their states are bit-identical.
    for a, b in zip(out[0]["leaves"], out[1]["leaves"]):
        np.testing.assert_array_equal(a, b)
    np.testing.assert_array_equal(out[0]["loss"], out[1]["loss"])
    # The full-batch step on one GPU: losses within 1e-4; parameters within the 2*lr*steps a
    # sign flip of Adam's noise-level updates can move them.
    F.use(cuda, "cuda")
    step, state, tokens = _model(F, 1, 0)
    c = F.compile(step, (state, tokens), validate="none", device="cuda")
    r = F.run(c, state, tokens, steps=3)
    ref = np.array(r.history["aux"])
    assert np.max(np.abs(out[0]["loss"] - ref) / np.abs(ref)) < 1e-4
    for a, b in zip(out[0]["leaves"], [np.asarray(x.numpy()) for x in F.tree_leaves(r.state)]):
        assert np.max(np.abs(a.astype(np.float64) - b)) <= 3 * 2e-3 + 1e-6


@pytest.mark.skipif(_gpus() < 2, reason="needs two GPUs")
def test_a_rank_that_stops_joining_ends_the_collective_with_an_error(cuda, tmp_path):
    out = _spawn(tmp_path, "stall")
    assert "collective waited more than" in out[0]["error"], out[0]
