"""Device-resident sessions on the CUDA device: the GPT training state stays in HBM between
runs, checkpoints stream from the device frame into a safetensors file (and back) through pinned
memory, and save / restore / continue reproduces one uninterrupted run bit for bit."""
import numpy as np
import pytest

from rustautograd_b200 import frontend as F
from helpers import assert_bits_equal

pytestmark = pytest.mark.gpu


def _gpt():
    model = F.gpt.GPT(vocab=40, block=16, d=32, heads=4, layers=2)
    params = model.init(F.random.key(0))
    opt = F.optim.adamw(1e-3, weight_decay=0.01)
    state = {"params": params, "opt": opt.init(params), "key": F.random.key(1)}
    tokens = F.tensor(np.random.default_rng(0).integers(0, 40, size=4000, dtype="int32"))
    return F.gpt.make_train_step(model, opt, 8), state, tokens


def test_gpu_session_checkpoint_round_trip(cuda, tmp_path):
    F.use(cuda, "cuda")
    step, state, tokens = _gpt()
    c = F.compile(step, (state, tokens), validate="none", device="cuda")
    full = F.run(c, state, tokens, steps=10)
    s = F.Session(c, state, tokens)
    h1 = s.run(4).history["aux"]
    h2 = s.run(2).history["aux"]
    path = str(tmp_path / "gpt.safetensors")
    s.save(path, {"steps": "6"})
    at6 = s.state
    h3 = s.run(4).history["aux"]
    assert list(h1) + list(h2) + list(h3) == list(full.history["aux"])
    for a, b in zip(F.tree_leaves(s.state), F.tree_leaves(full.state)):
        assert_bits_equal(a.numpy(), b.numpy(), "state after 10 steps")
    # The file is an ordinary checkpoint of the state at step 6 ...
    tree, meta = F.checkpoint.load(path, with_metadata=True)
    assert meta == {"steps": "6"}
    for a, b in zip(F.tree_leaves(tree), F.tree_leaves(at6)):
        assert_bits_equal(a.numpy(), b.numpy(), "checkpoint")
    # ... and a new session restored from it continues exactly.
    s2 = F.Session(c, state, tokens)
    s2.restore(path)
    assert list(s2.run(4).history["aux"]) == list(h3)
    for a, b in zip(F.tree_leaves(s2.state), F.tree_leaves(full.state)):
        assert_bits_equal(a.numpy(), b.numpy(), "restored run")
