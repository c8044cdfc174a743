"""Loads the golden fixtures and regenerates their (unstored) inputs from the seeds."""

from pathlib import Path

import numpy as np
import torch

from exp3_b200 import synthetic

GOLDEN = Path(__file__).resolve().parent / "golden"
SCALE = 128 ** -0.5


def load(name):
    """Returns (fixture dict, q, k, v) with bf16 inputs checked against the stored digest."""
    data = dict(np.load(GOLDEN / name, allow_pickle=False))
    shape = synthetic.LayerShape(1, int(data["length"]), int(data["heads"]), int(data["kv_heads"]),
                                 int(data.get("head_dim", 128)))
    q, k, v = synthetic.attention_inputs(shape, seed=int(data["seed"]), needles=2, apply_rope=True)
    digest = synthetic.tensor_digest(q, k, v)
    assert digest == str(data["digest"]), (
        f"{name}: regenerated inputs differ from those the fixture was made from; "
        "rerun tests/golden/make_golden.py")
    return data, q, k, v


def t(array, dtype=None):
    x = torch.from_numpy(np.asarray(array))
    return x if dtype is None else x.to(dtype)
