"""Helpers shared by the GPU tests (fixtures only; the reference is not imported)."""

import json
import os

import numpy as np
import torch

from oracle.gate import bf16_round
from tests.golden.cases import build_tree_ops

HERE = os.path.dirname(os.path.abspath(__file__))
TORCH_DT = {"f32": torch.float32, "bf16": torch.bfloat16, "f16": torch.float16}


def load_streams():
    with open(os.path.join(HERE, "golden", "alloc_streams.json")) as f:
        return json.load(f)


def round_np(a, dtype):
    if dtype == "bf16":
        return bf16_round(a)
    if dtype == "f16":
        return a.astype(np.float16).astype(np.float32)
    return a.astype(np.float32)


def build_tree(mgr, c, inp, dev="cuda"):
    """Run the case's tree ops through a cache manager; return the leaf seq ids."""
    dt = TORCH_DT[c["dtype"]]
    leaves = []
    for op in build_tree_ops(c):
        if op[0] == "append":
            k = torch.from_numpy(inp[op[2]]).to(dev).to(dt)
            v = torch.from_numpy(inp[op[3]]).to(dev).to(dt)
            mgr.append_tokens(op[1], 0, k, v)
        elif op[0] == "alloc":
            mgr.allocate_sequence()
        elif op[0] == "fork":
            mgr.fork_sequence(op[1])
        elif op[0] == "free":
            mgr.free_sequence(op[1])
        else:
            leaves = op[1]
    return leaves
