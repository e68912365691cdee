"""Semantic pruning's pair resolution on the device (``mentat_prune_similar``)
against the reference's ``_prune_similar`` (``generator.py:400-497``, fixtures in
tests/golden/prune.json: the reference's own similarity matrices and pruned
leaves) and against the oracle (``oracle.prune``) on random trees: many leaves
(rows of several 32-column chunks), thresholds at and below zero, tied and NaN
log-probs, sibling groups, several trees in one call.  Integer decisions:
bit-exact."""

import json
import os

import numpy as np
import pytest
import torch

from oracle.prune import prune_pairs
from tests.gpu_util import HERE, TORCH_DT

pytestmark = pytest.mark.gpu


def _run(blocks, dtype):
    """blocks: list of (sim (m, m) float32 already rounded to dtype, parents, logp,
    thr); all trees in one block-diagonal matrix and one call."""
    from mentat_b200 import ops
    sizes = [b[0].shape[0] for b in blocks]
    off = np.concatenate([[0], np.cumsum(sizes)]).astype(np.int32)
    m = int(off[-1])
    sim = np.full((m, m), np.nan, np.float32)  # entries between trees must not be read
    keys, logp = [], []
    for g, (s, par, lp, _) in enumerate(blocks):
        a = off[g]
        sim[a:a + s.shape[0], a:a + s.shape[0]] = s
        keys += [(-1 - (a + i)) if p is None else int(p) for i, p in enumerate(par)]
        logp += list(lp)
    thr = blocks[0][3]
    assert all(b[3] == thr for b in blocks)
    dev = "cuda"
    flags = ops.prune_similar(torch.from_numpy(sim).to(dev).to(TORCH_DT[dtype]),
                              torch.from_numpy(off).to(dev), torch.tensor(keys, dtype=torch.int64, device=dev),
                              torch.tensor(logp, dtype=torch.float64, device=dev), thr, max(sizes) if sizes else 0)
    f = flags.cpu().numpy()
    return [set(np.nonzero(f[off[g]:off[g + 1]])[0].tolist()) for g in range(len(blocks))]


def test_prune_matches_reference_fixtures():
    with open(os.path.join(HERE, "golden", "prune.json")) as fh:
        g = json.load(fh)
    for name, c in g.items():
        n = len(c["node_id"])
        if n == 0:
            continue
        sim = np.asarray(c["sim"], np.float32).reshape(n, n)
        (gone,) = _run([(sim, c["parent"], c["logp"], c["thr"])], c["dtype"])
        assert [c["node_id"][i] for i in sorted(gone)] == c["pruned"], name


def _round(a, dtype):
    return torch.from_numpy(a).to(TORCH_DT[dtype]).float().numpy()


@pytest.mark.parametrize("dtype,thr", [("f32", 0.85), ("bf16", 0.85), ("f32", 0.0), ("bf16", -0.1)])
def test_prune_matches_oracle_random_trees(dtype, thr):
    rng = np.random.default_rng(7)
    thr_r = float(torch.tensor(thr, dtype=TORCH_DT[dtype]).item())
    blocks = []
    for m in (1, 2, 31, 32, 33, 64, 97, 300):
        x = rng.standard_normal((m, 16)) + 3.0 * rng.standard_normal((1, 16))  # correlated: many sims near 1
        x /= np.linalg.norm(x, axis=1, keepdims=True)
        s = _round((x @ x.T).astype(np.float32), dtype)
        par = [None if p < 0 else int(p) for p in rng.integers(-1, max(1, m // 5), m)]
        lp = np.round(rng.standard_normal(m), 1)
        lp[rng.random(m) < 0.05] = np.nan
        blocks.append((s, par, lp.tolist(), thr_r))
    got = _run(blocks, dtype)
    for (s, par, lp, t), gone in zip(blocks, got):
        assert gone == prune_pairs(s, par, lp, t), (s.shape, dtype, thr)


def test_prune_argument_errors():
    from mentat_b200 import _lib
    lib = _lib.load()
    assert lib.mentat_prune_similar(None, 0, 0, None, 0, 0, None, None, 0.0, None, None) == 0
    assert lib.mentat_prune_similar(None, 0, 0, None, 1, 5000, None, None, 0.0, None, None) == -1  # MENTAT_ERR_ARG: a tree above 4,096 leaves
