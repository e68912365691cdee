"""Host-side pieces of the rollout, on CPU: the growable history arrays and the
semantic-vector table (its batched EMA update must give the reference's
per-leaf ``clone`` / ``mul_(1 - a).add_(h, alpha=a)``, ``generator.py:376-398``)."""

import numpy as np
import torch

from mentat_b200.rollout import Node, _Hist, _SemTable


def test_history_grows_and_branches_copy():
    h = _Hist()
    for t in range(150):
        h.append(t)
    g = h.plus(999)
    h.append(7)
    assert h.view().tolist() == list(range(150)) + [7]
    assert g.view().tolist() == list(range(150)) + [999]
    assert h.view().dtype == np.int32


def test_semantic_table_matches_per_leaf_updates():
    torch.manual_seed(0)
    tab = _SemTable(16, torch.bfloat16, "cpu", cap=2)
    leaves = [Node(node_id=i) for i in range(3)]
    ref = [None] * 3
    a = 0.3
    for step in range(5):
        hidden = torch.randn(len(leaves), 16).to(torch.bfloat16)
        tab.update(leaves, hidden, a)
        for i in range(len(leaves)):
            if ref[i] is None:
                ref[i] = hidden[i].clone()
            else:
                ref[i].mul_(1.0 - a).add_(hidden[i], alpha=a)
        if step == 2:  # leaf 0 branches: its child starts from a copy of its row
            leaves.append(Node(node_id=9, sem_row=tab.copy_row(leaves[0].sem_row)))
            ref.append(ref[0].clone())
    got = tab.rows([lf.sem_row for lf in leaves])
    # bf16 to one rounding step: torch's CPU kernels round the vectorised body and the
    # scalar tail of a row differently, so a batched and a per-row update can differ in
    # the last bit (on the GPU every element takes the same path)
    for i in range(len(leaves)):
        torch.testing.assert_close(got[i].float(), ref[i].float(), rtol=8e-3, atol=8e-3)
    assert tab.n == 4 and tab.t.shape[0] >= 4  # grown past its initial capacity of 2
