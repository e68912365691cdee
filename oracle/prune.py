"""Oracle of semantic diversity pruning (test infrastructure only).

Restates the pair resolution of ``MentatGenerator._prune_similar``
(``core/generator.py:400-497``) on one tree's similarity matrix:

* the mask keeps the strict upper triangle (``torch.triu(..., diagonal=1)``,
  ``:447``) minus sibling pairs, the leaves sharing a non-None parent
  (``:451-455``);
* ``(sim * mask) > threshold`` (``:458-463``): a masked entry is compared as
  ``sim x 0``, and the comparison is made in the matrix's dtype (torch rounds
  the Python threshold to it);
* the pairs come in row-major order (``nonzero``), and a pair whose two leaves
  are both still unpruned prunes the one with the lower cumulative log-prob,
  the second leaf when ``lp_i >= lp_j`` (``:470-484``; False for NaN, which
  prunes the first).

``sim`` is a float array already rounded to the matrix dtype; ``threshold`` the
threshold rounded to that dtype.  Returns the set of pruned leaf indices.
"""

from __future__ import annotations

import numpy as np


def prune_pairs(sim: np.ndarray, parents, logp, threshold: float) -> set:
    m = sim.shape[0]
    mask = np.triu(np.ones((m, m), dtype=bool), k=1)
    for i in range(m):
        for j in range(i + 1, m):
            if parents[i] is not None and parents[i] == parents[j]:
                mask[i, j] = False
    with np.errstate(invalid="ignore"):
        masked = np.where(mask, sim, sim * np.float32(0.0))
        above = np.argwhere(masked > threshold)  # row-major, as nonzero()
    gone: set = set()
    for i, j in above:
        i, j = int(i), int(j)
        if i in gone or j in gone:
            continue
        gone.add(j if logp[i] >= logp[j] else i)
    return gone
