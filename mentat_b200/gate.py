"""Batched entropy gate: one kernel launch and one device-to-host read per step.

``Gate`` evaluates, for every active leaf at once, what the reference's
``MentatGenerator._step_leaf`` (``core/generator.py:333-374``) computes one leaf
at a time with several host synchronisations: the entropy at temperature T
(``generator_utils.py:196-202``), the EMA and threshold
(``generator.py:345-360``, ``generator_utils.py:247-253``,
``generator.py:319-331``), the repetition penalty over the leaf's generated
tokens (``generator_utils.py:205-230``), the branch decision
(``generator.py:368-369``) and the top-K / argmax of the penalised
log-softmax (``generator.py:283-287,308-310``).
"""

from __future__ import annotations

import ctypes as C
import math
from dataclasses import dataclass

import numpy as np
import torch

from . import _lib, ops

_DT = {torch.bfloat16: _lib.MENTAT_BF16, torch.float16: _lib.MENTAT_F16, torch.float32: _lib.MENTAT_F32}

GATE_OUT_DTYPE = np.dtype([
    ("entropy", "<f8"), ("entropy_acc", "<f8"), ("pen_entropy", "<f8"), ("ema", "<f8"),
    ("tau", "<f8"), ("branch", "<i4"), ("argmax", "<i4"), ("argmax_lp", "<f4"),
    ("topk_ids", "<i4", (_lib.GATE_MAXK,)), ("topk_lps", "<f4", (_lib.GATE_MAXK,)),
    ("pad", "<i4", (3,)),
])
assert GATE_OUT_DTYPE.itemsize == C.sizeof(_lib.GateOut)


@dataclass
class GateConfig:
    """Generator knobs the gate reads (``generator.py:29-52`` defaults)."""
    temperature: float = 0.7
    repetition_penalty: float = 1.2
    entropy_ema_alpha: float = 0.3
    relative_entropy_multiplier: float = 1.25
    soft_explore_initial: float = 0.3
    branching_factor: int = 3
    max_active_branches: int = 10
    soft_explore_window: int = 10
    # the penalised entropy serves only the reference's branch-point diagnostics
    # (generator.py:291-293); False leaves it out of the kernel (0 in the record)
    pen_entropy: bool = True
    # log-softmax rounding: "cpu" rounds log(sum) to the logits dtype as torch's
    # CPU kernels do (pinned by the golden fixtures); "cuda" keeps it in float as
    # torch's CUDA kernels do
    log_softmax: str = "cpu"


class Gate:
    """Reusable gate with pinned staging buffers for one device."""

    def __init__(self, device, cfg: GateConfig):
        self.device = torch.device(device)
        self.cfg = cfg
        self.lib = _lib.load()
        self._cap = 0
        self._hist_cap = 0
        self._n = 0

    def _ensure(self, n: int, nh: int):
        if n > self._cap:
            self._cap = max(n, 2 * self._cap, 16)
            nb = self._cap * GATE_OUT_DTYPE.itemsize
            self._out_dev = torch.empty(nb, dtype=torch.uint8, device=self.device)
            self._out_host = torch.empty(nb, dtype=torch.uint8, pin_memory=True)
            self._ptr_host = torch.empty(self._cap + 1, dtype=torch.int32, pin_memory=True)
            self._ptr_dev = torch.empty(self._cap + 1, dtype=torch.int32, device=self.device)
            self._ema_host = torch.empty(self._cap, dtype=torch.float64, pin_memory=True)
            self._ema_dev = torch.empty(self._cap, dtype=torch.float64, device=self.device)
        if nh > self._hist_cap or self._hist_cap == 0:
            self._hist_cap = max(nh, 2 * self._hist_cap, 1024)
            self._hist_host = torch.empty(self._hist_cap, dtype=torch.int32, pin_memory=True)
            self._hist_dev = torch.empty(self._hist_cap, dtype=torch.int32, device=self.device)

    def launch(self, logits: torch.Tensor, histories, ema_old, *, num_active: int, step: int) -> None:
        """Enqueue the gate for ``logits`` (N, V); read results with :meth:`result`."""
        n, V = logits.shape
        if logits.stride(1) != 1:
            logits = logits.contiguous()
        lens = [len(h) for h in histories]
        nh = sum(lens)
        self._ensure(n, nh)
        ptr = np.zeros(n + 1, np.int32)
        ptr[1:] = np.cumsum(lens)
        self._ptr_host.numpy()[: n + 1] = ptr
        if nh:
            self._hist_host.numpy()[:nh] = np.concatenate([np.asarray(h, dtype=np.int32) for h in histories if len(h)])
        self._ema_host.numpy()[:n] = [math.nan if e is None else e for e in ema_old]
        self._ptr_dev[: n + 1].copy_(self._ptr_host[: n + 1], non_blocking=True)
        if nh:
            self._hist_dev[:nh].copy_(self._hist_host[:nh], non_blocking=True)
        self._ema_dev[:n].copy_(self._ema_host[:n], non_blocking=True)
        c = self.cfg
        nb = n * GATE_OUT_DTYPE.itemsize
        ops.gate_step(
            logits, self._ptr_dev[: n + 1], self._hist_dev, self._ema_dev[:n],
            [c.temperature, c.repetition_penalty, c.entropy_ema_alpha, c.relative_entropy_multiplier,
             c.soft_explore_initial],
            [c.branching_factor, c.max_active_branches, num_active, step, c.soft_explore_window,
             (0 if c.pen_entropy else _lib.GATE_SKIP_PEN_ENTROPY)
             | (_lib.GATE_FLOAT_LOGSUM if c.log_softmax == "cuda" else 0)],
            self._out_dev[:nb])
        self._out_host[:nb].copy_(self._out_dev[:nb], non_blocking=True)
        self._n = n

    def result(self) -> np.ndarray:
        torch.cuda.current_stream(self.device).synchronize()
        nb = self._n * GATE_OUT_DTYPE.itemsize
        return np.frombuffer(self._out_host.numpy()[:nb].tobytes(), dtype=GATE_OUT_DTYPE)


def gate_step(logits: torch.Tensor, histories, ema_old, cfg: GateConfig, *, num_active: int, step: int) -> np.ndarray:
    """One-shot convenience wrapper around :class:`Gate`."""
    g = Gate(logits.device, cfg)
    g.launch(logits, histories, ema_old, num_active=num_active, step=step)
    return g.result()
