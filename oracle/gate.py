"""Oracle for the entropy gate (test infrastructure only).

Restates, in numpy, the reference's per-leaf gate on bf16 logits with the
rounding chain the reference's PyTorch CPU path applies (measured against the
reference itself; see ``tests/golden/make_golden.py``):

* ``compute_entropy`` (``core/generator_utils.py:196-202``)::

      xt = bf16(x / T)                     # float32 divide, one rounding
      m  = max(xt);  e = exp(xt - m);  S = sum(e)   (float32)
      p  = bf16(e / S)                     # softmax output
      lp = bf16((xt - m) - bf16(log(bf16(S))))   # log_softmax output
      H  = -float(bf16(sum_f32(bf16(p * lp))))   # nan_to_num(nan=0)

  The reference's CPU bf16 ``sum`` rounds per-thread partial sums to bf16, so
  its value depends on ``torch.get_num_threads()``.  The oracle (and the CUDA
  kernel) follow the single-thread result, which is the round-once sum.
* ``apply_repetition_penalty`` (``generator_utils.py:205-230``): over the
  unique generated tokens of the leaf, ``x > 0 -> bf16(x / p)`` else
  ``bf16(x * p)``.
* ``_do_extend`` (``core/generator.py:301-314``): ``argmax`` of the bf16
  ``log_softmax`` of the penalised logits, lowest index among equal values.
* ``_do_branch`` (``generator.py:275-298``): ``topk(K)`` of the same.  Ties are
  ordered by value, then lowest index.  (torch's CPU ``topk`` orders exactly
  equal values in an implementation-defined way; tests compare tie groups.)
* ``_step_leaf`` (``generator.py:333-374``), ``adaptive_threshold``
  (``generator_utils.py:247-253``), ``_soft_explore_factor``
  (``generator.py:319-331``): EMA, threshold and decision in Python double
  arithmetic.
"""

from __future__ import annotations

import math

import numpy as np


def bf16_round(a) -> np.ndarray:
    """Round float32 values to bf16 (round-to-nearest-even); float32 result."""
    a = np.array(a, dtype=np.float32)
    u = a.view(np.uint32).astype(np.uint64)
    r = (((u + 0x7FFF + ((u >> 16) & 1)) >> 16) << 16).astype(np.uint32)
    out = r.view(np.float32).copy()
    nan = np.isnan(a)
    if nan.any():
        out[nan] = np.float32("nan")
    return out.reshape(a.shape)


def bf16_bits_to_f32(bits) -> np.ndarray:
    return (np.asarray(bits, np.uint16).astype(np.uint32) << 16).view(np.float32)


def f32_to_bf16_bits(a) -> np.ndarray:
    return (bf16_round(a).view(np.uint32) >> 16).astype(np.uint16)


def _sum_f32(a: np.ndarray) -> np.float32:
    return np.float32(np.sum(a, dtype=np.float64))


_F = np.float32


def _hexf(h: str) -> np.float32:
    return np.float32(float.fromhex(h))  # the literals are exact float32 values


_LOG2E, _LN2_HI, _LN2_LO = _hexf("0x1.715476p+0"), _hexf("0x1.62e4p-1"), _hexf("0x1.7f7d1cp-20")
_EXP_POLY = [_hexf(h) for h in ("0x1.a01a02p-13", "0x1.6c16c2p-10", "0x1.111112p-7", "0x1.555556p-5",
                                "0x1.555556p-3")] + [_F(0.5), _F(1.0), _F(1.0)]


def exp_cw(d) -> np.ndarray:
    """e^d (d <= 0) in IEEE float32 multiplies and adds only: Cody and Waite's
    argument reduction (Cody, Waite, "Software Manual for the Elementary
    Functions", 1980; k = rint(d / ln2) by adding 1.5 * 2^23) and the degree-7
    Taylor polynomial of e^r, exactly the operations of the CUDA gate kernel's
    ``exp_cw``, so both give the same bits.
    The reference's torch CPU softmax uses its own vectorised expf; the two
    differ by about an ulp on some elements, which can move a probability
    across a bf16 rounding boundary (the residual mismatch the tests measure).
    Inputs below -87 give 0."""
    d = np.asarray(d, np.float32)
    ok = d >= _F(-87.0)
    d = np.where(ok, d, _F(0))
    # k = rint(d log2(e)): adding 1.5 * 2^23 rounds to an integer, ties to even
    kb = (d * _LOG2E + _F(12582912.0)).astype(np.float32)
    k = (kb - _F(12582912.0)).astype(np.float32)
    ki = kb.view(np.int32) - np.int32(0x4B400000)
    r = ((d - k * _LN2_HI) - k * _LN2_LO).astype(np.float32)
    p = _EXP_POLY[0]
    for c in _EXP_POLY[1:]:
        p = (p * r + c).astype(np.float32)
    scale = ((ki + 127) << 23).astype(np.int32).view(np.float32)
    return np.where(ok, (p * scale).astype(np.float32), _F(0)).astype(np.float32)


def softmax_parts(xt: np.ndarray, float_logsum: bool = False):
    """(m, e, S, L) of the bf16 softmax / log_softmax of bf16 values ``xt``:
    e = exp(xt - m) (float32), S = the float32 rounding of the exact sum of e,
    L = bf16(log(bf16(S))) with log correctly rounded to float32 (torch's CPU
    log_softmax), or L = log(S) in float32 with ``float_logsum`` (its CUDA one)."""
    m = np.float32(xt.max())
    with np.errstate(invalid="ignore", over="ignore"):
        e = exp_cw((xt - m).astype(np.float32))
    S = _sum_f32(e)
    if float_logsum:
        L = np.float32(np.log(np.float64(S)))
    else:
        L = bf16_round(np.float32(np.log(np.float64(bf16_round(S)[()]))))[()]
    return m, e, S, np.float32(L)


def log_softmax_bf16(z: np.ndarray, float_logsum: bool = False) -> np.ndarray:
    m, _, _, L = softmax_parts(z, float_logsum)
    with np.errstate(invalid="ignore"):
        return bf16_round((z - m).astype(np.float32) - L)


def entropy_bf16(x: np.ndarray, temperature: float = 1.0, float_logsum: bool = False) -> float:
    """``compute_entropy`` (``generator_utils.py:196-202``); x holds bf16 values."""
    x = np.asarray(x, np.float32)
    xt = bf16_round(x / np.float32(temperature)) if temperature != 1.0 else x.copy()
    m, e, S, L = softmax_parts(xt, float_logsum)
    with np.errstate(invalid="ignore", divide="ignore"):
        p = bf16_round(e / S)
        lp = bf16_round((xt - m).astype(np.float32) - L)
        plogp = bf16_round(p * lp)
    plogp = np.where(np.isnan(plogp), np.float32(0), plogp)
    s = bf16_round(_sum_f32(plogp))[()]
    return -float(s)


def entropy_f64(x: np.ndarray, temperature: float = 1.0) -> float:
    """Accurate entropy of softmax(x / T) (for the 1e-3-nat check)."""
    y = np.asarray(x, np.float64) / temperature
    y = y - y.max()
    p = np.exp(y)
    s = p.sum()
    p /= s
    lp = y - math.log(s)
    return float(-(p * lp)[p > 0].sum())


def apply_penalty(x: np.ndarray, history, penalty: float) -> np.ndarray:
    """``apply_repetition_penalty`` (``generator_utils.py:205-230``)."""
    x = np.asarray(x, np.float32)
    if len(history) == 0 or penalty == 1.0:
        return x
    z = x.copy()
    u = np.unique(np.asarray(list(history), np.int64))
    g = z[u]
    pf = np.float32(penalty)
    z[u] = np.where(g > 0, bf16_round(g / pf), bf16_round(g * pf))
    return z


def argmax_lowest(lp: np.ndarray) -> int:
    return int(np.argmax(lp))  # numpy returns the first maximal index


def topk_lowest(lp: np.ndarray, k: int):
    """Top-k by value desc, then index asc."""
    idx = np.lexsort((np.arange(lp.size), -lp.astype(np.float64)))[:k]
    return idx.astype(np.int64), lp[idx]


def adaptive_threshold(base: float, max_active: int, current: int) -> float:
    util = current / max(max_active, 1)
    return base * (1.0 + 2.0 * util * util)


def soft_explore_factor(step: int, window: int, initial: float) -> float:
    if step >= window:
        return 1.0
    t = step / max(window, 1)
    return initial + (1.0 - initial) * t


def decide(entropy: float, ema_old, *, alpha, mult, M, num_active, K, step,
           window, initial):
    """Branch decision of ``_step_leaf`` (``generator.py:342-369``).

    Returns ``(branch, ema_new, tau)``.
    """
    ema = entropy if ema_old is None else (alpha * entropy) + ((1.0 - alpha) * ema_old)
    dyn = adaptive_threshold(mult, M, num_active)
    warm = soft_explore_factor(step, window, initial)
    tau = ema * dyn * warm
    branch = (entropy > tau) and ((M - num_active) >= K)
    return branch, ema, tau


def gate_leaf(x, history, *, temperature, penalty, K, ema_old, alpha, mult, M,
              num_active, step, window, initial, float_logsum=False):
    """Everything ``_step_leaf`` computes for one leaf (``float_logsum``: the
    log-softmax rounding of torch's CUDA kernels instead of its CPU ones)."""
    x = np.asarray(x, np.float32)
    H = entropy_bf16(x, temperature, float_logsum)
    branch, ema, tau = decide(H, ema_old, alpha=alpha, mult=mult, M=M,
                              num_active=num_active, K=K, step=step,
                              window=window, initial=initial)
    z = apply_penalty(x, history, penalty)
    lp = log_softmax_bf16(z, float_logsum)
    am = argmax_lowest(lp)
    tk, tv = topk_lowest(lp, K)
    return {
        "entropy": H,
        "entropy_f64": entropy_f64(x, temperature),
        "ema": ema,
        "tau": tau,
        "branch": bool(branch),
        "argmax": am,
        "argmax_lp": float(lp[am]),
        "topk_ids": tk.tolist(),
        "topk_lps": [float(v) for v in tv],
        "pen_entropy": entropy_bf16(z, 1.0, float_logsum),
    }
