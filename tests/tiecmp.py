"""Tie-aware comparison of product-key top-k results.

Two implementations can legitimately disagree on the order or membership of
top-k entries whose scores differ by less than the rounding of the score
arithmetic (``torch.topk`` also leaves exact-tie order unspecified).  The
check used here:

* the score lists, both sorted descending, agree position by position
  within ``bound``;
* wherever the chosen slots differ, the other side's slot, re-scored with
  the checker's own full score matrix, is within ``bound`` of the checker's
  score at that position, i.e. the disagreement is a near-tie.

Rows that pass only through the second rule are counted and returned so the
tests can report (and bound) them.
"""
from __future__ import annotations

import numpy as np


def rescore(full_scores: np.ndarray, slots: np.ndarray, bf16: bool = False) -> np.ndarray:
    """Score of ``slot = i1*n + i2`` from full sub-scores ``[R, 2, n]``."""
    from oracle.pkm_oracle import bf16_round

    n = full_scores.shape[-1]
    i1 = slots // n
    i2 = slots % n
    s1 = np.take_along_axis(full_scores[:, 0, :], i1, axis=1)
    s2 = np.take_along_axis(full_scores[:, 1, :], i2, axis=1)
    s = (s1 + s2).astype(np.float32)
    return bf16_round(s) if bf16 else s


def compare_topk(check_scores, check_idx, other_scores, other_idx, full_scores, bound,
                 bf16: bool = False):
    """Return (n_exact_rows, n_tie_rows, worst) or raise AssertionError.

    ``check_*`` come from the checker whose ``full_scores`` are given;
    ``bound`` is an absolute tolerance (scalar or per-row array).
    """
    cs = np.asarray(check_scores, dtype=np.float64)
    os_ = np.asarray(other_scores, dtype=np.float64)
    ci = np.asarray(check_idx, dtype=np.int64)
    oi = np.asarray(other_idx, dtype=np.int64)
    assert cs.shape == os_.shape == ci.shape == oi.shape, (cs.shape, os_.shape)
    R, k = ci.shape
    b = np.broadcast_to(np.asarray(bound, dtype=np.float64).reshape(-1, 1) if np.ndim(bound) else bound,
                        (R, 1))
    gap = np.abs(cs - os_)
    bad_score = gap > b
    if bad_score.any():
        r = int(np.argwhere(bad_score.any(axis=1))[0][0])
        raise AssertionError(f"row {r}: score lists differ beyond bound: {cs[r]} vs {os_[r]}")
    exact = (ci == oi).all(axis=1)
    tie_rows = np.nonzero(~exact)[0]
    worst = 0.0
    if len(tie_rows):
        rs = rescore(full_scores[tie_rows], oi[tie_rows], bf16=bf16).astype(np.float64)
        d = np.abs(rs - cs[tie_rows])
        mism = ci[tie_rows] != oi[tie_rows]
        d = np.where(mism, d, 0.0)
        worst = float(d.max())
        viol = d > b[tie_rows]
        if viol.any():
            r = int(tie_rows[np.argwhere(viol.any(axis=1))[0][0]])
            raise AssertionError(
                f"row {r}: index mismatch not explained by a near-tie: {ci[r]} vs {oi[r]}")
    return int(exact.sum()), int(len(tie_rows)), worst
