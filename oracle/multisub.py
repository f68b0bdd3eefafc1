"""Numpy restatement of one step of the multi-subbox input-split BaB (test
oracle: only tests import it).

Follows the inner loop of ``_multi_sub_input_split_bab``
(``verify_graph.py:11180-11922``) after the forward-LiRPA bound:

* ``leaf_fate``: safe when any query's margin (lower bound + the sub-box's
  query bias) is positive (:11640-11660); otherwise ``clip_iters`` rounds of
  ``_clip_input_domain`` (:11121-11177) over the varying dimensions, the
  leaf safe when the box comes out empty (:11695-11734); otherwise the
  smart-branching score max_q(max(|A_qk|, 0.1) * width_k * 0.5 + margin_q)
  on the pre-clip widths, -inf on dimensions that do not vary or are at most
  1e-12 wide after the clip (:11780-11802);
* ``emit_children``: top-K dimensions in CPU torch.topk order, 2^K children
  per leaf, bit j set = high half of the j-th ranked dimension, a dimension
  at most 1e-12 wide left whole (:11816-11852).

Every operation is float32 and rounded as the reference's tensor expression
rounds it; sums over dimensions run in dimension order.
"""
from __future__ import annotations

import numpy as np

from .bab import topk_cpu_order

F32 = np.float32


def clip_input_domain(xl, xh, lA, lbias, num_iters=1):
    """(x_L, x_U) after ``num_iters`` rounds of the closed-form clip:
    xl, xh (B, K); lA (B, S, K); lbias (B, S) including the query bias."""
    xl = np.array(xl, F32)
    xh = np.array(xh, F32)
    lA = np.asarray(lA, F32)
    lbias = np.asarray(lbias, F32)
    B, S, K = lA.shape
    for _ in range(num_iters):
        lo = np.zeros((B, S), F32)
        for k in range(K):
            a = lA[:, :, k]
            lo = lo + (np.maximum(a, F32(0)) * xl[:, None, k]
                       + np.minimum(a, F32(0)) * xh[:, None, k])
        lo = lo + lbias
        mid = (xh + xl) * F32(0.5)
        rad = (xh - xl) * F32(0.5)
        rest = lo[:, :, None] - (lA * mid[:, None, :] - np.abs(lA) * rad[:, None, :])
        denom = np.where(np.abs(lA) > F32(1e-30), lA, F32(1))
        x0 = -rest / denom
        nh = np.where(lA > 0, x0, F32(np.inf)).min(axis=1)
        nl = np.where(lA < 0, x0, F32(-np.inf)).max(axis=1)
        xh, xl = np.minimum(nh, xh), np.maximum(nl, xl)
    return xl, xh


def leaf_fate(xl, xh, var_idx, spec_A, spec_b, lb, sub_bias, sub, clip_iters=2):
    """(fate (B + 1), box_lo, box_hi, score) as ``vcb_multisub_fate`` defines
    them; rows that are not split keep NaN in box_lo / box_hi / score."""
    xl = np.asarray(xl, F32)
    xh = np.asarray(xh, F32)
    var_idx = np.asarray(var_idx, np.int64)
    B, n = xl.shape
    bias = np.asarray(sub_bias, F32)[np.asarray(sub, np.int64)]
    margin = np.asarray(lb, F32) + bias
    safe = (margin > 0).any(axis=1)
    fate = np.zeros(B + 1, np.int32)
    box_lo = np.full((B, n), np.nan, F32)
    box_hi = np.full((B, n), np.nan, F32)
    score = np.full((B, n), np.nan, F32)
    u = np.nonzero(~safe)[0]
    if u.size:
        cl0, ch0 = xl[u][:, var_idx], xh[u][:, var_idx]
        lA = np.asarray(spec_A, F32)[u]
        cl, ch = clip_input_domain(cl0, ch0, lA, np.asarray(spec_b, F32)[u] + bias[u],
                                   clip_iters)
        empty = (cl > ch).any(axis=1)
        fate[u] = np.where(empty, 1, 2)
        s = u[~empty]
        keep = ~empty
        box_lo[s], box_hi[s] = xl[s], xh[s]
        box_lo[s[:, None], var_idx[None, :]] = cl[keep]
        box_hi[s[:, None], var_idx[None, :]] = ch[keep]
        w0 = (ch0 - cl0)[keep]
        sc = (np.maximum(np.abs(lA[keep]), F32(0.1)) * w0[:, None, :] * F32(0.5)
              + margin[s][:, :, None] * F32(1.0)).max(axis=1)
        full = np.full((s.size, n), -np.inf, F32)
        full[:, var_idx] = sc
        wide = (box_hi[s] - box_lo[s]) > F32(1e-12)
        score[s] = np.where(wide, full, F32(-np.inf))
        fate[B] = int(wide.sum(axis=1).max()) if s.size else 0
    return fate, box_lo, box_hi, score


def emit_children(rows, xl, xh, score, sub, k):
    """(kid_xl, kid_xh, kid_sub) as ``vcb_multisub_emit`` defines them."""
    xl = np.asarray(xl, F32)
    xh = np.asarray(xh, F32)
    sub = np.asarray(sub)
    n = xl.shape[1]
    nch = 1 << k
    kxl, kxh, ksub = [], [], []
    for b in np.asarray(rows, np.int64):
        top = topk_cpu_order(np.asarray(score[b], F32), k)
        for c in range(nch):
            lo, hi = xl[b].copy(), xh[b].copy()
            for j, d in enumerate(top):
                if xh[b, d] - xl[b, d] > F32(1e-12):
                    mid = (xl[b, d] + xh[b, d]) * F32(0.5)
                    if (c >> j) & 1:
                        lo[d] = mid
                    else:
                        hi[d] = mid
            kxl.append(lo)
            kxh.append(hi)
            ksub.append(sub[b])
    if not kxl:
        return np.zeros((0, n), F32), np.zeros((0, n), F32), np.zeros(0, np.int32)
    return np.stack(kxl), np.stack(kxh), np.asarray(ksub, np.int32)
