"""Numpy restatement of the batched input-split BaB driver (test oracle).

Follows ``_input_split_batched_inner`` (``verify_graph.py:12511-13464``) on the
default path: LIFO chunk worklist (:12695-12726), pop B (:12846), bound with
CROWN or zonotope intermediates + CROWN spec backward with the input-space
linear form (:12855-12870), closure "every disjunct has a query with lb > 0"
(:12901-12908), one round of halfspace clipping (:13030-13130), widest-axis
(or sum-|A| sensitivity) split dim via first-max argmax (:13236-13295), the
vectorised bisection with the 1e-12 degenerate guard and children pushed
low-chunk then high-chunk (:13353-13382), the max_worklist overflow check
(:13424-13429) and the verdict (:13452-13464).  Root PGD, alpha-CROWN,
leaf-PGD and MILP escalation are not part of this restatement.
"""
from __future__ import annotations

import time

import numpy as np

from . import bounds as ob


def input_split_bab(gg, x_lo, x_hi, spec_W, spec_b, disj_q=None,
                    batch_size=4096, max_worklist=200_000,
                    crown_intermediate=True, clip_enabled=True,
                    branch_sb=False, timeout=60.0, max_iters=None,
                    dtype=np.float32, trace=None):
    """Returns (verdict, details) like the reference driver."""
    spec_W = np.asarray(spec_W, dtype)
    spec_b = np.asarray(spec_b, dtype)
    Q = spec_W.shape[0]
    if disj_q is None:
        disj_q = [list(range(Q))]
    multi = len(disj_q) > 1
    t0 = time.perf_counter()
    wl_xl = [np.asarray(x_lo, dtype).reshape(1, -1)]
    wl_xh = [np.asarray(x_hi, dtype).reshape(1, -1)]
    n_leaves = 0
    n_iters = 0
    n_open = 0

    def wl_size():
        return sum(c.shape[0] for c in wl_xl)

    def wl_pop(n):
        got = 0
        pxl, pxh = [], []
        while got < n:
            cxl, cxh = wl_xl[-1], wl_xh[-1]
            m = cxl.shape[0]
            if got + m <= n:
                pxl.append(cxl)
                pxh.append(cxh)
                wl_xl.pop()
                wl_xh.pop()
                got += m
            else:
                need = n - got
                pxl.append(cxl[m - need:])
                pxh.append(cxh[m - need:])
                wl_xl[-1] = cxl[:m - need]
                wl_xh[-1] = cxh[:m - need]
                got = n
        return (pxl[0] if len(pxl) == 1 else np.concatenate(pxl, 0),
                pxh[0] if len(pxh) == 1 else np.concatenate(pxh, 0))

    while wl_xl:
        wn = wl_size()
        if time.perf_counter() - t0 > timeout - 0.5 or (
                max_iters is not None and n_iters >= max_iters):
            n_open = wn
            break
        B = min(batch_size, wn)
        xl_b, xh_b = wl_pop(B)
        if crown_intermediate:
            sb_b = ob.crown_intermediate_batched(gg, xl_b, xh_b, dtype=dtype)
        else:
            sb_b, _ = ob.forward_zonotope_batched(xl_b, xh_b, gg, dtype)
        if clip_enabled:
            lbs, A_lin, b_lin = ob.spec_backward_batched(
                sb_b, xl_b, xh_b, gg, spec_W, spec_b,
                return_input_linear=True, dtype=dtype)
        else:
            lbs = ob.spec_backward_batched(sb_b, xl_b, xh_b, gg, spec_W,
                                           spec_b, dtype=dtype)
            A_lin = b_lin = None
        closed = np.ones(B, bool)
        for q_idx in disj_q:
            closed &= (lbs[:, q_idx] > 0).any(axis=1)
        unclosed = np.nonzero(~closed)[0]
        n_leaves += B
        rec = {'iter': n_iters, 'B': B, 'closed_crown': int(closed.sum())}
        if clip_enabled and unclosed.size > 0:
            xl_u, xh_u = xl_b[unclosed], xh_b[unclosed]
            A_u, b_u = A_lin[unclosed], b_lin[unclosed]
            if multi:
                pxl, pxh, pf = [], [], []
                for q_idx in disj_q:
                    xl_d, xh_d, f_d = ob.clip_box_by_halfspaces_batched(
                        xl_u, xh_u, A_u[:, q_idx], b_u[:, q_idx])
                    pxl.append(np.where(f_d[:, None], xl_d, np.inf))
                    pxh.append(np.where(f_d[:, None], xh_d, -np.inf))
                    pf.append(f_d)
                feas = np.stack(pf, 0).any(axis=0)
                xl_c = np.where(feas[:, None], np.stack(pxl, 0).min(axis=0),
                                xl_u).astype(dtype)
                xh_c = np.where(feas[:, None], np.stack(pxh, 0).max(axis=0),
                                xh_u).astype(dtype)
            else:
                xl_c, xh_c, feas = ob.clip_box_by_halfspaces_batched(
                    xl_u, xh_u, A_u, b_u)
            fidx = np.nonzero(feas)[0]
            xl_s, xh_s = xl_c[fidx], xh_c[fidx]
            rec['closed_clip'] = int((~feas).sum())
        else:
            fidx = np.arange(unclosed.size)
            xl_s, xh_s = xl_b[unclosed], xh_b[unclosed]
            rec['closed_clip'] = 0
        if xl_s.shape[0] > 0:
            widths = xh_s - xl_s
            if branch_sb and A_lin is not None:
                A_s = A_lin[unclosed][fidx] if clip_enabled else A_lin[unclosed]
                scores = widths * np.abs(A_s).sum(axis=1)
                ax = scores.argmax(axis=1)
            else:
                ax = widths.argmax(axis=1)
            rows = np.arange(xl_s.shape[0])
            lo_ax = xl_s[rows, ax]
            hi_ax = xh_s[rows, ax]
            usable = (hi_ax - lo_ax) > dtype(1e-12)
            n_open += int((~usable).sum())
            if usable.any():
                u = np.nonzero(usable)[0]
                xl_u2, xh_u2 = xl_s[u], xh_s[u]
                mid = ((lo_ax[u] + hi_ax[u]) * dtype(0.5)).astype(dtype)
                xh_low = xh_u2.copy()
                xh_low[np.arange(u.size), ax[u]] = mid
                xl_high = xl_u2.copy()
                xl_high[np.arange(u.size), ax[u]] = mid
                wl_xl.append(xl_u2)
                wl_xh.append(xh_low)
                wl_xl.append(xl_high)
                wl_xh.append(xh_u2)
            rec['split'] = int(usable.sum())
            rec['split_dims'] = ax.copy()
            if wl_size() > max_worklist:
                return 'unknown', {'phase': 'batched_worklist_overflow',
                                   'batched_n_leaves': n_leaves,
                                   'batched_n_iters': n_iters,
                                   'worklist_size': wl_size()}
        if trace is not None:
            trace.append(rec)
        n_iters += 1
    if not wl_xl and n_open == 0:
        return 'verified', {'phase': 'batched_verified',
                            'batched_n_leaves': n_leaves,
                            'batched_n_iters': n_iters,
                            'batched_batch_size': batch_size}
    return 'unknown', {'phase': 'batched_timeout',
                       'batched_n_leaves': n_leaves,
                       'batched_n_iters': n_iters,
                       'batched_worklist_left': wl_size(),
                       'batched_open_degenerate': n_open,
                       'batched_batch_size': batch_size}
