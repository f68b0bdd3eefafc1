"""Numpy restatement of the batched input-split BaB driver (test oracle).

Follows ``_input_split_batched_inner`` (``verify_graph.py:12511-13464``) on the
default path: LIFO chunk worklist (:12695-12726), pop B (:12846), bound with
CROWN or zonotope intermediates + CROWN spec backward with the input-space
linear form (:12855-12870), closure "every disjunct has a query with lb > 0"
(:12901-12908), halfspace clipping repeated up to clip_iters times while any
box of the batch shrinks (:13030-13084), the branching score -- width, SB
width * sum_q |A_q|, or the SB margin score max_q(max(|A_q|, thr) * width /
2 + lb_q * mw), times the branch boost (:13236-13295) -- with the first-max
argmax, the vectorised bisection with the 1e-12 degenerate guard and
children pushed low-chunk then high-chunk (:13353-13382), the K-dimension
split of bab_split_depth while the popped batch is below the batch size
(top-K scores, 2^K' children per leaf in one chunk, :13320-13423), the
max_worklist overflow check (:13424-13429) and the verdict (:13452-13464);
``branch_boost`` restates the root boost (:12744-12800).  Root PGD,
alpha-CROWN, leaf-PGD and MILP escalation are not part of this restatement.
"""
from __future__ import annotations

import time

import numpy as np

from . import bounds as ob


# Top-K in the order torch.topk(largest, sorted) returns on the CPU, ties
# included (the reference ranks its K split dimensions with it,
# verify_graph.py:13347): (score, index) pairs in index order,
# std::nth_element at k - 1 then std::sort of the first k - 1 when 64 k > n,
# else std::partial_sort -- the published standard-library algorithms
# (introselect with a median-of-three pivot, insertion sort; binary heaps).

def _before(a, b):
    return (np.isnan(a[0]) and not np.isnan(b[0])) or a[0] > b[0]


def _insertion_sort(q, first, last):
    for i in range(first + 1, last):
        v = q[i]
        if _before(v, q[first]):
            q[first + 1:i + 1] = q[first:i]
            q[first] = v
        else:
            j, nxt = i, i - 1
            while _before(v, q[nxt]):
                q[j] = q[nxt]
                j, nxt = nxt, nxt - 1
            q[j] = v


def _median_to_first(q, r, a, b, c):
    def sw(x):
        q[r], q[x] = q[x], q[r]
    if _before(q[a], q[b]):
        sw(b if _before(q[b], q[c]) else (c if _before(q[a], q[c]) else a))
    elif _before(q[a], q[c]):
        sw(a)
    else:
        sw(c if _before(q[b], q[c]) else b)


def _partition(q, first, last, pivot):
    while True:
        while _before(q[first], q[pivot]):
            first += 1
        last -= 1
        while _before(q[pivot], q[last]):
            last -= 1
        if not first < last:
            return first
        q[first], q[last] = q[last], q[first]
        first += 1


def _adjust_heap(q, first, hole, n, value):
    top = second = hole
    while second < (n - 1) // 2:
        second = 2 * (second + 1)
        if _before(q[first + second], q[first + second - 1]):
            second -= 1
        q[first + hole] = q[first + second]
        hole = second
    if n % 2 == 0 and second == (n - 2) // 2:
        second = 2 * (second + 1)
        q[first + hole] = q[first + second - 1]
        hole = second - 1
    parent = (hole - 1) // 2
    while hole > top and _before(q[first + parent], value):
        q[first + hole] = q[first + parent]
        hole, parent = parent, (parent - 1) // 2
    q[first + hole] = value


def _heap_select(q, first, middle, last):
    n = middle - first
    for parent in range((n - 2) // 2, -1, -1):
        _adjust_heap(q, first, parent, n, q[first + parent])
    for i in range(middle, last):
        if _before(q[i], q[first]):
            v = q[i]
            q[i] = q[first]
            _adjust_heap(q, first, 0, n, v)


def topk_cpu_order(scores, k):
    """Indices of the k largest scores in torch's CPU topk order."""
    q = [(float(v), i) for i, v in enumerate(scores)]
    n = len(q)
    if k * 64 <= n:
        _heap_select(q, 0, k, n)
        last = k
        while last > 1:
            last -= 1
            v = q[last]
            q[last] = q[0]
            _adjust_heap(q, 0, 0, last, v)
        return [i for _, i in q[:k]]
    first, last, nth = 0, n, k - 1
    depth = 2 * (n.bit_length() - 1)
    done = False
    while last - first > 3:
        if depth == 0:
            _heap_select(q, first, nth + 1, last)
            q[first], q[nth] = q[nth], q[first]
            done = True
            break
        depth -= 1
        mid = first + (last - first) // 2
        _median_to_first(q, first, first + 1, mid, last - 1)
        cut = _partition(q, first + 1, last, first)
        if cut <= nth:
            first = cut
        else:
            last = cut
    if not done:
        _insertion_sort(q, first, last)
    _insertion_sort(q, 0, k - 1)
    return [i for _, i in q[:k]]


def branch_boost(gg, x_lo, x_hi, exp=1.0, dtype=np.float32):
    """The reference's per-dimension SB boost (verify_graph.py:12744-12800):
    for each varying input dimension the shallow ReLU layer (first half of
    the layers) whose mean zonotope width drops most -- by more than 1e-5 --
    when the dimension is halved at the root, and (1 + that layer's unstable
    count at the root) ** exp.  Widths are averaged in float64 and rounded
    to float32 (torch's CPU mean of a float32 tensor)."""
    xl0 = np.asarray(x_lo, dtype).ravel()
    xh0 = np.asarray(x_hi, dtype).ravel()
    vary = np.nonzero((xh0 - xl0) > dtype(1e-9))[0]
    sb_root, _ = ob.forward_zonotope_batched(xl0[None], xh0[None], gg, dtype)
    Ls = sorted(L for L in sb_root if isinstance(L, int))
    shallow = Ls[:max(1, len(Ls) // 2)]

    def mean_w(sb, L):
        w = (sb[L][1][0] - sb[L][0][0]).astype(dtype)
        return float(dtype(w.astype(np.float64).sum() / w.size))

    root_w = {L: mean_w(sb_root, L) for L in shallow}
    n_unst = {L: int(((sb_root[L][0][0] < 0) & (sb_root[L][1][0] > 0)).sum()) for L in shallow}
    boost = np.ones(xl0.size, dtype)
    for d in vary:
        xh_h = xh0.copy()
        xh_h[d] = dtype(xl0[d] + dtype(dtype(0.5) * dtype(xh0[d] - xl0[d])))
        sb_h, _ = ob.forward_zonotope_batched(xl0[None], xh_h[None], gg, dtype)
        best_L, best_delta = None, 1e-5
        for L in shallow:
            delta = root_w[L] - mean_w(sb_h, L)
            if delta > best_delta:
                best_delta, best_L = delta, L
        if best_L is not None:
            boost[d] = dtype((1.0 + float(n_unst[best_L])) ** exp)
    return boost


def input_split_bab(gg, x_lo, x_hi, spec_W, spec_b, disj_q=None,
                    batch_size=4096, max_worklist=200_000,
                    crown_intermediate=True, clip_enabled=True,
                    branch_sb=False, timeout=60.0, max_iters=None,
                    dtype=np.float32, trace=None, clip_iters=1, margin=None,
                    split_depth=1, boost=None):
    """Returns (verdict, details) like the reference driver.  ``margin``:
    None or (coeff_thresh, margin_weight); ``boost``: (n_in,) multipliers of
    the SB score or None."""
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
            xl_c, xh_c = xl_u, xh_u
            for _ in range(clip_iters):
                if multi:
                    pxl, pxh, pf = [], [], []
                    for q_idx in disj_q:
                        xl_d, xh_d, f_d = ob.clip_box_by_halfspaces_batched(
                            xl_c, xh_c, A_u[:, q_idx], b_u[:, q_idx])
                        pxl.append(np.where(f_d[:, None], xl_d, np.inf))
                        pxh.append(np.where(f_d[:, None], xh_d, -np.inf))
                        pf.append(f_d)
                    feas = np.stack(pf, 0).any(axis=0)
                    xl_n = np.where(feas[:, None], np.stack(pxl, 0).min(axis=0),
                                    xl_c).astype(dtype)
                    xh_n = np.where(feas[:, None], np.stack(pxh, 0).max(axis=0),
                                    xh_c).astype(dtype)
                else:
                    xl_n, xh_n, feas = ob.clip_box_by_halfspaces_batched(
                        xl_c, xh_c, A_u, b_u)
                shrunk = bool(((xl_n > xl_c) | (xh_n < xh_c)).any())
                xl_c, xh_c = xl_n, xh_n
                if not shrunk:
                    break
            fidx = np.nonzero(feas)[0]
            xl_s, xh_s = xl_c[fidx], xh_c[fidx]
            rec['closed_clip'] = int((~feas).sum())
        else:
            fidx = np.arange(unclosed.size)
            xl_s, xh_s = xl_b[unclosed], xh_b[unclosed]
            rec['closed_clip'] = 0
        if xl_s.shape[0] > 0:
            widths = xh_s - xl_s
            sb_on = branch_sb and A_lin is not None
            if sb_on:
                A_s = A_lin[unclosed][fidx] if clip_enabled else A_lin[unclosed]
                if margin is not None:
                    lb_s = lbs[unclosed][fidx] if clip_enabled else lbs[unclosed]
                    base = (np.maximum(np.abs(A_s), dtype(margin[0]))
                            * widths[:, None, :]) / dtype(2)
                    base = base + lb_s[:, :, None] * dtype(margin[1])
                    scores = base.max(axis=1)
                else:
                    scores = widths * np.abs(A_s).sum(axis=1)
                if boost is not None:
                    scores = scores * np.asarray(boost, dtype)[None]
                ax = scores.argmax(axis=1)
            else:
                ax = widths.argmax(axis=1)
            if split_depth > 1 and B < batch_size and sb_on:
                # K-dimension split: 2^K' children per leaf, one chunk
                top = [topk_cpu_order(scores[i], split_depth) for i in range(scores.shape[0])]
                kxl, kxh = [], []
                for i in range(xl_s.shape[0]):
                    dims = [int(d) for d in top[i]
                            if float(xh_s[i, d] - xl_s[i, d]) > 1e-12]
                    if not dims:
                        n_open += 1
                        continue
                    mids = [dtype((xl_s[i, d] + xh_s[i, d]) / dtype(2)) for d in dims]
                    for combo in range(1 << len(dims)):
                        cl, ch = xl_s[i].copy(), xh_s[i].copy()
                        for k, d in enumerate(dims):
                            if (combo >> k) & 1:
                                cl[d] = mids[k]
                            else:
                                ch[d] = mids[k]
                        kxl.append(cl)
                        kxh.append(ch)
                if kxl:
                    wl_xl.append(np.stack(kxl).astype(dtype))
                    wl_xh.append(np.stack(kxh).astype(dtype))
                rec['split'] = len(kxl)
                if wl_size() > max_worklist:
                    return 'unknown', {'phase': 'batched_worklist_overflow',
                                       'batched_n_leaves': n_leaves,
                                       'batched_n_iters': n_iters,
                                       'worklist_size': wl_size()}
                if trace is not None:
                    trace.append(rec)
                n_iters += 1
                continue
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
