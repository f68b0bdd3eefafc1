"""Batched sign-gradient PGD on ``vcb_mlp_pgd``.

``_simple_pgd`` / ``_simple_pgd_batched`` keep the reference's signatures
(verify_hybrid_acasxu.py:39, :103): margin rows per disjunct from the spec,
``torch.manual_seed(seed)`` then ``lo + (hi - lo) * torch.rand(...)`` for the
restarts (the same draw as the reference on the same device), and the
(sat, witness) result.  The iterations run in one kernel launch.
"""
from __future__ import annotations

import numpy as np
import torch

from . import _lib
from .netdesc import mlp_desc
from .ops import F32, _dev

NO_SAT = 0xFFFFFFFFFFFFFFFF


def _constraint_rows(spec, n_output):
    """Margin rows (C, cb) and the disjunct of each row
    (verify_hybrid_acasxu.py:117-130).  Returns None for a constraint kind
    the reference's PGD does not handle (it then reports no witness)."""
    rows, bs, dis = [], [], []
    disjuncts = getattr(spec, 'disjuncts_raw', None)
    if disjuncts is not None:
        for d, conj in enumerate(disjuncts):
            for c in conj:
                w = np.zeros(n_output)
                if c[0] == 'pair':
                    w[c[1]], w[c[2]] = 1.0, -1.0
                    b = 0.0
                elif c[0] == 'ge':
                    w[c[1]] = -1.0
                    b = float(c[2])
                else:
                    w[c[1]] = 1.0
                    b = -float(c[2])
                rows.append(w), bs.append(b), dis.append(d)
    else:
        for d, conj in enumerate(spec.disjuncts):
            for c in conj.constraints:
                w = np.zeros(n_output)
                if hasattr(c, 'pred'):
                    w[c.pred], w[c.comp] = 1.0, -1.0
                    b = 0.0
                elif c.op == '>=':
                    w[c.index] = -1.0
                    b = float(c.value)
                elif c.op == '<=':
                    w[c.index] = 1.0
                    b = -float(c.value)
                else:
                    return None
                rows.append(w), bs.append(b), dis.append(d)
    D = (max(dis) + 1) if dis else 0
    return np.stack(rows).astype(np.float32), np.asarray(bs, np.float32), \
        np.asarray(dis, np.int32), D


def pgd_run(desc, x, lo, hi, R, C, cb, cdis, D, n_iter, lr):
    """Raw launch; returns (best_key, x) with x updated in place."""
    dev = x.device
    best = torch.full((1,), -1, dtype=torch.int64, device=dev)  # all ones
    P = _lib.ptr
    rc = _lib.lib().vcb_mlp_pgd(desc.struct, x.shape[0], R, P(x), P(lo), P(hi),
                                C.shape[0], P(C), P(cb), P(cdis), D, n_iter,
                                float(lr), P(best), _lib.stream_of(dev))
    _lib.check(rc, 'vcb_mlp_pgd')
    key = int(best.item()) & NO_SAT
    return key, x


def _simple_pgd_batched(xl, xh, spec, gg, n_output, device, dtype,
                        n_restarts=128, n_iter=50, lr=0.1, seed=0, box_expand=0.0):
    """Sign-gradient PGD over many boxes at once (verify_hybrid_acasxu.py:103).
    Returns (sat: bool, witness np.ndarray or None)."""
    device = _dev(device)
    xl = torch.as_tensor(xl, device=device).to(F32)
    xh = torch.as_tensor(xh, device=device).to(F32)
    B, n_in = xl.shape
    if box_expand:
        xl = xl - box_expand
        xh = xh + box_expand
    rows = _constraint_rows(spec, n_output)
    if rows is None or B == 0:
        return False, None
    C, cb, cdis, D = rows
    desc = mlp_desc(gg, device)
    torch.manual_seed(seed)
    R = n_restarts
    lo = xl.unsqueeze(1).expand(B, R, n_in).reshape(B * R, n_in)
    hi = xh.unsqueeze(1).expand(B, R, n_in).reshape(B * R, n_in)
    x = (lo + (hi - lo) * torch.rand(B * R, n_in, device=device, dtype=F32)).contiguous()
    key, x = pgd_run(desc, x, xl.contiguous(), xh.contiguous(), R,
                     torch.as_tensor(C, device=device), torch.as_tensor(cb, device=device),
                     torch.as_tensor(cdis, device=device), D, n_iter, lr)
    if key == NO_SAT:
        return False, None
    idx = key & 0xFFFFFFFF
    return True, x[idx].detach().cpu().numpy()


def _simple_pgd(xl, xh, spec, gg, n_output, device, dtype, n_restarts=10000,
                n_iter=50, lr=0.1, seed=0, min_restarts=64, box_expand=0.0):
    """Sign-gradient PGD over one input box (verify_hybrid_acasxu.py:39);
    halves the restarts on OOM down to ``min_restarts``."""
    device = _dev(device)
    xl0 = torch.as_tensor(xl, device=device).to(F32).flatten() - box_expand
    xh0 = torch.as_tensor(xh, device=device).to(F32).flatten() + box_expand
    n_in = xl0.numel()
    rows = _constraint_rows(spec, n_output)
    if rows is None:
        return False, None
    C, cb, cdis, D = rows
    desc = mlp_desc(gg, device)
    cur = n_restarts
    while cur >= min_restarts:
        try:
            torch.manual_seed(seed)
            x = (xl0 + (xh0 - xl0) * torch.rand(cur, n_in, device=device, dtype=F32)).contiguous()
            key, x = pgd_run(desc, x, xl0.reshape(1, -1).contiguous(),
                             xh0.reshape(1, -1).contiguous(), cur,
                             torch.as_tensor(C, device=device),
                             torch.as_tensor(cb, device=device),
                             torch.as_tensor(cdis, device=device), D, n_iter, lr)
            if key == NO_SAT:
                return False, None
            return True, x[key & 0xFFFFFFFF].detach().cpu().numpy()
        except torch.cuda.OutOfMemoryError:
            cur //= 2
    return False, None


def root_pgd(spec, gg, n_output, device, settings):
    """Root SAT search before the BaB: the reference's simple-PGD stage
    (10,000 restarts x 50 iterations, verify_graph.py:12604-12619)."""
    xl = torch.as_tensor(np.asarray(spec.x_lo), dtype=F32, device=device).flatten()
    xh = torch.as_tensor(np.asarray(spec.x_hi), dtype=F32, device=device).flatten()
    return _simple_pgd(xl.unsqueeze(0), xh.unsqueeze(0), spec, gg, n_output,
                       device, torch.float32, n_restarts=10000, n_iter=50)


def leaf_pgd(xl_b, xh_b, lb, qd, D, spec, gg, n_output, device, settings):
    """Leaf PGD on the worst unclosed leaves (verify_graph.py:13000-13019)."""
    lp_max = int(getattr(settings, 'input_split_leaf_pgd_max_leaves', 64) or 64)
    restarts = int(getattr(settings, 'input_split_leaf_pgd_restarts', 128) or 128)
    iters = int(getattr(settings, 'input_split_leaf_pgd_iters', 50) or 50)
    qd = qd.long()
    per_disj = []
    closed = torch.ones(lb.shape[0], dtype=torch.bool, device=lb.device)
    for d in range(D):
        cols = (qd == d).nonzero(as_tuple=True)[0]
        sub = lb[:, cols]
        per_disj.append(sub.max(dim=1).values)
        closed &= (sub > 0).any(dim=1)
    unclosed = (~closed).nonzero(as_tuple=True)[0]
    if unclosed.numel() == 0:
        return False, None
    worst = torch.stack([pd[unclosed] for pd in per_disj], dim=1).min(dim=1).values
    sel = unclosed[worst.argsort()[:lp_max]]
    return _simple_pgd_batched(xl_b[sel], xh_b[sel], spec, gg, n_output, device,
                               torch.float32, n_restarts=restarts, n_iter=iters)
