"""Batched PGD counterexample search on ``vcb_mlp_pgd`` / ``vcb_mlp_pgd_general``.

``_simple_pgd`` / ``_simple_pgd_batched`` keep the reference's signatures
(verify_hybrid_acasxu.py:39, :103): margin rows per disjunct from the spec,
``torch.manual_seed(seed)`` then ``lo + (hi - lo) * torch.rand(...)`` for the
restarts (the same draw as the reference on the same device), and the
(sat, witness) result.  ``pgd_attack_general`` keeps the signature and the
random draws of pgd.py:233 (restart init, OSI projections).  The iterations
run in one kernel launch each.
"""
from __future__ import annotations

import math
import time

import numpy as np
import torch

from . import _lib
from .netdesc import MlpDesc, mlp_desc
from .ops import F32, _dev

NO_SAT = 0xFFFFFFFFFFFFFFFF
INT32_MAX = 2 ** 31 - 1


def _disjunct_tuples(spec):
    """The spec's DNF as lists of ('pair', pred, comp) | ('ge', i, v) |
    ('le', i, v), from a LinearSpec or the reference's VNNSpec; None for a
    constraint kind PGD does not handle."""
    raw = getattr(spec, 'disjuncts_raw', None)
    if raw is not None:
        return [list(conj) for conj in raw]
    out = []
    for conj in spec.disjuncts:
        cur = []
        for c in conj.constraints:
            if hasattr(c, 'pred'):
                cur.append(('pair', int(c.pred), int(c.comp)))
            elif c.op in ('>=', '<='):
                cur.append(('ge' if c.op == '>=' else 'le', int(c.index), float(c.value)))
            else:
                return None
        out.append(cur)
    return out


def _rows_of(disjuncts, n_output):
    """Margin rows (margin > 0 = safe; pgd.py:75-118): w, b and the disjunct of
    each row."""
    rows, bs, dis = [], [], []
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
    return rows, bs, dis


def _constraint_rows(spec, n_output):
    """Margin rows (C, cb) and the disjunct of each row
    (verify_hybrid_acasxu.py:117-130).  Returns None for a constraint kind
    the reference's PGD does not handle (it then reports no witness)."""
    disjuncts = _disjunct_tuples(spec)
    if disjuncts is None:
        return None
    rows, bs, dis = _rows_of(disjuncts, n_output)
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


def _graph(gg, device):
    from .graph import graph_net
    return graph_net(gg, device)


def _screen(G_out, t, y, rows, R, simple, best, gmin_t, g, hinge=0.0, bloat=0.0,
            prd=False, n_act=1):
    C, cb, cdis, cact, D = rows
    rc = _lib.lib().vcb_pgd_screen(
        y.shape[0], G_out, _lib.ptr(y), y.shape[1], C.shape[0], _lib.ptr(C), _lib.ptr(cb),
        _lib.ptr(cdis), _lib.ptr(cact), D, n_act, int(prd), R, int(simple), float(hinge),
        float(bloat), t, best, gmin_t, _lib.ptr(g), g.shape[1], _lib.stream_of(y.device))
    _lib.check(rc, 'vcb_pgd_screen')


def _step(x, lo, hi, R, g, mode, optim=0, t=0, step0=None, cur=None, m1=None, m2=None,
          sc1=1.0, sc2=1.0, decay=1.0, lr=0.0):
    N, n_in = x.shape
    rc = _lib.lib().vcb_pgd_step(
        N, R, n_in, _lib.ptr(x), _lib.ptr(lo), _lib.ptr(hi), _lib.ptr(g), g.shape[1], mode,
        optim, t, _lib.ptr(step0), 1 if step0 is None else step0.shape[0], _lib.ptr(cur),
        _lib.ptr(m1), _lib.ptr(m2), float(sc1), float(sc2), float(decay), float(lr),
        _lib.stream_of(x.device))
    _lib.check(rc, 'vcb_pgd_step')


def simple_layerwise(G, x, lo, hi, R, C, cb, cdis, D, n_iter, lr):
    """_simple_pgd's loop on the layer kernels for networks outside the
    shared-memory kernel: per iteration forward, screen (SAT at loss
    <= 1e-6), backward, sign step.  x (N, n_in) is updated in place; returns
    the first SAT sample's index or None."""
    from .graph import graph_forward, graph_vjp
    dev = x.device
    best = torch.full((1,), -1, dtype=torch.int64, device=dev)
    g = torch.empty((x.shape[0], G.n_out), dtype=F32, device=dev)
    rows = (C, cb, cdis, None, D)
    for it in range(n_iter):
        y, pre = graph_forward(G, x, keep=True)
        _screen(G.n_out, it, y, rows, R, True, best.data_ptr(), None, g)
        key = int(best.item()) & NO_SAT  # the reference checks sat_mask.any() here too
        if key != NO_SAT:
            return key & 0xFFFFFFFF
        gx = graph_vjp(G, pre, g)
        _step(x, lo, hi, R, gx, 2, lr=lr)
    return None


def _simple_run(gg, x, lo, hi, R, C, cb, cdis, D, n_iter, lr):
    """One simple-PGD attack: the fused kernel for MLPs that fit it, the
    layer kernels otherwise.  Returns the witness row index or None."""
    dev = x.device
    try:
        desc = mlp_desc(gg, dev)
        key, _ = pgd_run(desc, x, lo, hi, R, C, cb, cdis, D, n_iter, lr)
        return None if key == NO_SAT else key & 0xFFFFFFFF
    except _lib.UnsupportedInput:
        pass
    return simple_layerwise(_graph(gg, dev), x, lo, hi, R, C, cb, cdis, D, n_iter, lr)


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
    torch.manual_seed(seed)
    R = n_restarts
    lo = xl.unsqueeze(1).expand(B, R, n_in).reshape(B * R, n_in)
    hi = xh.unsqueeze(1).expand(B, R, n_in).reshape(B * R, n_in)
    x = (lo + (hi - lo) * torch.rand(B * R, n_in, device=device, dtype=F32)).contiguous()
    idx = _simple_run(gg, x, xl.contiguous(), xh.contiguous(), R,
                      torch.as_tensor(C, device=device), torch.as_tensor(cb, device=device),
                      torch.as_tensor(cdis, device=device), D, n_iter, lr)
    if idx is None:
        return False, None
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
    cur = n_restarts
    while cur >= min_restarts:
        try:
            torch.manual_seed(seed)
            x = (xl0 + (xh0 - xl0) * torch.rand(cur, n_in, device=device, dtype=F32)).contiguous()
            idx = _simple_run(gg, x, xl0.reshape(1, -1).contiguous(),
                              xh0.reshape(1, -1).contiguous(), cur,
                              torch.as_tensor(C, device=device),
                              torch.as_tensor(cb, device=device),
                              torch.as_tensor(cdis, device=device), D, n_iter, lr)
            if idx is None:
                return False, None
            return True, x[idx].detach().cpu().numpy()
        except torch.cuda.OutOfMemoryError:
            torch.cuda.empty_cache()
            cur //= 2
    return False, None


def pgd_box_expand_amount(settings):
    """Per-side widening of the search box (pgd.py:190-203): 0 when
    ``pgd_input_box_expand`` is unset; it may not exceed
    ``sat_validate_atol``."""
    b = float(getattr(settings, 'pgd_input_box_expand', 0.0) or 0.0)
    if b <= 0.0:
        return 0.0
    atol = float(getattr(settings, 'sat_validate_atol', 1e-4))
    assert b <= atol + 1e-12, (
        f'pgd_input_box_expand ({b}) must be <= sat_validate_atol ({atol})')
    return b


def expand_search_box(lo, hi, settings):
    """(lo, hi) widened by ``pgd_box_expand_amount`` (pgd.py:206-212)."""
    b = pgd_box_expand_amount(settings)
    return (lo, hi) if b == 0.0 else (lo - b, hi + b)


_OPTIM = {'sign_sgd': 0, 'adam_sign': 1, 'adam_clipping': 2}


def _num(settings, key, default):
    v = getattr(settings, key, default)
    return default if v is None or not isinstance(v, (int, float, str, bool)) else v


def _decode_min(u):
    """Inverse of the kernel's order encoding of a float32."""
    u &= 0xFFFFFFFF
    bits = (u & 0x7FFFFFFF) if u & 0x80000000 else (~u & 0xFFFFFFFF)
    return float(np.array([bits], np.uint32).view(np.float32)[0])


def _bc_tables(n_iter, device):
    """float32 reciprocals of the Adam bias corrections, rounded as the GPU
    divides a tensor by a Python scalar: float32(1) / float32(c)."""
    t = np.arange(1, n_iter + 1, dtype=np.float64)
    bc1 = (1.0 - 0.9 ** t).astype(np.float32)
    sbc2 = ((1.0 - 0.999 ** t) ** 0.5).astype(np.float32)
    inv1 = (np.float32(1.0) / bc1).astype(np.float32)
    inv2 = (np.float32(1.0) / sbc2).astype(np.float32)
    return (torch.as_tensor(inv1, device=device), torch.as_tensor(inv2, device=device))


def pgd_attack_general(xl, xh, spec, gg, settings, restrict_disj=None,
                       time_budget=None, per_restart_disj=None, seed=None, defer=False):
    """PGD counterexample search for a DNF spec (pgd.py:233-524): restarts
    drawn uniformly in the box, optional OSI initialisation, hinge loss over
    the attacked disjuncts, sign_sgd / adam_sign / adam_clipping steps with
    step decay, plateau give-up and wall-time budget.  For MLPs that fit the
    shared-memory kernel one launch runs every restart and iteration; other
    networks run the same loop on the layer kernels.  Returns (is_sat,
    witness ndarray or None); with ``defer`` the launch is queued on the
    current stream and a callable that waits for it and returns the same
    pair comes back instead (or the pair itself when nothing was launched).
    """
    t_start = time.perf_counter()
    xl, xh = expand_search_box(xl, xh, settings)
    dev = xl.device
    dt = xl.dtype
    if dt != F32:
        raise _lib.UnsupportedInput('vibecheck_nn_b200: pgd_attack_general runs in float32')
    if isinstance(seed, (int, float)):
        torch.manual_seed(int(seed))
    n_restarts = int(_num(settings, 'pgd_restarts', 10))
    n_iter = int(_num(settings, 'pgd_iter', 100))
    lr_decay = float(_num(settings, 'pgd_lr_decay', 0.99))
    hinge_thr = float(_num(settings, 'pgd_hinge_threshold', -1e-5))
    alpha_frac = float(_num(settings, 'pgd_alpha_frac', 0.25))
    if time_budget is None:
        tb = getattr(settings, 'pgd_time_budget', None)
        if isinstance(tb, (int, float)):
            time_budget = float(tb)
    eps_input = (xh - xl) / 2.0
    if bool(_num(settings, 'pgd_alpha_multi', False)):
        fr = list(getattr(settings, 'pgd_alpha_multi_fractions', [0.25, 0.05, 0.01, 0.002]))
        pra = torch.tensor([fr[i % len(fr)] for i in range(n_restarts)], dtype=dt, device=dev)
        while pra.dim() < eps_input.dim() + 1:
            pra = pra.unsqueeze(-1)
        step = eps_input.unsqueeze(0) * pra
    else:
        step = eps_input * alpha_frac
    optim = str(_num(settings, 'pgd_optim', 'adam_sign'))
    if optim not in _OPTIM:
        raise AssertionError(f'unknown pgd_optim {optim!r}; valid: {tuple(_OPTIM)}')
    disjuncts = _disjunct_tuples(spec)
    if disjuncts is None:
        raise ValueError('unknown constraint op')
    act = list(range(len(disjuncts))) if restrict_disj is None else sorted(restrict_disj)
    if not act:
        return False, None
    act = [d for d in act if disjuncts[d]]
    if not act:
        return False, None
    if per_restart_disj is None:
        per_restart_disj = bool(_num(settings, 'pgd_per_restart_disjunct', False))
    prd = bool(per_restart_disj) and len(act) > 1
    init_mode = str(_num(settings, 'pgd_init_mode', 'uniform'))
    x = xl + (xh - xl) * torch.rand(n_restarts, *xl.shape, dtype=dt, device=dev)
    try:
        net = mlp_desc(gg, dev)
        n_out, n_in = net.n_out, net.dims[0]
    except _lib.UnsupportedInput:
        net = _graph(gg, dev)
        n_out, n_in = net.n_out, x[0].numel()
    w_d = None
    n_osi = 0
    if init_mode == 'osi':
        w_d = ((torch.rand(n_restarts, n_out, dtype=dt, device=dev) - 0.5) * 2.0).contiguous()
        n_osi = int(_num(settings, 'pgd_osi_iters', 50))
    plateau = int(_num(settings, 'pgd_plateau_iters', 100))
    bloat = float(getattr(spec, 'unsat_margin_bloat', 0.0) or 0.0)
    x = x.reshape(n_restarts, n_in).contiguous()
    args = (x, xl.reshape(1, n_in), xh.reshape(1, n_in), step.reshape(-1, n_in), w_d, n_osi,
            n_iter, optim, lr_decay, hinge_thr, plateau, disjuncts, act, prd, bloat)
    def result(idx):
        if idx is None:
            return False, None
        return True, x[idx].reshape(xl.shape).detach().cpu().numpy()

    idx = -1
    if isinstance(net, MlpDesc):
        budget_ns = 0
        if time_budget is not None:
            left = time_budget - (time.perf_counter() - t_start)
            budget_ns = max(1, int(left * 1e9))
        try:
            fin = pgd_general_launch(net, *args, budget_ns)
            if defer:
                stream = torch.cuda.current_stream(dev)

                def finish():
                    i = fin()
                    with torch.cuda.stream(stream):
                        return result(i)
                return finish
            idx = fin()
        except _lib.UnsupportedInput:  # wider than the shared-memory kernel
            net = _graph(gg, dev)
    if idx == -1:
        deadline = None if time_budget is None else t_start + time_budget
        idx = general_layerwise(net, *args, deadline)
    out = result(idx)
    return (lambda: out) if defer else out


def pgd_general_run(desc, x, lo, hi, step, w_d, n_osi, n_iter, optim, lr_decay, hinge_thr,
                    plateau, disjuncts, act, prd, bloat=0.0, budget_ns=0):
    """One ``vcb_mlp_pgd_general`` launch over the restarts x (R, n_in)
    (updated in place) and the host replay of the loop's give-up rules.
    Returns the restart index of the confirmed witness or None."""
    return pgd_general_launch(desc, x, lo, hi, step, w_d, n_osi, n_iter, optim, lr_decay,
                              hinge_thr, plateau, disjuncts, act, prd, bloat, budget_ns)()


def pgd_general_launch(desc, x, lo, hi, step, w_d, n_osi, n_iter, optim, lr_decay, hinge_thr,
                       plateau, disjuncts, act, prd, bloat=0.0, budget_ns=0):
    """pgd_general_run up to its launch: returns ``finish()``, which waits
    for the kernel (the one host synchronisation, on the stream current at
    launch) and replays the give-up rules."""
    dev = x.device
    R, n_in = x.shape
    n_out = desc.n_out
    rows, bs, dis = _rows_of(disjuncts, n_out)
    ordinal = {d: i for i, d in enumerate(act)}
    cact = [ordinal.get(d, -1) for d in dis]
    lo = lo.to(F32).contiguous()
    hi = hi.to(F32).contiguous()
    step = step.to(F32).contiguous()
    C = torch.as_tensor(np.stack(rows), dtype=F32, device=dev)
    cb = torch.as_tensor(np.asarray(bs, np.float32), device=dev)
    cdis = torch.as_tensor(np.asarray(dis, np.int32), device=dev)
    cact_t = torch.as_tensor(np.asarray(cact, np.int32), device=dev)
    inv1, inv2 = _bc_tables(max(n_iter, 1), dev)
    # [best (2 x int32) | gmin (n_iter + 2) | t_stop]
    state = torch.full((2 + n_iter + 2 + 1,), -1, dtype=torch.int32, device=dev)
    state[-1] = INT32_MAX
    base = state.data_ptr()
    rc = _lib.lib().vcb_mlp_pgd_general(
        desc.struct, R, R, _lib.ptr(x), _lib.ptr(lo), _lib.ptr(hi), _lib.ptr(step),
        step.shape[0], _lib.ptr(w_d), n_osi if w_d is not None else 0, n_iter,
        _OPTIM[optim], lr_decay, hinge_thr, int(plateau), _lib.ptr(inv1), _lib.ptr(inv2), len(rows),
        _lib.ptr(C), _lib.ptr(cb), _lib.ptr(cdis), _lib.ptr(cact_t), len(disjuncts),
        len(act), int(prd), float(bloat), int(budget_ns), base, base + 8,
        base + 4 * (2 + n_iter + 2), _lib.stream_of(dev))
    _lib.check(rc, 'vcb_mlp_pgd_general')
    stream = torch.cuda.current_stream(dev)

    def finish():
        with torch.cuda.stream(stream):
            host = state.cpu().numpy().view(np.uint32)  # the one host sync
        return _general_replay(host, n_iter, hinge_thr, plateau)
    return finish


def _general_replay(host, n_iter, hinge_thr, plateau):
    """The host side of pgd_general_run: the witness key and the replay of
    the loop's give-up rules from the kernel's per-iteration record."""
    key = int(host[0]) | (int(host[1]) << 32)
    t_w = (key >> 32) if key != NO_SAT else None
    t_stop = int(np.int32(host[-1]))
    gmin = host[2:2 + n_iter + 2]
    # replay of the loop's control flow (pgd.py:440-467, :494-512)
    best_min = float('inf')
    nimp = 0
    final = n_iter + 1
    for t in range(1, n_iter + 1):
        if t >= t_stop:
            final = t
            break
        if t_w == t:
            return key & 0xFFFFFFFF
        curr_min = _decode_min(int(gmin[t]))
        if curr_min > hinge_thr:
            if curr_min < best_min - 1e-6:
                best_min = curr_min
                nimp = 0
            else:
                nimp += 1
            if nimp >= plateau:
                return None
        else:
            nimp = 0
    if t_w == final:
        return key & 0xFFFFFFFF
    return None


def general_layerwise(G, x, lo, hi, step, w_d, n_osi, n_iter, optim, lr_decay, hinge_thr,
                      plateau, disjuncts, act, prd, bloat=0.0, deadline=None):
    """pgd_attack_general's loop on the layer kernels (networks outside the
    shared-memory kernel): OSI steps, then per iteration forward, screen,
    host check (the reference's ``cand.any()`` sync), plateau / deadline,
    backward and the optimiser step.  x (R, n_in) is updated in place;
    returns the witness row or None."""
    from .graph import graph_forward, graph_vjp
    dev = x.device
    R, n_in = x.shape
    n_out = G.n_out
    lo = lo.to(F32).contiguous()
    hi = hi.to(F32).contiguous()
    step = step.to(F32).contiguous()
    for _ in range(n_osi if w_d is not None else 0):
        _, pre = graph_forward(G, x, keep=True)
        gx = graph_vjp(G, pre, w_d)
        _step(x, lo, hi, R, gx, 1, step0=step)
    rows_np, bs, dis = _rows_of(disjuncts, n_out)
    ordinal = {d: i for i, d in enumerate(act)}
    rows = (torch.as_tensor(np.stack(rows_np), dtype=F32, device=dev),
            torch.as_tensor(np.asarray(bs, np.float32), device=dev),
            torch.as_tensor(np.asarray(dis, np.int32), device=dev),
            torch.as_tensor(np.asarray([ordinal.get(d, -1) for d in dis], np.int32),
                            device=dev),
            len(disjuncts))
    t_ = np.arange(1, max(n_iter, 1) + 1, dtype=np.float64)
    sc1 = np.float32(1.0) / (1.0 - 0.9 ** t_).astype(np.float32)
    sc2 = np.float32(1.0) / ((1.0 - 0.999 ** t_) ** 0.5).astype(np.float32)
    cur = step.expand(R, n_in).contiguous().clone()
    m1 = torch.zeros_like(x)
    m2 = torch.zeros_like(x)
    g = torch.empty((R, n_out), dtype=F32, device=dev)
    state = torch.full((4,), -1, dtype=torch.int32, device=dev)  # best (2) | gmin | pad
    base = state.data_ptr()
    best_min = float('inf')
    nimp = 0
    for t in range(1, n_iter + 2):
        final = t == n_iter + 1 or (deadline is not None and time.perf_counter() > deadline)
        state[2] = -1
        y, pre = graph_forward(G, x, keep=True)
        _screen(n_out, t, y, rows, R, False, base, base + 8, g, hinge_thr, bloat, prd,
                len(act))
        host = state.cpu().numpy().view(np.uint32)
        key = int(host[0]) | (int(host[1]) << 32)
        if key != NO_SAT:
            return key & 0xFFFFFFFF
        if final:
            return None
        curr_min = _decode_min(int(host[2]))
        if curr_min > hinge_thr:
            if curr_min < best_min - 1e-6:
                best_min = curr_min
                nimp = 0
            else:
                nimp += 1
            if nimp >= plateau:
                return None
        else:
            nimp = 0
        gx = graph_vjp(G, pre, g)
        _step(x, lo, hi, R, gx, 0, _OPTIM[optim], t, cur=cur, m1=m1, m2=m2,
              sc1=sc1[t - 1], sc2=sc2[t - 1], decay=lr_decay)
    return None


def root_pgd(spec, gg, n_output, device, settings):
    """Root SAT search before the BaB (verify_graph.py:12586-12619):
    ``pgd_attack_general`` within ``pgd_time_budget_phase0``, then the
    simple-PGD stage (10,000 restarts x 50 iterations).  Each is best-effort:
    a RuntimeError (NotImplementedError included) or OOM falls through.
    Returns (sat, witness, phase)."""
    xl = torch.as_tensor(np.asarray(spec.x_lo), dtype=F32, device=device)
    xh = torch.as_tensor(np.asarray(spec.x_hi), dtype=F32, device=device)
    # The two stages are independent searches; the general one (a few
    # restarts: one CTA) runs on a side stream while the simple one fills the
    # other SMs.  Random draws happen on the host in the sequential order and
    # the results are consulted in it (the simple stage's only when the
    # general one found nothing), so the outcome is the sequential one.
    dev = _dev(device)
    main = torch.cuda.current_stream(dev)
    side = torch.cuda.Stream(device=dev)
    side.wait_stream(main)
    general = None
    try:
        budget = float(_num(settings, 'pgd_time_budget_phase0', 5.0))
        with torch.cuda.stream(side):
            r = pgd_attack_general(xl, xh, spec, gg, settings, time_budget=budget, defer=True)
        general = r if callable(r) else (lambda: r)
    except _BEST_EFFORT:
        pass
    # the simple stage reseeds torch's generators; when the general stage
    # wins, the sequential order would not have run it, so its states return
    rng = (torch.get_rng_state(), torch.cuda.get_rng_state(dev))
    simple = (False, None)
    try:
        simple = _simple_pgd(xl.flatten().unsqueeze(0), xh.flatten().unsqueeze(0), spec,
                             gg, n_output, device, torch.float32, n_restarts=10000, n_iter=50)
    except _BEST_EFFORT:
        pass
    gen = (False, None)
    if general is not None:
        try:
            gen = general()
        except _BEST_EFFORT:
            pass
    main.wait_stream(side)
    if gen[0] and gen[1] is not None:
        torch.set_rng_state(rng[0])
        torch.cuda.set_rng_state(rng[1], dev)
        return True, gen[1], 'batched_pgd'
    if simple[0]:
        return True, simple[1], 'batched_simple_pgd'
    return False, None, None


# The root PGD stages are best-effort SAT finders (verify_graph.py:12566-12605
# skips a stage that fails for lack of memory or support); a KernelError is a
# fault and propagates.
_BEST_EFFORT = (_lib.UnsupportedInput, torch.cuda.OutOfMemoryError)


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
