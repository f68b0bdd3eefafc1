"""Freeze-replay alpha-CROWN BaB (the reference's hybrid ACAS-Xu pipeline) on
the B200 kernels.

``_full_freeze``, ``_replay_batched`` and ``verify_hybrid`` keep the
signatures, settings and results of verify_hybrid_acasxu.py:164-539:

* ``_full_freeze``: forward zonotope bounds; then per ReLU layer L, in order,
  up to ``n_iters_per_layer`` Adam steps (lr x 0.98 per step) on per-row
  slopes of every earlier ReLU, bounding +-e_j at layer L's input,
  best-of-iterations, stopping once the sum of the best bounds improves by
  less than 1e-6, the result intersected into the layer's bounds; then the
  same for the spec rows (``n_iters_spec``).  Returns (tight,
  alpha_per_layer, alpha_spec, best_spec).
* ``_replay_batched``: forward zonotope, each layer's frozen slopes replayed
  once (no Adam), then ``spec_iters`` Adam steps on the spec slopes
  warm-started from the frozen ones; returns (best lb, A of the best iterate
  per leaf).
* ``verify_hybrid``: root PGD, fan-out to ``init_leaves`` by widest-dimension
  bisection, the freeze on those leaves (one slope group each), then the BaB
  loop: LIFO worklist, replay, closure (worst disjunct's best query > 0), PGD
  on the worst open leaves every ``pgd_between_every`` iterations,
  widest-dimension bisection of the rest.

How it maps onto the device:

* Slopes are per (box, row) tensors (B, Q, n_k): one row of the wide CROWN
  kernels each.  The bound of ReLU L's input is the spec bound of the
  network cut after fc layer L with the rows [I; -I], so every stage is one
  ``wide.wide_alpha_grad`` call (``vcb_wide_back_layer`` down,
  ``vcb_wide_adjoint_layer`` up) plus one fused Adam + clamp launch per
  layer (``vcb_wtc_adam`` with one row per domain).  No autograd, no
  ``torch.optim``.
* The early stop is decided on the device: a flag, cleared when the best
  bounds' sum improves by less than 1e-6, gates the Adam kernel and the
  best-of update, so the iterations queued after the stop change nothing.
  The host reads the flag once every ``_STOP_POLL`` iterations to stop
  queuing work.
* The BaB worklist is a device stack of boxes and slope-group ids.  A batch
  is bounded in one replay -- each leaf gathers its group's frozen slopes --
  closed, and bisected with a handful of tensor operations; the host reads
  one count per iteration.  The between-round PGD runs the worst open
  leaves' restarts in one launch sequence.
"""
from __future__ import annotations

import time
import types
from collections import defaultdict

import numpy as np
import torch

from . import _lib
from .interm import _forward_zonotope_graph_batched
from .ops import F32, _dev, spec_matrix
from .pgd import _constraint_rows, _simple_pgd, _simple_run, pgd_box_expand_amount
from .wide import wide_alpha_grad, wide_crown, wide_net

P = _lib.ptr
_STOP_POLL = 8  # Adam iterations queued between reads of the stop flag

# Adam steps taken by each stage of the last _full_freeze (int32 device
# tensors, in stage order: the ReLU layers that have earlier layers, then
# the spec rows); reading them synchronises.
last_stats = {'stage_steps': []}


def _min_area(lo, hi, dtype=F32):
    """Lower slope of the CROWN min-area rule: 1 where up_s > 0.5 on unstable
    neurons (verify_zono_bnb.py:503-522)."""
    lb_r = torch.clamp(lo, max=0)
    ub_r = torch.maximum(torch.clamp(hi, min=0), lb_r + 1e-8)
    up_s = ub_r / (ub_r - lb_r)
    unstable = (lo < 0) & (hi > 0)
    return (up_s > 0.5).to(dtype) * unstable.to(dtype)


def _seed_rows(n, device):
    """Rows [I; -I] (2n, n) and zero biases: lower bounds of +-z_j at a
    layer input give its lower and (negated) upper bounds."""
    eye = torch.eye(n, dtype=F32, device=device)
    return torch.cat([eye, -eye]).contiguous(), torch.zeros(2 * n, dtype=F32, device=device)


class _Head:
    """The network up to and including fc layer L, in the layout the wide
    kernels read: its spec bound with ``_seed_rows`` bounds ReLU L's input."""

    def __init__(self, wn, L):
        self.W, self.Wabs = wn.W[:L + 1], wn.Wabs[:L + 1]
        self.b, self.Waug = wn.b[:L + 1], wn.Waug[:L + 1]


def _per_row(alpha, Q):
    """(B, n) slopes -> (B, Q, n), one copy per row."""
    return alpha.unsqueeze(1).expand(-1, Q, -1).contiguous()


def _intersect(old, lb_rows, n):
    lo_t = torch.maximum(old[0], lb_rows[:, :n])
    hi_t = torch.minimum(old[1], -lb_rows[:, n:])
    return torch.minimum(lo_t, hi_t), hi_t


def _adam_step(alpha, contrib, m1, m2, lr, step, gate, D, Q):
    """One gated Adam step (torch defaults) on -sum(lb) and the clamp to
    [0, 1] for every layer's per-row slopes (D, Q, n_k)."""
    L_ = _lib.lib()
    for k, a in alpha.items():
        dc, ldc = contrib[k]
        rc = L_.vcb_wtc_adam(D * Q, 1, a.shape[-1], P(dc), ldc, P(a), P(m1[k]), P(m2[k]),
                             float(lr), int(step), P(gate), _lib.stream_of(a.device))
        _lib.check(rc, 'vcb_wtc_adam')


def _optimise(net, xl, xh, tight, W_q, b_q, alpha, n_iters, lr, lr_decay=0.98,
              deadline=None):
    """The freeze's Adam stage (verify_hybrid_acasxu.py:206-231, :246-264):
    per-row slopes ``alpha`` {k: (D, Q, n_k)} optimised in place on
    -sum(lb); returns the best-of-iterations lb (D, Q).  Stops after the
    first iteration whose best-sum improvement is below 1e-6 (that
    iteration's Adam step included), or at ``deadline`` (host clock, checked
    from the second iteration)."""
    dev = xl.device
    D, Q = xl.shape[0], W_q.shape[0]
    m1 = {k: torch.zeros_like(a) for k, a in alpha.items()}
    m2 = {k: torch.zeros_like(a) for k, a in alpha.items()}
    gate = torch.ones(1, dtype=torch.int32, device=dev)
    steps = torch.zeros(1, dtype=torch.int32, device=dev)
    last_stats['stage_steps'].append(steps)
    best = prev = None
    cur_lr = lr
    for it in range(max(1, n_iters)):
        if deadline is not None and it > 0 and time.perf_counter() > deadline:
            break
        lb, contrib = wide_alpha_grad(net, xl, xh, tight, W_q, b_q, alpha)
        if best is None:
            best = lb.clone()
        else:
            best = torch.where(gate.bool(), torch.maximum(best, lb), best)
        cur = best.sum().double()
        _adam_step(alpha, contrib, m1, m2, cur_lr, it + 1, gate, D, Q)
        steps += gate
        if prev is not None:
            gate = gate * (~(cur - prev < 1e-6)).to(torch.int32)
        prev = cur
        cur_lr *= lr_decay
        if (it + 1) % _STOP_POLL == 0 and not bool(gate.item()):
            break
    return best


def _full_freeze(xl, xh, gg, spec_ew, device, dtype, n_iters_per_layer=100, n_iters_spec=100,
                 lr=0.25, deadline=None):
    device = _dev(device)
    wn = wide_net(gg, device)
    last_stats['stage_steps'] = []
    xl = xl.to(device=device, dtype=F32).contiguous()
    xh = xh.to(device=device, dtype=F32).contiguous()
    sb, _ = _forward_zonotope_graph_batched(xl, xh, gg, device, F32)
    tight = {L: (lo.clone(), hi.clone()) for L, (lo, hi) in sb.items()}
    order = sorted(tight)
    alpha_per_layer = {}
    for L in order:
        if deadline is not None and time.perf_counter() > deadline:
            alpha_per_layer[L] = {}
            continue
        n = tight[L][0].shape[1]
        alpha = {k: _per_row(_min_area(*tight[k]), 2 * n) for k in order if k < L}
        if alpha:
            W_q, b_q = _seed_rows(n, device)
            best = _optimise(_Head(wn, L), xl, xh, tight, W_q, b_q, alpha,
                             n_iters_per_layer, lr)
            tight[L] = _intersect(tight[L], best, n)
        alpha_per_layer[L] = alpha
    W_s, b_s = spec_matrix(spec_ew, device)
    alpha_spec = {L: _per_row(_min_area(*tight[L]), W_s.shape[0]) for L in order}
    best_spec = _optimise(wn, xl, xh, tight, W_s, b_s, alpha_spec, n_iters_spec, lr,
                          deadline=deadline)
    return tight, alpha_per_layer, alpha_spec, best_spec


def _replay(wn, gg, xl, xh, W_s, b_s, layer_alpha, spec_alpha, gid, spec_iters, spec_lr,
            want_A=False):
    """Bounds of a batch under frozen slopes (verify_hybrid_acasxu.py:
    270-330): leaf b takes the slopes of group gid[b] from the banks
    ``layer_alpha`` {L: {k: (G, 2 n_L, n_k)}} and ``spec_alpha`` {k: (G, Q,
    n_k)}; per layer the seeded bound with the layer's slopes, then
    ``spec_iters`` Adam steps (constant lr) on the spec slopes.  Returns
    (best (B, Q), best_A (B, Q, n0) or None): a row's best takes a bound only
    when it is larger; a leaf's A is the one of its last iteration that
    improved some row."""
    dev = xl.device
    B, Q = xl.shape[0], W_s.shape[0]
    sb, _ = _forward_zonotope_graph_batched(xl, xh, gg, dev, F32)
    tight = {L: (lo.clone(), hi.clone()) for L, (lo, hi) in sb.items()}
    for L in sorted(tight):
        bank = layer_alpha.get(L)
        if not bank:
            continue
        n = tight[L][0].shape[1]
        W_q, b_q = _seed_rows(n, dev)
        al = {k: a[gid] for k, a in bank.items()}
        lb = wide_crown(_Head(wn, L), xl, xh, tight, W_q, b_q, alpha=al)['lb']
        del al
        tight[L] = _intersect(tight[L], lb, n)
    alpha = {k: a[gid] for k, a in spec_alpha.items()}
    m1 = {k: torch.zeros_like(a) for k, a in alpha.items()}
    m2 = {k: torch.zeros_like(a) for k, a in alpha.items()}
    best = best_A = None
    n_it = max(1, spec_iters)
    for it in range(n_it):
        out = wide_alpha_grad(wn, xl, xh, tight, W_s, b_s, alpha, want_A=want_A)
        lb, contrib = out[0], out[1]
        if best is None:
            best = lb.clone()
            best_A = out[2].clone() if want_A else None
        else:
            imp = lb > best
            best = torch.where(imp, lb, best)
            if want_A:
                best_A = torch.where(imp.any(dim=1)[:, None, None], out[2], best_A)
        if it + 1 < n_it:  # the last step's slopes are not used
            _adam_step(alpha, contrib, m1, m2, spec_lr, it + 1, None, B, Q)
    return best, best_A


def _replay_batched(xl_b, xh_b, gg, spec_ew, alpha_layer_b, alpha_spec_b, device, dtype,
                    spec_iters=10, spec_lr=0.1):
    device = _dev(device)
    wn = wide_net(gg, device)
    xl_b = xl_b.to(device=device, dtype=F32).contiguous()
    xh_b = xh_b.to(device=device, dtype=F32).contiguous()
    W_s, b_s = spec_matrix(spec_ew, device)
    gid = torch.zeros(xl_b.shape[0], dtype=torch.long, device=device)  # one group
    return _replay(wn, gg, xl_b, xh_b, W_s, b_s, alpha_layer_b, alpha_spec_b, gid, spec_iters,
                   spec_lr, want_A=True)


def _fan_out(x_lo, x_hi, init_leaves):
    """Initial leaves by widest-dimension bisection in the reference's order
    (verify_hybrid_acasxu.py:377-390): each round splits the boxes in order
    and stops once ``init_leaves`` children exist."""
    boxes = [(x_lo, x_hi)]
    while len(boxes) < init_leaves:
        new = []
        for lo, hi in boxes:
            d = int(np.argmax(hi - lo))
            mid = np.float32((lo[d] + hi[d]) / np.float32(2))
            a_hi, b_lo = hi.copy(), lo.copy()
            a_hi[d] = mid
            b_lo[d] = mid
            new += [(lo, a_hi), (b_lo, hi)]
            if len(new) >= init_leaves:
                break
        boxes = new
    boxes = boxes[:init_leaves]
    return np.stack([b[0] for b in boxes]), np.stack([b[1] for b in boxes])


class _Stack:
    """LIFO worklist of boxes and slope-group ids on the device."""

    def __init__(self, xl, xh, gid):
        self.xl, self.xh, self.gid = xl.contiguous(), xh.contiguous(), gid.contiguous()
        self.n = xl.shape[0]

    def pop(self, take):
        s = self.n - take
        self.n = s
        return self.xl[s:s + take].clone(), self.xh[s:s + take].clone(), \
            self.gid[s:s + take].clone()

    def push(self, xl, xh, gid):
        m = xl.shape[0]
        if self.n + m > self.xl.shape[0]:
            cap = max(2 * self.xl.shape[0], self.n + m)
            grow = lambda t: torch.cat([t[:self.n], t.new_empty((cap - self.n,) + t.shape[1:])])  # noqa: E731
            self.xl, self.xh, self.gid = grow(self.xl), grow(self.xh), grow(self.gid)
        self.xl[self.n:self.n + m] = xl
        self.xh[self.n:self.n + m] = xh
        self.gid[self.n:self.n + m] = gid
        self.n += m


def _pgd_leaves(xl, xh, spec, gg, n_output, restarts, n_iter, box_expand):
    """``_simple_pgd`` on each of the k boxes (xl, xh) (k, n), as one attack
    of k x restarts rows: every box draws the same seed-0 starts the
    reference draws in its per-box calls (verify_hybrid_acasxu.py:488-505).
    Returns (sat, witness)."""
    dev = xl.device
    rows = _constraint_rows(spec, n_output)
    if rows is None:
        return False, None
    C, cb, cdis, D = rows
    lo = (xl - box_expand).contiguous()
    hi = (xh + box_expand).contiguous()
    k, n = lo.shape
    torch.manual_seed(0)
    u = torch.rand(restarts, n, device=dev, dtype=F32)
    lo_r = lo.repeat_interleave(restarts, dim=0)
    hi_r = hi.repeat_interleave(restarts, dim=0)
    x = (lo_r + (hi_r - lo_r) * u.repeat(k, 1)).contiguous()
    idx = _simple_run(gg, x, lo, hi, restarts, torch.as_tensor(C, device=dev),
                      torch.as_tensor(cb, device=dev), torch.as_tensor(cdis, device=dev), D,
                      n_iter, 0.1)
    if idx is None:
        return False, None
    return True, x[idx].detach().cpu().numpy()


def verify_hybrid(graph, spec, settings=None, timeout=120.0, init_leaves=32, k_freeze=5,
                  batch=4096, verbose=False, pgd_between_every=1, pgd_between_k=5,
                  pgd_between_restarts=1000, pgd_between_iter=50):
    """Returns {verdict in 'sat' / 'unsat' / 'unknown', time, phase, ...}."""
    if settings is None:
        settings = types.SimpleNamespace()
    settings.total_timeout = timeout
    disable_sat = bool(getattr(settings, 'disable_sat_finding', False))
    pgd_between_every = int(getattr(settings, 'hybrid_pgd_between_every', pgd_between_every))
    pgd_between_restarts = int(getattr(settings, 'hybrid_pgd_between_restarts',
                                       pgd_between_restarts))
    freeze_iters = int(getattr(settings, 'hybrid_freeze_iters', 100))
    box_expand = pgd_box_expand_amount(settings)

    t_start = time.perf_counter()
    device = torch.device('cuda')
    gg = graph.gpu_graph(device, F32)
    wn = wide_net(gg, device)
    n_output = int(wn.W[-1].shape[0])
    queries = spec.as_linear_queries(n_output)
    spec_ew = {qi: (torch.as_tensor(w, dtype=F32, device=device).flatten(), float(b))
               for qi, (di, w, b) in enumerate(queries)}
    W_s, b_s = spec_matrix(spec_ew, device)
    disj = defaultdict(list)
    for qi, (di, _, _) in enumerate(queries):
        disj[di].append(qi)
    disj_cols = [torch.as_tensor(sorted(q), device=device) for q in disj.values()]

    def worst_disjunct(best):
        return torch.stack([best[:, c].max(dim=1).values for c in disj_cols], 1).min(1).values

    x_lo = np.asarray(spec.x_lo, np.float64).reshape(-1).astype(np.float32)
    x_hi = np.asarray(spec.x_hi, np.float64).reshape(-1).astype(np.float32)
    xl_root = torch.as_tensor(x_lo, device=device)[None]
    xh_root = torch.as_tensor(x_hi, device=device)[None]

    # phase 0: root PGD
    if bool(getattr(settings, 'pgd_phase0_enabled', True)) and not disable_sat:
        sat, witness = _simple_pgd(xl_root, xh_root, spec, gg, n_output, device, F32,
                                   n_restarts=10000, n_iter=50, lr=0.1, box_expand=box_expand)
        if sat:
            return {'verdict': 'sat', 'time': time.perf_counter() - t_start,
                    'phase': 'root_pgd', 'witness': witness}
        torch.cuda.empty_cache()

    # phase 2: fan-out and the freeze
    lo_k, hi_k = _fan_out(x_lo, x_hi, init_leaves)
    xl_init = torch.as_tensor(lo_k, device=device)
    xh_init = torch.as_tensor(hi_k, device=device)
    try:
        _, alpha_layer_K, alpha_spec_K, best_K = _full_freeze(
            xl_init, xh_init, gg, spec_ew, device, F32, n_iters_per_layer=freeze_iters,
            n_iters_spec=freeze_iters, deadline=t_start + 0.8 * timeout)
    except torch.cuda.OutOfMemoryError:
        torch.cuda.empty_cache()
        return {'verdict': 'unknown', 'time': time.perf_counter() - t_start,
                'phase': 'freeze_oom'}
    n_init = xl_init.shape[0]
    open_K = (worst_disjunct(best_K) <= 0).nonzero(as_tuple=True)[0]
    stack = _Stack(xl_init[open_K], xh_init[open_K], open_K)
    n_evaluated = n_init
    n_closed = n_init - stack.n
    if verbose:
        print(f'  depth-K closure: {n_closed}/{n_init}  open={stack.n}')

    # phase 3: BaB
    cur_batch = batch
    iters = 0
    while stack.n:
        if time.perf_counter() - t_start > timeout - 0.5:
            return {'verdict': 'unknown', 'time': time.perf_counter() - t_start,
                    'phase': 'bab_timeout', 'residual': stack.n,
                    'evaluated': n_evaluated, 'closed': n_closed}
        take = min(cur_batch, stack.n)
        xl_b, xh_b, gid = stack.pop(take)
        try:
            best, _ = _replay(wn, gg, xl_b, xh_b, W_s, b_s, alpha_layer_K, alpha_spec_K, gid,
                              10, 0.1)
        except torch.cuda.OutOfMemoryError:
            torch.cuda.empty_cache()
            stack.n += take  # the popped rows are still in place
            if cur_batch <= 8:
                return {'verdict': 'unknown', 'time': time.perf_counter() - t_start,
                        'phase': 'bab_oom'}
            cur_batch = max(8, cur_batch // 2)
            continue
        n_evaluated += take
        worst = worst_disjunct(best)
        open_idx = (~(worst > 0)).nonzero(as_tuple=True)[0]
        n_open = int(open_idx.numel())
        n_closed += take - n_open
        if verbose and iters % 10 == 0:
            print(f'    iter {iters} t={time.perf_counter() - t_start:.1f} wl={stack.n} '
                  f'eval={n_evaluated} closed={n_closed}')
        if (pgd_between_every > 0 and not disable_sat and n_open > 0
                and iters % pgd_between_every == 0):
            pick = open_idx[worst[open_idx].argsort()[:min(pgd_between_k, n_open)]]
            sat, witness = _pgd_leaves(xl_b[pick], xh_b[pick], spec, gg, n_output,
                                       pgd_between_restarts, pgd_between_iter, box_expand)
            if sat:
                return {'verdict': 'sat', 'time': time.perf_counter() - t_start,
                        'phase': 'between_pgd', 'witness': witness}
        if n_open:
            lo, hi, g = xl_b[open_idx], xh_b[open_idx], gid[open_idx]
            d = (hi - lo).argmax(dim=1, keepdim=True)
            mid = (lo.gather(1, d) + hi.gather(1, d)) / 2
            # children low, high per leaf, leaves in batch order
            kid_lo = torch.stack([lo, lo.scatter(1, d, mid)], 1).reshape(2 * n_open, -1)
            kid_hi = torch.stack([hi.scatter(1, d, mid), hi], 1).reshape(2 * n_open, -1)
            stack.push(kid_lo, kid_hi, g.repeat_interleave(2))
        iters += 1
    return {'verdict': 'unsat', 'time': time.perf_counter() - t_start, 'phase': 'bab_complete',
            'evaluated': n_evaluated, 'closed': n_closed, 'bab_iters': iters}
