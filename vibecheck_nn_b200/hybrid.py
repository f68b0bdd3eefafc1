"""Freeze-replay alpha-CROWN BaB (the reference's hybrid ACAS-Xu pipeline) on
the B200 kernels.

``_full_freeze``, ``_replay_batched`` and ``verify_hybrid`` keep the
signatures, settings and results of verify_hybrid_acasxu.py:164-539:

* ``_full_freeze``: forward zonotope bounds, then per relu layer L (in order)
  ``n_iters_per_layer`` Adam steps on per-query slopes alpha (B, 2 n_L, n_k)
  of every earlier layer k, bounding +-e_j at layer L's input (the seeded
  backward), best-of-iterations, sum-based early stop, lr x 0.98 per step,
  bounds intersected into ``tight``; then the same for the spec rows
  (``n_iters_spec``).  Returns (tight, alpha_per_layer, alpha_spec,
  best_spec).
* ``_replay_batched``: forward zonotope, the frozen layer alphas replayed once
  per layer (no Adam), then ``spec_iters`` Adam steps on the spec alphas
  warm-started from the group's frozen ones; returns (best lb, A of the best
  iterate per leaf).
* ``verify_hybrid``: root PGD, fan-out to ``init_leaves`` by widest-dimension
  bisection, the freeze on those leaves (one alpha group each), then the BaB
  loop: LIFO worklist, batches grouped by alpha group, replay, closure
  (worst disjunct's best query > 0), PGD on the worst open leaves every
  ``pgd_between_every`` iterations, widest-dimension split of the rest.

Every bound runs on this package's kernels (``interm._forward_zonotope_graph_
batched``, ``ops._spec_backward_graph_batched`` with per-query alphas on the
layer-wise CROWN kernels and the hand-written adjoint); the optimiser is
``torch.optim.Adam`` as in the reference.
"""
from __future__ import annotations

import time
import types
from collections import defaultdict

import torch

from .interm import _forward_zonotope_graph_batched
from .ops import _dev, _spec_backward_graph_batched
from .pgd import _simple_pgd, pgd_box_expand_amount


def _min_area(lo, hi, dtype):
    """Lower slope of the CROWN min-area rule: 1 where up_s > 0.5 on unstable
    neurons (verify_zono_bnb.py:503-522)."""
    lb_r = torch.clamp(lo, max=0)
    ub_r = torch.maximum(torch.clamp(hi, min=0), lb_r + 1e-8)
    up_s = ub_r / (ub_r - lb_r)
    unstable = (lo < 0) & (hi > 0)
    return (up_s > 0.5).to(dtype) * unstable.to(dtype)


def _layer_seeds(gg, n_layer, B, device, dtype):
    eye = torch.eye(n_layer, dtype=dtype, device=device)
    W_q = torch.cat([eye, -eye], dim=0)
    return W_q.unsqueeze(0).expand(B, -1, -1), torch.zeros(B, 2 * n_layer, dtype=dtype,
                                                          device=device)


def _full_freeze(xl, xh, gg, spec_ew, device, dtype, n_iters_per_layer=100, n_iters_spec=100,
                 lr=0.25, deadline=None):
    device = _dev(device)
    B = xl.shape[0]
    sb_init, _ = _forward_zonotope_graph_batched(xl, xh, gg, device, dtype)
    tight = {L: (lo.clone(), hi.clone()) for L, (lo, hi) in sb_init.items()}
    layer_order = sorted(tight.keys())
    relu_op_by_L = {op['layer_idx']: op for op in gg['ops']
                    if op['type'] == 'relu' and 'layer_idx' in op}
    alpha_per_layer = {}
    for L in layer_order:
        if deadline is not None and time.perf_counter() > deadline:
            alpha_per_layer[L] = {}
            continue
        feed = relu_op_by_L[L]['inputs'][0]
        n_layer = tight[L][0].shape[1]
        Q = 2 * n_layer
        seed, seed_acc = _layer_seeds(gg, n_layer, B, device, dtype)
        seed_ew = {feed: seed}
        alpha_at = {}
        for k in layer_order:
            if k >= L:
                break
            init = _min_area(*tight[k], dtype).unsqueeze(1).expand(-1, Q, -1).contiguous()
            alpha_at[k] = init.detach().clone().requires_grad_(True)
        if alpha_at:
            opt = torch.optim.Adam([alpha_at[k] for k in alpha_at], lr=lr)
            best = None
            prev = -float('inf')
            for it in range(n_iters_per_layer):
                opt.zero_grad()
                sl = _spec_backward_graph_batched(tight, xl, xh, gg, None, device, dtype,
                                                  alpha_at_layer=alpha_at, seed_ew_at=seed_ew,
                                                  seed_acc=seed_acc)
                with torch.no_grad():
                    best = sl.detach().clone() if best is None else torch.maximum(best, sl.detach())
                    cur = float(best.sum().item())
                (-sl.sum()).backward()
                opt.step()
                with torch.no_grad():
                    for k in alpha_at:
                        alpha_at[k].clamp_(0.0, 1.0)
                if it > 0 and cur - prev < 1e-6:
                    break
                prev = cur
                for gp in opt.param_groups:
                    gp['lr'] *= 0.98
            new_lo, new_hi = best[:, :n_layer], -best[:, n_layer:]
            lo_t = torch.maximum(tight[L][0], new_lo)
            hi_t = torch.minimum(tight[L][1], new_hi)
            tight[L] = (torch.minimum(lo_t, hi_t), hi_t)
        alpha_per_layer[L] = {k: a.detach().clone() for k, a in alpha_at.items()}
    Q_spec = len(spec_ew)
    alpha_spec = {}
    for L in layer_order:
        init = _min_area(*tight[L], dtype).unsqueeze(1).expand(-1, Q_spec, -1).contiguous()
        alpha_spec[L] = init.detach().clone().requires_grad_(True)
    opt = torch.optim.Adam([alpha_spec[L] for L in alpha_spec], lr=lr)
    best_spec = None
    prev = -float('inf')
    for it in range(n_iters_spec):
        if deadline is not None and it > 0 and time.perf_counter() > deadline:
            break
        opt.zero_grad()
        sl = _spec_backward_graph_batched(tight, xl, xh, gg, spec_ew, device, dtype,
                                          alpha_at_layer=alpha_spec)
        with torch.no_grad():
            best_spec = sl.detach().clone() if best_spec is None else \
                torch.maximum(best_spec, sl.detach())
            cur = float(best_spec.sum().item())
        (-sl.sum()).backward()
        opt.step()
        with torch.no_grad():
            for L in alpha_spec:
                alpha_spec[L].clamp_(0.0, 1.0)
        if it > 0 and cur - prev < 1e-6:
            break
        prev = cur
        for gp in opt.param_groups:
            gp['lr'] *= 0.98
    return (tight, alpha_per_layer, {k: a.detach().clone() for k, a in alpha_spec.items()},
            best_spec.detach())


def _replay_batched(xl_b, xh_b, gg, spec_ew, alpha_layer_b, alpha_spec_b, device, dtype,
                    spec_iters=10, spec_lr=0.1):
    device = _dev(device)
    B = xl_b.shape[0]
    with torch.no_grad():
        sb, _ = _forward_zonotope_graph_batched(xl_b, xh_b, gg, device, dtype)
        tight = {L: (lo.clone(), hi.clone()) for L, (lo, hi) in sb.items()}
        relu_op_by_L = {op['layer_idx']: op for op in gg['ops']
                        if op['type'] == 'relu' and 'layer_idx' in op}
        for L in sorted(tight.keys()):
            if not alpha_layer_b[L]:
                continue
            feed = relu_op_by_L[L]['inputs'][0]
            n_layer = tight[L][0].shape[1]
            seed, seed_acc = _layer_seeds(gg, n_layer, B, device, dtype)
            alpha_b = {k: a.expand(B, -1, -1).contiguous() for k, a in alpha_layer_b[L].items()}
            sl = _spec_backward_graph_batched(tight, xl_b, xh_b, gg, None, device, dtype,
                                              alpha_at_layer=alpha_b, seed_ew_at={feed: seed},
                                              seed_acc=seed_acc)
            lo_t = torch.maximum(tight[L][0], sl[:, :n_layer])
            hi_t = torch.minimum(tight[L][1], -sl[:, n_layer:])
            tight[L] = (torch.minimum(lo_t, hi_t), hi_t)
    alpha_spec = {k: a.expand(B, -1, -1).contiguous().clone().detach().requires_grad_(True)
                  for k, a in alpha_spec_b.items()}
    opt = torch.optim.Adam([alpha_spec[k] for k in alpha_spec], lr=spec_lr)
    best = best_A = None
    for _ in range(max(1, spec_iters)):
        opt.zero_grad()
        sl, A, _acc = _spec_backward_graph_batched(tight, xl_b, xh_b, gg, spec_ew, device, dtype,
                                                   alpha_at_layer=alpha_spec,
                                                   return_input_linear=True)
        with torch.no_grad():
            if best is None:
                best, best_A = sl.detach().clone(), A.detach().clone()
            else:
                imp = sl.detach() > best
                best = torch.where(imp, sl.detach(), best)
                leaf_imp = imp.any(dim=1)
                if leaf_imp.any():
                    best_A[leaf_imp] = A.detach()[leaf_imp]
        (-sl.sum()).backward()
        opt.step()
        with torch.no_grad():
            for k in alpha_spec:
                alpha_spec[k].clamp_(0.0, 1.0)
    return best, best_A


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

    t_start = time.perf_counter()
    device = torch.device('cuda')
    dtype = torch.float32
    gg = graph.gpu_graph(device, dtype)
    n_output = None
    for op in reversed(gg['ops']):
        if op['type'] == 'fc':
            n_output = int(op['W'].shape[0])
            break
    queries = spec.as_linear_queries(n_output)
    spec_ew = {qi: (torch.as_tensor(w, dtype=dtype, device=device).flatten(), float(b))
               for qi, (di, w, b) in enumerate(queries)}
    disj_q_idx = defaultdict(list)
    for qi, (di, w, b) in enumerate(queries):
        disj_q_idx[di].append(qi)
    xl_root = torch.as_tensor(spec.x_lo, dtype=dtype, device=device).flatten()[None, :]
    xh_root = torch.as_tensor(spec.x_hi, dtype=dtype, device=device).flatten()[None, :]

    # phase 0: root PGD
    if bool(getattr(settings, 'pgd_phase0_enabled', True)) and not disable_sat:
        sat, witness = _simple_pgd(xl_root, xh_root, spec, gg, n_output, device, dtype,
                                   n_restarts=10000, n_iter=50, lr=0.1,
                                   box_expand=pgd_box_expand_amount(settings))
        if sat:
            return {'verdict': 'sat', 'time': time.perf_counter() - t_start,
                    'phase': 'root_pgd', 'witness': witness}
        torch.cuda.empty_cache()

    # phase 2: fan-out and the freeze
    boxes = [(xl_root, xh_root)]
    while len(boxes) < init_leaves:
        new = []
        for xl, xh in boxes:
            d = int((xh[0] - xl[0]).argmax().item())
            mid = ((xl[0, d] + xh[0, d]) / 2).item()
            a_xh = xh.clone()
            a_xh[0, d] = mid
            b_xl = xl.clone()
            b_xl[0, d] = mid
            new.append((xl, a_xh))
            new.append((b_xl, xh))
            if len(new) >= init_leaves:
                break
        boxes = new
    boxes = boxes[:init_leaves]
    xl_init = torch.stack([b[0][0] for b in boxes])
    xh_init = torch.stack([b[1][0] for b in boxes])
    try:
        _, alpha_layer_K, alpha_spec_K, best_K = _full_freeze(
            xl_init, xh_init, gg, spec_ew, device, dtype, n_iters_per_layer=freeze_iters,
            n_iters_spec=freeze_iters, deadline=t_start + 0.8 * timeout)
    except torch.cuda.OutOfMemoryError:
        torch.cuda.empty_cache()
        return {'verdict': 'unknown', 'time': time.perf_counter() - t_start,
                'phase': 'freeze_oom'}
    per_disj_K = torch.stack([best_K[:, sorted(qids)].max(dim=1).values
                              for qids in disj_q_idx.values()], dim=1)
    worst_K = per_disj_K.min(dim=1).values
    alpha_groups = []
    for i in range(init_leaves):
        layer_i = {L: {k: a[i:i + 1].contiguous() for k, a in alpha_layer_K[L].items()}
                   for L in alpha_layer_K}
        spec_i = {k: a[i:i + 1].contiguous() for k, a in alpha_spec_K.items()}
        alpha_groups.append((layer_i, spec_i))
    open_idx_K = (worst_K <= 0).nonzero(as_tuple=True)[0].tolist()
    worklist = [(xl_init[i], xh_init[i], i) for i in open_idx_K]
    n_evaluated = init_leaves
    n_closed = init_leaves - len(open_idx_K)
    if verbose:
        print(f'  depth-K closure: {n_closed}/{init_leaves}  open={len(open_idx_K)}  '
              f'worst@K={float(worst_K.min()):+.4f}')

    # phase 3: BaB
    cur_batch = batch
    iters = 0
    n_in = xl_root.shape[1]
    while worklist:
        if time.perf_counter() - t_start > timeout - 0.5:
            return {'verdict': 'unknown', 'time': time.perf_counter() - t_start,
                    'phase': 'bab_timeout', 'residual': len(worklist),
                    'evaluated': n_evaluated, 'closed': n_closed}
        take = min(cur_batch, len(worklist))
        batch_entries = worklist[-take:]
        del worklist[-take:]
        groups = defaultdict(list)
        for idx, (xl_, xh_, gid) in enumerate(batch_entries):
            groups[gid].append((idx, xl_, xh_))
        all_best = torch.empty(len(batch_entries), len(spec_ew), dtype=dtype, device=device)
        all_A = torch.empty(len(batch_entries), len(spec_ew), n_in, dtype=dtype, device=device)
        try:
            for gid, entries in groups.items():
                idx_t = torch.tensor([e[0] for e in entries], device=device, dtype=torch.long)
                layer_g, spec_g = alpha_groups[gid]
                best_g, A_g = _replay_batched(torch.stack([e[1] for e in entries]),
                                              torch.stack([e[2] for e in entries]), gg, spec_ew,
                                              layer_g, spec_g, device, dtype)
                all_best[idx_t] = best_g
                all_A[idx_t] = A_g
        except torch.cuda.OutOfMemoryError:
            torch.cuda.empty_cache()
            worklist.extend(batch_entries)
            if cur_batch <= 8:
                return {'verdict': 'unknown', 'time': time.perf_counter() - t_start,
                        'phase': 'bab_oom'}
            cur_batch = max(8, cur_batch // 2)
            continue
        n_evaluated += len(batch_entries)
        if verbose and iters % 10 == 0:
            print(f'    iter {iters} t={time.perf_counter() - t_start:.1f} wl={len(worklist)} '
                  f'eval={n_evaluated} closed={n_closed}')
        pdb = torch.stack([all_best[:, sorted(qids)].max(dim=1).values
                           for qids in disj_q_idx.values()], dim=1)
        worst_per_leaf, _ = pdb.min(dim=1)
        closed_mask = worst_per_leaf > 0
        n_closed += int(closed_mask.sum().item())
        open_idx = (~closed_mask).nonzero(as_tuple=True)[0]
        if (pgd_between_every > 0 and not disable_sat and open_idx.numel() > 0
                and iters % pgd_between_every == 0):
            wv = worst_per_leaf[open_idx]
            for j in wv.argsort()[:min(pgd_between_k, open_idx.numel())].tolist():
                j_global = int(open_idx[j].item())
                sat, witness = _simple_pgd(
                    batch_entries[j_global][0][None, :], batch_entries[j_global][1][None, :],
                    spec, gg, n_output, device, dtype, n_restarts=pgd_between_restarts,
                    n_iter=pgd_between_iter, box_expand=pgd_box_expand_amount(settings))
                if sat:
                    return {'verdict': 'sat', 'time': time.perf_counter() - t_start,
                            'phase': 'between_pgd', 'witness': witness}
        if open_idx.numel() > 0:
            xl_b = torch.stack([batch_entries[i][0] for i in open_idx.tolist()])
            xh_b = torch.stack([batch_entries[i][1] for i in open_idx.tolist()])
            split_dims = (xh_b - xl_b).argmax(dim=1)
            mids = (xl_b.gather(1, split_dims.unsqueeze(1)).squeeze(1)
                    + xh_b.gather(1, split_dims.unsqueeze(1)).squeeze(1)) / 2
            for j_local, j_global in enumerate(open_idx.tolist()):
                d = int(split_dims[j_local].item())
                m = float(mids[j_local].item())
                xl_p, xh_p, gid_p = batch_entries[j_global]
                a_xh = xh_p.clone()
                a_xh[d] = m
                b_xl = xl_p.clone()
                b_xl[d] = m
                worklist.append((xl_p, a_xh, gid_p))
                worklist.append((b_xl, xh_p, gid_p))
        iters += 1
    return {'verdict': 'unsat', 'time': time.perf_counter() - t_start, 'phase': 'bab_complete',
            'evaluated': n_evaluated, 'closed': n_closed, 'bab_iters': iters}
