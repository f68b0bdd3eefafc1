"""Multi-subbox batched input-split BaB on the B200 kernels.

``_multi_sub_input_split_bab`` keeps the signature and results of
verify_graph.py:11180-11922 for its default configuration (forward-LiRPA
bounds, clipping before the split, smart branching over the varying input
dimensions):

* one worklist of (sub-box index, leaf box) over every sub-box of the call;
  each iteration takes the first ``input_split_batch_size`` leaves of the
  sub-boxes still open;
* bounds: batched forward linear bounds of the leaves over the varying input
  dimensions and the spec rows (``vcb_mlp_flirpa``); a leaf is safe when any
  of its sub-box's queries has a positive margin (lower bound + the sub-box's
  query bias); a sub-box closes when its last live leaf is safe;
* unsafe leaves are clipped twice (``_clip_input_domain``,
  verify_graph.py:11121-11177); a leaf clipped to an empty box is safe;
* the rest split on their top K (``bab_split_depth``, at most the number of
  non-degenerate dimensions) smart-branching dimensions at once, 2^K
  children each, appended to the worklist.

Networks the forward-LiRPA kernel does not take (widths > 64, more than 31
varying dimensions) use the zonotope + CROWN bounds per query and split on
the widest dimensions, as the reference does when its forward LiRPA fails.
Returns the set of closed sub-box indices; ``last_stats`` holds the
iteration and visited-leaf counts of the last call.
"""
from __future__ import annotations

import time

import numpy as np
import torch

from . import _lib
from .bab import LinearSpec
from .netdesc import mlp_desc
from .ops import F32, _dev
from .pgd import _disjunct_tuples

last_stats = {}


def forward_linear_spec(desc, xl, xh, var_idx, W_q, want_bounds=False):
    """``vcb_mlp_flirpa``: (spec_A (B, Q, K), spec_b (B, Q), lb (B, Q)) and,
    with ``want_bounds``, the output bounds (A_lo, A_up, b_lo, b_up)."""
    dev = xl.device
    B, _ = xl.shape
    K = int(var_idx.numel())
    Q = W_q.shape[0]
    nL = desc.n_out
    spec_A = torch.empty((B, Q, K), dtype=F32, device=dev)
    spec_b = torch.empty((B, Q), dtype=F32, device=dev)
    lb = torch.empty((B, Q), dtype=F32, device=dev)
    outs = [None] * 4
    if want_bounds:
        outs = [torch.empty((B, nL, K), dtype=F32, device=dev),
                torch.empty((B, nL, K), dtype=F32, device=dev),
                torch.empty((B, nL), dtype=F32, device=dev),
                torch.empty((B, nL), dtype=F32, device=dev)]
    P = _lib.ptr
    rc = _lib.lib().vcb_mlp_flirpa(desc.struct, B, K, P(xl.contiguous()), P(xh.contiguous()),
                                   P(var_idx), Q, P(W_q.contiguous()), P(spec_A), P(spec_b),
                                   P(lb), *[P(o) for o in outs], _lib.stream_of(dev))
    _lib.check(rc, 'vcb_mlp_flirpa')
    res = (spec_A, spec_b, lb)
    return res + tuple(outs) if want_bounds else res


def _clip_input_domain(x_L, x_U, lA, lbias, num_iters=1):
    """Closed-form input-domain shrinking (verify_graph.py:11121-11177): for
    every dimension k and query j, the point where the query's linear lower
    bound (other dimensions at their worst) crosses 0; the part of the box
    beyond it is verified by that query and dropped, minimum over queries."""
    x_L = x_L.clone()
    x_U = x_U.clone()
    for _ in range(num_iters):
        xhat = (x_U + x_L) / 2
        eps = (x_U - x_L) / 2
        lA_pos = lA.clamp(min=0)
        lA_neg = lA.clamp(max=0)
        dm_lb = (lA_pos * x_L.unsqueeze(1) + lA_neg * x_U.unsqueeze(1)).sum(dim=2) + lbias
        contrib = lA * xhat.unsqueeze(1) - lA.abs() * eps.unsqueeze(1)
        concrete_minus_one = dm_lb.unsqueeze(2) - contrib
        denom = torch.where(lA.abs() > 1e-30, lA, torch.ones_like(lA))
        curr_x = -concrete_minus_one / denom
        x_U_cand = torch.where(lA > 0, curr_x, torch.full_like(curr_x, float('inf')))
        x_L_cand = torch.where(lA < 0, curr_x, torch.full_like(curr_x, float('-inf')))
        x_U = torch.min(x_U_cand.amin(dim=1), x_U)
        x_L = torch.max(x_L_cand.amax(dim=1), x_L)
    return x_L, x_U


def _sub_queries(group, n_out):
    """(disjunct, w, bias) queries of one sub-box (x_lo, x_hi, conjuncts),
    as VNNSpec.as_linear_queries (spec.py:218-248) computes them."""
    x_lo, x_hi, conjs = group
    if conjs and isinstance(conjs[0], (list, tuple)):
        tuples = [list(c) for c in conjs]
    else:
        tuples = _disjunct_tuples(type('S', (), {'disjuncts': conjs})())
    if tuples is None:
        return None
    return LinearSpec(x_lo, x_hi, tuples).as_linear_queries(n_out)


def _multi_sub_input_split_bab(sub_idx_list, groups, order, gg, device, dtype, total_budget,
                               n_out, settings):
    t0 = time.perf_counter()
    device = _dev(device)
    closed = set()
    last_stats.clear()
    if not sub_idx_list:
        return closed
    sub_specs = {}
    for ki in sub_idx_list:
        qs = _sub_queries(groups[order[ki]], n_out)
        if qs is None:
            return closed
        sub_specs[ki] = qs
    q_counts = [len(sub_specs[ki]) for ki in sub_idx_list]
    if not q_counts or max(q_counts) == 0:
        return closed
    max_q = q_counts[0]
    uniform_q = all(c == max_q for c in q_counts)
    same_w = uniform_q and all(
        all(np.array_equal(np.asarray(sub_specs[ki][qi][1]),
                           np.asarray(sub_specs[sub_idx_list[0]][qi][1]))
            for ki in sub_idx_list) for qi in range(max_q))
    if not (uniform_q and same_w):
        return closed
    W_q = torch.as_tensor(np.stack([np.asarray(sub_specs[sub_idx_list[0]][qi][1], np.float64)
                                    for qi in range(max_q)]), dtype=F32, device=device)
    bias_np = np.zeros((max(sub_idx_list) + 1, max_q), np.float32)
    for ki in sub_idx_list:
        bias_np[ki] = [float(sub_specs[ki][qi][2]) for qi in range(max_q)]
    bias_table = torch.as_tensor(bias_np, device=device)
    xl_t = torch.as_tensor(np.stack([groups[order[ki]][0] for ki in sub_idx_list])
                           .astype(np.float64), dtype=F32, device=device)
    xh_t = torch.as_tensor(np.stack([groups[order[ki]][1] for ki in sub_idx_list])
                           .astype(np.float64), dtype=F32, device=device)
    sub_idx_t = torch.as_tensor(sub_idx_list, dtype=torch.long, device=device)
    batch_size = int(getattr(settings, 'input_split_batch_size', 1024))
    K_max = int(getattr(settings, 'bab_split_depth', 4))
    live = {int(ki): 1 for ki in sub_idx_list}
    try:
        desc = mlp_desc(gg, device)
    except _lib.UnsupportedInput:
        desc = None
    n_iters = 0
    n_visited = 0
    while xl_t.shape[0] > 0:
        if time.perf_counter() - t0 > total_budget:
            break
        B = min(batch_size, xl_t.shape[0])
        keep = torch.as_tensor([live.get(int(s), 0) > 0 for s in sub_idx_t.tolist()],
                               device=device)
        if not bool(keep.all()):
            xl_t, xh_t, sub_idx_t = xl_t[keep], xh_t[keep], sub_idx_t[keep]
            B = min(batch_size, xl_t.shape[0])
            if B == 0:
                break
        xl_b, xh_b, si_b = xl_t[:B], xh_t[:B], sub_idx_t[:B]
        # varying dimensions of this batch (the forward LiRPA's compression)
        varying = (((xh_b - xl_b) / 2).abs().max(dim=0).values > 0)
        var_idx = varying.nonzero(as_tuple=True)[0].to(torch.int32)
        lirpa = None
        if desc is not None:
            try:
                lirpa = forward_linear_spec(desc, xl_b, xh_b, var_idx, W_q)
            except (_lib.UnsupportedInput, torch.cuda.OutOfMemoryError):
                # the reference falls back on these (verify_graph.py:11458); a
                # KernelError is a fault and propagates
                lirpa = None
        clip_lA = clip_lbias = margins = None
        if lirpa is not None:
            spec_A, spec_b, lbs = lirpa
            biases = bias_table[si_b]
            margins = lbs + biases
            safe = (margins > 0).any(dim=1)
            clip_lA, clip_lbias = spec_A, spec_b + biases
            xl_c, xh_c = xl_b[:, varying], xh_b[:, varying]
        else:
            from .interm import _forward_zonotope_graph_batched
            from .ops import _spec_backward_graph_batched
            sb, _ = _forward_zonotope_graph_batched(xl_b, xh_b, gg, device, dtype)
            safe = torch.zeros(B, dtype=torch.bool, device=device)
            for qi in range(max_q):
                lbs_q = _spec_backward_graph_batched(sb, xl_b, xh_b, gg, {0: (W_q[qi], 0.0)},
                                                     device, dtype)[:, 0]
                safe |= (lbs_q + bias_table[si_b, qi]) > 0
        n_visited += B
        si_h = si_b.tolist()
        for i in np.nonzero(safe.cpu().numpy())[0].tolist():
            sk = si_h[i]
            live[sk] -= 1
            if live[sk] == 0:
                closed.add(sk)
        unsafe_idx = (~safe).nonzero(as_tuple=True)[0]
        rest_xl, rest_xh, rest_si = xl_t[B:], xh_t[B:], sub_idx_t[B:]
        if clip_lA is not None and unsafe_idx.numel() > 0:
            xl_cl, xh_cl = _clip_input_domain(xl_c[unsafe_idx], xh_c[unsafe_idx],
                                              clip_lA[unsafe_idx], clip_lbias[unsafe_idx],
                                              num_iters=2)
            vfull = varying.nonzero(as_tuple=True)[0]
            rows = unsafe_idx.unsqueeze(1).expand(-1, vfull.numel())
            cols = vfull.unsqueeze(0).expand(unsafe_idx.numel(), -1)
            xl_b = xl_b.clone()
            xh_b = xh_b.clone()
            xl_b[rows, cols] = xl_cl
            xh_b[rows, cols] = xh_cl
            newly = (xl_b[unsafe_idx] > xh_b[unsafe_idx]).any(dim=1)
            if bool(newly.any()):
                safe = safe.clone()
                add = unsafe_idx[newly]
                safe[add] = True
                for ai in add.tolist():
                    sk = si_h[ai]
                    live[sk] -= 1
                    if live[sk] == 0:
                        closed.add(sk)
                unsafe_idx = (~safe).nonzero(as_tuple=True)[0]
        if unsafe_idx.numel() > 0:
            n_in = xl_b.shape[1]
            xl_u, xh_u, si_u = xl_b[unsafe_idx], xh_b[unsafe_idx], si_b[unsafe_idx]
            widths = xh_u - xl_u
            n_u = xl_u.shape[0]
            nz = (widths > 1e-12).sum(dim=1)
            K_eff = max(1, int(min(K_max, int(nz.max().item()), n_in)))
            if clip_lA is not None:
                lA_u = clip_lA[unsafe_idx]
                wK = xh_c[unsafe_idx] - xl_c[unsafe_idx]
                score = (lA_u.abs().clamp(min=0.1) * wK.unsqueeze(1) * 0.5
                         + margins[unsafe_idx].unsqueeze(-1) * 1.0)
                sb_score = score.amax(dim=1)
                sb_full = torch.full((n_u, n_in), float('-inf'), dtype=F32, device=device)
                sb_full[:, varying.nonzero(as_tuple=True)[0]] = sb_score
                sb_full = torch.where(widths > 1e-12, sb_full, torch.full_like(sb_full,
                                                                               float('-inf')))
                # ranked on the host: tie order as the reference's CPU topk
                top = torch.topk(sb_full.cpu(), K_eff, dim=1).indices.to(device)
            else:
                top = torch.topk(widths.cpu(), K_eff, dim=1).indices.to(device)
            xl_top, xh_top = xl_u.gather(1, top), xh_u.gather(1, top)
            mids = (xl_top + xh_top) * 0.5
            usable = (xh_top - xl_top) > 1e-12
            n_ch = 1 << K_eff
            combos = torch.arange(n_ch, device=device)
            bits = (combos.unsqueeze(-1) >> torch.arange(K_eff, device=device)) & 1
            xl_e = xl_u.unsqueeze(1).expand(-1, n_ch, -1).contiguous()
            xh_e = xh_u.unsqueeze(1).expand(-1, n_ch, -1).contiguous()
            leaf_ax = torch.arange(n_u, device=device).unsqueeze(1).expand(-1, n_ch)
            child_ax = combos.unsqueeze(0).expand(n_u, -1)
            for k in range(K_eff):
                dim_k = top[:, k:k + 1].expand(-1, n_ch)
                mid_k = mids[:, k:k + 1].expand(-1, n_ch)
                use_k = usable[:, k:k + 1].expand(-1, n_ch)
                bit_k = bits[:, k].unsqueeze(0).expand(n_u, -1).bool()
                hi_m = bit_k & use_k
                lo_m = (~bit_k) & use_k
                if bool(hi_m.any()):
                    xl_e[leaf_ax[hi_m], child_ax[hi_m], dim_k[hi_m]] = mid_k[hi_m]
                if bool(lo_m.any()):
                    xh_e[leaf_ax[lo_m], child_ax[lo_m], dim_k[lo_m]] = mid_k[lo_m]
            xl_new = xl_e.reshape(-1, n_in)
            xh_new = xh_e.reshape(-1, n_in)
            si_new = si_u.unsqueeze(1).expand(-1, n_ch).reshape(-1)
            for s_val in si_u.tolist():
                live[int(s_val)] += n_ch - 1
            xl_t = torch.cat([rest_xl, xl_new])
            xh_t = torch.cat([rest_xh, xh_new])
            sub_idx_t = torch.cat([rest_si, si_new])
        else:
            xl_t, xh_t, sub_idx_t = rest_xl, rest_xh, rest_si
        n_iters += 1
    last_stats.update(iters=n_iters, leaves=n_visited, closed=len(closed),
                      subs=len(sub_idx_list))
    if getattr(settings, 'print_progress', False):
        print(f'[multi-sub BAB] {n_iters} iters, {n_visited} leaves, {len(closed)}/'
              f'{len(sub_idx_list)} closed, {time.perf_counter() - t0:.1f}s', flush=True)
    return closed
