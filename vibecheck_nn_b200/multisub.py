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
* one kernel (``vcb_mlp_flirpa_fate``: the forward-LiRPA bound with the
  leaf fate in its epilogue) decides every leaf of the batch: safe
  by its bound, safe because two rounds of input-domain clipping
  (``_clip_input_domain``, verify_graph.py:11121-11177) leave an empty box,
  or to split, with its clipped box and smart-branching scores;
* a second (``vcb_multisub_emit``) ranks the dimensions of the leaves to
  split in CPU torch.topk order and writes their children: the top K
  (``bab_split_depth``, at most the number of non-degenerate dimensions)
  dimensions at once, 2^K children per leaf, appended to the worklist.
  One device-to-host copy per iteration (the fates) keeps the per-sub-box
  live-leaf counts on the host.

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


def forward_fate(desc, xl, xh, var_idx, W_q, sub_bias, sub, clip_iters=2):
    """``vcb_mlp_flirpa_fate``: the forward-LiRPA spec bound and the leaf fate
    in one kernel; returns (fate, box_lo, box_hi, score) as ``leaf_fate``."""
    dev = xl.device
    B, n = xl.shape
    K = int(var_idx.numel())
    fate = torch.empty(B + 1, dtype=torch.int32, device=dev)
    box_lo = torch.empty((B, n), dtype=F32, device=dev)
    box_hi = torch.empty((B, n), dtype=F32, device=dev)
    score = torch.empty((B, n), dtype=F32, device=dev)
    P = _lib.ptr
    rc = _lib.lib().vcb_mlp_flirpa_fate(desc.struct, B, K, P(xl.contiguous()), P(xh.contiguous()),
                                        P(var_idx), W_q.shape[0], P(W_q.contiguous()),
                                        P(sub_bias.contiguous()), P(sub), int(clip_iters),
                                        P(fate), P(box_lo), P(box_hi), P(score),
                                        _lib.stream_of(dev))
    _lib.check(rc, 'vcb_mlp_flirpa_fate')
    return fate, box_lo, box_hi, score


def leaf_fate(xl, xh, var_idx, spec_A, spec_b, lb, sub_bias, sub, clip_iters=2):
    """``vcb_multisub_fate``: (fate, box_lo, box_hi, score) of a batch.

    ``fate`` (B + 1, int32, on the device): 0 safe by its bound, 1 safe by
    the input-domain clip (``_clip_input_domain``, verify_graph.py:11121-11177,
    ``clip_iters`` rounds), 2 to split; ``fate[B]`` is the largest number of
    dimensions wider than 1e-12 among the leaves to split.  For those leaves
    ``box_lo``/``box_hi`` hold the clipped box and ``score`` the smart-branching
    score of every input dimension (verify_graph.py:11780-11802)."""
    dev = xl.device
    B, n = xl.shape
    K = int(var_idx.numel())
    Q = lb.shape[1]
    fate = torch.empty(B + 1, dtype=torch.int32, device=dev)
    box_lo = torch.empty((B, n), dtype=F32, device=dev)
    box_hi = torch.empty((B, n), dtype=F32, device=dev)
    score = torch.empty((B, n), dtype=F32, device=dev)
    P = _lib.ptr
    rc = _lib.lib().vcb_multisub_fate(B, n, K, Q, P(xl.contiguous()), P(xh.contiguous()),
                                      P(var_idx), P(spec_A), P(spec_b), P(lb),
                                      P(sub_bias.contiguous()), P(sub), int(clip_iters),
                                      P(fate), P(box_lo), P(box_hi), P(score),
                                      _lib.stream_of(dev))
    _lib.check(rc, 'vcb_multisub_fate')
    return fate, box_lo, box_hi, score


def emit_children(rows, xl, xh, score, sub, k):
    """``vcb_multisub_emit``: the 2^k children of each batch row in ``rows``
    (int32, on the device), leaf by leaf, split on its top-k dimensions by
    ``score`` in CPU torch.topk order (verify_graph.py:11804-11852).  Returns
    (kid_xl, kid_xh, kid_sub)."""
    dev = xl.device
    U = int(rows.numel())
    n = xl.shape[1]
    kid_xl = torch.empty((U << k, n), dtype=F32, device=dev)
    kid_xh = torch.empty((U << k, n), dtype=F32, device=dev)
    kid_sub = torch.empty(U << k, dtype=torch.int32, device=dev)
    lib = _lib.lib()
    ws = torch.empty(max(1, int(lib.vcb_multisub_emit_workspace(U, n, k))), dtype=torch.uint8,
                     device=dev)
    P = _lib.ptr
    rc = lib.vcb_multisub_emit(U, n, k, P(rows), P(xl.contiguous()), P(xh.contiguous()),
                               P(score.contiguous()), P(sub), P(ws), P(kid_xl), P(kid_xh),
                               P(kid_sub), _lib.stream_of(dev))
    _lib.check(rc, 'vcb_multisub_emit')
    return kid_xl, kid_xh, kid_sub


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
    sub_idx_t = torch.as_tensor(sub_idx_list, dtype=torch.int32, device=device)
    batch_size = int(getattr(settings, 'input_split_batch_size', 1024))
    K_max = int(getattr(settings, 'bab_split_depth', 4))
    live = {int(ki): 1 for ki in sub_idx_list}
    open_sub = torch.zeros(bias_np.shape[0], dtype=torch.bool, device=device)
    open_sub[sub_idx_t.long()] = True
    try:
        desc = mlp_desc(gg, device)
    except _lib.UnsupportedInput:
        desc = None
    n_iters = 0
    n_visited = 0
    newly_closed = []

    def retire(rows, si_h):
        for i in rows:
            sk = si_h[i]
            live[sk] -= 1
            if live[sk] == 0:
                closed.add(sk)
                newly_closed.append(sk)

    while xl_t.shape[0] > 0:
        if time.perf_counter() - t0 > total_budget:
            break
        if newly_closed:
            # leaves of closed sub-boxes leave the worklist
            open_sub[torch.as_tensor(newly_closed, dtype=torch.long, device=device)] = False
            newly_closed.clear()
            keep = open_sub[sub_idx_t.long()]
            xl_t, xh_t, sub_idx_t = xl_t[keep], xh_t[keep], sub_idx_t[keep]
            if xl_t.shape[0] == 0:
                break
        B = min(batch_size, xl_t.shape[0])
        xl_b, xh_b, si_b = xl_t[:B], xh_t[:B], sub_idx_t[:B]
        # varying dimensions of this batch (the forward LiRPA's compression)
        varying = (((xh_b - xl_b) / 2).abs().max(dim=0).values > 0)
        var_idx = varying.nonzero(as_tuple=True)[0].to(torch.int32)
        lirpa = None
        if desc is not None and var_idx.numel() > 0:
            try:
                lirpa = forward_fate(desc, xl_b, xh_b, var_idx, W_q, bias_table, si_b,
                                     clip_iters=2)
            except (_lib.UnsupportedInput, torch.cuda.OutOfMemoryError):
                # the reference falls back on these (verify_graph.py:11458); a
                # KernelError is a fault and propagates
                lirpa = None
        if lirpa is not None:
            fate_d, box_lo, box_hi, score = lirpa
        else:
            from .interm import _forward_zonotope_graph_batched
            from .ops import _spec_backward_graph_batched
            sb, _ = _forward_zonotope_graph_batched(xl_b, xh_b, gg, device, dtype)
            safe = torch.zeros(B, dtype=torch.bool, device=device)
            for qi in range(max_q):
                lbs_q = _spec_backward_graph_batched(sb, xl_b, xh_b, gg, {0: (W_q[qi], 0.0)},
                                                     device, dtype)[:, 0]
                safe |= (lbs_q + bias_table[si_b.long(), qi]) > 0
            # widest dimensions (verify_graph.py:11816)
            box_lo, box_hi, score = xl_b, xh_b, xh_b - xl_b
            nz = ((score > 1e-12).sum(dim=1) * (~safe)).max().reshape(1)
            fate_d = torch.cat([torch.where(safe, 0, 2), nz]).to(torch.int32)
        fate = fate_d.cpu().numpy()
        n_visited += B
        si_h = si_b.tolist()
        retire(np.nonzero(fate[:B] == 0)[0].tolist(), si_h)
        retire(np.nonzero(fate[:B] == 1)[0].tolist(), si_h)
        split = np.nonzero(fate[:B] == 2)[0]
        rest_xl, rest_xh, rest_si = xl_t[B:], xh_t[B:], sub_idx_t[B:]
        if split.size:
            n_in = xl_b.shape[1]
            k = max(1, min(K_max, int(fate[B]), n_in))
            rows = torch.as_tensor(split.astype(np.int32), device=device)
            kid_xl, kid_xh, kid_si = emit_children(rows, box_lo, box_hi, score, si_b, k)
            for i in split.tolist():
                live[si_h[i]] += (1 << k) - 1
            xl_t = torch.cat([rest_xl, kid_xl])
            xh_t = torch.cat([rest_xh, kid_xh])
            sub_idx_t = torch.cat([rest_si, kid_si])
        else:
            xl_t, xh_t, sub_idx_t = rest_xl, rest_xh, rest_si
        n_iters += 1
    last_stats.update(iters=n_iters, leaves=n_visited, closed=len(closed),
                      subs=len(sub_idx_list))
    if getattr(settings, 'print_progress', False):
        print(f'[multi-sub BAB] {n_iters} iters, {n_visited} leaves, {len(closed)}/'
              f'{len(sub_idx_list)} closed, {time.perf_counter() - t0:.1f}s', flush=True)
    return closed
