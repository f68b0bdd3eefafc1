"""alpha-CROWN on the B200 kernels (no autograd through any kernel).

* ``_run_alpha_crown_inputsplit_batched`` -- reference signature
  (verify_zono_bnb.py:5137-5288): zonotope intermediates, min-area alpha
  init, Adam(lr) with per-iteration lr decay on -sum(lb), clamp to [0, 1],
  best-of-iterations lb, stop when every lb > 0 or the batch max improves by
  less than ``early_stop_eps``.
* ``alpha_boundary_refine`` -- the BaB's selective alpha-CROWN on boundary
  leaves (verify_graph.py:12927-12975).
* ``spec_backward_with_grad`` -- ``_spec_backward_graph_batched`` with alpha
  and beta tensors that require grad: a ``torch.autograd.Function`` whose
  backward is the hand-written adjoint kernel (beta, added after each
  relaxation, gets the adjoint itself as its gradient), so the reference's
  own ``(-lbs.sum()).backward()`` loops work unchanged -- the alpha-beta loop
  of ``_ibp_crown_bab`` (verify_milp.py:2762-2807) included.
"""
from __future__ import annotations

import torch

from .interm import mlp_zono
from .netdesc import mlp_desc
from .ops import F32, _check_dtype, _dev, _f32, _unpack_layers, spec_matrix
from . import _lib, wide


def _sb_dict(desc, B, lo, hi):
    lo_d = _unpack_layers(desc, B, lo)
    hi_d = _unpack_layers(desc, B, hi)
    return {L: (lo_d[L].contiguous(), hi_d[L].contiguous()) for L in lo_d}


def zonotope_sb(desc, xl, xh):
    try:
        lo, hi, _, _ = mlp_zono(desc, xl, xh)
    except _lib.UnsupportedInput:  # too wide for the shared-memory kernel
        from .zono_wide import wide_zono
        wn = desc.__dict__.get('_wide') or wide.WideNet(desc)
        desc.__dict__['_wide'] = wn
        return wide_zono(wn, xl, xh)
    return _sb_dict(desc, xl.shape[0], lo, hi)


def _run_alpha_crown_inputsplit_batched(xl, xh, gg, spec_ew, device, dtype,
                                        n_iters=10, lr=0.25, lr_decay=0.98,
                                        early_stop_eps=1e-6):
    """Batched alpha-CROWN for input-split leaves; returns best lb (B, Q)."""
    _check_dtype(dtype)
    device = _dev(device)
    xl = _f32(xl, device)
    xh = _f32(xh, device)
    desc = mlp_desc(gg, device)
    W_q, b_q = spec_ew if isinstance(spec_ew, tuple) else spec_matrix(spec_ew, device)
    sb = zonotope_sb(desc, xl, xh)
    wn = wide.wide_net(gg, device)
    return wide.alpha_loop(wn, xl, xh, sb, W_q, b_q, n_iters, lr, lr_decay,
                           early_stop_eps)


def alpha_boundary_refine(desc, xl, xh, lb, W_q, b_q, qd, D, eps, iters,
                          max_leaves, alpha_all, gg=None):
    """Tighten the spec lbs of the unclosed leaves whose worst disjunct's best
    query is within ``eps`` of 0 (or all unclosed leaves), at most
    ``max_leaves`` of them ordered by that margin, with alpha-CROWN
    (lr 0.25, decay 0.98) and keep the elementwise max."""
    qd = qd.long()
    closed = torch.ones(lb.shape[0], dtype=torch.bool, device=lb.device)
    best_per = []
    for d in range(D):
        cols = (qd == d).nonzero(as_tuple=True)[0]
        sub = lb[:, cols]
        closed &= (sub > 0).any(dim=1)
        best_per.append(sub.max(dim=1).values)
    if bool(closed.all()):
        return lb
    worst = torch.stack(best_per, dim=1).min(dim=1).values
    mask = ~closed if alpha_all else (~closed) & (worst > -eps)
    idx = mask.nonzero(as_tuple=True)[0]
    if idx.numel() == 0:
        return lb
    if not alpha_all:
        order = worst[idx].argsort(descending=True)
        idx = idx[order[:max_leaves]]
    xl_c, xh_c = xl[idx].contiguous(), xh[idx].contiguous()
    sb = zonotope_sb(desc, xl_c, xh_c)
    wn = desc.__dict__.get('_wide') or wide.WideNet(desc)
    desc.__dict__['_wide'] = wn
    try:
        # SIMT layer kernels: the BaB engines' leaf counts are pinned to the
        # reference's with this path's fp32 arithmetic
        new = wide.alpha_loop(wn, xl_c, xh_c, sb, W_q, b_q, iters, 0.25, 0.98, 1e-6,
                              tc=False)
    except torch.cuda.OutOfMemoryError:
        # an opportunistic tightener, as in the reference (verify_graph.py:
        # 12970-12974); a kernel fault is not swallowed
        return lb
    lb = lb.clone()
    lb[idx] = torch.maximum(lb[idx], new)
    return lb


class _SpecBackwardAlpha(torch.autograd.Function):
    """lb = CROWN(alpha, beta); backward by the hand-written adjoint.  alpha
    per layer is (D, n) (one slope per domain) or (D, Q, n) (one per spec
    row); with ``want_A`` the input-space linear bound (A, acc) is returned
    too, without gradient."""

    @staticmethod
    def forward(ctx, wn, xl, xh, sb, W_q, b_q, Ls, Lb, want_A, *params):
        alpha = {L: a.detach().contiguous() for L, a in zip(Ls, params[:len(Ls)])}
        beta = {L: b.detach().contiguous() for L, b in zip(Lb, params[len(Ls):])}
        with torch.no_grad():
            lb, contrib, bcontrib, A, acc = wide.wide_alpha_grad(
                wn, xl, xh, sb, W_q, b_q, alpha, beta=beta or None, beta_grad=True,
                want_A=True)
        ctx.Q = W_q.shape[0]
        ctx.Ls, ctx.Lb = Ls, Lb
        ctx.shapes = [tuple(alpha[L].shape) for L in Ls]
        ctx.bwidths = [beta[L].shape[1] for L in Lb]
        ctx.contrib, ctx.bcontrib = contrib, bcontrib
        if want_A:
            ctx.mark_non_differentiable(A, acc)
            return lb, A, acc
        return lb

    @staticmethod
    def backward(ctx, grad, *unused):
        w = grad.flatten()
        if not bool((w == w[0]).all()):
            raise _lib.UnsupportedInput(
                'vibecheck_nn_b200: alpha / beta gradients only for a uniform weighting '
                'of the spec lower bounds (the loss -sum(lb) the reference uses)')
        scale = w[0]

        def per_domain(store, L, n):
            dc, ldo = store[L]
            D = dc.shape[0] // ctx.Q
            return dc.view(D, ctx.Q, ldo).sum(dim=1)[:, :n] * scale

        def per_row(store, L, shape):
            dc, ldo = store[L]
            D, Q, n = shape
            return dc.view(D, Q, ldo)[:, :, :n] * scale

        res = [None] * 9
        res += [per_row(ctx.contrib, L, sh) if len(sh) == 3 else per_domain(ctx.contrib, L, sh[1])
                for L, sh in zip(ctx.Ls, ctx.shapes)]
        res += [per_domain(ctx.bcontrib, L, n) for L, n in zip(ctx.Lb, ctx.bwidths)]
        return tuple(res)


def spec_backward_with_grad(desc, lo, hi, xl, xh, spec, alpha_at_layer,
                            relu_split_beta, return_input_linear):
    """_spec_backward_graph_batched with alpha (and beta) tensors that may
    require grad: lb carries the hand-written adjoint as its backward;
    with ``return_input_linear`` also A (B, Q, n_in) and acc (B, Q), which
    carry no gradient."""
    B = xl.shape[0]
    sb = _sb_dict(desc, B, lo, hi)
    wn = desc.__dict__.get('_wide') or wide.WideNet(desc)
    desc.__dict__['_wide'] = wn
    W_q, b_q = spec
    Ls = sorted(alpha_at_layer or {})
    beta = relu_split_beta or {}
    Lb = sorted(beta)
    params = [alpha_at_layer[L] for L in Ls] + [beta[L].to(F32) for L in Lb]
    return _SpecBackwardAlpha.apply(wn, xl, xh, sb, W_q, b_q, Ls, Lb,
                                    bool(return_input_linear), *params)
