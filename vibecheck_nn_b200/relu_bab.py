"""ReLU-split branch-and-bound for one query on the B200 kernels.

``_ibp_crown_bab`` keeps the signature, settings and results of the
reference driver (verify_milp.py:2658-2960):

* a min-heap frontier of domains (lower bound, insertion counter, split
  clamps {(layer, neuron): side}); each step pops the ``batch`` lowest;
* per-domain pre-ReLU bounds: the IBP forward under the domain's clamps,
  intersected with the root bounds (``ops._ibp_forward_graph_batched``), or
  with ``no_reforward`` the root bounds intersected with the clamps;
* ``alpha_iters`` Adam steps (lr) on alpha (min-area or ``alpha_init``) and
  on the split multipliers beta (sign +1 for OFF, -1 for ON, beta >= 0)
  through ``ops._spec_backward_graph_batched``, whose gradient is the
  hand-written adjoint kernel; best-of-iterations lower bound; early stop
  when every domain is positive;
* kfsb branching: per unpruned domain the top ``kfsb_k`` unstable neurons by
  the BaBSR intercept score ``-lo hi / (hi - lo)`` (times ``ew_w`` when
  given; with ``no_reforward`` the score's |coefficient| factor is recomputed
  per domain from that domain's bounds), both children of every candidate
  bounded in one batched CROWN pass
  (``alpha_init`` or the default slopes, no Adam), the candidate whose worse
  child is best wins, and its unpruned children enter the frontier with
  their evaluated bounds.

Returns (closed, n_domains, reason): reason in {'closed', 'time',
'max_domains', 'exhausted_pattern'}.
"""
from __future__ import annotations

import heapq

import numpy as np
import torch

from . import _lib
from .netdesc import mlp_desc
from .ops import _check_dtype, _dev, _ibp_forward_graph_batched, _spec_backward_graph_batched


def _clamp_tensors(domains, sizes, B, device, dtype):
    """{L: (cl, ch)} (B, n_L) for the layers any of the B domains splits:
    OFF (side 0) caps the pre-activation at 0, ON (side 1) floors it at 0."""
    out = {}
    for bi, clamps in enumerate(domains):
        for (L, j), side in clamps.items():
            if L not in out:
                out[L] = (torch.full((B, sizes[L]), -np.inf, device=device, dtype=dtype),
                          torch.full((B, sizes[L]), np.inf, device=device, dtype=dtype))
            if side == 0:
                out[L][1][bi, j] = 0.0
            else:
                out[L][0][bi, j] = 0.0
    return out


def _domain_relu_coeffs(gg, sb, w_t, device, dtype):
    """Per domain, |coefficient| of the query at every ReLU output under
    that domain's bounds with the default CROWN slopes: the ``return_ew``
    output of the single-domain spec backward (verify_zono_bnb.py:2557-2560),
    for all B domains at once.  NotImplementedError for non-MLP graphs (the
    caller then keeps the given scores, as the reference does)."""
    desc = mlp_desc(gg, device)
    B = next(iter(sb.values()))[0].shape[0]
    ew = w_t.reshape(1, -1).expand(B, -1)
    out = [None] * len(desc.relu_widths)
    for L in reversed(range(len(desc.relu_widths))):
        ew = ew @ desc.Ws[L + 1].to(dtype)
        out[L] = ew.abs()
        lo, hi = sb[L]
        lb_r = torch.clamp(lo, max=0)
        ub_r = torch.maximum(torch.clamp(hi, min=0), lb_r + 1e-8)
        up_s = ub_r / (ub_r - lb_r)
        active = lo >= 0
        unstable = ~active & ~(hi <= 0)
        lo_s = ((up_s > 0.5) & unstable).to(dtype) + active.to(dtype)
        ew = ew.clamp(min=0) * lo_s + ew.clamp(max=0) * up_s
    return [{L: out[L][bi] for L in range(len(out))} for bi in range(B)]


def _ibp_crown_bab(gg, xl, xh, sb_root, w_q, b_q, device, dtype, *, time_left, ew_w=None,
                   batch=64, alpha_iters=8, lr=0.25, max_domains=500000,
                   print_progress=False, alpha_init=None, kfsb_k=4, split_deepest=False,
                   no_reforward=False):
    _check_dtype(dtype)
    device = _dev(device)
    w_t = (w_q.to(device=device, dtype=dtype) if torch.is_tensor(w_q)
           else torch.as_tensor(np.asarray(w_q), device=device, dtype=dtype))
    spec = {0: (w_t, float(b_q))}
    root = {L: (lo.detach().to(device), hi.detach().to(device)) for L, (lo, hi) in sb_root.items()}
    sizes = {L: lo.numel() for L, (lo, _) in root.items()}
    xl = torch.as_tensor(xl, device=device, dtype=dtype).flatten()
    xh = torch.as_tensor(xh, device=device, dtype=dtype).flatten()

    def boxes(n):
        return (xl.unsqueeze(0).expand(n, -1).contiguous(),
                xh.unsqueeze(0).expand(n, -1).contiguous())

    def domain_bounds(clamps, n):
        if no_reforward:
            sb = {}
            for L, (lo_r, hi_r) in root.items():
                lo = lo_r.unsqueeze(0).expand(n, -1).clone()
                hi = hi_r.unsqueeze(0).expand(n, -1).clone()
                if L in clamps:
                    lo = torch.maximum(lo, clamps[L][0])
                    hi = torch.minimum(hi, clamps[L][1])
                    hi = torch.maximum(hi, lo)
                sb[L] = (lo, hi)
            return sb
        bl, bh = boxes(n)
        return _ibp_forward_graph_batched(bl, bh, gg, device, dtype,
                                          relu_clamps=clamps or None, root_sb=root)

    counter = 0
    frontier = [(-float('inf'), counter, {})]
    n_domains = 0
    n_report = 0
    while frontier:
        if time_left() <= 3.0:
            return False, n_domains, 'time'
        if n_domains >= max_domains:
            return False, n_domains, 'max_domains'
        popped = [heapq.heappop(frontier) for _ in range(min(batch, len(frontier)))]
        B = len(popped)
        n_domains += B
        doms = [d[2] for d in popped]
        clamps = _clamp_tensors(doms, sizes, B, device, dtype)
        with torch.no_grad():
            sb = domain_bounds(clamps, B)
        bl, bh = boxes(B)
        # alpha: the caller's root alpha or the min-area choice; beta per
        # split layer with the halfspace sign of each clamp
        alpha = {}
        for L, (lo, hi) in sb.items():
            if alpha_init is not None and L in alpha_init:
                a0 = alpha_init[L].detach().to(device=device, dtype=dtype).unsqueeze(0).expand(B, -1)
            else:
                lb_r = torch.clamp(lo, max=0)
                ub_r = torch.maximum(torch.clamp(hi, min=0), lb_r + 1e-8)
                up_s = ub_r / (ub_r - lb_r)
                unstable = (lo < 0) & (hi > 0)
                a0 = (up_s > 0.5).to(dtype) * unstable.to(dtype)
            alpha[L] = a0.detach().clone().requires_grad_(True)
        sign = {}
        beta = {}
        for L, (cl, ch) in clamps.items():
            s = torch.zeros_like(cl)
            s[ch == 0] = 1.0
            s[cl == 0] = -1.0
            sign[L] = s
            beta[L] = torch.zeros_like(cl).requires_grad_(True)
        opt = torch.optim.Adam(list(alpha.values()) + list(beta.values()), lr=lr)
        best = None
        for _ in range(max(1, alpha_iters)):
            opt.zero_grad()
            rsb = {L: beta[L] * sign[L] for L in beta} or None
            lbs = _spec_backward_graph_batched(sb, bl, bh, gg, spec, device, dtype,
                                               alpha_at_layer=alpha, relu_split_beta=rsb)[:, 0]
            with torch.no_grad():
                best = lbs.detach().clone() if best is None else torch.maximum(best, lbs.detach())
            if bool((best > 0).all()) or time_left() <= 3.0:
                break
            (-lbs.sum()).backward()
            opt.step()
            with torch.no_grad():
                for a in alpha.values():
                    a.clamp_(0.0, 1.0)
                for b in beta.values():
                    b.clamp_(min=0.0)
        best_h = best.cpu().numpy()
        with torch.no_grad():
            cands = []   # (bi, (L, j)) in evaluation order
            ew_dom = None
            if no_reforward and ew_w is not None:
                try:
                    ew_dom = _domain_relu_coeffs(gg, sb, w_t, device, dtype)
                except _lib.UnsupportedInput:
                    ew_dom = None
            for bi in range(B):
                if float(best_h[bi]) > 0:
                    continue
                ew_bi = ew_dom[bi] if ew_dom is not None else ew_w
                if split_deepest:
                    layers = [L for L in sorted(sb)
                              if bool(((sb[L][0][bi] < 0) & (sb[L][1][bi] > 0)).any())][-1:]
                else:
                    layers = list(sb)
                scored = []
                for L in layers:
                    lo, hi = sb[L][0][bi], sb[L][1][bi]
                    unstable = (lo < 0) & (hi > 0)
                    if not bool(unstable.any()):
                        continue
                    gap = (-lo * hi) / (hi - lo).clamp(min=1e-12)
                    score = gap * unstable.to(dtype)
                    if ew_bi is not None and L in ew_bi:
                        score = score * ew_bi[L]
                    k = min(kfsb_k, int(unstable.sum()))
                    vals, idxs = torch.topk(score, k)
                    scored += [(v, (L, int(j))) for v, j in zip(vals.tolist(), idxs.tolist())
                               if v > 0]
                if not scored:
                    # every neuron of this domain is fixed and its bound is
                    # still <= 0: splitting cannot help
                    return False, n_domains, 'exhausted_pattern'
                scored.sort(reverse=True)
                cands += [(bi, key) for _, key in scored[:kfsb_k]]
            if not cands:
                continue
            # both children of every candidate, in chunks, default slopes
            n_child = 2 * len(cands)
            child_lb = np.empty(n_child)
            chunk = max(8, batch)
            for c0 in range(0, n_child, chunk):
                rows = range(c0, min(c0 + chunk, n_child))
                kids = []
                for r in rows:
                    bi, key = cands[r // 2]
                    c = dict(doms[bi])
                    c[key] = r % 2
                    kids.append(c)
                Bc = len(kids)
                kc = _clamp_tensors(kids, sizes, Bc, device, dtype)
                sbc = domain_bounds(kc, Bc)
                alc = {}
                if alpha_init is not None:
                    for L in sbc:
                        if L in alpha_init:
                            alc[L] = alpha_init[L].detach().to(device=device, dtype=dtype) \
                                .unsqueeze(0).expand(Bc, -1)
                cl_, ch_ = boxes(Bc)
                lbs = _spec_backward_graph_batched(sbc, cl_, ch_, gg, spec, device, dtype,
                                                   alpha_at_layer=alc or None)[:, 0]
                child_lb[c0:c0 + Bc] = lbs.detach().cpu().numpy()
            # per domain: the candidate whose worse child is best
            choice = {}
            for slot, (bi, key) in enumerate(cands):
                worse = min(child_lb[2 * slot], child_lb[2 * slot + 1])
                if bi not in choice or worse > choice[bi][0]:
                    choice[bi] = (worse, slot, key)
            for bi in sorted(choice):
                _, slot, key = choice[bi]
                for side in (0, 1):
                    lb_child = float(child_lb[2 * slot + side])
                    if lb_child > 0:
                        continue
                    counter += 1
                    child = dict(doms[bi])
                    child[key] = side
                    heapq.heappush(frontier, (lb_child, counter, child))
        if print_progress and n_domains >= n_report + 2048:
            n_report = n_domains
            worst = min((d[0] for d in frontier), default=0.0)
            print(f'    [ibp-bab] {n_domains} domains, frontier {len(frontier)}, '
                  f'worst lb {worst:.4f}', flush=True)
    return True, n_domains, 'closed'
