"""Layer-wise bounds for MLPs too wide for the shared-memory-resident kernels.

One ``vcb_wide_*`` launch per layer (a tiled fp32 GEMM with the layer's bound
arithmetic in its epilogue) plus small reduction kernels:

* ``wide_ibp`` -- IBP with ReLU-split clamps (verify_zono_bnb.py:1066-1153);
* ``wide_crown`` -- CROWN back-substitution with optional alpha / beta,
  optionally recording the coefficients entering each relaxation
  (verify_zono_bnb.py:4270-5134);
* ``wide_alpha_grad`` -- lb and d(sum lb)/d(alpha) by the hand-written
  adjoint (the gradient autograd computes through the back-substitution);
* ``alpha_crown_domains`` -- the alpha loop of the ReLU-split BaB
  (verify_milp.py:2762-2807, beta held at 0): IBP intermediates under each
  domain's clamps, min-area init, Adam + clamp on -sum(lb), best-of-iterations.
"""
from __future__ import annotations

import torch

from . import _lib
from .netdesc import mlp_desc
from .ops import F32, _dev

P = _lib.ptr


def _pad4(n):
    return (n + 3) // 4 * 4


class WideNet:
    """Per-layer device weights in the layouts the wide kernels read."""

    def __init__(self, desc):
        self.desc = desc
        self.dims = desc.dims
        self.W, self.Wabs, self.b, self.Waug = [], [], [], []
        for W, b in zip(desc.Ws, desc.bs):
            W = W.contiguous()
            nout, nin = W.shape
            self.W.append(W)
            self.Wabs.append(W.abs().contiguous())
            self.b.append(b.contiguous())
            aug = torch.zeros((nout, _pad4(nin + 1)), dtype=F32, device=W.device)
            aug[:, :nin] = W
            aug[:, nin] = b
            self.Waug.append(aug)


def wide_net(gg, device):
    desc = mlp_desc(gg, device)
    wn = desc.__dict__.get('_wide')
    if wn is None:
        wn = WideNet(desc)
        desc.__dict__['_wide'] = wn
    return wn


def wide_ibp(wn, xl, xh, clamps=None):
    """IBP over D domains.  clamps: {L: (cl, ch)} (D, n_L) or None.
    Returns {L: (lo, hi)} (D, n_L)."""
    dev = xl.device
    D, n0 = xl.shape
    st = _lib.stream_of(dev)
    L_ = _lib.lib()
    lda = _pad4(n0)
    mid = torch.zeros((D, lda), dtype=F32, device=dev)
    rad = torch.zeros((D, lda), dtype=F32, device=dev)
    mid[:, :n0] = (xl + xh) * 0.5
    rad[:, :n0] = (xh - xl) * 0.5
    sb = {}
    nfc = len(wn.W)
    for l in range(nfc - 1):
        nout, nin = wn.W[l].shape
        ldo = _pad4(nout)
        lo = torch.empty((D, nout), dtype=F32, device=dev)
        hi = torch.empty((D, nout), dtype=F32, device=dev)
        mid_o = torch.empty((D, ldo), dtype=F32, device=dev)
        rad_o = torch.empty((D, ldo), dtype=F32, device=dev)
        cl = ch = None
        if clamps is not None and l in clamps:
            cl = clamps[l][0].to(F32).expand(D, nout).contiguous()
            ch = clamps[l][1].to(F32).expand(D, nout).contiguous()
        rc = L_.vcb_wide_ibp_layer(D, nin, nout, P(mid), P(rad), lda, P(wn.W[l]),
                                   P(wn.Wabs[l]), P(wn.b[l]), P(cl), P(ch), P(lo),
                                   P(hi), P(mid_o), P(rad_o), ldo, st)
        _lib.check(rc, 'vcb_wide_ibp_layer')
        sb[l] = (lo, hi)
        mid, rad, lda = mid_o, rad_o, ldo
    return sb


def wide_crown(wn, xl, xh, sb, W_q, b_q, alpha=None, beta=None, want_A=False,
               record=False, want_g0=False):
    """CROWN back-substitution for D boxes x Q spec rows.

    sb {L: (lo, hi)} (D, n_L); alpha {L: (D, n_L) or (D, Q, n_L), the latter
    one slope per spec row (verify_zono_bnb.py:4423)}, beta {L: (D, n_L)} or
    None.
    Returns dict(lb (D, Q), acc (D, Q), A (D, Q, n0) if want_A, rec {L: (R, ld)}
    if record, g0 (R, ld0) if want_g0)."""
    dev = xl.device
    D, n0 = xl.shape
    Q = W_q.shape[0]
    R = D * Q
    st = _lib.stream_of(dev)
    L_ = _lib.lib()
    nfc = len(wn.W)
    nL = wn.W[-1].shape[0]
    ldc = _pad4(nL)
    coef = torch.zeros((R, ldc), dtype=F32, device=dev)
    coef[:, :nL] = W_q.repeat(D, 1)
    acc = b_q.repeat(D).contiguous().clone()
    rec = {}
    out = {}
    for l in range(nfc - 1, -1, -1):
        nout, nin = wn.W[l].shape
        ldo = _pad4(nin + 1)
        coef_o = torch.empty((R, ldo), dtype=F32, device=dev)
        bd = torch.empty(R, dtype=F32, device=dev)
        nparts = L_.vcb_wide_back_parts(R, nin)
        part = torch.empty((R, nparts), dtype=F32, device=dev)
        Lr = l - 1
        lo = hi = al = be = None
        r_buf = None
        if Lr >= 0:
            lo, hi = sb[Lr]
            lo, hi = lo.contiguous(), hi.contiguous()
            al = alpha.get(Lr) if alpha is not None else None
            be = beta.get(Lr) if beta is not None else None
            if record:
                r_buf = torch.empty((R, ldo), dtype=F32, device=dev)
                rec[Lr] = r_buf
        rc = L_.vcb_wide_back_layer(R, Q, nin, nout, P(coef), ldc, P(wn.Waug[l]),
                                    wn.Waug[l].shape[1], P(lo), P(hi),
                                    P(None if al is None else al.contiguous()),
                                    int(al is not None and al.dim() == 3),
                                    P(None if be is None else be.contiguous()),
                                    P(coef_o), P(r_buf), ldo, P(bd), P(part), st)
        _lib.check(rc, 'vcb_wide_back_layer')
        rc = L_.vcb_wide_rowsum(R, nparts, int(Lr >= 0), P(bd), P(part), P(acc), st)
        _lib.check(rc, 'vcb_wide_rowsum')
        coef, ldc = coef_o, ldo
    lb = torch.empty(R, dtype=F32, device=dev)
    A = torch.empty((R, n0), dtype=F32, device=dev) if want_A else None
    g0 = torch.empty((R, ldc), dtype=F32, device=dev) if want_g0 else None
    rc = L_.vcb_wide_concretize(R, Q, n0, ldc, P(coef), P(acc), P(xl.contiguous()),
                                P(xh.contiguous()), P(lb), P(A), P(g0), st)
    _lib.check(rc, 'vcb_wide_concretize')
    out['lb'] = lb.view(D, Q)
    out['acc'] = acc.view(D, Q)
    if want_A:
        out['A'] = A.view(D, Q, n0)
    if record:
        out['rec'] = rec
    if want_g0:
        out['g0'] = (g0, ldc)
    return out


def wide_alpha_grad(wn, xl, xh, sb, W_q, b_q, alpha, beta=None, beta_grad=False,
                    want_A=False):
    """lb (D, Q) and the per-row gradient contributions {L: (R, ld)} of
    d(sum lb)/d(alpha) (summed over the Q rows of a domain for per-domain
    alpha); with ``beta_grad`` also those of d(sum lb)/d(beta) for the split
    multipliers ``beta`` {L: (D, n_L)} added after each relaxation; with
    ``want_A`` also A (D, Q, n0) and acc (D, Q) (appended to the tuple)."""
    dev = xl.device
    D, n0 = xl.shape
    Q = W_q.shape[0]
    R = D * Q
    st = _lib.stream_of(dev)
    L_ = _lib.lib()
    res = wide_crown(wn, xl, xh, sb, W_q, b_q, alpha=alpha, beta=beta, record=True,
                     want_g0=True, want_A=want_A)
    g, ldg = res['g0']
    contrib = {}
    bcontrib = {}
    for l in range(len(wn.W) - 1):
        nout, nin = wn.W[l].shape
        rec = res['rec'][l]
        ldo = rec.shape[1]
        g_o = torch.empty((R, ldo), dtype=F32, device=dev)
        dc = torch.empty((R, ldo), dtype=F32, device=dev)
        db = torch.empty((R, ldo), dtype=F32, device=dev) if beta_grad else None
        lo, hi = sb[l]
        al = alpha.get(l) if alpha is not None else None
        rc = L_.vcb_wide_adjoint_layer(R, Q, nin, nout, P(g), ldg, P(wn.W[l]), P(wn.b[l]),
                                       P(rec), P(lo.contiguous()), P(hi.contiguous()),
                                       P(None if al is None else al.contiguous()),
                                       int(al is not None and al.dim() == 3),
                                       P(g_o), P(dc), P(db), ldo, st)
        _lib.check(rc, 'vcb_wide_adjoint_layer')
        contrib[l] = (dc, ldo)
        if beta_grad:
            bcontrib[l] = (db, ldo)
        g, ldg = g_o, ldo
    out = (res['lb'], contrib) + ((bcontrib,) if beta_grad else ())
    if want_A:
        out += (res['A'], res['acc'])
    return out


def min_area_alpha(sb):
    """alpha init = (up_s > 0.5) on unstable neurons (verify_zono_bnb.py:5170-5173)."""
    out = {}
    for L, (lo, hi) in sb.items():
        lb_r = torch.clamp(lo, max=0)
        ub_r = torch.maximum(torch.clamp(hi, min=0), lb_r + 1e-8)
        up_s = ub_r / (ub_r - lb_r)
        unstable = (lo < 0) & (hi > 0)
        out[L] = ((up_s > 0.5) & unstable).to(F32).contiguous()
    return out


def alpha_loop(wn, xl, xh, sb, W_q, b_q, n_iters, lr, lr_decay=1.0,
               early_stop_eps=None):
    """Adam on -sum(lb) over alpha with clamp to [0,1] and best-of-iterations
    lb; stops when every best lb is > 0 (and, when early_stop_eps is given,
    when the batch max improves by less than it -- verify_zono_bnb.py:5248-5288)."""
    dev = xl.device
    D = xl.shape[0]
    Q = W_q.shape[0]
    st = _lib.stream_of(dev)
    L_ = _lib.lib()
    alpha = min_area_alpha(sb)
    m1 = {L: torch.zeros_like(a) for L, a in alpha.items()}
    m2 = {L: torch.zeros_like(a) for L, a in alpha.items()}
    best = None
    prev_max = -float('inf')
    cur_lr = lr
    for it in range(max(1, n_iters)):
        lb, contrib = wide_alpha_grad(wn, xl, xh, sb, W_q, b_q, alpha)
        best = lb.clone() if best is None else torch.maximum(best, lb)
        curr_max = float(best.max().item()) if early_stop_eps is not None else 0.0
        if bool((best > 0).all().item()):
            break
        for L, a in alpha.items():
            dc, ldc = contrib[L]
            rc = L_.vcb_wide_alpha_adam(D, Q, a.shape[1], ldc, P(dc), P(a), P(m1[L]),
                                        P(m2[L]), float(cur_lr), it + 1, st)
            _lib.check(rc, 'vcb_wide_alpha_adam')
        if early_stop_eps is not None:
            if it > 0 and curr_max - prev_max < early_stop_eps:
                break
            prev_max = curr_max
        cur_lr *= lr_decay
    return best


def alpha_crown_domains(xl, xh, gg, spec_W, spec_b, relu_clamps, device='cuda',
                        n_iters=20, lr=0.1):
    """alpha-CROWN over ReLU-split domains (cfg3; verify_milp.py:2762-2807
    with beta = 0).  xl, xh (D, n_in).  Returns (best lb (D, Q), sb)."""
    device = _dev(device)
    wn = wide_net(gg, device)
    xl = torch.as_tensor(xl, device=device).to(F32).contiguous()
    xh = torch.as_tensor(xh, device=device).to(F32).contiguous()
    W_q = torch.as_tensor(spec_W, device=device).to(F32).contiguous()
    b_q = torch.as_tensor(spec_b, device=device).to(F32).contiguous()
    clamps = None
    if relu_clamps:
        clamps = {L: (torch.as_tensor(c[0], device=device), torch.as_tensor(c[1], device=device))
                  for L, c in relu_clamps.items()}
    sb = wide_ibp(wn, xl, xh, clamps)
    best = alpha_loop(wn, xl, xh, sb, W_q, b_q, n_iters, lr)
    return best, sb
