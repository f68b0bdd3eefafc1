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


# Domains x spec rows from which alpha_loop runs on the tensor cores (3xTF32
# GEMMs with fused relaxation / adjoint / Adam stages) instead of the SIMT
# layer kernels; below it the GEMMs are too small to fill the SMs.
_TC_MIN_ROWS = 4096

# What the last alpha_loop ran: {'path': 'tc' | 'simt', 'iterations': k} (for
# the tensor-core path 'iterations' is a callable, as reading the device
# stop flags synchronises).
last_stats = {}


def _split_pad(t):
    """(rows x cols) fp32 -> TF32 (hi, lo, ld) with ld = cols rounded up to 4
    (the layout the tensor-core GEMM reads)."""
    rows, cols = t.shape
    ld = _pad4(cols)
    buf = torch.zeros((rows, ld), dtype=F32, device=t.device)
    buf[:, :cols] = t
    hi, lo = torch.empty_like(buf), torch.empty_like(buf)
    rc = _lib.lib().vcb_tf32_split(buf.numel(), P(buf), P(hi), P(lo), _lib.stream_of(t.device))
    _lib.check(rc, 'vcb_tf32_split')
    return hi, lo, ld


def _tc_operands(wn):
    """Per layer l the GEMM operands of W_l (n_out x n_in): W_l^T for the
    back-substitution C = coef @ W_l and W_l for the adjoint g @ W_l^T."""
    ops = wn.__dict__.get('_tc_ops')
    if ops is None:
        ops = ([_split_pad(W.t()) for W in wn.W], [_split_pad(W) for W in wn.W])
        wn.__dict__['_tc_ops'] = ops
    return ops


def _tc_eligible(wn, D, Q):
    return len(wn.W) >= 2 and D * Q >= _TC_MIN_ROWS


class _TcAlphaPlan:
    """Buffers and launch sequence of the tensor-core alpha loop for one
    (net, D domains, Q spec rows, iterations, lr, decay).

    Per Adam iteration, top layer down, one 3xTF32 GEMM per layer with the
    bound arithmetic in its epilogue: vcb_wtc_back_gemm (C_l = coef @ W_l
    kept as the record, the relaxation of ReLU l-1 written as the next coef's
    TF32 split, intercept and next-bias partial sums), vcb_wtc_input_gemm
    (the input box's partial sums, the adjoint seed), vcb_wtc_finish (lb,
    best, stop flag); then bottom up vcb_wtc_adj_gemm (ga = g @ W_l^T + b_l,
    alpha gradient rows, next adjoint) and vcb_wtc_adam.  Each iteration's
    launches are gated on the previous iteration's "some best lb <= 0" flag,
    so without an early-stop epsilon the whole loop is queued with no host
    synchronisation -- and, replayed from fixed buffers, captured once as a
    CUDA graph."""

    def __init__(self, wn, D, n0, Q, dev, n_iters, lr, lr_decay):
        self.wn, self.D, self.n0, self.Q, self.dev = wn, D, n0, Q, dev
        self.n_it, self.lr, self.lr_decay = max(1, n_iters), lr, lr_decay
        self.key = (id(wn), D, n0, Q, str(dev), self.n_it, lr, lr_decay)
        nfc = len(wn.W)
        self.dims = dims = [wn.W[0].shape[1]] + [W.shape[0] for W in wn.W]
        R = D * Q
        e = lambda *shape: torch.empty(shape, dtype=F32, device=dev)  # noqa: E731
        # inputs (copied in by load)
        self.xl, self.xh = e(D, n0), e(D, n0)
        self.sb = {L: (e(D, dims[L + 1]), e(D, dims[L + 1])) for L in range(nfc - 1)}
        self.W_q, self.b_q = e(Q, dims[nfc]), e(Q)
        # working buffers: records C_l (l >= 1), two split operand pairs
        # (a GEMM reads one and writes the other), alpha-gradient rows,
        # per-row partial sums (one per 64 columns of every layer)
        self.C = {l: e(R, _pad4(dims[l])) for l in range(1, nfc)}
        ldmax = max(_pad4(d) for d in dims)
        self.ops = [(e(R, ldmax), e(R, ldmax)) for _ in range(2)]
        self.ldd = max(_pad4(d) for d in dims[1:nfc])
        self.dcontrib = e(R, self.ldd)
        self.part0 = {}
        off = 0
        for l in range(nfc - 1, -1, -1):
            self.part0[l] = off
            off += (dims[l] + 63) // 64
        self.nparts = off
        self.part = e(R, off)
        self.lb, self.best = e(R), e(R)
        self.opens = torch.zeros(self.n_it, dtype=torch.int32, device=dev)
        self.err = torch.zeros(1, dtype=torch.int32, device=dev)
        self.graph = None
        self.last_it = 0

    def load(self, xl, xh, sb, W_q, b_q):
        self.xl.copy_(xl)
        self.xh.copy_(xh)
        for L, (lo, hi) in sb.items():
            self.sb[L][0].copy_(lo)
            self.sb[L][1].copy_(hi)
        self.W_q.copy_(W_q)
        self.b_q.copy_(b_q)

    def launch(self, early_stop_eps=None):
        """Queue the loop on the current stream (one host synchronisation per
        iteration only with ``early_stop_eps``)."""
        wn, D, Q, dims = self.wn, self.D, self.Q, self.dims
        R, n0, nfc = D * Q, self.n0, len(wn.W)
        st = _lib.stream_of(self.dev)
        L_ = _lib.lib()
        fwd, adj = _tc_operands(wn)
        err, C, part, ldp = self.err, self.C, self.part, self.part.shape[1]
        self.opens.zero_()
        # alpha-independent: the spec rows as the top layer's coef, and
        # acc0 = b_q + W_q . b_last
        wq = _split_pad(self.W_q.repeat(D, 1))
        qh, ql, ldq = _split_pad(self.W_q)
        bl = _split_pad(wn.b[-1][None, :])
        wb = torch.empty((Q, 4), dtype=F32, device=self.dev)
        rc = L_.vcb_tc_gemm(Q, 1, dims[nfc], P(qh), P(ql), ldq, P(bl[0]), P(bl[1]), bl[2], None,
                            P(wb), 4, P(err), st)
        _lib.check(rc, 'vcb_tc_gemm')
        acc0 = (self.b_q + wb[:, 0]).repeat(D).contiguous()
        # per ReLU layer: upper slope / intercept records and the lower
        # slopes (alpha on unstable neurons, min-area init; 1 / 0 fixed on
        # active / dead ones)
        alpha, rx = {}, {}
        for L, (s_lo, s_hi) in self.sb.items():
            alpha[L] = torch.empty_like(s_lo)
            rx[L] = torch.empty(s_lo.shape + (2,), dtype=F32, device=self.dev)
            rc = L_.vcb_wtc_relax_init(s_lo.numel(), P(s_lo), P(s_hi), P(rx[L]), P(alpha[L]),
                                       None, st)
            _lib.check(rc, 'vcb_wtc_relax_init')
        m1 = {L: torch.zeros_like(a) for L, a in alpha.items()}
        m2 = {L: torch.zeros_like(a) for L, a in alpha.items()}
        prev_max = -float('inf')
        cur_lr = self.lr
        for it in range(self.n_it):
            self.last_it = it
            gate_f = P(None if it == 0 else self.opens[it - 1:it])
            gate_a = P(self.opens[it:it + 1])
            src, ld_src = (wq[0], wq[1]), wq[2]
            k = 0
            for l in range(nfc - 1, 0, -1):
                dst = self.ops[k]
                n = dims[l]
                rc = L_.vcb_wtc_back_gemm(R, Q, n, dims[l + 1], P(src[0]), P(src[1]), ld_src,
                                          P(fwd[l][0]), P(fwd[l][1]), fwd[l][2], P(C[l]),
                                          C[l].shape[1], P(alpha[l - 1]), P(rx[l - 1]),
                                          None, P(wn.b[l - 1]), P(dst[0]), P(dst[1]), _pad4(n),
                                          P(part), ldp, self.part0[l], P(err), gate_f, st)
                _lib.check(rc, 'vcb_wtc_back_gemm')
                src, ld_src, k = dst, _pad4(n), 1 - k
            dst = self.ops[k]
            rc = L_.vcb_wtc_input_gemm(R, Q, n0, dims[1], P(src[0]), P(src[1]), ld_src,
                                       P(fwd[0][0]), P(fwd[0][1]), fwd[0][2], P(self.xl),
                                       P(self.xh), P(dst[0]), P(dst[1]), _pad4(n0), P(part), ldp,
                                       self.part0[0], P(err), gate_f, st)
            _lib.check(rc, 'vcb_wtc_input_gemm')
            rc = L_.vcb_wtc_finish(R, P(acc0), P(part), ldp, self.nparts, P(self.lb),
                                   P(self.best), int(it == 0), gate_a, gate_f, st)
            _lib.check(rc, 'vcb_wtc_finish')
            src, k = dst, 1 - k
            for l in range(nfc - 1):
                nin, nout = dims[l], dims[l + 1]
                dst = self.ops[k]
                last = l == nfc - 2
                rc = L_.vcb_wtc_adj_gemm(R, Q, nout, nin, P(src[0]), P(src[1]), _pad4(nin),
                                         P(adj[l][0]), P(adj[l][1]), adj[l][2], P(wn.b[l]),
                                         P(C[l + 1]), C[l + 1].shape[1], P(alpha[l]),
                                         P(rx[l]), P(self.dcontrib), self.ldd,
                                         None if last else P(dst[0]), None if last else P(dst[1]),
                                         _pad4(nout), P(err), gate_a, st)
                _lib.check(rc, 'vcb_wtc_adj_gemm')
                rc = L_.vcb_wtc_adam(D, Q, nout, P(self.dcontrib), self.ldd, P(alpha[l]),
                                     P(m1[l]), P(m2[l]), float(cur_lr), it + 1, gate_a, st)
                _lib.check(rc, 'vcb_wtc_adam')
                src, k = dst, 1 - k
            if early_stop_eps is not None:
                if not bool(self.opens[it].item()):
                    break
                curr_max = float(self.best.max().item())
                if it > 0 and curr_max - prev_max < early_stop_eps:
                    break
                prev_max = curr_max
            cur_lr *= self.lr_decay

    def replay(self):
        """Run the loop as one CUDA graph (captured on the first replay)."""
        if self.graph is None:
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g):
                self.launch()
            self.graph = g
        self.graph.replay()

    def finish(self):
        if int(self.err.item()):
            raise TimeoutError('vcb_tc_gemm_gated: a bounded pipeline wait expired')
        opens, it = self.opens, self.last_it
        last_stats.clear()
        last_stats.update(path='tc', iterations=lambda: 1 + int(opens[:it].sum().item()))


# The plan of the last graph-eligible call: a repeat with the same shapes and
# settings replays it as a CUDA graph (one entry bounds the memory held).
_tc_plan_cache = {}


def _tc_alpha_loop(wn, xl, xh, sb, W_q, b_q, n_iters, lr, lr_decay, early_stop_eps):
    """alpha_loop on the tensor cores (_TcAlphaPlan).  Without an early-stop
    epsilon a repeated call with the same net, shapes and settings replays
    the previous call's plan as a CUDA graph."""
    dev = xl.device
    D, n0 = xl.shape
    Q = W_q.shape[0]
    if early_stop_eps is not None:
        plan = _TcAlphaPlan(wn, D, n0, Q, dev, n_iters, lr, lr_decay)
        plan.load(xl, xh, sb, W_q, b_q)
        plan.launch(early_stop_eps)
        plan.finish()
        return plan.best.view(D, Q)
    key = (id(wn), D, n0, Q, str(dev), max(1, n_iters), lr, lr_decay)
    plan = _tc_plan_cache.get('plan')
    if plan is not None and plan.key == key and plan.wn is wn:
        plan.load(xl, xh, sb, W_q, b_q)
        plan.replay()
    else:
        _tc_plan_cache.clear()
        plan = _TcAlphaPlan(wn, D, n0, Q, dev, n_iters, lr, lr_decay)
        plan.load(xl, xh, sb, W_q, b_q)
        plan.launch()
        _tc_plan_cache['plan'] = plan
    plan.finish()
    return plan.best.view(D, Q).clone()


def alpha_loop(wn, xl, xh, sb, W_q, b_q, n_iters, lr, lr_decay=1.0,
               early_stop_eps=None, tc=None):
    """Adam on -sum(lb) over alpha with clamp to [0,1] and best-of-iterations
    lb; stops when every best lb is > 0 (and, when early_stop_eps is given,
    when the batch max improves by less than it -- verify_zono_bnb.py:5248-5288).
    ``tc``: run on the tensor cores (True), on the SIMT layer kernels (False)
    or by size (None: from _TC_MIN_ROWS domains x spec rows)."""
    if tc is None:
        tc = _tc_eligible(wn, xl.shape[0], W_q.shape[0])
    if tc and len(wn.W) >= 2:
        return _tc_alpha_loop(wn, xl, xh, sb, W_q, b_q, n_iters, lr, lr_decay, early_stop_eps)
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
    last_stats.clear()
    last_stats['path'] = 'simt'
    for it in range(max(1, n_iters)):
        last_stats['iterations'] = it + 1
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
                        n_iters=20, lr=0.1, tc=None):
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
    best = alpha_loop(wn, xl, xh, sb, W_q, b_q, n_iters, lr, tc=tc)
    return best, sb
