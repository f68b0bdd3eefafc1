"""Batched input-split branch-and-bound on the B200 kernels.

``_input_split_batched(graph, spec, settings, gg, device, dtype)`` has the
signature, settings keys, worklist semantics and return values of the
reference driver (verify_graph.py:12466-13464).  Per iteration:

1. pop up to ``input_split_batch_size`` boxes from the end of the chunk
   worklist (LIFO; a chunk popped in part keeps its head) -- :12695-12726;
2. bound them: CROWN intermediates (``vcb_mlp_zono`` + one ``vcb_mlp_crown``
   per layer + ``vcb_interm_intersect``) or zonotope intermediates, then the
   spec back-substitution with its input-space linear form -- :12855-12870;
3. optional alpha-CROWN on boundary leaves and leaf PGD (settings-gated, as
   in the reference);
4. ``vcb_bab_step``: closure, clipping, branching and both child blocks;
5. push the low block then the high block as two chunks -- :13381-13382.

The only host round trip per iteration is the 4-word counter read that the
chunk sizes need.  Root PGD, alpha-CROWN and leaf PGD use the same kernels as
their stand-alone operators.
"""
from __future__ import annotations

import time

import numpy as np
import torch

from . import _lib
from .interm import crown_intermediate_packed, mlp_zono
from .netdesc import mlp_desc
from .ops import F32, _dev, mlp_crown


WIDE_IN = 64  # input widths above this take the one-CTA-per-leaf step kernel


class LinearSpec:
    """Minimal stand-in for the reference ``VNNSpec``: input box plus a DNF of
    output constraints.  ``disjuncts`` is a list of lists of
    ('pair', pred, comp) | ('ge', idx, value) | ('le', idx, value)."""

    def __init__(self, x_lo, x_hi, disjuncts):
        self.x_lo = np.asarray(x_lo, np.float64)
        self.x_hi = np.asarray(x_hi, np.float64)
        self.disjuncts_raw = disjuncts

    def as_linear_queries(self, n_output):
        """spec.py:218-248: (disjunct, w, bias), safe iff w.y + bias > 0."""
        out = []
        for di, conj in enumerate(self.disjuncts_raw):
            for c in conj:
                w = np.zeros(n_output)
                if c[0] == 'pair':
                    w[c[1]], w[c[2]] = 1.0, -1.0
                    out.append((di, w, 0.0))
                elif c[0] == 'ge':
                    w[c[1]] = -1.0
                    out.append((di, w, float(c[2])))
                else:
                    w[c[1]] = 1.0
                    out.append((di, w, -float(c[2])))
        return out


def _setting(settings, name, default):
    v = getattr(settings, name, default) if settings is not None else default
    return default if v is None else v


def dedup_queries(queries, device):
    """Unique (w, b) halfspaces in first-seen order and the disjunct of each
    (verify_graph.py:12658-12681).  Returns (W_q, b_q, qd, disj_q)."""
    pos_of = {}
    ws, bs, qd = [], [], []
    disj_q = {}
    for di, w, b in queries:
        w_arr = np.asarray(w, np.float64).flatten()
        key = (w_arr.tobytes(), round(float(b), 12))
        pos = pos_of.get(key)
        if pos is None:
            pos = len(ws)
            pos_of[key] = pos
            ws.append(w_arr)
            bs.append(float(b))
            qd.append(di)
        disj_q.setdefault(di, []).append(pos)
    # the kernel maps each unique query to one disjunct; a query shared by
    # several disjuncts is replicated per disjunct for the closure/clip rule
    W = list(ws)
    B_ = list(bs)
    QD = list(qd)
    remap = {}
    for di, plist in disj_q.items():
        for p_ in plist:
            if QD[p_] != di:
                key = (p_, di)
                if key not in remap:
                    remap[key] = len(W)
                    W.append(ws[p_])
                    B_.append(bs[p_])
                    QD.append(di)
    disj_ids = sorted(disj_q)
    dmap = {d: i for i, d in enumerate(disj_ids)}
    W_q = torch.tensor(np.stack(W), dtype=F32, device=device)
    b_q = torch.tensor(B_, dtype=F32, device=device)
    qd_t = torch.tensor([dmap[d] for d in QD], dtype=torch.int32, device=device)
    return W_q, b_q, qd_t, len(disj_ids), len(ws)


class Worklist:
    """Chunked LIFO stack of (xl, xh) device blocks (verify_graph.py:12695-12726)."""

    def __init__(self, xl0, xh0):
        self.xl = [xl0.reshape(1, -1)]
        self.xh = [xh0.reshape(1, -1)]
        self.sizes = [1]

    @classmethod
    def empty(cls, n_in=None, device=None):
        wl = cls.__new__(cls)
        wl.xl, wl.xh, wl.sizes = [], [], []
        return wl

    def size(self):
        return sum(self.sizes)

    def __bool__(self):
        return bool(self.xl)

    def push(self, xl, xh):
        self.xl.append(xl)
        self.xh.append(xh)
        self.sizes.append(int(xl.shape[0]))

    def pop(self, n):
        got = 0
        pxl, pxh = [], []
        while got < n:
            m = self.sizes[-1]
            if got + m <= n:
                pxl.append(self.xl.pop())
                pxh.append(self.xh.pop())
                self.sizes.pop()
                got += m
            else:
                need = n - got
                cxl, cxh = self.xl[-1], self.xh[-1]
                pxl.append(cxl[m - need:])
                pxh.append(cxh[m - need:])
                self.xl[-1] = cxl[:m - need]
                self.xh[-1] = cxh[:m - need]
                self.sizes[-1] = m - need
                got = n
        if len(pxl) == 1:
            return pxl[0].contiguous(), pxh[0].contiguous()
        return torch.cat(pxl, 0), torch.cat(pxh, 0)


def bound_batch(desc, xl, xh, W_q, b_q, crown_intermediate, want_A):
    """Spec lower bounds (and the input-space linear form) of a batch."""
    if crown_intermediate:
        lo, hi = crown_intermediate_packed(desc, xl, xh)
    else:
        lo, hi, _, _ = mlp_zono(desc, xl, xh)
    out = mlp_crown(desc, xl, xh, sb_in=(lo, hi), spec=(W_q, b_q), want_A=want_A)
    return out['lb'], out.get('A'), out.get('acc')


def bab_step(xl, xh, lb, A, acc, qd, D, clip, branch_sb, q_sens=None):
    """Launch vcb_bab_step.  Returns (lo_xl, lo_xh, hi_xl, hi_xh, counters)."""
    B, n = xl.shape
    Q = lb.shape[1]
    dev = xl.device
    lo_xl = torch.empty((B, n), dtype=F32, device=dev)
    lo_xh = torch.empty_like(lo_xl)
    hi_xl = torch.empty_like(lo_xl)
    hi_xh = torch.empty_like(lo_xl)
    cnt = torch.zeros(4, dtype=torch.int64, device=dev)
    P = _lib.ptr
    L_ = _lib.lib()
    qs = Q if q_sens is None else q_sens
    if n <= WIDE_IN:
        rc = L_.vcb_bab_step(B, n, Q, D, qs, P(qd), P(xl), P(xh), P(lb), P(A),
                             P(acc), int(bool(clip)), int(bool(branch_sb)),
                             P(lo_xl), P(lo_xh), P(hi_xl), P(hi_xh), P(cnt),
                             _lib.stream_of(dev))
        _lib.check(rc, 'vcb_bab_step')
    else:
        ws_n = L_.vcb_bab_step_wide_workspace(B, n)
        ws = _lib.workspace(ws_n, dev)
        rc = L_.vcb_bab_step_wide(B, n, Q, D, qs, P(qd), P(xl), P(xh), P(lb), P(A), P(acc),
                                  int(bool(clip)), int(bool(branch_sb)), P(lo_xl), P(lo_xh),
                                  P(hi_xl), P(hi_xh), P(cnt), P(ws), ws_n, _lib.stream_of(dev))
        _lib.check(rc, 'vcb_bab_step_wide')
    return lo_xl, lo_xh, hi_xl, hi_xh, cnt


class BabConfig:
    """The driver's settings keys with the reference's default_settings
    values (settings.py)."""

    def __init__(self, settings):
        g = lambda k, d: _setting(settings, k, d)  # noqa: E731
        self.total_budget = float(g('total_timeout', 120.0))
        self.batch_size = int(g('input_split_batch_size', 4096))
        self.max_worklist = int(g('input_split_batched_max_worklist', 200_000))
        self.clip = bool(g('input_split_batched_clip_enabled', True))
        self.crown_intermediate = bool(g('input_split_crown_intermediate', False))
        self.branch_sb = bool(g('input_split_batched_branch_sb', False))
        self.alpha_eps = float(g('input_split_batched_alpha_boundary_eps', 0.0))
        self.alpha_iters = int(g('input_split_batched_alpha_iters', 0))
        self.alpha_all = bool(g('input_split_batched_alpha_all_leaves', False))
        self.alpha_max_leaves = int(g('input_split_batched_alpha_max_leaves', 200))
        self.leaf_pgd_every = int(g('input_split_leaf_pgd_every', 0))
        self.sat_finding = not bool(g('disable_sat_finding', False))
        self.pgd_phase0 = bool(g('pgd_phase0_enabled', True))
        self.raise_on_oom = bool(g('raise_on_oom', True))


class StepResult:
    """One bounded-and-split batch: the two child blocks (low half, high
    half), the degenerate count and a witness if leaf PGD found one."""
    __slots__ = ('lo', 'hi', 'n_split', 'n_degen', 'witness')

    def __init__(self, lo, hi, n_split, n_degen, witness=None):
        self.lo, self.hi = lo, hi
        self.n_split, self.n_degen, self.witness = n_split, n_degen, witness


class BoundEngine:
    """Bounds and splits one popped batch on the GPU (steps 2-4 above)."""

    def __init__(self, spec, gg, settings, device):
        self.cfg = BabConfig(settings)
        self.spec, self.gg, self.settings = spec, gg, settings
        self.device = device
        self.desc = mlp_desc(gg, device)
        self.n_output = self.desc.n_out
        self.n_in = self.desc.n_in
        self.queries = spec.as_linear_queries(self.n_output)
        if self.queries:
            (self.W_q, self.b_q, self.qd, self.D,
             self.q_sens) = dedup_queries(self.queries, device)

    def root(self):
        xl0 = torch.as_tensor(np.asarray(self.spec.x_lo), dtype=F32, device=self.device).flatten()
        xh0 = torch.as_tensor(np.asarray(self.spec.x_hi), dtype=F32, device=self.device).flatten()
        return xl0, xh0

    def bounds(self, xl_b, xh_b, want_A):
        return bound_batch(self.desc, xl_b, xh_b, self.W_q, self.b_q,
                           self.cfg.crown_intermediate, want_A)

    def process(self, xl_b, xh_b, n_iter):
        c = self.cfg
        lb, A, acc = self.bounds(xl_b, xh_b, c.clip or c.branch_sb)
        if c.alpha_iters > 0 and (c.alpha_all or c.alpha_eps > 0):
            from .alpha import alpha_boundary_refine
            lb = alpha_boundary_refine(self.desc, xl_b, xh_b, lb, self.W_q, self.b_q, self.qd,
                                       self.D, c.alpha_eps, c.alpha_iters, c.alpha_max_leaves,
                                       c.alpha_all)
        if c.leaf_pgd_every > 0 and c.sat_finding and n_iter % c.leaf_pgd_every == 0:
            from .pgd import leaf_pgd
            sat, wit = leaf_pgd(xl_b, xh_b, lb, self.qd, self.D, self.spec, self.gg,
                                self.n_output, self.device, self.settings)
            if sat:
                return StepResult(None, None, 0, 0, wit)
        lo_xl, lo_xh, hi_xl, hi_xh, cnt = bab_step(
            xl_b, xh_b, lb, A, acc, self.qd, self.D, c.clip, c.branch_sb, self.q_sens)
        cnt = cnt.tolist()  # host sync: chunk sizes
        n_split, n_degen = int(cnt[2]), int(cnt[3])
        return StepResult((lo_xl[:n_split], lo_xh[:n_split]), (hi_xl[:n_split], hi_xh[:n_split]),
                          n_split, n_degen)


class WideBoundEngine(BoundEngine):
    """BoundEngine for MLPs outside the shared-memory kernels (the cfg5 shape):
    zonotope intermediates on the tcgen05 GEMM (``zono_wide.wide_zono``),
    then the layer-wise CROWN back-substitution with the input-space linear
    form (``wide.wide_crown``); the split runs on the wide step kernel."""

    def __init__(self, spec, gg, settings, device):
        super().__init__(spec, gg, settings, device)
        if self.cfg.crown_intermediate:
            raise _lib.UnsupportedInput(
                'vibecheck_nn_b200: CROWN intermediates for networks outside the '
                'shared-memory kernels')
        from .wide import wide_net
        self.wn = wide_net(gg, device)

    stats = None  # a dict here collects the zonotope GEMMs' FLOPs and timing

    def bounds(self, xl_b, xh_b, want_A):
        from .wide import wide_crown
        from .zono_wide import wide_zono
        sb = wide_zono(self.wn, xl_b, xh_b, stats=self.stats)
        out = wide_crown(self.wn, xl_b, xh_b, sb, self.W_q, self.b_q, want_A=want_A)
        return out['lb'], out.get('A'), out.get('acc')


def make_engine(spec, gg, settings, device):
    """The fused shared-memory engine when the network fits its kernels, the
    wide engine otherwise."""
    eng = BoundEngine(spec, gg, settings, device)
    if not eng.queries:
        return eng
    from .ops import fits_smem
    fused = fits_smem(eng.desc, eng.W_q.shape[0])
    if fused:
        try:  # the zonotope kernel has its own limits
            xl0, xh0 = eng.root()
            mlp_zono(eng.desc, xl0.reshape(1, -1), xh0.reshape(1, -1))
        except _lib.UnsupportedInput:
            fused = False
    return eng if fused else WideBoundEngine(spec, gg, settings, device)


class LocalState:
    """Per-process BaB state: the worklist and its counters."""

    def __init__(self, wl, batch_size):
        self.wl = wl
        self.batch_size = batch_size
        self.n_leaves = 0
        self.n_iters = 0
        self.n_open = 0
        self.witness = None
        self.oom = False


def is_oom(e):
    """Out of memory, as main.py:89-99 (``_is_oom_exception``) decides it: a
    host MemoryError, torch's OutOfMemoryError (what VCB_ERR_OOM maps to), or
    a RuntimeError whose message says so.  A KernelError is never an OOM."""
    if isinstance(e, _lib.KernelError):
        return False
    return isinstance(e, (MemoryError, torch.cuda.OutOfMemoryError)) or (
        isinstance(e, RuntimeError) and 'out of memory' in str(e).lower())


def local_iteration(engine, st):
    """Pop a batch, bound and split it, push the children (LIFO: low block,
    then high block) -- one iteration of verify_graph.py:12840-13429.  On a
    bound failure the batch goes back and the batch size halves
    (:12872-12897); ``st.oom`` is set when it cannot halve further."""
    wl = st.wl
    B = min(st.batch_size, wl.size())
    xl_b, xh_b = wl.pop(B)
    try:
        res = engine.process(xl_b, xh_b, st.n_iters)
    except (MemoryError, RuntimeError) as e:
        if not is_oom(e):
            raise
        new_bs = max(1, st.batch_size // 2)
        wl.push(xl_b, xh_b)
        if new_bs == st.batch_size:
            if engine.cfg.raise_on_oom:
                raise
            st.oom = True
            return
        st.batch_size = new_bs
        return
    if res.witness is not None:
        st.witness = res.witness
        return
    st.n_leaves += B
    st.n_open += res.n_degen
    if res.n_split > 0:
        wl.push(*res.lo)
        wl.push(*res.hi)
    st.n_iters += 1


def _input_split_batched(graph, spec, settings, gg, device, dtype):
    """Worklist-based input-split BaB with batched leaf evaluation
    (verify_graph.py:12466).  Returns (verdict, details) with verdict in
    {'verified', 'unknown', 'sat'}."""
    device = _dev(device)
    t_start = time.perf_counter()
    engine = make_engine(spec, gg, settings, device)
    cfg = engine.cfg
    if cfg.sat_finding and cfg.pgd_phase0:
        from .pgd import root_pgd
        sat, wit, phase = root_pgd(spec, gg, engine.n_output, device, settings)
        if sat:
            return 'sat', {'phase': phase, 'witness': wit}
    if not engine.queries:
        return 'verified', {'phase': 'batched_no_queries'}
    st = LocalState(Worklist(*engine.root()), cfg.batch_size)
    wl = st.wl
    while wl:
        if time.perf_counter() - t_start > cfg.total_budget - 0.5:
            st.n_open = wl.size()
            break
        local_iteration(engine, st)
        if st.oom:
            return 'unknown', {'phase': 'batched_oom', 'batch_size': st.batch_size}
        if st.witness is not None:
            return 'sat', {'phase': 'batched_leaf_pgd', 'witness': st.witness}
        if wl.size() > cfg.max_worklist:
            return 'unknown', {'phase': 'batched_worklist_overflow',
                               'batched_n_leaves': st.n_leaves,
                               'batched_n_iters': st.n_iters,
                               'worklist_size': wl.size()}
    _lib.fault_check(device)  # a bounded-wait expiry makes the verdict void
    if not wl and st.n_open == 0:
        return 'verified', {'phase': 'batched_verified',
                            'batched_n_leaves': st.n_leaves,
                            'batched_n_iters': st.n_iters,
                            'batched_batch_size': st.batch_size}
    return 'unknown', {'phase': 'batched_timeout',
                       'batched_n_leaves': st.n_leaves,
                       'batched_n_iters': st.n_iters,
                       'batched_worklist_left': wl.size(),
                       'batched_open_degenerate': st.n_open,
                       'batched_batch_size': st.batch_size}
