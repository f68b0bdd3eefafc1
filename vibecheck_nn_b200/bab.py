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
4. ``vcb_bab_step_ex``: closure, (iterated) clipping, branching and the
   children -- :13030-13423;
5. push the low block then the high block as two chunks (:13381-13382), or,
   for a K-dimension split, all 2^K children as one chunk (:13419-13423).

The only host round trip per iteration is the 4-word counter read that the
chunk sizes need.  Root PGD, alpha-CROWN and leaf PGD use the same kernels as
their stand-alone operators.
"""
from __future__ import annotations

import ctypes
import os
import time

import numpy as np
import torch
from torch.cuda import nvtx

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


def bab_step(xl, xh, lb, A, acc, qd, D, clip, branch_sb, q_sens=None, clip_iters=1,
             margin=None, split_depth=1, boost=None):
    """Launch vcb_bab_step_ex (vcb_bab_step_wide_ex for n_in > 64).
    ``margin`` is None or (coeff_thresh, margin_weight) for the SB margin
    score; ``boost`` an (n_in,) device tensor of SB score multipliers.
    Returns (lo_xl, lo_xh, hi_xl, hi_xh, counters); for split_depth > 1 the
    children are (lo_xl, lo_xh), all of them, and hi_xl = hi_xh = None."""
    B, n = xl.shape
    Q = lb.shape[1]
    dev = xl.device
    K = int(split_depth)
    rows = B if K == 1 else B << K
    lo_xl = torch.empty((rows, n), dtype=F32, device=dev)
    lo_xh = torch.empty_like(lo_xl)
    hi_xl = torch.empty_like(lo_xl) if K == 1 else None
    hi_xh = torch.empty_like(lo_xl) if K == 1 else None
    cnt = torch.zeros(4, dtype=torch.int64, device=dev)
    o = _lib.VcbBabOpts()
    o.clip = int(bool(clip))
    o.clip_iters = int(clip_iters)
    o.branch_sb = int(bool(branch_sb))
    o.margin_score = int(margin is not None)
    o.split_depth = K
    o.coeff_thresh = margin[0] if margin is not None else 0.01
    o.margin_weight = margin[1] if margin is not None else 1.0
    o.boost = boost.data_ptr() if boost is not None else None
    P = _lib.ptr
    L_ = _lib.lib()
    qs = Q if q_sens is None else q_sens
    kids = (P(lo_xl), P(lo_xh)) if K > 1 else (None, None)
    lohi = (P(lo_xl), P(lo_xh), P(hi_xl), P(hi_xh)) if K == 1 else (None,) * 4
    if n <= WIDE_IN:
        rc = L_.vcb_bab_step_ex(B, n, Q, D, qs, P(qd), P(xl), P(xh), P(lb), P(A), P(acc),
                                ctypes.byref(o), *lohi, *kids, P(cnt), _lib.stream_of(dev))
        _lib.check(rc, 'vcb_bab_step')
    else:
        ws_n = L_.vcb_bab_step_wide_workspace(B, n)
        ws = _lib.workspace(ws_n, dev)
        rc = L_.vcb_bab_step_wide_ex(B, n, Q, D, qs, P(qd), P(xl), P(xh), P(lb), P(A), P(acc),
                                     ctypes.byref(o), *lohi, *kids, P(cnt), P(ws), ws_n,
                                     _lib.stream_of(dev))
        _lib.check(rc, 'vcb_bab_step_wide')
    return lo_xl, lo_xh, hi_xl, hi_xh, cnt


class BabConfig:
    """The driver's settings keys, with the defaults the reference driver
    falls back to when a key is absent (its getattr defaults,
    verify_graph.py:12511-13429).  Keys whose feature is not on the B200
    path (the Gurobi LP clip and MILP escalation) raise UnsupportedInput
    when set, so the installed binding hands the call to the reference's own
    driver."""

    def __init__(self, settings):
        g = lambda k, d: _setting(settings, k, d)  # noqa: E731
        for key in ('input_split_batched_clip_full_lp', 'input_split_batched_milp_escalate'):
            if bool(g(key, False)):
                raise _lib.UnsupportedInput(
                    f'vibecheck_nn_b200: {key} (Gurobi LP / MILP) is not on the B200 path')
        self.total_budget = float(g('total_timeout', 60.0))
        self.batch_size = int(g('input_split_batch_size', 4096))
        self.max_worklist = int(g('input_split_batched_max_worklist', 200_000))
        self.clip = bool(g('input_split_batched_clip_enabled', True))
        self.clip_iters = int(g('input_split_batched_clip_iters', 1))
        self.crown_intermediate = bool(g('input_split_crown_intermediate', False))
        self.branch_sb = bool(g('input_split_batched_branch_sb', True))
        self.margin = None
        if bool(g('input_split_sb_margin_score', False)):
            self.margin = (float(g('input_split_sb_coeff_thresh', 0.01)),
                           float(g('input_split_sb_margin_weight', 1.0)))
        self.split_depth = int(g('bab_split_depth', 1))
        self.branch_boost = bool(g('input_split_batched_branch_boost', True))
        self.boost_exp = float(os.environ.get(
            'BRANCH_BOOST_EXP', str(g('input_split_batched_branch_boost_exp', 1.0))))
        self.phase_timing = (bool(g('input_split_batched_phase_timing', False))
                             or os.environ.get('VC_PHASE_TIMING', '') == '1')
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
    half) -- or, for a K-dimension split, ``lo`` holds all children and
    ``hi`` is None -- the number of rows in each block, the degenerate count,
    the leaves closed by CROWN and by clipping, and a witness if leaf PGD
    found one."""
    __slots__ = ('lo', 'hi', 'n_split', 'n_degen', 'witness', 'closed')

    def __init__(self, lo, hi, n_split, n_degen, witness=None, closed=(0, 0)):
        self.lo, self.hi = lo, hi
        self.n_split, self.n_degen, self.witness = n_split, n_degen, witness
        self.closed = closed


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

    def zonotope_bounds(self, xl_b, xh_b):
        """{relu layer: (lo, hi)} of the DeepZ forward (the branch boost's
        probe, verify_graph.py:12758-12790)."""
        lo, hi, _, _ = mlp_zono(self.desc, xl_b, xh_b)
        B = xl_b.shape[0]
        out, off = {}, 0
        for L, n in enumerate(self.desc.relu_widths):
            out[L] = (lo[off:off + B * n].view(B, n), hi[off:off + B * n].view(B, n))
            off += B * n
        return out

    boost = None  # (n_in,) SB score multipliers when the branch boost is on

    def process(self, xl_b, xh_b, n_iter, batch_size=None, timer=None):
        """Bound and split one popped batch.  ``batch_size`` (the driver's
        current one) decides the split depth: bab_split_depth while the
        popped batch is smaller, else 1 (verify_graph.py:13320-13344).
        ``timer`` (phase timing) records the bound and split phases."""
        c = self.cfg
        if timer is not None:
            timer.mark()
        # NVTX ranges name the phases for a profiler's timeline (no cost
        # without one attached)
        nvtx.range_push('vcb.bound')
        # the input-space linear form exists only with clipping, and SB
        # scoring needs it (verify_graph.py:12862-12870, :13244)
        lb, A, acc = self.bounds(xl_b, xh_b, c.clip)
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
                nvtx.range_pop()
                return StepResult(None, None, 0, 0, wit)
        nvtx.range_pop()
        if timer is not None:
            timer.mark('bound')
        nvtx.range_push('vcb.step')
        sb = c.branch_sb and c.clip
        B = xl_b.shape[0]
        K = c.split_depth if (sb and batch_size is not None and B < batch_size) else 1
        lo_xl, lo_xh, hi_xl, hi_xh, cnt = bab_step(
            xl_b, xh_b, lb, A, acc, self.qd, self.D, c.clip, sb, self.q_sens,
            clip_iters=c.clip_iters, margin=c.margin, split_depth=K,
            boost=self.boost if sb else None)
        cnt = cnt.tolist()  # host sync: chunk sizes
        nvtx.range_pop()
        if timer is not None:
            timer.mark('step')
        n_split, n_degen = int(cnt[2]), int(cnt[3])
        closed = (int(cnt[0]), int(cnt[1]))
        if K > 1:
            return StepResult((lo_xl[:n_split], lo_xh[:n_split]), None, n_split, n_degen,
                              closed=closed)
        return StepResult((lo_xl[:n_split], lo_xh[:n_split]), (hi_xl[:n_split], hi_xh[:n_split]),
                          n_split, n_degen, closed=closed)


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

    def zonotope_bounds(self, xl_b, xh_b):
        from .zono_wide import wide_zono
        return wide_zono(self.wn, xl_b, xh_b)


def branch_boost(engine, exp):
    """Per-dimension SB score multipliers (verify_graph.py:12744-12800): at
    the root, each varying input dimension's dominant shallow ReLU layer --
    the layer among the first half whose mean pre-activation width drops
    most (by more than 1e-5) when that dimension is halved -- and the boost
    (1 + unstable neurons of that layer at the root) ** exp; 1 elsewhere.
    The zonotope probes of all halved boxes run as one batch; widths are
    averaged as the reference's CPU run does (float64 sum of the float32
    widths, rounded to float32)."""
    xl0, xh0 = engine.root()
    n_in = xl0.numel()
    vary = ((xh0 - xl0) > 1e-9).nonzero(as_tuple=True)[0].tolist()
    xl = xl0.reshape(1, -1).repeat(1 + len(vary), 1)
    xh = xh0.reshape(1, -1).repeat(1 + len(vary), 1)
    for r, d in enumerate(vary, start=1):
        xh[r, d] = xl0[d] + 0.5 * (xh0[d] - xl0[d])
    sb = engine.zonotope_bounds(xl.contiguous(), xh.contiguous())
    Ls = sorted(L for L in sb if isinstance(L, int))
    shallow = Ls[:max(1, len(Ls) // 2)]
    lo = {L: sb[L][0].cpu().numpy() for L in shallow}
    hi = {L: sb[L][1].cpu().numpy() for L in shallow}

    def mean_width(L, r):
        w = (hi[L][r] - lo[L][r]).astype(np.float32)
        return float(np.float32(w.astype(np.float64).sum() / w.size))

    root_w = {L: mean_width(L, 0) for L in shallow}
    n_unst = {L: int(((lo[L][0] < 0) & (hi[L][0] > 0)).sum()) for L in shallow}
    boost = torch.ones(n_in, dtype=F32, device=engine.device)
    for r, d in enumerate(vary, start=1):
        best_L, best_delta = None, 1e-5
        for L in shallow:
            delta = root_w[L] - mean_width(L, r)
            if delta > best_delta:
                best_delta, best_L = delta, L
        if best_L is not None:
            boost[d] = (1.0 + float(n_unst[best_L])) ** exp
    return boost


def make_engine(spec, gg, settings, device):
    """The fused shared-memory engine when the network fits its kernels, the
    wide engine otherwise; with bab_split_depth > 1 and the branch boost on,
    its boost is computed at the root."""
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
    if not fused:
        eng = WideBoundEngine(spec, gg, settings, device)
    if eng.cfg.branch_boost and eng.cfg.split_depth > 1:
        try:
            eng.boost = branch_boost(eng, eng.cfg.boost_exp)
        except _lib.UnsupportedInput:  # as the reference, no boost then
            eng.boost = None
    return eng


class PhaseTimer:
    """Per-phase profile of the driver (input_split_batched_phase_timing or
    VC_PHASE_TIMING=1, verify_graph.py:12814-12833, :13436-13450): wall time
    of the bound phase (bounding, alpha-CROWN, leaf PGD) and of the step
    (closure, clipping, branching and children: one kernel here, the
    reference's clip and split phases), each ended by a device
    synchronisation, and the leaves closed by CROWN and by clipping."""

    def __init__(self, device):
        self.device = device
        self.t0 = time.perf_counter()
        self.last = None
        self.t = {'bound': 0.0, 'step': 0.0}
        self.crown_closed = 0
        self.clip_closed = 0

    def mark(self, key=None):
        torch.cuda.synchronize(self.device)
        now = time.perf_counter()
        if key is not None and self.last is not None:
            self.t[key] += now - self.last
        self.last = now

    def closed(self, crown, clip):
        self.crown_closed += crown
        self.clip_closed += clip

    def report(self, n_iters, n_leaves):
        tot = max(time.perf_counter() - self.t0, 1e-12)
        other = tot - self.t['bound'] - self.t['step']
        pct = lambda x: 100.0 * x / tot  # noqa: E731
        print(f"[vc-phase] BAB total={tot:.2f}s | bound={self.t['bound']:.2f}s "
              f"({pct(self.t['bound']):.0f}%) clip+split={self.t['step']:.2f}s "
              f"({pct(self.t['step']):.0f}%) other={other:.2f}s ({pct(other):.0f}%) | "
              f'iters={n_iters} leaves={n_leaves}', flush=True)
        print(f'[vc-phase] closures: crown={self.crown_closed} clip={self.clip_closed}',
              flush=True)
        return {'total_s': tot, 'bound_s': self.t['bound'], 'clip_split_s': self.t['step'],
                'other_s': other, 'crown_closed': self.crown_closed,
                'clip_closed': self.clip_closed}


class LocalState:
    """Per-process BaB state: the worklist and its counters."""

    def __init__(self, wl, batch_size, timer=None):
        self.wl = wl
        self.batch_size = batch_size
        self.n_leaves = 0
        self.n_iters = 0
        self.n_open = 0
        self.witness = None
        self.oom = False
        self.timer = timer


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
        res = engine.process(xl_b, xh_b, st.n_iters, st.batch_size, st.timer)
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
    if st.timer is not None:
        st.timer.closed(*res.closed)
    if res.n_split > 0:
        wl.push(*res.lo)
        if res.hi is not None:
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
    timer = PhaseTimer(device) if cfg.phase_timing else None
    st = LocalState(Worklist(*engine.root()), cfg.batch_size, timer)
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
    extra = {}
    if timer is not None:
        extra['phase_timing'] = timer.report(st.n_iters, st.n_leaves)
    if not wl and st.n_open == 0:
        return 'verified', {'phase': 'batched_verified',
                            'batched_n_leaves': st.n_leaves,
                            'batched_n_iters': st.n_iters,
                            'batched_batch_size': st.batch_size, **extra}
    return 'unknown', {'phase': 'batched_timeout',
                       'batched_n_leaves': st.n_leaves,
                       'batched_n_iters': st.n_iters,
                       'batched_worklist_left': wl.size(),
                       'batched_open_degenerate': st.n_open,
                       'batched_batch_size': st.batch_size, **extra}
