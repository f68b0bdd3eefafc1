"""Generate golden vectors by running the reference's own Python code.

Usage::

    python tests/golden/make_golden.py --ref-src <vibecheck checkout>/src

Imports ``vibecheck`` from the given source tree (with an empty ``gurobipy``
stub: only ``gurobi_util.py:22`` imports it at module level and the bound
path never calls it), runs the hot-path functions on small seeded cases on
CPU, and writes ``tests/golden/*.npz``.  The committed fixtures are what the
CPU tests check the oracle against; the reference itself is not needed at
test time.
"""
from __future__ import annotations

import argparse
import os
import sys
import types

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(os.path.dirname(HERE)))


def _import_reference(src):
    sys.modules.setdefault('gurobipy', types.ModuleType('gurobipy'))
    sys.path.insert(0, src)
    import torch
    torch.set_num_threads(4)
    import vibecheck.verify_zono_bnb as vz
    import vibecheck.verify_graph as vg
    import vibecheck.verify_hybrid_acasxu as vh
    import vibecheck.settings as vs
    import vibecheck.spec as vspec
    return vz, vg, vh, vs, vspec


def _t(a, dtype):
    import torch
    return torch.as_tensor(np.asarray(a), dtype=dtype)


def _n(t):
    return t.detach().cpu().numpy()


def _save(name, **arrays):
    path = os.path.join(HERE, name + '.npz')
    np.savez_compressed(path, **arrays)
    print('wrote', path, sum(a.nbytes for a in arrays.values()), 'bytes raw')


def _net_arrays(layers):
    out = {}
    for i, (W, b) in enumerate(layers):
        out[f'W{i}'] = np.asarray(W, np.float32)
        out[f'b{i}'] = np.asarray(b, np.float32)
    out['n_layers'] = np.array(len(layers))
    return out


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument('--ref-src', required=True)
    ap.add_argument('--only', default=None,
                    choices=['pgd_general', 'forward', 'relu_bab', 'hybrid', 'multisub',
                             'cfg2', 'bab_branching', 'acasxu'],
                    help='regenerate one fixture only')
    args = ap.parse_args()
    vz, vg, vh, vs, vspec = _import_reference(args.ref_src)
    import torch
    from vibecheck_nn_b200 import workloads as wk
    if args.only == 'pgd_general':
        _golden_pgd_general(vspec, wk)
        return
    if args.only == 'forward':
        _golden_forward(vz, wk)
        return
    if args.only == 'relu_bab':
        _golden_relu_bab(vz, wk)
        return
    if args.only == 'hybrid':
        _golden_hybrid(wk)
        return
    if args.only == 'multisub':
        _golden_multisub(wk)
        return
    if args.only == 'cfg2':
        _golden_cfg2(vz, wk)
        return
    if args.only == 'bab_branching':
        _golden_bab_branching(vg, vs, vspec, wk)
        return
    if args.only == 'acasxu':
        _golden_acasxu(args.ref_src, vg, vs)
        return

    # ------------------------------------------------------------------ slopes
    lo = np.array([1.0, 2.0, -3.0, -2.0, -1.0, 1.0, -1.0, -3.0, 0.0, -0.0,
                   -5e-9, -1e-9, -0.2, -0.7], np.float32)
    hi = np.array([3.0, 4.0, -1.0, -0.5, 3.0, 2.0, 1.0, -1.0, 0.0, 0.3,
                   -1e-9, 0.0, 0.6, 0.3], np.float32)
    rng = np.random.default_rng(11)
    rl = rng.normal(size=200).astype(np.float32)
    rh = (rl + np.abs(rng.normal(size=200))).astype(np.float32)
    lo = np.concatenate([lo, rl])
    hi = np.concatenate([hi, rh])
    res = vz._make_slopes(_t(lo, torch.float32), _t(hi, torch.float32))
    _save('slopes', lo=lo, hi=hi, lo_s=_n(res[0]), up_s=_n(res[1]),
          up_t=_n(res[2]), active=_n(res[3]), dead=_n(res[4]),
          unstable=_n(res[5]))

    # --------------------------------------------- IBP + CROWN, small + ACAS
    for tag, dims, B, Q, seed in (('small', (6, 9, 7, 4), 5, 3, 1),
                                  ('acas', wk.ACAS_DIMS, 24, 4, 2)):
        rng = np.random.default_rng(seed)
        layers = wk.mlp_params(dims, rng)
        centre = rng.uniform(-0.5, 0.5, (B, dims[0]))
        half = rng.uniform(0.001, 0.3, (B, dims[0]))
        xl = (centre - half).astype(np.float32)
        xh = (centre + half).astype(np.float32)
        SW = rng.integers(-1, 2, (Q, dims[-1])).astype(np.float32)
        Sb = rng.normal(size=Q).astype(np.float32)
        # clamps on layer 0: two neurons ON/OFF in alternating domains
        n0 = dims[1]
        cl = np.full((B, n0), -np.inf, np.float32)
        ch = np.full((B, n0), np.inf, np.float32)
        cl[::2, 0] = 0.0
        ch[1::2, 0] = 0.0
        ch[::3, 1] = 0.0
        out = dict(_net_arrays(layers), xl=xl, xh=xh, spec_W=SW, spec_b=Sb,
                   clamp_lo0=cl, clamp_hi0=ch)
        for bits, dt in ((32, torch.float32), (64, torch.float64)):
            gg = wk.mlp_gg(layers, 'cpu', dt)
            spec_ew = {q: (_t(SW[q], dt), float(Sb[q])) for q in range(Q)}
            txl, txh = _t(xl, dt), _t(xh, dt)
            sb = vz._ibp_forward_graph_batched(txl, txh, gg, 'cpu', dt)
            for L, (l_, h_) in sb.items():
                out[f'ibp{bits}_lo{L}'] = _n(l_)
                out[f'ibp{bits}_hi{L}'] = _n(h_)
            lb, A, acc = vz._spec_backward_graph_batched(
                sb, txl, txh, gg, spec_ew, 'cpu', dt, return_input_linear=True)
            out[f'crown{bits}_lb'] = _n(lb)
            out[f'crown{bits}_A'] = _n(A)
            out[f'crown{bits}_acc'] = _n(acc)
            sbc = vz._ibp_forward_graph_batched(
                txl, txh, gg, 'cpu', dt,
                relu_clamps={0: (_t(cl, dt), _t(ch, dt))})
            for L, (l_, h_) in sbc.items():
                out[f'ibpc{bits}_lo{L}'] = _n(l_)
                out[f'ibpc{bits}_hi{L}'] = _n(h_)
            lbc = vz._spec_backward_graph_batched(sbc, txl, txh, gg, spec_ew,
                                                  'cpu', dt)
            out[f'crownc{bits}_lb'] = _n(lbc)
            # zonotope forward + CROWN intermediates + spec on them
            zsb, (zc, zG) = vz._forward_zonotope_graph_batched(
                txl, txh, gg, 'cpu', dt)
            for L, (l_, h_) in zsb.items():
                out[f'zono{bits}_lo{L}'] = _n(l_)
                out[f'zono{bits}_hi{L}'] = _n(h_)
            out[f'zono{bits}_c'] = _n(zc)
            if bits == 32:
                out[f'zono{bits}_G'] = _n(zG)
            tight = vz._crown_intermediate_batched(gg, txl, txh, 'cpu', dt)
            for L, (l_, h_) in tight.items():
                out[f'interm{bits}_lo{L}'] = _n(l_)
                out[f'interm{bits}_hi{L}'] = _n(h_)
            lbi, Ai, acci = vz._spec_backward_graph_batched(
                tight, txl, txh, gg, spec_ew, 'cpu', dt,
                return_input_linear=True)
            out[f'spec_interm{bits}_lb'] = _n(lbi)
            out[f'spec_interm{bits}_A'] = _n(Ai)
            out[f'spec_interm{bits}_acc'] = _n(acci)
            # alpha-CROWN on the input-split leaves
            lba = vz._run_alpha_crown_inputsplit_batched(
                txl, txh, gg, spec_ew, 'cpu', dt, n_iters=6, lr=0.25,
                lr_decay=0.98)
            out[f'alpha{bits}_lb'] = _n(lba)
        _save(f'mlp_{tag}', **out)

    # zero-radius input dim (generator dropping) ------------------------------
    rng = np.random.default_rng(5)
    layers = wk.mlp_params((4, 6, 3), rng)
    xl = rng.uniform(-1, 0, (3, 4)).astype(np.float32)
    xh = (xl + rng.uniform(0.1, 1, (3, 4))).astype(np.float32)
    xh[:, 2] = xl[:, 2]
    gg = wk.mlp_gg(layers, 'cpu', torch.float32)
    zsb, (zc, zG) = vz._forward_zonotope_graph_batched(
        _t(xl, torch.float32), _t(xh, torch.float32), gg, 'cpu', torch.float32)
    _save('zono_zero_radius', **_net_arrays(layers), xl=xl, xh=xh,
          lo0=_n(zsb[0][0]), hi0=_n(zsb[0][1]), c=_n(zc), G=_n(zG))

    # --------------------------------------------------------------- clipping
    rng = np.random.default_rng(7)
    B, Q, n = 40, 3, 5
    xl = rng.uniform(-1, 0, (B, n)).astype(np.float32)
    xh = (xl + rng.uniform(0.05, 1, (B, n))).astype(np.float32)
    A = rng.normal(size=(B, Q, n)).astype(np.float32)
    A[0, 0, 1] = 0.0
    A[1, :, 2] = 1e-13
    bb = rng.normal(size=(B, Q)).astype(np.float32)
    xl2, xh2, feas = vg._clip_box_by_halfspaces_batched(
        _t(xl, torch.float32), _t(xh, torch.float32), _t(A, torch.float32),
        _t(bb, torch.float32))
    _save('clip', xl=xl, xh=xh, A=A, b=bb, xl_new=_n(xl2), xh_new=_n(xh2),
          feasible=_n(feas))

    # ------------------------------------------------- alpha-CROWN on domains
    # The alpha loop of verify_milp._ibp_crown_bab (:2762-2807) with beta
    # held at zero, restated with the reference's own kernels + torch Adam.
    rng = np.random.default_rng(9)
    dims = (12, 16, 16, 16, 5)
    layers = wk.mlp_params(dims, rng)
    x0 = rng.uniform(0, 1, dims[0])
    xl1 = np.clip(x0 - 0.08, 0, 1).astype(np.float32)
    xh1 = np.clip(x0 + 0.08, 0, 1).astype(np.float32)
    y0 = wk._mlp_forward64(layers, x0[None])[0]
    t_lab = int(np.argmax(y0))
    SW, Sb = wk.margin_rows(dims[-1], t_lab)
    gg = wk.mlp_gg(layers, 'cpu', torch.float32)
    dt = torch.float32
    root = vz._ibp_forward_graph_batched(_t(xl1[None], dt), _t(xh1[None], dt),
                                         gg, 'cpu', dt)
    picked, clamps = wk.split_domains(
        {L: _n(v[0][0]) for L, v in root.items()},
        {L: _n(v[1][0]) for L, v in root.items()}, 3)
    D = 1 << len(picked)
    xl = np.broadcast_to(xl1, (D, dims[0])).copy()
    xh = np.broadcast_to(xh1, (D, dims[0])).copy()
    txl, txh = _t(xl, dt), _t(xh, dt)
    rc = {L: (_t(c_[0], dt), _t(c_[1], dt)) for L, c_ in clamps.items()}
    sb = vz._ibp_forward_graph_batched(txl, txh, gg, 'cpu', dt, relu_clamps=rc)
    alpha = {}
    for L, (l_, h_) in sb.items():
        _, up_s, _, _, _, unst = vz._make_slopes(l_, h_)
        alpha[L] = ((up_s > 0.5).to(dt) * unst.to(dt)).clone().requires_grad_(True)
    spec_ew = {q: (_t(SW[q], dt), float(Sb[q])) for q in range(SW.shape[0])}
    opt = torch.optim.Adam(list(alpha.values()), lr=0.1)
    best = None
    for _ in range(8):
        opt.zero_grad()
        lbs = vz._spec_backward_graph_batched(sb, txl, txh, gg, spec_ew, 'cpu',
                                              dt, alpha_at_layer=alpha)
        best = lbs.detach().clone() if best is None else torch.maximum(
            best, lbs.detach())
        if (best > 0).all():
            break
        (-lbs.sum()).backward()
        opt.step()
        with torch.no_grad():
            for L in alpha:
                alpha[L].clamp_(0.0, 1.0)
    clamp_arrays = {}
    for L, (c0, c1) in clamps.items():
        clamp_arrays[f'clamp_lo{L}'] = c0
        clamp_arrays[f'clamp_hi{L}'] = c1
    _save('alpha_domains', **_net_arrays(layers), **clamp_arrays, xl=xl, xh=xh,
          spec_W=SW, spec_b=Sb, n_iters=np.array(8), lr=np.array(0.1),
          best_lb=_n(best))

    # ------------------------------------------------------------------- conv
    rng = np.random.default_rng(13)
    k1 = (rng.standard_normal((4, 2, 3, 3)) * 0.4).astype(np.float32)
    b1 = (rng.standard_normal(4) * 0.01).astype(np.float32)
    W2 = (rng.standard_normal((6, 4 * 4 * 4)) * 0.2).astype(np.float32)
    b2 = (rng.standard_normal(6) * 0.01).astype(np.float32)
    W3 = (rng.standard_normal((3, 6)) * 0.5).astype(np.float32)
    b3 = (rng.standard_normal(3) * 0.01).astype(np.float32)
    ins = (2, 8, 8)
    ggc = _small_cnn_gg(k1, b1, W2, b2, W3, b3, ins, dt)
    B = 4
    x0 = rng.uniform(0, 1, (B, int(np.prod(ins))))
    xl = (x0 - 0.05).astype(np.float32)
    xh = (x0 + 0.05).astype(np.float32)
    SW = rng.integers(-1, 2, (2, 3)).astype(np.float32)
    Sb = np.zeros(2, np.float32)
    txl, txh = _t(xl, dt), _t(xh, dt)
    spec_ew = {q: (_t(SW[q], dt), float(Sb[q])) for q in range(2)}
    sb = vz._ibp_forward_graph_batched(txl, txh, ggc, 'cpu', dt)
    lb, A, acc = vz._spec_backward_graph_batched(sb, txl, txh, ggc, spec_ew,
                                                 'cpu', dt,
                                                 return_input_linear=True)
    zsb, (zc, zG) = vz._forward_zonotope_graph_batched(txl, txh, ggc, 'cpu', dt)
    out = dict(k1=k1, b1=b1, W2=W2, b2=b2, W3=W3, b3=b3, xl=xl, xh=xh,
               spec_W=SW, spec_b=Sb, lb=_n(lb), A=_n(A), acc=_n(acc),
               zc=_n(zc))
    for L, (l_, h_) in sb.items():
        out[f'ibp_lo{L}'] = _n(l_)
        out[f'ibp_hi{L}'] = _n(h_)
    for L, (l_, h_) in zsb.items():
        out[f'zono_lo{L}'] = _n(l_)
        out[f'zono_hi{L}'] = _n(h_)
    _save('conv_small', **out)

    # ---------------------------------------------------------- batched PGD
    rng = np.random.default_rng(17)
    layers = wk.mlp_params((5, 20, 20, 4), rng)
    gg = wk.mlp_gg(layers, 'cpu', dt)
    Bp, R = 6, 16
    c_ = rng.uniform(-0.5, 0.5, (Bp, 5))
    h_ = rng.uniform(0.05, 0.3, (Bp, 5))
    xl = (c_ - h_).astype(np.float32)
    xh = (c_ + h_).astype(np.float32)
    pts = xl[:, None, :] + (xh - xl)[:, None, :] * rng.random((Bp, 64, 5))
    ys = wk._mlp_forward64(layers, pts.reshape(-1, 5).astype(np.float64))
    spec_results = {}
    for tag, thr in (('unsat', float(ys[:, 0].max() + 0.2)),
                     ('sat', float(np.median(ys[:, 0])))):
        spec = vspec.VNNSpec(
            x_lo=xl[0].astype(np.float64), x_hi=xh[0].astype(np.float64),
            disjuncts=[vspec.Conjunct([vspec.Constraint(0, '>=', thr)]),
                       vspec.Conjunct([vspec.PairwiseConstraint(1, 2),
                                       vspec.Constraint(3, '<=', -50.0)])])
        torch.manual_seed(0)
        lo_e = _t(xl, dt).unsqueeze(1).expand(Bp, R, 5).reshape(Bp * R, 5)
        hi_e = _t(xh, dt).unsqueeze(1).expand(Bp, R, 5).reshape(Bp * R, 5)
        x_init = lo_e + (hi_e - lo_e) * torch.rand(Bp * R, 5, dtype=dt)
        sat, wit = vh._simple_pgd_batched(_t(xl, dt), _t(xh, dt), spec, gg, 4,
                                          torch.device('cpu'), dt,
                                          n_restarts=R, n_iter=30, lr=0.1,
                                          seed=0)
        spec_results[f'{tag}_thr'] = np.array(thr)
        spec_results[f'{tag}_sat'] = np.array(bool(sat))
        spec_results[f'{tag}_witness'] = (np.zeros(5, np.float32) if wit is None
                                          else np.asarray(wit, np.float32))
        spec_results[f'{tag}_x_init'] = _n(x_init)
    _save('pgd', **_net_arrays(layers), xl=xl, xh=xh, R=np.array(R),
          n_iter=np.array(30), **spec_results)

    # --------------------------------------------------- full BaB driver cfg1
    for seed in (0, 1):
        w = wk.cfg1(seed)
        gg = wk.mlp_gg(w['layers'], 'cpu', torch.float32)
        spec = vspec.VNNSpec(
            x_lo=w['xl'].astype(np.float64), x_hi=w['xh'].astype(np.float64),
            disjuncts=[vspec.Conjunct([vspec.PairwiseConstraint(pred=1,
                                                                comp=0)])])
        res = {}
        for ci, crown_i in ((1, True), (0, False)):
            st = vs.default_settings(
                device='cpu', bits=32, input_split_batched_enabled=True,
                input_split_batch_size=2048, input_split_crown_intermediate=crown_i,
                disable_sat_finding=True, total_timeout=600.0)
            verdict, det = vg._input_split_batched(
                types.SimpleNamespace(onnx_path=None), spec, st, gg,
                torch.device('cpu'), torch.float32)
            res[f'verdict_ci{ci}'] = np.array(verdict)
            res[f'n_leaves_ci{ci}'] = np.array(det.get('batched_n_leaves', -1))
            res[f'n_iters_ci{ci}'] = np.array(det.get('batched_n_iters', -1))
            print('cfg1 seed', seed, 'crown_interm', crown_i, verdict, det)
        _save(f'bab_cfg1_seed{seed}', **_net_arrays(w['layers']), xl=w['xl'],
              xh=w['xh'], d=np.array(w['d']), **res)


# Cases of pgd_attack_general: (tag, net, case seed, threshold offsets q0, q3,
# settings).  q0 puts the 'Y0 >= thr' disjunct q0 sample-std above the
# sampled max of y0; q3 puts 'Y3 <= thr3' q3 std below the sampled min of y3.
PGD_GENERAL_CASES = (
    ('clip_osi_a', 'deep', 0, 0.1, 5.0, {}),
    ('clip_osi_b', 'deep', 1, 0.2, 5.0, {}),
    ('clip_osi_c', 'deep', 2, 0.4, 5.0, {}),
    ('clip_osi_unsat', 'deep', 3, 3.0, 5.0, {}),
    ('sign_sgd_uniform', 'deep', 4, 0.1, 0.1,
     {'pgd_optim': 'sign_sgd', 'pgd_init_mode': 'uniform'}),
    ('adam_sign_multi_prd', 'deep', 5, 0.1, 0.1,
     {'pgd_optim': 'adam_sign', 'pgd_init_mode': 'uniform', 'pgd_alpha_multi': True,
      'pgd_per_restart_disjunct': True}),
    ('restrict_disj1', 'deep', 6, 0.0, 0.05, {'restrict_disj': {1}}),
    ('plateau', 'deep', 7, 3.0, 5.0, {'pgd_plateau_iters': 6, 'no_pair': True}),
    ('small_osi10', 'small', 8, 0.05, 5.0, {'pgd_osi_iters': 10, 'pgd_iter': 30,
                                            'pgd_restarts': 16}),
    ('small_unsat', 'small', 9, 2.0, 5.0, {'pgd_osi_iters': 10, 'pgd_iter': 30,
                                           'pgd_restarts': 16}),
)


def _golden_pgd_general(vspec, wk):
    """pgd_attack_general (pgd.py:233-524) on two seeded MLPs: the restarts'
    initial draw, the OSI projections, the (sat, witness) result and the
    last iterate the reference screened (recorded by wrapping the traced
    forward, so UNSAT trajectories are pinned too)."""
    import torch
    import vibecheck.pgd as vp
    nets = {'deep': wk.mlp_params(wk.ACAS_DIMS, np.random.default_rng(5)),
            'small': wk.mlp_params((5, 20, 20, 4), np.random.default_rng(2))}
    out = {}
    for name, layers in nets.items():
        for k, v in _net_arrays(layers).items():
            out[f'{name}_{k}'] = v
    orig = vp._get_traced_forward
    for tag, net, cs, q0, q3, extra in PGD_GENERAL_CASES:
        layers = nets[net]
        gg = wk.mlp_gg(layers, 'cpu', torch.float32)
        n_in, n_out = layers[0][0].shape[1], layers[-1][0].shape[0]
        rng = np.random.default_rng(1000 + cs)
        c = rng.uniform(-0.5, 0.5, n_in)
        h = rng.uniform(0.05, 0.3, n_in)
        xl = (c - h).astype(np.float32)
        xh = (c + h).astype(np.float32)
        pts = xl + (xh - xl) * rng.random((4096, n_in))
        ys = wk._mlp_forward64(layers, pts)
        thr = float(ys[:, 0].max() + q0 * ys[:, 0].std())
        thr3 = float(ys[:, 3].min() - q3 * ys[:, 3].std())
        second = [vspec.Constraint(3, '<=', thr3)]
        if not extra.get('no_pair'):
            second.insert(0, vspec.PairwiseConstraint(1, 2))
        spec = vspec.VNNSpec(
            x_lo=xl.astype(np.float64), x_hi=xh.astype(np.float64),
            disjuncts=[vspec.Conjunct([vspec.Constraint(0, '>=', thr)]),
                       vspec.Conjunct(second)])
        st = dict(pgd_restarts=30, pgd_iter=100, pgd_optim='adam_clipping',
                  pgd_init_mode='osi', pgd_osi_iters=50, pgd_plateau_iters=100)
        st.update({k: v for k, v in extra.items() if k not in ('restrict_disj', 'no_pair')})
        restrict = extra.get('restrict_disj')
        R = st['pgd_restarts']
        xlt, xht = torch.tensor(xl), torch.tensor(xh)
        torch.manual_seed(cs)
        x_init = xlt + (xht - xlt) * torch.rand(R, n_in)
        w_d = (torch.rand(R, n_out) - 0.5) * 2.0
        seen = []

        def wrapped(gg_, sample, _seen=seen):
            fn = orig(gg_, sample)

            def rec(x):
                if x.shape[0] == R:
                    _seen.append(x.detach().clone())
                return fn(x)
            return rec
        vp._get_traced_forward = wrapped
        try:
            sat, wit = vp.pgd_attack_general(xlt, xht, spec, gg, types.SimpleNamespace(**st),
                                             restrict_disj=restrict, seed=cs)
        finally:
            vp._get_traced_forward = orig
        n_osi = st['pgd_osi_iters'] if st['pgd_init_mode'] == 'osi' else 0
        print('pgd_general', tag, 'sat', sat, 'screens', len(seen) - n_osi)
        p = f'{tag}_'
        out[p + 'net'] = np.array(net)
        out[p + 'xl'] = xl
        out[p + 'xh'] = xh
        out[p + 'thr'] = np.array(thr)
        out[p + 'thr3'] = np.array(thr3)
        out[p + 'settings'] = np.array(repr(sorted(st.items())))
        out[p + 'no_pair'] = np.array(bool(extra.get('no_pair')))
        out[p + 'restrict'] = np.array(-1 if restrict is None else sorted(restrict)[0])
        out[p + 'x_init'] = _n(x_init)
        out[p + 'w_d'] = _n(w_d)
        out[p + 'sat'] = np.array(bool(sat))
        out[p + 'witness'] = (np.zeros(n_in, np.float32) if wit is None
                              else np.asarray(wit, np.float32))
        out[p + 'screens'] = np.array(len(seen) - n_osi)
        out[p + 'x_last'] = _n(seen[-1])
    out['tags'] = np.array([c[0] for c in PGD_GENERAL_CASES])
    _save('pgd_general', **out)


# ReLU-split BaB cases: (tag, seed, dims, eps, keyword settings)
RELU_BAB_CASES = (
    ('closed20', 0, (20, 32, 32, 32, 5), 0.005, {}),
    ('exhausted', 0, (20, 32, 32, 32, 5), 0.01, {}),
    ('closed229', 3, (12, 24, 24, 24, 4), 0.04, {}),
    ('capped', 2, (10, 40, 40, 5), 0.05, {'max_domains': 400}),
    ('deepest', 3, (12, 24, 24, 24, 4), 0.04, {'split_deepest': True}),
    ('noreforward', 3, (12, 24, 24, 24, 4), 0.04, {'no_reforward': True}),
    ('warm', 3, (12, 24, 24, 24, 4), 0.04, {'alpha_half': True, 'ew_ones': True}),
    ('warm_noref', 3, (12, 24, 24, 24, 4), 0.04,
     {'alpha_half': True, 'ew_ones': True, 'no_reforward': True}),
    # cfg3's input and layer widths (784 -> 256 ...), depth and radius chosen
    # so that the run closes after tens to hundreds of domains
    ('wide2', 0, (784, 256, 256, 10), 0.001, {}),
    ('wide3', 0, (784, 256, 256, 256, 10), 0.0002, {}),
    ('wide4', 0, (784, 256, 256, 256, 256, 10), 0.000035, {}),
)


def relu_bab_kwargs(kw, root):
    """Keyword arguments of a case: 'alpha_half' becomes alpha_init = 0.5
    at every ReLU, 'ew_ones' a unit coefficient score ew_w at every ReLU."""
    import torch
    out = dict(time_left=lambda: 1e9, batch=16, alpha_iters=8, max_domains=3000)
    for k, v in kw.items():
        if k == 'alpha_half':
            out['alpha_init'] = {L: torch.full_like(lo, 0.5) for L, (lo, _) in root.items()}
        elif k == 'ew_ones':
            out['ew_w'] = {L: torch.ones_like(lo) for L, (lo, _) in root.items()}
        else:
            out[k] = v
    return out


def relu_bab_problem(seed, dims, eps):
    """Network, box and margin query (y_top - y_second > 0 at the centre) of
    a ReLU-split BaB case."""
    from vibecheck_nn_b200 import workloads as wk
    rng = np.random.default_rng(seed)
    layers = wk.mlp_params(dims, rng)
    x0 = rng.uniform(0, 1, dims[0])
    y = wk._mlp_forward64(layers, x0[None])[0]
    t, j = int(np.argmax(y)), int(np.argsort(y)[-2])
    w = np.zeros(dims[-1])
    w[t], w[j] = 1.0, -1.0
    return layers, (x0 - eps).astype(np.float32), (x0 + eps).astype(np.float32), w


def _golden_relu_bab(vz, wk):
    """_ibp_crown_bab (verify_milp.py:2658-2960) in float32 on CPU: closed
    flag, domain count and reason per case (batch 16, 8 alpha-beta Adam
    iterations)."""
    import torch
    import vibecheck.verify_milp as vm
    out = {}
    for tag, seed, dims, eps, kw in RELU_BAB_CASES:
        layers, xl, xh, w = relu_bab_problem(seed, dims, eps)
        dt = torch.float32
        gg = wk.mlp_gg(layers, 'cpu', dt)
        xlt, xht = torch.as_tensor(xl), torch.as_tensor(xh)
        sb = vz._ibp_forward_graph_batched(xlt[None], xht[None], gg, 'cpu', dt)
        root = {L: (lo[0], hi[0]) for L, (lo, hi) in sb.items()}
        closed, n, reason = vm._ibp_crown_bab(gg, xlt, xht, root, w, 0.0, 'cpu', dt,
                                              **relu_bab_kwargs(kw, root))
        print('relu_bab', tag, closed, n, reason)
        out[f'{tag}_closed'] = np.array(bool(closed))
        out[f'{tag}_n'] = np.array(int(n))
        out[f'{tag}_reason'] = np.array(reason)
    out['tags'] = np.array([c[0] for c in RELU_BAB_CASES])
    _save('relu_bab', **out)


# freeze-replay hybrid cases: (tag, cfg1 seed, offset added to the property
# threshold d, settings)
HYBRID_CASES = (
    ('unsat0', 0, 0.0, {}),
    ('unsat1', 1, 0.0, {}),
    ('unsat0_short', 0, 0.0, {'hybrid_freeze_iters': 20, 'hybrid_pgd_between_every': 3}),
    ('sat0', 0, -2.0, {}),
)


def hybrid_problem(seed, offset):
    """cfg1 network with the property y0 - y1 <= d + offset folded into the
    last bias (unsafe iff Y1' >= Y0' after the fold)."""
    from vibecheck_nn_b200 import workloads as wk
    w = wk.cfg1(seed)
    layers = [(np.array(W), np.array(b)) for W, b in w['layers']]
    layers[-1][1][0] -= np.float32(offset) if offset else 0
    return layers, w['xl'], w['xh']


def _golden_hybrid(wk):
    """verify_hybrid (verify_hybrid_acasxu.py:321-539) on CPU in float32:
    verdict, phase and the BaB counters per case."""
    import types as _types
    import torch
    import vibecheck.spec as vspec
    import vibecheck.verify_hybrid_acasxu as vhy
    out = {}
    for tag, seed, offset, st in HYBRID_CASES:
        layers, xl, xh = hybrid_problem(seed, offset)
        gg = wk.mlp_gg(layers, 'cpu', torch.float32)
        graph = _types.SimpleNamespace(gpu_graph=lambda device, dtype, gg=gg: gg)
        spec = vspec.VNNSpec(x_lo=np.asarray(xl, np.float64), x_hi=np.asarray(xh, np.float64),
                             disjuncts=[vspec.Conjunct([vspec.PairwiseConstraint(pred=1,
                                                                                 comp=0)])])
        settings = _types.SimpleNamespace(**st)
        res = vhy.verify_hybrid(graph, spec, settings, timeout=1e6)
        print('hybrid', tag, {k: v for k, v in res.items() if k != 'witness'})
        out[f'{tag}_verdict'] = np.array(res['verdict'])
        out[f'{tag}_phase'] = np.array(res.get('phase', ''))
        for k in ('evaluated', 'closed', 'bab_iters'):
            out[f'{tag}_{k}'] = np.array(int(res.get(k, -1)))
    out['tags'] = np.array([c[0] for c in HYBRID_CASES])
    _save('hybrid', **out)


# multi-subbox BaB cases: (tag, net seed, sub-boxes, margins (lo, hi),
# half-widths of the varying dimensions (lo, hi), batch, split depth, budget);
# 'unsafe' has one sub-box whose property fails (only its closed set is
# deterministic: the loop runs until the budget)
MULTISUB_CASES = (
    ('mixed', 5, 16, (0.01, 0.05), (0.1, 0.3), 1024, 4, 1e6),
    ('small_batch', 6, 12, (0.005, 0.03), (0.1, 0.3), 64, 2, 1e6),
    ('wide', 7, 16, (0.01, 0.1), (0.3, 0.5), 1024, 4, 1e6),
    ('unsafe', 5, 1, (-0.3, -0.3), (0.1, 0.3), 1024, 4, 3.0),
)


def multisub_problem(seed, n_sub, margins, half=(0.1, 0.3)):
    """A 6 -> [24] x 3 -> 2 MLP and sub-boxes whose dimensions 0-3 are fixed
    and 4-5 vary.  Sub-box k is unsafe iff y0 >= t0_k and y1 <= t1_k, with
    t0_k = max y0 + m_k and t1_k = min y1 - m_k over samples (the property
    holds when m_k > 0 and the sampled extremes are the true ones).  Returns
    (layers, [(x_lo, x_hi, [[('ge', 0, t0), ('le', 1, t1)]])])."""
    from vibecheck_nn_b200 import workloads as wk
    rng = np.random.default_rng(seed)
    layers = wk.mlp_params((6, 24, 24, 24, 2), rng)
    subs = []
    for k in range(n_sub):
        fixed = rng.uniform(0, 1, 4)
        c = rng.uniform(0.2, 0.8, 2)
        h = rng.uniform(half[0], half[1], 2)
        lo = np.concatenate([fixed, c - h]).astype(np.float32)
        hi = np.concatenate([fixed, c + h]).astype(np.float32)
        pts = lo + (hi - lo) * rng.random((4096, 6))
        y = wk._mlp_forward64(layers, pts.astype(np.float64))
        m = margins[0] + (margins[1] - margins[0]) * (k / max(1, n_sub - 1))
        t0 = float(y[:, 0].max() + m)
        t1 = float(y[:, 1].min() - m)
        subs.append((lo, hi, [[('ge', 0, t0), ('le', 1, t1)]]))
    return layers, subs


def _golden_acasxu(ref_src, vg, vs):
    """The reference's bundled ACAS Xu example (README.md:40-75): the
    network as this package's ONNX reader lowers it (weights and biases of
    the fc layers), and for examples/prop_1 and prop_2 the property as the
    reference's vnnlib_loader parses it (box, linear queries) and the
    reference driver's verdict, leaves, iterations, phase and witness under
    configs/acasxu_2023.yaml (_input_split_batched on CPU in float32, 60 s)."""
    import types as _types
    import torch
    import vibecheck.config_loader as cl
    import vibecheck.vnnlib_loader as vl
    from vibecheck_nn_b200 import netdesc, onnx_graph
    root = os.path.dirname(os.path.abspath(ref_src))
    g = onnx_graph.read_onnx(os.path.join(root, 'examples', 'ACASXU_run2a_2_2_batch_2000.onnx'))
    gg = g.to_gg('cpu', torch.float32)
    layers = netdesc.lower_mlp(gg)
    out = _net_arrays(layers)
    out['op_types'] = np.array(' '.join(op['type'] for op in gg['ops']))
    over = cl.load_config(os.path.join(root, 'configs', 'acasxu_2023.yaml'))
    for prop in (1, 2):
        spec = vl.load_vnnlib(os.path.join(root, 'examples', f'prop_{prop}.vnnlib'))
        st = vs.default_settings(device='cpu', bits=32, total_timeout=60.0, **over)
        verdict, det = vg._input_split_batched(_types.SimpleNamespace(onnx_path=None), spec, st,
                                               gg, torch.device('cpu'), torch.float32)
        print('acasxu prop', prop, verdict, {k: v for k, v in det.items() if k != 'witness'},
              flush=True)
        q = spec.as_linear_queries(5)
        p = f'p{prop}_'
        from vibecheck_nn_b200.pgd import _disjunct_tuples
        out[p + 'disj'] = np.array(repr(_disjunct_tuples(spec)))
        out[p + 'x_lo'] = np.asarray(spec.x_lo, np.float64).reshape(-1)
        out[p + 'x_hi'] = np.asarray(spec.x_hi, np.float64).reshape(-1)
        out[p + 'qd'] = np.array([d for d, _, _ in q])
        out[p + 'qw'] = np.stack([np.asarray(w, np.float64).reshape(-1) for _, w, _ in q])
        out[p + 'qb'] = np.array([float(b) for _, _, b in q])
        out[p + 'verdict'] = np.array(verdict)
        out[p + 'phase'] = np.array(det.get('phase', ''))
        out[p + 'n_leaves'] = np.array(det.get('batched_n_leaves', -1))
        out[p + 'n_iters'] = np.array(det.get('batched_n_iters', -1))
        if det.get('witness') is not None:
            out[p + 'witness'] = np.asarray(det['witness'], np.float64).reshape(-1)
    _save('acasxu', **out)


# Branching variants of the input-split BaB driver on cfg1 networks: (tag,
# seed, settings overrides).  'sb' scores width x sum_q |A_q| (verify_graph.py:
# 13285-13286), 'margin' the margin-augmented worst-query score (:13275-13283),
# 'clip3' iterates the halfspace clip (:13036-13084), 'depth2' / 'depth3'
# split 2^K ways while the popped batch is below the batch size, with the
# branch boost (:12744-12800, :13320-13423).
BAB_BRANCHING_CASES = (
    ('sb', 0, {'input_split_batched_branch_sb': True}),
    ('margin', 0, {'input_split_batched_branch_sb': True, 'input_split_sb_margin_score': True}),
    ('margin_thr', 1, {'input_split_batched_branch_sb': True, 'input_split_sb_margin_score': True,
                       'input_split_sb_coeff_thresh': 0.5, 'input_split_sb_margin_weight': 0.25}),
    ('clip3', 0, {'input_split_batched_clip_iters': 3}),
    ('clip3_s1', 1, {'input_split_batched_clip_iters': 3}),
    ('depth2', 0, {'input_split_batched_branch_sb': True, 'bab_split_depth': 2}),
    ('depth3_noboost', 1, {'input_split_batched_branch_sb': True, 'bab_split_depth': 3,
                           'input_split_batched_branch_boost': False}),
    ('depth2_b64', 0, {'input_split_batched_branch_sb': True, 'bab_split_depth': 2,
                       'input_split_batch_size': 64}),
    ('depth2_margin_exp2', 1, {'input_split_batched_branch_sb': True, 'bab_split_depth': 2,
                               'input_split_sb_margin_score': True,
                               'input_split_batched_branch_boost_exp': 2.0}),
)


def _golden_bab_branching(vg, vs, vspec, wk):
    """_input_split_batched (verify_graph.py:12466) on cfg1 networks with
    CROWN intermediates under each BAB_BRANCHING_CASES setting, on CPU in
    float32: verdict, visited leaves, iterations and open degenerate leaves."""
    import types as _types
    import torch
    out = {}
    for tag, seed, over in BAB_BRANCHING_CASES:
        w = wk.cfg1(seed)
        gg = wk.mlp_gg(w['layers'], 'cpu', torch.float32)
        spec = vspec.VNNSpec(
            x_lo=w['xl'].astype(np.float64), x_hi=w['xh'].astype(np.float64),
            disjuncts=[vspec.Conjunct([vspec.PairwiseConstraint(pred=1, comp=0)])])
        kw = dict(device='cpu', bits=32, input_split_batched_enabled=True,
                  input_split_batch_size=2048, input_split_crown_intermediate=True,
                  disable_sat_finding=True, total_timeout=600.0)
        kw.update(over)
        st = vs.default_settings(**kw)
        verdict, det = vg._input_split_batched(_types.SimpleNamespace(onnx_path=None), spec,
                                               st, gg, torch.device('cpu'), torch.float32)
        print('bab branching', tag, verdict, det, flush=True)
        out[f'{tag}_verdict'] = np.array(verdict)
        out[f'{tag}_n_leaves'] = np.array(det.get('batched_n_leaves', -1))
        out[f'{tag}_n_iters'] = np.array(det.get('batched_n_iters', -1))
        out[f'{tag}_open'] = np.array(det.get('batched_open_degenerate', 0))
    _save('bab_branching', **out)


# cfg2 benchmark workloads whose tensor-core IBP bounds put a ReLU at the
# min-area tie, and one box of each that sits there
CFG2_SEEDS = (0, 1, 3)
CFG2_TIE_BOXES = (53604, 60678, 53706)
CFG2_LB_BOXES = 4096


def ibp_digest(arrays):
    """SHA-256 of a list of float32 arrays' bytes (bit-exact equality of
    65,536-box IBP bounds without committing them)."""
    import hashlib
    h = hashlib.sha256()
    for a in arrays:
        h.update(np.ascontiguousarray(a, np.float32).tobytes())
    return h.hexdigest()


def _golden_cfg2(vz, wk):
    """The reference's own float32 IBP forward + CROWN back-substitution
    (_ibp_forward_graph_batched, verify_zono_bnb.py:1066, then
    _spec_backward_graph_batched, :4270) on the full 65,536-box cfg2
    workload, on CPU: a digest of every layer's IBP bounds and the lower
    bounds of the first CFG2_LB_BOXES boxes plus the tie box."""
    import torch
    out = {}
    for seed, tie in zip(CFG2_SEEDS, CFG2_TIE_BOXES):
        w = wk.cfg2(seed=seed)
        gg = wk.mlp_gg(w['layers'])
        xl, xh = _t(w['xl'], torch.float32), _t(w['xh'], torch.float32)
        spec_ew = wk.spec_ew_from(w['spec_W'], w['spec_b'], 'cpu')
        sb = vz._ibp_forward_graph_batched(xl, xh, gg, 'cpu', torch.float32)
        lb = _n(vz._spec_backward_graph_batched(sb, xl, xh, gg, spec_ew, 'cpu',
                                                torch.float32))
        keys = sorted(sb)
        out[f's{seed}_ibp_digest'] = np.array(
            ibp_digest([_n(sb[L][k]) for L in keys for k in (0, 1)]))
        idx = np.concatenate([np.arange(CFG2_LB_BOXES), [tie]])
        out[f's{seed}_idx'] = idx
        out[f's{seed}_lb'] = lb[idx]
    _save('cfg2_ref', **out)


def _golden_multisub(wk):
    """_multi_sub_input_split_bab (verify_graph.py:11180) on CPU in float32:
    closed sub-boxes, iterations and visited leaves per case."""
    import contextlib
    import io
    import re
    import types as _types
    import torch
    import vibecheck.spec as vspec
    import vibecheck.verify_graph as vg
    out = {}
    for tag, seed, n_sub, margins, half, batch, depth, budget in MULTISUB_CASES:
        layers, subs = multisub_problem(seed, n_sub, margins, half)
        gg = wk.mlp_gg(layers, 'cpu', torch.float32)
        groups = []
        for lo, hi, conj in subs:
            cons = [vspec.Constraint(i, '>=' if op == 'ge' else '<=', v) for op, i, v in conj[0]]
            groups.append((lo.astype(np.float64), hi.astype(np.float64), [vspec.Conjunct(cons)]))
        order = list(range(len(groups)))
        st = _types.SimpleNamespace(input_split_batch_size=batch, bab_split_depth=depth,
                                    print_progress=True)
        buf = io.StringIO()
        with contextlib.redirect_stdout(buf):
            closed = vg._multi_sub_input_split_bab(list(range(len(groups))), groups, order, gg,
                                                   torch.device('cpu'), torch.float32, budget,
                                                   2, st)
        mt = re.search(r'(\d+) iters, (\d+) leaves', buf.getvalue())
        print('multisub', tag, sorted(closed), mt.group(0) if mt else buf.getvalue()[-200:])
        out[f'{tag}_closed'] = np.array(sorted(closed), np.int64)
        out[f'{tag}_iters'] = np.array(int(mt.group(1)) if mt else -1)
        out[f'{tag}_leaves'] = np.array(int(mt.group(2)) if mt else -1)
    # forward linear bounds of the first net on its sub-boxes (varying dims 4, 5)
    import vibecheck.forward_lirpa as fl
    layers, subs = multisub_problem(*MULTISUB_CASES[0][1:5])
    gg = wk.mlp_gg(layers, 'cpu', torch.float32)
    xl = torch.as_tensor(np.stack([sb[0] for sb in subs]))
    xh = torch.as_tensor(np.stack([sb[1] for sb in subs]))
    bb = fl.chunked_batched_forward_linear_bounds(gg, xl, xh, torch.device('cpu'), torch.float32)
    for k in ('A_lo', 'A_up', 'b_lo', 'b_up', 'lo_box', 'hi_box'):
        out[f'flirpa_{k}'] = getattr(bb, k).numpy()
    out['flirpa_mask'] = fl.chunked_batched_forward_linear_bounds.last_varying_mask.numpy()
    out['tags'] = np.array([c[0] for c in MULTISUB_CASES])
    _save('multisub', **out)


def forward_cnn_gg(k1, b1, cb, W2, b2, W3, b3, fb, ins, dt):
    """CNN of the concrete-forward fixture: conv -> add (per-channel bias)
    -> relu -> flatten -> fc -> relu -> fc -> sub (elementwise bias)."""
    import torch
    g = _small_cnn_gg(k1, b1, W2, b2, W3, b3, ins, dt)
    ops = g['ops']
    conv = ops[0]
    add = {'name': 'cadd', 'type': 'add', 'inputs': ['conv0'],
           'bias': torch.as_tensor(cb, dtype=dt), 'out_shape_nd': conv['out_shape']}
    ops[1]['inputs'] = ['cadd']
    sub = {'name': 'fsub', 'type': 'sub', 'inputs': ['fc1'],
           'bias': torch.as_tensor(fb, dtype=dt), 'out_shape_nd': (fb.size,)}
    g['ops'] = [conv, add] + ops[1:] + [sub]
    return g


def _golden_forward(vz, wk):
    """_forward_batch_graph (verify_zono_bnb.py:554) on a CNN with bias ops and
    on an ACAS-sized MLP: outputs, two captures and the autograd gradient of
    g . f(x)."""
    import torch
    dt = torch.float32
    rng = np.random.default_rng(41)
    ins = (3, 12, 12)
    k1 = (rng.standard_normal((8, 3, 4, 4)) * 0.3).astype(np.float32)
    b1 = (rng.standard_normal(8) * 0.05).astype(np.float32)
    cb = (rng.standard_normal((8, 1, 1)) * 0.05).astype(np.float32)
    W2 = (rng.standard_normal((20, 8 * 6 * 6)) * 0.08).astype(np.float32)
    b2 = (rng.standard_normal(20) * 0.05).astype(np.float32)
    W3 = (rng.standard_normal((5, 20)) * 0.3).astype(np.float32)
    b3 = (rng.standard_normal(5) * 0.05).astype(np.float32)
    fb = (rng.standard_normal(5) * 0.05).astype(np.float32)
    gg = forward_cnn_gg(k1, b1, cb, W2, b2, W3, b3, fb, ins, dt)
    N = 19
    x = rng.uniform(0, 1, (N, int(np.prod(ins)))).astype(np.float32)
    gw = rng.standard_normal((N, 5)).astype(np.float32)
    xt = torch.as_tensor(x).requires_grad_(True)
    out = vz._forward_batch_graph(xt, gg)
    (out * torch.as_tensor(gw)).sum().backward()
    with torch.no_grad():
        cap_relu = vz._forward_batch_graph(torch.as_tensor(x), gg, capture='relu0')
        cap_fc = vz._forward_batch_graph(torch.as_tensor(x), gg, capture='fc0')
    res = dict(k1=k1, b1=b1, cb=cb, W2=W2, b2=b2, W3=W3, b3=b3, fb=fb, x=x, gw=gw,
               out=_n(out), grad=_n(xt.grad), cap_relu0=_n(cap_relu), cap_fc0=_n(cap_fc))
    layers = wk.mlp_params(wk.ACAS_DIMS, np.random.default_rng(43))
    ggm = wk.mlp_gg(layers, 'cpu', dt)
    xm = rng.uniform(-1, 1, (N, 5)).astype(np.float32)
    gm = rng.standard_normal((N, 5)).astype(np.float32)
    xmt = torch.as_tensor(xm).requires_grad_(True)
    outm = vz._forward_batch_graph(xmt, ggm)
    (outm * torch.as_tensor(gm)).sum().backward()
    res.update(mlp_x=xm, mlp_gw=gm, mlp_out=_n(outm), mlp_grad=_n(xmt.grad),
               **{f'mlp_{k}': v for k, v in _net_arrays(layers).items()})
    _save('forward', **res)


def _small_cnn_gg(k1, b1, W2, b2, W3, b3, ins, dt):
    import torch
    from vibecheck_nn_b200 import workloads as wk
    stride, pad = (2, 2), (1, 1)
    Ho, Wo = wk.conv_out_hw(ins[1], ins[2], k1.shape[2:], stride, pad)
    out_shape = (k1.shape[0], Ho, Wo)
    oph = ins[1] - ((Ho - 1) * stride[0] - 2 * pad[0] + k1.shape[2])
    opw = ins[2] - ((Wo - 1) * stride[1] - 2 * pad[1] + k1.shape[3])
    ops = [
        {'name': 'conv0', 'type': 'conv', 'inputs': ['x'],
         'kernel': torch.as_tensor(k1, dtype=dt),
         'bias': torch.as_tensor(b1, dtype=dt),
         'kernel_np': k1.astype(np.float64), 'bias_np': b1.astype(np.float64),
         'in_shape': ins, 'out_shape': out_shape, 'stride': stride,
         'padding': pad, 'output_padding': (oph, opw),
         'n_out': int(np.prod(out_shape))},
        {'name': 'relu0', 'type': 'relu', 'inputs': ['conv0'], 'layer_idx': 0},
        {'name': 'flat', 'type': 'reshape', 'inputs': ['relu0']},
        {'name': 'fc0', 'type': 'fc', 'inputs': ['flat'],
         'W': torch.as_tensor(W2, dtype=dt), 'bias': torch.as_tensor(b2, dtype=dt),
         'W_np': W2.astype(np.float64), 'bias_np': b2.astype(np.float64)},
        {'name': 'relu1', 'type': 'relu', 'inputs': ['fc0'], 'layer_idx': 1},
        {'name': 'fc1', 'type': 'fc', 'inputs': ['relu1'],
         'W': torch.as_tensor(W3, dtype=dt), 'bias': torch.as_tensor(b3, dtype=dt),
         'W_np': W3.astype(np.float64), 'bias_np': b3.astype(np.float64)},
    ]
    return {'ops': ops, 'relu_names': ['relu0', 'relu1'], 'fork_points': set(),
            'n_relu': 2, 'input_name': 'x', 'input_n': int(np.prod(ins)),
            'input_shape': (1,) + tuple(ins)}


if __name__ == '__main__':
    main()
