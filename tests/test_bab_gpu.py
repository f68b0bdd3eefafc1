"""GPU parity of the zonotope forward, CROWN intermediates and the input-split
BaB driver against the reference's golden vectors and the numpy oracle."""
import numpy as np
import pytest
import torch

from conftest import close, golden_layers, load_golden, max_excess
from oracle import bab as obab
from oracle import bounds as ob
from vibecheck_nn_b200 import bab, interm, ops, workloads as wk

pytestmark = pytest.mark.gpu
DEV = torch.device('cuda:0') if torch.cuda.is_available() else None


def T(a):
    return torch.as_tensor(np.asarray(a), device=DEV)


def N(t):
    return t.detach().cpu().numpy()


def gram(G):
    """Column-order-free fingerprint of a generator matrix: G G^T per box."""
    G = np.asarray(G, np.float64)
    return np.einsum('bik,bjk->bij', G, G)


@pytest.mark.parametrize('tag', ['small', 'acas'])
def test_zonotope_golden(tag):
    g = load_golden(f'mlp_{tag}')
    gg = wk.mlp_gg(golden_layers(g), DEV)
    sb, (c, G) = interm._forward_zonotope_graph_batched(T(g['xl']), T(g['xh']), gg,
                                                       DEV, torch.float32)
    for L, (lo, hi) in sb.items():
        assert close(N(lo), g[f'zono32_lo{L}']), (L, max_excess(N(lo), g[f'zono32_lo{L}']))
        assert close(N(hi), g[f'zono32_hi{L}'])
    assert close(N(c), g['zono32_c'])
    ref = gram(g['zono32_G'])
    got = gram(N(G))
    assert np.allclose(got, ref, rtol=1e-4, atol=1e-4 * np.abs(ref).max())


def test_zonotope_zero_radius_golden():
    g = load_golden('zono_zero_radius')
    gg = wk.mlp_gg(golden_layers(g), DEV)
    sb, (c, G) = interm._forward_zonotope_graph_batched(T(g['xl']), T(g['xh']), gg,
                                                       DEV, torch.float32)
    assert close(N(sb[0][0]), g['lo0']) and close(N(sb[0][1]), g['hi0'])
    assert close(N(c), g['c'])
    assert np.allclose(gram(N(G)), gram(g['G']), rtol=1e-5, atol=1e-6)


@pytest.mark.parametrize('tag', ['small', 'acas'])
def test_crown_intermediate_golden(tag):
    g = load_golden(f'mlp_{tag}')
    gg = wk.mlp_gg(golden_layers(g), DEV)
    tight = interm._crown_intermediate_batched(gg, T(g['xl']), T(g['xh']), DEV,
                                               torch.float32)
    for L, (lo, hi) in tight.items():
        assert close(N(lo), g[f'interm32_lo{L}']), (L, max_excess(N(lo), g[f'interm32_lo{L}']))
        assert close(N(hi), g[f'interm32_hi{L}']), (L, max_excess(N(hi), g[f'interm32_hi{L}']))
    spec_ew = wk.spec_ew_from(g['spec_W'], g['spec_b'], DEV)
    lb, A, acc = ops._spec_backward_graph_batched(
        tight, T(g['xl']), T(g['xh']), gg, spec_ew, DEV, torch.float32,
        return_input_linear=True)
    assert close(N(lb), g['spec_interm32_lb'])
    assert close(N(A), g['spec_interm32_A']) and close(N(acc), g['spec_interm32_acc'])


def test_seeded_spec_backward_matches_oracle():
    w = wk.cfg2(seed=5, n_boxes=12)
    gg = wk.mlp_gg(w['layers'], DEV)
    ggc = wk.mlp_gg(w['layers'])
    sb = ob.forward_zonotope_batched(w['xl'], w['xh'], ggc)[0]
    n = 50
    seed = np.concatenate([np.eye(n), -np.eye(n)]).astype(np.float32)
    seed_b = np.broadcast_to(seed, (12, 2 * n, n))
    ref = ob.spec_backward_batched(sb, w['xl'], w['xh'], ggc, seed_ew_at={'fc2': seed_b},
                                   seed_acc=np.zeros((12, 2 * n), np.float32))
    tight = {L: (T(v[0]), T(v[1])) for L, v in sb.items()}
    got = ops._spec_backward_graph_batched(
        tight, T(w['xl']), T(w['xh']), gg, None, DEV, torch.float32,
        seed_ew_at={'fc2': T(seed).unsqueeze(0).expand(12, -1, -1)},
        seed_acc=torch.zeros(12, 2 * n, device=DEV))
    assert close(N(got), ref), max_excess(N(got), ref)


def test_bab_step_matches_oracle():
    rng = np.random.default_rng(3)
    B, Q, n = 700, 3, 5
    xl = rng.uniform(-1, 0, (B, n)).astype(np.float32)
    xh = (xl + rng.uniform(0.0, 1, (B, n))).astype(np.float32)
    xh[:5, 2] = xl[:5, 2]          # zero-width dims
    xh[5, :] = xl[5, :] + 1e-13    # degenerate leaf
    A = rng.normal(size=(B, Q, n)).astype(np.float32)
    acc = rng.normal(size=(B, Q)).astype(np.float32)
    lb = rng.normal(size=(B, Q)).astype(np.float32)
    qd = torch.zeros(Q, dtype=torch.int32, device=DEV)
    for sb_ in (False, True):
        lo_xl, lo_xh, hi_xl, hi_xh, cnt = bab.bab_step(
            T(xl), T(xh), T(lb), T(A), T(acc), qd, 1, True, sb_)
        closed = (lb > 0).any(axis=1)
        un = np.nonzero(~closed)[0]
        xl_c, xh_c, feas = ob.clip_box_by_halfspaces_batched(xl[un], xh[un], A[un], acc[un])
        f = np.nonzero(feas)[0]
        xs_l, xs_h = xl_c[f], xh_c[f]
        widths = xs_h - xs_l
        if sb_:
            score = widths * np.abs(A[un][f]).sum(axis=1)
        else:
            score = widths
        ax = score.argmax(axis=1)
        rows = np.arange(len(f))
        usable = (xs_h[rows, ax] - xs_l[rows, ax]) > np.float32(1e-12)
        c = N(cnt)
        assert c[0] == closed.sum() and c[1] == (~feas).sum()
        assert c[2] == usable.sum() and c[3] == (~usable).sum()
        u = np.nonzero(usable)[0]
        mid = ((xs_l[u, ax[u]] + xs_h[u, ax[u]]) * np.float32(0.5)).astype(np.float32)
        exp_lo_xh = xs_h[u].copy()
        exp_lo_xh[np.arange(len(u)), ax[u]] = mid
        exp_hi_xl = xs_l[u].copy()
        exp_hi_xl[np.arange(len(u)), ax[u]] = mid
        k = int(c[2])
        assert close(N(lo_xl)[:k], xs_l[u]) and close(N(lo_xh)[:k], exp_lo_xh)
        assert close(N(hi_xl)[:k], exp_hi_xl) and close(N(hi_xh)[:k], xs_h[u])


@pytest.mark.parametrize('seed', [0, 1])
@pytest.mark.parametrize('ci', [1, 0])
def test_bab_cfg1_matches_reference_leaf_counts(seed, ci):
    g = load_golden(f'bab_cfg1_seed{seed}')
    gg = wk.mlp_gg(golden_layers(g), DEV)
    spec = bab.LinearSpec(g['xl'], g['xh'], [[('pair', 1, 0)]])
    st = wk.reference_bab_settings(input_split_batch_size=2048,
                                   input_split_crown_intermediate=bool(ci),
                                   disable_sat_finding=True, total_timeout=600.0)
    verdict, det = bab._input_split_batched(None, spec, st, gg, DEV, torch.float32)
    assert verdict == str(g[f'verdict_ci{ci}'])
    assert det['batched_n_leaves'] == int(g[f'n_leaves_ci{ci}']), det
    assert det['batched_n_iters'] == int(g[f'n_iters_ci{ci}']), det


def test_bab_multi_disjunct_matches_oracle():
    """Two disjuncts (per-disjunct clip + union) against the numpy driver."""
    w = wk.cfg1(2)
    gg = wk.mlp_gg(w['layers'], DEV)
    ggc = wk.mlp_gg(w['layers'])
    y = wk._mlp_forward64(w['layers'], ((w['xl'] + w['xh']) / 2)[None].astype(np.float64))[0]
    disj = [[('pair', 1, 0)], [('ge', 2, float(y[2]) + 60.0), ('le', 3, float(y[3]) - 60.0)]]
    spec = bab.LinearSpec(w['xl'], w['xh'], disj)
    st = wk.reference_bab_settings(input_split_batch_size=512, disable_sat_finding=True)
    verdict, det = bab._input_split_batched(None, spec, st, gg, DEV, torch.float32)
    queries = spec.as_linear_queries(5)
    W = np.stack([q[1] for q in queries]).astype(np.float32)
    b = np.array([q[2] for q in queries], np.float32)
    v2, d2 = obab.input_split_bab(ggc, w['xl'], w['xh'], W, b, disj_q=[[0], [1, 2]],
                                  batch_size=512, crown_intermediate=False,
                                  timeout=600)
    assert verdict == v2
    assert det['batched_n_leaves'] == d2['batched_n_leaves']
    assert det['batched_n_iters'] == d2['batched_n_iters']
