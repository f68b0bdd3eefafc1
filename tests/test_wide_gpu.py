"""GPU parity of the layer-wise (wide-network) IBP / CROWN / alpha-CROWN path."""
import numpy as np
import pytest
import torch

from conftest import close, golden_layers, load_golden, max_excess
from oracle import bounds as ob
from vibecheck_nn_b200 import wide, workloads as wk

pytestmark = pytest.mark.gpu
DEV = torch.device('cuda:0') if torch.cuda.is_available() else None


def T(a):
    return torch.as_tensor(np.asarray(a), device=DEV)


def N(t):
    return t.detach().cpu().numpy()


@pytest.mark.parametrize('tag', ['small', 'acas'])
def test_wide_ibp_crown_golden(tag):
    g = load_golden(f'mlp_{tag}')
    gg = wk.mlp_gg(golden_layers(g), DEV)
    wn = wide.wide_net(gg, DEV)
    sb = wide.wide_ibp(wn, T(g['xl']), T(g['xh']))
    for L, (lo, hi) in sb.items():
        assert close(N(lo), g[f'ibp32_lo{L}']) and close(N(hi), g[f'ibp32_hi{L}'])
    out = wide.wide_crown(wn, T(g['xl']), T(g['xh']), sb, T(g['spec_W']), T(g['spec_b']),
                          want_A=True)
    assert close(N(out['lb']), g['crown32_lb']), max_excess(N(out['lb']), g['crown32_lb'])
    assert close(N(out['A']), g['crown32_A']) and close(N(out['acc']), g['crown32_acc'])
    clamps = {0: (T(g['clamp_lo0']), T(g['clamp_hi0']))}
    sbc = wide.wide_ibp(wn, T(g['xl']), T(g['xh']), clamps)
    for L, (lo, hi) in sbc.items():
        assert close(N(lo), g[f'ibpc32_lo{L}']) and close(N(hi), g[f'ibpc32_hi{L}'])
    lbc = wide.wide_crown(wn, T(g['xl']), T(g['xh']), sbc, T(g['spec_W']), T(g['spec_b']))['lb']
    assert close(N(lbc), g['crownc32_lb'])


def test_wide_alpha_gradient_matches_oracle():
    """One adjoint evaluation against the oracle's hand-written adjoint, which
    is itself pinned to torch autograd through the reference (float64)."""
    rng = np.random.default_rng(21)
    dims = (40, 64, 64, 48, 7)
    layers = wk.mlp_params(dims, rng)
    D, Q = 37, 3
    x0 = rng.uniform(0, 1, (D, dims[0]))
    xl = (x0 - 0.05).astype(np.float32)
    xh = (x0 + 0.05).astype(np.float32)
    SW = rng.normal(size=(Q, dims[-1])).astype(np.float32)
    Sb = rng.normal(size=Q).astype(np.float32)
    ggc = wk.mlp_gg(layers)
    sb = ob.ibp_forward_batched(xl, xh, ggc)
    alpha = {}
    for L, (lo, hi) in sb.items():
        alpha[L] = rng.uniform(0, 1, lo.shape).astype(np.float32)
    lb_ref, grads = ob.alpha_grad(sb, xl, xh, ggc, SW, Sb, alpha)
    gg = wk.mlp_gg(layers, DEV)
    wn = wide.wide_net(gg, DEV)
    sbd = {L: (T(lo), T(hi)) for L, (lo, hi) in sb.items()}
    lb, contrib = wide.wide_alpha_grad(wn, T(xl), T(xh), sbd, T(SW), T(Sb),
                                       {L: T(a) for L, a in alpha.items()})
    assert close(N(lb), lb_ref), max_excess(N(lb), lb_ref)
    for L, g in grads.items():
        dc, ldo = contrib[L]
        got = N(dc)[:, :g.shape[1]].reshape(D, Q, -1).sum(axis=1)
        scale = np.abs(g).max() + 1e-12
        assert np.allclose(got, g, rtol=1e-4, atol=1e-5 * scale), (L, np.abs(got - g).max())


def test_alpha_domains_golden():
    """The cfg3-style alpha loop against the reference's recorded best lb
    (fp32 alpha trajectories agree to ~1e-3 relative; see the oracle tests)."""
    g = load_golden('alpha_domains')
    layers = golden_layers(g)
    gg = wk.mlp_gg(layers, DEV)
    clamps = {}
    for L in range(len(layers) - 1):
        if f'clamp_lo{L}' in g:
            clamps[L] = (g[f'clamp_lo{L}'], g[f'clamp_hi{L}'])
    best, _ = wide.alpha_crown_domains(g['xl'], g['xh'], gg, g['spec_W'], g['spec_b'],
                                       clamps, DEV, n_iters=int(g['n_iters']),
                                       lr=float(g['lr']))
    assert close(N(best), g['best_lb'], rtol=5e-3, atol=1e-5), max_excess(
        N(best), g['best_lb'], rtol=5e-3, atol=1e-5)


def test_cfg3_small_domains_against_oracle():
    """cfg3 network and domain construction at 64 domains x 4 iterations."""
    w = wk.cfg3(seed=0)
    ggc = wk.mlp_gg(w['layers'])
    root = ob.ibp_forward_batched(w['xl'][None], w['xh'][None], ggc)
    picked, clamps = wk.split_domains({L: v[0][0] for L, v in root.items()},
                                      {L: v[1][0] for L, v in root.items()}, 6)
    Dn = 1 << len(picked)
    xl = np.broadcast_to(w['xl'], (Dn, w['xl'].size)).copy()
    xh = np.broadcast_to(w['xh'], (Dn, w['xh'].size)).copy()
    ref, _ = ob.alpha_beta_crown_domains(xl, xh, ggc, w['spec_W'], w['spec_b'], clamps,
                                         n_iters=4, lr=0.1)
    gg = wk.mlp_gg(w['layers'], DEV)
    best, _ = wide.alpha_crown_domains(xl, xh, gg, w['spec_W'], w['spec_b'], clamps, DEV,
                                       n_iters=4, lr=0.1)
    assert close(N(best), ref, rtol=5e-3, atol=1e-4), max_excess(N(best), ref, rtol=5e-3,
                                                                 atol=1e-4)


@pytest.mark.parametrize('tag', ['small', 'acas'])
def test_alpha_inputsplit_golden(tag):
    """_run_alpha_crown_inputsplit_batched vs the reference's recorded lb
    (6 iterations, lr 0.25, decay 0.98; fp32 alpha trajectories agree to
    ~1e-3 relative)."""
    from vibecheck_nn_b200 import alpha
    g = load_golden(f'mlp_{tag}')
    gg = wk.mlp_gg(golden_layers(g), DEV)
    spec_ew = wk.spec_ew_from(g['spec_W'], g['spec_b'], DEV)
    lb = alpha._run_alpha_crown_inputsplit_batched(T(g['xl']), T(g['xh']), gg, spec_ew, DEV,
                                                   torch.float32, n_iters=6, lr=0.25,
                                                   lr_decay=0.98)
    assert close(N(lb), g['alpha32_lb'], rtol=5e-3, atol=1e-5), max_excess(
        N(lb), g['alpha32_lb'], rtol=5e-3, atol=1e-5)


def test_reference_style_autograd_loop():
    """The reference's own alpha loop (torch Adam, (-lb.sum()).backward())
    through ops._spec_backward_graph_batched, whose gradient is the
    hand-written adjoint, reproduces the recorded best lb."""
    from vibecheck_nn_b200 import ops
    g = load_golden('alpha_domains')
    layers = golden_layers(g)
    gg = wk.mlp_gg(layers, DEV)
    clamps = {}
    for L in range(len(layers) - 1):
        if f'clamp_lo{L}' in g:
            clamps[L] = (T(g[f'clamp_lo{L}']), T(g[f'clamp_hi{L}']))
    xl, xh = T(g['xl']), T(g['xh'])
    sb = ops._ibp_forward_graph_batched(xl, xh, gg, DEV, torch.float32, relu_clamps=clamps)
    alpha = {}
    for L, (lo, hi) in sb.items():
        lb_r = torch.clamp(lo, max=0)
        ub_r = torch.maximum(torch.clamp(hi, min=0), lb_r + 1e-8)
        up_s = ub_r / (ub_r - lb_r)
        unst = (lo < 0) & (hi > 0)
        alpha[L] = ((up_s > 0.5).float() * unst.float()).clone().requires_grad_(True)
    spec_ew = wk.spec_ew_from(g['spec_W'], g['spec_b'], DEV)
    opt = torch.optim.Adam(list(alpha.values()), lr=float(g['lr']))
    best = None
    for _ in range(int(g['n_iters'])):
        opt.zero_grad()
        lbs = ops._spec_backward_graph_batched(sb, xl, xh, gg, spec_ew, DEV, torch.float32,
                                               alpha_at_layer=alpha)
        best = lbs.detach().clone() if best is None else torch.maximum(best, lbs.detach())
        if (best > 0).all():
            break
        (-lbs.sum()).backward()
        opt.step()
        with torch.no_grad():
            for a in alpha.values():
                a.clamp_(0.0, 1.0)
    assert close(N(best), g['best_lb'], rtol=5e-3, atol=1e-5), max_excess(
        N(best), g['best_lb'], rtol=5e-3, atol=1e-5)


def test_bab_with_boundary_alpha_and_leaf_pgd():
    """acasxu_2023.yaml-style settings (CROWN intermediates, boundary
    alpha-CROWN, leaf PGD every 3 iterations) on cfg1: still verified, with
    no more leaves than plain CROWN (alpha only tightens)."""
    from vibecheck_nn_b200 import bab
    w = wk.cfg1(0)
    gg = wk.mlp_gg(w['layers'], DEV)
    spec = bab.LinearSpec(w['xl'], w['xh'], [[('pair', 1, 0)]])
    # the reference's default_settings values (width branching) plus the
    # preset's keys
    st = wk.reference_bab_settings(
        input_split_batch_size=2048, input_split_crown_intermediate=True,
        input_split_batched_alpha_boundary_eps=10.0, input_split_batched_alpha_iters=20,
        input_split_batched_alpha_max_leaves=2048, input_split_leaf_pgd_every=3,
        input_split_leaf_pgd_max_leaves=128, input_split_leaf_pgd_restarts=256,
        input_split_leaf_pgd_iters=50, total_timeout=600.0)
    v, det = bab._input_split_batched(None, spec, st, gg, DEV, torch.float32)
    assert v == 'verified', det
    assert det['batched_n_leaves'] <= int(load_golden('bab_cfg1_seed0')['n_leaves_ci1'])


def _small_cnn(g, device):
    import importlib.util
    import os
    spec = importlib.util.spec_from_file_location(
        'mkg', os.path.join(os.path.dirname(__file__), 'golden', 'make_golden.py'))
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    gg = mod._small_cnn_gg(g['k1'], g['b1'], g['W2'], g['b2'], g['W3'], g['b3'], (2, 8, 8),
                           torch.float32)
    return wk.gg_to(gg, device)


def test_conv_ibp_crown_golden():
    from vibecheck_nn_b200 import ops
    g = load_golden('conv_small')
    gg = _small_cnn(g, DEV)
    sb = ops._ibp_forward_graph_batched(T(g['xl']), T(g['xh']), gg, DEV, torch.float32)
    for L, (lo, hi) in sb.items():
        assert close(N(lo), g[f'ibp_lo{L}']) and close(N(hi), g[f'ibp_hi{L}']), L
    spec_ew = wk.spec_ew_from(g['spec_W'], g['spec_b'], DEV)
    lb, A, acc = ops._spec_backward_graph_batched(sb, T(g['xl']), T(g['xh']), gg, spec_ew, DEV,
                                                  torch.float32, return_input_linear=True)
    assert close(N(lb), g['lb']), max_excess(N(lb), g['lb'])
    assert close(N(A), g['A']) and close(N(acc), g['acc'])


def test_cfg4_cnn_against_oracle():
    """cfg4 CNN (3x32x32 -> conv16 -> conv32 -> fc100 -> fc10), 16 split
    domains, IBP with clamps + CROWN through conv-transpose."""
    from vibecheck_nn_b200 import ops
    w = wk.cfg4(seed=0)
    ggc = wk.cnn_gg(w['params'])
    root = ob.ibp_forward_batched(w['xl'][None], w['xh'][None], ggc)
    picked, clamps = wk.split_domains({L: v[0][0] for L, v in root.items()},
                                      {L: v[1][0] for L, v in root.items()}, 4)
    Dn = 1 << len(picked)
    xl = np.broadcast_to(w['xl'], (Dn, w['xl'].size)).copy()
    xh = np.broadcast_to(w['xh'], (Dn, w['xh'].size)).copy()
    y0 = ob.ibp_forward_batched(w['x0'][None], w['x0'][None], ggc)
    SW, Sb = wk.margin_rows(10, 3)
    sb_ref = ob.ibp_forward_batched(xl, xh, ggc, relu_clamps=clamps)
    lb_ref, A_ref, acc_ref = ob.spec_backward_batched(sb_ref, xl, xh, ggc, SW, Sb,
                                                      return_input_linear=True)
    gg = wk.cnn_gg(w['params'], DEV)
    tclamps = {L: (T(c[0]), T(c[1])) for L, c in clamps.items()}
    sb = ops._ibp_forward_graph_batched(T(xl), T(xh), gg, DEV, torch.float32, relu_clamps=tclamps)
    for L in sb_ref:
        assert close(N(sb[L][0]), sb_ref[L][0]) and close(N(sb[L][1]), sb_ref[L][1]), L
    lb, A, acc = ops._spec_backward_graph_batched(sb, T(xl), T(xh), gg,
                                                  wk.spec_ew_from(SW, Sb, DEV), DEV,
                                                  torch.float32, return_input_linear=True)
    assert close(N(lb), lb_ref), max_excess(N(lb), lb_ref)
    assert close(N(acc), acc_ref)
    _ = y0


def _cfg3_domains(n_split, n_iters_unused=None):
    w = wk.cfg3(seed=0)
    ggc = wk.mlp_gg(w['layers'])
    root = ob.ibp_forward_batched(w['xl'][None], w['xh'][None], ggc)
    picked, clamps = wk.split_domains({L: v[0][0] for L, v in root.items()},
                                      {L: v[1][0] for L, v in root.items()}, n_split)
    Dn = 1 << len(picked)
    xl = np.broadcast_to(w['xl'], (Dn, w['xl'].size)).copy()
    xh = np.broadcast_to(w['xh'], (Dn, w['xh'].size)).copy()
    return w, ggc, xl, xh, clamps


def test_tc_alpha_loop_against_oracle():
    """The tensor-core alpha loop (3xTF32 GEMMs, fused relaxation / adjoint /
    Adam stages) on the cfg3 network against the numpy oracle."""
    w, ggc, xl, xh, clamps = _cfg3_domains(5)
    ref, _ = ob.alpha_beta_crown_domains(xl, xh, ggc, w['spec_W'], w['spec_b'], clamps,
                                         n_iters=4, lr=0.1)
    gg = wk.mlp_gg(w['layers'], DEV)
    best, _ = wide.alpha_crown_domains(xl, xh, gg, w['spec_W'], w['spec_b'], clamps, DEV,
                                       n_iters=4, lr=0.1, tc=True)
    assert wide.last_stats['path'] == 'tc'
    assert close(N(best), ref, rtol=5e-3, atol=1e-4), max_excess(N(best), ref, rtol=5e-3,
                                                                 atol=1e-4)


def test_tc_alpha_loop_matches_simt_at_cfg3_size():
    """cfg3 itself (1,024 domains x 9 rows, 20 iterations): the size routing
    picks the tensor cores, and they agree with the SIMT layer kernels."""
    w, ggc, xl, xh, clamps = _cfg3_domains(10)
    gg = wk.mlp_gg(w['layers'], DEV)
    tcl = {L: (T(c[0]), T(c[1])) for L, c in clamps.items()}
    best_tc, _ = wide.alpha_crown_domains(xl, xh, gg, w['spec_W'], w['spec_b'], tcl, DEV,
                                          n_iters=20, lr=0.1)
    assert wide.last_stats['path'] == 'tc'
    best_s, _ = wide.alpha_crown_domains(xl, xh, gg, w['spec_W'], w['spec_b'], tcl, DEV,
                                         n_iters=20, lr=0.1, tc=False)
    assert close(N(best_tc), N(best_s), rtol=5e-3, atol=1e-4), max_excess(
        N(best_tc), N(best_s), rtol=5e-3, atol=1e-4)


@pytest.mark.parametrize('eps', [None, 1e-6])
def test_tc_alpha_loop_stops_like_simt(eps):
    """Stop rule (every best lb > 0, then the early-stop epsilon): shift the
    spec offsets so that the batch closes after a few iterations; the device
    gates must end the tensor-core loop at the same iteration as the SIMT loop
    (lb is b_q + an alpha-dependent part, and alpha's trajectory does not
    depend on b_q)."""
    w, ggc, xl, xh, clamps = _cfg3_domains(5)
    gg = wk.mlp_gg(w['layers'], DEV)
    wn = wide.wide_net(gg, DEV)
    xlt, xht = T(xl).float(), T(xh).float()
    tcl = {L: (T(c[0]), T(c[1])) for L, c in clamps.items()}
    sb = wide.wide_ibp(wn, xlt, xht, tcl)
    W_q, b_q = T(w['spec_W']).float(), T(w['spec_b']).float()
    mins = []
    for k in range(1, 7):
        b = wide.alpha_loop(wn, xlt, xht, sb, W_q, b_q, k, 0.1, tc=False)
        mins.append(float(b.min()))
    gaps = [mins[k] - mins[k - 1] for k in range(1, 6)]
    k = max(range(1, 6), key=lambda i: gaps[i - 1])   # widest step: closes after k + 1 iterations
    assert gaps[k - 1] > 1e-3
    shift = -(mins[k - 1] + mins[k]) / 2
    b_s = b_q + shift
    out_s = wide.alpha_loop(wn, xlt, xht, sb, W_q, b_s, 10, 0.1, early_stop_eps=eps, tc=False)
    it_s = wide.last_stats['iterations']
    out_t = wide.alpha_loop(wn, xlt, xht, sb, W_q, b_s, 10, 0.1, early_stop_eps=eps, tc=True)
    it_t = wide.last_stats['iterations']()
    assert it_t == it_s and (eps is not None or it_s == k + 1), (it_t, it_s, k)
    assert bool((out_t > 0).all()) == bool((out_s > 0).all())
    assert close(N(out_t), N(out_s), rtol=5e-3, atol=1e-4)


def test_tc_alpha_loop_graph_replay():
    """Repeated calls with the same shapes replay the loop as a CUDA graph
    from fixed buffers: each call's result follows its own inputs."""
    w, ggc, xl, xh, clamps = _cfg3_domains(9)
    gg = wk.mlp_gg(w['layers'], DEV)
    wn = wide.wide_net(gg, DEV)
    xlt, xht = T(xl).float(), T(xh).float()
    tcl = {L: (T(c[0]), T(c[1])) for L, c in clamps.items()}
    sb = wide.wide_ibp(wn, xlt, xht, tcl)
    W_q, b_q = T(w['spec_W']).float(), T(w['spec_b']).float()
    wide._tc_plan_cache.clear()
    for k, shift in enumerate([0.0, 3.0, -2.0, 0.5]):
        rng = np.random.default_rng(k)
        W_k = W_q * T(rng.uniform(0.5, 1.5, W_q.shape)).float()
        got = wide.alpha_loop(wn, xlt, xht, sb, W_k, b_q + shift, 6, 0.1, tc=True)
        assert (wide._tc_plan_cache['plan'].graph is not None) == (k > 0)
        ref = wide.alpha_loop(wn, xlt, xht, sb, W_k, b_q + shift, 6, 0.1, tc=False)
        assert close(N(got), N(ref), rtol=5e-3, atol=1e-4), (k, max_excess(N(got), N(ref),
                                                                           rtol=5e-3, atol=1e-4))


@pytest.mark.parametrize('dims, D', [((41, 50, 66, 30, 7), 48), ((9, 130, 3, 70, 5), 48),
                                     ((40, 64, 64, 48, 8), 37)])
def test_tc_alpha_loop_odd_widths_match_simt(dims, D):
    """Widths that are not multiples of 4 (the GEMM epilogue's one-column-per-
    lane path, partial 32- and 64-column groups, K tails) and row counts that
    end in a partial warp (37 x 3 rows on the 16-byte path) on the tensor
    cores against the SIMT layer kernels."""
    rng = np.random.default_rng(sum(dims))
    layers = wk.mlp_params(dims, rng)
    Q = 3
    x0 = rng.uniform(0, 1, (D, dims[0]))
    xl = (x0 - 0.08).astype(np.float32)
    xh = (x0 + 0.08).astype(np.float32)
    SW = rng.normal(size=(Q, dims[-1])).astype(np.float32)
    Sb = (rng.normal(size=Q) - 5.0).astype(np.float32)
    gg = wk.mlp_gg(layers, DEV)
    wn = wide.wide_net(gg, DEV)
    xlt, xht = T(xl), T(xh)
    sb = wide.wide_ibp(wn, xlt, xht)
    got = wide.alpha_loop(wn, xlt, xht, sb, T(SW), T(Sb), 6, 0.1, tc=True)
    assert wide.last_stats['path'] == 'tc'
    ref = wide.alpha_loop(wn, xlt, xht, sb, T(SW), T(Sb), 6, 0.1, tc=False)
    assert close(N(got), N(ref), rtol=5e-3, atol=1e-4), max_excess(N(got), N(ref), rtol=5e-3,
                                                                   atol=1e-4)
