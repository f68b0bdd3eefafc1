"""GPU parity of the fused IBP + CROWN kernel (vcb_mlp_crown).

Checked against (a) golden vectors recorded from the reference and (b) the
numpy oracle on seeded cfg2 inputs, at |a-b| <= 1e-6 + 1e-5 |b|.
"""
import numpy as np
import pytest
import torch

from conftest import close, golden_layers, load_golden, max_excess
from oracle import bounds as ob
from vibecheck_nn_b200 import ops, workloads as wk

pytestmark = pytest.mark.gpu
DEV = torch.device('cuda:0') if torch.cuda.is_available() else None


def T(a):
    return torch.as_tensor(np.asarray(a), device=DEV)


def N(t):
    return t.detach().cpu().numpy()


@pytest.mark.parametrize('tag', ['small', 'acas'])
def test_golden_ibp_and_crown(tag):
    g = load_golden(f'mlp_{tag}')
    gg = wk.mlp_gg(golden_layers(g), DEV)
    spec_ew = wk.spec_ew_from(g['spec_W'], g['spec_b'], DEV)
    sb = ops._ibp_forward_graph_batched(T(g['xl']), T(g['xh']), gg, DEV,
                                        torch.float32)
    for L, (lo, hi) in sb.items():
        assert close(N(lo), g[f'ibp32_lo{L}']), max_excess(N(lo), g[f'ibp32_lo{L}'])
        assert close(N(hi), g[f'ibp32_hi{L}'])
    lb, A, acc = ops._spec_backward_graph_batched(
        sb, T(g['xl']), T(g['xh']), gg, spec_ew, DEV, torch.float32,
        return_input_linear=True)
    assert close(N(lb), g['crown32_lb']), max_excess(N(lb), g['crown32_lb'])
    assert close(N(A), g['crown32_A'])
    assert close(N(acc), g['crown32_acc'])
    # fused single launch
    lb2, A2, acc2 = ops.ibp_crown_batched(T(g['xl']), T(g['xh']), gg, spec_ew,
                                          DEV, return_input_linear=True)
    assert close(N(lb2), g['crown32_lb'])
    assert close(N(A2), g['crown32_A']) and close(N(acc2), g['crown32_acc'])


@pytest.mark.parametrize('tag', ['small', 'acas'])
def test_golden_clamped(tag):
    g = load_golden(f'mlp_{tag}')
    gg = wk.mlp_gg(golden_layers(g), DEV)
    spec_ew = wk.spec_ew_from(g['spec_W'], g['spec_b'], DEV)
    clamps = {0: (T(g['clamp_lo0']), T(g['clamp_hi0']))}
    sb = ops._ibp_forward_graph_batched(T(g['xl']), T(g['xh']), gg, DEV,
                                        torch.float32, relu_clamps=clamps)
    for L, (lo, hi) in sb.items():
        assert close(N(lo), g[f'ibpc32_lo{L}']) and close(N(hi), g[f'ibpc32_hi{L}'])
    lb = ops.ibp_crown_batched(T(g['xl']), T(g['xh']), gg, spec_ew, DEV,
                               relu_clamps=clamps)
    assert close(N(lb), g['crownc32_lb'])


@pytest.mark.parametrize('tag', ['small', 'acas'])
def test_golden_spec_on_crown_intermediates(tag):
    """Spec backward given externally computed (CROWN-intermediate) bounds."""
    g = load_golden(f'mlp_{tag}')
    gg = wk.mlp_gg(golden_layers(g), DEV)
    spec_ew = wk.spec_ew_from(g['spec_W'], g['spec_b'], DEV)
    n_relu = int(g['n_layers']) - 1
    tight = {L: (T(g[f'interm32_lo{L}']), T(g[f'interm32_hi{L}']))
             for L in range(n_relu)}
    lb, A, acc = ops._spec_backward_graph_batched(
        tight, T(g['xl']), T(g['xh']), gg, spec_ew, DEV, torch.float32,
        return_input_linear=True)
    assert close(N(lb), g['spec_interm32_lb'])
    assert close(N(A), g['spec_interm32_A'])
    assert close(N(acc), g['spec_interm32_acc'])


@pytest.mark.parametrize('B,Q', [(1, 4), (17, 4), (33, 1), (40, 9), (4096, 4)])
def test_cfg2_vs_oracle(B, Q):
    w = wk.cfg2(seed=3, n_boxes=B, n_q=Q)
    gg = wk.mlp_gg(w['layers'], DEV)
    spec_ew = wk.spec_ew_from(w['spec_W'], w['spec_b'], DEV)
    lb, A, acc, sbd = ops.ibp_crown_batched(T(w['xl']), T(w['xh']), gg, spec_ew,
                                            DEV, return_input_linear=True,
                                            return_sb=True)
    ggc = wk.mlp_gg(w['layers'])
    sb = ob.ibp_forward_batched(w['xl'], w['xh'], ggc)
    r_lb, r_A, r_acc = ob.spec_backward_batched(sb, w['xl'], w['xh'], ggc,
                                                w['spec_W'], w['spec_b'],
                                                return_input_linear=True)
    for L in sb:
        assert close(N(sbd[L][0]), sb[L][0]) and close(N(sbd[L][1]), sb[L][1])
    assert close(N(lb), r_lb), max_excess(N(lb), r_lb)
    assert close(N(A), r_A) and close(N(acc), r_acc)


def test_cfg2_full_size_against_oracle():
    """The benchmark workload itself (65,536 boxes, Q=4)."""
    w = wk.cfg2(seed=0)
    gg = wk.mlp_gg(w['layers'], DEV)
    spec_ew = wk.spec_ew_from(w['spec_W'], w['spec_b'], DEV)
    lb = ops.ibp_crown_batched(T(w['xl']), T(w['xh']), gg, spec_ew, DEV)
    ggc = wk.mlp_gg(w['layers'])
    sb = ob.ibp_forward_batched(w['xl'], w['xh'], ggc)
    r_lb = ob.spec_backward_batched(sb, w['xl'], w['xh'], ggc, w['spec_W'],
                                    w['spec_b'])
    assert close(N(lb), r_lb), max_excess(N(lb), r_lb)
    # soundness against concrete samples of the first 256 boxes
    rng = np.random.default_rng(1)
    xs = w['xl'][:256, None, :] + (w['xh'] - w['xl'])[:256, None, :] * \
        rng.random((256, 64, 5))
    ys = wk._mlp_forward64(w['layers'], xs.reshape(-1, 5)).reshape(256, 64, -1)
    spec_vals = ys @ w['spec_W'].T.astype(np.float64)
    assert (N(lb)[:256, None, :] <= spec_vals.min(axis=1, keepdims=True) + 1e-5).all()


def test_empty_batch_and_zero_width_boxes():
    w = wk.cfg2(seed=4, n_boxes=8)
    gg = wk.mlp_gg(w['layers'], DEV)
    spec_ew = wk.spec_ew_from(w['spec_W'], w['spec_b'], DEV)
    lb = ops.ibp_crown_batched(T(w['xl'][:0]), T(w['xh'][:0]), gg, spec_ew, DEV)
    assert lb.shape == (0, 4)
    x = w['xl']
    lb = ops.ibp_crown_batched(T(x), T(x), gg, spec_ew, DEV)
    y = wk._mlp_forward64(w['layers'], x.astype(np.float64)) @ \
        w['spec_W'].T.astype(np.float64)
    assert np.allclose(N(lb), y, rtol=1e-5, atol=1e-5)


def test_unsupported_graph_raises_notimplemented():
    gg = wk.mlp_gg(wk.mlp_params((4, 6, 3), np.random.default_rng(0)), DEV)
    gg['ops'].insert(1, {'name': 'sg', 'type': 'sigmoid', 'inputs': ['fc0']})
    with pytest.raises(NotImplementedError):
        ops._ibp_forward_graph_batched(torch.zeros(2, 4, device=DEV),
                                       torch.ones(2, 4, device=DEV), gg, DEV,
                                       torch.float32)
