"""Gradients of the CROWN lower bound with respect to alpha AND the split
multipliers beta through _spec_backward_graph_batched (the hand-written
adjoint), against the float64 oracle: alpha by its hand-written adjoint,
beta by central differences (lb is piecewise linear in beta)."""
import numpy as np
import pytest
import torch

from conftest import golden_layers, load_golden
from oracle import bounds as ob
from vibecheck_nn_b200 import ops, workloads as wk

pytestmark = pytest.mark.gpu
DEV = torch.device('cuda:0') if torch.cuda.is_available() else None


def _oracle_lb(tight, xl, xh, ggc, SW, Sb, alpha, beta):
    return ob.spec_backward_batched(tight, xl, xh, ggc, SW, Sb, alpha=alpha, beta=beta,
                                    dtype=np.float64)


@pytest.mark.parametrize('tag', ['small', 'acas'])
def test_alpha_and_beta_gradients(tag):
    g = load_golden(f'mlp_{tag}')
    layers = golden_layers(g)
    ggc = wk.mlp_gg(layers)
    xl, xh = g['xl'].astype(np.float64), g['xh'].astype(np.float64)
    SW, Sb = g['spec_W'].astype(np.float64), g['spec_b'].astype(np.float64)
    tight = ob.ibp_forward_batched(xl, xh, ggc, dtype=np.float64)
    rng = np.random.default_rng(7)
    B = xl.shape[0]
    alpha = {L: rng.uniform(0, 1, lo.shape) for L, (lo, hi) in tight.items()}
    beta = {L: rng.uniform(-0.3, 0.3, lo.shape) * (rng.random(lo.shape) < 0.3)
            for L, (lo, hi) in tight.items()}
    # GPU: the reference's usage (leaf tensors requiring grad, loss -sum(lb))
    T = lambda a, rg=False: torch.tensor(np.asarray(a, np.float32), device=DEV,  # noqa: E731
                                         requires_grad=rg)
    al_t = {L: T(a, True) for L, a in alpha.items()}
    be_t = {L: T(b, True) for L, b in beta.items()}
    tight_t = {L: (T(lo), T(hi)) for L, (lo, hi) in tight.items()}
    spec_ew = wk.spec_ew_from(g['spec_W'], g['spec_b'], DEV)
    lb = ops._spec_backward_graph_batched(tight_t, T(xl), T(xh), wk.mlp_gg(layers, DEV), spec_ew,
                                          DEV, torch.float32, alpha_at_layer=al_t,
                                          relu_split_beta=be_t)
    (-lb.sum()).backward()
    lb_ref = _oracle_lb(tight, xl, xh, ggc, SW, Sb, alpha, beta)
    np.testing.assert_allclose(lb.detach().cpu().numpy(), lb_ref, rtol=1e-4, atol=1e-4)
    # alpha: the oracle's float64 adjoint (d sum lb / d alpha)
    _, ga = ob.alpha_grad(tight, xl, xh, ggc, SW, Sb, alpha, dtype=np.float64, beta=beta)
    for L in alpha:
        np.testing.assert_allclose(al_t[L].grad.cpu().numpy(), -ga[L], rtol=1e-3,
                                   atol=1e-3 * (np.abs(ga[L]).max() + 1e-6))
    # beta: central differences of sum lb in float64
    h = 1e-6
    for L in beta:
        num = np.zeros_like(beta[L])
        for j in range(beta[L].shape[1]):
            bp = {k: v.copy() for k, v in beta.items()}
            bm = {k: v.copy() for k, v in beta.items()}
            bp[L][:, j] += h
            bm[L][:, j] -= h
            dp = _oracle_lb(tight, xl, xh, ggc, SW, Sb, alpha, bp).sum(axis=1)
            dm = _oracle_lb(tight, xl, xh, ggc, SW, Sb, alpha, bm).sum(axis=1)
            num[:, j] = (dp - dm) / (2 * h)
        got = be_t[L].grad.cpu().numpy()
        np.testing.assert_allclose(got, -num, rtol=1e-3, atol=1e-3 * (np.abs(num).max() + 1e-6))
        assert np.abs(num).max() > 0
