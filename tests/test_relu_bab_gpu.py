"""GPU parity of the ReLU-split BaB driver (verify_milp.py:2658-2960) against
verdicts, domain counts and stop reasons recorded from the reference
(tests/golden/make_golden.py --only relu_bab): the same frontier order,
alpha-beta Adam steps, kfsb branching and pruning on the B200 bound kernels
must visit exactly as many domains."""
import numpy as np
import pytest
import torch

from conftest import golden_script, load_golden
from vibecheck_nn_b200 import ops, relu_bab, workloads as wk

pytestmark = pytest.mark.gpu
DEV = torch.device('cuda:0') if torch.cuda.is_available() else None
G = load_golden('relu_bab')
CASES = {c[0]: c for c in golden_script().RELU_BAB_CASES}


def _problem(tag):
    _, seed, dims, eps, kw = CASES[tag]
    layers, xl, xh, w = golden_script().relu_bab_problem(seed, dims, eps)
    gg = wk.mlp_gg(layers, DEV, torch.float32)
    xlt = torch.as_tensor(xl, device=DEV)
    xht = torch.as_tensor(xh, device=DEV)
    sb = ops._ibp_forward_graph_batched(xlt[None], xht[None], gg, DEV, torch.float32)
    root = {L: (lo[0], hi[0]) for L, (lo, hi) in sb.items()}
    return gg, xlt, xht, root, w, kw


@pytest.mark.parametrize('tag', [str(t) for t in G['tags']])
def test_relu_bab_matches_reference(tag):
    gg, xl, xh, root, w, kw = _problem(tag)
    args = golden_script().relu_bab_kwargs(kw, root)
    closed, n, reason = relu_bab._ibp_crown_bab(gg, xl, xh, root, w, 0.0, DEV, torch.float32,
                                                **args)
    assert (closed, n, reason) == (bool(G[f'{tag}_closed']), int(G[f'{tag}_n']),
                                   str(G[f'{tag}_reason']))


def test_relu_bab_time_budget():
    gg, xl, xh, root, w, _ = _problem('closed229')
    assert relu_bab._ibp_crown_bab(gg, xl, xh, root, w, 0.0, DEV, torch.float32,
                                   time_left=lambda: 2.0) == (False, 0, 'time')


def test_domain_coefficients_match_host_chain():
    gg, xl, xh, root, w, _ = _problem('closed20')
    B = 3
    g = torch.Generator().manual_seed(0)
    sb = {}
    for L, (lo, hi) in root.items():
        jl = torch.rand((B, lo.numel()), generator=g).to(DEV) * 0.2
        sb[L] = (lo[None] + jl * (hi - lo)[None], hi[None] - jl * (hi - lo)[None])
    wt = torch.as_tensor(w, device=DEV, dtype=torch.float32)
    got = relu_bab._domain_relu_coeffs(gg, sb, wt, DEV, torch.float32)
    layers = [(np.asarray(W, np.float64), np.asarray(b, np.float64))
              for W, b in wk.mlp_params(CASES['closed20'][2], np.random.default_rng(0))]
    for bi in range(B):
        ew = np.asarray(w, np.float64)
        for L in reversed(range(len(layers) - 1)):
            ew = ew @ layers[L + 1][0]
            assert np.allclose(got[bi][L].cpu().numpy(), np.abs(ew), rtol=1e-4, atol=1e-5)
            lo = sb[L][0][bi].double().cpu().numpy()
            hi = sb[L][1][bi].double().cpu().numpy()
            lb_r, ub_r = np.minimum(lo, 0), np.maximum(np.maximum(hi, 0), np.minimum(lo, 0) + 1e-8)
            up = ub_r / (ub_r - lb_r)
            act, uns = lo >= 0, (lo < 0) & (hi > 0)
            lo_s = ((up > 0.5) & uns) + act
            ew = np.maximum(ew, 0) * lo_s + np.minimum(ew, 0) * up
