"""GPU parity of the freeze-replay hybrid pipeline (verify_hybrid_acasxu.py:
164-539) against outcomes recorded from the reference on CPU
(tests/golden/make_golden.py --only hybrid): verdict, phase and the BaB
counters, plus the per-query alpha machinery it needs (seeded backward with
per-row slopes and their gradient, input-linear outputs with alpha
gradients)."""
import types

import numpy as np
import pytest
import torch

from conftest import golden_script, load_golden
from vibecheck_nn_b200 import hybrid, ops, workloads as wk
from vibecheck_nn_b200.bab import LinearSpec

pytestmark = pytest.mark.gpu
DEV = torch.device('cuda:0') if torch.cuda.is_available() else None
G = load_golden('hybrid')
CASES = {c[0]: c for c in golden_script().HYBRID_CASES}


def _problem(tag):
    _, seed, offset, st = CASES[tag]
    layers, xl, xh = golden_script().hybrid_problem(seed, offset)
    gg = wk.mlp_gg(layers, DEV, torch.float32)
    graph = types.SimpleNamespace(gpu_graph=lambda device, dtype: gg)
    spec = LinearSpec(xl, xh, [[('pair', 1, 0)]])  # unsafe iff Y0' >= Y1'
    return layers, gg, graph, spec, types.SimpleNamespace(**st)


@pytest.mark.parametrize('tag', [str(t) for t in G['tags']])
def test_verify_hybrid_matches_reference(tag):
    layers, gg, graph, spec, st = _problem(tag)
    res = hybrid.verify_hybrid(graph, spec, st, timeout=600.0)
    assert res['verdict'] == str(G[f'{tag}_verdict']), res
    assert res['phase'] == str(G[f'{tag}_phase'])
    if res['verdict'] == 'sat':
        x = np.asarray(res['witness'], np.float64).reshape(1, -1)
        assert (x >= spec.x_lo - 1e-6).all() and (x <= spec.x_hi + 1e-6).all()
        y = wk._mlp_forward64(layers, x)[0]
        assert y[0] >= y[1]  # the unsafe region
    else:
        # 100-step fp32 Adam trajectories round differently on the GPU than on
        # the reference's CPU run, which moves a handful of leaves that sit at
        # the closure boundary: counts agree within 0.1 %, iterations within 1
        for k in ('evaluated', 'closed'):
            ref = int(G[f'{tag}_{k}'])
            assert abs(res[k] - ref) <= max(4, ref // 1000), (k, res[k], ref)
        assert abs(res['bab_iters'] - int(G[f'{tag}_bab_iters'])) <= 1


def test_per_query_alpha_gradient_matches_finite_differences():
    """d sum(lb) / d alpha for (B, Q, n) slopes on the seeded backward."""
    _, gg, _, spec, _ = _problem('unsat0')
    xl = torch.as_tensor(spec.x_lo, device=DEV, dtype=torch.float32)[None].repeat(3, 1)
    xh = torch.as_tensor(spec.x_hi, device=DEV, dtype=torch.float32)[None].repeat(3, 1)
    xh[1] = xl[1] + (xh[1] - xl[1]) * 0.5
    xh[2] = xl[2] + (xh[2] - xl[2]) * 0.25
    from vibecheck_nn_b200.interm import _forward_zonotope_graph_batched
    sb, _ = _forward_zonotope_graph_batched(xl, xh, gg, DEV, torch.float32)
    L = 2
    n = sb[L][0].shape[1]
    seed, acc = hybrid._layer_seeds(gg, n, 3, DEV, torch.float32)
    feed = [op for op in gg['ops'] if op['type'] == 'relu' and op.get('layer_idx') == L][0]['inputs'][0]
    g = torch.Generator(device=DEV).manual_seed(0)
    alpha = {k: torch.rand((3, 2 * n, sb[k][0].shape[1]), generator=g, device=DEV).requires_grad_(True)
             for k in range(L)}
    lb = ops._spec_backward_graph_batched(sb, xl, xh, gg, None, DEV, torch.float32,
                                          alpha_at_layer=alpha, seed_ew_at={feed: seed},
                                          seed_acc=acc)
    lb.sum().backward()
    # the same bounds through the shared-memory kernel with the slopes of one row
    with torch.no_grad():
        for k in range(L):
            for (b, q) in ((0, 3), (2, 71)):
                unstable = (sb[k][0][b] < 0) & (sb[k][1][b] > 0)
                j = int(torch.nonzero(unstable)[0]) if bool(unstable.any()) else 0
                h = 1e-2
                a_p = {kk: v.detach().clone() for kk, v in alpha.items()}
                a_m = {kk: v.detach().clone() for kk, v in alpha.items()}
                a_p[k][b, q, j] += h
                a_m[k][b, q, j] -= h
                f = [ops._spec_backward_graph_batched(sb, xl, xh, gg, None, DEV, torch.float32,
                                                      alpha_at_layer=a, seed_ew_at={feed: seed},
                                                      seed_acc=acc).sum().double()
                     for a in (a_p, a_m)]
                fd = float((f[0] - f[1]) / (2 * h))
                assert abs(float(alpha[k].grad[b, q, j]) - fd) <= 2e-3 * max(1.0, abs(fd)), \
                    (k, b, q, j, float(alpha[k].grad[b, q, j]), fd)


def test_input_linear_with_alpha_gradient():
    _, gg, _, spec, _ = _problem('unsat0')
    xl = torch.as_tensor(spec.x_lo, device=DEV, dtype=torch.float32)[None].repeat(2, 1)
    xh = torch.as_tensor(spec.x_hi, device=DEV, dtype=torch.float32)[None].repeat(2, 1)
    sb = ops._ibp_forward_graph_batched(xl, xh, gg, DEV, torch.float32)
    spec_ew = {0: (torch.tensor([-1.0, 1.0, 0, 0, 0], device=DEV), 0.0)}
    alpha = {L: torch.full((2, 1, lo.shape[1]), 0.5, device=DEV).requires_grad_(True)
             for L, (lo, _) in sb.items()}
    lb, A, acc = ops._spec_backward_graph_batched(sb, xl, xh, gg, spec_ew, DEV, torch.float32,
                                                  alpha_at_layer=alpha,
                                                  return_input_linear=True)
    lb2 = ops._spec_backward_graph_batched(sb, xl, xh, gg, spec_ew, DEV, torch.float32,
                                           alpha_at_layer={L: a.detach() for L, a in alpha.items()})
    assert torch.allclose(lb, lb2)
    conc = acc + (A.clamp(min=0) * xl[:, None]).sum(-1) + (A.clamp(max=0) * xh[:, None]).sum(-1)
    assert torch.allclose(conc, lb, rtol=1e-5, atol=1e-5)
    (-lb.sum()).backward()
    assert all(a.grad is not None for a in alpha.values())
