"""GPU parity of the batched PGD kernel (vcb_mlp_pgd) with the reference's
recorded results and with the numpy oracle on the same initial samples."""
import numpy as np
import pytest
import torch

from conftest import golden_layers, load_golden
from oracle import pgd as opgd
from vibecheck_nn_b200 import netdesc, pgd, workloads as wk
from vibecheck_nn_b200.bab import LinearSpec

pytestmark = pytest.mark.gpu
DEV = torch.device('cuda:0') if torch.cuda.is_available() else None


def _run(desc, x0, xl, xh, R, spec, n_out, n_iter):
    C, cb, cdis, D = pgd._constraint_rows(spec, n_out)
    x = torch.as_tensor(x0, device=DEV).contiguous().clone()
    key, x = pgd.pgd_run(desc, x, torch.as_tensor(xl, device=DEV),
                         torch.as_tensor(xh, device=DEV), R,
                         torch.as_tensor(C, device=DEV), torch.as_tensor(cb, device=DEV),
                         torch.as_tensor(cdis, device=DEV), D, n_iter, 0.1)
    if key == pgd.NO_SAT:
        return False, None
    return True, x[key & 0xFFFFFFFF].cpu().numpy()


@pytest.mark.parametrize('tag', ['unsat', 'sat'])
def test_pgd_golden(tag):
    g = load_golden('pgd')
    layers = golden_layers(g)
    desc = netdesc.mlp_desc(wk.mlp_gg(layers, DEV), DEV)
    thr = float(g[f'{tag}_thr'])
    spec = LinearSpec(g['xl'][0], g['xh'][0],
                      [[('ge', 0, thr)], [('pair', 1, 2), ('le', 3, -50.0)]])
    sat, wit = _run(desc, g[f'{tag}_x_init'], g['xl'], g['xh'], int(g['R']), spec, 4,
                    int(g['n_iter']))
    assert sat == bool(g[f'{tag}_sat'])
    if sat:
        np.testing.assert_allclose(wit, g[f'{tag}_witness'], rtol=1e-5, atol=1e-6)


@pytest.mark.parametrize('seed', [0, 1, 2])
def test_pgd_matches_oracle(seed):
    rng = np.random.default_rng(100 + seed)
    layers = wk.mlp_params((5, 50, 50, 50, 5), rng)
    B, R = 12, 32
    c = rng.uniform(-0.5, 0.5, (B, 5))
    h = rng.uniform(0.05, 0.4, (B, 5))
    xl = (c - h).astype(np.float32)
    xh = (c + h).astype(np.float32)
    x0 = (np.repeat(xl, R, 0) + np.repeat(xh - xl, R, 0) * rng.random((B * R, 5))).astype(np.float32)
    y = wk._mlp_forward64(layers, x0.astype(np.float64))
    thr = float(np.quantile(y[:, 0], 0.97 if seed else 0.5))
    disj = [[('ge', 0, thr), ('pair', 1, 2)], [('le', 4, float(y[:, 4].min()) - 1.0)]]
    spec = LinearSpec(xl[0], xh[0], disj)
    desc = netdesc.mlp_desc(wk.mlp_gg(layers, DEV), DEV)
    sat, wit = _run(desc, x0, xl, xh, R, spec, 5, 40)
    mats = opgd.margin_matrices(disj, 5)
    osat, owit, _ = opgd.pgd_batched(x0, np.repeat(xl, R, 0), np.repeat(xh, R, 0),
                                     wk.mlp_gg(layers), mats, n_iter=40)
    assert sat == osat
    if sat:
        np.testing.assert_allclose(wit, owit, rtol=1e-5, atol=1e-6)


def test_simple_pgd_finds_easy_witness_and_respects_box():
    w = wk.cfg1(0)
    gg = wk.mlp_gg(w['layers'], DEV)
    # unsafe region y0' >= y1' is unreachable (d has margin 0.5): no witness
    spec = LinearSpec(w['xl'], w['xh'], [[('pair', 1, 0)]])
    sat, _ = pgd._simple_pgd(torch.as_tensor(w['xl']).unsqueeze(0),
                             torch.as_tensor(w['xh']).unsqueeze(0), spec, gg, 5, DEV,
                             torch.float32, n_restarts=2048, n_iter=50)
    assert not sat
    # the reversed property is violated almost everywhere: witness inside the box
    spec2 = LinearSpec(w['xl'], w['xh'], [[('pair', 0, 1)]])
    sat, wit = pgd._simple_pgd(torch.as_tensor(w['xl']).unsqueeze(0),
                               torch.as_tensor(w['xh']).unsqueeze(0), spec2, gg, 5,
                               DEV, torch.float32, n_restarts=256, n_iter=50)
    assert sat and np.all(wit >= w['xl'] - 1e-7) and np.all(wit <= w['xh'] + 1e-7)
    # PairwiseConstraint(pred=0, comp=1) is violated where y1 >= y0
    y = wk._mlp_forward64(w['layers'], wit[None].astype(np.float64))[0]
    assert y[0] - y[1] <= 1e-5
