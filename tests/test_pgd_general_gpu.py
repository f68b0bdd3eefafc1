"""GPU parity of ``vcb_mlp_pgd_general`` (pgd_attack_general, pgd.py:233-524)
with the reference's recorded attacks and with the numpy oracle fed the same
draws."""
import types

import numpy as np
import pytest
import torch

from conftest import load_golden, oracle_pgd_general, pgd_general_case
from oracle import pgd as opgd
from vibecheck_nn_b200 import netdesc, pgd, workloads as wk
from vibecheck_nn_b200.bab import LinearSpec

pytestmark = pytest.mark.gpu
DEV = torch.device('cuda:0') if torch.cuda.is_available() else None
TAGS = [str(t) for t in load_golden('pgd_general')['tags']]
FRACS = [0.25, 0.05, 0.01, 0.002]


def _kernel_case(case, budget_ns=0, n_iter=None):
    """The kernel on the fixture's own draws; returns (sat, witness, x)."""
    st = case['st']
    gg = wk.mlp_gg(case['layers'], DEV)
    desc = netdesc.mlp_desc(gg, DEV)
    R = st['pgd_restarts']
    xl = torch.as_tensor(case['xl'], device=DEV)
    xh = torch.as_tensor(case['xh'], device=DEV)
    eps = (xh - xl) / 2.0
    if st.get('pgd_alpha_multi'):
        pra = torch.tensor([FRACS[i % 4] for i in range(R)], device=DEV).unsqueeze(-1)
        step = eps.unsqueeze(0) * pra
    else:
        step = (eps * 0.25).unsqueeze(0)
    osi = st['pgd_init_mode'] == 'osi'
    w_d = torch.as_tensor(case['w_d'], device=DEV).contiguous() if osi else None
    x = torch.as_tensor(case['x_init'], device=DEV).contiguous().clone()
    act = sorted(case['restrict']) if case['restrict'] else [0, 1]
    prd = bool(st.get('pgd_per_restart_disjunct')) and len(act) > 1
    idx = pgd.pgd_general_run(desc, x, xl.unsqueeze(0), xh.unsqueeze(0), step, w_d,
                              st['pgd_osi_iters'], st['pgd_iter'] if n_iter is None else n_iter,
                              st['pgd_optim'], 0.99, -1e-5, st['pgd_plateau_iters'],
                              case['disj'], act, prd, 0.0, budget_ns)
    xs = x.cpu().numpy()
    if idx is None:
        return False, None, xs
    return True, xs[idx], xs


@pytest.mark.parametrize('tag', TAGS)
def test_pgd_general_matches_reference_and_oracle(tag):
    case = pgd_general_case(load_golden('pgd_general'), tag)
    sat, wit, xs = _kernel_case(case)
    osat, owit, info = oracle_pgd_general(case, wk.mlp_gg(case['layers']), 'cuda')
    assert sat == case['sat'] == osat
    if sat:
        np.testing.assert_allclose(wit, case['witness'], rtol=1e-5, atol=1e-6)
        np.testing.assert_allclose(wit, owit, rtol=1e-5, atol=1e-6)
    else:
        # the whole trajectory: the last iterate of every restart
        np.testing.assert_allclose(xs, case['x_last'], rtol=1e-5, atol=1e-6)
        np.testing.assert_allclose(xs, info['x'], rtol=1e-5, atol=1e-6)


def test_pgd_general_budget_ends_after_first_screen():
    """An exhausted wall-time budget leaves only the final check of the
    initial (post-OSI) iterate -- the oracle with no loop iterations."""
    g = load_golden('pgd_general')
    for tag in TAGS:
        case = pgd_general_case(g, tag)
        sat, wit, _ = _kernel_case(case, budget_ns=1)
        c0 = dict(case, st=dict(case['st'], pgd_iter=0))
        osat, owit, _ = oracle_pgd_general(c0, wk.mlp_gg(case['layers']), 'cuda')
        assert sat == osat, tag
        if sat:
            np.testing.assert_allclose(wit, owit, rtol=1e-5, atol=1e-6)


@pytest.mark.parametrize('seed', [0, 1, 2, 3])
def test_pgd_attack_general_api(seed):
    """Reference signature end to end: the CUDA draws after
    torch.manual_seed(seed) are the oracle's input too; the verdict agrees and
    a witness lies in the box and violates the property."""
    w = wk.cfg1(seed)
    gg = wk.mlp_gg(w['layers'], DEV)
    y = wk._mlp_forward64(w['layers'], (w['xl'] + (w['xh'] - w['xl'])
                                       * np.random.default_rng(seed).random((2048, 5))))
    disj = [[('ge', 0, float(y[:, 0].max()))], [('pair', 1, 2), ('le', 4, float(y[:, 4].min()))]]
    spec = LinearSpec(w['xl'], w['xh'], disj)
    st = types.SimpleNamespace(pgd_restarts=30, pgd_iter=100, pgd_optim='adam_clipping',
                               pgd_init_mode='osi', pgd_osi_iters=50)
    xl = torch.as_tensor(w['xl'], device=DEV)
    xh = torch.as_tensor(w['xh'], device=DEV)
    sat, wit = pgd.pgd_attack_general(xl, xh, spec, gg, st, seed=seed)
    torch.manual_seed(seed)
    x0 = xl + (xh - xl) * torch.rand(30, 5, device=DEV)
    w_d = (torch.rand(30, 5, device=DEV) - 0.5) * 2.0
    osat, owit, _ = opgd.pgd_attack_general(w['xl'], w['xh'], wk.mlp_gg(w['layers']), disj,
                                            x0.cpu().numpy(), w_d.cpu().numpy(), div='cuda')
    assert sat == osat
    if sat:
        np.testing.assert_allclose(wit, owit, rtol=1e-5, atol=1e-6)
        assert np.all(wit >= w['xl']) and np.all(wit <= w['xh'])
        yw = wk._mlp_forward64(w['layers'], wit[None].astype(np.float64))[0]
        viol0 = yw[0] >= disj[0][0][2] - 1e-4
        viol1 = yw[2] >= yw[1] - 1e-4 and yw[4] <= disj[1][1][2] + 1e-4
        assert viol0 or viol1


def test_root_pgd_sequence_reports_phase():
    """root_pgd runs pgd_attack_general first; an easy property is found
    there and reported as the 'batched_pgd' phase."""
    w = wk.cfg1(0)
    gg = wk.mlp_gg(w['layers'], DEV)
    spec = LinearSpec(w['xl'], w['xh'], [[('pair', 0, 1)]])
    st = types.SimpleNamespace(pgd_restarts=30, pgd_iter=100, pgd_optim='adam_clipping',
                               pgd_init_mode='osi', pgd_osi_iters=50)
    sat, wit, phase = pgd.root_pgd(spec, gg, 5, DEV, st)
    assert sat and phase == 'batched_pgd'
    y = wk._mlp_forward64(w['layers'], wit[None].astype(np.float64))[0]
    assert y[1] >= y[0] - 1e-5


def _root_pgd_sequential(spec, gg, st):
    """root_pgd's stages one after the other on one stream (the reference's
    order), for comparison with the overlapped version."""
    xl = torch.as_tensor(np.asarray(spec.x_lo), dtype=torch.float32, device=DEV)
    xh = torch.as_tensor(np.asarray(spec.x_hi), dtype=torch.float32, device=DEV)
    sat, wit = pgd.pgd_attack_general(xl, xh, spec, gg, st, time_budget=5.0)
    if sat and wit is not None:
        return True, wit, 'batched_pgd'
    sat, wit = pgd._simple_pgd(xl.flatten().unsqueeze(0), xh.flatten().unsqueeze(0), spec,
                               gg, 5, DEV, torch.float32, n_restarts=10000, n_iter=50)
    return (True, wit, 'batched_simple_pgd') if sat else (False, None, None)


@pytest.mark.parametrize('case', ['general_finds', 'none_finds', 'simple_finds'])
def test_root_pgd_overlapped_stages_match_sequential(case):
    """The general and simple stages overlap on two streams; verdict, phase,
    witness and the generators' states afterwards equal the sequential run."""
    w = wk.cfg1(0)
    gg = wk.mlp_gg(w['layers'], DEV)
    st = types.SimpleNamespace(pgd_restarts=10, pgd_iter=100, pgd_optim='adam_sign')
    pair = (1, 0) if case == 'none_finds' else (0, 1)
    spec = LinearSpec(w['xl'], w['xh'], [[('pair',) + pair]])
    if case == 'simple_finds':
        st.pgd_iter = 1  # one step from uniform draws: the general stage gives up
        st.pgd_restarts = 1
    outs = []
    for fn in (lambda: pgd.root_pgd(spec, gg, 5, DEV, st),
               lambda: _root_pgd_sequential(spec, gg, st)):
        torch.manual_seed(1234)
        outs.append((fn(), torch.get_rng_state(), torch.cuda.get_rng_state(DEV)))
    (a, ca, ga), (b, cb_, gb) = outs
    assert a[0] == b[0] and a[2] == b[2], (a[:1] + a[2:], b[:1] + b[2:])
    if a[0]:
        np.testing.assert_array_equal(a[1], b[1])
    assert torch.equal(ca, cb_) and torch.equal(ga, gb)
    if case == 'none_finds':
        assert not a[0]
