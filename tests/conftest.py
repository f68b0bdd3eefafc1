import os
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

GOLDEN = os.path.join(ROOT, 'tests', 'golden')


def pytest_configure(config):
    config.addinivalue_line('markers', 'gpu: needs a CUDA GPU (B200)')
    config.addinivalue_line('markers', 'slow: long-running CPU test')


def load_golden(name):
    return dict(np.load(os.path.join(GOLDEN, name + '.npz')))


def golden_layers(g):
    n = int(g['n_layers'])
    return [(g[f'W{i}'], g[f'b{i}']) for i in range(n)]


def close(a, b, rtol=1e-5, atol=1e-6):
    """Reference-parity tolerance: |a - b| <= atol + rtol * |b|."""
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    return np.allclose(a, b, rtol=rtol, atol=atol)


def max_excess(a, b, rtol=1e-5, atol=1e-6):
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    return float(np.max(np.abs(a - b) - (atol + rtol * np.abs(b)), initial=-1))


@pytest.fixture(scope='session')
def cuda_available():
    import torch
    return torch.cuda.is_available()


def pgd_general_case(g, tag):
    """One pgd_attack_general fixture case: net layers, box, spec disjuncts
    (tuple form), settings dict, restrict set, draws and reference results."""
    import ast
    p = tag + '_'
    net = str(g[p + 'net'])
    n = int(g[f'{net}_n_layers'])
    layers = [(g[f'{net}_W{i}'], g[f'{net}_b{i}']) for i in range(n)]
    second = [('le', 3, float(g[p + 'thr3']))]
    if not bool(g[p + 'no_pair']):
        second.insert(0, ('pair', 1, 2))
    disj = [[('ge', 0, float(g[p + 'thr']))], second]
    st = dict(ast.literal_eval(str(g[p + 'settings'])))
    r = int(g[p + 'restrict'])
    return dict(layers=layers, xl=g[p + 'xl'], xh=g[p + 'xh'], disj=disj, st=st,
                restrict=None if r < 0 else {r}, x_init=g[p + 'x_init'],
                w_d=g[p + 'w_d'], sat=bool(g[p + 'sat']), witness=g[p + 'witness'],
                screens=int(g[p + 'screens']), x_last=g[p + 'x_last'])


def oracle_pgd_general(case, gg, div):
    from oracle import pgd as opgd
    st = case['st']
    return opgd.pgd_attack_general(
        case['xl'], case['xh'], gg, case['disj'], case['x_init'],
        case['w_d'] if st['pgd_init_mode'] == 'osi' else None,
        n_iter=st['pgd_iter'], optim=st['pgd_optim'], osi_iters=st['pgd_osi_iters'],
        plateau_iters=st['pgd_plateau_iters'],
        alpha_fracs=[0.25, 0.05, 0.01, 0.002] if st.get('pgd_alpha_multi') else None,
        per_restart_disj=st.get('pgd_per_restart_disjunct', False),
        active=case['restrict'], div=div)
