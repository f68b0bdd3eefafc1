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


def close_linear_form(A, A_ref, rtol=1e-5, atol=1e-6):
    """Input-space linear forms (the A output, one row per box and spec row):
    each coefficient within atol + rtol * the largest |coefficient| of its
    reference row.  The coefficients of a row are the sums whose signs
    cancel in the concretisation, so their rounding is relative to the row's
    scale; the bounds themselves are held to ``close``."""
    A = np.asarray(A, np.float64)
    A_ref = np.asarray(A_ref, np.float64)
    scale = np.abs(A_ref).max(axis=-1, keepdims=True)
    return bool((np.abs(A - A_ref) <= atol + rtol * scale).all())


def fp32_equivalent(ours, ref32, ref64, rtol=1e-5, atol=1e-6, slack=2.0):
    """fp32-equivalence against exact (float64) arithmetic: every element of
    ``ours`` within the parity tolerance of the float64 result plus ``slack``
    times the float32 reference's own worst error on the same output.
    Returns (ok, worst excess, worst error of ours, worst error of ref32)."""
    ours = np.asarray(ours, np.float64)
    ref32 = np.asarray(ref32, np.float64)
    ref64 = np.asarray(ref64, np.float64)
    ref_err = float(np.abs(ref32 - ref64).max(initial=0.0))
    err = np.abs(ours - ref64)
    excess = err - (atol + rtol * np.abs(ref64) + slack * ref_err)
    worst = float(excess.max(initial=-1.0))
    return worst <= 0, worst, float(err.max(initial=0.0)), ref_err


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


def golden_script():
    """tests/golden/make_golden.py as a module (graph builders shared by the
    fixtures and the tests; it imports the reference only when run)."""
    import importlib.util
    spec = importlib.util.spec_from_file_location('make_golden',
                                                  os.path.join(GOLDEN, 'make_golden.py'))
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def forward_fixture(device='cpu'):
    """The concrete-forward fixture: (CNN gg, MLP gg, arrays)."""
    import torch
    from vibecheck_nn_b200 import workloads as wk
    g = load_golden('forward')
    mg = golden_script()
    gg = mg.forward_cnn_gg(g['k1'], g['b1'], g['cb'], g['W2'], g['b2'], g['W3'], g['b3'],
                           g['fb'], (3, 12, 12), torch.float32)
    if str(device) != 'cpu':
        for op in gg['ops']:
            for k in ('W', 'bias', 'kernel'):
                if isinstance(op.get(k), torch.Tensor):
                    op[k] = op[k].to(device)
    n = int(g['mlp_n_layers'])
    layers = [(g[f'mlp_W{i}'], g[f'mlp_b{i}']) for i in range(n)]
    return gg, wk.mlp_gg(layers, device), g
