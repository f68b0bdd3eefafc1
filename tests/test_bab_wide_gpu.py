"""BaB on wide inputs and wide networks: the one-CTA-per-leaf step kernel
(vcb_bab_step_wide) and the wide engine (tcgen05 zonotope + layer-wise CROWN)
against the single-CTA kernel, the reference's cfg1 leaf count and the
numpy oracle's BaB."""
import types

import numpy as np
import pytest
import torch

from conftest import load_golden
from oracle import bab as obab
from vibecheck_nn_b200 import bab, workloads as wk
from vibecheck_nn_b200.bab import LinearSpec

pytestmark = pytest.mark.gpu
DEV = torch.device('cuda:0') if torch.cuda.is_available() else None


def _cfg1_run(monkeypatch, wide_step):
    if wide_step:
        monkeypatch.setattr(bab, 'WIDE_IN', 0)
    w = wk.cfg1(0)
    gg = wk.mlp_gg(w['layers'], DEV)
    spec = LinearSpec(w['xl'], w['xh'], [[('pair', 1, 0)]])
    st = wk.reference_bab_settings(input_split_batch_size=2048, input_split_crown_intermediate=True,
                                   disable_sat_finding=True, total_timeout=600.0)
    return bab._input_split_batched(None, spec, st, gg, DEV, torch.float32)


def test_wide_step_kernel_reproduces_reference_leaf_count(monkeypatch):
    """The wide step kernel on cfg1 (forced for n_in = 5) gives the
    reference's verdict and leaf count."""
    g = load_golden('bab_cfg1_seed0')
    verdict, det = _cfg1_run(monkeypatch, True)
    assert verdict == str(g['verdict_ci1'])
    assert det['batched_n_leaves'] == int(g['n_leaves_ci1'])


def test_wide_step_matches_small_kernel_on_random_batches(monkeypatch):
    rng = np.random.default_rng(3)
    B, n, Q, D = 300, 40, 6, 3
    xl = rng.uniform(-1, 0, (B, n)).astype(np.float32)
    xh = (xl + rng.uniform(0.0, 1.0, (B, n))).astype(np.float32)
    xh[:5, 7] = xl[:5, 7]  # degenerate width on the split axis candidates
    lb = rng.normal(size=(B, Q)).astype(np.float32)
    A = rng.normal(size=(B, Q, n)).astype(np.float32)
    acc = rng.normal(size=(B, Q)).astype(np.float32) * 3
    qd = torch.as_tensor(np.arange(Q) % D, dtype=torch.int32, device=DEV)
    T = lambda a: torch.as_tensor(a, device=DEV)  # noqa: E731
    for clip in (True, False):
        for sb in (False, True):
            small = bab.bab_step(T(xl), T(xh), T(lb), T(A), T(acc), qd, D, clip, sb)
            monkeypatch.setattr(bab, 'WIDE_IN', 0)
            wide = bab.bab_step(T(xl), T(xh), T(lb), T(A), T(acc), qd, D, clip, sb)
            monkeypatch.setattr(bab, 'WIDE_IN', 64)
            cs, cw = small[4].tolist(), wide[4].tolist()
            assert cs == cw, (clip, sb, cs, cw)
            k = cs[2]
            for a, b in zip(small[:4], wide[:4]):
                np.testing.assert_allclose(a[:k].cpu().numpy(), b[:k].cpu().numpy(),
                                           rtol=1e-5, atol=1e-6)


def test_wide_engine_bab_matches_oracle():
    """An MLP outside the shared-memory kernels (80 -> [200] x 3 -> 5) with
    zonotope intermediates: verdict and leaf count against the oracle's BaB
    on the same property."""
    rng = np.random.default_rng(11)
    dims = (80, 200, 200, 200, 5)
    layers = wk.mlp_params(dims, rng)
    x0 = rng.uniform(-0.5, 0.5, dims[0])
    xl = (x0 - 0.003).astype(np.float32)
    xh = (x0 + 0.003).astype(np.float32)
    pts = xl + (xh - xl) * np.random.default_rng(5).random((4096, dims[0]))
    y = wk._mlp_forward64(layers, pts)
    d = float((y[:, 0] - y[:, 1]).max()) + 0.05  # oracle: verified, ~5.7k leaves
    W_last, b_last = layers[-1]
    b_last = b_last.copy()
    b_last[0] = np.float32(b_last[0] - d)
    layers = layers[:-1] + [(W_last, b_last)]
    spec_W = np.zeros((1, 5), np.float32)
    spec_W[0, 1], spec_W[0, 0] = 1.0, -1.0
    ref_v, ref_d = obab.input_split_bab(wk.mlp_gg(layers), xl, xh, spec_W, np.zeros(1, np.float32),
                                        batch_size=256, crown_intermediate=False, timeout=120.0)
    gg = wk.mlp_gg(layers, DEV)
    spec = LinearSpec(xl, xh, [[('pair', 1, 0)]])
    st = wk.reference_bab_settings(input_split_batch_size=256, disable_sat_finding=True,
                                   total_timeout=600.0)
    eng = bab.make_engine(spec, gg, st, DEV)
    assert isinstance(eng, bab.WideBoundEngine)
    verdict, det = bab._input_split_batched(None, spec, st, gg, DEV, torch.float32)
    print('wide BaB', verdict, det.get('batched_n_leaves'), 'oracle', ref_v,
          ref_d.get('batched_n_leaves'))
    assert verdict == ref_v
    assert ref_d['batched_n_leaves'] > 1000
    assert det['batched_n_leaves'] == ref_d['batched_n_leaves']
