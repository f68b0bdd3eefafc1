"""GPU parity of the multi-subbox input-split BaB (verify_graph.py:11180-11922)
and its forward-LiRPA bound (forward_lirpa.py:443-687) against outputs
recorded from the reference on CPU (tests/golden/make_golden.py --only
multisub): closed sub-boxes, iterations and visited leaves, and the linear
output bounds of the first network."""
import types

import numpy as np
import pytest
import torch

from conftest import close, golden_script, load_golden, max_excess
from vibecheck_nn_b200 import multisub, netdesc, workloads as wk

pytestmark = pytest.mark.gpu
DEV = torch.device('cuda:0') if torch.cuda.is_available() else None
G = load_golden('multisub')
CASES = {c[0]: c for c in golden_script().MULTISUB_CASES}


@pytest.mark.parametrize('tag', [str(t) for t in G['tags']])
def test_multi_sub_bab_matches_reference(tag):
    _, seed, n_sub, margins, half, batch, depth, budget = CASES[tag]
    layers, subs = golden_script().multisub_problem(seed, n_sub, margins, half)
    gg = wk.mlp_gg(layers, DEV, torch.float32)
    groups = [(lo.astype(np.float64), hi.astype(np.float64), conj) for lo, hi, conj in subs]
    st = types.SimpleNamespace(input_split_batch_size=batch, bab_split_depth=depth)
    closed = multisub._multi_sub_input_split_bab(list(range(len(groups))), groups,
                                                 list(range(len(groups))), gg, DEV,
                                                 torch.float32, budget, 2, st)
    assert sorted(closed) == G[f'{tag}_closed'].tolist()
    if tag != 'unsafe':  # the unsafe case runs until its time budget
        assert multisub.last_stats['iters'] == int(G[f'{tag}_iters'])
        assert multisub.last_stats['leaves'] == int(G[f'{tag}_leaves'])


def test_forward_linear_bounds_match_reference():
    _, seed, n_sub, margins, half = CASES['mixed'][:5]
    layers, subs = golden_script().multisub_problem(seed, n_sub, margins, half)
    desc = netdesc.mlp_desc(wk.mlp_gg(layers, DEV, torch.float32), DEV)
    xl = torch.as_tensor(np.stack([s[0] for s in subs]), device=DEV)
    xh = torch.as_tensor(np.stack([s[1] for s in subs]), device=DEV)
    var_idx = torch.nonzero(torch.as_tensor(G['flirpa_mask'], device=DEV)).flatten().to(torch.int32)
    W_q = torch.eye(2, device=DEV)
    spec_A, spec_b, lb, A_lo, A_up, b_lo, b_up = multisub.forward_linear_spec(
        desc, xl, xh, var_idx, W_q, want_bounds=True)
    for k, v in (('A_lo', A_lo), ('A_up', A_up), ('b_lo', b_lo), ('b_up', b_up)):
        assert close(v.cpu().numpy(), G[f'flirpa_{k}']), (k, max_excess(v.cpu().numpy(),
                                                                           G[f'flirpa_{k}']))
    # identity spec rows: lb is the output lower box bound
    assert close(lb.cpu().numpy(), G['flirpa_lo_box']), max_excess(lb.cpu().numpy(),
                                                                   G['flirpa_lo_box'])
    # soundness on samples
    rng = np.random.default_rng(0)
    lo, hi = xl.cpu().numpy(), xh.cpu().numpy()
    pts = lo[:, None] + (hi - lo)[:, None] * rng.random((len(lo), 256, 6))
    y = wk._mlp_forward64(layers, pts.reshape(-1, 6)).reshape(len(lo), 256, 2)
    assert (lb.cpu().numpy()[:, None, :] <= y + 1e-5).all()


def _fate_problem(seed, B=512, n=8, Q=3, nsub=4):
    rng = np.random.default_rng(seed)
    var = np.array([0, 1, 3, 4, 6, 7])
    xl = rng.random((B, n), np.float32)
    xh = xl + rng.random((B, n), np.float32)
    xh[:, [2, 5]] = xl[:, [2, 5]]
    xh[::7, 1] = xl[::7, 1]  # a varying dimension that is degenerate in some leaves
    A = rng.standard_normal((B, Q, var.size)).astype(np.float32)
    sb = (rng.standard_normal((B, Q)) * 2 - 1).astype(np.float32)
    lb = sb.copy()
    for k, d in enumerate(var):
        a = A[:, :, k]
        lb += np.maximum(a, 0) * xl[:, None, d] + np.minimum(a, 0) * xh[:, None, d]
    bias = (rng.standard_normal((nsub, Q)) * 0.3).astype(np.float32)
    sub = rng.integers(0, nsub, B).astype(np.int32)
    return xl, xh, var, A, sb, lb, bias, sub


def _same(a, b):
    return np.array_equal(a.view(np.uint32), b.view(np.uint32))


@pytest.mark.parametrize('seed', [0, 1, 2])
def test_leaf_fate_and_children_match_the_oracle_bitwise(seed):
    """vcb_multisub_fate / vcb_multisub_emit against the numpy restatement
    of the reference's tensor expressions: fates, clipped boxes, scores and
    children bit for bit."""
    from oracle import multisub as oms
    prob = _fate_problem(seed)
    xl, xh, var, A, sb, lb, bias, sub = prob
    T = [torch.as_tensor(v, device=DEV) for v in prob]
    T[2] = T[2].to(torch.int32)
    fate, lo, hi, sc = multisub.leaf_fate(*T, clip_iters=2)
    fo, loo, hio, sco = oms.leaf_fate(*prob, clip_iters=2)
    fate = fate.cpu().numpy()
    assert fate.tolist() == fo.tolist()
    assert set(fo[:-1].tolist()) == {0, 1, 2}
    s = np.nonzero(fo[:-1] == 2)[0]
    for got, want in ((lo, loo), (hi, hio), (sc, sco)):
        assert _same(got.cpu().numpy()[s], want[s])
    for k in (1, 2, 3):
        rows = torch.as_tensor(s.astype(np.int32), device=DEV)
        kid = multisub.emit_children(rows, lo, hi, sc, T[7], k)
        want = oms.emit_children(s, loo, hio, sco, sub, k)
        for g, w in zip(kid, want):
            assert np.array_equal(g.cpu().numpy(), w), k


def test_fused_forward_fate_equals_the_two_calls():
    """vcb_mlp_flirpa_fate gives the fates, boxes and scores of
    vcb_mlp_flirpa followed by vcb_multisub_fate, bit for bit."""
    _, seed, n_sub, margins, half = CASES['mixed'][:5]
    layers, subs = golden_script().multisub_problem(seed, n_sub, margins, half)
    desc = netdesc.mlp_desc(wk.mlp_gg(layers, DEV, torch.float32), DEV)
    rng = np.random.default_rng(1)
    lo = np.concatenate([s[0] for s in subs for _ in range(8)]).reshape(-1, 6).astype(np.float32)
    hi = np.concatenate([s[1] for s in subs for _ in range(8)]).reshape(-1, 6).astype(np.float32)
    # widen the fixed dimensions 0-3, shrink some boxes, fix dimension 4
    lo[:, :4] -= 0.05 * rng.random((lo.shape[0], 4)).astype(np.float32)
    hi[:, :4] += 0.05 * rng.random((lo.shape[0], 4)).astype(np.float32)
    f = rng.random(lo.shape).astype(np.float32)
    hi = np.where(rng.random(lo.shape) < 0.5, lo + (hi - lo) * f, hi).astype(np.float32)
    hi[:, 4] = lo[:, 4]
    xl, xh = torch.as_tensor(lo, device=DEV), torch.as_tensor(hi, device=DEV)
    var_idx = torch.tensor([0, 1, 2, 3, 5], dtype=torch.int32, device=DEV)
    W_q = torch.tensor([[1.0, -1.0], [-1.0, 1.0]], device=DEV)
    bias = torch.as_tensor(rng.normal(0, 0.5, (n_sub, 2)).astype(np.float32), device=DEV)
    sub = torch.as_tensor(np.repeat(np.arange(n_sub), 8).astype(np.int32), device=DEV)
    fused = multisub.forward_fate(desc, xl, xh, var_idx, W_q, bias, sub, clip_iters=2)
    spec_A, spec_b, lb = multisub.forward_linear_spec(desc, xl, xh, var_idx, W_q)
    two = multisub.leaf_fate(xl, xh, var_idx, spec_A, spec_b, lb, bias, sub, clip_iters=2)
    f1, f2 = fused[0].cpu().numpy(), two[0].cpu().numpy()
    assert np.array_equal(f1, f2) and len(set(f1[:-1].tolist())) >= 2, np.bincount(f1[:-1])
    s = np.nonzero(f1[:-1] == 2)[0]
    for a, b in zip(fused[1:], two[1:]):
        assert _same(a.cpu().numpy()[s], b.cpu().numpy()[s])
