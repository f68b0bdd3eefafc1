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


def test_clip_input_domain_is_sound_and_shrinks():
    g = torch.Generator(device=DEV).manual_seed(0)
    B, S, K = 64, 3, 4
    xl = torch.rand((B, K), generator=g, device=DEV)
    xh = xl + torch.rand((B, K), generator=g, device=DEV)
    lA = torch.randn((B, S, K), generator=g, device=DEV)
    lb = torch.randn((B, S), generator=g, device=DEV)
    cl, ch = multisub._clip_input_domain(xl, xh, lA, lb, num_iters=2)
    assert (cl >= xl).all() and (ch <= xh).all()
    # every removed point is verified by some query (its linear bound >= 0)
    pts = xl[:, None] + (xh - xl)[:, None] * torch.rand((B, 512, K), generator=g, device=DEV)
    inside = ((pts >= cl[:, None]) & (pts <= ch[:, None])).all(-1)
    val = torch.einsum('bsk,bpk->bps', lA, pts) + lb[:, None]
    assert (val[~inside].max(dim=-1).values >= -1e-4).all()
