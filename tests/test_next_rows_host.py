"""CPU tests of the host logic of the next-row drivers: the input-domain clip
and sub-box query extraction of the multi-subbox BaB (verify_graph.py:
11121-11177, 11205-11215), the min-area slope and layer seeds of the
freeze-replay hybrid (verify_hybrid_acasxu.py:186-199), and the split clamps
of the ReLU-split BaB (verify_milp.py:2738-2752)."""
import types

import numpy as np
import torch

from vibecheck_nn_b200 import hybrid, multisub, relu_bab


def test_clip_input_domain_sound_and_shrinking():
    g = torch.Generator().manual_seed(0)
    B, S, K = 64, 3, 4
    xl = torch.rand((B, K), generator=g)
    xh = xl + torch.rand((B, K), generator=g)
    lA = torch.randn((B, S, K), generator=g)
    lb = torch.randn((B, S), generator=g)
    cl, ch = multisub._clip_input_domain(xl, xh, lA, lb, num_iters=2)
    assert (cl >= xl).all() and (ch <= xh).all()
    assert bool(((cl > xl) | (ch < xh)).any())
    pts = xl[:, None] + (xh - xl)[:, None] * torch.rand((B, 512, K), generator=g)
    inside = ((pts >= cl[:, None]) & (pts <= ch[:, None])).all(-1)
    val = torch.einsum('bsk,bpk->bps', lA, pts) + lb[:, None]
    # every removed point is verified by some query
    assert (val[~inside].max(dim=-1).values >= -1e-4).all()


def test_clip_input_domain_one_dimension_closed_form():
    # bound 2 x - 1 >= 0 on [0, 1]: x >= 0.5 is verified, so x_U drops to 0.5
    cl, ch = multisub._clip_input_domain(torch.tensor([[0.0]]), torch.tensor([[1.0]]),
                                         torch.tensor([[[2.0]]]), torch.tensor([[-1.0]]))
    assert float(cl) == 0.0 and abs(float(ch) - 0.5) < 1e-7


def test_sub_queries_from_tuples_and_reference_objects():
    lo, hi = np.zeros(3), np.ones(3)
    q = multisub._sub_queries((lo, hi, [[('ge', 0, 1.5), ('le', 1, -2.0)]]), 2)
    assert [(d, list(w), b) for d, w, b in q] == [(0, [-1.0, 0.0], 1.5), (0, [0.0, 1.0], 2.0)]
    cons = [types.SimpleNamespace(index=0, op='>=', value=1.5),
            types.SimpleNamespace(pred=1, comp=0)]
    q2 = multisub._sub_queries((lo, hi, [types.SimpleNamespace(constraints=cons)]), 2)
    assert [(d, list(w), b) for d, w, b in q2] == [(0, [-1.0, 0.0], 1.5), (0, [-1.0, 1.0], 0.0)]
    bad = [types.SimpleNamespace(index=0, op='==', value=1.0)]
    assert multisub._sub_queries((lo, hi, [types.SimpleNamespace(constraints=bad)]), 2) is None


def test_min_area_slope_and_layer_seeds():
    lo = torch.tensor([[-1.0, -1.0, 0.5, -2.0]])
    hi = torch.tensor([[3.0, 0.5, 1.0, -0.5]])
    # unstable with up_s 0.75 -> 1; unstable with up_s 1/3 -> 0; active / dead -> 0
    assert hybrid._min_area(lo, hi, torch.float32).tolist() == [[1.0, 0.0, 0.0, 0.0]]
    seed, acc = hybrid._layer_seeds(None, 3, 2, 'cpu', torch.float32)
    assert seed.shape == (2, 6, 3) and acc.shape == (2, 6) and float(acc.abs().sum()) == 0
    assert torch.equal(seed[1, :3], torch.eye(3)) and torch.equal(seed[0, 3:], -torch.eye(3))


def test_relu_split_clamp_tensors():
    doms = [{(0, 1): 0}, {(0, 1): 1, (1, 0): 0}]
    out = relu_bab._clamp_tensors(doms, {0: 3, 1: 2}, 2, 'cpu', torch.float32)
    cl0, ch0 = out[0]
    assert ch0[0, 1] == 0 and cl0[0, 1] == -np.inf   # OFF: z <= 0
    assert cl0[1, 1] == 0 and ch0[1, 1] == np.inf    # ON: z >= 0
    assert out[1][1][1, 0] == 0 and set(out) == {0, 1}
