"""CPU tests of the host logic of the next-row drivers: the input-domain clip
and sub-box query extraction of the multi-subbox BaB (verify_graph.py:
11121-11177, 11205-11215), the min-area slope and layer seeds of the
freeze-replay hybrid (verify_hybrid_acasxu.py:186-199), and the split clamps
of the ReLU-split BaB (verify_milp.py:2738-2752)."""
import types

import numpy as np
import torch

from oracle import multisub as oms
from vibecheck_nn_b200 import hybrid, multisub, relu_bab


def test_clip_input_domain_sound_and_shrinking():
    rng = np.random.default_rng(0)
    B, S, K = 64, 3, 4
    xl = rng.random((B, K), np.float32)
    xh = xl + rng.random((B, K), np.float32)
    lA = rng.standard_normal((B, S, K)).astype(np.float32)
    lb = rng.standard_normal((B, S)).astype(np.float32)
    cl, ch = oms.clip_input_domain(xl, xh, lA, lb, num_iters=2)
    assert (cl >= xl).all() and (ch <= xh).all()
    assert ((cl > xl) | (ch < xh)).any()
    pts = xl[:, None] + (xh - xl)[:, None] * rng.random((B, 512, K))
    inside = ((pts >= cl[:, None]) & (pts <= ch[:, None])).all(-1)
    val = np.einsum('bsk,bpk->bps', lA, pts) + lb[:, None]
    # every removed point is verified by some query
    assert (val[~inside].max(axis=-1) >= -1e-4).all()


def test_clip_input_domain_one_dimension_closed_form():
    # bound 2 x - 1 >= 0 on [0, 1]: x >= 0.5 is verified, so x_U drops to 0.5
    cl, ch = oms.clip_input_domain([[0.0]], [[1.0]], [[[2.0]]], [[-1.0]])
    assert float(cl[0, 0]) == 0.0 and float(ch[0, 0]) == 0.5


def test_multisub_leaf_fate_and_children_oracle():
    """Fates of a hand-made batch: one leaf safe by its margin, one whose
    clip empties the box, one split on the higher-scoring dimension."""
    xl = np.zeros((3, 3), np.float32)
    xh = np.array([[1, 1, 0], [1, 1, 0], [1, 2, 0]], np.float32)
    var = np.array([0, 1])
    # leaf 1: x0 <= 0.6 and x0 >= 0.4 are each verified by one query
    A = np.array([[[1, 0], [0, 0]], [[-1, 0], [1, 0]], [[1, 1], [0, 0]]], np.float32)
    sb = np.array([[0.5, -5], [0.6, -0.4], [-3, -5]], np.float32)
    lb = np.array([[0.5, -5], [-0.4, -0.4], [-3, -5]], np.float32)
    fate, lo, hi, sc = oms.leaf_fate(xl, xh, var, A, sb, lb, np.zeros((1, 2), np.float32),
                                     np.zeros(3, np.int64))
    assert fate.tolist() == [0, 1, 2, 2]
    # leaf 2: x0 + x1 - 3 >= 0 nowhere inside [0,1] x [0,2]
    assert lo[2].tolist() == [0, 0, 0] and hi[2].tolist() == [1, 2, 0]
    assert sc[2].tolist() == [-2.5, -2.0, -np.inf]  # 1 * width / 2 - 3
    kxl, kxh, ks = oms.emit_children([2], lo, hi, sc, np.array([0, 0, 5]), 2)
    assert ks.tolist() == [5] * 4
    assert kxl.tolist() == [[0, 0, 0], [0, 1, 0], [0.5, 0, 0], [0.5, 1, 0]]
    assert kxh.tolist() == [[0.5, 1, 0], [0.5, 2, 0], [1, 1, 0], [1, 2, 0]]


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
    W_q, b_q = hybrid._seed_rows(3, 'cpu')
    assert W_q.shape == (6, 3) and float(b_q.abs().sum()) == 0
    assert torch.equal(W_q[:3], torch.eye(3)) and torch.equal(W_q[3:], -torch.eye(3))
    # seeded bounds intersect into the layer's box, lower never above upper
    old = (torch.tensor([[-1.0, 0.0]]), torch.tensor([[1.0, 2.0]]))
    lo, hi = hybrid._intersect(old, torch.tensor([[-0.5, 3.0, -0.5, -1.0]]), 2)
    assert lo.tolist() == [[-0.5, 1.0]] and hi.tolist() == [[0.5, 1.0]]


def test_hybrid_fan_out_order():
    """Widest-dimension bisection, children low then high, rounds in order."""
    lo, hi = hybrid._fan_out(np.zeros(2, np.float32), np.array([4, 2], np.float32), 4)
    # [0,4]x[0,2] -> x0 at 2; then both halves are square: first max, x0
    assert lo.tolist() == [[0, 0], [1, 0], [2, 0], [3, 0]]
    assert hi.tolist() == [[1, 2], [2, 2], [3, 2], [4, 2]]
    lo3, _ = hybrid._fan_out(np.zeros(2, np.float32), np.array([4, 2], np.float32), 3)
    assert lo3.tolist() == [[0, 0], [1, 0], [2, 0]]  # the reference drops the rest


def test_relu_split_clamp_tensors():
    doms = [{(0, 1): 0}, {(0, 1): 1, (1, 0): 0}]
    out = relu_bab._clamp_tensors(doms, {0: 3, 1: 2}, 2, 'cpu', torch.float32)
    cl0, ch0 = out[0]
    assert ch0[0, 1] == 0 and cl0[0, 1] == -np.inf   # OFF: z <= 0
    assert cl0[1, 1] == 0 and ch0[1, 1] == np.inf    # ON: z >= 0
    assert out[1][1][1, 0] == 0 and set(out) == {0, 1}
