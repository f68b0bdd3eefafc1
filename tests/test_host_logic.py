"""CPU tests of host-side logic that needs no kernel: PGD bookkeeping,
spec conversion, cfg5 leaf generation, graph lowering and bias folding."""
import types

import numpy as np
import pytest
import torch

from vibecheck_nn_b200 import bab, graph, pgd, workloads as wk


def _order_code(f):
    u = int(np.array([f], np.float32).view(np.uint32)[0])
    return (~u & 0xFFFFFFFF) if u & 0x80000000 else (u | 0x80000000)


def test_order_code_round_trip_and_monotone():
    vals = [-3e38, -2.5, -1e-30, -0.0, 0.0, 1e-30, 1.0, 7.5, 3e38]
    codes = [_order_code(v) for v in vals]
    assert codes == sorted(codes)
    for v, c in zip(vals, codes):
        assert pgd._decode_min(c) == np.float32(v)
    assert np.isnan(pgd._decode_min(0xFFFFFFFF))  # the "no margin recorded" code


def test_bias_correction_tables_round_like_a_gpu_scalar_divisor():
    inv1, inv2 = pgd._bc_tables(5, 'cpu')
    for t in range(1, 6):
        bc1 = np.float32(1.0 - 0.9 ** t)
        assert inv1[t - 1].item() == np.float32(np.float32(1.0) / bc1)
        sb2 = np.float32((1.0 - 0.999 ** t) ** 0.5)
        assert inv2[t - 1].item() == np.float32(np.float32(1.0) / sb2)


def test_disjunct_tuples_from_reference_style_spec():
    Pw = types.SimpleNamespace
    spec = Pw(disjuncts=[Pw(constraints=[Pw(pred=2, comp=0, strict=False)]),
                         Pw(constraints=[Pw(index=1, op='>=', value=0.5),
                                         Pw(index=3, op='<=', value=-1.0)])])
    assert pgd._disjunct_tuples(spec) == [[('pair', 2, 0)], [('ge', 1, 0.5), ('le', 3, -1.0)]]
    bad = Pw(disjuncts=[Pw(constraints=[Pw(index=0, op='==', value=0.0)])])
    assert pgd._disjunct_tuples(bad) is None
    rows, bs, dis = pgd._rows_of([[('pair', 2, 0)], [('ge', 1, 0.5)]], 4)
    np.testing.assert_array_equal(rows[0], [-1, 0, 1, 0])
    np.testing.assert_array_equal(rows[1], [0, -1, 0, 0])
    assert bs == [0.0, 0.5] and dis == [0, 1]


def test_box_expand_is_capped_by_the_validation_tolerance():
    st = types.SimpleNamespace(pgd_input_box_expand=1e-5, sat_validate_atol=1e-4)
    lo, hi = pgd.expand_search_box(np.zeros(2), np.ones(2), st)
    np.testing.assert_allclose(lo, -1e-5)
    np.testing.assert_allclose(hi, 1 + 1e-5)
    with pytest.raises(AssertionError):
        pgd.pgd_box_expand_amount(types.SimpleNamespace(pgd_input_box_expand=1e-3,
                                                        sat_validate_atol=1e-4))


def test_cfg5_leaves_partition_the_box():
    rng = np.random.default_rng(0)
    xl = rng.uniform(0, 1, 64).astype(np.float32)
    xh = (xl + rng.uniform(0.5, 1.0, 64)).astype(np.float32)
    xh[5] = xl[5] + 2.0  # the widest dimension is split first
    dims = wk.cfg5_split_dims(xl, xh, depth=6)
    assert dims[0] == 5 and dims[1] == 5  # still the widest after one halving
    lo, hi = wk.cfg5_leaves(xl, xh, 0, 64, depth=6)
    assert np.all(lo >= xl) and np.all(hi <= xh) and np.all(lo < hi)
    vol = np.prod((hi - lo).astype(np.float64), axis=1).sum()
    assert np.isclose(vol, np.prod((xh - xl).astype(np.float64)), rtol=1e-5)
    centres = (lo + hi) / 2
    assert len({tuple(c) for c in centres}) == 64


def test_robustness_disjuncts():
    assert wk.robustness_disjuncts(4, 2) == [[('pair', 2, 0)], [('pair', 2, 1)], [('pair', 2, 3)]]


def test_graph_folds_bias_ops_and_tracks_names():
    rng = np.random.default_rng(1)
    layers = wk.mlp_params((6, 8, 3), rng)
    gg = wk.mlp_gg(layers)
    ops = gg['ops']
    fc0 = ops[0]['name']
    ops.insert(1, {'name': 'badd', 'type': 'add', 'inputs': [fc0],
                   'bias': torch.full((8,), 0.25)})
    ops[2]['inputs'] = ['badd']
    ops.append({'name': 'flat', 'type': 'reshape', 'inputs': [ops[-1]['name']]})
    G = graph.GraphNet(gg, torch.device('cpu'))
    fc = [L for L in G.layers if L['type'] == 'fc']
    np.testing.assert_allclose(fc[0]['b'].numpy(), layers[0][1] + 0.25, rtol=1e-6)
    np.testing.assert_allclose(fc[0]['Waug'][:, 6].numpy(), layers[0][1] + 0.25, rtol=1e-6)
    assert G.layer_of('badd') == 0
    assert G.layer_of('flat') == len(G.layers) - 1
    assert G.layer_of(gg['input_name']) == -1
    with pytest.raises(NotImplementedError):
        G.layer_of(fc0)  # its own output no longer exists after folding
    ops.insert(2, {'name': 'bcast', 'type': 'add', 'inputs': ['badd'],
                   'bias': torch.zeros(3)})  # neither scalar nor per-output
    ops[3]['inputs'] = ['bcast']
    with pytest.raises(NotImplementedError):
        graph.GraphNet(gg, torch.device('cpu'))


def test_dedup_queries_replicates_shared_halfspaces_per_disjunct():
    spec = bab.LinearSpec(np.zeros(2), np.ones(2),
                          [[('pair', 0, 1), ('ge', 2, 1.0)], [('pair', 0, 1)]])
    W, b, qd, D, q_sens = bab.dedup_queries(spec.as_linear_queries(3), 'cpu')
    assert D == 2 and q_sens == 2
    assert W.shape[0] == 3  # the shared pair is replicated for disjunct 1
    assert qd.tolist() == [0, 0, 1]
    np.testing.assert_array_equal(W[2].numpy(), W[0].numpy())


def test_engine_choice_by_input_width():
    assert bab.WIDE_IN == 64
