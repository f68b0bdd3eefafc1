"""Front end: the ONNX reader and the float64 witness replay (CPU).

The reader is pinned to tests/golden/acasxu.npz, made by make_golden.py from
the reference's bundled ACAS Xu example: the same op sequence as the
reference's loader produces (sub, reshape, then fc / add / relu) and the
same fc weights.  The reference's own prop_2 witness must pass the replay.
"""
import ast
import os

import numpy as np
import pytest
import torch

from conftest import ROOT, golden_layers, load_golden
from vibecheck_nn_b200 import bab, frontend, netdesc, onnx_graph, workloads as wk

REF = os.environ.get('VIBECHECK_REF_SRC', os.path.join(os.path.dirname(ROOT), 'reference', 'src'))
ONNX = os.path.join(os.path.dirname(REF), 'examples', 'ACASXU_run2a_2_2_batch_2000.onnx')


@pytest.mark.skipif(not os.path.exists(ONNX), reason='no reference checkout')
def test_reader_matches_fixture():
    g = load_golden('acasxu')
    graph = onnx_graph.read_onnx(ONNX)
    assert graph.input_shape == (1, 1, 1, 5) and len(graph.nodes) == 22
    gg = graph.to_gg('cpu', torch.float32)
    assert ' '.join(op['type'] for op in gg['ops']) == str(g['op_types'])
    for (W, b), (W2, b2) in zip(netdesc.lower_mlp(gg), golden_layers(g)):
        assert np.array_equal(W.astype(np.float32), W2) and np.array_equal(b.astype(np.float32), b2)
    x = np.random.default_rng(0).uniform(-0.5, 0.5, 5)
    assert np.allclose(graph.forward64(x), wk._mlp_forward64(netdesc.lower_mlp(gg), x[None])[0],
                       rtol=0, atol=1e-12)


def test_reader_decodes_bytes_and_structure():
    """A rebuilt graph of the same structure lowers to the same layers."""
    g = load_golden('acasxu')
    layers = golden_layers(g)
    graph = wk.onnx_mlp_graph(layers, (1, 1, 1, 5))
    gg = graph.to_gg('cpu', torch.float32)
    assert ' '.join(op['type'] for op in gg['ops']) == str(g['op_types'])
    low = netdesc.lower_mlp(gg)
    assert all(np.array_equal(W.astype(np.float32), W2) for (W, _), (W2, _) in zip(low, layers))


def _spec(g, prop):
    p = f'p{prop}_'
    return bab.LinearSpec(g[p + 'x_lo'], g[p + 'x_hi'], ast.literal_eval(str(g[p + 'disj'])))


def test_spec_queries_are_the_reference_parse():
    """The tuple form of each property gives the linear queries the
    reference's VNNSpec gave (safe iff w . y + b > 0)."""
    g = load_golden('acasxu')
    for prop in (1, 2):
        p = f'p{prop}_'
        q = _spec(g, prop).as_linear_queries(5)
        assert [d for d, _, _ in q] == list(g[p + 'qd'])
        assert np.array_equal(np.stack([w for _, w, _ in q]), g[p + 'qw'])
        assert np.array_equal(np.array([b for _, _, b in q]), g[p + 'qb'])


def test_reference_witness_replays():
    g = load_golden('acasxu')
    graph = wk.onnx_mlp_graph(golden_layers(g), (1, 1, 1, 5))
    spec = _spec(g, 2)
    ok, info = frontend.witness_violates(graph, spec, g['p2_witness'])
    assert ok and info['worst_margin'] <= 0, info
    # the centre of prop_1's box is not a counterexample of prop_1 (it holds)
    ok1, _ = frontend.witness_violates(graph, _spec(g, 1), (g['p1_x_lo'] + g['p1_x_hi']) / 2)
    assert not ok1
    # outside the box beyond the tolerance
    ok2, info2 = frontend.witness_violates(graph, spec, g['p2_witness'] + 1.0)
    assert not ok2 and 'outside' in info2['reason']
