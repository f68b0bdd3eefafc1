"""The reference's bundled ACAS Xu example end to end on the GPU
(README.md:40-75): examples/prop_1 is verified with the reference's leaves
and iterations under configs/acasxu_2023.yaml, examples/prop_2 is sat with a
witness the float64 replay confirms.  The network is rebuilt from the
weights in tests/golden/acasxu.npz in the structure of the ONNX export
(test_frontend.py pins the reader to the same weights)."""
import ast

import numpy as np
import pytest
import torch

from conftest import golden_layers, load_golden
from vibecheck_nn_b200 import bab, frontend, workloads as wk

pytestmark = pytest.mark.gpu
DEV = torch.device('cuda:0') if torch.cuda.is_available() else None


def _case(prop):
    g = load_golden('acasxu')
    graph = wk.onnx_mlp_graph(golden_layers(g), (1, 1, 1, 5))
    gg = graph.to_gg(DEV, torch.float32)
    p = f'p{prop}_'
    spec = bab.LinearSpec(g[p + 'x_lo'], g[p + 'x_hi'], ast.literal_eval(str(g[p + 'disj'])))
    st = wk.reference_bab_settings(total_timeout=60.0, **wk.ACASXU_2023)
    return g, p, graph, gg, spec, st


def test_prop_1_verified_like_the_reference():
    g, p, graph, gg, spec, st = _case(1)
    verdict, det = frontend.verify(graph, gg, spec, st, DEV)
    assert verdict == str(g[p + 'verdict']) == 'verified', det
    assert det['batched_n_leaves'] == int(g[p + 'n_leaves']), det
    assert det['batched_n_iters'] == int(g[p + 'n_iters']), det


def test_prop_2_sat_with_a_replayed_witness():
    g, p, graph, gg, spec, st = _case(2)
    verdict, det = frontend.verify(graph, gg, spec, st, DEV)
    assert verdict == str(g[p + 'verdict']) == 'sat', det
    assert det['witness_check']['worst_margin'] <= 0
    w = np.asarray(det['witness'], np.float64)
    assert (w >= g[p + 'x_lo'] - 1e-4).all() and (w <= g[p + 'x_hi'] + 1e-4).all()
