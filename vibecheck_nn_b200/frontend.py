"""Front end around the input-split BaB: ONNX network and VNN-LIB property in,
validated verdict out.

The ``vibecheck verify`` path of the reference (main.py -> verify_graph ->
``_input_split_batched``, verify_graph.py:9947) on the B200 kernels, for
fc / ReLU networks:

* ``load_network`` parses the ONNX file without the ``onnx`` package
  (``onnx_graph.read_onnx``) and builds the reference's ``gg`` op dict;
* ``load_spec`` parses the property with the reference's own
  ``vibecheck.vnnlib_loader.load_vnnlib`` when the reference is importable
  (``bab.LinearSpec`` carries an already-parsed property);
* ``verify`` runs the batched driver under the given settings and replays a
  SAT witness through the network in float64 (``OnnxGraph.forward64``), in
  place of the reference's onnxruntime replay (verify_graph.py:5423-5467,
  :9987-10012): the witness must lie in the input box up to ``atol`` and its
  output must satisfy every constraint of some disjunct of the unsafe region
  (w . y + b <= 0 for each of its queries); otherwise the verdict becomes
  ``unknown`` with phase ``spurious_sat_<phase>``, as in the reference.
"""
from __future__ import annotations

import numpy as np
import torch

from . import bab
from .onnx_graph import read_onnx


def load_network(path, device='cuda', dtype=torch.float32):
    """(OnnxGraph, gg) of an ONNX file (.onnx or .onnx.gz)."""
    g = read_onnx(path)
    return g, g.to_gg(torch.device(device), dtype)


def load_spec(path):
    """The reference's VNNSpec of a VNN-LIB file (needs the reference package
    importable as ``vibecheck``)."""
    from vibecheck.vnnlib_loader import load_vnnlib
    return load_vnnlib(str(path))


def witness_violates(graph, spec, witness, atol=1e-4):
    """(ok, info): the witness lies in the input box (within atol) and the
    network's float64 output satisfies every query of some disjunct of the
    unsafe region."""
    x = np.asarray(witness, np.float64).reshape(-1)
    lo, hi = spec.x_lo.reshape(-1), spec.x_hi.reshape(-1)
    info = {'max_box_violation': float(max(0.0, np.max(lo - x), np.max(x - hi)))}
    if info['max_box_violation'] > atol:
        info['reason'] = 'witness outside the input box'
        return False, info
    y = graph.forward64(x)
    info['output'] = y
    margins = {}
    for d, w, b in spec.as_linear_queries(y.size):
        m = float(np.dot(np.asarray(w, np.float64).reshape(-1), y) + b)
        margins[d] = max(margins.get(d, -np.inf), m)
    info['worst_margin'] = min(margins.values()) if margins else None
    ok = any(m <= 0.0 for m in margins.values())
    if not ok:
        info['reason'] = 'float64 replay does not violate the property'
    return ok, info


def verify(graph, gg, spec, settings, device='cuda', atol=1e-4):
    """Verdict and details of the batched input-split BaB on the B200
    kernels, with the SAT witness replayed in float64."""
    verdict, details = bab._input_split_batched(None, spec, settings, gg, device,
                                                torch.float32)
    if verdict == 'sat' and details.get('witness') is not None:
        ok, info = witness_violates(graph, spec, details['witness'], atol)
        details['witness_check'] = info
        if not ok:
            details['spurious_witness'] = info
            details['original_phase'] = details.get('phase')
            details['phase'] = f'spurious_sat_{details.get("phase")}'
            verdict = 'unknown'
    return verdict, details
