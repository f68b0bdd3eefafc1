"""Bind the B200 operators in place of vibecheck's batched bound kernels.

The reference driver imports its kernels at call time
(verify_graph.py:12485-12486, :12514-12515, :12858, :12937), so rebinding the
module attributes before ``verify_graph`` runs routes the input-split BaB
through this package.  ``verify_hybrid_acasxu`` binds its PGD helpers at
import (verify_hybrid_acasxu.py:31-34), so they are rebound there too; the
general PGD attack is rebound in ``vibecheck.pgd``, which the reference's
``_pgd_attack_general`` wrapper imports at call time; the MILP phase's
ReLU-split BaB is rebound in ``vibecheck.verify_milp`` when that module
imports (it needs gurobipy).
"""
from __future__ import annotations

import importlib

from . import _lib

BINDINGS = {
    'vibecheck.verify_zono_bnb': {
        '_ibp_forward_graph_batched': ('ops', '_ibp_forward_graph_batched'),
        '_spec_backward_graph_batched': ('ops', '_spec_backward_graph_batched'),
        '_forward_zonotope_graph_batched': ('interm', '_forward_zonotope_graph_batched'),
        '_crown_intermediate_batched': ('interm', '_crown_intermediate_batched'),
        '_run_alpha_crown_inputsplit_batched': ('alpha', '_run_alpha_crown_inputsplit_batched'),
        '_forward_batch_graph': ('forward', '_forward_batch_graph', 'delegate'),
    },
    'vibecheck.verify_graph': {
        # settings or graphs outside the B200 path (the Gurobi LP clip, MILP
        # escalation, CPU / float64) run the reference's own driver
        '_input_split_batched': ('bab', '_input_split_batched', 'delegate'),
        # per-disjunct sub-box verification calls it as a module global
        # (verify_graph.py:9337); CPU calls go to the reference's own
        '_multi_sub_input_split_bab': ('multisub', '_multi_sub_input_split_bab', 'delegate'),
    },
    'vibecheck.verify_hybrid_acasxu': {
        '_simple_pgd': ('pgd', '_simple_pgd'),
        '_simple_pgd_batched': ('pgd', '_simple_pgd_batched'),
        '_forward_batch_graph': ('forward', '_forward_batch_graph', 'delegate'),
        # the freeze-replay pipeline; verify_graph imports verify_hybrid at
        # call time (verify_graph.py:9890); networks other than fc / ReLU
        # MLPs run the reference's own
        '_full_freeze': ('hybrid', '_full_freeze', 'delegate'),
        '_replay_batched': ('hybrid', '_replay_batched', 'delegate'),
        'verify_hybrid': ('hybrid', 'verify_hybrid', 'delegate'),
    },
    # verify_milp._pgd_attack_general (verify_milp.py:111-124), which every
    # caller uses, looks this attribute up at call time
    'vibecheck.pgd': {
        'pgd_attack_general': ('pgd', 'pgd_attack_general'),
    },
    # the MILP phase calls its ReLU-split BaB through the module global
    # (verify_milp.py:3874); float64 or CPU calls go to the reference's own
    'vibecheck.verify_milp': {
        '_ibp_crown_bab': ('relu_bab', '_ibp_crown_bab', 'delegate'),
    },
}
# modules whose import needs an optional solver (verify_milp imports
# gurobipy): without it the phase that would call the binding cannot run
OPTIONAL = {'vibecheck.verify_milp'}


def _delegating(impl, original):
    """``impl`` for the inputs it supports; the reference's own function for
    the rest.  Used for the concrete forward, which the reference also calls
    off the hot path (CPU / float64 tensors, merge graphs, ND fc ops) where no
    caller catches NotImplementedError, and for the multi-subbox and
    ReLU-split drivers on CPU or float64 calls.  Only ``UnsupportedInput``
    (inputs outside the B200 path, raised before any kernel runs) hands the
    call over; a kernel failure (``KernelError``), a time-out or an
    out-of-memory error propagates to the caller unchanged."""
    if original is None:
        return impl

    def fn(*args, **kwargs):
        try:
            return impl(*args, **kwargs)
        except _lib.UnsupportedInput:
            return original(*args, **kwargs)
    fn.__wrapped__ = impl
    fn.__name__ = getattr(impl, '__name__', 'fn')
    return fn


def install(modules=None):
    """Rebind the reference's functions; returns {module: [names]} of what
    was rebound.  ``modules`` maps module names to already-imported module
    objects (default: import them)."""
    done = {}
    for mod_name, names in BINDINGS.items():
        mod = (modules or {}).get(mod_name)
        if mod is None:
            try:
                mod = importlib.import_module(mod_name)
            except ImportError:
                if mod_name in OPTIONAL:
                    continue
                raise
        for attr, spec in names.items():
            sub, fn = spec[0], spec[1]
            impl = getattr(importlib.import_module(f'{__package__}.{sub}'), fn)
            if len(spec) > 2 and spec[2] == 'delegate':
                impl = _delegating(impl, getattr(mod, attr, None))
            setattr(mod, attr, impl)
            done.setdefault(mod_name, []).append(attr)
    return done
