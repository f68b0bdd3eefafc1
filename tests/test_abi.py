"""CPU checks of the C ABI and the host-side lowering (no GPU compute)."""
import ctypes
import os
import re

import numpy as np
import pytest
import torch

from vibecheck_nn_b200 import _lib, netdesc, workloads as wk

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def header_functions():
    src = open(os.path.join(ROOT, 'include', 'vcb.h')).read()
    src = re.sub(r'/\*.*?\*/', '', src, flags=re.S)
    return sorted(set(re.findall(
        r'^\s*(?:int|const char\*|size_t)\s+(vcb_\w+)\s*\(', src, flags=re.M)))


def test_library_builds_and_loads():
    from vibecheck_nn_b200 import build
    build.build()
    lib = _lib.lib()
    assert lib.vcb_version() >= 100


def test_exports_every_header_symbol():
    lib = ctypes.CDLL(_lib.LIB_PATH)
    names = header_functions()
    assert 'vcb_mlp_crown' in names
    for name in names:
        assert hasattr(lib, name), name
        assert name in _lib.SIGNATURES, f'{name} missing from _lib.SIGNATURES'


def test_invalid_arguments_return_status_not_crash():
    lib = _lib.lib()
    rc = lib.vcb_mlp_crown(None, 4, None, None, None, None, None, None, None,
                           None, 1, None, None, None, None, None, None, None,
                           None, 0, None)
    assert rc == _lib.VCB_ERR_INVALID
    assert 'NULL' in _lib.last_error()
    with pytest.raises(ValueError):
        _lib.check(rc, 'x')
    s = _lib.VcbMlp()
    s.n_fc = 0
    rc = lib.vcb_mlp_crown(ctypes.byref(s), 4, None, None, None, None, None,
                           None, None, None, 1, None, None, None, None, None,
                           None, None, None, 0, None)
    assert rc == _lib.VCB_ERR_INVALID  # NULL weights are caught first
    assert lib.vcb_mlp_crown_workspace(ctypes.byref(s), 4, 1) == 0
    # non-NULL (never dereferenced) pointers: the n_fc check rejects it first
    s.W = s.b = 16
    fake = ctypes.c_void_p(16)
    rc = lib.vcb_mlp_crown(ctypes.byref(s), 4, fake, fake, None, None, None,
                           None, None, None, 0, None, None, None, None, None,
                           None, None, None, 0, None)
    assert rc == _lib.VCB_ERR_UNSUPPORTED
    with pytest.raises(NotImplementedError):
        _lib.check(rc, 'x')
    rc = lib.vcb_probe_ffma(None, 0, 0, None)
    assert rc == _lib.VCB_ERR_INVALID


def test_status_mapping():
    with pytest.raises(torch.cuda.OutOfMemoryError):
        _lib.check(_lib.VCB_ERR_OOM)
    with pytest.raises(_lib.KernelError):
        _lib.check(_lib.VCB_ERR_CUDA)
    with pytest.raises(TimeoutError):
        _lib.check(_lib.VCB_ERR_TIMEOUT)


def test_lower_mlp_chain_and_folding():
    rng = np.random.default_rng(0)
    layers = wk.mlp_params((4, 6, 3), rng)
    gg = wk.mlp_gg(layers)
    out = netdesc.lower_mlp(gg)
    assert len(out) == 2
    np.testing.assert_array_equal(out[0][0], layers[0][0].astype(np.float64))
    # add-bias after the last fc folds into its bias
    gg['ops'].append({'name': 'badd', 'type': 'add', 'inputs': ['fc1'],
                      'is_merge': False, 'bias': np.ones(3)})
    out = netdesc.lower_mlp(gg)
    np.testing.assert_allclose(out[1][1], layers[1][1].astype(np.float64) + 1)


def test_lower_rejects_unsupported():
    rng = np.random.default_rng(0)
    gg = wk.mlp_gg(wk.mlp_params((4, 6, 3), rng))
    gg['ops'].insert(1, {'name': 'sg', 'type': 'sigmoid', 'inputs': ['fc0']})
    with pytest.raises(NotImplementedError):
        netdesc.lower_mlp(gg)


def test_cpu_device_is_refused():
    from vibecheck_nn_b200 import ops
    gg = wk.mlp_gg(wk.mlp_params((4, 6, 3), np.random.default_rng(0)))
    with pytest.raises(_lib.UnsupportedInput):
        ops._ibp_forward_graph_batched(torch.zeros(2, 4), torch.ones(2, 4), gg,
                                       'cpu', torch.float32)


def test_install_rebinds_reference_functions():
    import types
    from vibecheck_nn_b200 import install, ops, bab, pgd
    mods = {name: types.ModuleType(name) for name in install.BINDINGS}
    done = install.install(mods)
    assert mods['vibecheck.verify_zono_bnb']._spec_backward_graph_batched is \
        ops._spec_backward_graph_batched
    assert mods['vibecheck.verify_graph']._input_split_batched is bab._input_split_batched
    assert mods['vibecheck.verify_hybrid_acasxu']._simple_pgd_batched is pgd._simple_pgd_batched
    assert mods['vibecheck.pgd'].pgd_attack_general is pgd.pgd_attack_general
    assert sum(len(v) for v in done.values()) == 16


def test_install_relu_bab_delegates_and_is_optional():
    import types
    from vibecheck_nn_b200 import install, relu_bab
    mods = {name: types.ModuleType(name) for name in install.BINDINGS}
    mods['vibecheck.verify_milp']._ibp_crown_bab = lambda *a, **k: 'reference'
    install.install(mods)
    fn = mods['vibecheck.verify_milp']._ibp_crown_bab
    assert fn.__wrapped__ is relu_bab._ibp_crown_bab
    # CPU and float64 calls are the reference's
    assert fn(None, None, None, {}, None, 0.0, 'cpu', torch.float32, time_left=None) == 'reference'
    assert fn(None, None, None, {}, None, 0.0, 'cuda', torch.float64, time_left=None) == 'reference'
    # without the optional module (it needs a MILP solver) the rest still binds
    del mods['vibecheck.verify_milp']
    done = install.install(mods)
    assert 'vibecheck.verify_milp' not in done and len(done) == len(install.BINDINGS) - 1


def test_install_forward_delegates_outside_the_kernels():
    import types
    from vibecheck_nn_b200 import install, forward
    calls = []
    mod = types.ModuleType('vibecheck.verify_zono_bnb')
    mod._forward_batch_graph = lambda x, gg, capture=None: calls.append(x) or 'reference'
    mods = {name: types.ModuleType(name) for name in install.BINDINGS}
    mods['vibecheck.verify_zono_bnb'] = mod
    install.install(mods)
    fn = mod._forward_batch_graph
    assert fn.__wrapped__ is forward._forward_batch_graph
    # a CPU tensor is outside the kernels: the reference's function answers
    assert fn(torch.zeros(2, 3), {}) == 'reference' and len(calls) == 1
