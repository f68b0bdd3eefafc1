"""No silent fallbacks: a kernel failure propagates.

The library's status codes map to exception types (``_lib.check``); only
``UnsupportedInput`` (inputs outside the B200 path, refused before any kernel
runs) may hand a call to the reference's own function, and only an
out-of-memory error halves the BaB batch (main.py:89-99,
verify_graph.py:12872-12897).  These run on the CPU with a stand-in for the
loaded library whose compute entry points return a chosen status.
"""
import types

import numpy as np
import pytest
import torch

from vibecheck_nn_b200 import _lib, bab, install, ops, workloads as wk


class FakeLib:
    """libvcb stand-in: size queries answer, compute calls return OK except
    the ones named in ``fail``, which return ``status``."""

    def __init__(self, fail=(), status=_lib.VCB_ERR_CUDA):
        self.fail, self.status = set(fail), status
        self.calls = []

    def vcb_last_error(self):
        return b'injected status'

    def vcb_mlp_crown_workspace(self, *a):
        return 4096

    def vcb_mlp_crown_path(self, *a):
        return 0

    def vcb_mlp_zono_kmax(self, *a):
        return 16

    def __getattr__(self, name):
        def fn(*a):
            self.calls.append(name)
            return self.status if name in self.fail else _lib.VCB_OK
        return fn


@pytest.fixture
def fake(monkeypatch):
    def make(**kw):
        f = FakeLib(**kw)
        monkeypatch.setattr(_lib, '_lib', f)
        monkeypatch.setattr(_lib, 'stream_of', lambda device: None)
        monkeypatch.setattr(bab, '_dev', lambda device: torch.device('cpu'))
        return f
    return make


def _problem():
    layers = wk.mlp_params((3, 8, 8, 2), np.random.default_rng(0))
    gg = wk.mlp_gg(layers)
    spec = bab.LinearSpec(np.zeros(3), np.ones(3), [[('pair', 0, 1)]])
    settings = types.SimpleNamespace(input_split_batch_size=8, disable_sat_finding=True,
                                     input_split_crown_intermediate=False, raise_on_oom=False)
    return spec, gg, settings


def test_status_codes_map_to_distinct_exceptions():
    assert issubclass(_lib.KernelError, RuntimeError)
    assert issubclass(_lib.UnsupportedInput, NotImplementedError)
    with pytest.raises(_lib.KernelError):
        _lib.check(_lib.VCB_ERR_CUDA)
    with pytest.raises(_lib.UnsupportedInput):
        _lib.check(_lib.VCB_ERR_UNSUPPORTED)
    with pytest.raises(TimeoutError):
        _lib.check(_lib.VCB_ERR_TIMEOUT)


def test_kernel_error_propagates_out_of_the_bab_driver(fake):
    """A VCB_ERR_CUDA from the spec bound leaves _input_split_batched as a
    KernelError on the first iteration: no batch halving, no verdict."""
    f = fake(fail={'vcb_mlp_crown'})
    spec, gg, settings = _problem()
    with pytest.raises(_lib.KernelError):
        bab._input_split_batched(None, spec, settings, gg, 'cuda', torch.float32)
    assert f.calls.count('vcb_mlp_crown') == 1


def test_timeout_status_propagates_out_of_the_bab_driver(fake):
    f = fake(fail={'vcb_bab_step_ex'}, status=_lib.VCB_ERR_TIMEOUT)
    spec, gg, settings = _problem()
    with pytest.raises(TimeoutError):
        bab._input_split_batched(None, spec, settings, gg, 'cuda', torch.float32)
    assert f.calls.count('vcb_bab_step_ex') == 1


def test_out_of_memory_halves_the_batch(fake):
    """An OOM status halves the batch down to 1, then the driver reports
    batched_oom (raise_on_oom=False), as the reference does."""
    f = fake(fail={'vcb_mlp_crown'}, status=_lib.VCB_ERR_OOM)
    spec, gg, settings = _problem()
    verdict, details = bab._input_split_batched(None, spec, settings, gg, 'cuda',
                                                torch.float32)
    assert verdict == 'unknown' and details['phase'] == 'batched_oom'
    assert details['batch_size'] == 1
    assert f.calls.count('vcb_mlp_crown') == 4  # batch 8, 4, 2, 1 (one box in the worklist)


def test_is_oom_matches_the_reference_rule():
    assert bab.is_oom(MemoryError())
    assert bab.is_oom(torch.cuda.OutOfMemoryError('CUDA out of memory'))
    assert bab.is_oom(RuntimeError('CUDA error: out of memory'))
    assert not bab.is_oom(RuntimeError('illegal memory access'))
    assert not bab.is_oom(_lib.KernelError('vcb_mlp_crown: out of memory in a kernel'))


def test_installed_binding_delegates_only_unsupported_inputs(fake):
    """The delegating bindings hand UnsupportedInput to the reference's
    function; a KernelError from the B200 implementation propagates and the
    reference function is not run."""
    fake(fail={'vcb_mlp_crown'})
    ran = []

    def original(*a, **k):
        ran.append(a)
        return 'reference'

    def impl_fault(*a, **k):
        _lib.check(_lib.lib().vcb_mlp_crown(), 'vcb_mlp_crown')

    def impl_unsupported(*a, **k):
        raise _lib.UnsupportedInput('CPU tensor')

    with pytest.raises(_lib.KernelError):
        install._delegating(impl_fault, original)(1)
    assert not ran
    assert install._delegating(impl_unsupported, original)(1) == 'reference'
    with pytest.raises(TimeoutError):
        install._delegating(lambda *a: _lib.check(_lib.VCB_ERR_TIMEOUT), original)(1)
    assert len(ran) == 1


def test_cpu_tensors_are_unsupported_input():
    gg = wk.mlp_gg(wk.mlp_params((4, 6, 3), np.random.default_rng(0)))
    with pytest.raises(_lib.UnsupportedInput):
        ops._ibp_forward_graph_batched(torch.zeros(2, 4), torch.ones(2, 4), gg, 'cpu',
                                       torch.float32)
    with pytest.raises(_lib.UnsupportedInput):
        ops._ibp_forward_graph_batched(torch.zeros(2, 4), torch.ones(2, 4), gg, 'cuda',
                                       torch.float64)


@pytest.mark.parametrize('key', ['input_split_batched_clip_full_lp',
                                 'input_split_batched_milp_escalate'])
def test_settings_outside_the_b200_path_are_refused(key):
    """The Gurobi LP clip and MILP escalation are not on the B200 path: the
    driver refuses them with UnsupportedInput (so the installed binding runs
    the reference's own driver) instead of ignoring them."""
    assert bab.BabConfig(types.SimpleNamespace()).split_depth == 1
    with pytest.raises(_lib.UnsupportedInput):
        bab.BabConfig(types.SimpleNamespace(**{key: True}))


def test_branching_settings_are_read():
    c = bab.BabConfig(types.SimpleNamespace(
        bab_split_depth=3, input_split_batched_clip_iters=2, input_split_sb_margin_score=True,
        input_split_sb_coeff_thresh=0.5, input_split_sb_margin_weight=0.25,
        input_split_batched_branch_boost=False, input_split_batched_branch_boost_exp=2.0))
    assert (c.split_depth, c.clip_iters, c.margin, c.branch_boost, c.boost_exp) == \
        (3, 2, (0.5, 0.25), False, 2.0)
    # the reference driver's fallbacks for absent keys
    d = bab.BabConfig(types.SimpleNamespace())
    assert d.branch_sb and d.branch_boost and d.total_budget == 60.0 and d.margin is None
