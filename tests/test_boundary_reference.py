"""The drop-in boundary against the reference's own modules.

Imports vibecheck's modules from a reference checkout (with an empty
``gurobipy`` stub: only gurobi_util.py imports it at module level), runs
``install()`` on them and checks that every rebound name exists in the
reference module and that each replacement accepts every parameter of the
function it replaces -- same names, kinds, positions and defaults -- so a
renamed or reordered keyword on either side fails here.  Skipped when no
reference checkout is available (``VIBECHECK_REF_SRC`` or a ``reference/src``
beside this repository).
"""
import importlib
import inspect
import os
import sys
import types

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
REF_SRC = os.environ.get('VIBECHECK_REF_SRC',
                         os.path.join(os.path.dirname(ROOT), 'reference', 'src'))

pytestmark = pytest.mark.skipif(not os.path.isdir(os.path.join(REF_SRC, 'vibecheck')),
                                reason='no reference checkout')


def _compatible(orig, impl):
    """Problems that keep ``impl`` from accepting every call ``orig``
    accepts (empty when compatible)."""
    so, si = inspect.signature(orig), inspect.signature(impl)
    po, pi = list(so.parameters.values()), list(si.parameters.values())
    byname = {p.name: p for p in pi}
    pos_o = [p.name for p in po if p.kind in (p.POSITIONAL_ONLY, p.POSITIONAL_OR_KEYWORD)]
    pos_i = [p.name for p in pi if p.kind in (p.POSITIONAL_ONLY, p.POSITIONAL_OR_KEYWORD)]
    bad = []
    if pos_i[:len(pos_o)] != pos_o:
        bad.append(f'positional order {pos_o} vs {pos_i}')
    for p in po:
        q = byname.get(p.name)
        if q is None:
            bad.append(f'missing parameter {p.name}')
            continue
        if p.kind == p.KEYWORD_ONLY and q.kind not in (q.KEYWORD_ONLY, q.POSITIONAL_OR_KEYWORD):
            bad.append(f'{p.name}: keyword-only in the reference')
        if p.default is not p.empty and q.default != p.default:
            bad.append(f'{p.name}: default {p.default!r} vs {q.default!r}')
    for q in pi:
        if q.name not in {p.name for p in po} and q.default is q.empty and \
                q.kind not in (q.VAR_POSITIONAL, q.VAR_KEYWORD):
            bad.append(f'extra required parameter {q.name}')
    return bad


def test_install_rebinds_the_reference_modules(monkeypatch):
    from vibecheck_nn_b200 import install
    monkeypatch.setitem(sys.modules, 'gurobipy', types.ModuleType('gurobipy'))
    monkeypatch.syspath_prepend(REF_SRC)
    mods = {name: importlib.import_module(name) for name in install.BINDINGS}
    originals = {}
    for mod_name, names in install.BINDINGS.items():
        for attr in names:
            assert hasattr(mods[mod_name], attr), f'{mod_name}.{attr} is not in the reference'
            originals[(mod_name, attr)] = getattr(mods[mod_name], attr)
            # restored at teardown: the reference modules stay untouched
            monkeypatch.setattr(mods[mod_name], attr, originals[(mod_name, attr)])
    done = install.install(mods)
    assert sum(len(v) for v in done.values()) == sum(len(v) for v in install.BINDINGS.values())
    problems = {}
    for mod_name, names in install.BINDINGS.items():
        for attr, spec in names.items():
            new = getattr(mods[mod_name], attr)
            impl = getattr(importlib.import_module(f'vibecheck_nn_b200.{spec[0]}'), spec[1])
            assert getattr(new, '__wrapped__', new) is impl, (mod_name, attr)
            bad = _compatible(originals[(mod_name, attr)], impl)
            if bad:
                problems[f'{mod_name}.{attr}'] = bad
    assert not problems, problems


def test_compatibility_check_catches_renames():
    def ref(a, b, *, c=1, d=None):
        pass

    def renamed(a, b, *, c=1, e=None):
        pass

    def reordered(b, a, *, c=1, d=None):
        pass

    def new_default(a, b, *, c=2, d=None):
        pass

    def ok(a, b, c=1, d=None, extra=False):
        pass

    assert _compatible(ref, renamed)
    assert _compatible(ref, reordered)
    assert _compatible(ref, new_default)
    assert not _compatible(ref, ok)
