"""The allocation-free CROWN entry point agrees with the workspace one.

``vcb_mlp_crown_noalloc`` serves callers that may not allocate GPU memory
while they bound boxes (a host application whose memory pool already owns the
device, or a tight loop where cudaMalloc is not allowed): its scratch is a
fixed static device array instead of a caller workspace.  This test calls it
through the C ABI twice in a row (the second call reuses the array the first
one left behind) and compares every output with ``vcb_mlp_crown`` at the
parity tolerance used throughout the tests.  It lives in its own file, named
to be collected last.
"""
import ctypes

import numpy as np
import pytest
import torch

from conftest import close, max_excess
from vibecheck_nn_b200 import _lib, netdesc, ops, workloads as wk

pytestmark = pytest.mark.gpu


def _ptr(t):
    return None if t is None else ctypes.c_void_p(t.data_ptr())


@pytest.mark.parametrize('n_boxes,n_q,with_sb', [(8192, 4, False), (3001, 9, True)])
def test_noalloc_matches_workspace_entry_point(n_boxes, n_q, with_sb):
    dev = torch.device('cuda:0')
    lib = _lib.lib()
    w = wk.cfg2(seed=11, n_boxes=n_boxes, n_q=n_q)
    gg = wk.mlp_gg(w['layers'], dev)
    desc = netdesc.mlp_desc(gg, dev)
    xl = torch.as_tensor(w['xl'], device=dev)
    xh = torch.as_tensor(w['xh'], device=dev)
    W_q = torch.as_tensor(w['spec_W'], device=dev)
    b_q = torch.as_tensor(w['spec_b'], device=dev)
    ref = ops.mlp_crown(desc, xl, xh, spec=(W_q, b_q), want_A=True, want_sb=with_sb)
    torch.cuda.synchronize(dev)
    _, total = desc.relu_offsets(n_boxes)
    for call in range(2):
        lb = torch.full((n_boxes, n_q), float('nan'), device=dev)
        A = torch.full((n_boxes, n_q, desc.n_in), float('nan'), device=dev)
        acc = torch.full((n_boxes, n_q), float('nan'), device=dev)
        sbl = torch.full((total,), float('nan'), device=dev) if with_sb else None
        sbh = torch.full((total,), float('nan'), device=dev) if with_sb else None
        torch.cuda.synchronize(dev)
        rc = lib.vcb_mlp_crown_noalloc(
            desc.struct, n_boxes, _ptr(xl), _ptr(xh), None, None, None, None, None,
            None, n_q, _ptr(W_q), _ptr(b_q), _ptr(lb), _ptr(A), _ptr(acc),
            _ptr(sbl), _ptr(sbh), _lib.stream_of(dev))
        _lib.check(rc, f'vcb_mlp_crown_noalloc call {call}')
        torch.cuda.synchronize(dev)
        for got, want in ((lb, ref['lb']), (A, ref['A']), (acc, ref['acc'])):
            g, r = got.cpu().numpy(), want.cpu().numpy()
            assert np.isfinite(g).all()
            assert close(g, r), max_excess(g, r)
        if with_sb:
            assert close(sbl.cpu().numpy(), ref['sb_lo'].cpu().numpy())
            assert close(sbh.cpu().numpy(), ref['sb_hi'].cpu().numpy())
    assert lib.vcb_mlp_crown_noalloc_capacity() == 4 << 20
