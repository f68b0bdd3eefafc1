"""DeepZ zonotope for MLPs too wide for the shared-memory kernel (cfg5).

``wide_zono`` follows _forward_zonotope_graph_batched
(verify_zono_bnb.py:3079-4074) layer by layer on the kernels of
vcb_zono_wide.cu and the tcgen05 3xTF32 GEMM:

* layer 0: centre ``c W0^T + b0`` and radius ``r |W0|^T`` (its generators are
  r_i W0[:, i], so the pre-ReLU bounds are exact without a GEMM);
* every later layer: the ReLU transformer (``vcb_zw_relu``), one host read of
  the per-leaf unstable counts (the reference syncs at the same point), the
  next generator matrix of the whole batch as one ``vcb_tc_gemm`` over
  generator-major rows built by ``vcb_zw_build``, and the fixed-order
  per-leaf radius ``vcb_zw_colsum``.

Generators of leaf b are rows [off[b], off[b+1]) of one matrix; the first
k[b] rows are its generators in the reference's column order (input
dimensions, then each ReLU layer's unstable neurons in index order), the rest
zero padding to a multiple of 128 rows (one GEMM tile).
"""
from __future__ import annotations

import numpy as np
import torch

from . import _lib
from .ops import F32

P = _lib.ptr
ROW_TILE = 128
COL_CHUNK = 128  # rows per partial radius sum (vcb_zw_colsum)


def _pad4(n):
    return (n + 3) // 4 * 4


def _split(x):
    hi = torch.empty_like(x)
    lo = torch.empty_like(x)
    _lib.check(_lib.lib().vcb_tf32_split(x.numel(), P(x), P(hi), P(lo), _lib.stream_of(x.device)),
               'vcb_tf32_split')
    return hi, lo


class WideZonoNet:
    """Per-layer weights in the layouts the wide zonotope reads: W (n_out x
    n_in) TF32-split with leading dimension pad4(n_in), |W0| and W0^T."""

    def __init__(self, wn):
        self.dims = wn.dims
        self.W = wn.W
        self.b = wn.b
        self.W0abs = wn.Wabs[0]
        self.W0T = wn.W[0].t().contiguous()
        self.zero_b0 = torch.zeros_like(wn.b[0])
        self.split = [None]
        for W in wn.W[1:]:
            nout, nin = W.shape
            Wp = torch.zeros((nout, _pad4(nin)), dtype=F32, device=W.device)
            Wp[:, :nin] = W
            self.split.append(_split(Wp))


def zono_net(wn):
    z = wn.__dict__.get('_zono')
    if z is None:
        z = WideZonoNet(wn)
        wn.__dict__['_zono'] = z
    return z


def _fc(x, W, b):
    N, nin = x.shape
    nout = W.shape[0]
    z = torch.empty((N, nout), dtype=F32, device=x.device)
    rc = _lib.lib().vcb_fc_forward(N, nin, nout, P(x), x.stride(0), P(W), P(b), P(z), nout, None,
                                   0, _lib.stream_of(x.device))
    _lib.check(rc, 'vcb_fc_forward')
    return z


def wide_zono(wn, xl, xh, want_output=False, stats=None):
    """Zonotope bounds of B boxes.  Returns sb {L: (lo, hi) (B, n_L)} and,
    with ``want_output``, (c_out (B, n_out), G (B, n_out, K)) as the
    reference returns them (generator columns in its order, zero-padded to
    the batch maximum).  ``stats`` (a dict) collects the generator GEMMs'
    algorithmic FLOPs (unpadded rows) and CUDA events around each launch."""
    z = zono_net(wn)
    dev = xl.device
    st = _lib.stream_of(dev)
    L_ = _lib.lib()
    B, n0 = xl.shape
    nfc = len(z.W)
    xl = xl.to(F32).contiguous()
    xh = xh.to(F32).contiguous()
    c = (xl + xh) / 2
    r = ((xh - xl) / 2).contiguous()
    cur_c = _fc(c, z.W[0], z.b[0])
    rad = _fc(r, z.W0abs, z.zero_b0)
    lo, hi = cur_c - rad, cur_c + rad
    sb = {0: (lo, hi)} if nfc > 1 else {}
    k_in = torch.full((B,), n0, dtype=torch.int32, device=dev)
    k_host = np.full(B, n0, dtype=np.int64)
    in_off = None
    C = None
    ldc = 0
    err = torch.zeros(1, dtype=torch.int32, device=dev)
    for l in range(1, nfc):
        if l == nfc - 1 and not want_output:
            break  # the output layer's generators are not needed for the bounds
        n = wn.dims[l]
        ld = _pad4(n)
        lam = torch.empty((B, n), dtype=F32, device=dev)
        mu = torch.empty_like(lam)
        c_relu = torch.empty_like(lam)
        cnt = torch.empty(B, dtype=torch.int32, device=dev)
        idx = torch.empty((B, n), dtype=torch.int32, device=dev)
        rc = L_.vcb_zw_relu(B, n, P(cur_c), P(lo.contiguous()), P(hi.contiguous()), P(lam), P(mu),
                            P(c_relu), P(cnt), P(idx), st)
        _lib.check(rc, 'vcb_zw_relu')
        k_out = k_host + cnt.cpu().numpy().astype(np.int64)  # host sync: row counts
        rows = (k_out + ROW_TILE - 1) // ROW_TILE * ROW_TILE
        out_off_h = np.zeros(B + 1, dtype=np.int64)
        out_off_h[1:] = np.cumsum(rows)
        M = int(out_off_h[-1])
        out_off = torch.as_tensor(out_off_h, device=dev)
        A_hi = torch.empty((M, ld), dtype=F32, device=dev)
        A_lo = torch.empty_like(A_hi)
        rc = L_.vcb_zw_build(B, n, ld, P(in_off), P(k_in), P(C), ldc, P(r), n0, P(z.W0T), P(lam),
                             P(mu), P(cnt), P(idx), P(out_off), M, P(A_hi), P(A_lo), st)
        _lib.check(rc, 'vcb_zw_build')
        nout = wn.dims[l + 1]
        ldc = _pad4(nout)
        C = torch.empty((M, ldc), dtype=F32, device=dev)
        W_hi, W_lo = z.split[l]
        if stats is not None:
            ev = (torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
            ev[0].record()
        rc = L_.vcb_tc_gemm(M, nout, n, P(A_hi), P(A_lo), ld, P(W_hi), P(W_lo), ld, None, P(C),
                            ldc, P(err), st)
        _lib.check(rc, 'vcb_tc_gemm')
        if stats is not None:
            ev[1].record()
            stats.setdefault('gemm_events', []).append(ev)
            stats['gemm_flop'] = stats.get('gemm_flop', 0) + 2.0 * float(k_out.sum()) * nout * n
            stats['gemm_launches'] = stats.get('gemm_launches', 0) + 1
        del A_hi, A_lo
        cur_c = _fc(c_relu, z.W[l], z.b[l])
        k_host = k_out
        k_in = torch.as_tensor(k_out.astype(np.int32), device=dev)
        in_off = out_off
        if l < nfc - 1 or want_output:
            lo = torch.empty((B, nout), dtype=F32, device=dev)
            hi = torch.empty_like(lo)
            nch = (k_out + COL_CHUNK - 1) // COL_CHUNK
            ch_off = np.zeros(B + 1, dtype=np.int64)
            ch_off[1:] = np.cumsum(nch)
            ws_n = L_.vcb_zw_colsum_workspace(int(ch_off[-1]), nout)
            ws = _lib.workspace(ws_n, dev)
            rc = L_.vcb_zw_colsum(B, nout, P(in_off), P(k_in),
                                  P(torch.as_tensor(ch_off, device=dev)), int(nch.max()), P(C),
                                  ldc, P(cur_c), P(lo), P(hi), P(ws), ws_n, st)
            _lib.check(rc, 'vcb_zw_colsum')
            if l < nfc - 1:
                sb[l] = (lo, hi)
    if int(err.item()) != 0:
        raise TimeoutError('vibecheck_nn_b200: vcb_tc_gemm pipeline wait expired')
    if not want_output:
        return sb
    nout = wn.dims[-1]
    if nfc == 1:
        Kmax = n0
        G = torch.zeros((B, nout, Kmax), dtype=F32, device=dev)
        G[:] = z.W[0].unsqueeze(0) * r.unsqueeze(1)
        return sb, (cur_c, G)
    Kmax = int(k_host.max()) if B else 0
    G = torch.zeros((B, nout, Kmax), dtype=F32, device=dev)
    offs = in_off.cpu().numpy()
    for b in range(B):
        kb = int(k_host[b])
        G[b, :, :kb] = C[int(offs[b]):int(offs[b]) + kb, :nout].t()
    return sb, (cur_c, G)
