"""Layer-wise IBP and CROWN for fc / conv / relu / reshape chains.

Networks with convolutions (cfg4) run op by op: conv layers as implicit GEMMs
(``vcb_conv_ibp``, ``vcb_conv_back``), fc layers on the wide GEMM kernels,
ReLU as element-wise kernels (``vcb_ibp_relu``, ``vcb_relu_back``) -- the
reference's ``_ibp_forward_graph_batched`` (verify_zono_bnb.py:1093-1152) and
``_spec_backward_graph_batched`` (:4379-4593) op handlers, each as a CUDA
launch.  Activations are NCHW-flattened rows exactly as the reference's
``reshape(B, *in_shape)`` / ``reshape(B, -1)``.
"""
from __future__ import annotations

import numpy as np
import torch

from . import _lib
from .netdesc import _as_np
from .ops import F32

P = _lib.ptr


def _pad4(n):
    return (n + 3) // 4 * 4


class GraphNet:
    """Device-side layers of a gg chain of fc / conv / relu / reshape ops; a
    single-input ``add`` / ``sub`` of a bias right after an fc or conv is
    folded into that layer's bias.  ``names[i]`` lists the op names whose
    output is layer i's output (reshapes alias the previous value; ``-1`` is
    the network input); ``stale`` holds fc / conv names whose own output no
    longer exists because a later bias was folded in."""

    def __init__(self, gg, device):
        self.layers = []
        self.relu_widths = []
        self.names = {-1: [gg['input_name']]}
        self.stale = set()
        cur = gg['input_name']
        n = int(gg.get('input_n') or 0)
        for op in gg['ops']:
            t = op['type']
            if op['inputs'][0] != cur:
                raise _lib.UnsupportedInput(f'vibecheck_nn_b200: non-chain graph at {op["name"]!r}')
            if t in ('add', 'sub') and not op.get('is_merge') and op.get('bias') is not None \
                    and self.layers and self.layers[-1]['type'] in ('fc', 'conv'):
                self._fold_bias(op, t, device)
                cur = op['name']
                continue
            if t == 'fc':
                W = torch.as_tensor(_as_np(op['W']), dtype=F32, device=device).contiguous()
                b = torch.as_tensor(_as_np(op['bias']), dtype=F32, device=device).flatten()
                nout, nin = W.shape
                aug = torch.zeros((nout, _pad4(nin + 1)), dtype=F32, device=device)
                aug[:, :nin] = W
                aug[:, nin] = b
                self.layers.append({'type': 'fc', 'W': W, 'Wabs': W.abs().contiguous(),
                                    'b': b.contiguous(), 'Waug': aug, 'nin': nin,
                                    'nout': nout})
                n = nout
            elif t == 'conv':
                K = torch.as_tensor(_as_np(op['kernel']), dtype=F32, device=device).contiguous()
                b = torch.as_tensor(_as_np(op['bias']), dtype=F32, device=device).flatten()
                C, H, Wd = (int(v) for v in op['in_shape'])
                Co, Ho, Wo = (int(v) for v in op['out_shape'])
                kh, kw = int(K.shape[2]), int(K.shape[3])
                sh, sw = (int(v) for v in op['stride'])
                ph, pw = (int(v) for v in op['padding'])
                if K.shape[1] != C or K.shape[0] != Co:
                    raise _lib.UnsupportedInput('vibecheck_nn_b200: grouped conv')
                if (C * H * Wd) % 4 or (Co * Ho * Wo) % 4:
                    raise _lib.UnsupportedInput('vibecheck_nn_b200: conv sizes must be multiples of 4')
                geom = np.array([C, H, Wd, Co, Ho, Wo, kh, kw, sh, sw, ph, pw], np.int32)
                self.layers.append({'type': 'conv', 'K': K, 'Kabs': K.abs().contiguous(),
                                    'b': b.contiguous(), 'geom': geom, 'nin': C * H * Wd,
                                    'nout': Co * Ho * Wo, 'Co': Co, 'hw': Ho * Wo})
                n = Co * Ho * Wo
            elif t == 'relu':
                self.layers.append({'type': 'relu', 'L': op['layer_idx'], 'n': n})
                self.relu_widths.append(n)
            elif t == 'reshape':
                self.names.setdefault(len(self.layers) - 1, []).append(op['name'])
                cur = op['name']
                continue
            else:
                raise _lib.UnsupportedInput(f'vibecheck_nn_b200: unsupported op {t!r}')
            self.names[len(self.layers) - 1] = [op['name']]
            cur = op['name']
        self.n_out = n

    def _fold_bias(self, op, t, device):
        """Bias add / sub after an fc or conv (the reference broadcasts it as
        _point_bcast_bias, verify_zono_bnb.py:525-551): a scalar, an fc's
        full-width vector or a conv's per-channel (Co, 1, 1) block folds into
        the layer bias; other broadcasts are not supported."""
        layer = self.layers[-1]
        raw = np.asarray(_as_np(op['bias']))
        shape = tuple(int(d) for d in raw.shape)
        while shape and shape[0] == 1 and len(shape) > 1:
            shape = shape[1:]
        if raw.size == 1:
            n_ch = layer['nout'] if layer['type'] == 'fc' else layer['Co']
            vec = np.full(n_ch, float(raw.reshape(-1)[0]))
        elif layer['type'] == 'fc' and raw.size == layer['nout']:
            vec = raw.reshape(-1)
        elif layer['type'] == 'conv' and shape == (layer['Co'], 1, 1):
            vec = raw.reshape(-1)
        else:
            raise _lib.UnsupportedInput('vibecheck_nn_b200: broadcast bias')
        bias = torch.as_tensor(vec, dtype=F32, device=device)
        layer['b'] = (layer['b'] + bias if t == 'add' else layer['b'] - bias).contiguous()
        if layer['type'] == 'fc':
            layer['Waug'][:, layer['nin']] = layer['b']
        idx = len(self.layers) - 1
        self.stale.update(self.names.get(idx, []))
        self.names[idx] = [op['name']]

    def layer_of(self, name):
        """Index of the layer whose output is op ``name`` (-1: the input)."""
        if name in self.stale:
            raise _lib.UnsupportedInput(
                f'vibecheck_nn_b200: {name!r} has a bias folded into it; capture the add')
        for idx, names in self.names.items():
            if name in names:
                return idx
        raise KeyError(name)


def graph_net(gg, device):
    cache = gg.setdefault('_vcb_cache', {})
    key = ('_graph', str(device))
    ent = cache.get(key)
    if ent is not None and ent[0] is gg['ops']:
        return ent[1]
    g = GraphNet(gg, device)
    cache[key] = (gg['ops'], g)
    return g


def _geom_ptr(a):
    return a.ctypes.data_as(_lib.ctypes.POINTER(_lib.ctypes.c_int32))


def graph_ibp(G, xl, xh, clamps=None):
    """IBP through the chain; returns sb {L: (lo, hi)} (D, n_L)."""
    dev = xl.device
    D, n0 = xl.shape
    st = _lib.stream_of(dev)
    L_ = _lib.lib()
    ld = _pad4(n0)
    mid = torch.zeros((D, ld), dtype=F32, device=dev)
    rad = torch.zeros((D, ld), dtype=F32, device=dev)
    mid[:, :n0] = (xl + xh) * 0.5
    rad[:, :n0] = (xh - xl) * 0.5
    lo = hi = None
    sb = {}
    for layer in G.layers:
        t = layer['type']
        if t == 'fc':
            lo = torch.empty((D, layer['nout']), dtype=F32, device=dev)
            hi = torch.empty_like(lo)
            rc = L_.vcb_wide_ibp_layer(D, layer['nin'], layer['nout'], P(mid), P(rad), ld,
                                       P(layer['W']), P(layer['Wabs']), P(layer['b']), None,
                                       None, P(lo), P(hi), None, None, 4, st)
            _lib.check(rc, 'vcb_wide_ibp_layer')
        elif t == 'conv':
            lo = torch.empty((D, layer['nout']), dtype=F32, device=dev)
            hi = torch.empty_like(lo)
            rc = L_.vcb_conv_ibp(D, _geom_ptr(layer['geom']), P(mid), P(rad), P(layer['K']),
                                 P(layer['Kabs']), P(layer['b']), P(lo), P(hi), st)
            _lib.check(rc, 'vcb_conv_ibp')
        else:  # relu
            n = layer['n']
            L = layer['L']
            ld = _pad4(n)
            sl = torch.empty((D, n), dtype=F32, device=dev)
            sh = torch.empty_like(sl)
            mid = torch.zeros((D, ld), dtype=F32, device=dev)
            rad = torch.zeros((D, ld), dtype=F32, device=dev)
            cl = ch = None
            if clamps is not None and L in clamps:
                cl = clamps[L][0].to(F32).expand(D, n).contiguous()
                ch = clamps[L][1].to(F32).expand(D, n).contiguous()
            rc = L_.vcb_ibp_relu(D, n, P(lo), P(hi), P(cl), P(ch), P(sl), P(sh), P(mid),
                                 P(rad), ld, st)
            _lib.check(rc, 'vcb_ibp_relu')
            sb[L] = (sl, sh)
    return sb


def graph_crown(G, xl, xh, sb, W_q, b_q, alpha=None, beta=None, want_A=False):
    """CROWN back-substitution through the chain for D boxes x Q spec rows.
    Returns dict(lb (D, Q), acc (D, Q)[, A (D, Q, n0)])."""
    dev = xl.device
    D, n0 = xl.shape
    Q = W_q.shape[0]
    R = D * Q
    st = _lib.stream_of(dev)
    L_ = _lib.lib()
    nL = G.n_out
    ldc = _pad4(nL)
    coef = torch.zeros((R, ldc), dtype=F32, device=dev)
    coef[:, :nL] = W_q.repeat(D, 1)
    acc = b_q.repeat(D).contiguous().clone()
    zeros_bd = torch.zeros(R, dtype=F32, device=dev)
    layers = G.layers
    for idx in range(len(layers) - 1, -1, -1):
        layer = layers[idx]
        t = layer['type']
        # the op consuming this op's output coefficients (next in backward
        # order) decides the layout: conv wants dense rows
        nxt = layers[idx - 1]['type'] if idx > 0 else None
        if t == 'fc':
            nin = layer['nin']
            ldo = _pad4(nin + 1)
            coef_o = torch.empty((R, ldo), dtype=F32, device=dev)
            bd = torch.empty(R, dtype=F32, device=dev)
            nparts = L_.vcb_wide_back_parts(R, nin)
            part = torch.empty((R, nparts), dtype=F32, device=dev)
            rc = L_.vcb_wide_back_layer(R, Q, nin, layer['nout'], P(coef), ldc, P(layer['Waug']),
                                        layer['Waug'].shape[1], None, None, None, 0, None,
                                        P(coef_o), None, ldo, P(bd), P(part), st)
            _lib.check(rc, 'vcb_wide_back_layer')
            rc = L_.vcb_wide_rowsum(R, nparts, 0, P(bd), P(part), P(acc), st)
            _lib.check(rc, 'vcb_wide_rowsum')
            coef, ldc = coef_o, ldo
        elif t == 'conv':
            if ldc != layer['nout']:
                coef = coef[:, :layer['nout']].contiguous()
                ldc = layer['nout']
            bd = torch.empty(R, dtype=F32, device=dev)
            rc = L_.vcb_conv_bias_dot(R, layer['Co'], layer['hw'], P(coef), P(layer['b']),
                                      P(bd), st)
            _lib.check(rc, 'vcb_conv_bias_dot')
            e_in = torch.empty((R, layer['nin']), dtype=F32, device=dev)
            ws_n = L_.vcb_conv_back_workspace(R, _geom_ptr(layer['geom']))
            ws = _lib.workspace(ws_n, dev)
            rc = L_.vcb_conv_back(R, _geom_ptr(layer['geom']), P(coef), P(layer['K']),
                                  P(e_in), P(ws), ws_n, st)
            _lib.check(rc, 'vcb_conv_back')
            rc = L_.vcb_wide_rowsum(R, 1, 0, P(bd), P(bd), P(acc), st)
            _lib.check(rc, 'vcb_wide_rowsum')
            coef, ldc = e_in, layer['nin']
        else:  # relu
            n = layer['n']
            L = layer['L']
            ldo = n if nxt == 'conv' else _pad4(n)
            coef_o = torch.zeros((R, ldo), dtype=F32, device=dev)
            part = torch.empty(R, dtype=F32, device=dev)
            lo, hi = sb[L]
            al = alpha.get(L) if alpha is not None else None
            be = beta.get(L) if beta is not None else None
            rc = L_.vcb_relu_back(R, Q, n, P(coef), ldc, P(coef_o), ldo,
                                  P(lo.contiguous()), P(hi.contiguous()),
                                  P(None if al is None else al.contiguous()),
                                  P(None if be is None else be.contiguous()), P(part), st)
            _lib.check(rc, 'vcb_relu_back')
            rc = L_.vcb_wide_rowsum(R, 1, 1, P(zeros_bd), P(part), P(acc), st)
            _lib.check(rc, 'vcb_wide_rowsum')
            coef, ldc = coef_o, ldo
    lb = torch.empty(R, dtype=F32, device=dev)
    A = torch.empty((R, n0), dtype=F32, device=dev) if want_A else None
    rc = L_.vcb_wide_concretize(R, Q, n0, ldc, P(coef), P(acc), P(xl.contiguous()),
                                P(xh.contiguous()), P(lb), P(A), None, st)
    _lib.check(rc, 'vcb_wide_concretize')
    out = {'lb': lb.view(D, Q), 'acc': acc.view(D, Q)}
    if want_A:
        out['A'] = A.view(D, Q, n0)
    return out


def graph_forward(G, x, upto=None, keep=False):
    """Concrete forward of N points x (N, n0) through the chain (the
    fc / conv / relu branches of _forward_batch_graph,
    verify_zono_bnb.py:554-596).  Returns the output of layer ``upto``
    (default: the last) and, with ``keep``, the pre-activation of every layer
    that feeds a ReLU {layer index: (N, n)} for graph_vjp."""
    dev = x.device
    N = x.shape[0]
    st = _lib.stream_of(dev)
    L_ = _lib.lib()
    layers = G.layers
    last = len(layers) - 1 if upto is None else upto
    cur = x.contiguous()
    pre = {}
    for idx in range(last + 1):
        layer = layers[idx]
        t = layer['type']
        if t == 'relu':
            continue  # written by the producer's epilogue
        nxt_relu = idx + 1 < len(layers) and layers[idx + 1]['type'] == 'relu'
        want_a = nxt_relu and idx + 1 <= last
        want_z = keep or not want_a
        z = torch.empty((N, layer['nout']), dtype=F32, device=dev) if want_z else None
        a = torch.empty((N, layer['nout']), dtype=F32, device=dev) if want_a else None
        if t == 'fc':
            rc = L_.vcb_fc_forward(N, layer['nin'], layer['nout'], P(cur), cur.shape[1],
                                   P(layer['W']), P(layer['b']), P(z), layer['nout'], P(a),
                                   layer['nout'], st)
            _lib.check(rc, 'vcb_fc_forward')
        else:
            rc = L_.vcb_conv_forward(N, _geom_ptr(layer['geom']), P(cur), P(layer['K']),
                                     P(layer['b']), P(z), P(a), st)
            _lib.check(rc, 'vcb_conv_forward')
        if keep and nxt_relu:
            pre[idx] = z
        cur = a if want_a else z
    return (cur, pre) if keep else cur


def graph_vjp(G, pre, g):
    """d(g . f(x))/dx for the points whose pre-activations ``pre`` came from
    graph_forward(keep=True): the transposed layers, each masked by the ReLU
    in front of it (F.relu passes the gradient where z > 0)."""
    dev = g.device
    N = g.shape[0]
    st = _lib.stream_of(dev)
    L_ = _lib.lib()
    layers = G.layers
    if layers[-1]['type'] == 'relu':
        raise _lib.UnsupportedInput('vibecheck_nn_b200: network output after a relu')
    cur = g.contiguous()
    for idx in range(len(layers) - 1, -1, -1):
        layer = layers[idx]
        if layer['type'] == 'relu':
            continue
        mask = pre.get(idx - 2) if idx >= 1 and layers[idx - 1]['type'] == 'relu' else None
        out = torch.empty((N, layer['nin']), dtype=F32, device=dev)
        if layer['type'] == 'fc':
            rc = L_.vcb_fc_backward(N, layer['nin'], layer['nout'], P(cur), cur.shape[1],
                                    P(layer['W']), P(mask), layer['nin'], P(out),
                                    layer['nin'], st)
            _lib.check(rc, 'vcb_fc_backward')
        else:
            ws_n = L_.vcb_conv_back_workspace(N, _geom_ptr(layer['geom']))
            ws = _lib.workspace(ws_n, dev)
            rc = L_.vcb_conv_backward(N, _geom_ptr(layer['geom']), P(cur), P(layer['K']),
                                      P(mask), P(out), P(ws), ws_n, st)
            _lib.check(rc, 'vcb_conv_backward')
        cur = out
    return cur
