"""Network descriptors built once per ``gg`` op dict (and cached on it).

The reference's op dicts (``ComputeGraph.gpu_graph``, network.py:1707-2910)
are lowered here to the packed layouts the kernels read:

* ``MlpDesc`` -- an fc/relu chain: fc weights back to back (layer l row-major
  ``(n_{l+1}, n_l)``), biases back to back, plus a ``vcb_mlp`` ctypes struct.
  ``reshape`` ops are identities, and so is an all-zero ``add``/``sub`` of
  the input; a single-input ``add``/``sub`` with a bias vector right after
  an fc is folded into that fc's bias.

Anything else raises ``NotImplementedError`` -- the exception type the
reference's callers already treat as "route elsewhere"
(verify_graph.py:9949-9980).
"""
from __future__ import annotations

import numpy as np
import torch

from . import _lib


class MlpDesc:
    def __init__(self, dims, W_all, b_all, Ws, bs):
        self.dims = tuple(int(d) for d in dims)
        self.n_fc = len(self.dims) - 1
        self.W_all = W_all
        self.b_all = b_all
        self.Ws = Ws
        self.bs = bs
        self.relu_widths = self.dims[1:-1]
        self.struct = _lib.VcbMlp()
        self.struct.n_fc = self.n_fc
        for i, d in enumerate(self.dims):
            self.struct.dims[i] = d
        self.struct.W = W_all.data_ptr()
        self.struct.b = b_all.data_ptr()

    @property
    def n_in(self):
        return self.dims[0]

    @property
    def n_out(self):
        return self.dims[-1]

    def relu_offsets(self, B):
        """Element offsets of each relu layer's (B, n_L) block in a packed
        per-layer array, and the total length."""
        offs = []
        o = 0
        for n in self.relu_widths:
            offs.append(o)
            o += B * n
        return offs, o


def _as_np(t):
    if isinstance(t, torch.Tensor):
        return t.detach().cpu().to(torch.float64).numpy()
    return np.asarray(t, np.float64)


def lower_mlp(gg):
    """fc/relu chain of a gg -> ([(W (out,in), b (out,)) float64], relu idx)."""
    ops = gg['ops']
    layers = []
    cur = gg['input_name']
    expect_fc = True
    relu_seen = 0
    for op in ops:
        t = op['type']
        if op['inputs'][0] != cur:
            raise _lib.UnsupportedInput(
                f'vibecheck_nn_b200: op {op["name"]!r} does not consume the '
                f'previous op (non-chain graph)')
        if t == 'fc':
            if not expect_fc:
                raise _lib.UnsupportedInput('vibecheck_nn_b200: fc after fc')
            W = _as_np(op['W'])
            b = _as_np(op['bias']) if op.get('bias') is not None else np.zeros(W.shape[0])
            if W.ndim != 2 or (layers and W.shape[1] != layers[-1][0].shape[0]):
                raise _lib.UnsupportedInput(
                    f'vibecheck_nn_b200: fc {op["name"]!r} shape {W.shape}')
            in_nd = op.get('in_shapes_nd', [None])[0]
            if in_nd is not None and len(in_nd) >= 2 and W.shape[1] == in_nd[-1] \
                    and int(np.prod(in_nd)) != W.shape[1]:
                raise _lib.UnsupportedInput('vibecheck_nn_b200: ND-batched fc')
            layers.append([W, b.reshape(-1)])
            expect_fc = False
        elif t == 'relu':
            if expect_fc:
                raise _lib.UnsupportedInput('vibecheck_nn_b200: relu not after fc')
            if op.get('layer_idx', relu_seen) != relu_seen:
                raise _lib.UnsupportedInput('vibecheck_nn_b200: relu layer_idx order')
            relu_seen += 1
            expect_fc = True
        elif t == 'reshape':
            pass
        elif t in ('add', 'sub') and not op.get('is_merge') and not layers \
                and op.get('bias') is not None and not np.any(_as_np(op['bias'])):
            pass  # a zero offset of the input (ACAS Xu's input_Sub): exact identity
        elif t in ('add', 'sub') and not op.get('is_merge') and not expect_fc \
                and op.get('bias') is not None:
            bias = _as_np(op['bias']).reshape(-1)
            if bias.size != layers[-1][1].size:
                raise _lib.UnsupportedInput('vibecheck_nn_b200: broadcast bias')
            layers[-1][1] = layers[-1][1] + (bias if t == 'add' else -bias)
        else:
            raise _lib.UnsupportedInput(
                f'vibecheck_nn_b200: unsupported op {t!r} at {op["name"]!r}')
        cur = op['name']
    if expect_fc or not layers:
        raise _lib.UnsupportedInput('vibecheck_nn_b200: graph must end in an fc')
    if len(layers) > _lib.MAX_FC:
        raise _lib.UnsupportedInput(f'vibecheck_nn_b200: more than {_lib.MAX_FC} fc layers')
    return layers


def mlp_desc(gg, device):
    """Cached ``MlpDesc`` for gg on device (fp32)."""
    device = torch.device(device)
    key = ('_vcb_mlp', str(device))
    cache = gg.get('_vcb_cache')
    if cache is None:
        cache = {}
        gg['_vcb_cache'] = cache
    ent = cache.get(key)
    if ent is not None and ent[0] is gg['ops']:
        return ent[1]
    layers = lower_mlp(gg)
    dims = [layers[0][0].shape[1]] + [W.shape[0] for W, _ in layers]
    Ws = [torch.as_tensor(W, dtype=torch.float32, device=device) for W, _ in layers]
    bs = [torch.as_tensor(b, dtype=torch.float32, device=device) for _, b in layers]
    W_all = torch.cat([w.reshape(-1) for w in Ws]).contiguous()
    b_all = torch.cat(bs).contiguous()
    desc = MlpDesc(dims, W_all, b_all, Ws, bs)
    cache[key] = (gg['ops'], desc)
    return desc
