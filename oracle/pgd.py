"""Numpy restatement of the batched sign-gradient PGD (test oracle).

Follows ``_simple_pgd_batched`` (``verify_hybrid_acasxu.py:103-161``): per
disjunct margin rows (W, b) (:117-130), per-sample loss
``min_d max_c (W_d y + b_d)_c`` (:145-149), SAT when a sample's loss is
<= 1e-6 (:150-154, first such sample in row order), otherwise
``x <- clamp(x - lr * sign(grad) * width, lo, hi)`` (:155-159).  The initial
samples are an input (the reference draws them from torch's generator after
``torch.manual_seed(seed)``; tests feed both implementations the same draw).
Gradients follow torch autograd: F.relu passes gradient where the
pre-activation is > 0; max/min route it to the first extremal index.
"""
from __future__ import annotations

import numpy as np

from . import bounds as ob


def margin_matrices(disjuncts, n_out, dtype=np.float32):
    """disjuncts: list of lists of ('pair', pred, comp) | ('ge', idx, val) |
    ('le', idx, val).  Returns [(W (n_c, n_out), b (n_c,))] per disjunct."""
    out = []
    for conj in disjuncts:
        W = np.zeros((len(conj), n_out), dtype)
        b = np.zeros(len(conj), dtype)
        for i, c in enumerate(conj):
            if c[0] == 'pair':
                W[i, c[1]] = 1.0
                W[i, c[2]] = -1.0
            elif c[0] == 'ge':
                W[i, c[1]] = -1.0
                b[i] = c[2]
            elif c[0] == 'le':
                W[i, c[1]] = 1.0
                b[i] = -c[2]
            else:
                raise ValueError(c)
        out.append((W, b))
    return out


def _mlp_layers(gg, dtype):
    layers = []
    for op in gg['ops']:
        if op['type'] == 'fc':
            a = ob.op_arrays(op, dtype)
            layers.append((a['W'], a['b']))
        elif op['type'] not in ('relu', 'reshape'):
            raise NotImplementedError('oracle pgd: fc/relu chains only')
    return layers


def pgd_batched(x0, lo, hi, gg, mats, n_iter=50, lr=0.1, dtype=np.float32):
    """x0, lo, hi: (N, n_in) samples and their (expanded) box bounds.

    Returns (sat, witness or None, iterations run)."""
    layers = _mlp_layers(gg, dtype)
    x = np.asarray(x0, dtype).copy()
    lo = np.asarray(lo, dtype)
    hi = np.asarray(hi, dtype)
    width = hi - lo
    lr = dtype(lr)
    for it in range(n_iter):
        acts = []
        a = x
        for i, (W, b) in enumerate(layers):
            z = a @ W.T + b
            if i < len(layers) - 1:
                acts.append(z)
                a = np.maximum(z, 0)
            else:
                a = z
        out = a
        per_d = []
        arg_c = []
        for W, b in mats:
            m = out @ W.T + b
            arg_c.append(m.argmax(axis=1))
            per_d.append(m.max(axis=1))
        stacked = np.stack(per_d, axis=1)
        d_arg = stacked.argmin(axis=1)
        min_m = stacked.min(axis=1)
        sat = min_m <= dtype(1e-6)
        if sat.any():
            idx = int(np.nonzero(sat)[0][0])
            return True, x[idx].copy(), it
        g = np.zeros_like(out)
        for d, (W, b) in enumerate(mats):
            sel = d_arg == d
            if sel.any():
                g[sel] += W[arg_c[d][sel]]
        for i in range(len(layers) - 1, -1, -1):
            W, _ = layers[i]
            g = g @ W
            if i > 0:
                g = g * (acts[i - 1] > 0)
        step = lr * np.sign(g) * width
        x = np.maximum(np.minimum(x - step, hi), lo)
    return False, None, n_iter
