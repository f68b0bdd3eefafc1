"""Numpy restatement of the reference's batched bound kernels (test oracle).

Follows ``src/vibecheck/verify_zono_bnb.py`` and ``verify_graph.py`` of
stanleybak/vibecheck-nn.  All arrays are numpy; ``dtype`` selects float32
(the reference's ``bits=32`` arithmetic) or float64 (to separate rounding
from algorithmic differences).  Supported ops: fc, relu, reshape, add (bias),
sub (bias), conv -- the ops the hot-path configurations use.
"""
from __future__ import annotations

import numpy as np


def _np(t, dtype):
    """torch tensor / array -> numpy array of dtype."""
    if t is None:
        return None
    if hasattr(t, 'detach'):
        t = t.detach().cpu().numpy()
    return np.asarray(t, dtype=dtype)


def op_arrays(op, dtype):
    """Per-op numpy parameters, cached on the op dict per dtype."""
    key = '_oracle_np_' + np.dtype(dtype).name
    cached = op.get(key)
    if cached is not None:
        return cached
    t = op['type']
    if t == 'fc':
        arr = {'W': _np(op['W'], dtype), 'b': _np(op['bias'], dtype)}
    elif t == 'conv':
        arr = {'K': _np(op['kernel'], dtype), 'b': _np(op['bias'], dtype)}
    elif t in ('add', 'sub'):
        b = op.get('bias')
        arr = {'b': None if b is None else _np(b, dtype).reshape(-1)}
    else:
        arr = {}
    op[key] = arr
    return arr


# ---------------------------------------------------------------------------
# convolution helpers (NCHW, square stride/padding tuples)
# ---------------------------------------------------------------------------

def _im2col(x, kh, kw, stride, pad):
    N, C, H, W = x.shape
    xp = np.pad(x, ((0, 0), (0, 0), (pad[0], pad[0]), (pad[1], pad[1])))
    Ho = (H + 2 * pad[0] - kh) // stride[0] + 1
    Wo = (W + 2 * pad[1] - kw) // stride[1] + 1
    cols = np.empty((N, C, kh, kw, Ho, Wo), dtype=x.dtype)
    for i in range(kh):
        for j in range(kw):
            cols[:, :, i, j] = xp[:, :, i:i + stride[0] * Ho:stride[0],
                                  j:j + stride[1] * Wo:stride[1]]
    return cols, Ho, Wo


def conv2d(x, K, b, stride, pad):
    """torch.nn.functional.conv2d semantics (cross-correlation)."""
    Co, Ci, kh, kw = K.shape
    cols, Ho, Wo = _im2col(x, kh, kw, stride, pad)
    N = x.shape[0]
    cm = cols.transpose(0, 4, 5, 1, 2, 3).reshape(N * Ho * Wo, Ci * kh * kw)
    out = cm @ K.reshape(Co, -1).T
    out = out.reshape(N, Ho, Wo, Co).transpose(0, 3, 1, 2)
    if b is not None:
        out = out + b.reshape(1, Co, 1, 1)
    return np.ascontiguousarray(out)


def conv_transpose2d(g, K, stride, pad, in_hw):
    """Adjoint of conv2d (= F.conv_transpose2d with the output_padding that
    restores ``in_hw``)."""
    N, Co, Ho, Wo = g.shape
    _, Ci, kh, kw = K.shape
    H, W = in_hw
    gm = g.transpose(0, 2, 3, 1).reshape(N * Ho * Wo, Co)
    cols = (gm @ K.reshape(Co, -1)).reshape(N, Ho, Wo, Ci, kh, kw)
    Hp, Wp = H + 2 * pad[0], W + 2 * pad[1]
    Hp = max(Hp, (Ho - 1) * stride[0] + kh)
    Wp = max(Wp, (Wo - 1) * stride[1] + kw)
    out = np.zeros((N, Ci, Hp, Wp), dtype=g.dtype)
    for i in range(kh):
        for j in range(kw):
            out[:, :, i:i + stride[0] * Ho:stride[0],
                j:j + stride[1] * Wo:stride[1]] += \
                cols[:, :, :, :, i, j].transpose(0, 3, 1, 2)
    return np.ascontiguousarray(out[:, :, pad[0]:pad[0] + H, pad[1]:pad[1] + W])


# ---------------------------------------------------------------------------
# concrete forward  (verify_zono_bnb.py:554-596) and its vector-Jacobian product
# ---------------------------------------------------------------------------

def _point_bias(a, op, sign, dtype):
    """a + sign * bias with the reference's broadcast (_point_bcast_bias,
    verify_zono_bnb.py:525-551): scalar or full-width biases add elementwise,
    others right-align against the op's ``out_shape_nd``."""
    b = _np(op.get('bias'), dtype)
    if b is None:
        return a
    sb = b * dtype(sign)
    if b.size in (1, a.shape[1]):
        return a + sb.reshape(-1)
    N = a.shape[0]
    out_sh = tuple(int(d) for d in op['out_shape_nd'])
    if int(np.prod(out_sh)) != a.shape[1]:
        raise NotImplementedError('oracle forward: outer broadcast')
    return (a.reshape(N, *out_sh) + sb).reshape(N, -1)


def forward_batch_graph(x, gg, dtype=np.float32, capture=None, keep=False):
    """Concrete forward of N points (N, n_in) through fc / conv / relu /
    reshape / bias add-sub ops.  Returns the output (or ``capture``'s
    activation); with ``keep`` also {relu op name: its input}."""
    x = np.asarray(x, dtype)
    N = x.shape[0]
    act = {gg['input_name']: x.reshape(N, -1)}
    relu_in = {}
    out = act[gg['input_name']]
    for op in gg['ops']:
        t = op['type']
        a = act[op['inputs'][0]]
        if t == 'conv':
            p = op_arrays(op, dtype)
            v = conv2d(a.reshape(N, *op['in_shape']), p['K'], p['b'], op['stride'],
                       op['padding']).reshape(N, -1)
        elif t == 'fc':
            p = op_arrays(op, dtype)
            v = a @ p['W'].T + p['b']
        elif t == 'relu':
            relu_in[op['name']] = a
            v = np.maximum(a, 0)
        elif t == 'reshape':
            v = a
        elif t in ('add', 'sub') and not op.get('is_merge'):
            v = _point_bias(a, op, 1.0 if t == 'add' else -1.0, dtype)
        else:
            raise NotImplementedError(f'oracle forward: unsupported op {t!r}')
        act[op['name']] = v
        out = v
        if capture is not None and op['name'] == capture:
            break
    if capture is not None:
        out = act[capture]
    return (out, relu_in) if keep else out


def forward_vjp(gg, relu_in, g, dtype=np.float32):
    """d(g . f(x))/dx for a chain (autograd's rules: F.relu passes the
    gradient where its input is > 0)."""
    g = np.asarray(g, dtype)
    N = g.shape[0]
    for op in reversed(gg['ops']):
        t = op['type']
        if t == 'fc':
            g = g @ op_arrays(op, dtype)['W']
        elif t == 'conv':
            K = op_arrays(op, dtype)['K']
            ins = op['in_shape']
            Co, Ho, Wo = op['out_shape']
            g = conv_transpose2d(g.reshape(N, Co, Ho, Wo), K, op['stride'], op['padding'],
                                 ins[1:]).reshape(N, -1)
        elif t == 'relu':
            g = g * (relu_in[op['name']] > 0)
        elif t in ('reshape', 'add', 'sub'):
            pass
        else:
            raise NotImplementedError(f'oracle vjp: unsupported op {t!r}')
    return g


# ---------------------------------------------------------------------------
# ReLU slopes  (verify_zono_bnb.py:503-522)
# ---------------------------------------------------------------------------

def make_slopes(lo, hi):
    """CROWN adaptive slopes: returns (lo_s, up_s, up_t, active, dead, unstable).

    verify_zono_bnb.py:511-521 -- ``ub_r = max(max(hi,0), min(lo,0)+1e-8)``,
    ``up_s = ub_r/(ub_r-lb_r)``, ``up_t = -lb_r*up_s``, lower slope 1 where
    active, else (up_s > 0.5) for unstable, 0 for dead."""
    dt = lo.dtype
    lb_r = np.minimum(lo, dt.type(0))
    ub_r = np.maximum(hi, dt.type(0))
    ub_r = np.maximum(ub_r, lb_r + dt.type(1e-8))
    up_s = ub_r / (ub_r - lb_r)
    up_t = -lb_r * up_s
    active = lo >= 0
    dead = hi <= 0
    unstable = ~active & ~dead
    lm = active.astype(dt)
    um = dead.astype(dt)
    lo_s = (up_s > 0.5).astype(dt) * (1 - lm) * (1 - um) + lm
    return lo_s, up_s, up_t, active, dead, unstable


# ---------------------------------------------------------------------------
# IBP  (verify_zono_bnb.py:1066-1153)
# ---------------------------------------------------------------------------

def ibp_forward_batched(xl, xh, gg, relu_clamps=None, root_sb=None,
                        dtype=np.float32):
    """Batched interval forward; returns sb {layer_idx: (lo, hi)} (B, n).

    Mirrors ``_ibp_forward_graph_batched``: fc via mid/rad
    (verify_zono_bnb.py:1115-1120), relu applies root_sb then clamps then
    ``h = max(h, l)`` before recording (:1123-1138)."""
    xl = np.asarray(xl, dtype)
    xh = np.asarray(xh, dtype)
    B = xl.shape[0]
    lo = {gg['input_name']: xl}
    hi = {gg['input_name']: xh}
    sb = {}
    half = dtype(0.5) if isinstance(dtype, type) else np.dtype(dtype).type(0.5)
    for op in gg['ops']:
        t = op['type']
        name = op['name']
        l, h = lo[op['inputs'][0]], hi[op['inputs'][0]]
        if t == 'conv':
            a = op_arrays(op, dtype)
            mid, rad = (l + h) * half, (h - l) * half
            ins = op['in_shape']
            mc = conv2d(mid.reshape(B, *ins), a['K'], a['b'], op['stride'],
                        op['padding'])
            rc = conv2d(rad.reshape(B, *ins), np.abs(a['K']), None,
                        op['stride'], op['padding'])
            lo[name] = (mc - rc).reshape(B, -1)
            hi[name] = (mc + rc).reshape(B, -1)
        elif t == 'fc':
            a = op_arrays(op, dtype)
            mid, rad = (l + h) * half, (h - l) * half
            mc = mid @ a['W'].T + a['b']
            rc = rad @ np.abs(a['W']).T
            lo[name], hi[name] = mc - rc, mc + rc
        elif t == 'relu':
            L = op.get('layer_idx')
            if L is not None:
                if root_sb is not None and L in root_sb:
                    l = np.maximum(l, np.asarray(root_sb[L][0], dtype)[None])
                    h = np.minimum(h, np.asarray(root_sb[L][1], dtype)[None])
                if relu_clamps is not None and L in relu_clamps:
                    cl, ch = relu_clamps[L]
                    l = np.maximum(l, np.asarray(cl, dtype))
                    h = np.minimum(h, np.asarray(ch, dtype))
                h = np.maximum(h, l)
                sb[L] = (l.copy(), h.copy())
            lo[name], hi[name] = np.maximum(l, 0), np.maximum(h, 0)
        elif t == 'reshape':
            lo[name], hi[name] = l, h
        elif t == 'add':
            b = op_arrays(op, dtype)['b']
            lo[name], hi[name] = l + b, h + b
        elif t == 'sub':
            b = op_arrays(op, dtype)['b']
            lo[name], hi[name] = l - b, h - b
        else:
            raise NotImplementedError(f'oracle ibp: unsupported op {t!r}')
    return sb


# ---------------------------------------------------------------------------
# CROWN back-substitution  (verify_zono_bnb.py:4270-5134)
# ---------------------------------------------------------------------------

def spec_backward_batched(tight, xl, xh, gg, spec_W=None, spec_b=None,
                          return_input_linear=False, alpha=None, beta=None,
                          seed_ew_at=None, seed_acc=None, dtype=np.float32,
                          record=None):
    """Batched CROWN spec backward.  Returns lb (B,Q) [, A (B,Q,n_in), acc].

    spec_W (Q, n_out), spec_b (Q,) replace the reference's ``spec_ew`` dict
    (sorted-key order, verify_zono_bnb.py:4315-4321).  ``alpha`` {L: (B, n)}
    replaces the min-area lower slope for unstable neurons (:4420-4433);
    ``beta`` {L: (B, n)} adds the signed split multiplier to the
    pre-activation coefficient (:4448-4449).  ``record`` (dict) receives the
    per-relu incoming coefficients ``ew`` for the hand-written alpha adjoint.
    """
    xl = np.asarray(xl, dtype)
    xh = np.asarray(xh, dtype)
    ops = gg['ops']
    B, n_in = xl.shape
    if seed_ew_at is not None:
        ew_at = {k: np.array(v, dtype=dtype, copy=True)
                 for k, v in seed_ew_at.items()}
        Q = next(iter(ew_at.values())).shape[1]
        acc = (np.zeros((B, Q), dtype) if seed_acc is None
               else np.array(seed_acc, dtype=dtype, copy=True))
    else:
        W_q = np.asarray(spec_W, dtype)
        b_q = np.asarray(spec_b, dtype)
        Q = W_q.shape[0]
        ew_at = {ops[-1]['name']: np.broadcast_to(W_q, (B,) + W_q.shape).copy()}
        acc = np.broadcast_to(b_q, (B, Q)).copy()
    for op in reversed(ops):
        name = op['name']
        if name not in ew_at:
            continue
        ew = ew_at[name]
        t = op['type']
        if t == 'fc':
            a = op_arrays(op, dtype)
            acc = acc + ew @ a['b']
            ew_back = ew @ a['W']
        elif t == 'relu':
            if 'layer_idx' in op:
                L = op['layer_idx']
                lo, hi = tight[L]
                lo = np.asarray(lo, dtype)
                hi = np.asarray(hi, dtype)
                lo_s_def, up_s, up_t, active, dead, unstable = make_slopes(lo, hi)
                if record is not None:
                    record[L] = ew.copy()
                ep = np.maximum(ew, 0)
                en = np.minimum(ew, 0)
                acc = acc + (en * up_t[:, None, :]).sum(axis=-1)
                if alpha is not None and L in alpha:
                    aL = np.asarray(alpha[L], dtype)
                    lo_s = (active.astype(dtype) + unstable.astype(dtype) * aL)
                    ew_back = ep * lo_s[:, None, :] + en * up_s[:, None, :]
                else:
                    ew_back = ep * lo_s_def[:, None, :] + en * up_s[:, None, :]
                if beta is not None and L in beta:
                    ew_back = ew_back + np.asarray(beta[L], dtype)[:, None, :]
            else:
                ew_back = ew
        elif t == 'add':
            b = op_arrays(op, dtype)['b']
            if b is not None:
                acc = acc + (ew * b).sum(axis=-1)
            ew_back = ew.copy()
        elif t == 'sub':
            b = op_arrays(op, dtype)['b']
            if b is not None:
                acc = acc - (ew * b).sum(axis=-1)
            ew_back = ew.copy()
        elif t == 'reshape':
            ew_back = ew.copy()
        elif t == 'conv':
            a = op_arrays(op, dtype)
            Co, Ho, Wo = op['out_shape']
            bias_flat = np.repeat(a['b'], Ho * Wo)
            acc = acc + (ew * bias_flat).sum(axis=-1)
            ins = op['in_shape']
            g = conv_transpose2d(ew.reshape(B * Q, Co, Ho, Wo), a['K'],
                                 op['stride'], op['padding'], ins[1:])
            ew_back = g.reshape(B, Q, -1)
        else:
            raise ValueError(f'oracle spec backward: unknown op {t!r}')
        inp = op['inputs'][0]
        existing = ew_at.get(inp)
        ew_at[inp] = ew_back if existing is None else existing + ew_back
    ew_inp = ew_at.get(gg['input_name'])
    if ew_inp is None:
        if return_input_linear:
            return acc, np.zeros((B, Q, n_in), dtype), acc
        return acc
    pos = np.maximum(ew_inp, 0)
    neg = np.minimum(ew_inp, 0)
    lbs = (acc + (pos * xl[:, None, :]).sum(axis=-1)
           + (neg * xh[:, None, :]).sum(axis=-1))
    if return_input_linear:
        return lbs, ew_inp, acc
    return lbs


# ---------------------------------------------------------------------------
# Zonotope forward  (verify_zono_bnb.py:3079-4074)
# ---------------------------------------------------------------------------

def forward_zonotope_batched(xl, xh, gg, dtype=np.float32):
    """DeepZ forward.  Returns (sb, (c, G)) with G (B, n_out, K).

    Input generators: one column per input dim with a non-zero radius in any
    leaf (verify_zono_bnb.py:3098-3110).  ReLU: lambda = hi/(hi-lo),
    mu = -hi*lo/(2(hi-lo)) on unstable neurons, one compacted new generator
    column per unstable neuron, padded to the batch max (:3175-3211)."""
    xl = np.asarray(xl, dtype)
    xh = np.asarray(xh, dtype)
    B, n_in = xl.shape
    half = np.dtype(dtype).type(0.5)
    c = (xl + xh) / 2
    radii = (xh - xl) / 2
    varying = np.abs(radii).max(axis=0) > 0
    var_idx = np.nonzero(varying)[0]
    K = var_idx.size
    G = np.zeros((B, n_in, K), dtype)
    G[:, var_idx, np.arange(K)] = radii[:, var_idx]
    state = {gg['input_name']: (c, G)}
    sb = {}
    for op in gg['ops']:
        name = op['name']
        t = op['type']
        c_in, G_in = state[op['inputs'][0]]
        if t == 'fc':
            a = op_arrays(op, dtype)
            c_out = c_in @ a['W'].T + a['b']
            G_out = np.einsum('oi,bik->bok', a['W'], G_in)
            state[name] = (c_out, G_out)
        elif t == 'relu':
            abs_sum = np.abs(G_in).sum(axis=2)
            lo = c_in - abs_sum
            hi = c_in + abs_sum
            ust = (lo < 0) & (hi > 0)
            dead = hi <= 0
            with np.errstate(divide='ignore', invalid='ignore'):
                lam = np.where(ust, hi / (hi - lo),
                               np.where(dead, 0, 1)).astype(dtype)
                mu = np.where(ust, -hi * lo / (2 * (hi - lo)), 0).astype(dtype)
            c_out = lam * c_in + mu
            G_scaled = G_in * lam[:, :, None]
            cnt = ust.sum(axis=1)
            max_k = int(cnt.max()) if B else 0
            if max_k == 0:
                G_out = G_scaled
            else:
                n = c_in.shape[1]
                new = np.zeros((B, n, max_k), dtype)
                rank = np.cumsum(ust, axis=1) - 1
                bi, ri = np.nonzero(ust)
                new[bi, ri, rank[bi, ri]] = mu[bi, ri]
                G_out = np.concatenate([G_scaled, new], axis=2)
            state[name] = (c_out, G_out)
            if 'layer_idx' in op:
                sb[op['layer_idx']] = (lo.copy(), hi.copy())
        elif t == 'reshape':
            state[name] = (c_in, G_in)
        elif t == 'add':
            b = op_arrays(op, dtype)['b']
            state[name] = (c_in + b if b is not None else c_in, G_in)
        elif t == 'sub':
            b = op_arrays(op, dtype)['b']
            state[name] = (c_in - b if b is not None else c_in, G_in)
        elif t == 'conv':
            a = op_arrays(op, dtype)
            ins = op['in_shape']
            c_out = conv2d(c_in.reshape(B, *ins), a['K'], a['b'], op['stride'],
                           op['padding']).reshape(B, -1)
            Kg = G_in.shape[2]
            if Kg == 0:
                G_out = np.zeros((B, c_out.shape[1], 0), dtype)
            else:
                gp = G_in.transpose(0, 2, 1).reshape(B * Kg, *ins)
                go = conv2d(gp, a['K'], None, op['stride'], op['padding'])
                G_out = go.reshape(B, Kg, -1).transpose(0, 2, 1).copy()
            state[name] = (c_out, G_out)
        else:
            raise ValueError(f'oracle zonotope: unknown op type {t!r}')
    _ = half
    return sb, state[gg['ops'][-1]['name']]


# ---------------------------------------------------------------------------
# CROWN intermediate bounds  (verify_zono_bnb.py:4077-4147)
# ---------------------------------------------------------------------------

def crown_intermediate_batched(gg, xl, xh, chunk=2048, dtype=np.float32,
                               sb=None):
    """Backward-CROWN pre-ReLU bounds intersected with the zonotope bounds.

    Seeds ``[+e_j; -e_j]`` at each ReLU's feeding op for the neurons unstable
    in ANY leaf of the batch (verify_zono_bnb.py:4123), walks back to the
    input through the earlier layers' already-tightened relaxations, and
    intersects (:4142-4145)."""
    xl = np.asarray(xl, dtype)
    xh = np.asarray(xh, dtype)
    if sb is None:
        sb, _ = forward_zonotope_batched(xl, xh, gg, dtype)
    tight = {L: (lo.copy(), hi.copy()) for L, (lo, hi) in sb.items()}
    relu_op_by_L = {op['layer_idx']: op for op in gg['ops']
                    if op['type'] == 'relu' and 'layer_idx' in op}
    B = xl.shape[0]
    for L in sorted(tight):
        if L not in relu_op_by_L:
            continue
        feed = relu_op_by_L[L]['inputs'][0]
        lo_L, hi_L = tight[L]
        n = lo_L.shape[1]
        idx = np.nonzero(((lo_L < 0) & (hi_L > 0)).any(axis=0))[0]
        m = idx.size
        if m == 0:
            continue
        new_lo = lo_L.copy()
        new_hi = hi_L.copy()
        for c0 in range(0, m, max(1, int(chunk))):
            cidx = idx[c0:c0 + chunk]
            k = cidx.size
            eye = np.zeros((k, n), dtype)
            eye[np.arange(k), cidx] = 1
            seed = np.broadcast_to(np.concatenate([eye, -eye], 0),
                                   (B, 2 * k, n))
            sl = spec_backward_batched(tight, xl, xh, gg, seed_ew_at={feed: seed},
                                       seed_acc=np.zeros((B, 2 * k), dtype),
                                       dtype=dtype)
            lo_c = np.maximum(lo_L[:, cidx], sl[:, :k])
            hi_c = np.maximum(np.minimum(hi_L[:, cidx], -sl[:, k:]), lo_c)
            new_lo[:, cidx] = lo_c
            new_hi[:, cidx] = hi_c
        tight[L] = (new_lo, new_hi)
    return tight


# ---------------------------------------------------------------------------
# Halfspace box clip  (verify_graph.py:12363-12426)
# ---------------------------------------------------------------------------

def clip_box_by_halfspaces_batched(xl, xh, A, b):
    """Per-(query, dim) projection of {A_q.x + b_q <= 0} onto the box."""
    dt = xl.dtype.type
    A_pos = np.maximum(A, 0)
    A_neg = np.minimum(A, 0)
    total_min = ((A_pos * xl[:, None, :]).sum(axis=-1)
                 + (A_neg * xh[:, None, :]).sum(axis=-1))
    contrib = A_pos * xl[:, None, :] + A_neg * xh[:, None, :]
    L_other = total_min[..., None] - contrib
    A_nz = np.abs(A) > dt(1e-12)
    A_safe = np.where(A_nz, A, dt(1))
    threshold = (-b[..., None] - L_other) / A_safe
    pos_mask = A > dt(1e-12)
    neg_mask = A < dt(-1e-12)
    xh_per_q = np.where(pos_mask, threshold, xh[:, None, :])
    xl_per_q = np.where(neg_mask, threshold, xl[:, None, :])
    xh_new = np.minimum(xh_per_q.min(axis=1), xh)
    xl_new = np.maximum(xl_per_q.max(axis=1), xl)
    halfspace_empty = (total_min + b > 0).any(axis=1)
    box_empty = (xl_new > xh_new).any(axis=-1)
    feasible = ~(halfspace_empty | box_empty)
    return xl_new, xh_new, feasible


# ---------------------------------------------------------------------------
# alpha-CROWN  (verify_zono_bnb.py:5137-5288, verify_milp.py:2762-2807)
# ---------------------------------------------------------------------------

def alpha_grad(tight, xl, xh, gg, spec_W, spec_b, alpha, dtype=np.float32,
               beta=None):
    """lb and d(sum lb)/d(alpha) by a hand-written adjoint (MLP graphs).

    Reproduces torch autograd through ``_spec_backward_graph_batched``:
    clamp(min=0)/clamp(max=0) both pass gradient at exactly 0, so the
    derivative of pos(e)*x + neg(e)*y at e == 0 is x + y."""
    rec = {}
    lb = spec_backward_batched(tight, xl, xh, gg, spec_W, spec_b,
                               alpha=alpha, beta=beta, dtype=dtype, record=rec)
    xl = np.asarray(xl, dtype)
    xh = np.asarray(xh, dtype)
    ops = gg['ops']
    # forward-in-adjoint: walk input -> output
    # g = d(sum lb)/d(ew at current point)
    B = xl.shape[0]
    ew_in_rec = None
    # recompute ew at the input from the recorded first relu output: easier to
    # rerun the primal from the lowest relu.
    relu_ops = [op for op in ops if op['type'] == 'relu' and 'layer_idx' in op]
    fcs = [op for op in ops if op['type'] == 'fc']
    if len(fcs) != len(relu_ops) + 1 or any(
            op['type'] not in ('fc', 'relu') for op in ops):
        raise NotImplementedError('alpha_grad oracle: fc/relu chains only')
    Ls = [op['layer_idx'] for op in relu_ops]
    # primal ew at input
    L0 = Ls[0]
    lo, hi = tight[L0]
    lo_s_def, up_s, up_t, active, dead, unstable = make_slopes(
        np.asarray(lo, dtype), np.asarray(hi, dtype))
    ew = rec[L0]
    if alpha is not None and L0 in alpha:
        lo_s = active.astype(dtype) + unstable.astype(dtype) * np.asarray(alpha[L0], dtype)
    else:
        lo_s = lo_s_def
    e_after = np.maximum(ew, 0) * lo_s[:, None, :] + np.minimum(ew, 0) * up_s[:, None, :]
    if beta is not None and L0 in beta:
        e_after = e_after + np.asarray(beta[L0], dtype)[:, None, :]
    W0 = op_arrays(fcs[0], dtype)['W']
    ew_in_rec = e_after @ W0
    g = (np.where(ew_in_rec >= 0, xl[:, None, :], 0)
         + np.where(ew_in_rec <= 0, xh[:, None, :], 0)).astype(dtype)
    grads = {}
    for i, L in enumerate(Ls):
        W = op_arrays(fcs[i], dtype)['W']
        bvec = op_arrays(fcs[i], dtype)['b']
        # d/d(e_after_L): ew_back = e_after @ W, acc += e_after . b
        g_after = g @ W.T + bvec
        lo, hi = tight[L]
        lo_s_def, up_s, up_t, active, dead, unstable = make_slopes(
            np.asarray(lo, dtype), np.asarray(hi, dtype))
        if alpha is not None and L in alpha:
            lo_s = active.astype(dtype) + unstable.astype(dtype) * np.asarray(alpha[L], dtype)
        else:
            lo_s = lo_s_def
        e = rec[L]
        pmask = (e >= 0).astype(dtype)
        nmask = (e <= 0).astype(dtype)
        grads[L] = ((np.maximum(e, 0) * g_after).sum(axis=1)
                    * unstable.astype(dtype))
        g = (pmask * lo_s[:, None, :] * g_after
             + nmask * (up_s[:, None, :] * g_after + up_t[:, None, :]))
    return lb, grads


class Adam:
    """torch.optim.Adam (defaults betas=(0.9,0.999), eps=1e-8) restated."""

    def __init__(self, params, lr, dtype=np.float32):
        self.p = params
        self.lr = lr
        self.t = 0
        self.m = {k: np.zeros_like(v) for k, v in params.items()}
        self.v = {k: np.zeros_like(v) for k, v in params.items()}
        self.dt = np.dtype(dtype).type

    def step(self, grads):
        dt = self.dt
        self.t += 1
        b1, b2, eps = dt(0.9), dt(0.999), dt(1e-8)
        bc1 = 1 - 0.9 ** self.t
        bc2 = 1 - 0.999 ** self.t
        step_size = dt(self.lr / bc1)
        bc2_sqrt = dt(np.sqrt(bc2))
        for k in self.p:
            g = grads[k]
            self.m[k] = self.m[k] * b1 + g * (1 - b1)
            self.v[k] = self.v[k] * b2 + (g * g) * (1 - b2)
            denom = np.sqrt(self.v[k]) / bc2_sqrt + eps
            self.p[k] = self.p[k] - step_size * (self.m[k] / denom)


def alpha_crown_inputsplit_batched(xl, xh, gg, spec_W, spec_b, n_iters=10,
                                   lr=0.25, lr_decay=0.98, early_stop_eps=1e-6,
                                   dtype=np.float32, sb_init=None):
    """Batched alpha-CROWN on input-split leaves (verify_zono_bnb.py:5137-5288).

    Intermediates: forward zonotope (:5166-5168).  alpha init = min-area
    choice on unstable neurons (:5170-5173).  Adam on -sum(lb), clamp to
    [0,1], best-of-iterations lb, early stop when all lb > 0 or the batch max
    improves by < eps, lr decay per iteration (:5248-5288)."""
    xl = np.asarray(xl, dtype)
    xh = np.asarray(xh, dtype)
    if sb_init is None:
        sb_init, _ = forward_zonotope_batched(xl, xh, gg, dtype)
    alpha = {}
    for L, (lo, hi) in sb_init.items():
        _, up_s, _, active, dead, unstable = make_slopes(lo, hi)
        alpha[L] = ((up_s > 0.5).astype(dtype) * unstable.astype(dtype))
    opt = Adam(alpha, lr, dtype)
    best = None
    prev_max = -np.inf
    for it in range(n_iters):
        lb, grads = alpha_grad(sb_init, xl, xh, gg, spec_W, spec_b, opt.p,
                               dtype)
        best = lb.copy() if best is None else np.maximum(best, lb)
        curr_max = float(best.max())
        if (best > 0).all():
            break
        # loss = -sum(lb): gradient is -grads
        opt.step({L: -g for L, g in grads.items()})
        for L in opt.p:
            opt.p[L] = np.clip(opt.p[L], 0, 1).astype(dtype)
        if it > 0 and curr_max - prev_max < early_stop_eps:
            break
        prev_max = curr_max
        opt.lr *= lr_decay
    return best


def alpha_beta_crown_domains(xl, xh, gg, spec_W, spec_b, relu_clamps,
                             n_iters=20, lr=0.1, dtype=np.float32):
    """alpha-CROWN for ReLU-split domains with beta = 0 (cfg3 oracle).

    Follows the alpha loop of ``_ibp_crown_bab`` (verify_milp.py:2762-2807)
    with beta fixed at zero: per-domain IBP intermediates under the split
    clamps, min-area alpha init, Adam (no lr decay) on -sum(lb), clamp to
    [0,1], best-of-iterations lb.  xl/xh are (D, n_in)."""
    xl = np.asarray(xl, dtype)
    xh = np.asarray(xh, dtype)
    sb = ibp_forward_batched(xl, xh, gg, relu_clamps=relu_clamps, dtype=dtype)
    alpha = {}
    for L, (lo, hi) in sb.items():
        _, up_s, _, active, dead, unstable = make_slopes(lo, hi)
        alpha[L] = ((up_s > 0.5).astype(dtype) * unstable.astype(dtype))
    opt = Adam(alpha, lr, dtype)
    best = None
    for it in range(max(1, n_iters)):
        lb, grads = alpha_grad(sb, xl, xh, gg, spec_W, spec_b, opt.p, dtype)
        best = lb.copy() if best is None else np.maximum(best, lb)
        if (best > 0).all():
            break
        opt.step({L: -g for L, g in grads.items()})
        for L in opt.p:
            opt.p[L] = np.clip(opt.p[L], 0, 1).astype(dtype)
    return best, sb
