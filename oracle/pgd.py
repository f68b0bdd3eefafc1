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

``pgd_attack_general`` restates ``pgd_attack_general`` (``pgd.py:233-524``)
with its optimiser ``_PGDOptim`` (:127-187) and margin rows
``_build_constraint_matrices`` (:75-118).  Test infrastructure only: nothing
in the product imports this module.
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
    fwd, bwd = _net_fns(gg, dtype)
    x = np.asarray(x0, dtype).copy()
    lo = np.asarray(lo, dtype)
    hi = np.asarray(hi, dtype)
    width = hi - lo
    lr = dtype(lr)
    for it in range(n_iter):
        out, acts = fwd(x)
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
        g = bwd(acts, g)
        step = lr * np.sign(g) * width
        x = np.maximum(np.minimum(x - step, hi), lo)
    return False, None, n_iter


def _forward_acts(layers, x):
    """Forward pass keeping the pre-activations of the hidden layers."""
    acts = []
    a = x
    for i, (W, b) in enumerate(layers):
        z = a @ W.T + b
        if i < len(layers) - 1:
            acts.append(z)
            a = np.maximum(z, 0)
        else:
            a = z
    return a, acts


def _backward(layers, acts, g):
    """d(g . f(x))/dx with autograd's ReLU rule (gradient where z > 0)."""
    for i in range(len(layers) - 1, -1, -1):
        W, _ = layers[i]
        g = g @ W
        if i > 0:
            g = g * (acts[i - 1] > 0)
    return g


def _net_fns(gg, dtype):
    """(forward(x) -> (out, acts), backward(acts, g) -> dx): the MLP
    matrices for fc/relu chains, the graph walker (conv, bias ops) else."""
    try:
        layers = _mlp_layers(gg, dtype)
    except NotImplementedError:
        return (lambda x: ob.forward_batch_graph(x, gg, dtype, keep=True),
                lambda acts, g: ob.forward_vjp(gg, acts, g, dtype))
    return (lambda x: _forward_acts(layers, x), lambda acts, g: _backward(layers, acts, g))


def _fma32(a, b, c):
    """fl32(a * b + c) with one rounding of the exact product (float64 holds
    the product of two float32 values exactly)."""
    return (a.astype(np.float64) * np.float64(b) + c.astype(np.float64)).astype(np.float32)


def pgd_attack_general(xl, xh, gg, disjuncts, x_init, w_d=None, *, n_iter=100,
                       lr_decay=0.99, hinge_thr=-1e-5, alpha_frac=0.25,
                       alpha_fracs=None, optim='adam_clipping', osi_iters=50,
                       plateau_iters=100, per_restart_disj=False, active=None,
                       div='cuda', max_iters=None):
    """Restatement of ``pgd_attack_general`` (pgd.py:233-524) in float32.

    xl, xh (n_in,): the (already widened) search box.  disjuncts: the spec's
    DNF in the tuple form of ``margin_matrices``.  x_init (R, n_in): the
    restarts' uniform draw (pgd.py:375); w_d (R, n_out): the OSI projection
    draw (pgd.py:384) or None for ``pgd_init_mode='uniform'``.  ``active``:
    indices of the disjuncts to attack (``restrict_disj``), None = all.
    ``alpha_fracs``: the multi-alpha list (pgd.py:306-321), None = single
    ``alpha_frac``.  ``div``: how ``base_step / bc1`` rounds -- 'cuda'
    multiplies by the float32 reciprocal (ATen's scalar-divisor path on the
    GPU), 'cpu' divides.  ``max_iters`` stops the loop early without a final
    screen (trajectory comparisons only).

    Returns (sat, witness or None, info) with info = dict(t=screen index of
    the witness, x=final iterate).
    """
    f32 = np.float32
    fwd, bwd = _net_fns(gg, f32)
    xl = np.asarray(xl, f32).reshape(-1)
    xh = np.asarray(xh, f32).reshape(-1)
    x = np.asarray(x_init, f32).copy()
    R = x.shape[0]
    n_out = fwd(x[:1])[0].shape[1]
    mats_all = margin_matrices(disjuncts, n_out, f32)
    act_idx = list(range(len(disjuncts))) if active is None else sorted(active)
    act_idx = [d for d in act_idx if len(disjuncts[d])]
    mats = [mats_all[d] for d in act_idx]
    if not mats:
        return False, None, {'t': None, 'x': x}
    eps_input = (xh - xl) / f32(2.0)
    if alpha_fracs is not None:
        pra = np.asarray([alpha_fracs[i % len(alpha_fracs)] for i in range(R)], f32)
        step0 = eps_input[None, :] * pra[:, None]
    else:
        step0 = np.broadcast_to(eps_input * f32(alpha_frac), x.shape).astype(f32)
    # OSI init (pgd.py:378-402): ascend w_d . f(x) with sign steps
    if w_d is not None:
        w_d = np.asarray(w_d, f32)
        for _ in range(osi_iters):
            _, acts = fwd(x)
            g = bwd(acts, w_d)
            x = np.minimum(np.maximum(x + step0 * np.sign(g).astype(f32), xl), xh)
    n_act = len(mats)
    prd = bool(per_restart_disj) and n_act > 1
    assign = np.arange(R) % n_act

    def screen(out):
        """Index of the first confirmed witness (pgd.py:443-451) or None."""
        flat = np.concatenate([out @ W.T + b for W, b in mats], axis=1)
        cand = flat.min(axis=1) <= 0
        for bi in np.nonzero(cand)[0]:
            worst = min(float((out[bi] @ W.T + b).max()) for W, b in mats_all
                        if W.shape[0])
            if worst <= 0.0:
                return int(bi), flat
        return None, flat

    m1 = np.zeros_like(x)
    m2 = np.zeros_like(x)
    cur = step0.copy()
    best_min = float('inf')
    nimp = 0
    b1, b2, eps_a = 0.9, 0.999, 1e-8
    t_run = 0
    for t in range(1, n_iter + 1):
        if max_iters is not None and t > max_iters:
            return False, None, {'t': None, 'x': x}
        out, acts = fwd(x)
        bi, flat = screen(out)
        if bi is not None:
            return True, x[bi].copy(), {'t': t, 'x': x}
        curr_min = float(flat.min())
        if curr_min > hinge_thr:
            if curr_min < best_min - 1e-6:
                best_min = curr_min
                nimp = 0
            else:
                nimp += 1
            if nimp >= plateau_iters:
                break
        else:
            nimp = 0
        # d/dy of sum clamp(margin, min=thr): rows with margin >= thr
        g = np.zeros_like(out)
        col = 0
        for d, (W, b) in enumerate(mats):
            m = flat[:, col:col + W.shape[0]]
            sel = (m >= f32(hinge_thr)).astype(f32)
            if prd:
                sel = sel * (assign == d)[:, None]
            g = g + sel @ W
            col += W.shape[0]
        grad = bwd(acts, g)
        t_run = t
        if optim == 'sign_sgd':
            delta = cur * np.sign(grad).astype(f32)
        else:
            m1 = _fma32(grad, f32(1 - b1), (m1 * f32(b1)).astype(f32))
            m2 = _fma32(grad * grad, f32(1 - b2), (m2 * f32(b2)).astype(f32))
            bc1 = 1.0 - b1 ** t
            bc2 = 1.0 - b2 ** t
            denom = np.sqrt(m2) / f32(bc2 ** 0.5) + f32(eps_a)
            direction = np.sign(m1 / denom).astype(f32)
            if optim == 'adam_sign':
                delta = cur * direction
            elif div == 'cuda':
                delta = (cur * (f32(1.0) / f32(bc1))) * direction
            else:
                delta = (cur / f32(bc1)) * direction
        x = np.minimum(np.maximum(x - delta, xl), xh)
        cur = cur * f32(lr_decay)
    out, _ = fwd(x)
    bi, _ = screen(out)
    if bi is not None:
        return True, x[bi].copy(), {'t': t_run + 1, 'x': x}
    return False, None, {'t': None, 'x': x}
