"""Seeded synthetic workloads for the bound-propagation path.

Every network, input box and spec used by the tests and by ``bench.py`` is
built here from ``numpy.random.default_rng(seed)``.  Draw order per layer is
``W_l`` then ``b_l`` (He-normal weights ``N(0, 2/fan_in)``, biases
``N(0, 0.01^2)``), then the input box / points, all cast to fp32.

The returned ``gg`` dicts use the reference's op-dict schema
(``vibecheck/network.py:1707-2910``: ``{'ops': [...], 'input_name', 'fork_points',
'relu_names', 'n_relu', 'input_n', 'input_shape'}`` with ``fc`` ops carrying
``W``/``bias`` torch tensors and ``W_np``/``bias_np`` float64 copies, ``relu``
ops carrying ``layer_idx``, ``conv`` ops carrying ``kernel``/``bias``/
``in_shape``/``out_shape``/``stride``/``padding``/``output_padding``), so the
same dict drives the reference, the oracle and this package.

Configurations (the reference has no public dataset for this path, so these
seeded inputs stand in for its benchmarks):

* cfg1 -- 5->[50]x6->5 MLP, one box (centre U(-0.5,0.5), half-width
  U(0.05,0.5)), spec ``y0 - y1 <= d`` folded into the last bias.
* cfg2 -- same MLP, 65,536 sub-boxes (half-widths U(0.001,0.1)), 4 spec rows
  with coefficients in {-1,0,1}.
* cfg3 -- 784->[256]x6->10 MLP, eps=0.03 ball, 9 margin rows, 1024 ReLU-split
  domains.
* cfg4 -- CNN 3x32x32 -> conv16 -> conv32 -> fc100 -> fc10, eps=2/255, 9
  margin rows, 256 ReLU-split domains.
* cfg5 -- 3072->[1024]x8->10 MLP, eps=1/255, 9 margin rows.
"""
from __future__ import annotations

import numpy as np
import torch

ACAS_DIMS = (5, 50, 50, 50, 50, 50, 50, 5)
CFG3_DIMS = (784, 256, 256, 256, 256, 256, 256, 10)
CFG5_DIMS = (3072,) + (1024,) * 8 + (10,)


# ---------------------------------------------------------------------------
# networks
# ---------------------------------------------------------------------------

def mlp_params(dims, rng):
    """He-normal fp32 weights and N(0, 0.01^2) biases, drawn W_l then b_l."""
    layers = []
    for i in range(len(dims) - 1):
        fan_in, fan_out = dims[i], dims[i + 1]
        W = (rng.standard_normal((fan_out, fan_in)) * np.sqrt(2.0 / fan_in))
        b = rng.standard_normal(fan_out) * 0.01
        layers.append((W.astype(np.float32), b.astype(np.float32)))
    return layers


def mlp_gg(layers, device='cpu', dtype=torch.float32, input_name='x'):
    """Reference-schema op dict for an fc/relu chain (last fc has no relu)."""
    ops = []
    prev = input_name
    relu_names = []
    for i, (W, b) in enumerate(layers):
        name = f'fc{i}'
        ops.append({
            'name': name, 'type': 'fc', 'inputs': [prev],
            'W': torch.as_tensor(np.asarray(W), dtype=dtype, device=device),
            'bias': torch.as_tensor(np.asarray(b), dtype=dtype, device=device),
            'W_np': np.asarray(W, np.float64),
            'bias_np': np.asarray(b, np.float64),
        })
        prev = name
        if i < len(layers) - 1:
            rname = f'relu{i}'
            ops.append({'name': rname, 'type': 'relu', 'inputs': [prev],
                        'layer_idx': i})
            relu_names.append(rname)
            prev = rname
    n_in = int(np.asarray(layers[0][0]).shape[1])
    return {
        'ops': ops, 'relu_names': relu_names, 'fork_points': set(),
        'n_relu': len(relu_names), 'input_name': input_name,
        'input_n': n_in, 'input_shape': (n_in,),
    }


def conv_out_hw(h, w, k, stride, pad):
    return ((h + 2 * pad[0] - k[0]) // stride[0] + 1,
            (w + 2 * pad[1] - k[1]) // stride[1] + 1)


def cnn_cfg4_params(rng):
    """cfg4 CNN: conv(3->16,4x4,s2,p1) relu conv(16->32,4x4,s2,p1) relu
    flatten fc(2048->100) relu fc(100->10).  He-normal (fan_in = C_in*kh*kw)."""
    spec = []
    c1 = rng.standard_normal((16, 3, 4, 4)) * np.sqrt(2.0 / (3 * 16))
    b1 = rng.standard_normal(16) * 0.01
    c2 = rng.standard_normal((32, 16, 4, 4)) * np.sqrt(2.0 / (16 * 16))
    b2 = rng.standard_normal(32) * 0.01
    W3 = rng.standard_normal((100, 2048)) * np.sqrt(2.0 / 2048)
    b3 = rng.standard_normal(100) * 0.01
    W4 = rng.standard_normal((10, 100)) * np.sqrt(2.0 / 100)
    b4 = rng.standard_normal(10) * 0.01
    for a in (c1, b1, c2, b2, W3, b3, W4, b4):
        spec.append(a.astype(np.float32))
    return spec


def cnn_gg(params, device='cpu', dtype=torch.float32, input_name='x',
           in_shape=(3, 32, 32)):
    """Reference-schema op dict for the cfg4 CNN (conv/relu/reshape/fc)."""
    c1, b1, c2, b2, W3, b3, W4, b4 = params
    ops = []
    shape = tuple(in_shape)
    prev = input_name
    relu_i = 0
    relu_names = []
    for ci, (k, b) in enumerate(((c1, b1), (c2, b2))):
        stride, pad = (2, 2), (1, 1)
        Ho, Wo = conv_out_hw(shape[1], shape[2], k.shape[2:], stride, pad)
        out_shape = (k.shape[0], Ho, Wo)
        oph = shape[1] - ((Ho - 1) * stride[0] - 2 * pad[0] + k.shape[2])
        opw = shape[2] - ((Wo - 1) * stride[1] - 2 * pad[1] + k.shape[3])
        name = f'conv{ci}'
        ops.append({
            'name': name, 'type': 'conv', 'inputs': [prev],
            'kernel': torch.as_tensor(k, dtype=dtype, device=device),
            'bias': torch.as_tensor(b, dtype=dtype, device=device),
            'kernel_np': k.astype(np.float64), 'bias_np': b.astype(np.float64),
            'in_shape': shape, 'out_shape': out_shape,
            'stride': stride, 'padding': pad, 'output_padding': (oph, opw),
            'n_out': int(np.prod(out_shape)),
        })
        rname = f'relu{relu_i}'
        ops.append({'name': rname, 'type': 'relu', 'inputs': [name],
                    'layer_idx': relu_i})
        relu_names.append(rname)
        relu_i += 1
        prev = rname
        shape = out_shape
    ops.append({'name': 'flat', 'type': 'reshape', 'inputs': [prev]})
    prev = 'flat'
    for li, (W, b) in enumerate(((W3, b3), (W4, b4))):
        name = f'fc{li}'
        ops.append({
            'name': name, 'type': 'fc', 'inputs': [prev],
            'W': torch.as_tensor(W, dtype=dtype, device=device),
            'bias': torch.as_tensor(b, dtype=dtype, device=device),
            'W_np': W.astype(np.float64), 'bias_np': b.astype(np.float64),
        })
        prev = name
        if li == 0:
            rname = f'relu{relu_i}'
            ops.append({'name': rname, 'type': 'relu', 'inputs': [name],
                        'layer_idx': relu_i})
            relu_names.append(rname)
            relu_i += 1
            prev = rname
    n_in = int(np.prod(in_shape))
    return {
        'ops': ops, 'relu_names': relu_names, 'fork_points': set(),
        'n_relu': len(relu_names), 'input_name': input_name,
        'input_n': n_in, 'input_shape': (1,) + tuple(in_shape),
    }


def gg_to(gg, device, dtype=torch.float32):
    """Copy of a reference-schema gg with its tensors moved to device/dtype."""
    out = dict(gg)
    ops = []
    for op in gg['ops']:
        o = dict(op)
        for k in ('W', 'bias', 'kernel'):
            if isinstance(o.get(k), torch.Tensor):
                o[k] = o[k].to(device=device, dtype=dtype)
        ops.append(o)
    out['ops'] = ops
    out['fork_points'] = set(gg['fork_points'])
    return out


def spec_ew_from(W_q, b_q, device='cpu', dtype=torch.float32):
    """Reference ``spec_ew`` dict {q: (w (n_out,), bias float)}."""
    W_q = np.asarray(W_q)
    return {q: (torch.as_tensor(W_q[q], dtype=dtype, device=device),
                float(b_q[q])) for q in range(W_q.shape[0])}


def margin_rows(n_out, true_label):
    """9 rows y_true - y_j (j != true) with zero bias."""
    rows = []
    for j in range(n_out):
        if j == true_label:
            continue
        w = np.zeros(n_out, np.float32)
        w[true_label] = 1.0
        w[j] = -1.0
        rows.append(w)
    return np.stack(rows), np.zeros(len(rows), np.float32)


# ---------------------------------------------------------------------------
# configurations
# ---------------------------------------------------------------------------

def cfg2(seed=0, n_boxes=65536, n_q=4):
    """CROWN microbench: ACAS-shaped MLP, many small boxes, {-1,0,1} spec."""
    rng = np.random.default_rng(seed)
    layers = mlp_params(ACAS_DIMS, rng)
    n_in = ACAS_DIMS[0]
    centre = rng.uniform(-0.5, 0.5, (n_boxes, n_in))
    half = rng.uniform(0.001, 0.1, (n_boxes, n_in))
    xl = (centre - half).astype(np.float32)
    xh = (centre + half).astype(np.float32)
    C = rng.integers(-1, 2, (n_q, ACAS_DIMS[-1])).astype(np.float32)
    bq = np.zeros(n_q, np.float32)
    return {'layers': layers, 'xl': xl, 'xh': xh, 'spec_W': C, 'spec_b': bq,
            'name': f'cfg2 acas-mlp 5x[50]x6x5 crown B={n_boxes} Q={n_q}'}


def _mlp_forward64(layers, x):
    a = x
    for i, (W, b) in enumerate(layers):
        a = a @ W.astype(np.float64).T + b.astype(np.float64)
        if i < len(layers) - 1:
            a = np.maximum(a, 0.0)
    return a


def _margin_ascent64(layers, xl, xh, w_out, seed, n_restarts=10000, n_iter=50,
                     lr=0.1):
    """Sign-gradient ascent of w_out . y over the box in float64 (numpy RNG).

    Returns the largest value seen.  Used only to place the spec threshold
    so that the cfg1 property holds with a margin."""
    rng = np.random.default_rng(seed + 1_000_003)
    width = xh - xl
    x = xl + width * rng.random((n_restarts, xl.size))
    best = -np.inf
    Ws = [W.astype(np.float64) for W, _ in layers]
    bs = [b.astype(np.float64) for _, b in layers]
    for _ in range(n_iter + 1):
        acts = [x]
        masks = []
        a = x
        for i in range(len(Ws)):
            a = a @ Ws[i].T + bs[i]
            if i < len(Ws) - 1:
                masks.append(a > 0)
                a = np.maximum(a, 0.0)
            acts.append(a)
        val = a @ w_out
        best = max(best, float(val.max()))
        g = np.broadcast_to(w_out, a.shape).copy()
        for i in range(len(Ws) - 1, -1, -1):
            g = g @ Ws[i]
            if i > 0:
                g = g * masks[i - 1]
        x = np.clip(x + lr * np.sign(g) * width, xl, xh)
    return best


def cfg1(seed=0):
    """Small input-split BaB: one box, spec y0 - y1 <= d (holds by margin 0.5).

    ``d`` is folded into the last-layer bias (b0 <- b0 - d) so the spec is the
    pairwise query ``y1' - y0' > 0``: w = e1 - e0, b = 0."""
    rng = np.random.default_rng(seed)
    layers = mlp_params(ACAS_DIMS, rng)
    n_in = ACAS_DIMS[0]
    centre = rng.uniform(-0.5, 0.5, n_in)
    half = rng.uniform(0.05, 0.5, n_in)
    xl = (centre - half).astype(np.float32)
    xh = (centre + half).astype(np.float32)
    w_out = np.zeros(ACAS_DIMS[-1])
    w_out[0], w_out[1] = 1.0, -1.0
    m = _margin_ascent64(layers, xl.astype(np.float64), xh.astype(np.float64),
                         w_out, seed)
    d = np.float32(m + 0.5)
    W_last, b_last = layers[-1]
    b_last = b_last.copy()
    b_last[0] = np.float32(b_last[0] - d)
    layers = layers[:-1] + [(W_last, b_last)]
    spec_W = np.zeros((1, ACAS_DIMS[-1]), np.float32)
    spec_W[0, 1], spec_W[0, 0] = 1.0, -1.0
    return {'layers': layers, 'xl': xl, 'xh': xh, 'spec_W': spec_W,
            'spec_b': np.zeros(1, np.float32), 'd': float(d),
            'name': 'cfg1 acas-mlp 5x[50]x6x5 input-split BaB y0-y1<=d'}


def cfg3(seed=0, n_domains=1024, n_split=10, eps=0.03):
    """alpha-CROWN on 784->[256]x6->10 with 2^n_split ReLU-split domains."""
    rng = np.random.default_rng(seed)
    layers = mlp_params(CFG3_DIMS, rng)
    x0 = rng.uniform(0.0, 1.0, CFG3_DIMS[0])
    xl = np.clip(x0 - eps, 0.0, 1.0).astype(np.float32)
    xh = np.clip(x0 + eps, 0.0, 1.0).astype(np.float32)
    y0 = _mlp_forward64(layers, x0[None, :])[0]
    t = int(np.argmax(y0))
    W_q, b_q = margin_rows(CFG3_DIMS[-1], t)
    return {'layers': layers, 'xl': xl, 'xh': xh, 'spec_W': W_q,
            'spec_b': b_q, 'true_label': t, 'n_domains': n_domains,
            'n_split': n_split,
            'name': f'cfg3 mlp 784x[256]x6x10 alpha-crown D={n_domains}'}


def cfg4(seed=0, n_domains=256, n_split=8, eps=2.0 / 255.0):
    """Conv CROWN on the cfg4 CNN with 2^n_split ReLU-split domains."""
    rng = np.random.default_rng(seed)
    params = cnn_cfg4_params(rng)
    x0 = rng.uniform(0.0, 1.0, 3 * 32 * 32)
    xl = np.clip(x0 - eps, 0.0, 1.0).astype(np.float32)
    xh = np.clip(x0 + eps, 0.0, 1.0).astype(np.float32)
    return {'params': params, 'x0': x0.astype(np.float32), 'xl': xl, 'xh': xh,
            'n_domains': n_domains, 'n_split': n_split,
            'name': f'cfg4 cnn 3x32x32 conv-crown D={n_domains}'}


def cfg5(seed=0, eps=1.0 / 255.0):
    """Large zonotope: 3072->[1024]x8->10, eps ball around U[0,1]^3072."""
    rng = np.random.default_rng(seed)
    layers = mlp_params(CFG5_DIMS, rng)
    x0 = rng.uniform(0.0, 1.0, CFG5_DIMS[0])
    xl = np.clip(x0 - eps, 0.0, 1.0).astype(np.float32)
    xh = np.clip(x0 + eps, 0.0, 1.0).astype(np.float32)
    y0 = _mlp_forward64(layers, x0[None, :])[0]
    t = int(np.argmax(y0))
    W_q, b_q = margin_rows(CFG5_DIMS[-1], t)
    return {'layers': layers, 'xl': xl, 'xh': xh, 'spec_W': W_q,
            'spec_b': b_q, 'true_label': t,
            'name': 'cfg5 mlp 3072x[1024]x8x10 zonotope'}


def split_domains(sb_lo, sb_hi, n_split):
    """ReLU-split domains from the n_split widest unstable neurons.

    ``sb_lo/sb_hi``: {layer: (n_layer,)} root IBP bounds.  Neurons are ranked
    by width (descending), ties broken by (layer, index).  Returns
    (picked [(layer, idx)], clamps {layer: (cl, ch)} of shape
    (2^n_split, n_layer)) where bit i of the domain index chooses OFF (0:
    ch=0) or ON (1: cl=0) for picked neuron i."""
    cand = []
    for L in sorted(sb_lo):
        lo, hi = np.asarray(sb_lo[L]), np.asarray(sb_hi[L])
        for j in np.nonzero((lo < 0) & (hi > 0))[0]:
            cand.append((-(float(hi[j]) - float(lo[j])), L, int(j)))
    cand.sort()
    picked = [(L, j) for _, L, j in cand[:n_split]]
    D = 1 << len(picked)
    clamps = {}
    for L in sb_lo:
        n = np.asarray(sb_lo[L]).size
        clamps[L] = (np.full((D, n), -np.inf, np.float32),
                     np.full((D, n), np.inf, np.float32))
    for i, (L, j) in enumerate(picked):
        on = ((np.arange(D) >> i) & 1).astype(bool)
        clamps[L][0][on, j] = 0.0
        clamps[L][1][~on, j] = 0.0
    return picked, clamps


def cfg5_split_dims(xl, xh, depth=18):
    """The dimensions the first ``depth`` widest-axis bisections of the box
    split, in order (ties -> lowest index, as torch.argmax): each split halves
    one dimension, so while at least ``depth`` dimensions share the largest
    width the splits walk them in index order."""
    width = (np.asarray(xh, np.float64) - np.asarray(xl, np.float64)).copy()
    dims = []
    for _ in range(depth):
        d = int(np.argmax(width))
        dims.append(d)
        width[d] *= 0.5
    return dims


def cfg5_leaves(xl, xh, start, count, depth=18):
    """Leaves start .. start+count-1 of the depth-``depth`` input-split tree
    of the box: bit t of the leaf index picks the lower (0) or upper (1) half
    along the t-th split dimension.  Returns (count, n) float32 arrays."""
    xl = np.asarray(xl, np.float32)
    xh = np.asarray(xh, np.float32)
    dims = cfg5_split_dims(xl, xh, depth)
    lo = np.repeat(xl[None], count, 0)
    hi = np.repeat(xh[None], count, 0)
    idx = np.arange(start, start + count)
    for t, d in enumerate(dims):
        upper = (idx >> t) & 1
        mid = ((lo[:, d].astype(np.float32) + hi[:, d]) * np.float32(0.5)).astype(np.float32)
        lo[:, d] = np.where(upper == 1, mid, lo[:, d])
        hi[:, d] = np.where(upper == 1, hi[:, d], mid)
    return lo, hi


def robustness_disjuncts(n_out, true_label):
    """Unsafe iff some y_j >= y_true: one pairwise disjunct per j != true."""
    return [[('pair', true_label, j)] for j in range(n_out) if j != true_label]


def reference_bab_settings(**overrides):
    """The input-split driver's settings keys with the values of the
    reference's default_settings (settings.py:319-438, :1364), as a plain
    namespace, plus overrides.  The driver's getattr fallbacks for absent
    keys differ for some (branch_sb True, total_timeout 60 s), so tests that
    mirror a default_settings run pass these explicitly."""
    import types
    d = dict(total_timeout=120.0, input_split_batch_size=4096,
             input_split_batched_max_worklist=200_000,
             input_split_batched_clip_enabled=True, input_split_batched_clip_iters=1,
             input_split_batched_branch_sb=False, input_split_sb_margin_score=False,
             input_split_sb_coeff_thresh=0.01, input_split_sb_margin_weight=1.0,
             input_split_crown_intermediate=False, bab_split_depth=1,
             input_split_batched_branch_boost_exp=1.0, input_split_leaf_pgd_every=0,
             input_split_batched_alpha_boundary_eps=0.0, input_split_batched_alpha_iters=10,
             input_split_batched_alpha_max_leaves=200,
             input_split_batched_alpha_all_leaves=False, disable_sat_finding=False,
             pgd_phase0_enabled=True, raise_on_oom=True)
    d.update(overrides)
    return types.SimpleNamespace(**d)


# configs/acasxu_2023.yaml of the reference (its low-dimensional ReLU FC
# preset): CROWN intermediates, OSI root PGD, leaf PGD every 3 iterations,
# alpha-CROWN on boundary leaves within 10 of closing.
ACASXU_2023 = dict(
    use_hybrid_acasxu=False, input_split_batched_enabled=True,
    input_split_crown_intermediate=True, pgd_init_mode='osi', pgd_time_budget_phase0=5.0,
    input_split_leaf_pgd_every=3, input_split_leaf_pgd_max_leaves=128,
    input_split_leaf_pgd_restarts=256, input_split_leaf_pgd_iters=50,
    input_split_batched_alpha_boundary_eps=10.0, input_split_batched_alpha_iters=20,
    input_split_batched_alpha_max_leaves=2048, input_split_serial_disjuncts=True)


def onnx_mlp_graph(layers, input_shape, offset=None):
    """An OnnxGraph of the ACAS Xu export's structure for fc layers (W (out,
    in), b): Sub(input, offset) -> Flatten -> MatMul(W^T) -> Add(b) -> Relu
    ... -> MatMul -> Add, as onnx_graph.read_onnx returns such a file."""
    from .onnx_graph import OnnxGraph
    n_in = layers[0][0].shape[1]
    consts = {'offset': np.zeros((1,) * (len(input_shape) - 1) + (n_in,))
              if offset is None else np.asarray(offset, np.float64)}
    nodes = [('Sub', ['input', 'offset'], ['sub'], {}),
             ('Flatten', ['sub'], ['flat'], {'axis': 1})]
    cur = 'flat'
    for i, (W, b) in enumerate(layers):
        consts[f'W{i}'] = np.asarray(W, np.float64).T
        consts[f'b{i}'] = np.asarray(b, np.float64)
        nodes.append(('MatMul', [cur, f'W{i}'], [f'mm{i}'], {}))
        nodes.append(('Add', [f'mm{i}', f'b{i}'], [f'add{i}'], {}))
        cur = f'add{i}'
        if i < len(layers) - 1:
            nodes.append(('Relu', [cur], [f'relu{i}'], {}))
            cur = f'relu{i}'
    return OnnxGraph(nodes, consts, 'input', list(input_shape), cur)
