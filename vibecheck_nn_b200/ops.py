"""Reference-signature operators backed by libvcb.so.

Each public function here has the name, arguments, return structure and
error behaviour of the vibecheck function it replaces (cited per function),
so it can be bound in place of the reference's
(``vibecheck_nn_b200.install``).  All work runs on the current CUDA stream of
``device``; there is no CPU path.
"""
from __future__ import annotations

import math

import numpy as np
import torch

from . import _lib
from .netdesc import mlp_desc

F32 = torch.float32


def _dev(device):
    device = torch.device(device) if device is not None else torch.device('cuda')
    if device.type != 'cuda':
        raise _lib.UnsupportedInput('vibecheck_nn_b200 runs on CUDA devices only '
                                    f'(got device={device}); there is no CPU fallback')
    return device


def _f32(t, device):
    t = torch.as_tensor(t, device=device)
    if t.dtype != F32:
        t = t.to(F32)
    return t.contiguous()


def _check_dtype(dtype):
    if dtype not in (None, torch.float32):
        raise _lib.UnsupportedInput(
            f'vibecheck_nn_b200 computes in float32 (bits=32); got {dtype}')


def spec_matrix(spec_ew, device):
    """``spec_ew`` {qid: (w, bias)} -> (W_q (Q, n_out), b_q (Q,)) in sorted
    qid order (verify_zono_bnb.py:4315-4321)."""
    qids = sorted(spec_ew.keys())
    W_q = torch.stack([torch.as_tensor(spec_ew[q][0]).flatten().to(device=device, dtype=F32)
                       for q in qids])
    b_q = torch.tensor([float(spec_ew[q][1]) for q in qids], dtype=F32, device=device)
    return W_q.contiguous(), b_q


def _packed_layers(desc, B, per_layer, device, fill=None):
    """Pack {L: (B, n_L)} tensors layer-major into one flat buffer.

    Returns the flat tensor (a view-free fast path when the inputs already
    are consecutive slices of one buffer).  Missing layers get ``fill``."""
    offs, total = desc.relu_offsets(B)
    Ls = range(len(desc.relu_widths))
    ts = [per_layer.get(L) if per_layer is not None else None for L in Ls]
    if all(t is not None for t in ts):
        base = ts[0]
        if (base.dtype == F32 and base.is_cuda and base.is_contiguous()
                and all(t.is_contiguous() and t.dtype == F32 for t in ts)):
            st = base.untyped_storage().data_ptr()
            ok = all(t.untyped_storage().data_ptr() == st for t in ts)
            ok = ok and all(t.data_ptr() == base.data_ptr() + 4 * offs[i]
                            for i, t in enumerate(ts))
            ok = ok and all(tuple(t.shape) == (B, desc.relu_widths[i])
                            for i, t in enumerate(ts))
            if ok:
                return torch.as_strided(base, (total,), (1,))
    out = torch.empty(total, dtype=F32, device=device)
    for i, t in enumerate(ts):
        n = desc.relu_widths[i]
        seg = out[offs[i]:offs[i] + B * n].view(B, n)
        if t is None:
            if fill is None:
                raise ValueError(f'missing per-layer tensor for layer {i}')
            seg.fill_(fill)
        else:
            seg.copy_(torch.as_tensor(t, device=device).to(F32).expand(B, n))
    return out


def _unpack_layers(desc, B, flat):
    offs, _ = desc.relu_offsets(B)
    return {L: flat[offs[L]:offs[L] + B * n].view(B, n)
            for L, n in enumerate(desc.relu_widths)}


def _clamp_arrays(desc, B, relu_clamps, root_sb, device):
    """Fold root_sb and relu_clamps into one packed (lo, hi) clamp pair.
    max(max(l, root_lo), cl) == max(l, max(root_lo, cl)) exactly, so the fold
    reproduces verify_zono_bnb.py:1126-1133."""
    if not relu_clamps and not root_sb:
        return None, None
    offs, total = desc.relu_offsets(B)
    lo = torch.full((total,), -math.inf, dtype=F32, device=device)
    hi = torch.full((total,), math.inf, dtype=F32, device=device)
    for L, n in enumerate(desc.relu_widths):
        seg_lo = lo[offs[L]:offs[L] + B * n].view(B, n)
        seg_hi = hi[offs[L]:offs[L] + B * n].view(B, n)
        if root_sb is not None and L in root_sb:
            seg_lo.copy_(_f32(root_sb[L][0], device).reshape(1, n).expand(B, n))
            seg_hi.copy_(_f32(root_sb[L][1], device).reshape(1, n).expand(B, n))
        if relu_clamps is not None and L in relu_clamps:
            cl, ch = relu_clamps[L]
            torch.maximum(seg_lo, _f32(cl, device).expand(B, n), out=seg_lo)
            torch.minimum(seg_hi, _f32(ch, device).expand(B, n), out=seg_hi)
    return lo, hi


def mlp_crown(desc, xl, xh, *, clamps=(None, None), sb_in=(None, None),
              alpha=None, beta=None, spec=None, want_A=False, want_sb=False):
    """Raw launch of ``vcb_mlp_crown`` on packed arguments.

    Returns dict with lb (B,Q), A (B,Q,n_in), acc (B,Q), sb_lo/sb_hi packed."""
    device = xl.device
    B = xl.shape[0]
    out = {}
    if spec is not None:
        W_q, b_q = spec
        Q = W_q.shape[0]
        out['lb'] = torch.empty((B, Q), dtype=F32, device=device)
        if want_A:
            out['A'] = torch.empty((B, Q, desc.n_in), dtype=F32, device=device)
            out['acc'] = torch.empty((B, Q), dtype=F32, device=device)
    else:
        W_q = b_q = None
        Q = 0
    if want_sb:
        _, total = desc.relu_offsets(B)
        out['sb_lo'] = torch.empty(total, dtype=F32, device=device)
        out['sb_hi'] = torch.empty(total, dtype=F32, device=device)
    P = _lib.ptr
    L = _lib.lib()
    ws_bytes = L.vcb_mlp_crown_workspace(desc.struct, B, Q) if B > 0 else 0
    ws = _lib.workspace(ws_bytes, device)
    rc = L.vcb_mlp_crown(
        desc.struct, B, P(xl), P(xh), P(clamps[0]), P(clamps[1]),
        P(sb_in[0]), P(sb_in[1]), P(alpha), P(beta), Q, P(W_q), P(b_q),
        P(out.get('lb')), P(out.get('A')), P(out.get('acc')),
        P(out.get('sb_lo')), P(out.get('sb_hi')), P(ws), ws_bytes,
        _lib.stream_of(device))
    _lib.check(rc, 'vcb_mlp_crown')
    return out


# ---------------------------------------------------------------------------
# reference-signature operators
# ---------------------------------------------------------------------------

def fits_smem(desc, Q):
    """True when the shared-memory-resident kernel takes this network (else
    the layer-wise wide path runs)."""
    key = ('_fits', Q)
    v = desc.__dict__.get(key)
    if v is None:
        v = bool(_lib.lib().vcb_mlp_crown_workspace(desc.struct, 64, Q))
        desc.__dict__[key] = v
    return v


def _mlp_or_graph(gg, device):
    """(MlpDesc, None) for fc/relu chains, else (None, GraphNet) for chains
    with convolutions; NotImplementedError for anything else."""
    try:
        return mlp_desc(gg, device), None
    except _lib.UnsupportedInput:
        from .graph import graph_net
        return None, graph_net(gg, device)


def _graph_clamps(G, B, relu_clamps, root_sb, device):
    if not relu_clamps and not root_sb:
        return None
    out = {}
    for L, n in enumerate(G.relu_widths):
        lo = torch.full((B, n), -math.inf, dtype=F32, device=device)
        hi = torch.full((B, n), math.inf, dtype=F32, device=device)
        if root_sb is not None and L in root_sb:
            lo.copy_(_f32(root_sb[L][0], device).reshape(1, n).expand(B, n))
            hi.copy_(_f32(root_sb[L][1], device).reshape(1, n).expand(B, n))
        if relu_clamps is not None and L in relu_clamps:
            torch.maximum(lo, _f32(relu_clamps[L][0], device).expand(B, n), out=lo)
            torch.minimum(hi, _f32(relu_clamps[L][1], device).expand(B, n), out=hi)
        out[L] = (lo, hi)
    return out


def _ibp_forward_graph_batched(xl, xh, gg, device, dtype, relu_clamps=None,
                               root_sb=None):
    """Batched interval forward (verify_zono_bnb.py:1066-1153).

    Returns ``sb`` {relu layer: (lo, hi)} of (B, n_L) pre-activation bounds
    after the root/clamp intersection and crossing repair."""
    _check_dtype(dtype)
    device = _dev(device)
    xl = _f32(xl, device)
    xh = _f32(xh, device)
    desc, G = _mlp_or_graph(gg, device)
    if G is not None:
        from .graph import graph_ibp
        return graph_ibp(G, xl, xh, _graph_clamps(G, xl.shape[0], relu_clamps, root_sb, device))
    B = xl.shape[0]
    clo, chi = _clamp_arrays(desc, B, relu_clamps, root_sb, device)
    if not fits_smem(desc, 0):
        from . import wide
        clamps = None
        if clo is not None:
            lo_d, hi_d = _unpack_layers(desc, B, clo), _unpack_layers(desc, B, chi)
            clamps = {L: (lo_d[L], hi_d[L]) for L in lo_d}
        return wide.wide_ibp(wide.wide_net(gg, device), xl, xh, clamps)
    out = mlp_crown(desc, xl, xh, clamps=(clo, chi), want_sb=True)
    lo = _unpack_layers(desc, B, out['sb_lo'])
    hi = _unpack_layers(desc, B, out['sb_hi'])
    return {L: (lo[L], hi[L]) for L in lo}


def _spec_backward_graph_batched(tight, xl, xh, gg, spec_ew, device, dtype,
                                 return_input_linear=False,
                                 alpha_at_layer=None,
                                 relu_split_beta=None,
                                 alpha_mccormick=None,
                                 alpha_recip=None,
                                 bilinear_op_bounds=None,
                                 seed_ew_at=None, seed_acc=None):
    """Batched CROWN spec backward (verify_zono_bnb.py:4270-5134).

    Returns spec_lbs (B, Q), or (spec_lbs, A (B, Q, n_in), acc (B, Q)) when
    ``return_input_linear``.  alpha_at_layer {L: (B, n_L)} gives the lower
    slope of unstable neurons; relu_split_beta {L: (B, n_L)} the signed split
    multiplier.  When alpha or beta require grad, the result carries a
    hand-written adjoint (no autograd through the kernel)."""
    _check_dtype(dtype)
    device = _dev(device)
    if seed_ew_at is not None:
        from .interm import spec_backward_seeded
        return spec_backward_seeded(tight, xl, xh, gg, seed_ew_at, seed_acc,
                                    device, alpha_at_layer=alpha_at_layer)
    if alpha_mccormick or alpha_recip:
        raise _lib.UnsupportedInput('vibecheck_nn_b200: bilinear alpha terms')
    xl = _f32(xl, device)
    xh = _f32(xh, device)
    desc, G = _mlp_or_graph(gg, device)
    if G is not None:
        from .graph import graph_crown
        if alpha_at_layer is not None and any(bool(a.requires_grad) for a in alpha_at_layer.values()) \
                and torch.is_grad_enabled():
            raise _lib.UnsupportedInput('vibecheck_nn_b200: alpha gradients on conv graphs')
        W_q, b_q = spec_matrix(spec_ew, device)
        sb = {L: (_f32(v[0], device), _f32(v[1], device)) for L, v in tight.items()}
        out = graph_crown(G, xl, xh, sb, W_q, b_q,
                          alpha=None if alpha_at_layer is None else
                          {L: _f32(a.detach(), device) for L, a in alpha_at_layer.items()},
                          beta=None if relu_split_beta is None else
                          {L: _f32(b.detach(), device) for L, b in relu_split_beta.items()},
                          want_A=return_input_linear)
        if return_input_linear:
            return out['lb'], out['A'], out['acc']
        return out['lb']
    B = xl.shape[0]
    lo = _packed_layers(desc, B, {L: v[0] for L, v in tight.items()}, device)
    hi = _packed_layers(desc, B, {L: v[1] for L, v in tight.items()}, device)
    spec = spec_matrix(spec_ew, device)
    needs_grad = False
    per_query = False  # alpha (B, Q, n): one slope per spec row (verify_zono_bnb.py:4423)
    if alpha_at_layer is not None:
        for a in alpha_at_layer.values():
            if a.dim() not in (2, 3):
                raise _lib.UnsupportedInput('vibecheck_nn_b200: alpha must be (B, n) or (B, Q, n)')
            per_query |= a.dim() == 3
            needs_grad |= bool(a.requires_grad)
    if relu_split_beta is not None:
        needs_grad |= any(bool(b.requires_grad) for b in relu_split_beta.values())
    if needs_grad and torch.is_grad_enabled():
        from .alpha import spec_backward_with_grad
        return spec_backward_with_grad(desc, lo, hi, xl, xh, spec,
                                       alpha_at_layer, relu_split_beta,
                                       return_input_linear)
    if per_query or not fits_smem(desc, spec[0].shape[0]):
        from . import wide
        sb = {L: (tight[L][0].to(F32).contiguous(), tight[L][1].to(F32).contiguous())
              for L in range(len(desc.relu_widths))}
        out = wide.wide_crown(
            wide.wide_net(gg, device), xl, xh, sb, spec[0], spec[1],
            alpha=None if alpha_at_layer is None else
            {L: a.detach().to(F32).contiguous() for L, a in alpha_at_layer.items()},
            beta=None if relu_split_beta is None else
            {L: b.detach().to(F32).contiguous() for L, b in relu_split_beta.items()},
            want_A=return_input_linear)
        if return_input_linear:
            return out['lb'], out['A'], out['acc']
        return out['lb']
    alpha = (None if alpha_at_layer is None else
             _packed_layers(desc, B, {L: a.detach() for L, a in alpha_at_layer.items()},
                            device, fill=0.0))
    beta = (None if relu_split_beta is None else
            _packed_layers(desc, B, {L: b.detach() for L, b in relu_split_beta.items()},
                           device, fill=0.0))
    out = mlp_crown(desc, xl, xh, sb_in=(lo, hi), alpha=alpha, beta=beta,
                    spec=spec, want_A=return_input_linear)
    if return_input_linear:
        return out['lb'], out['A'], out['acc']
    return out['lb']


def ibp_crown_batched(xl, xh, gg, spec_ew, device='cuda', relu_clamps=None,
                      root_sb=None, return_input_linear=False, return_sb=False):
    """Fused ``_ibp_forward_graph_batched`` -> ``_spec_backward_graph_batched``
    in one kernel launch (the composition the ReLU-split BaB uses,
    verify_milp.py:2762-2807, and the CROWN microbenchmark).  The
    intermediate bounds never leave shared memory unless ``return_sb``."""
    device = _dev(device)
    xl = _f32(xl, device)
    xh = _f32(xh, device)
    desc = mlp_desc(gg, device)
    B = xl.shape[0]
    clo, chi = _clamp_arrays(desc, B, relu_clamps, root_sb, device)
    spec = spec_ew if isinstance(spec_ew, tuple) else spec_matrix(spec_ew, device)
    out = mlp_crown(desc, xl, xh, clamps=(clo, chi), spec=spec,
                    want_A=return_input_linear, want_sb=return_sb)
    res = [out['lb']]
    if return_input_linear:
        res += [out['A'], out['acc']]
    if return_sb:
        lo = _unpack_layers(desc, B, out['sb_lo'])
        hi = _unpack_layers(desc, B, out['sb_hi'])
        res.append({L: (lo[L], hi[L]) for L in lo})
    return res[0] if len(res) == 1 else tuple(res)


def to_numpy(x):
    if isinstance(x, torch.Tensor):
        return x.detach().cpu().numpy()
    return np.asarray(x)
