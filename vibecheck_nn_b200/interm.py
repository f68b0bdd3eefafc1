"""Zonotope forward and CROWN intermediate bounds on libvcb.so.

* ``_forward_zonotope_graph_batched`` -- the DeepZ forward
  (verify_zono_bnb.py:3079-4074) as one ``vcb_mlp_zono`` launch.
* ``_crown_intermediate_batched`` -- backward-CROWN pre-ReLU bounds
  intersected with the zonotope's (verify_zono_bnb.py:4077-4147).  Layer L's
  seeds ``[+e_j; -e_j]`` at its feeding fc are exactly a spec of 2 n_L one-hot
  rows on the network truncated after fc L, so each layer is one
  ``vcb_mlp_crown`` launch (caller-supplied bounds for the earlier layers)
  followed by ``vcb_interm_intersect``.  All neurons are seeded; the
  intersection is applied to the batch-wide unstable set only, which gives
  the reference's union-over-batch semantics without a host round trip.
"""
from __future__ import annotations

import torch

from . import _lib
from .netdesc import MlpDesc, mlp_desc
from .ops import F32, _check_dtype, _dev, _f32, mlp_crown, _unpack_layers

_SEED_CACHE = {}


def truncated(desc, n_fc):
    """Descriptor of the first n_fc fc layers (a prefix of desc's buffers)."""
    key = ('_trunc', n_fc)
    sub = desc.__dict__.get(key)
    if sub is None:
        sub = MlpDesc(desc.dims[:n_fc + 1], desc.W_all, desc.b_all,
                      desc.Ws[:n_fc], desc.bs[:n_fc])
        desc.__dict__[key] = sub
    return sub


def _seed_spec(n, device):
    key = (n, str(device))
    s = _SEED_CACHE.get(key)
    if s is None:
        eye = torch.eye(n, dtype=F32, device=device)
        s = (torch.cat([eye, -eye], 0).contiguous(),
             torch.zeros(2 * n, dtype=F32, device=device))
        _SEED_CACHE[key] = s
    return s


def mlp_zono(desc, xl, xh, want_union=False, full=False):
    """Raw ``vcb_mlp_zono`` launch.  Returns (sb_lo, sb_hi packed,
    unstable_any or None, (c, G, K) or None)."""
    device = xl.device
    B = xl.shape[0]
    _, total = desc.relu_offsets(B)
    sb_lo = torch.empty(total, dtype=F32, device=device)
    sb_hi = torch.empty(total, dtype=F32, device=device)
    unst = (torch.zeros(max(1, sum(desc.relu_widths)), dtype=torch.int32,
                        device=device) if want_union else None)
    out_full = None
    P = _lib.ptr
    L = _lib.lib()
    if full:
        kmax = L.vcb_mlp_zono_kmax(desc.struct)
        c = torch.empty((B, desc.n_out), dtype=F32, device=device)
        G = torch.empty((B, desc.n_out, kmax), dtype=F32, device=device)
        K = torch.empty((B,), dtype=torch.int32, device=device)
        out_full = (c, G, K)
    rc = L.vcb_mlp_zono(desc.struct, B, P(xl), P(xh), P(sb_lo), P(sb_hi),
                        P(unst), P(out_full[0] if full else None),
                        P(out_full[1] if full else None),
                        P(out_full[2] if full else None), _lib.stream_of(device))
    _lib.check(rc, 'vcb_mlp_zono')
    return sb_lo, sb_hi, unst, out_full


def _forward_zonotope_graph_batched(xl, xh, gg, device, dtype):
    """Batched DeepZ forward (verify_zono_bnb.py:3079-4074).

    Returns ``(sb, (c, G))``: sb {relu layer: (lo, hi)} (B, n_L); c (B, n_out);
    G (B, n_out, K) with K the largest per-box generator count.  Each box's
    generators are its input dimensions of nonzero radius followed by its
    unstable neurons in layer/neuron order, zero-padded; the reference keeps
    batch-union input columns and per-layer padding instead, so the column
    order can differ while the zonotope (and every bound) is the same."""
    _check_dtype(dtype)
    device = _dev(device)
    xl = _f32(xl, device)
    xh = _f32(xh, device)
    desc = mlp_desc(gg, device)
    B = xl.shape[0]
    try:
        sb_lo, sb_hi, _, (c, G, K) = mlp_zono(desc, xl, xh, full=True)
    except _lib.UnsupportedInput:  # too wide for the shared-memory kernel
        from .wide import wide_net
        from .zono_wide import wide_zono
        sb, (c, G) = wide_zono(wide_net(gg, device), xl, xh, want_output=True)
        _forward_zonotope_graph_batched.last_bilinear_op_bounds = {}
        return sb, (c, G)
    kmax = int(K.max().item()) if B > 0 else 0
    G = G[:, :, :kmax]
    lo = _unpack_layers(desc, B, sb_lo)
    hi = _unpack_layers(desc, B, sb_hi)
    _forward_zonotope_graph_batched.last_bilinear_op_bounds = {}
    return {L: (lo[L], hi[L]) for L in lo}, (c, G)


_forward_zonotope_graph_batched.last_bilinear_op_bounds = {}


def crown_intermediate_packed(desc, xl, xh):
    """Packed (lo, hi) CROWN-intermediate bounds (layer-major (B, n_L))."""
    B = xl.shape[0]
    lo, hi, unst, _ = mlp_zono(desc, xl, xh, want_union=True)
    if B == 0:
        return lo, hi
    offs, _ = desc.relu_offsets(B)
    uoff = 0
    L_ = _lib.lib()
    for L, n in enumerate(desc.relu_widths):
        sub = truncated(desc, L + 1)
        spec = _seed_spec(n, xl.device)
        lb = mlp_crown(sub, xl, xh, sb_in=(lo, hi), spec=spec)['lb']
        seg = slice(offs[L], offs[L] + B * n)
        rc = L_.vcb_interm_intersect(B, n, _lib.ptr(lb), _lib.ptr(unst[uoff:uoff + n]),
                                     _lib.ptr(lo[seg]), _lib.ptr(hi[seg]),
                                     _lib.stream_of(xl.device))
        _lib.check(rc, 'vcb_interm_intersect')
        uoff += n
    return lo, hi


def _crown_intermediate_batched(gg, xl, xh, device, dtype, chunk=2048):
    """Backward-CROWN intermediate bounds intersected with the zonotope's
    (verify_zono_bnb.py:4077-4147).  Returns tight {L: (lo, hi)} (B, n_L).
    ``chunk`` only bounded the reference's peak memory; results do not
    depend on it."""
    _check_dtype(dtype)
    device = _dev(device)
    xl = _f32(xl, device)
    xh = _f32(xh, device)
    desc = mlp_desc(gg, device)
    B = xl.shape[0]
    lo, hi = crown_intermediate_packed(desc, xl, xh)
    lo_d = _unpack_layers(desc, B, lo)
    hi_d = _unpack_layers(desc, B, hi)
    return {L: (lo_d[L], hi_d[L]) for L in lo_d}


def spec_backward_seeded(tight, xl, xh, gg, seed_ew_at, seed_acc, device, alpha_at_layer=None):
    """``_spec_backward_graph_batched(..., seed_ew_at=..., seed_acc=...)`` for
    a seed at the output of one fc layer that is identical across the batch
    (the form ``_crown_intermediate_batched`` uses, verify_zono_bnb.py:4131-4139,
    and the per-layer alpha freeze of verify_hybrid_acasxu.py:186-215).  With
    ``alpha_at_layer`` ({L: (B, n_L) or (B, Q, n_L)} for the relu layers below
    the seed, possibly requiring grad) the layer-wise kernels run the
    relaxation with those slopes."""
    device = _dev(device)
    if len(seed_ew_at) != 1:
        raise _lib.UnsupportedInput('vibecheck_nn_b200: one seed op supported')
    (name, seed), = seed_ew_at.items()
    names = [op['name'] for op in gg['ops'] if op['type'] == 'fc']
    if name not in names:
        raise _lib.UnsupportedInput(f'vibecheck_nn_b200: seed at non-fc op {name!r}')
    L = names.index(name)
    seed = torch.as_tensor(seed, device=device)
    B = xl.shape[0]
    s0 = seed[0]
    if B > 1 and not (seed.stride(0) == 0 or bool((seed == s0).all())):
        raise _lib.UnsupportedInput('vibecheck_nn_b200: per-box seeds')
    acc0 = torch.zeros(s0.shape[0], dtype=F32, device=device) if seed_acc is None \
        else torch.as_tensor(seed_acc, device=device)[0].to(F32)
    if seed_acc is not None and B > 1 and not bool(
            (torch.as_tensor(seed_acc, device=device) == acc0).all()):
        raise _lib.UnsupportedInput('vibecheck_nn_b200: per-box seed_acc')
    desc = mlp_desc(gg, device)
    sub = truncated(desc, L + 1)
    xl = _f32(xl, device)
    xh = _f32(xh, device)
    from .ops import _packed_layers
    lo = _packed_layers(sub, B, {l: tight[l][0] for l in range(L)}, device) if L > 0 \
        else torch.zeros(1, dtype=F32, device=device)
    hi = _packed_layers(sub, B, {l: tight[l][1] for l in range(L)}, device) if L > 0 \
        else torch.zeros(1, dtype=F32, device=device)
    spec = (_f32(s0, device), _f32(acc0, device))
    alpha = {k: a for k, a in (alpha_at_layer or {}).items() if k < L}
    if alpha:
        if any(bool(a.requires_grad) for a in alpha.values()) and torch.is_grad_enabled():
            from .alpha import spec_backward_with_grad
            return spec_backward_with_grad(sub, lo, hi, xl, xh, spec, alpha, None, False)
        from . import wide
        from .alpha import _sb_dict
        wn = sub.__dict__.get('_wide') or wide.WideNet(sub)
        sub.__dict__['_wide'] = wn
        return wide.wide_crown(wn, xl, xh, _sb_dict(sub, B, lo, hi), spec[0], spec[1],
                               alpha={k: a.detach().to(F32).contiguous()
                                      for k, a in alpha.items()})['lb']
    return mlp_crown(sub, xl, xh, sb_in=(lo, hi), spec=spec)['lb']
