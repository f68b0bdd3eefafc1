"""Concrete batched forward pass on the layer kernels.

``_forward_batch_graph`` keeps the reference's signature
(verify_zono_bnb.py:554): N points ``x`` (N, *input_shape) through an
fc / conv / relu / reshape chain (bias add / sub folded), returning the
network output (N, n_out) or, with ``capture``, the activation of that op.
Every fc and conv runs as a ``vcb_fc_forward`` / ``vcb_conv_forward`` launch
with its ReLU fused into the epilogue; when ``x`` requires grad the result
carries the transposed-layer kernels as its backward.
"""
from __future__ import annotations

import torch

from .graph import graph_forward, graph_net, graph_vjp
from . import _lib
from .ops import F32


class _Forward(torch.autograd.Function):
    """Network output with the layer kernels' vector-Jacobian product as its
    backward, so callers that differentiate through the forward (PGD
    losses) keep working."""

    @staticmethod
    def forward(ctx, x2, G):
        y, pre = graph_forward(G, x2.detach(), keep=True)
        ctx.G = G
        ctx.pre = pre
        return y

    @staticmethod
    def backward(ctx, gy):
        return graph_vjp(ctx.G, ctx.pre, gy.contiguous().to(F32)), None


def _forward_batch_graph(x, gg, capture=None):
    if not isinstance(x, torch.Tensor) or x.device.type != 'cuda':
        raise _lib.UnsupportedInput("vibecheck_nn_b200: _forward_batch_graph needs a CUDA tensor")
    if x.dtype != F32:
        raise _lib.UnsupportedInput('vibecheck_nn_b200: _forward_batch_graph runs in float32')
    G = graph_net(gg, x.device)
    N = x.shape[0]
    x2 = x.reshape(N, -1).contiguous()
    if capture is None:
        if x.requires_grad and torch.is_grad_enabled():
            return _Forward.apply(x2, G)
        return graph_forward(G, x2)
    if x.requires_grad and torch.is_grad_enabled():
        raise _lib.UnsupportedInput('vibecheck_nn_b200: capture with gradients')
    idx = G.layer_of(capture)
    if idx < 0:
        return x2
    return graph_forward(G, x2, upto=idx)
