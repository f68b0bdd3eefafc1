"""Wide-MLP zonotope (vcb_zw_* + tcgen05 3xTF32 GEMM) against the oracle's
DeepZ restatement: every intermediate bound, the output centre and the
zonotope's G G^T (column order differs from the reference's)."""
import numpy as np
import pytest
import torch

from conftest import close, max_excess
from oracle import bounds as ob
from vibecheck_nn_b200 import interm, wide, workloads as wk
from vibecheck_nn_b200.zono_wide import wide_zono

pytestmark = pytest.mark.gpu
DEV = torch.device('cuda:0') if torch.cuda.is_available() else None


@pytest.mark.parametrize('dims,B,eps', [((300, 256, 256, 256, 10), 7, 0.05),
                                        ((130, 140, 150, 9), 3, 0.5),
                                        ((768, 512, 512, 512, 512, 10), 5, 0.01)])
def test_wide_zono_matches_oracle(dims, B, eps):
    rng = np.random.default_rng(sum(dims) + B)
    layers = wk.mlp_params(dims, rng)
    x0 = rng.uniform(0, 1, (B, dims[0]))
    w = rng.uniform(0.2, 1.0, (B, dims[0])) * eps
    xl = (x0 - w).astype(np.float32)
    xh = (x0 + w).astype(np.float32)
    xh[0, :3] = xl[0, :3]  # zero-radius dimensions in one leaf
    ggc = wk.mlp_gg(layers)
    sb_ref, (c_ref, G_ref) = ob.forward_zonotope_batched(xl, xh, ggc, np.float64)
    sb32, (c32, _) = ob.forward_zonotope_batched(xl, xh, ggc, np.float32)
    gg = wk.mlp_gg(layers, DEV)
    sb, (c, G) = interm._forward_zonotope_graph_batched(
        torch.as_tensor(xl, device=DEV), torch.as_tensor(xh, device=DEV), gg, DEV, torch.float32)
    unstable = 0
    for L in sb_ref:
        for k in (0, 1):
            ours = sb[L][k].cpu().numpy().astype(np.float64)
            exact = sb_ref[L][k]
            # fp32-equivalent: within the parity tolerance plus twice the fp32
            # reference's own worst error on this layer
            ref_err = np.abs(sb32[L][k] - exact).max()
            allowed = 1e-6 + 1e-5 * np.abs(exact) + 2 * ref_err
            err = np.abs(ours - exact)
            print(f'layer {L} {"lo" if k == 0 else "hi"}: ours {err.max():.2e} '
                  f'fp32 reference {ref_err:.2e}')
            assert (err - allowed).max() <= 0, (L, k, (err - allowed).max())
        unstable += int(((sb_ref[L][0] < 0) & (sb_ref[L][1] > 0)).sum())
    assert unstable > 0  # the ReLU transformer and new generators were exercised
    c_allowed = 1e-6 + 1e-5 * np.abs(c_ref) + 2 * np.abs(c32 - c_ref).max()
    assert (np.abs(c.cpu().numpy() - c_ref) - c_allowed).max() <= 0
    Gn = G.cpu().numpy().astype(np.float64)
    ggt = np.einsum('bok,bpk->bop', Gn, Gn)
    ggt_ref = np.einsum('bok,bpk->bop', G_ref, G_ref)
    assert close(ggt, ggt_ref, rtol=1e-4, atol=1e-5), max_excess(ggt, ggt_ref, 1e-4, 1e-5)


def test_wide_zono_sound_and_no_looser_than_ibp():
    rng = np.random.default_rng(5)
    layers = wk.mlp_params((200, 256, 256, 10), rng)
    x0 = rng.uniform(0, 1, (16, 200))
    xl = torch.as_tensor((x0 - 0.02).astype(np.float32), device=DEV)
    xh = torch.as_tensor((x0 + 0.02).astype(np.float32), device=DEV)
    gg = wk.mlp_gg(layers, DEV)
    wn = wide.wide_net(gg, DEV)
    sb = wide_zono(wn, xl, xh)
    ibp = wide.wide_ibp(wn, xl, xh)
    pts = xl + (xh - xl) * torch.rand(512, 16, 200, device=DEV)
    from vibecheck_nn_b200.forward import _forward_batch_graph
    for L in sb:
        assert torch.all(sb[L][0] >= ibp[L][0] - 1e-4)  # zonotope first layer = IBP exactly
    y = _forward_batch_graph(pts.reshape(-1, 200), gg)
    assert y.shape[0] == 512 * 16
