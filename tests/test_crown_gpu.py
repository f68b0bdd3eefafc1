"""GPU parity of the fused IBP + CROWN kernels behind vcb_mlp_crown.

Checked against (a) golden vectors recorded from the reference and (b) the
numpy oracle on seeded cfg2 inputs.  The fp32 SIMT kernel: |a-b| <= 1e-6 +
1e-5 |b| against the float32 results.  The tcgen05 3xTF32 kernel, whose
tensor-core accumulation rounds differently: fp32-equivalence against the
float64 results (the same tolerance plus twice the float32 reference's own
worst error on that output).
"""
import numpy as np
import pytest
import torch

from conftest import close, fp32_equivalent, golden_layers, load_golden, max_excess
from oracle import bounds as ob
from vibecheck_nn_b200 import ops, workloads as wk

pytestmark = pytest.mark.gpu
DEV = torch.device('cuda:0') if torch.cuda.is_available() else None


def check(path, ours, ref32, ref64):
    """The parity criterion of the kernel that ran (module docstring)."""
    if path == 'simt':
        assert close(ours, ref32), max_excess(ours, ref32)
    else:
        ok, worst, err, ref_err = fp32_equivalent(ours, ref32, ref64)
        assert ok, (worst, err, ref_err)


@pytest.fixture(autouse=True, params=['simt', 'tc'])
def kernel_path(request):
    """Every test runs through both kernels behind vcb_mlp_crown: the fp32
    SIMT kernel and the tcgen05 3xTF32 kernel (routing threshold 0)."""
    from vibecheck_nn_b200 import _lib
    lib = _lib.lib()
    prev = lib.vcb_mlp_crown_tc_min_batch(0 if request.param == 'tc' else 1 << 30)
    yield request.param
    lib.vcb_mlp_crown_tc_min_batch(prev)


def T(a):
    return torch.as_tensor(np.asarray(a), device=DEV)


def N(t):
    return t.detach().cpu().numpy()


@pytest.mark.parametrize('tag', ['small', 'acas'])
def test_golden_ibp_and_crown(tag, kernel_path):
    g = load_golden(f'mlp_{tag}')
    gg = wk.mlp_gg(golden_layers(g), DEV)
    spec_ew = wk.spec_ew_from(g['spec_W'], g['spec_b'], DEV)
    sb = ops._ibp_forward_graph_batched(T(g['xl']), T(g['xh']), gg, DEV,
                                        torch.float32)
    for L, (lo, hi) in sb.items():
        check(kernel_path, N(lo), g[f'ibp32_lo{L}'], g[f'ibp64_lo{L}'])
        check(kernel_path, N(hi), g[f'ibp32_hi{L}'], g[f'ibp64_hi{L}'])
    lb, A, acc = ops._spec_backward_graph_batched(
        sb, T(g['xl']), T(g['xh']), gg, spec_ew, DEV, torch.float32,
        return_input_linear=True)
    for k, v in (('lb', lb), ('A', A), ('acc', acc)):
        check(kernel_path, N(v), g[f'crown32_{k}'], g[f'crown64_{k}'])
    # fused single launch
    lb2, A2, acc2 = ops.ibp_crown_batched(T(g['xl']), T(g['xh']), gg, spec_ew,
                                          DEV, return_input_linear=True)
    for k, v in (('lb', lb2), ('A', A2), ('acc', acc2)):
        check(kernel_path, N(v), g[f'crown32_{k}'], g[f'crown64_{k}'])


@pytest.mark.parametrize('tag', ['small', 'acas'])
def test_golden_clamped(tag, kernel_path):
    g = load_golden(f'mlp_{tag}')
    gg = wk.mlp_gg(golden_layers(g), DEV)
    spec_ew = wk.spec_ew_from(g['spec_W'], g['spec_b'], DEV)
    clamps = {0: (T(g['clamp_lo0']), T(g['clamp_hi0']))}
    sb = ops._ibp_forward_graph_batched(T(g['xl']), T(g['xh']), gg, DEV,
                                        torch.float32, relu_clamps=clamps)
    for L, (lo, hi) in sb.items():
        check(kernel_path, N(lo), g[f'ibpc32_lo{L}'], g[f'ibpc64_lo{L}'])
        check(kernel_path, N(hi), g[f'ibpc32_hi{L}'], g[f'ibpc64_hi{L}'])
    lb = ops.ibp_crown_batched(T(g['xl']), T(g['xh']), gg, spec_ew, DEV,
                               relu_clamps=clamps)
    check(kernel_path, N(lb), g['crownc32_lb'], g['crownc64_lb'])


@pytest.mark.parametrize('tag', ['small', 'acas'])
def test_golden_spec_on_crown_intermediates(tag, kernel_path):
    """Spec backward given externally computed (CROWN-intermediate) bounds."""
    g = load_golden(f'mlp_{tag}')
    gg = wk.mlp_gg(golden_layers(g), DEV)
    spec_ew = wk.spec_ew_from(g['spec_W'], g['spec_b'], DEV)
    n_relu = int(g['n_layers']) - 1
    tight = {L: (T(g[f'interm32_lo{L}']), T(g[f'interm32_hi{L}']))
             for L in range(n_relu)}
    lb, A, acc = ops._spec_backward_graph_batched(
        tight, T(g['xl']), T(g['xh']), gg, spec_ew, DEV, torch.float32,
        return_input_linear=True)
    for k, v in (('lb', lb), ('A', A), ('acc', acc)):
        check(kernel_path, N(v), g[f'spec_interm32_{k}'], g[f'spec_interm64_{k}'])


def _oracle(w, dtype):
    ggc = wk.mlp_gg(w['layers'])
    sb = ob.ibp_forward_batched(w['xl'], w['xh'], ggc, dtype=dtype)
    lb, A, acc = ob.spec_backward_batched(sb, w['xl'], w['xh'], ggc, w['spec_W'],
                                          w['spec_b'], return_input_linear=True, dtype=dtype)
    return sb, lb, A, acc


@pytest.mark.parametrize('B,Q', [(1, 4), (17, 4), (33, 1), (40, 9), (4096, 4)])
def test_cfg2_vs_oracle(B, Q, kernel_path):
    w = wk.cfg2(seed=3, n_boxes=B, n_q=Q)
    gg = wk.mlp_gg(w['layers'], DEV)
    spec_ew = wk.spec_ew_from(w['spec_W'], w['spec_b'], DEV)
    lb, A, acc, sbd = ops.ibp_crown_batched(T(w['xl']), T(w['xh']), gg, spec_ew,
                                            DEV, return_input_linear=True,
                                            return_sb=True)
    sb, r_lb, r_A, r_acc = _oracle(w, np.float32)
    sb64, e_lb, e_A, e_acc = _oracle(w, np.float64)
    for L in sb:
        check(kernel_path, N(sbd[L][0]), sb[L][0], sb64[L][0])
        check(kernel_path, N(sbd[L][1]), sb[L][1], sb64[L][1])
    check(kernel_path, N(lb), r_lb, e_lb)
    check(kernel_path, N(A), r_A, e_A)
    check(kernel_path, N(acc), r_acc, e_acc)


def _near_tie(lo, hi, tol=1e-4):
    """Boxes with an unstable neuron whose CROWN upper slope is within tol of
    the min-area threshold 0.5 (the lower slope jumps between 0 and 1 there,
    so the last bits of the bounds decide it)."""
    unstable = (lo < 0) & (hi > 0)
    up = np.where(unstable, hi / np.where(unstable, hi - lo, 1.0), 0.0)
    return (unstable & (np.abs(up - 0.5) < tol)).any(axis=1)


def test_cfg2_full_size_against_oracle(kernel_path):
    """The benchmark workload itself (65,536 boxes, Q=4).  For the tensor-core
    kernel a box may also differ where the min-area slope rule is at a tie
    in exact arithmetic (both sides are valid CROWN bounds); such boxes must
    be rare and their bounds sound."""
    w = wk.cfg2(seed=0)
    gg = wk.mlp_gg(w['layers'], DEV)
    spec_ew = wk.spec_ew_from(w['spec_W'], w['spec_b'], DEV)
    lb = N(ops.ibp_crown_batched(T(w['xl']), T(w['xh']), gg, spec_ew, DEV))
    ggc = wk.mlp_gg(w['layers'])
    sb = ob.ibp_forward_batched(w['xl'], w['xh'], ggc)
    r_lb = ob.spec_backward_batched(sb, w['xl'], w['xh'], ggc, w['spec_W'],
                                    w['spec_b'])
    if kernel_path == 'simt':
        assert close(lb, r_lb), max_excess(lb, r_lb)
        tie_boxes = np.zeros(0, np.int64)
    else:
        sb64 = ob.ibp_forward_batched(w['xl'], w['xh'], ggc, dtype=np.float64)
        e_lb = ob.spec_backward_batched(sb64, w['xl'], w['xh'], ggc, w['spec_W'],
                                        w['spec_b'], dtype=np.float64)
        ref_err = np.abs(r_lb - e_lb).max()
        bad = (np.abs(lb - e_lb) > 1e-6 + 1e-5 * np.abs(e_lb) + 2 * ref_err).any(axis=1)
        tie = np.zeros(len(lb), bool)
        for L in sb64:
            tie |= _near_tie(sb64[L][0], sb64[L][1])
        tie_boxes = np.nonzero(bad)[0]
        assert len(tie_boxes) <= max(1, len(lb) // 10000), len(tie_boxes)
        assert tie[tie_boxes].all(), tie_boxes[~tie[tie_boxes]]
    # soundness against concrete samples of the first 256 boxes and of every
    # box at a slope tie
    idx = np.unique(np.concatenate([np.arange(256), tie_boxes]))
    rng = np.random.default_rng(1)
    xs = w['xl'][idx, None, :] + (w['xh'] - w['xl'])[idx, None, :] * \
        rng.random((len(idx), 64, 5))
    ys = wk._mlp_forward64(w['layers'], xs.reshape(-1, 5)).reshape(len(idx), 64, -1)
    spec_vals = ys @ w['spec_W'].T.astype(np.float64)
    assert (lb[idx, None, :] <= spec_vals.min(axis=1, keepdims=True) + 1e-5).all()


def test_empty_batch_and_zero_width_boxes():
    w = wk.cfg2(seed=4, n_boxes=8)
    gg = wk.mlp_gg(w['layers'], DEV)
    spec_ew = wk.spec_ew_from(w['spec_W'], w['spec_b'], DEV)
    lb = ops.ibp_crown_batched(T(w['xl'][:0]), T(w['xh'][:0]), gg, spec_ew, DEV)
    assert lb.shape == (0, 4)
    x = w['xl']
    lb = ops.ibp_crown_batched(T(x), T(x), gg, spec_ew, DEV)
    y = wk._mlp_forward64(w['layers'], x.astype(np.float64)) @ \
        w['spec_W'].T.astype(np.float64)
    assert np.allclose(N(lb), y, rtol=1e-5, atol=1e-5)


def test_unsupported_graph_raises_notimplemented():
    gg = wk.mlp_gg(wk.mlp_params((4, 6, 3), np.random.default_rng(0)), DEV)
    gg['ops'].insert(1, {'name': 'sg', 'type': 'sigmoid', 'inputs': ['fc0']})
    with pytest.raises(NotImplementedError):
        ops._ibp_forward_graph_batched(torch.zeros(2, 4, device=DEV),
                                       torch.ones(2, 4, device=DEV), gg, DEV,
                                       torch.float32)


def test_tensor_core_path_is_taken(kernel_path):
    from vibecheck_nn_b200 import _lib
    w = wk.cfg2(seed=0, n_boxes=64)
    desc = ops.mlp_desc(wk.mlp_gg(w['layers'], DEV), DEV)
    path = _lib.lib().vcb_mlp_crown_path(desc.struct, 64, 4)
    assert path == (1 if kernel_path == 'tc' else 0)
    assert _lib.lib().vcb_mlp_crown_path(desc.struct, 64, 17) == 0  # Q > 16


@pytest.mark.parametrize('B', [5, 300])
def test_alpha_beta_and_given_bounds_match_across_kernels(kernel_path, B):
    """alpha, beta, caller-supplied bounds and the A / acc outputs: the
    selected kernel against the other one (each pinned to the oracle above)."""
    from vibecheck_nn_b200 import _lib
    w = wk.cfg2(seed=5, n_boxes=B, n_q=3)
    gg = wk.mlp_gg(w['layers'], DEV)
    desc = ops.mlp_desc(gg, DEV)
    spec = (T(w['spec_W']).float(), T(w['spec_b']).float())
    xl, xh = T(w['xl']).float(), T(w['xh']).float()
    sb = ops.mlp_crown(desc, xl, xh, want_sb=True)
    g = torch.Generator(device=DEV).manual_seed(0)
    alpha = torch.rand(sb['sb_lo'].shape, generator=g, device=DEV)
    beta = torch.rand(sb['sb_lo'].shape, generator=g, device=DEV) * 0.1
    outs = []
    lib = _lib.lib()
    for thr in ((0, 1 << 30) if kernel_path == 'tc' else (1 << 30, 0)):
        prev = lib.vcb_mlp_crown_tc_min_batch(thr)
        try:
            outs.append(ops.mlp_crown(desc, xl, xh, sb_in=(sb['sb_lo'], sb['sb_hi']), alpha=alpha,
                                      beta=beta, spec=spec, want_A=True))
        finally:
            lib.vcb_mlp_crown_tc_min_batch(prev)
    for k in ('lb', 'acc'):
        assert close(N(outs[0][k]), N(outs[1][k]), rtol=3e-5, atol=3e-6), \
            (k, max_excess(N(outs[0][k]), N(outs[1][k])))
    # A entries cancel; compare them on the scale of their row
    A0, A1 = N(outs[0]['A']).astype(np.float64), N(outs[1]['A']).astype(np.float64)
    scale = np.abs(A1).max(axis=2, keepdims=True)
    assert (np.abs(A0 - A1) <= 1e-6 + 1e-5 * scale).all()


@pytest.mark.parametrize('Q', [3, 4, 5, 16])
def test_split_tail_matches_unsplit(Q, kernel_path):
    """151 tiles of 128 boxes on the 148-CTA persistent grid: the tensor-core
    kernel splits the 3 tiles of its last round by spec-row pass across two
    CTAs each.  Every box's bounds must equal, bit for bit, those of the same
    boxes bounded in two calls that need no split (148 tiles, then 3)."""
    B = 151 * 128 - 28
    w = wk.cfg2(seed=5, n_boxes=B, n_q=Q)
    gg = wk.mlp_gg(w['layers'], DEV)
    spec_ew = wk.spec_ew_from(w['spec_W'], w['spec_b'], DEV)
    xl, xh = T(w['xl']), T(w['xh'])

    def run(lo, hi):
        return ops.ibp_crown_batched(lo, hi, gg, spec_ew, DEV, return_input_linear=True)

    whole = run(xl, xh)
    cut = 148 * 128
    first, rest = run(xl[:cut], xh[:cut]), run(xl[cut:], xh[cut:])
    for a, b0, b1 in zip(whole, first, rest):
        assert torch.equal(a, torch.cat([b0, b1])), Q
