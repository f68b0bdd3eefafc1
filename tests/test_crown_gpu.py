"""GPU parity of the fused IBP + CROWN kernels behind vcb_mlp_crown.

Checked against (a) golden vectors recorded from the reference and (b) the
numpy oracle on seeded cfg2 inputs, whose float32 IBP bounds are bit-equal to
the reference's on the cfg2 workload (tests/golden/cfg2_ref.npz pins that on
the CPU).  Both kernels -- the fp32 SIMT kernel and the tcgen05 3xTF32
kernel -- are held to north_star's tolerance |a-b| <= 1e-6 + 1e-5 |b| against
the float32 results on every bound (IBP bounds, lb, acc), with no exempted
boxes; the input-space coefficients A to the same tolerance on the scale of
their row (``close_linear_form``).  Where the tensor cores' rounding could
move a ReLU's upper slope across the min-area threshold, the kernel bounds
the box again with the SIMT kernel's fp32 operation order
(crown_tie_kernel); those boxes must equal the SIMT kernel's bit for bit.
"""
import numpy as np
import pytest
import torch

from conftest import close, close_linear_form, golden_layers, load_golden, max_excess
from oracle import bounds as ob
from vibecheck_nn_b200 import ops, workloads as wk

pytestmark = pytest.mark.gpu
DEV = torch.device('cuda:0') if torch.cuda.is_available() else None
TIE_BAND = np.float32(4e-6)  # crown_tc_kernel's band around up_s = 0.5


def check(ours, ref32, kind='bound'):
    """north_star's parity criterion against the float32 reference."""
    if kind == 'A':
        assert close_linear_form(ours, ref32), max_excess(ours, ref32)
    else:
        assert close(ours, ref32), max_excess(ours, ref32)


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
        check(N(lo), g[f'ibp32_lo{L}'])
        check(N(hi), g[f'ibp32_hi{L}'])
    lb, A, acc = ops._spec_backward_graph_batched(
        sb, T(g['xl']), T(g['xh']), gg, spec_ew, DEV, torch.float32,
        return_input_linear=True)
    for k, v in (('lb', lb), ('A', A), ('acc', acc)):
        check(N(v), g[f'crown32_{k}'], k)
    # fused single launch
    lb2, A2, acc2 = ops.ibp_crown_batched(T(g['xl']), T(g['xh']), gg, spec_ew,
                                          DEV, return_input_linear=True)
    for k, v in (('lb', lb2), ('A', A2), ('acc', acc2)):
        check(N(v), g[f'crown32_{k}'], k)


@pytest.mark.parametrize('tag', ['small', 'acas'])
def test_golden_clamped(tag, kernel_path):
    g = load_golden(f'mlp_{tag}')
    gg = wk.mlp_gg(golden_layers(g), DEV)
    spec_ew = wk.spec_ew_from(g['spec_W'], g['spec_b'], DEV)
    clamps = {0: (T(g['clamp_lo0']), T(g['clamp_hi0']))}
    sb = ops._ibp_forward_graph_batched(T(g['xl']), T(g['xh']), gg, DEV,
                                        torch.float32, relu_clamps=clamps)
    for L, (lo, hi) in sb.items():
        check(N(lo), g[f'ibpc32_lo{L}'])
        check(N(hi), g[f'ibpc32_hi{L}'])
    lb = ops.ibp_crown_batched(T(g['xl']), T(g['xh']), gg, spec_ew, DEV,
                               relu_clamps=clamps)
    check(N(lb), g['crownc32_lb'])


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
        check(N(v), g[f'spec_interm32_{k}'], k)


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
    for L in sb:
        check(N(sbd[L][0]), sb[L][0])
        check(N(sbd[L][1]), sb[L][1])
    check(N(lb), r_lb)
    check(N(A), r_A, 'A')
    check(N(acc), r_acc)


def _lower_multiplier(lo, hi, band=TIE_BAND):
    """The min-area lower multiplier the kernels' encode_slope gives each
    neuron (1 active, 0 dead, up_s > 0.5 for unstable) and whether the
    neuron is unstable with up_s within ``band`` of 0.5."""
    lo = lo.astype(np.float32)
    hi = hi.astype(np.float32)
    unstable = (lo < 0) & (hi > 0)
    ub = np.maximum(np.maximum(hi, np.float32(0)), lo + np.float32(1e-8))
    den = np.where(unstable, ub - lo, np.float32(1))
    up = np.where(unstable, ub / den, np.float32(0)).astype(np.float32)
    pos = np.where(lo >= 0, 1, np.where(hi <= 0, 0, (up > np.float32(0.5)).astype(int)))
    return pos, unstable & (np.abs(up - np.float32(0.5)) <= band)


@pytest.mark.parametrize('seed', [0, 1, 3])
def test_cfg2_full_size_against_oracle(kernel_path, seed):
    """The benchmark workload itself (65,536 boxes, Q=4), seeds whose
    tensor-core IBP bounds put a ReLU at the min-area tie: every lower bound
    and IBP bound within the tolerance of the float32 reference, none
    tighter than it by more than the tolerance, A on its row scale."""
    w = wk.cfg2(seed=seed)
    gg = wk.mlp_gg(w['layers'], DEV)
    spec_ew = wk.spec_ew_from(w['spec_W'], w['spec_b'], DEV)
    lb, A, acc, sbd = ops.ibp_crown_batched(T(w['xl']), T(w['xh']), gg, spec_ew, DEV,
                                            return_input_linear=True, return_sb=True)
    lb, A, acc = N(lb), N(A), N(acc)
    ggc = wk.mlp_gg(w['layers'])
    sb = ob.ibp_forward_batched(w['xl'], w['xh'], ggc)
    r_lb, r_A, r_acc = ob.spec_backward_batched(sb, w['xl'], w['xh'], ggc, w['spec_W'],
                                                w['spec_b'], return_input_linear=True)
    for L in sb:
        check(N(sbd[L][0]), sb[L][0])
        check(N(sbd[L][1]), sb[L][1])
    check(lb, r_lb)
    check(acc, r_acc)
    check(A, r_A, 'A')
    # one-sided: never tighter than the reference by more than the tolerance
    ref = r_lb.astype(np.float64)
    assert (lb.astype(np.float64) <= ref + 1e-6 + 1e-5 * np.abs(ref)).all()


@pytest.mark.parametrize('seed', [0, 1, 3])
def test_tie_boxes_are_rebound_with_the_fp32_order(seed):
    """crown_tc_kernel lists every box whose IBP bounds put an unstable ReLU
    within its band of the min-area threshold, and crown_tie_kernel bounds
    those boxes again in the SIMT kernel's order: their lb, A and acc equal
    the SIMT kernel's bit for bit.  Every neuron where the two kernels' slope
    decisions differ lies inside the band (so its box was re-bound)."""
    from vibecheck_nn_b200 import _lib
    lib = _lib.lib()
    w = wk.cfg2(seed=seed)
    gg = wk.mlp_gg(w['layers'], DEV)
    desc = ops.mlp_desc(gg, DEV)
    spec = (T(w['spec_W']).float(), T(w['spec_b']).float())
    xl, xh = T(w['xl']).float(), T(w['xh']).float()
    outs = {}
    for name, thr in (('tc', 0), ('simt', 1 << 30)):
        prev = lib.vcb_mlp_crown_tc_min_batch(thr)
        try:
            outs[name] = {k: N(v) for k, v in ops.mlp_crown(
                desc, xl, xh, spec=spec, want_A=True, want_sb=True).items()}
        finally:
            lib.vcb_mlp_crown_tc_min_batch(prev)
    _lib.fault_check(DEV)
    B = xl.shape[0]
    offs, _ = desc.relu_offsets(B)
    # the kernel lists by its own up_s, within 2 ulp of this exact one: boxes
    # inside 0.95 of the band are listed for certain, every flip lies inside
    # 1.05 of it
    listed = np.zeros(B, bool)
    flipped = np.zeros(B, bool)
    for off, n in zip(offs, desc.relu_widths):
        sl_ = slice(off, off + B * n)
        lo_t = outs['tc']['sb_lo'][sl_].reshape(B, n)
        hi_t = outs['tc']['sb_hi'][sl_].reshape(B, n)
        pos_t, band_in = _lower_multiplier(lo_t, hi_t, TIE_BAND * np.float32(0.95))
        _, band_out = _lower_multiplier(lo_t, hi_t, TIE_BAND * np.float32(1.05))
        pos_s, _ = _lower_multiplier(outs['simt']['sb_lo'][sl_].reshape(B, n),
                                     outs['simt']['sb_hi'][sl_].reshape(B, n))
        differ = pos_t != pos_s
        assert not (differ & ~band_out).any()  # every flip is inside the band
        flipped |= differ.any(axis=1)
        listed |= band_in.any(axis=1)
    assert flipped.sum() >= 1 and 50 <= listed.sum() <= B // 20, (flipped.sum(), listed.sum())
    for k in ('lb', 'A', 'acc'):
        assert np.array_equal(outs['tc'][k][listed], outs['simt'][k][listed]), k


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
    assert close_linear_form(N(outs[0]['A']), N(outs[1]['A']))


@pytest.mark.parametrize('Q', [3, 4, 5, 16])
def test_split_tail_matches_unsplit(Q, kernel_path):
    """A batch of (SMs + 3) tiles of 128 boxes on the persistent grid of one
    CTA per SM: the tensor-core kernel splits the 3 tiles of its last round
    by spec-row pass across two CTAs each.  Every box's bounds must equal,
    bit for bit, those of the same boxes bounded in two calls that need no
    split (SMs tiles, then 3)."""
    if kernel_path == 'simt':
        pytest.skip('the tail split is the tensor-core kernel\'s')
    sms = torch.cuda.get_device_properties(DEV).multi_processor_count
    B = (sms + 3) * 128 - 28
    w = wk.cfg2(seed=5, n_boxes=B, n_q=Q)
    gg = wk.mlp_gg(w['layers'], DEV)
    spec_ew = wk.spec_ew_from(w['spec_W'], w['spec_b'], DEV)
    xl, xh = T(w['xl']), T(w['xh'])

    def run(lo, hi):
        return ops.ibp_crown_batched(lo, hi, gg, spec_ew, DEV, return_input_linear=True)

    whole = run(xl, xh)
    cut = sms * 128
    first, rest = run(xl[:cut], xh[:cut]), run(xl[cut:], xh[cut:])
    for a, b0, b1 in zip(whole, first, rest):
        assert torch.equal(a, torch.cat([b0, b1])), Q
