"""ctypes binding of libvcb.so (the C ABI declared in include/vcb.h).

The library is built in-tree (``python -m vibecheck_nn_b200.build``).  There
is no fallback: if the library is missing or the device is not a CUDA GPU,
every operator raises.
"""
from __future__ import annotations

import ctypes
import os

import torch

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, 'libvcb.so')
MAX_FC = 16

VCB_OK = 0
VCB_ERR_INVALID = 1
VCB_ERR_UNSUPPORTED = 2
VCB_ERR_CUDA = 3
VCB_ERR_OOM = 4
VCB_ERR_TIMEOUT = 5


class VcbMlp(ctypes.Structure):
    _fields_ = [('n_fc', ctypes.c_int32),
                ('dims', ctypes.c_int32 * (MAX_FC + 1)),
                ('W', ctypes.c_void_p),
                ('b', ctypes.c_void_p)]


class VcbBabOpts(ctypes.Structure):
    _fields_ = [('clip', ctypes.c_int32),
                ('clip_iters', ctypes.c_int32),
                ('branch_sb', ctypes.c_int32),
                ('margin_score', ctypes.c_int32),
                ('split_depth', ctypes.c_int32),
                ('coeff_thresh', ctypes.c_float),
                ('margin_weight', ctypes.c_float),
                ('boost', ctypes.c_void_p)]


_P = ctypes.c_void_p
_I = ctypes.c_int32

# name -> argtypes; every function returns int (status) unless listed below.
SIGNATURES = {
    'vcb_version': [],
    'vcb_last_error': [],
    'vcb_mlp_crown': [ctypes.POINTER(VcbMlp), _I, _P, _P, _P, _P, _P, _P, _P,
                      _P, _I, _P, _P, _P, _P, _P, _P, _P, _P, ctypes.c_size_t,
                      _P],
    'vcb_mlp_crown_workspace': [ctypes.POINTER(VcbMlp), _I, _I],
    'vcb_mlp_crown_tc_min_batch': [_I],
    'vcb_mlp_crown_path': [ctypes.POINTER(VcbMlp), _I, _I],
    'vcb_fault_check': [_P],
    'vcb_mlp_flirpa': [ctypes.POINTER(VcbMlp), _I, _I, _P, _P, _P, _I, _P, _P, _P, _P, _P,
                       _P, _P, _P, _P],
    'vcb_mlp_flirpa_fate': [ctypes.POINTER(VcbMlp), _I, _I, _P, _P, _P, _I, _P, _P, _P, _I, _P,
                            _P, _P, _P, _P],
    'vcb_multisub_fate': [_I, _I, _I, _I, _P, _P, _P, _P, _P, _P, _P, _P, _I, _P, _P, _P, _P,
                          _P],
    'vcb_multisub_emit': [_I, _I, _I, _P, _P, _P, _P, _P, _P, _P, _P, _P, _P],
    'vcb_multisub_emit_workspace': [_I, _I, _I],
    'vcb_mlp_crown_noalloc': [ctypes.POINTER(VcbMlp), _I, _P, _P, _P, _P, _P,
                              _P, _P, _P, _I, _P, _P, _P, _P, _P, _P, _P, _P],
    'vcb_mlp_crown_noalloc_capacity': [],
    'vcb_probe_ffma': [_P, _I, _I, _P],
    'vcb_mlp_zono': [ctypes.POINTER(VcbMlp), _I, _P, _P, _P, _P, _P, _P, _P,
                     _P, _P],
    'vcb_mlp_zono_kmax': [ctypes.POINTER(VcbMlp)],
    'vcb_interm_intersect': [_I, _I, _P, _P, _P, _P, _P],
    'vcb_mlp_pgd': [ctypes.POINTER(VcbMlp), _I, _I, _P, _P, _P, _I, _P, _P, _P,
                    _I, _I, ctypes.c_float, _P, _P],
    'vcb_mlp_pgd_general': [ctypes.POINTER(VcbMlp), _I, _I, _P, _P, _P, _P, _I, _P, _I,
                            _I, _I, ctypes.c_float, ctypes.c_double, _I, _P, _P, _I, _P, _P,
                            _P, _P, _I, _I, _I, ctypes.c_double, ctypes.c_uint64, _P,
                            _P, _P, _P],
    'vcb_wide_ibp_layer': [_I, _I, _I, _P, _P, _I, _P, _P, _P, _P, _P, _P, _P,
                           _P, _P, _I, _P],
    'vcb_wide_back_layer': [_I, _I, _I, _I, _P, _I, _P, _I, _P, _P, _P, _I, _P, _P,
                            _P, _I, _P, _P, _P],
    'vcb_wide_back_parts': [_I, _I],
    'vcb_wide_rowsum': [_I, _I, _I, _P, _P, _P, _P],
    'vcb_wide_concretize': [_I, _I, _I, _I, _P, _P, _P, _P, _P, _P, _P, _P],
    'vcb_wide_adjoint_layer': [_I, _I, _I, _I, _P, _I, _P, _P, _P, _P, _P, _P, _I, _P, _P,
                               _P, _I, _P],
    'vcb_wide_alpha_adam': [_I, _I, _I, _I, _P, _P, _P, _P, ctypes.c_float, _I,
                            _P],
    'vcb_conv_ibp': [_I, _P, _P, _P, _P, _P, _P, _P, _P, _P],
    'vcb_conv_back': [_I, _P, _P, _P, _P, _P, ctypes.c_size_t, _P],
    'vcb_conv_back_workspace': [_I, _P],
    'vcb_pgd_screen': [_I, _I, _P, _I, _I, _P, _P, _P, _P, _I, _I, _I, _I, _I,
                       ctypes.c_float, ctypes.c_double, _I, _P, _P, _P, _I, _P],
    'vcb_pgd_step': [_I, _I, _I, _P, _P, _P, _P, _I, _I, _I, _I, _P, _I, _P, _P, _P,
                     ctypes.c_float, ctypes.c_float, ctypes.c_float, ctypes.c_float, _P],
    'vcb_tf32_split': [ctypes.c_int64, _P, _P, _P, _P],
    'vcb_tc_gemm': [_I, _I, _I, _P, _P, _I, _P, _P, _I, _P, _P, _I, _P, _P],
    'vcb_tc_gemm_gated': [_I, _I, _I, _P, _P, _I, _P, _P, _I, _P, _P, _I, _P, _P, _P],
    'vcb_wtc_relax_init': [ctypes.c_int64, _P, _P, _P, _P, _P, _P],
    'vcb_wtc_back_gemm': [_I, _I, _I, _I, _P, _P, _I, _P, _P, _I, _P, _I, _P, _P, _P, _P,
                          _P, _P, _I, _P, _I, _I, _P, _P, _P],
    'vcb_wtc_input_gemm': [_I, _I, _I, _I, _P, _P, _I, _P, _P, _I, _P, _P, _P, _P, _I, _P, _I,
                           _I, _P, _P, _P],
    'vcb_wtc_adj_gemm': [_I, _I, _I, _I, _P, _P, _I, _P, _P, _I, _P, _P, _I, _P, _P, _P,
                         _I, _P, _P, _I, _P, _P, _P],
    'vcb_wtc_finish': [_I, _P, _P, _I, _I, _P, _P, _I, _P, _P, _P],
    'vcb_wtc_adam': [_I, _I, _I, _P, _I, _P, _P, _P, ctypes.c_float, _I, _P, _P],
    'vcb_zw_relu': [_I, _I, _P, _P, _P, _P, _P, _P, _P, _P, _P],
    'vcb_zw_build': [_I, _I, _I, _P, _P, _P, _I, _P, _I, _P, _P, _P, _P, _P, _P,
                     ctypes.c_int64, _P, _P, _P],
    'vcb_zw_colsum': [_I, _I, _P, _P, _P, _I, _P, _I, _P, _P, _P, _P, ctypes.c_size_t, _P],
    'vcb_zw_colsum_workspace': [ctypes.c_int64, _I],
    'vcb_bab_step_wide': [_I, _I, _I, _I, _I, _P, _P, _P, _P, _P, _P, _I, _I, _P, _P, _P, _P,
                          _P, _P, ctypes.c_size_t, _P],
    'vcb_bab_step_wide_workspace': [_I, _I],
    'vcb_bab_step_ex': [_I, _I, _I, _I, _I, _P, _P, _P, _P, _P, _P, ctypes.POINTER(VcbBabOpts),
                        _P, _P, _P, _P, _P, _P, _P, _P],
    'vcb_bab_step_wide_ex': [_I, _I, _I, _I, _I, _P, _P, _P, _P, _P, _P,
                             ctypes.POINTER(VcbBabOpts), _P, _P, _P, _P, _P, _P, _P, _P,
                             ctypes.c_size_t, _P],
    'vcb_conv_forward': [_I, _P, _P, _P, _P, _P, _P, _P],
    'vcb_conv_backward': [_I, _P, _P, _P, _P, _P, _P, ctypes.c_size_t, _P],
    'vcb_fc_forward': [_I, _I, _I, _P, _I, _P, _P, _P, _I, _P, _I, _P],
    'vcb_fc_backward': [_I, _I, _I, _P, _I, _P, _P, _I, _P, _I, _P],
    'vcb_conv_bias_dot': [_I, _I, _I, _P, _P, _P, _P],
    'vcb_ibp_relu': [_I, _I, _P, _P, _P, _P, _P, _P, _P, _P, _I, _P],
    'vcb_relu_back': [_I, _I, _I, _P, _I, _P, _I, _P, _P, _P, _P, _P, _P],
    'vcb_bab_step': [_I, _I, _I, _I, _I, _P, _P, _P, _P, _P, _P, _I, _I, _P,
                     _P, _P, _P, _P, _P],
}
RESTYPES = {'vcb_last_error': ctypes.c_char_p,
            'vcb_mlp_crown_workspace': ctypes.c_size_t,
            'vcb_mlp_crown_noalloc_capacity': ctypes.c_size_t,
            'vcb_conv_back_workspace': ctypes.c_size_t,
            'vcb_bab_step_wide_workspace': ctypes.c_size_t,
            'vcb_zw_colsum_workspace': ctypes.c_size_t,
            'vcb_multisub_emit_workspace': ctypes.c_int64}

_lib = None


class KernelError(RuntimeError):
    """A kernel of this package failed: a CUDA launch or runtime error
    (VCB_ERR_CUDA).  Nothing in this package catches it; the reference's own
    callers report it like any RuntimeError (verify_graph.py:9949-9980 turns
    it into an ``unknown`` verdict that carries the message)."""


class UnsupportedInput(NotImplementedError):
    """Inputs outside the B200 path: CPU or float64 tensors, or a graph the
    kernels do not take.  A ``NotImplementedError``, the type the reference
    raises for an op it cannot bound (verify_zono_bnb.py:4071, :5115), so the
    reference's callers fall back exactly as they do for their own refusals;
    the installed delegating bindings hand these calls, and only these, to
    the reference's function."""


def lib():
    """Load libvcb.so once; raises if it has not been built."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise RuntimeError(
                f'{LIB_PATH} is missing: build it with '
                '`python -m vibecheck_nn_b200.build` (no CPU fallback exists)')
        handle = ctypes.CDLL(LIB_PATH)
        for name, args in SIGNATURES.items():
            fn = getattr(handle, name)
            fn.argtypes = args
            fn.restype = RESTYPES.get(name, ctypes.c_int)
        _lib = handle
    return _lib


def last_error():
    msg = lib().vcb_last_error()
    return msg.decode() if msg else ''


def check(rc, what='vcb'):
    """Map a VCB_* status to the exception type the reference's callers
    handle (ValueError / NotImplementedError / RuntimeError / OOM)."""
    if rc == VCB_OK:
        return
    msg = f'{what}: {last_error()}'
    if rc == VCB_ERR_INVALID:
        raise ValueError(msg)
    if rc == VCB_ERR_UNSUPPORTED:
        raise UnsupportedInput(msg)
    if rc == VCB_ERR_OOM:
        raise torch.cuda.OutOfMemoryError(msg)
    if rc == VCB_ERR_TIMEOUT:
        raise TimeoutError(msg)
    raise KernelError(msg)


def fault_check(device=None):
    """Synchronise ``device``'s current stream and raise ``TimeoutError`` if a
    kernel of the library gave up a bounded wait since the last check (its
    outputs for the unfinished boxes are NaN).  The drivers call it where
    they synchronise anyway (each BaB iteration's counter read, the end of a
    verdict); a caller of the raw operators calls it at its own sync points."""
    stream = stream_of(device if device is not None else torch.device('cuda'))
    check(lib().vcb_fault_check(stream), 'vcb_fault_check')


def ptr(t):
    """Device pointer of a tensor (None -> NULL)."""
    if t is None:
        return None
    return ctypes.c_void_p(t.data_ptr())


def workspace(nbytes, device):
    """Scratch buffer from torch's stream-aware caching allocator (>= 16-byte
    aligned); None when no scratch is needed."""
    if not nbytes:
        return None
    return torch.empty((nbytes + 15) // 16 * 4, dtype=torch.float32,
                       device=device)


def stream_of(device):
    return ctypes.c_void_p(torch.cuda.current_stream(device).cuda_stream)


def require_cuda(t, name='tensor'):
    if not (isinstance(t, torch.Tensor) and t.is_cuda):
        raise UnsupportedInput(
            f'vibecheck_nn_b200: {name} must be a CUDA tensor (the B200 path '
            'has no CPU fallback)')
