"""ctypes binding of the C ABI in ``include/thetascan_b200.h``.

The shared library is built in-tree (``thetascan_b200/libthetascan_b200.so``,
see :mod:`thetascan_b200.build`).  There is no fallback: if the library is
missing or cannot be loaded, every CUDA entry point raises.
"""
from __future__ import annotations

import ctypes
import os
import threading

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libthetascan_b200.so")

TS_OK, TS_ERR_VALUE, TS_ERR_NOT_IMPLEMENTED, TS_ERR_CUDA, TS_ERR_DEVICE = range(5)
TS_DTYPE_F32, TS_DTYPE_BF16 = 0, 1
MAX_RETENTIONS = 4

c_int64_3 = ctypes.c_int64 * 3
c_ptr4 = ctypes.c_void_p * MAX_RETENTIONS


class ScanArgs(ctypes.Structure):
    _fields_ = [
        ("batch", ctypes.c_int), ("heads", ctypes.c_int), ("tokens", ctypes.c_int),
        ("dk", ctypes.c_int), ("dv", ctypes.c_int),
        ("q", ctypes.c_void_p), ("k", ctypes.c_void_p), ("v", ctypes.c_void_p),
        ("q_strides", c_int64_3), ("k_strides", c_int64_3), ("v_strides", c_int64_3),
        ("v_append_unit", ctypes.c_int),
        ("n_retentions", ctypes.c_int),
        ("log_alpha", c_ptr4),
        ("out", c_ptr4),
        ("out_dtype", ctypes.c_int),
        ("workspace", ctypes.c_void_p), ("workspace_bytes", ctypes.c_size_t),
        ("init_state", ctypes.c_void_p), ("final_state", ctypes.c_void_p), ("stage", ctypes.c_int),
        ("stale", ctypes.c_int * MAX_RETENTIONS),
        ("f32_streams", ctypes.c_int),
        ("log_alpha_stream", c_ptr4),
    ]


class ScanGradArgs(ctypes.Structure):
    _fields_ = [
        ("dout", c_ptr4),
        ("dq", ctypes.c_void_p), ("dk", ctypes.c_void_p), ("dv", ctypes.c_void_p),
        ("grad_dtype", ctypes.c_int),
        ("dlog_alpha", c_ptr4),
        ("workspace", ctypes.c_void_p), ("workspace_bytes", ctypes.c_size_t),
        ("dv_strides", c_int64_3),
        ("dfinal_state", ctypes.c_void_p), ("dinit_state", ctypes.c_void_p), ("stage", ctypes.c_int),
        ("dlog_alpha_stream", c_ptr4),
    ]


# Every exported symbol declared in include/thetascan_b200.h, with its ctypes
# signature (restype, argtypes).  tests/test_capi_symbols.py checks this table
# against the header.
SIGNATURES = {
    "ts_b200_version": (ctypes.c_char_p, []),
    "ts_b200_launch_count": (ctypes.c_longlong, []),
    "ts_b200_last_error": (ctypes.c_int, [ctypes.c_char_p, ctypes.c_size_t]),
    "ts_b200_device_status": (ctypes.c_int, [ctypes.c_void_p, ctypes.POINTER(ctypes.c_int)]),
    "ts_b200_selftest_mma": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int,
                                            ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_void_p]),
    "ts_b200_selftest_tma_mma": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int,
                                                ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_void_p]),
    "ts_b200_scan_workspace_bytes": (ctypes.c_size_t, [ctypes.POINTER(ScanArgs)]),
    "ts_b200_scan_fwd": (ctypes.c_int, [ctypes.POINTER(ScanArgs), ctypes.c_void_p]),
    "ts_b200_scan_bwd_workspace_bytes": (ctypes.c_size_t, [ctypes.POINTER(ScanArgs)]),
    "ts_b200_scan_bwd": (ctypes.c_int, [ctypes.POINTER(ScanArgs), ctypes.POINTER(ScanGradArgs),
                                        ctypes.c_void_p]),
    "ts_b200_scan_fwd_static": (ctypes.c_int, [ctypes.POINTER(ScanArgs), ctypes.c_void_p]),
}
STATIC_SCRATCH_BYTES = 16 << 20


class FeatureArgs(ctypes.Structure):
    _fields_ = [
        ("batch", ctypes.c_int), ("heads", ctypes.c_int), ("tokens", ctypes.c_int),
        ("head_dim", ctypes.c_int), ("projections", ctypes.c_int), ("kind", ctypes.c_int),
        ("basis", ctypes.c_int), ("bound", ctypes.c_float), ("eps", ctypes.c_float),
        ("k", ctypes.c_void_p), ("q", ctypes.c_void_p),
        ("k_strides", c_int64_3), ("q_strides", c_int64_3),
        ("w1", ctypes.c_void_p), ("w2", ctypes.c_void_p),
        ("score_bias", ctypes.c_void_p), ("threshold", ctypes.c_void_p), ("gain", ctypes.c_void_p),
        ("gain_per_feature", ctypes.c_int), ("gain_scalar", ctypes.c_float),
        ("spline_scale", ctypes.c_void_p), ("spline_scale_scalar", ctypes.c_float),
        ("phi_k", ctypes.c_void_p), ("phi_q", ctypes.c_void_p), ("y0", ctypes.c_void_p),
        ("rope_rot", ctypes.c_int), ("rope_cos", ctypes.c_void_p), ("rope_sin", ctypes.c_void_p),
        ("rope_pos0", ctypes.c_int), ("l2norm", ctypes.c_int), ("l2norm_eps", ctypes.c_float),
        ("phi_q_f32", ctypes.c_void_p),
        ("sparsity", ctypes.c_int), ("threshold_temperature", ctypes.c_float),
        ("relative_threshold", ctypes.c_void_p), ("sparse_blend", ctypes.c_void_p),
    ]


class FeatureGradArgs(ctypes.Structure):
    _fields_ = [
        ("dphi_k", ctypes.c_void_p), ("dphi_q", ctypes.c_void_p), ("dphi_dtype", ctypes.c_int),
        ("dy0", ctypes.c_void_p), ("dk", ctypes.c_void_p), ("dq", ctypes.c_void_p),
        ("dw1", ctypes.c_void_p), ("dw2", ctypes.c_void_p),
        ("dscore_bias", ctypes.c_void_p), ("dthreshold", ctypes.c_void_p), ("dgain", ctypes.c_void_p),
        ("dspline_scale", ctypes.c_void_p),
        ("dk_bf16", ctypes.c_void_p), ("dq_bf16", ctypes.c_void_p),
        ("dk_strides", c_int64_3), ("dq_strides", c_int64_3),
        ("dy0_bf16", ctypes.c_void_p), ("dy0_strides", c_int64_3),
        ("dw2_transposed", ctypes.c_int),
        ("drelative_threshold", ctypes.c_void_p), ("dsparse_blend", ctypes.c_void_p),
    ]


class KReadArgs(ctypes.Structure):
    _fields_ = [
        ("batch", ctypes.c_int), ("heads", ctypes.c_int), ("tokens", ctypes.c_int), ("head_dim", ctypes.c_int),
        ("mode", ctypes.c_int), ("branches", ctypes.c_int), ("eps", ctypes.c_float),
        ("slots", c_ptr4), ("eta", ctypes.c_void_p), ("y0", ctypes.c_void_p), ("y", ctypes.c_void_p),
        ("mass_columns", ctypes.c_int), ("unnormalized", ctypes.c_int),
    ]


class KReadGradArgs(ctypes.Structure):
    _fields_ = [
        ("dy", ctypes.c_void_p), ("dy_dtype", ctypes.c_int), ("dslots", c_ptr4),
        ("dy0", ctypes.c_void_p), ("deta", ctypes.c_void_p),
    ]


class MassArgs(ctypes.Structure):
    _fields_ = [
        ("batch", ctypes.c_int), ("heads", ctypes.c_int), ("tokens", ctypes.c_int), ("width", ctypes.c_int),
        ("phi_k", ctypes.c_void_p), ("phi_q", ctypes.c_void_p), ("log_alpha", ctypes.c_void_p),
        ("stale", ctypes.c_int), ("eps", ctypes.c_float), ("q_scaled", ctypes.c_void_p),
        ("phi_q_f32", ctypes.c_void_p), ("q_scaled_f32", ctypes.c_int),
    ]


class MassGradArgs(ctypes.Structure):
    _fields_ = [
        ("dq_scaled", ctypes.c_void_p), ("dq_dtype", ctypes.c_int),
        ("dphi_q", ctypes.c_void_p), ("dphi_k", ctypes.c_void_p), ("dlog_alpha", ctypes.c_void_p),
        ("workspace", ctypes.c_void_p), ("workspace_bytes", ctypes.c_size_t),
    ]


class GnRowsArgs(ctypes.Structure):
    _fields_ = [
        ("batch", ctypes.c_int), ("heads", ctypes.c_int), ("tokens", ctypes.c_int),
        ("d", ctypes.c_int), ("m", ctypes.c_int), ("nonlinearity", ctypes.c_int), ("eps", ctypes.c_float),
        ("tau", ctypes.c_void_p), ("dtau", ctypes.c_void_p), ("stage", ctypes.c_int), ("flags", ctypes.c_int),
        ("inputs", ctypes.c_void_p * 8), ("outputs", ctypes.c_void_p * 4), ("out_bf16", ctypes.c_void_p),
    ]


class GnPrepArgs(ctypes.Structure):
    _fields_ = [
        ("batch", ctypes.c_int), ("heads", ctypes.c_int), ("tokens", ctypes.c_int), ("d", ctypes.c_int),
        ("rot", ctypes.c_int), ("cos", ctypes.c_void_p), ("sin", ctypes.c_void_p), ("eps", ctypes.c_float),
        ("qkv", ctypes.c_void_p), ("q", ctypes.c_void_p), ("k", ctypes.c_void_p), ("v", ctypes.c_void_p),
        ("dq", ctypes.c_void_p), ("dk", ctypes.c_void_p), ("dv", ctypes.c_void_p), ("dqkv", ctypes.c_void_p),
    ]


TS_GN_RELU2, TS_GN_SILU, TS_GN_TANH = 0, 1, 2
(TS_GN_WRITE_PRE, TS_GN_WRITE_LAM, TS_GN_WRITE_G, TS_GN_QUERY_PRE, TS_GN_FEATURES, TS_GN_OUT, TS_GN_OUT_BWD,
 TS_GN_FEATURES_BWD, TS_GN_QUERY_PRE_BWD, TS_GN_WRITE_G_BWD, TS_GN_WRITE_LAM_BWD, TS_GN_WRITE_PRE_BWD) = range(1, 13)

TS_FEATURE_RELU2, TS_FEATURE_SOFTMAX, TS_FEATURE_BSPLINE = 0, 1, 2
TS_VIEWS_SUM, TS_VIEWS_FAST, TS_VIEWS_STALE = 0, 1, 2

SIGNATURES.update({
    "ts_b200_feature_fwd": (ctypes.c_int, [ctypes.POINTER(FeatureArgs), ctypes.c_void_p]),
    "ts_b200_feature_bwd": (ctypes.c_int, [ctypes.POINTER(FeatureArgs), ctypes.POINTER(FeatureGradArgs),
                                           ctypes.c_void_p]),
    "ts_b200_kread_fwd": (ctypes.c_int, [ctypes.POINTER(KReadArgs), ctypes.c_void_p]),
    "ts_b200_kread_bwd": (ctypes.c_int, [ctypes.POINTER(KReadArgs), ctypes.POINTER(KReadGradArgs),
                                         ctypes.c_void_p]),
    "ts_b200_mass_query_fwd": (ctypes.c_int, [ctypes.POINTER(MassArgs), ctypes.c_void_p]),
    "ts_b200_mass_query_bwd_workspace_bytes": (ctypes.c_size_t, [ctypes.POINTER(MassArgs)]),
    "ts_b200_mass_query_bwd": (ctypes.c_int, [ctypes.POINTER(MassArgs), ctypes.POINTER(MassGradArgs),
                                              ctypes.c_void_p]),
    "ts_b200_gn_rows": (ctypes.c_int, [ctypes.POINTER(GnRowsArgs), ctypes.c_void_p]),
    "ts_b200_gn_prep_fwd": (ctypes.c_int, [ctypes.POINTER(GnPrepArgs), ctypes.c_void_p]),
    "ts_b200_gn_prep_bwd": (ctypes.c_int, [ctypes.POINTER(GnPrepArgs), ctypes.c_void_p]),
})

_lock = threading.Lock()
_lib = None


class ThetaScanB200Error(RuntimeError):
    """A CUDA-side failure reported by the library."""


def load():
    """Load the shared library (once) and bind every declared symbol."""
    global _lib
    with _lock:
        if _lib is None:
            if not os.path.exists(LIB_PATH):
                raise ImportError(
                    f"thetascan_b200: {LIB_PATH} is missing; build it with "
                    "`python -m thetascan_b200.build` (nvcc, sm_100a)")
            lib = ctypes.CDLL(LIB_PATH)
            for name, (restype, argtypes) in SIGNATURES.items():
                fn = getattr(lib, name)
                fn.restype = restype
                fn.argtypes = argtypes
            _lib = lib
    return _lib


def last_error() -> tuple[int, str]:
    buf = ctypes.create_string_buffer(512)
    code = load().ts_b200_last_error(buf, len(buf))
    return code, buf.value.decode(errors="replace")


def check(code: int) -> None:
    """Raise the Python exception matching a nonzero return code."""
    if code == TS_OK:
        return
    _, message = last_error()
    if code == TS_ERR_VALUE:
        raise ValueError(message)
    if code == TS_ERR_NOT_IMPLEMENTED:
        raise NotImplementedError(message)
    raise ThetaScanB200Error(message)


def device_status(stream_handle: int) -> int:
    """Synchronize the stream and return (and clear) the device status word."""
    status = ctypes.c_int(0)
    code = load().ts_b200_device_status(stream_handle, ctypes.byref(status))
    if code not in (TS_OK, TS_ERR_DEVICE):
        check(code)
    return status.value
