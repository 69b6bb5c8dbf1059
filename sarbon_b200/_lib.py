"""ctypes binding of ``libsarbon_sparse.so`` (C ABI declared in ``include/sarbon_sparse.h``).

There is no fallback: if the library is missing or cannot be loaded, every entry point
raises ``SarbonLibraryError``.  Build it with ``python -m sarbon_b200.build_lib``.
"""
from __future__ import annotations

import ctypes as C
from pathlib import Path

LIB_PATH = Path(__file__).resolve().parent / "libsarbon_sparse.so"

SB_OK, SB_EINVAL, SB_EOVERFLOW, SB_ETIMEOUT, SB_ECUDA, SB_ENOMEM = range(6)
SB_F16, SB_F32, SB_F8 = 0, 1, 2
SB_MODE_SKIP, SB_MODE_SPARSE, SB_MODE_DENSE = 0, 1, 2
MODE_NAMES = ("skip", "sparse", "dense")
SB_CREATE_BLOCK_UNITS = 1
SB_CREATE_FP8_S8 = 2
SB_CREATE_FP8_S4 = 4
SB_MAX_LAYERS = 32
SB_MAX_DILATIONS = 4

STATUS_NAMES = {SB_OK: "SB_OK", SB_EINVAL: "SB_EINVAL", SB_EOVERFLOW: "SB_EOVERFLOW",
                SB_ETIMEOUT: "SB_ETIMEOUT", SB_ECUDA: "SB_ECUDA", SB_ENOMEM: "SB_ENOMEM"}


class SarbonLibraryError(RuntimeError):
    """The CUDA library is missing, failed to load, or a call returned an error status."""

    def __init__(self, msg, status=None):
        super().__init__(msg)
        self.status = status


class GemmSrc(C.Structure):
    """sb_gemm_src: one NHWC fp16 source of sb_gemm_conv."""
    _fields_ = [("ptr", C.c_void_p), ("C", C.c_int), ("ld", C.c_longlong), ("img_stride", C.c_longlong)]


class LayerDesc(C.Structure):
    _fields_ = [("src", C.c_int32), ("res", C.c_int32), ("cin", C.c_int32), ("cout", C.c_int32),
                ("stride", C.c_int32), ("out_stride", C.c_int32), ("radius", C.c_int32),
                ("act", C.c_int32)]


class Stats(C.Structure):
    _fields_ = [("skip", C.c_int64), ("sparse", C.c_int64), ("dense", C.c_int64),
                ("last_count", C.c_int64), ("last_mode", C.c_int32), ("error", C.c_int32),
                ("counts", C.c_int32 * SB_MAX_DILATIONS), ("n_dilations", C.c_int32),
                ("dilations", C.c_int32 * SB_MAX_DILATIONS)]


_P = C.c_void_p
_I = C.c_int
_I64 = C.c_int64
_LL = C.c_longlong
# name -> (restype, argtypes); every symbol declared in include/sarbon_sparse.h
PROTOTYPES = {
    "sb_create": (_I, [C.POINTER(LayerDesc), _I, _I, _I, _I, _I, _I, C.c_double, _I, _I, C.POINTER(_P)]),
    "sb_create_ex": (_I, [C.POINTER(LayerDesc), _I, _I, _I, _I, _I, _I, C.c_double, _I, _I, _I, C.POINTER(_P)]),
    "sb_set_m0": (_I, [_P, _I, _I64]),
    "sb_upload_weights": (_I, [_P, _I, C.POINTER(C.c_float), C.POINTER(C.c_float)]),
    "sb_reset": (_I, [_P, _P, _P]),
    "sb_dense": (_I, [_P, _P, _P]),
    "sb_step": (_I, [_P, _P, _P, C.POINTER(_I), C.POINTER(_I64)]),
    "sb_step_u8": (_I, [_P, _P, C.POINTER(C.c_float), C.POINTER(C.c_float), _P, C.POINTER(_I),
                        C.POINTER(_I64)]),
    "sb_step_u8_resized": (_I, [_P, _P, _I, _I, C.POINTER(C.c_float), C.POINTER(C.c_float), _P,
                                C.POINTER(_I), C.POINTER(_I64)]),
    "sb_query": (_I, [_P, _P, C.POINTER(_I), C.POINTER(_I64)]),
    "sb_step_profiled": (_I, [_P, _P, _P, C.POINTER(C.c_float), _I, C.POINTER(_I)]),
    "sb_step_phases": (_I, [_P, _P, _P, C.POINTER(C.c_float)]),
    "sb_result_ptr": (_I, [_P, C.POINTER(_P)]),
    "sb_set_extra": (_I, [_P, _P, _P]),
    "sb_set_fallback": (_I, [_P, _I64, _P]),
    "sb_set_tau": (_I, [_P, C.c_double]),
    "sb_set_dense_check_every": (_I, [_P, _I, _P]),
    "sb_set_cell_gating": (_I, [_P, _I, C.POINTER(_I), _I]),
    "sb_run_sparse_forced": (_I, [_P, _P, _I64, _P]),
    "sb_dense_layers": (_I, [_P, _I, _I, _P]),
    "sb_set_step_graphs": (_I, [_P, _I]),
    "sb_debug_withhold_lookback": (_I, [_P, _I, _I]),
    "sb_cache_ptr": (_I, [_P, _I, C.POINTER(_P), C.POINTER(_I64)]),
    "sb_cache_dtype": (_I, [_P, _I, C.POINTER(_I), C.POINTER(C.c_float)]),
    "sb_set_act_scale": (_I, [_P, _I, C.c_float]),
    "sb_layer_wscale": (_I, [_P, _I, C.POINTER(C.c_float), _I]),
    "sb_layer_variant": (_I, [_P, _I, C.POINTER(_I)]),
    "sb_cell_active_blocks": (_I, [_P, _I, _I, _I, _I, _I, C.POINTER(_I), _I, _P, _P]),
    "sb_boxes_to_block_mask": (_I, [_P, _P, _I, _I, _I, _I, _I, _I, _P, _P]),
    "sb_gate_buffers": (_I, [_P, C.POINTER(_P), C.POINTER(_P), C.POINTER(_P), C.POINTER(_I), C.POINTER(_I)]),
    "sb_debug_lists": (_I, [_P, _I, C.POINTER(_P), C.POINTER(_P), C.POINTER(_P), C.POINTER(_I64), _P]),
    "sb_ms_deform_attn": (_I, [_P, _I, _I, _I, _I, _I, C.POINTER(_I), _I, _P, _P, _I, _I, _P, _P]),
    "sb_block_lists_static": (_I, [_P, _I, _I, _I, C.POINTER(_I), _I, _P, _P, _P, _P]),
    "sb_gemm_conv": (_I, [C.POINTER(GemmSrc), _I, _I, _I, _I, _I, _I, _P, _I, _P, _I, _P, _I,
                          C.c_longlong, C.c_longlong, _P, _I, C.c_longlong, C.c_longlong, _P]),
    "sb_kernels_error": (_I, [_I, C.POINTER(_I)]),
    "sb_layernorm": (_I, [_P, _I, _LL, _P, _I, _LL, _P, _P, C.c_float, _I, _I, _P, _LL, _P, _LL, _P, _LL, _I, C.c_float,
                          _P, _LL, _P]),
    "sb_add_rows": (_I, [_P, _I, _LL, _P, _I, _LL, _I, C.c_float, _I, _I, _P, _LL, _P]),
    "sb_dwconv3x3": (_I, [_P, _LL, _LL, _I, _I, _I, _I, _P, _P, _I, _P, _LL, _LL, _P]),
    "sb_upsample2x": (_I, [_P, _LL, _LL, _I, _I, _I, _I, _P, _LL, _LL, _P]),
    "sb_attention": (_I, [_P, _LL, _LL, _P, _LL, _LL, _P, _LL, _LL, _I, _I, _I, _I, _I, _P, _LL, _LL, _P]),
    "sb_topk_rows": (_I, [_P, _LL, _LL, _I, _I, _I, _P, _I, _P, _LL, _P]),
    "sb_gather_rows": (_I, [_P, _I, _LL, _LL, _I, _P, _LL, _I, _I, _I, _P, _LL, _LL, _P, _LL, _LL, _P]),
    "sb_deform_sample": (_I, [_P, _LL, _LL, C.POINTER(_I), _I, _P, _LL, _LL, _P, _LL, _LL, _P, _I, _LL, _LL, _I, _I, _I,
                              _I, _P, _LL, _LL, _P]),
    "sb_box_enc": (_I, [_P, _LL, _P, _I, _P, _I, _I, _P, _P, _LL, _P]),
    "sb_box_dec": (_I, [_I, _P, _LL, _P, _P, _LL, _P, _LL, _I, _P, C.c_float, _P, _P, _P, _LL, _I, _P]),
    "sb_l2norm_rows": (_I, [_P, _LL, _I, _I, _P, _LL, _P]),
    "sb_stats": (_I, [_P, _P, C.POINTER(Stats)]),
    "sb_last_launch_count": (_I, [_P]),
    "sb_destroy": (_I, [_P]),
    "sb_last_error": (C.c_char_p, []),
    "sb_version": (C.c_char_p, []),
}

_lib = None


def lib():
    """Load the library once; raise SarbonLibraryError if it is absent or incomplete."""
    global _lib
    if _lib is None:
        if not LIB_PATH.exists():
            raise SarbonLibraryError(f"{LIB_PATH} not found: build it with `python -m sarbon_b200.build_lib`")
        try:
            h = C.CDLL(str(LIB_PATH))
        except OSError as e:
            raise SarbonLibraryError(f"cannot load {LIB_PATH}: {e}") from e
        for name, (res, args) in PROTOTYPES.items():
            try:
                fn = getattr(h, name)
            except AttributeError as e:
                raise SarbonLibraryError(f"{LIB_PATH} does not export {name}") from e
            fn.restype, fn.argtypes = res, args
        _lib = h
    return _lib


def check(status, what=""):
    if status != SB_OK:
        msg = lib().sb_last_error().decode(errors="replace")
        raise SarbonLibraryError(f"{what}: {STATUS_NAMES.get(status, status)}: {msg}", status)
