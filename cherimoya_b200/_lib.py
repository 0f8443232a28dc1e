"""ctypes binding of libcherimoya_b200.so (C ABI: include/cherimoya_b200.h).

The library is the only compute path for CUDA tensors. If it is missing or
fails to load, every engine call raises; there is no CPU or PyTorch
fallback behind it.
"""

import ctypes
import os

LIB_PATH = os.path.join(os.path.dirname(os.path.abspath(__file__)), "libcherimoya_b200.so")

CHM_OK = 0
MODE_FP32 = 0
MODE_BF16 = 1
INPUT_F32 = 0
INPUT_BF16 = 1
ABI_VERSION = 1

# every symbol declared in include/cherimoya_b200.h
EXPORTED = (
    "chm_abi_version", "chm_error_string", "chm_validate", "chm_packed_weights_bytes",
    "chm_pack_weights", "chm_forward_workspace_bytes", "chm_forward", "chm_forward_bases",
    "chm_ism_workspace_bytes", "chm_ism", "chm_ism_ex", "chm_wrapper_epilogue",
    "chm_variant_workspace_bytes", "chm_variant",
    "chm_block_packed_bytes", "chm_pack_block", "chm_block_workspace_bytes",
    "chm_block_forward", "chm_forward_noalloc", "chm_noalloc_read_status", "chm_read_status",
    "chm_selftest_wait_timeout", "chm_last_launch_count", "chm_timing_enable",
    "chm_timing_collect",
)
TIMING_CLASSES = ("stem", "stats", "mlp", "profile_head", "count_head", "score", "other")


class ModelDesc(ctypes.Structure):
    """chm_model_desc."""
    _fields_ = [
        ("n_filters", ctypes.c_int32),
        ("n_layers", ctypes.c_int32),
        ("expansion", ctypes.c_int32),
        ("n_outputs", ctypes.c_int32),
        ("n_groups", ctypes.c_int32),
        ("n_control_tracks", ctypes.c_int32),
        ("trimming", ctypes.c_int32),
        ("seq_len", ctypes.c_int32),
        ("residual_scale", ctypes.c_float),
        ("mode", ctypes.c_int32),
    ]


_fp = ctypes.POINTER(ctypes.c_float)


class Params(ctypes.Structure):
    """chm_params (per-layer fields point to host arrays of device pointers)."""
    _fields_ = [
        ("iconv_weight", ctypes.c_void_p),
        ("iconv_bias", ctypes.c_void_p),
        ("conv_weight", ctypes.POINTER(ctypes.c_void_p)),
        ("linear1_weight", ctypes.POINTER(ctypes.c_void_p)),
        ("linear2_weight", ctypes.POINTER(ctypes.c_void_p)),
        ("fconv_weight", ctypes.c_void_p),
        ("fconv_bias", ctypes.c_void_p),
        ("linear_weight", ctypes.c_void_p),
        ("linear_bias", ctypes.c_void_p),
    ]


_lib = None
_load_error = None


def _declare(lib):
    vp, i32, sz = ctypes.c_void_p, ctypes.c_int32, ctypes.c_size_t
    desc_p = ctypes.POINTER(ModelDesc)
    sigs = {
        "chm_abi_version": (i32, []),
        "chm_error_string": (ctypes.c_char_p, [i32]),
        "chm_validate": (i32, [desc_p]),
        "chm_packed_weights_bytes": (sz, [desc_p]),
        "chm_pack_weights": (i32, [desc_p, ctypes.POINTER(Params), vp, sz, vp]),
        "chm_forward_workspace_bytes": (sz, [desc_p, i32]),
        "chm_forward": (i32, [desc_p, vp, i32, vp, i32, vp, vp, vp, vp, sz, vp]),
        "chm_forward_bases": (i32, [desc_p, vp, i32, vp, vp, vp, vp, vp, sz, vp]),
        "chm_ism_workspace_bytes": (sz, [desc_p, i32, i32]),
        "chm_ism": (i32, [desc_p, vp, i32, vp, i32, i32, i32, vp, vp, vp, sz, vp]),
        "chm_ism_ex": (i32, [desc_p, vp, i32, vp, i32, i32, i32, vp, vp, vp, vp, sz, vp]),
        "chm_wrapper_epilogue": (i32, [desc_p, i32, vp, vp, vp, vp, vp, vp, sz, vp]),
        "chm_variant_workspace_bytes": (sz, [desc_p, i32]),
        "chm_variant": (i32, [desc_p, vp, i32, vp, vp, vp, vp, vp, sz, vp]),
        "chm_block_packed_bytes": (sz, [i32, i32]),
        "chm_pack_block": (i32, [i32, i32, ctypes.c_float, vp, vp, vp, vp, sz, vp]),
        "chm_block_workspace_bytes": (sz, [i32, i32, i32, i32]),
        "chm_block_forward": (i32, [i32, i32, i32, i32, i32, i32, vp, vp, vp, vp, sz, vp]),
        "chm_forward_noalloc": (i32, [desc_p, vp, i32, vp, i32, vp, vp, vp, vp]),
        "chm_read_status": (i32, [vp, vp]),
        "chm_noalloc_read_status": (i32, [vp]),
        "chm_selftest_wait_timeout": (i32, [vp, sz, vp]),
        "chm_last_launch_count": (ctypes.c_int64, []),
        "chm_timing_enable": (None, [i32]),
        "chm_timing_collect": (i32, [ctypes.POINTER(ctypes.c_double),
                                     ctypes.POINTER(ctypes.c_int64)]),
    }
    for name, (res, args) in sigs.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args


def load():
    """Return the loaded library; raise RuntimeError if it is unavailable."""
    global _lib, _load_error
    if _lib is not None:
        return _lib
    if not os.path.exists(LIB_PATH):
        raise RuntimeError(
            "cherimoya_b200: {} is not built (run `python -m cherimoya_b200.csrc.build`); "
            "the CUDA engine has no fallback".format(LIB_PATH))
    try:
        lib = ctypes.CDLL(LIB_PATH)
        _declare(lib)
    except OSError as e:  # pragma: no cover - depends on the machine
        _load_error = e
        raise RuntimeError("cherimoya_b200: failed to load {}: {}".format(LIB_PATH, e))
    if lib.chm_abi_version() != ABI_VERSION:
        raise RuntimeError("cherimoya_b200: ABI version mismatch")
    _lib = lib
    return lib


def timing_enable(on=True):
    load().chm_timing_enable(1 if on else 0)


def timing_collect():
    """{class: (ms, launches)} of the engine launches timed since the last
    collect (synchronises their events)."""
    n = len(TIMING_CLASSES)
    ms = (ctypes.c_double * n)()
    cnt = (ctypes.c_int64 * n)()
    check(load().chm_timing_collect(ms, cnt), "timing_collect")
    return {name: (ms[i], cnt[i]) for i, name in enumerate(TIMING_CLASSES)}


def error_string(status):
    return load().chm_error_string(int(status)).decode()


def check(status, what):
    if status != CHM_OK:
        raise RuntimeError("cherimoya_b200.{}: {} (status {})".format(
            what, error_string(status), status))


def make_desc(n_filters, n_layers, expansion, n_outputs, n_groups, n_control_tracks,
              trimming, seq_len, residual_scale, mode):
    return ModelDesc(int(n_filters), int(n_layers), int(expansion), int(n_outputs),
                     int(n_groups), int(n_control_tracks), int(trimming), int(seq_len),
                     float(residual_scale), int(mode))
