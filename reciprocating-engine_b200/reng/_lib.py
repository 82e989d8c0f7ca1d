"""ctypes binding of libreng_cuda.so (the C ABI declared in include/reng_cuda.h).

The library is built in-tree (reng.build) and loaded from
reciprocating-engine_b200/lib/.  There is no fallback: if the library is
missing or fails to load, every caller gets the OSError.
"""
import ctypes as C
import os

from .build import LIB

RENG_OK = 0
RENG_E_INVAL = -1
RENG_E_CUDA = -2
RENG_E_NOMEM = -3
RENG_E_STATE = -4
RENG_E_UNSUPPORTED = -5
RENG_E_NCCL = -6
RENG_E_TIMEOUT = -7

RENG_MEM_DEVICE = 0
RENG_MEM_HOST = 1

RENG_FP8_E4M3 = 0
RENG_FP8_E5M2 = 1
RENG_SCALING_PCS = 0
RENG_SCALING_HW = 1
RENG_SCALING_UNIT = 2

RENG_WEIGHTS_BF16 = 0
RENG_WEIGHTS_FP8_E4M3 = 1


class RengError(RuntimeError):
    """A negative return code of the C ABI, with reng_last_error()'s message."""

    def __init__(self, code, msg):
        super().__init__("%s (code %d)" % (msg, code))
        self.code = code


class ModelDesc(C.Structure):
    _fields_ = [("hidden", C.c_int32), ("inter", C.c_int32), ("n_layers", C.c_int32),
                ("n_heads", C.c_int32), ("n_kv_heads", C.c_int32), ("head_dim", C.c_int32),
                ("vocab", C.c_int32), ("eps", C.c_float), ("attn_scale", C.c_float),
                ("has_qkv_bias", C.c_int32), ("weights", C.c_int32), ("batch", C.c_int32),
                ("capacity", C.c_int32), ("tp_rank", C.c_int32), ("tp_world", C.c_int32),
                ("device", C.c_int32), ("nccl_id", C.c_void_p), ("qk_norm", C.c_int32)]


class LayerWeights(C.Structure):
    _fields_ = [(n, C.c_void_p) for n in
                ("wq", "wk", "wv", "wo", "wg", "wu", "wd", "g1", "g2", "bq", "bk", "bv", "qn", "kn")] + \
               [("no_rope", C.c_int32)]


class StepTimes(C.Structure):
    _fields_ = [("upload_ms", C.c_float), ("device_ms", C.c_float), ("readback_ms", C.c_float),
                ("steps", C.c_int32), ("kernels_per_step", C.c_int32)]


# (major << 16) | minor of include/reng_cuda.h that the structs below mirror
ABI_VERSION = (0 << 16) | 3


class DeviceInfo(C.Structure):
    _fields_ = [("ordinal", C.c_int32), ("name", C.c_char * 96), ("pci_bus_id", C.c_char * 32),
                ("total_bytes", C.c_uint64), ("sm_count", C.c_int32), ("cc_major", C.c_int32),
                ("cc_minor", C.c_int32)]


# Every exported symbol with its argument types (restype int unless noted).
_P = C.c_void_p
SIGNATURES = {
    "reng_last_error": ([], C.c_char_p),
    "reng_version": ([], C.c_int),
    "reng_device_count": ([_P], C.c_int),
    "reng_device_info_get": ([C.c_int, _P], C.c_int),
    "reng_fp8_quantize": ([_P, C.c_int64, C.c_int64, C.c_int, C.c_int, C.c_float, _P, _P, _P,
                           C.c_int, _P], C.c_int),
    "reng_fp8_quantize_noalloc": ([_P, C.c_int64, C.c_int64, C.c_int, C.c_int, C.c_float, _P, _P,
                                   _P, _P], C.c_int),
    "reng_fp8_encode": ([_P, C.c_int64, C.c_int, _P, _P], C.c_int),
    "reng_fp8_decode": ([_P, C.c_int64, C.c_int, _P, _P], C.c_int),
    "reng_model_create": ([_P, _P, _P, _P, _P, _P, _P, C.c_int, _P], C.c_int),
    "reng_model_destroy": ([_P], C.c_int),
    "reng_model_prefill": ([_P, C.c_int, _P, C.c_int, _P, _P, _P], C.c_int),
    "reng_model_decode": ([_P, _P, C.c_int, _P], C.c_int),
    "reng_model_decode_device": ([_P, _P, C.c_int, _P, _P], C.c_int),
    "reng_model_step_logits": ([_P, _P, _P, _P], C.c_int),
    "reng_model_reset": ([_P, C.c_int], C.c_int),
    "reng_model_position": ([_P, C.c_int, _P], C.c_int),
    "reng_model_tp_exchange": ([_P, _P], C.c_int),
    "reng_tp_peer_wait_check": ([C.c_int], C.c_int),
    "reng_model_device_bytes": ([_P, _P], C.c_int),
    "reng_model_last_times": ([_P, _P], C.c_int),
    "reng_model_time_kernels": ([_P, C.c_int, _P], C.c_int),
    "reng_model_time_kernels_rows": ([_P, C.c_int, C.c_int, _P], C.c_int),
    "reng_model_time_exchange": ([_P, C.c_int, _P], C.c_int),
    "reng_tp_unique_id": ([_P], C.c_int),
    "reng_gemm_bf16": ([_P, C.c_int, C.c_int, _P, C.c_int, _P, C.c_int, C.c_int, _P, C.c_int], C.c_int),
}

_lib = None


def lib():
    """Load libreng_cuda.so once (raises OSError if it is not built)."""
    global _lib
    if _lib is None:
        path = os.environ.get("RENG_CUDA_LIB", LIB)  # another build of the library, for A/B runs
        if not os.path.exists(path):
            raise OSError("libreng_cuda.so is not built (%s); run reng.build.build()" % path)
        L = C.CDLL(path, mode=C.RTLD_GLOBAL)
        # the version first: a library of another version may lack symbols
        # these bindings name, and its structs may have another layout
        L.reng_version.argtypes = []
        L.reng_version.restype = C.c_int
        if L.reng_version() != ABI_VERSION:
            raise OSError("%s has ABI version %#x, these bindings %#x: rebuild the library"
                          % (path, L.reng_version(), ABI_VERSION))
        for name, (args, res) in SIGNATURES.items():
            try:
                f = getattr(L, name)
            except AttributeError:
                raise OSError("%s does not export %s: rebuild the library" % (path, name)) from None
            f.argtypes = args
            f.restype = res
        _lib = L
    return _lib


def check(rc):
    """Raise RengError for a negative return code."""
    if rc != RENG_OK:
        msg = lib().reng_last_error()
        raise RengError(rc, msg.decode() if msg else "")
    return rc


def call(name, *args):
    return check(getattr(lib(), name)(*args))


def devices():
    """The CUDA devices of this host, one dict each (reng-hal's
    enumerate_devices, crates/reng-hal/src/lib.rs:62: empty, not an error,
    on a host without devices)."""
    n = C.c_int(0)
    call("reng_device_count", C.byref(n))
    out = []
    for d in range(n.value):
        info = DeviceInfo()
        call("reng_device_info_get", d, C.byref(info))
        out.append({"ordinal": info.ordinal, "name": info.name.decode(errors="replace"),
                    "pci_bus_id": info.pci_bus_id.decode(errors="replace"),
                    "total_bytes": int(info.total_bytes), "sm_count": info.sm_count,
                    "compute_capability": (info.cc_major, info.cc_minor)})
    return out
