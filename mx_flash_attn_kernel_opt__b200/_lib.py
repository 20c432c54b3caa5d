"""ctypes binding of libpgqa.so (the C ABI declared in include/pgqa.h).

The library is loaded from this package directory only; there is no fallback
implementation: if the shared object is missing or does not export the ABI, every
entry point raises.
"""
import ctypes
import os
import threading

_PKG_DIR = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_PKG_DIR, "libpgqa.so")

# Every symbol declared in include/pgqa.h, with its ctypes signature.
c_void_p, c_int64, c_int32, c_size_t, c_float, c_char_p = (
    ctypes.c_void_p, ctypes.c_int64, ctypes.c_int32, ctypes.c_size_t, ctypes.c_float,
    ctypes.c_char_p)


class PgqaPlan(ctypes.Structure):
    _fields_ = [
        ("grid_ctas", ctypes.c_int32),
        ("warps_per_cta", ctypes.c_int32),
        ("stages", ctypes.c_int32),
        ("min_chunks_per_warp", ctypes.c_int32),
        ("head_groups", ctypes.c_int32),
        ("units_per_seq", ctypes.c_int32),
        ("smem_bytes", ctypes.c_int32),
        ("status", ctypes.c_int32),
        ("workspace_bytes", ctypes.c_int64),
        ("groups_per_unit", ctypes.c_int32),
        ("reserved", ctypes.c_int32),
    ]

    def as_dict(self):
        return {name: getattr(self, name) for name, _ in self._fields_}


class PgqaDecodeArgs(ctypes.Structure):
    """include/pgqa.h pgqa_decode_args (pgqa_decode_ex)."""
    _fields_ = [
        ("struct_size", c_size_t),
        ("q", c_void_p), ("k_cache", c_void_p), ("v_cache", c_void_p),
        ("k_new", c_void_p), ("v_new", c_void_p), ("out", c_void_p),
        ("softmax_lse", c_void_p), ("seq_lens", c_void_p), ("block_table", c_void_p),
        ("batch_size", c_int64), ("seqlen_q", c_int64), ("seqlen_new", c_int64),
        ("num_heads", c_int64), ("num_heads_k", c_int64), ("headdim", c_int64),
        ("page_size", c_int64), ("num_pages", c_int64), ("bt_stride", c_int64),
        ("max_seqlen", c_int64), ("causal", c_int64),
        ("scale", c_float), ("kv_format", ctypes.c_int32),
        ("k_scale", c_void_p), ("v_scale", c_void_p),
        ("workspace", c_void_p), ("workspace_bytes", c_size_t),
    ]


SIGNATURES = {
    "run_kernel": (None, [c_void_p] * 4 + [c_void_p, c_void_p] + [c_int64] * 9),
    "pgqa_decode_v1": (ctypes.c_int, [c_void_p] * 6 + [c_int64] * 8 +
                       [c_float, c_void_p, c_size_t, c_void_p]),
    "pgqa_decode_noalloc": (ctypes.c_int, [c_void_p] * 6 + [c_int64] * 8 + [c_float, c_void_p]),
    "pgqa_decode_v2": (ctypes.c_int, [c_void_p] * 6 + [c_int64] * 10 +
                       [c_float, c_void_p, c_size_t, c_void_p]),
    "pgqa_decode_ex": (ctypes.c_int, [ctypes.POINTER(PgqaDecodeArgs), c_void_p]),
    "pgqa_workspace_size_v2": (c_size_t, [c_int64] * 6),
    "pgqa_append_kv": (ctypes.c_int, [c_void_p] * 6 + [c_int64] * 7 + [c_void_p] * 2),
    "pgqa_decode_kvcache": (ctypes.c_int, [c_void_p] * 8 + [c_int64] * 11 +
                            [c_float, c_void_p, c_size_t, c_void_p]),
    "pgqa_append_kv_fp8": (ctypes.c_int, [c_void_p] * 6 + [c_int64] * 7 + [c_void_p] * 2),
    "pgqa_decode_fp8": (ctypes.c_int, [c_void_p] * 8 + [c_int64] * 11 +
                        [c_float, c_void_p, c_void_p, c_void_p, c_size_t, c_void_p]),
    "pgqa_workspace_size": (c_size_t, [c_int64] * 5),
    "pgqa_workspace_init": (ctypes.c_int, [c_void_p, c_size_t, c_void_p]),
    "pgqa_last_status": (ctypes.c_int, []),
    "pgqa_status_string": (c_char_p, [ctypes.c_int]),
    "pgqa_check_device_error": (ctypes.c_int, [c_void_p, c_void_p]),
    "pgqa_noalloc_check_device_error": (ctypes.c_int, [c_void_p]),
    "pgqa_make_plan": (ctypes.c_int, [c_int64] * 5 + [c_int32, c_int32,
                                                      ctypes.POINTER(PgqaPlan)]),
    "pgqa_simulate_partition": (c_int64, [c_void_p, c_int64, c_int64, c_int64,
                                          ctypes.POINTER(PgqaPlan), c_void_p, c_void_p]),
    "pgqa_version": (c_char_p, []),
}

STATUS = {
    0: "PGQA_OK", 1: "PGQA_ERR_NULL_POINTER", 2: "PGQA_ERR_BAD_SHAPE",
    3: "PGQA_ERR_UNSUPPORTED", 4: "PGQA_ERR_MISALIGNED", 5: "PGQA_ERR_WORKSPACE",
    6: "PGQA_ERR_CUDA", 7: "PGQA_ERR_NO_DEVICE", 8: "PGQA_ERR_DEVICE_TIMEOUT",
    9: "PGQA_ERR_DEVICE_BAD_PAGE", 10: "PGQA_ERR_DEVICE_BAD_SEQLEN", 11: "PGQA_ERR_SCRATCH_LIMIT",
}

_lock = threading.Lock()
_lib = None


class PgqaError(RuntimeError):
    def __init__(self, status, what=""):
        self.status = status
        name = STATUS.get(status, str(status))
        text = ""
        try:
            text = lib().pgqa_status_string(status).decode()
        except Exception:  # pragma: no cover - library unavailable
            pass
        super().__init__(f"{what}: {name} ({text})" if what else f"{name} ({text})")


def lib():
    """Load libpgqa.so (building it first if it is absent and nvcc is available)."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is None:
            if not os.path.exists(LIB_PATH):
                from . import build as _build
                _build.build()
            handle = ctypes.CDLL(LIB_PATH)
            for name, (res, args) in SIGNATURES.items():
                fn = getattr(handle, name)  # AttributeError if the ABI is incomplete
                fn.restype = res
                fn.argtypes = args
            _lib = handle
    return _lib


def check(status, what=""):
    if status != 0:
        raise PgqaError(status, what)
    return status
