"""B200 (sm_100a) paged grouped-query-attention decode.

Drop-in for the reference operator `run_kernel` (C ABI in include/pgqa.h, built as
libpgqa.so in this directory).  Python entry points:

  run_kernel(...)       the reference's operator surface (tensors + 9 integers)
  run_kernel_cabi(...)  the raw C symbol through ctypes, as the reference harness calls it
  decode(...)           general form: explicit scale, pool size and table stride,
                        several query tokens, optional append of new K/V tokens
  append_kv(...)        the append-KV step alone
  flash_attn_with_kvcache(...)  flash-attn's argument list, for the paged case
"""
from ._lib import LIB_PATH, PgqaError, lib  # noqa: F401
from .ops import (  # noqa: F401
    append_kv,
    check_device_error,
    decode,
    flash_attn_with_kvcache,
    make_plan,
    run_kernel,
    run_kernel_cabi,
    workspace_for,
)

__all__ = ["run_kernel", "run_kernel_cabi", "decode", "append_kv", "flash_attn_with_kvcache",
           "make_plan", "check_device_error", "workspace_for", "PgqaError", "lib", "LIB_PATH"]
