"""CPU oracle for the paged-GQA decode -- TEST INFRASTRUCTURE ONLY.

Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline / reference arm may
import this package, and only as the checker or the timed CPU baseline; the product
(mx_flash_attn_kernel_opt__b200) never calls it.

Parity pin: paged_decode_ref is checked (tests/test_oracle.py) against golden vectors
produced by the reference's own implementation of this path
(submission_c500_regions.py:run_kernel, run on the CPU under the Triton interpreter by
tests/golden/gen_golden.py).
"""
from .append_kv import append_kv_ref  # noqa: F401
from .paged_decode import (  # noqa: F401
    lse_combine_ref,
    paged_decode_fp8_ref,
    paged_decode_ref,
    split_partials_ref,
    split_decode_ref,
    match_stats,
)
