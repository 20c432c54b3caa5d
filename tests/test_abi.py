"""The C ABI: libpgqa.so loads, exports every symbol include/pgqa.h declares, and
validates its arguments on the host (no GPU needed)."""
import ctypes
import os
import re
import subprocess

import pytest
import torch

from mx_flash_attn_kernel_opt__b200 import _lib, make_plan

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(REPO, "include", "pgqa.h")


def declared_functions():
    text = open(HEADER).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    names = re.findall(r"^[A-Za-z_][\w \*]*?\b([A-Za-z_]\w*)\s*\(", text, flags=re.M)
    return sorted(set(n for n in names if n not in ("if", "while")))


def test_header_declares_the_reference_symbol():
    names = declared_functions()
    assert "run_kernel" in names
    assert {"pgqa_decode_v1", "pgqa_decode_v2", "pgqa_workspace_size", "pgqa_make_plan"} <= set(names)


def test_library_loads_and_exports_every_declared_symbol():
    L = _lib.lib()
    for name in declared_functions():
        assert hasattr(L, name), name
        assert name in _lib.SIGNATURES, f"{name} has no ctypes signature"
    out = subprocess.run(["nm", "-D", "--defined-only", _lib.LIB_PATH], capture_output=True,
                         text=True).stdout
    exported = set(line.split()[-1] for line in out.splitlines() if " T " in line)
    for name in declared_functions():
        assert name in exported, name


def test_status_strings():
    L = _lib.lib()
    for code in _lib.STATUS:
        assert L.pgqa_status_string(code).decode() != "unknown status"
    assert L.pgqa_status_string(999).decode() == "unknown status"
    assert L.pgqa_version().decode().startswith("pgqa-b200")


@pytest.mark.parametrize("shape", [(4, 32, 8, 16), (2, 64, 8, 16), (256, 32, 8, 16),
                                   (64, 28, 4, 64), (512, 64, 8, 16), (8, 32, 4, 16)])
def test_plan_for_benchmark_shapes(shape):
    B, Hq, Hkv, P = shape
    st, plan = make_plan(B, Hq, Hkv, 128, P)
    assert st == 0 and plan.status == 0
    assert plan.grid_ctas == 148
    assert plan.smem_bytes <= 232448
    assert plan.stages >= 2
    assert plan.head_groups == -(-(Hq // Hkv) // 8)
    assert plan.workspace_bytes > 0


def test_plan_rejects_bad_shapes():
    assert make_plan(0, 32, 8, 128, 16)[0] == 2
    assert make_plan(4, 30, 8, 128, 16)[0] == 2      # Hq % Hkv != 0
    assert make_plan(4, 32, 8, 64, 16)[0] == 3       # D != 128
    assert make_plan(4, 32, 8, 128, 8)[0] == 3       # page size not a multiple of 16
    st, plan = make_plan(4, 32, 8, 128, 16, num_sms=132, smem_optin=232448)
    assert st == 0 and plan.grid_ctas == 132


def test_plan_limits_batch_by_prefix_table():
    # the per-sequence chunk prefix lives in shared memory next to the TMA rings
    _, ok = make_plan(20000, 32, 8, 128, 16)
    assert ok.status == 0 and ok.smem_bytes <= 232448
    st, _ = make_plan(40000, 32, 8, 128, 16)
    assert st == 3


FAKE = ctypes.c_void_p(0x10000)


def _v1(**kw):
    a = dict(q=FAKE, k=FAKE, v=FAKE, out=FAKE, sl=FAKE, bt=FAKE, B=4, Hq=32, Hkv=8, D=128,
             P=16, num_pages=64, stride=16, max_seqlen=256, scale=0.088, ws=None, wsb=0,
             stream=None)
    a.update(kw)
    return _lib.lib().pgqa_decode_v1(a["q"], a["k"], a["v"], a["out"], a["sl"], a["bt"], a["B"],
                                     a["Hq"], a["Hkv"], a["D"], a["P"], a["num_pages"],
                                     a["stride"], a["max_seqlen"], a["scale"], a["ws"],
                                     a["wsb"], a["stream"])


def test_extended_entry_validates_arguments():
    assert _v1(q=None) == 1
    assert _v1(B=0) == 2
    assert _v1(Hq=31) == 2
    assert _v1(D=256) == 3
    assert _v1(P=24) == 3
    assert _v1(num_pages=0) == 2
    assert _v1(max_seqlen=10**6) == 2          # above stride * page_size
    assert _v1(scale=-1.0) == 2
    assert _v1(k=ctypes.c_void_p(0x10008)) == 4  # TMA base must be 16-byte aligned
    assert _lib.lib().pgqa_last_status() == 4


def _ex_args(**kw):
    a = _lib.PgqaDecodeArgs(
        struct_size=ctypes.sizeof(_lib.PgqaDecodeArgs), q=0x10000, k_cache=0x20000,
        v_cache=0x30000, out=0x40000, seq_lens=0x50000, block_table=0x60000, batch_size=2,
        seqlen_q=1, num_heads=32, num_heads_k=8, headdim=128, page_size=16, num_pages=8,
        bt_stride=4, scale=0.088, kv_format=0)
    for k, v in kw.items():
        setattr(a, k, v)
    return a


def test_struct_entry_validates_arguments():
    """pgqa_decode_ex checks its struct before anything else (no device needed)."""
    L = _lib.lib()
    assert L.pgqa_decode_ex(None, None) == 1
    assert L.pgqa_decode_ex(ctypes.byref(_ex_args(struct_size=8)), None) == 2
    assert L.pgqa_decode_ex(ctypes.byref(_ex_args(kv_format=2)), None) == 3
    assert L.pgqa_decode_ex(ctypes.byref(_ex_args(k_scale=0x70000)), None) == 2
    assert L.pgqa_decode_ex(ctypes.byref(_ex_args(softmax_lse=0x70002)), None) == 4
    assert L.pgqa_decode_ex(ctypes.byref(_ex_args(batch_size=0)), None) == 2
    assert L.pgqa_decode_ex(ctypes.byref(_ex_args(q=None)), None) == 1
    assert L.pgqa_last_status() == 1


def test_struct_layout_matches_the_header(tmp_path):
    """The ctypes mirror of pgqa_decode_args has the C struct's size and field offsets
    (a probe compiled with gcc against include/pgqa.h)."""
    import shutil
    if shutil.which("gcc") is None:
        pytest.skip("gcc not available")
    fields = [f for f, _ in _lib.PgqaDecodeArgs._fields_]
    src = tmp_path / "probe.c"
    src.write_text("#include <stdio.h>\n#include <stddef.h>\n#include \"pgqa.h\"\nint main(void) {\n"
                   + '  printf("%zu\\n", sizeof(pgqa_decode_args));\n'
                   + "".join(f'  printf("%zu\\n", offsetof(pgqa_decode_args, {f}));\n' for f in fields)
                   + "  return 0;\n}\n")
    exe = tmp_path / "probe"
    cuda_inc = "/usr/local/cuda/include"
    r = subprocess.run(["gcc", "-I", os.path.join(REPO, "include"), "-I", cuda_inc, str(src),
                        "-o", str(exe)], capture_output=True, text=True)
    assert r.returncode == 0, r.stderr
    got = [int(x) for x in subprocess.run([str(exe)], capture_output=True, text=True).stdout.split()]
    assert got[0] == ctypes.sizeof(_lib.PgqaDecodeArgs)
    assert got[1:] == [getattr(_lib.PgqaDecodeArgs, f).offset for f in fields]


@pytest.mark.skipif(torch.cuda.is_available(), reason="checks the no-device path")
def test_valid_call_without_device_reports_no_device():
    assert _v1() == 7


def test_reference_entry_validates_arguments():
    L = _lib.lib()
    args = [FAKE] * 6
    L.run_kernel(*args, 0, 16, 1, 32, 8, 128, 16, 64, 0)
    assert L.pgqa_last_status() == 2              # batch_size 0
    L.run_kernel(*args, 4, 16, 1, 32, 8, 128, 16, 63, 0)
    assert L.pgqa_last_status() == 2              # num_blocks % batch_size
    L.run_kernel(*args, 4, 16, 0, 32, 8, 128, 16, 64, 0)
    assert L.pgqa_last_status() == 2              # seqlen_q < 1
    L.run_kernel(*args, 4, 16, 1, 32, 8, 128, 16, 64, 2)
    assert L.pgqa_last_status() == 3              # causal not 0 / 1
    L.run_kernel(*args, 4, 1000, 1, 32, 8, 128, 16, 64, 0)
    assert L.pgqa_last_status() == 2              # seqlen_k above table capacity
    L.run_kernel(*args, 4, 16, 1, 32, 8, 96, 16, 64, 0)
    assert L.pgqa_last_status() == 3              # headdim


def test_workspace_size_is_zero_for_invalid_shapes():
    L = _lib.lib()
    assert L.pgqa_workspace_size(0, 32, 8, 128, 16) == 0
    assert L.pgqa_workspace_size(4, 32, 8, 128, 16) > 0
    assert L.pgqa_workspace_size_v2(4, 0, 32, 8, 128, 16) == 0
    assert L.pgqa_last_status() == 2
    # a batch whose length prefix does not fit in shared memory: unsupported, not bad
    assert L.pgqa_workspace_size(40000, 8, 2, 128, 16) == 0
    assert L.pgqa_last_status() == 3
    # more query tokens -> more row groups per KV head -> more arrival counters
    assert L.pgqa_workspace_size_v2(4, 4, 32, 8, 128, 16) > L.pgqa_workspace_size(4, 32, 8, 128, 16)


def test_plan_carries_two_row_groups_per_unit_when_a_kv_head_has_more():
    """g = 16: two groups of 8 query rows per KV head share every K/V tile (one unit per
    KV head instead of two); g <= 8 keeps one group per unit."""
    L = _lib.lib()
    wide = _lib.PgqaPlan()
    assert L.pgqa_make_plan(4, 64, 4, 128, 16, 148, 232448, ctypes.byref(wide)) == 0
    assert (wide.head_groups, wide.groups_per_unit, wide.units_per_seq) == (2, 2, 4)
    odd = _lib.PgqaPlan()  # 3 groups -> 2 units per KV head, the last one half empty
    assert L.pgqa_make_plan(4, 48, 2, 128, 16, 148, 232448, ctypes.byref(odd)) == 0
    assert (odd.head_groups, odd.groups_per_unit, odd.units_per_seq) == (3, 2, 4)
    narrow = _lib.PgqaPlan()
    assert L.pgqa_make_plan(4, 32, 8, 128, 16, 148, 232448, ctypes.byref(narrow)) == 0
    assert (narrow.head_groups, narrow.groups_per_unit, narrow.units_per_seq) == (1, 1, 8)


def test_a_c_program_builds_and_links_against_the_header(tmp_path):
    """A C caller compiles against include/pgqa.h alone (no CUDA or torch headers), links
    libpgqa.so and gets host-side answers: status strings, refused arguments, the struct
    entry point's checks."""
    import shutil
    if shutil.which("gcc") is None:
        pytest.skip("gcc not available")
    src = tmp_path / "caller.c"
    src.write_text(r"""
#include <stdio.h>
#include <string.h>
#include "pgqa.h"
int main(void) {
    int fails = 0;
    if (strlen(pgqa_status_string(PGQA_ERR_BAD_SHAPE)) == 0) fails++;
    /* null pointers are refused before anything touches a device */
    if (pgqa_decode_v1(0, 0, 0, 0, 0, 0, 2, 32, 8, 128, 16, 8, 4, 0, 0.088f, 0, 0, 0)
        != PGQA_ERR_NULL_POINTER) fails++;
    if (pgqa_last_status() != PGQA_ERR_NULL_POINTER) fails++;
    pgqa_decode_args a;
    memset(&a, 0, sizeof(a));
    a.struct_size = sizeof(a) - 8;   /* a caller built against another layout */
    if (pgqa_decode_ex(&a, 0) != PGQA_ERR_BAD_SHAPE) fails++;
    if (pgqa_decode_ex(0, 0) != PGQA_ERR_NULL_POINTER) fails++;
    printf("fails=%d\n", fails);
    return fails;
}
""")
    exe = tmp_path / "caller"
    libdir = os.path.dirname(_lib.LIB_PATH)
    r = subprocess.run(["gcc", "-std=c99", "-Wall", "-Werror", "-I", os.path.join(REPO, "include"),
                        str(src), "-L", libdir, "-lpgqa", "-Wl,-rpath," + libdir, "-o", str(exe)],
                       capture_output=True, text=True)
    assert r.returncode == 0, r.stderr
    r = subprocess.run([str(exe)], capture_output=True, text=True, timeout=120)
    assert r.returncode == 0 and "fails=0" in r.stdout, r.stdout + r.stderr
