"""The allocation-free entry point, pgqa_decode_noalloc, called through the C ABI.

Some callers cannot allocate device memory when they call the operator: serving engines
that keep nearly all of HBM in their own pool and allow no allocation on the hot path,
and plugin hosts that hand the operator only its inputs and outputs.  For them the
library keeps a fixed scratch array of its own.  These tests check that:

  * two calls in a row give exactly the bytes pgqa_decode_v1 gives with a caller
    workspace (the same kernel on the same plan; a difference would be a scratch layout
    fault, not rounding), and match the CPU oracle at the parity tolerance;
  * a bad block-table entry is reported through pgqa_noalloc_check_device_error, and
    the error word is clear again after it was read;
  * a shape needing more than the fixed scratch is refused before anything runs.

The file is named so that pytest collects it last.
"""
import ctypes

import pytest
import torch

import mx_flash_attn_kernel_opt__b200 as pgqa
from mx_flash_attn_kernel_opt__b200 import _lib, inputs, make_plan
from oracle import match_stats, paged_decode_ref

pytestmark = pytest.mark.gpu

ATOL = RTOL = 1e-2


def _noalloc(d, out, stream):
    vp = ctypes.c_void_p
    return _lib.lib().pgqa_decode_noalloc(
        vp(d.q.data_ptr()), vp(d.k.data_ptr()), vp(d.v.data_ptr()), vp(out.data_ptr()),
        vp(d.seq_lens.data_ptr()), vp(d.block_table.data_ptr()), d.batch, d.num_heads,
        d.num_heads_k, 128, d.page_size, d.num_pages, d.block_table.stride(0), 0,
        ctypes.c_float(d.scale), vp(stream.cuda_stream))


def _v1(d, out, ws, stream):
    vp = ctypes.c_void_p
    return _lib.lib().pgqa_decode_v1(
        vp(d.q.data_ptr()), vp(d.k.data_ptr()), vp(d.v.data_ptr()), vp(out.data_ptr()),
        vp(d.seq_lens.data_ptr()), vp(d.block_table.data_ptr()), d.batch, d.num_heads,
        d.num_heads_k, 128, d.page_size, d.num_pages, d.block_table.stride(0), 0,
        ctypes.c_float(d.scale), vp(ws.data_ptr()), ws.numel(), vp(stream.cuda_stream))


def _check_noalloc_errors(stream):
    return _lib.lib().pgqa_noalloc_check_device_error(ctypes.c_void_p(stream.cuda_stream))


@pytest.mark.parametrize("case", ["c1", "spj07", "c3", "g16"])
def test_noalloc_matches_workspace_entry_point_on_two_calls(case, cuda_device):
    if case.startswith("spj"):
        inp = inputs.spj_case(int(case[3:]), table="permuted")
    elif case == "g16":  # two row groups per unit
        inp = inputs.custom_case(6, 64, 4, 32, [1, 17, 300, 1025, 4000, 77], seed=5)
    else:
        inp = inputs.baseline_config(case)
    d = inp.to(cuda_device)
    stream = torch.cuda.current_stream(cuda_device)
    # the existing entry point, through the C ABI with a caller-provided workspace
    need = _lib.lib().pgqa_workspace_size(d.batch, d.num_heads, d.num_heads_k, 128, d.page_size)
    ws = torch.zeros(need, dtype=torch.uint8, device=cuda_device)
    ref_out = torch.full_like(d.q, float("nan"))
    assert _v1(d, ref_out, ws, stream) == 0
    torch.cuda.synchronize()
    for call in range(2):
        out = torch.full_like(d.q, float("nan"))
        st = _noalloc(d, out, stream)
        assert st == 0, _lib.lib().pgqa_status_string(st).decode()
        torch.cuda.synchronize()
        assert torch.equal(out, ref_out), f"call {call}: differs from pgqa_decode_v1"
        assert _check_noalloc_errors(stream) == 0
    ref = paged_decode_ref(inp.q, inp.k, inp.v, inp.block_table, inp.seq_lens)
    a = out.float().cpu()
    frac, outlier, maxd = match_stats(a, ref)
    assert not outlier and frac >= 0.99, (frac, maxd)
    assert torch.allclose(a, ref, atol=ATOL, rtol=RTOL), maxd


def test_noalloc_reports_a_bad_page_id(cuda_device):
    """A block-table entry outside [0, num_pages) is flagged, not dereferenced: the
    kernel checks each page id before its tile load.  The error stays in the scratch's
    error word across a later good call until it is read, and reading clears it."""
    inp = inputs.custom_case(3, 32, 8, 16, [40, 300, 17], seed=21)
    d = inp.to(cuda_device)
    stream = torch.cuda.current_stream(cuda_device)
    assert _check_noalloc_errors(stream) == 0
    bad = d.block_table.clone()
    bad[1, 5] = d.num_pages + 1000  # inside the row's first ceil(300/16) = 19 entries
    d_bad = inputs.DecodeInputs(q=d.q, k=d.k, v=d.v, block_table=bad, seq_lens=d.seq_lens,
                                scale=d.scale)
    out = torch.empty_like(d.q)
    assert _noalloc(d_bad, out, stream) == 0
    assert _noalloc(d, out, stream) == 0  # a good call does not hide the earlier error
    torch.cuda.synchronize()
    assert _check_noalloc_errors(stream) == 9  # PGQA_ERR_DEVICE_BAD_PAGE
    assert _check_noalloc_errors(stream) == 0
    ref = paged_decode_ref(inp.q, inp.k, inp.v, inp.block_table, inp.seq_lens)
    assert torch.allclose(out.float().cpu(), ref, atol=ATOL, rtol=RTOL)


def test_noalloc_refuses_shapes_beyond_its_scratch(cuda_device):
    # 12000 sequences x 64 KV heads need ~25 MB of arrival counters, far beyond 4 MiB
    st, plan = make_plan(12000, 512, 64, 128, 16)
    assert st == 0 and plan.workspace_bytes > (4 << 20)
    t = torch.zeros(1024, dtype=torch.bfloat16, device=cuda_device)
    i = torch.zeros(16, dtype=torch.int32, device=cuda_device)
    vp = ctypes.c_void_p
    st = _lib.lib().pgqa_decode_noalloc(
        vp(t.data_ptr()), vp(t.data_ptr()), vp(t.data_ptr()), vp(t.data_ptr()),
        vp(i.data_ptr()), vp(i.data_ptr()), 12000, 512, 64, 128, 16, 1, 1, 0,
        ctypes.c_float(0.088), None)
    assert st == 11
    assert "4 MiB" in _lib.lib().pgqa_status_string(st).decode()
