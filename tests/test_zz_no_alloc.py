"""The allocation-free entry point, pgqa_decode_noalloc, called through the C ABI.

Callers that cannot allocate device memory at call time (code inside a CUDA-graph
capture, engines that own all of HBM through their own pool, plugin hosts that only
pass the operator its inputs and outputs) use this entry point; its scratch is a fixed
array inside the library instead of a workspace from the caller.  These tests check
that two calls in a row give the same result as pgqa_decode_v1 with a caller workspace
(within the tolerance of the other parity tests), and that a shape needing more than
the fixed scratch is refused before anything runs.  The file is named so that pytest
collects it last.
"""
import ctypes

import pytest
import torch

import mx_flash_attn_kernel_opt__b200 as pgqa
from mx_flash_attn_kernel_opt__b200 import _lib, inputs, make_plan
from oracle import match_stats, paged_decode_ref

pytestmark = pytest.mark.gpu


def _noalloc(d, out, stream):
    vp = ctypes.c_void_p
    return _lib.lib().pgqa_decode_noalloc(
        vp(d.q.data_ptr()), vp(d.k.data_ptr()), vp(d.v.data_ptr()), vp(out.data_ptr()),
        vp(d.seq_lens.data_ptr()), vp(d.block_table.data_ptr()), d.batch, d.num_heads,
        d.num_heads_k, 128, d.page_size, d.num_pages, d.block_table.stride(0), 0,
        ctypes.c_float(d.scale), vp(stream.cuda_stream))


@pytest.mark.parametrize("case", ["c1", "spj07", "c3"])
def test_noalloc_matches_workspace_entry_point_on_two_calls(case, cuda_device):
    if case.startswith("spj"):
        inp = inputs.spj_case(int(case[3:]), table="permuted")
    else:
        inp = inputs.baseline_config(case)
    d = inp.to(cuda_device)
    # the existing entry point, with a caller-provided workspace
    ref_out = pgqa.decode(d.q, d.k, d.v, d.block_table, d.seq_lens, scale=inp.scale)
    torch.cuda.synchronize()
    stream = torch.cuda.current_stream(cuda_device)
    for call in range(2):
        out = torch.full_like(d.q, float("nan"))
        st = _noalloc(d, out, stream)
        assert st == 0, _lib.lib().pgqa_status_string(st).decode()
        torch.cuda.synchronize()
        a, b = out.float().cpu(), ref_out.float().cpu()
        assert torch.isfinite(a).all(), f"call {call}: non-finite output"
        frac, outlier, maxd = match_stats(a, b)
        assert not outlier and frac >= 0.99, (call, frac, maxd)
        assert torch.allclose(a, b, atol=1e-2, rtol=1e-2), (call, maxd)
    ref = paged_decode_ref(inp.q, inp.k, inp.v, inp.block_table, inp.seq_lens)
    assert torch.allclose(out.float().cpu(), ref, atol=1e-2, rtol=1e-2)


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
