"""GPU parity of the CUDA decode against the reference's golden vectors and the CPU oracle.

Acceptance, per case:
  * the reference's rule (verify_real.py:42-45): >= 99% of elements within
    1.6e-2 + 1.6e-2*|ref| (100% for its edge cases 1-3) and none beyond 8x that; and
  * every element within atol = rtol = 1e-2 of the fp32 oracle (torch.allclose);
  * block-table indexing bit-exact: pools poisoned with NaN in every slot a correct
    kernel must not read still give finite, matching outputs.
"""
import ctypes
import math
import os
import subprocess
import sys
import textwrap

import pytest
import torch

import mx_flash_attn_kernel_opt__b200 as pgqa
from mx_flash_attn_kernel_opt__b200 import _lib, inputs, ops
from oracle import match_stats, paged_decode_ref
from tests._golden import CASES, is_edge, load_rows, make_inputs

pytestmark = pytest.mark.gpu

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))

ATOL = RTOL = 1e-2


def assert_parity(out, ref, edge=False, what=""):
    out = out.float().cpu()
    ref = ref.float().cpu()
    assert torch.isfinite(out).all(), f"{what}: non-finite output"
    frac, outlier, maxd = match_stats(out, ref)
    assert not outlier, f"{what}: 8x-tolerance outlier (max |diff| {maxd})"
    assert frac >= (1.0 if edge else 0.99), f"{what}: match ratio {frac}"
    assert torch.allclose(out, ref, atol=ATOL, rtol=RTOL), f"{what}: max |diff| {maxd}"


def run_cabi(inp, dev):
    d = inp.to(dev)
    out = torch.zeros_like(d.q)
    B, Hq, D = d.q.shape
    pgqa.run_kernel_cabi(d.q, d.k, d.v, out, d.seq_lens, d.block_table, B, inp.seqlen_k, 1,
                         Hq, inp.num_heads_k, D, inp.page_size, inp.num_pages, 0)
    torch.cuda.synchronize(dev)
    pgqa.check_device_error()
    return out


def run_v1(inp, dev, **kw):
    d = inp.to(dev)
    out = pgqa.decode(d.q, d.k, d.v, d.block_table, d.seq_lens, scale=inp.scale, **kw)
    torch.cuda.synchronize(dev)
    return out


# ---- the reference's own outputs ----------------------------------------------------

@pytest.mark.parametrize("name", sorted(CASES))
def test_golden_case_through_reference_symbol(name, cuda_device):
    entry = CASES[name]
    inp = make_inputs(entry["spec"])
    assert inp.digest() == entry["digest"]
    out = run_cabi(inp, cuda_device)
    rows, gold = load_rows(name)
    assert_parity(out[rows], gold, edge=is_edge(name), what=f"{name} vs reference output")
    ref = paged_decode_ref(inp.q, inp.k, inp.v, inp.block_table, inp.seq_lens)
    assert_parity(out, ref, edge=is_edge(name), what=f"{name} vs oracle")


def test_python_operator_surface_matches_c_symbol(cuda_device):
    inp = inputs.spj_case(6, table="permuted")
    a = run_cabi(inp, cuda_device)
    d = inp.to(cuda_device)
    b = torch.zeros(d.batch, 1, d.num_heads, 128, dtype=torch.bfloat16, device=cuda_device)
    pgqa.run_kernel(d.q.view(d.batch, 1, d.num_heads, 128), d.k, d.v, b, d.seq_lens,
                    d.block_table, d.batch, inp.seqlen_k, 1, d.num_heads, d.num_heads_k, 128,
                    d.page_size, d.num_pages, 0)
    torch.cuda.synchronize()
    assert torch.equal(a, b.view_as(a))


# ---- the benchmark workloads ------------------------------------------------------

@pytest.mark.parametrize("name", ["c1", "c2", "c3", "c4"])
def test_baseline_config_vs_oracle(name, cuda_device):
    inp = inputs.baseline_config(name)
    out = run_v1(inp, cuda_device)
    ref = paged_decode_ref(inp.q, inp.k, inp.v, inp.block_table, inp.seq_lens)
    assert_parity(out, ref, what=name)


def test_c5_full_size_sampled_rows_and_page_permutation(cuda_device):
    """c5 at full size (~34 GB): 32 sequences spread over all 512 (every 16th, starting at
    a different offset in each half) against the oracle, and bit-identical output after
    moving every page to another physical slot (indexing is exact)."""
    dev = cuda_device
    inp = inputs.baseline_config("c5", device=dev)
    out = pgqa.decode(inp.q, inp.k, inp.v, inp.block_table, inp.seq_lens, scale=inp.scale)
    torch.cuda.synchronize()
    rows = list(range(0, 256, 16)) + list(range(263, 512, 16))
    assert len(rows) == 32 and rows[-1] == 503
    P = inp.page_size
    for b in rows:
        L = int(inp.seq_lens[b])
        ids = inp.block_table[b, :(L + P - 1) // P].to(torch.int64)
        sub = inputs.DecodeInputs(
            q=inp.q[b:b + 1].cpu(), k=inp.k.index_select(0, ids).cpu(),
            v=inp.v.index_select(0, ids).cpu(),
            block_table=torch.arange(len(ids), dtype=torch.int32).view(1, -1),
            seq_lens=inp.seq_lens[b:b + 1].cpu(), scale=inp.scale)
        ref = paged_decode_ref(sub.q, sub.k, sub.v, sub.block_table, sub.seq_lens)
        assert_parity(out[b:b + 1], ref, what=f"c5 row {b}")
    # permute physical pages: new_k[perm[i]] = k[i], table entries mapped through perm
    g = torch.Generator(device="cpu")
    g.manual_seed(11)
    perm = torch.randperm(inp.num_pages, generator=g).to(dev)
    k2 = torch.empty_like(inp.k)
    k2[perm] = inp.k
    del inp.k
    torch.cuda.empty_cache()
    v2 = torch.empty_like(inp.v)
    v2[perm] = inp.v
    del inp.v
    torch.cuda.empty_cache()
    bt2 = perm.to(torch.int32)[inp.block_table.to(torch.int64)]
    out2 = pgqa.decode(inp.q, k2, v2, bt2, inp.seq_lens, scale=inp.scale)
    torch.cuda.synchronize()
    assert torch.equal(out, out2)


# ---- edges: lengths, page sizes, group sizes, poisoned pools ------------------------

@pytest.mark.parametrize("P", [16, 32, 64, 128])
@pytest.mark.parametrize("Hq,Hkv", [(32, 8), (32, 4), (28, 4), (8, 8), (16, 1), (64, 2),
                                    (24, 3), (6, 2), (64, 1)])
def test_edge_lengths_poisoned(P, Hq, Hkv, cuda_device):
    lens = [1, 2, 15, 16, 17, P - 1, P, P + 1, 2 * P + 3, 100, 1000, 31, 33]
    width = max((L + P - 1) // P for L in lens) + 2
    inp = inputs.custom_case(len(lens), Hq, Hkv, P, lens, seed=P * 100 + Hq, width=width,
                             spare_pages=7)
    ref = paged_decode_ref(inp.q, inp.k, inp.v, inp.block_table, inp.seq_lens)
    out = run_v1(inputs.poison(inp), cuda_device)
    assert_parity(out, ref, edge=True, what=f"P={P} Hq={Hq} Hkv={Hkv}")


def test_zero_length_sequences_give_zeros(cuda_device):
    inp = inputs.custom_case(4, 32, 8, 16, [0, 40, 0, 3], seed=9, width=4)
    out = run_v1(inp, cuda_device)
    ref = paged_decode_ref(inp.q, inp.k, inp.v, inp.block_table, inp.seq_lens)
    assert torch.count_nonzero(out[0]) == 0 and torch.count_nonzero(out[2]) == 0
    assert_parity(out, ref, edge=True, what="zero lengths")


@pytest.mark.parametrize("lens", [[1], [16], [5000], [1] * 300, [2048, 1, 1, 7, 65536]])
def test_extreme_batches(lens, cuda_device):
    inp = inputs.custom_case(len(lens), 32, 4, 16, lens, seed=len(lens))
    out = run_v1(inp, cuda_device)
    ref = paged_decode_ref(inp.q, inp.k, inp.v, inp.block_table, inp.seq_lens)
    assert_parity(out, ref, what=f"lens={lens[:5]}")


def test_repeated_calls_are_bit_identical(cuda_device):
    """The fused combine's arrival counters must be left at zero by every call."""
    inp = inputs.baseline_config("c3").to(cuda_device)
    outs = [pgqa.decode(inp.q, inp.k, inp.v, inp.block_table, inp.seq_lens, scale=inp.scale)
            for _ in range(3)]
    torch.cuda.synchronize()
    assert torch.equal(outs[0], outs[1]) and torch.equal(outs[1], outs[2])


def test_caller_workspace_on_side_stream(cuda_device):
    inp = inputs.spj_case(11, table="permuted")
    d = inp.to(cuda_device)
    L = _lib.lib()
    need = L.pgqa_workspace_size(d.batch, d.num_heads, d.num_heads_k, 128, d.page_size)
    ws = torch.empty(need, dtype=torch.uint8, device=cuda_device)
    side = torch.cuda.Stream(cuda_device)
    with torch.cuda.stream(side):
        assert L.pgqa_workspace_init(ops._ptr(ws), need, ops._stream_handle(cuda_device)) == 0
        out = pgqa.decode(d.q, d.k, d.v, d.block_table, d.seq_lens, scale=inp.scale,
                          workspace=ws)
    side.synchronize()
    pgqa.check_device_error(ws)
    ref = paged_decode_ref(inp.q, inp.k, inp.v, inp.block_table, inp.seq_lens)
    assert_parity(out, ref, what="side stream")
    # a workspace that is too small is rejected before any launch
    with pytest.raises(pgqa.PgqaError):
        pgqa.decode(d.q, d.k, d.v, d.block_table, d.seq_lens, workspace=ws[:need // 2])


@pytest.mark.parametrize("skew", [16, -16, 1 << 20])
def test_speculative_prefix_is_rebuilt_when_lengths_change(skew, cuda_device, monkeypatch):
    """The pass before griddepcontrol.wait builds the prefix table from a first read of
    the lengths; PGQA_DEBUG_SPEC_SKEW makes that read disagree with the lengths the call
    really has (as when a predecessor rewrites them), so the table must be rebuilt after
    the wait and the output must not change."""
    inp = inputs.custom_case(6, 32, 4, 16, [1, 17, 300, 2048, 33, 4000], seed=41)
    d = inp.to(cuda_device)
    ref = paged_decode_ref(inp.q, inp.k, inp.v, inp.block_table, inp.seq_lens)
    plain = pgqa.decode(d.q, d.k, d.v, d.block_table, d.seq_lens, scale=inp.scale)
    monkeypatch.setenv("PGQA_DEBUG_SPEC_SKEW", str(skew))
    ws = _fresh_ws(inp, cuda_device)
    out = pgqa.decode(d.q, d.k, d.v, d.block_table, d.seq_lens, scale=inp.scale, workspace=ws)
    pgqa.check_device_error(ws)
    assert_parity(out, ref, what=f"skew {skew}")
    assert torch.equal(out, plain)


@pytest.mark.parametrize("kind", ["fp8", "multi_token_append"])
def test_speculative_pass_on_other_instantiations(kind, cuda_device, monkeypatch):
    """The same forced pass (PGQA_DEBUG_SPEC_SKEW) on e4m3 pages (two prefetch boxes a
    chunk) and on a causal two-token decode that appends its new tokens first (the pass
    reads lengths plus the appended count while the append may still be running)."""
    from oracle import append_kv_ref, paged_decode_fp8_ref
    lens = [1, 17, 300, 2048, 33]
    if kind == "fp8":
        f8 = inputs.to_fp8(inputs.custom_case(5, 32, 4, 16, lens, seed=43))
        d = f8.to(cuda_device)
        ref = paged_decode_fp8_ref(f8.q, f8.k, f8.v, f8.k_scale, f8.v_scale, f8.block_table,
                                   f8.seq_lens)
        call = lambda ws=None: pgqa.decode(d.q, d.k, d.v, d.block_table, d.seq_lens,
                                           k_scale=d.k_scale, v_scale=d.v_scale, workspace=ws)
    else:
        base = inputs.custom_case(5, 32, 4, 16, [L + 2 for L in lens], seed=44)
        base.seq_lens = torch.tensor(lens, dtype=torch.int32)
        g = torch.Generator().manual_seed(45)
        q2 = torch.randn(5, 2, 32, 128, generator=g).to(torch.bfloat16)
        kn = torch.randn(5, 2, 4, 128, generator=g).to(torch.bfloat16)
        vn = torch.randn(5, 2, 4, 128, generator=g).to(torch.bfloat16)
        ek, ev = append_kv_ref(base.k, base.v, kn, vn, base.seq_lens, base.block_table)
        ref = paged_decode_ref(q2, ek, ev, base.block_table, base.seq_lens + 2, causal=True)

        def call(ws=None):
            d = base.to(cuda_device)  # a fresh pool: the call appends into it
            return pgqa.decode(q2.to(cuda_device), d.k, d.v, d.block_table, d.seq_lens,
                               causal=True, k_new=kn.to(cuda_device), v_new=vn.to(cuda_device),
                               workspace=ws)
    plain = call()
    monkeypatch.setenv("PGQA_DEBUG_SPEC_SKEW", "16")
    ws = ops.workspace_for(5, 32, 4, 128, 16, cuda_device, seqlen_q=1 if kind == "fp8" else 2)
    out = call(ws)
    pgqa.check_device_error(ws)
    assert_parity(out, ref, what=f"{kind} with the forced pass")
    assert torch.equal(out, plain)


def test_custom_scale(cuda_device):
    inp = inputs.custom_case(3, 16, 2, 16, [7, 70, 700], seed=21)
    d = inp.to(cuda_device)
    out = pgqa.decode(d.q, d.k, d.v, d.block_table, d.seq_lens, scale=0.03)
    ref = paged_decode_ref(inp.q, inp.k, inp.v, inp.block_table, inp.seq_lens, scale=0.03)
    assert_parity(out, ref, what="scale 0.03")


# ---- device error word --------------------------------------------------------------

def _fresh_ws(inp, dev):
    L = _lib.lib()
    need = L.pgqa_workspace_size(inp.batch, inp.num_heads, inp.num_heads_k, 128, inp.page_size)
    return torch.zeros(need, dtype=torch.uint8, device=dev)


def test_bad_page_id_is_reported(cuda_device):
    inp = inputs.custom_case(2, 32, 8, 16, [40, 20], seed=5, width=3)
    bt = inp.block_table.clone()
    bt[0, 1] = inp.num_pages + 5
    d = inputs.DecodeInputs(q=inp.q, k=inp.k, v=inp.v, block_table=bt, seq_lens=inp.seq_lens,
                            scale=inp.scale).to(cuda_device)
    ws = _fresh_ws(inp, cuda_device)
    pgqa.decode(d.q, d.k, d.v, d.block_table, d.seq_lens, workspace=ws)
    with pytest.raises(pgqa.PgqaError) as e:
        pgqa.check_device_error(ws)
    assert e.value.status == 9
    pgqa.check_device_error(ws)  # cleared


def test_seq_len_above_capacity_is_reported(cuda_device):
    inp = inputs.custom_case(2, 32, 8, 16, [40, 20], seed=6, width=3)
    d = inp.to(cuda_device)
    d.seq_lens[1] = 10 ** 6
    ws = _fresh_ws(inp, cuda_device)
    pgqa.decode(d.q, d.k, d.v, d.block_table, d.seq_lens, workspace=ws)
    with pytest.raises(pgqa.PgqaError) as e:
        pgqa.check_device_error(ws)
    assert e.value.status == 10


def test_expired_wait_reports_timeout_and_context_survives(cuda_device, monkeypatch):
    """One stage barrier waits for 16 bytes nothing sends: its bounded wait expires, the
    kernel records PGQA_ERR_DEVICE_TIMEOUT and returns; the context stays usable and the
    workspace is left ready for the next call (no manual reset)."""
    inp = inputs.custom_case(2, 32, 8, 16, [300, 200], seed=8)
    d = inp.to(cuda_device)
    ws = _fresh_ws(inp, cuda_device)
    monkeypatch.setenv("PGQA_DEBUG_STUCK_BARRIER", "1")
    monkeypatch.setenv("PGQA_WAIT_LIMIT_NS", "20000000")
    pgqa.decode(d.q, d.k, d.v, d.block_table, d.seq_lens, workspace=ws)
    with pytest.raises(pgqa.PgqaError) as e:
        pgqa.check_device_error(ws)
    assert e.value.status == 8
    monkeypatch.delenv("PGQA_DEBUG_STUCK_BARRIER")
    monkeypatch.delenv("PGQA_WAIT_LIMIT_NS")
    out = pgqa.decode(d.q, d.k, d.v, d.block_table, d.seq_lens, workspace=ws)
    pgqa.check_device_error(ws)
    ref = paged_decode_ref(inp.q, inp.k, inp.v, inp.block_table, inp.seq_lens)
    assert_parity(out, ref, what="after timeout")


def _slice_begin(i, n, total):
    return i * total // n


def _sole_holder_case():
    """B=1, Hq=32, Hkv=8, L=240: 8 units of 15 chunks, 120 chunks over 7 CTAs of 8 warps
    (2 chunks per warp at least).  CTA 0 owns chunks [0, 17); its warp 7 owns [14, 17),
    the last chunk of unit 0 and the first two of unit 1, which continues in CTA 1.  So
    warp 7 is the only holder of unit 1 in CTA 0: if it stops, CTA 0 must still arrive
    on unit 1's counters, or the next call would merge unit 1 one CTA early."""
    inp = inputs.custom_case(1, 32, 8, 16, [240], seed=31)
    T, n_cta, W = 15 * 8, 120 // 16, 8
    cta0_end = _slice_begin(1, n_cta, T)
    w7 = (_slice_begin(7, W, cta0_end), _slice_begin(8, W, cta0_end))
    assert (n_cta, cta0_end, w7) == (7, 17, (14, 17))
    return inp


@pytest.mark.parametrize("path", ["caller_workspace", "run_kernel"])
def test_expired_wait_in_the_only_holder_of_a_cut_unit_leaves_counters_clean(
        path, cuda_device, monkeypatch):
    """The stalled warp parks a zero-weight state for each unit its slice cuts, so every
    arrival counter completes and is reset by its last arriver; the next call on the same
    workspace (the caller's, or run_kernel's library workspace, which the caller cannot
    reset) is correct without any manual reset."""
    inp = _sole_holder_case()
    d = inp.to(cuda_device)
    ws = _fresh_ws(inp, cuda_device) if path == "caller_workspace" else None

    def call():
        if ws is not None:
            return pgqa.decode(d.q, d.k, d.v, d.block_table, d.seq_lens, workspace=ws)
        out = torch.zeros_like(d.q)
        B, Hq, D = d.q.shape
        L = _lib.lib()
        with torch.cuda.device(cuda_device):
            L.run_kernel(ctypes.c_void_p(d.q.data_ptr()), ctypes.c_void_p(d.k.data_ptr()),
                         ctypes.c_void_p(d.v.data_ptr()), ctypes.c_void_p(out.data_ptr()),
                         ctypes.c_void_p(d.seq_lens.data_ptr()),
                         ctypes.c_void_p(d.block_table.data_ptr()), B, inp.seqlen_k, 1, Hq,
                         inp.num_heads_k, D, inp.page_size, inp.num_pages, 0)
        assert L.pgqa_last_status() == 0
        return out

    if ws is None:
        call()  # the library workspace exists (allocated, zeroed) before the failing call
        torch.cuda.synchronize()
        pgqa.check_device_error()
    monkeypatch.setenv("PGQA_DEBUG_STUCK_BARRIER", "8")  # warp 7 of CTA 0
    monkeypatch.setenv("PGQA_WAIT_LIMIT_NS", "20000000")
    call()
    with pytest.raises(pgqa.PgqaError) as e:
        pgqa.check_device_error(ws)
    assert e.value.status == 8
    monkeypatch.delenv("PGQA_DEBUG_STUCK_BARRIER")
    monkeypatch.delenv("PGQA_WAIT_LIMIT_NS")
    ref = paged_decode_ref(inp.q, inp.k, inp.v, inp.block_table, inp.seq_lens)
    for k in range(2):
        out = call()
        torch.cuda.synchronize()
        pgqa.check_device_error(ws)
        assert_parity(out, ref, what=f"call {k} after timeout ({path})")


def test_library_workspace_allocation_failure_is_reported(cuda_device):
    """The reference symbol runs on a library-owned workspace, allocated on first use.
    When that allocation fails (forced by PGQA_DEBUG_FAIL_WORKSPACE_ALLOC in a fresh
    process, where nothing is allocated yet) the call reports PGQA_ERR_WORKSPACE and
    leaves the output untouched; once the allocation succeeds the next call runs."""
    code = textwrap.dedent("""
        import os, sys, torch
        sys.path.insert(0, %r)
        import mx_flash_attn_kernel_opt__b200 as pgqa
        from mx_flash_attn_kernel_opt__b200 import inputs
        inp = inputs.spj_case(5, table="permuted")
        d = inp.to("cuda")
        out = torch.full_like(d.q, 7.0)
        B, Hq, D = d.q.shape
        args = (d.q, d.k, d.v, out, d.seq_lens, d.block_table, B, inp.seqlen_k, 1, Hq,
                inp.num_heads_k, D, inp.page_size, inp.num_pages, 0)
        try:
            pgqa.run_kernel_cabi(*args)
            print("status 0")
        except pgqa.PgqaError as e:
            print("status", e.status)
        torch.cuda.synchronize()
        print("untouched", bool((out == 7.0).all()))
        del os.environ["PGQA_DEBUG_FAIL_WORKSPACE_ALLOC"]
        pgqa.run_kernel_cabi(*args)
        torch.cuda.synchronize()
        pgqa.check_device_error()
        print("ran", bool(torch.isfinite(out.float()).all()) and bool((out != 7.0).any()))
    """ % REPO)
    env = dict(os.environ, PGQA_DEBUG_FAIL_WORKSPACE_ALLOC="1")  # same visible devices
    r = subprocess.run([sys.executable, "-c", code], env=env, capture_output=True, text=True,
                       timeout=600)
    assert r.returncode == 0, r.stderr[-2000:]
    lines = r.stdout.split("\n")
    assert "status 5" in lines and "untouched True" in lines and "ran True" in lines, r.stdout


def test_undersized_or_misaligned_workspace_is_refused(cuda_device):
    """A caller workspace below pgqa_workspace_size, or not 256-byte aligned, is refused
    before anything is launched (the output is left untouched)."""
    inp = inputs.baseline_config("c1").to(cuda_device)
    out = torch.full_like(inp.q, 7.0)
    small = torch.zeros(1024, dtype=torch.uint8, device=cuda_device)
    with pytest.raises(pgqa.PgqaError) as e:
        pgqa.decode(inp.q, inp.k, inp.v, inp.block_table, inp.seq_lens, out=out, workspace=small)
    assert e.value.status == 5
    need = _lib.lib().pgqa_workspace_size(inp.batch, inp.num_heads, inp.num_heads_k, 128,
                                          inp.page_size)
    big = torch.zeros(need + 512, dtype=torch.uint8, device=cuda_device)
    with pytest.raises(pgqa.PgqaError) as e:
        pgqa.decode(inp.q, inp.k, inp.v, inp.block_table, inp.seq_lens, out=out,
                    workspace=big[16:])
    assert e.value.status == 4
    torch.cuda.synchronize(cuda_device)
    assert bool((out == 7.0).all())


def test_large_batch_prefix_table(cuda_device):
    """B = 8000 short sequences: every CTA scans a long length table (31 per thread)."""
    g = torch.Generator().manual_seed(77)
    lens = torch.randint(1, 40, (8000,), generator=g).tolist()
    inp = inputs.custom_case(len(lens), 8, 2, 16, lens, seed=78)
    out = run_v1(inp, cuda_device)
    rows = list(range(0, 8000, 97))
    ref = paged_decode_ref(inp.q, inp.k, inp.v, inp.block_table, inp.seq_lens, rows=rows)
    assert_parity(out[rows], ref[rows], what="B=8000")
    f8 = inputs.to_fp8(inp)
    d8 = f8.to(cuda_device)
    out8 = pgqa.decode(d8.q, d8.k, d8.v, d8.block_table, d8.seq_lens, k_scale=d8.k_scale,
                       v_scale=d8.v_scale)
    torch.cuda.synchronize(cuda_device)
    from oracle import paged_decode_fp8_ref
    kd = f8.k.float() * f8.k_scale.view(1, 1, -1, 1)
    vd = f8.v.float() * f8.v_scale.view(1, 1, -1, 1)
    ref8 = paged_decode_ref(f8.q, kd, vd, f8.block_table, f8.seq_lens, rows=rows)
    assert_parity(out8[rows], ref8[rows], what="B=8000 fp8")


def test_batch_beyond_prefix_table_is_refused(cuda_device):
    inp = inputs.custom_case(40000, 8, 2, 16, [1] * 40000, seed=79).to(cuda_device)
    with pytest.raises(pgqa.PgqaError) as e:
        pgqa.decode(inp.q, inp.k, inp.v, inp.block_table, inp.seq_lens)
    assert e.value.status == 3


def test_python_surface_rejects_mismatched_output(cuda_device):
    """The operator refuses an output whose shape differs from q's (it would write past
    it) before anything is launched."""
    inp = inputs.baseline_config("c1").to(cuda_device)
    q4 = inp.q.unsqueeze(1).expand(-1, 2, -1, -1).contiguous()  # two query tokens
    small = torch.zeros_like(inp.q)                                 # one token's worth
    with pytest.raises(pgqa.PgqaError) as e:
        pgqa.decode(q4, inp.k, inp.v, inp.block_table, inp.seq_lens, out=small)
    assert e.value.status == 2
    with pytest.raises(ValueError):
        pgqa.decode(inp.q, inp.k, inp.v, inp.block_table, inp.seq_lens.cpu())
