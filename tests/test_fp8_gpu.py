"""GPU parity of the FP8 (e4m3) KV-page decode.

The oracle dequantises the same e4m3 bytes with the same per-KV-head factors and runs
the fp32 decode (paged_decode_fp8_ref), so the bar is the usual one: the reference's
rule and atol = rtol = 1e-2 against it, NaN-poisoned pools (the e4m3 NaN byte) in every
slot a correct kernel must not read.  The gap between an e4m3 pool and the bf16 pool it
was rounded from is the format's, not the kernel's, and is not measured here.
"""
import pytest
import torch

import mx_flash_attn_kernel_opt__b200 as pgqa
from mx_flash_attn_kernel_opt__b200 import inputs
from oracle import append_kv_ref, paged_decode_fp8_ref
from tests.test_parity_gpu import assert_parity

pytestmark = [pytest.mark.gpu, pytest.mark.usefixtures("both_kernels")]


def run_fp8(inp, dev, q=None, **kw):
    d = inp.to(dev)
    q = d.q if q is None else q.to(dev)
    out = pgqa.decode(q, d.k, d.v, d.block_table, d.seq_lens, scale=inp.scale,
                      k_scale=d.k_scale, v_scale=d.v_scale, **kw)
    torch.cuda.synchronize(dev)
    pgqa.check_device_error()
    return out


def ref_fp8(inp, q=None, **kw):
    return paged_decode_fp8_ref(inp.q if q is None else q, inp.k, inp.v, inp.k_scale,
                                inp.v_scale, inp.block_table, inp.seq_lens, scale=inp.scale,
                                **kw)


@pytest.mark.parametrize("P", [16, 32, 64, 128])
@pytest.mark.parametrize("Hq,Hkv", [(32, 8), (32, 4), (28, 4), (8, 8), (16, 1), (64, 8),
                                    (6, 2)])
def test_fp8_edge_lengths_poisoned(P, Hq, Hkv, cuda_device):
    lens = [1, 2, 15, 16, 17, P - 1, P, P + 1, 2 * P + 3, 100, 1000, 31, 33, 0]
    width = max((L + P - 1) // P for L in lens) + 2
    inp = inputs.to_fp8(inputs.custom_case(len(lens), Hq, Hkv, P, lens, seed=P * 7 + Hq,
                                           width=width, spare_pages=7))
    out = run_fp8(inputs.poison(inp), cuda_device)
    assert_parity(out, ref_fp8(inp), edge=True, what=f"fp8 P={P} Hq={Hq} Hkv={Hkv}")


@pytest.mark.parametrize("name", ["c1", "c3", "c4"])
def test_fp8_baseline_configs(name, cuda_device):
    inp = inputs.to_fp8(inputs.baseline_config(name))
    out = run_fp8(inp, cuda_device)
    assert_parity(out, ref_fp8(inp), what=f"fp8 {name}")


def test_fp8_c2_long_context(cuda_device):
    inp = inputs.to_fp8(inputs.baseline_config("c2"))
    out = run_fp8(inp, cuda_device)
    assert_parity(out, ref_fp8(inp), what="fp8 c2")


@pytest.mark.parametrize("q_mul", [3e4, 1e-5, 1.0])
def test_fp8_query_magnitudes(q_mul, cuda_device):
    """Rows far outside f16's range (or deep in its subnormals) are rescaled by an exact
    power of two before the f16 rounding."""
    lens = [700, 33, 4096]
    inp = inputs.to_fp8(inputs.custom_case(3, 32, 8, 16, lens, seed=11))
    q = (inp.q.float() * q_mul).to(torch.bfloat16)
    q[1, 5] *= 1e3  # one row much larger than the others
    out = run_fp8(inp, cuda_device, q=q)
    assert_parity(out, ref_fp8(inp, q=q), what=f"q x {q_mul}")


def test_fp8_distinct_head_scales_and_unit_scales(cuda_device):
    base = inputs.custom_case(4, 32, 8, 16, [300, 5, 2000, 77], seed=12)
    ks = torch.tensor([0.5, 0.01, 2.0, 0.003, 1.0, 0.25, 0.07, 4.0])
    vs = torch.tensor([0.02, 1.5, 0.3, 0.008, 1.0, 0.6, 0.09, 3.0])
    inp = inputs.to_fp8(base, k_scale=ks, v_scale=vs)
    assert_parity(run_fp8(inp, cuda_device), ref_fp8(inp), what="per-head scales")
    ones = inputs.to_fp8(base, k_scale=1.0 / 64, v_scale=1.0 / 64)
    d = ones.to(cuda_device)
    out = pgqa.decode(d.q, d.k, d.v, d.block_table, d.seq_lens, scale=ones.scale)  # no scales
    torch.cuda.synchronize(cuda_device)
    ref = paged_decode_fp8_ref(ones.q, ones.k, ones.v, 1.0, 1.0, ones.block_table,
                               ones.seq_lens, scale=ones.scale)
    assert_parity(out, ref, what="scales = 1")


@pytest.mark.parametrize("Sq,causal", [(2, 1), (4, 1), (4, 0), (8, 1)])
def test_fp8_multi_query(Sq, causal, cuda_device):
    lens = [1, 3, Sq, 17, 500, 0]
    inp = inputs.to_fp8(inputs.custom_case(len(lens), 32, 8, 16, lens, seed=Sq + 100,
                                           spare_pages=3))
    g = torch.Generator().manual_seed(Sq)
    q = torch.randn(len(lens), Sq, 32, 128, generator=g).to(torch.bfloat16)
    out = run_fp8(inputs.poison(inp), cuda_device, q=q, causal=bool(causal))
    assert_parity(out, ref_fp8(inp, q=q, causal=bool(causal)), edge=True,
                  what=f"fp8 Sq={Sq} causal={causal}")


def test_fp8_append_then_decode(cuda_device):
    lens, S_new, Hkv = [0, 5, 16, 250], 3, 8
    base = inputs.custom_case(4, 32, Hkv, 16, [L + S_new for L in lens], seed=21,
                              spare_pages=2)
    base.seq_lens = torch.tensor(lens, dtype=torch.int32)
    inp = inputs.poison(inputs.to_fp8(base))
    g = torch.Generator().manual_seed(22)
    kn = (torch.randn(4, S_new, Hkv, 128, generator=g) * 50).clamp(-448, 448).to(torch.float8_e4m3fn)
    vn = (torch.randn(4, S_new, Hkv, 128, generator=g) * 50).clamp(-448, 448).to(torch.float8_e4m3fn)
    ek, ev = append_kv_ref(inp.k.view(torch.uint8), inp.v.view(torch.uint8),
                           kn.view(torch.uint8), vn.view(torch.uint8), inp.seq_lens,
                           inp.block_table)
    ref = paged_decode_fp8_ref(inp.q, ek.view(torch.float8_e4m3fn), ev.view(torch.float8_e4m3fn),
                               inp.k_scale, inp.v_scale, inp.block_table, inp.seq_lens + S_new,
                               scale=inp.scale)
    d = inp.to(cuda_device)
    out = pgqa.decode(d.q, d.k, d.v, d.block_table, d.seq_lens, scale=inp.scale,
                      k_scale=d.k_scale, v_scale=d.v_scale, k_new=kn.to(cuda_device),
                      v_new=vn.to(cuda_device))
    torch.cuda.synchronize(cuda_device)
    pgqa.check_device_error()
    assert_parity(out, ref, edge=True, what="fp8 append")
    assert torch.equal(d.k.view(torch.uint8).cpu(), ek) and torch.equal(d.v.view(torch.uint8).cpu(), ev)
    # the append step alone
    d2 = inp.to(cuda_device)
    pgqa.append_kv(kn.to(cuda_device), vn.to(cuda_device), d2.k, d2.v, d2.block_table, d2.seq_lens)
    torch.cuda.synchronize(cuda_device)
    assert torch.equal(d2.k.view(torch.uint8).cpu(), ek) and torch.equal(d2.v.view(torch.uint8).cpu(), ev)


def test_fp8_repeated_calls_bit_identical(cuda_device):
    inp = inputs.to_fp8(inputs.baseline_config("c3")).to(cuda_device)
    outs = [pgqa.decode(inp.q, inp.k, inp.v, inp.block_table, inp.seq_lens, scale=inp.scale,
                        k_scale=inp.k_scale, v_scale=inp.v_scale) for _ in range(3)]
    torch.cuda.synchronize(cuda_device)
    assert torch.equal(outs[0], outs[1]) and torch.equal(outs[0], outs[2])
