"""The log-sum-exp output (pgqa_decode_ex's softmax_lse; decode(return_lse=True)) against
the oracle's, on every path a row's result can take: a unit finished inside one warp, a
unit merged across the warps of one CTA, and a unit merged across CTAs -- for one and
several query tokens (rows that see no key give -inf), e4m3 pages and appended tokens.
The output itself must be the same as without the LSE."""
import pytest
import torch

import mx_flash_attn_kernel_opt__b200 as pgqa
from mx_flash_attn_kernel_opt__b200 import inputs
from oracle import append_kv_ref, paged_decode_fp8_ref, paged_decode_ref
from tests.test_parity_gpu import assert_parity

pytestmark = [pytest.mark.gpu, pytest.mark.usefixtures("both_kernels")]

# fp32 log-sum-exp: the kernel uses ex2.approx / lg2.approx on the same bf16 inputs
LSE_ATOL = LSE_RTOL = 1e-3


def assert_lse(lse, ref, what):
    lse, ref = lse.float().cpu(), ref.float().cpu()
    assert lse.shape == ref.shape, f"{what}: shape {tuple(lse.shape)} vs {tuple(ref.shape)}"
    empty = torch.isneginf(ref)
    assert torch.equal(torch.isneginf(lse), empty), f"{what}: -inf rows differ"
    assert torch.isfinite(lse[~empty]).all(), f"{what}: non-finite lse"
    diff = (lse[~empty] - ref[~empty]).abs().max().item() if (~empty).any() else 0.0
    assert torch.allclose(lse[~empty], ref[~empty], atol=LSE_ATOL, rtol=LSE_RTOL), \
        f"{what}: max |diff| {diff}"


BF16_CASES = {
    "one_unit_split_over_warps": (1, 8, 1, 16, [40]),
    "tiny_units": (2, 32, 8, 16, [16, 3]),
    "spj5_permuted": None,
    "c1_split_over_ctas": None,
    "ragged_g7_P64": (5, 28, 4, 64, [1, 129, 2000, 64, 7000]),
}


@pytest.mark.parametrize("name", sorted(BF16_CASES))
def test_lse_single_token(name, cuda_device):
    if name == "spj5_permuted":
        inp = inputs.spj_case(5, table="permuted")
    elif name == "c1_split_over_ctas":
        inp = inputs.baseline_config("c1")
    else:
        B, Hq, Hkv, P, lens = BF16_CASES[name]
        inp = inputs.custom_case(B, Hq, Hkv, P, lens, seed=B * 7 + P)
    d = inp.to(cuda_device)
    ref, ref_lse = paged_decode_ref(inp.q, inp.k, inp.v, inp.block_table, inp.seq_lens,
                                    return_lse=True)
    plain = pgqa.decode(d.q, d.k, d.v, d.block_table, d.seq_lens, scale=inp.scale)
    out, lse = pgqa.decode(d.q, d.k, d.v, d.block_table, d.seq_lens, scale=inp.scale,
                           return_lse=True)
    torch.cuda.synchronize()
    assert_parity(out, ref, what=name)
    assert_lse(lse, ref_lse, name)
    assert torch.equal(out, plain)


@pytest.mark.parametrize("Sq,lens", [(4, [2, 40, 1000]), (3, [1, 3, 17]), (8, [5, 300])])
def test_lse_several_query_tokens(Sq, lens, cuda_device):
    B = len(lens)
    inp = inputs.custom_case(B, 32, 8, 16, lens, seed=Sq + B)
    g = torch.Generator().manual_seed(Sq)
    q = torch.randn(B, Sq, 32, 128, generator=g).to(torch.bfloat16)
    ref, ref_lse = paged_decode_ref(q, inp.k, inp.v, inp.block_table, inp.seq_lens,
                                    causal=True, return_lse=True)
    d = inp.to(cuda_device)
    out, lse = pgqa.decode(q.to(cuda_device), d.k, d.v, d.block_table, d.seq_lens,
                           causal=True, return_lse=True)
    torch.cuda.synchronize()
    assert_parity(out, ref, edge=True, what=f"Sq={Sq}")
    assert_lse(lse, ref_lse, f"Sq={Sq}")


@pytest.mark.parametrize("Sq", [1, 3])
def test_lse_fp8_pages(Sq, cuda_device):
    """e4m3 pages, one token (one row group per unit) and three causal tokens (two row
    groups per unit, the second partly padding; rows that see no key)."""
    f8 = inputs.to_fp8(inputs.custom_case(4, 32, 4, 16, [1, 300, 2048, 33], seed=61))
    d = f8.to(cuda_device)
    q = f8.q
    if Sq > 1:
        g = torch.Generator().manual_seed(64)
        q = torch.randn(4, Sq, 32, 128, generator=g).to(torch.bfloat16)
    ref, ref_lse = paged_decode_fp8_ref(q, f8.k, f8.v, f8.k_scale, f8.v_scale,
                                        f8.block_table, f8.seq_lens, causal=Sq > 1,
                                        return_lse=True)
    out, lse = pgqa.decode(q.to(cuda_device), d.k, d.v, d.block_table, d.seq_lens,
                           k_scale=d.k_scale, v_scale=d.v_scale, causal=Sq > 1,
                           return_lse=True)
    torch.cuda.synchronize()
    assert_parity(out, ref, edge=Sq > 1, what=f"fp8 Sq={Sq}")
    assert_lse(lse, ref_lse, f"fp8 Sq={Sq}")


def test_lse_with_appended_tokens(cuda_device):
    lens = [3, 40, 1500]
    base = inputs.custom_case(3, 16, 4, 16, [L + 2 for L in lens], seed=62)
    base.seq_lens = torch.tensor(lens, dtype=torch.int32)
    g = torch.Generator().manual_seed(63)
    q2 = torch.randn(3, 2, 16, 128, generator=g).to(torch.bfloat16)
    kn = torch.randn(3, 2, 4, 128, generator=g).to(torch.bfloat16)
    vn = torch.randn(3, 2, 4, 128, generator=g).to(torch.bfloat16)
    ek, ev = append_kv_ref(base.k, base.v, kn, vn, base.seq_lens, base.block_table)
    ref, ref_lse = paged_decode_ref(q2, ek, ev, base.block_table, base.seq_lens + 2,
                                    causal=True, return_lse=True)
    d = base.to(cuda_device)
    out, lse = pgqa.decode(q2.to(cuda_device), d.k, d.v, d.block_table, d.seq_lens,
                           causal=True, k_new=kn.to(cuda_device), v_new=vn.to(cuda_device),
                           return_lse=True)
    torch.cuda.synchronize()
    assert_parity(out, ref, what="append")
    assert_lse(lse, ref_lse, "append")


@pytest.mark.parametrize("Sq", [1, 3])
def test_lse_zero_length_sequences(Sq, cuda_device):
    """Sequences with no keys give zeros and a log-sum-exp of -inf in every row.  Both
    buffers hold NaN when the kernel starts (out is passed in; the LSE buffer is a
    NaN-filled block of the same size handed back by the caching allocator), so an entry
    the kernel skipped would show."""
    lens = [0, 300, 0, 17]
    inp = inputs.custom_case(4, 32, 8, 16, lens, seed=71 + Sq)
    q = inp.q
    if Sq > 1:
        g = torch.Generator().manual_seed(72)
        q = torch.randn(4, Sq, 32, 128, generator=g).to(torch.bfloat16)
    ref, ref_lse = paged_decode_ref(q, inp.k, inp.v, inp.block_table, inp.seq_lens,
                                    causal=Sq > 1, return_lse=True)
    d = inp.to(cuda_device)
    qd = q.to(cuda_device)
    # a first call creates the cached workspace, so that the loop's only allocation
    # between freeing the poison and the kernel is the LSE buffer
    pgqa.decode(qd, d.k, d.v, d.block_table, d.seq_lens, causal=Sq > 1, return_lse=True)
    for _ in range(2):
        out = torch.full_like(qd, float("nan"))
        poison = torch.full((4, 32, Sq), float("nan"), device=cuda_device)
        poison_ptr = poison.data_ptr()
        del poison
        out, lse = pgqa.decode(qd, d.k, d.v, d.block_table, d.seq_lens, out=out,
                               causal=Sq > 1, return_lse=True)
        torch.cuda.synchronize()
        assert lse.data_ptr() == poison_ptr, "the LSE buffer was not the poisoned block"
        assert_parity(out, ref, edge=Sq > 1, what=f"empty Sq={Sq}")
        assert_lse(lse, ref_lse, f"empty Sq={Sq}")
        assert torch.isneginf(lse[0]).all() and torch.isneginf(lse[2]).all()
        assert (out[0] == 0).all() and (out[2] == 0).all()
