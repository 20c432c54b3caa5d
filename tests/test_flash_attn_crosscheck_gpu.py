"""Cross-check against flash_attn_with_kvcache, the operator the reference's own harness
compares with (verify_real.py:40-41; task.md:16-26), where that library runs on this GPU.

The library is only a second checker here (it is called, never inspected).  Its paged
mode needs page sizes that are multiples of 256, so these cases use P = 256.  Skipped
when flash_attn is missing or has no kernel for this device.
"""
import pytest
import torch

import mx_flash_attn_kernel_opt__b200 as pgqa
from mx_flash_attn_kernel_opt__b200 import inputs
from tests.test_parity_gpu import ATOL, RTOL

pytestmark = pytest.mark.gpu

P = 256


def _fa():
    try:
        from flash_attn import flash_attn_with_kvcache
    except Exception as e:  # pragma: no cover - depends on the image
        pytest.skip(f"flash_attn unavailable: {e}")
    return flash_attn_with_kvcache


def _case(lens, S_new, Sq, Hq, Hkv, seed):
    inp = inputs.custom_case(len(lens), Hq, Hkv, P, [L + S_new for L in lens], seed=seed,
                             spare_pages=2)
    inp.seq_lens = torch.tensor(lens, dtype=torch.int32)
    g = torch.Generator().manual_seed(seed + 1)
    B = len(lens)
    q = torch.randn(B, Sq, Hq, 128, generator=g).to(torch.bfloat16)
    kn = torch.randn(B, S_new, Hkv, 128, generator=g).to(torch.bfloat16) if S_new else None
    vn = torch.randn(B, S_new, Hkv, 128, generator=g).to(torch.bfloat16) if S_new else None
    return inp, q, kn, vn


@pytest.mark.parametrize("Sq,S_new,causal", [(1, 0, 0), (4, 0, 1), (4, 0, 0), (4, 4, 1),
                                              (1, 1, 0), (8, 8, 1)])
@pytest.mark.parametrize("Hq,Hkv", [(32, 8), (28, 4), (64, 8)])
def test_matches_flash_attn_with_kvcache(Sq, S_new, causal, Hq, Hkv, cuda_device):
    fa = _fa()
    lens = [1, 7, 255, 256, 1000, 5000]
    inp, q, kn, vn = _case(lens, S_new, Sq, Hq, Hkv, seed=Sq * 5 + S_new + Hq)
    d = inp.to(cuda_device)
    qd = q.to(cuda_device)
    knd = kn.to(cuda_device) if kn is not None else None
    vnd = vn.to(cuda_device) if vn is not None else None
    k_fa, v_fa = d.k.clone(), d.v.clone()
    try:
        ref = fa(qd, k_fa, v_fa, k=knd, v=vnd, cache_seqlens=d.seq_lens,
                 block_table=d.block_table, softmax_scale=inp.scale, causal=bool(causal))
        torch.cuda.synchronize(cuda_device)
    except RuntimeError as e:  # no kernel image for this GPU, unsupported shape ...
        pytest.skip(f"flash_attn_with_kvcache did not run here: {e}")
    out = pgqa.decode(qd, d.k, d.v, d.block_table, d.seq_lens, scale=inp.scale,
                      causal=bool(causal), k_new=knd, v_new=vnd)
    torch.cuda.synchronize(cuda_device)
    assert torch.isfinite(out).all()
    assert torch.allclose(out.float(), ref.float(), atol=ATOL, rtol=RTOL), \
        f"max |diff| {(out.float() - ref.float()).abs().max().item()}"
    if S_new:
        assert torch.equal(d.k.view(torch.int16), k_fa.view(torch.int16))
        assert torch.equal(d.v.view(torch.int16), v_fa.view(torch.int16))


@pytest.mark.parametrize("Sq,S_new,causal", [(1, 0, False), (4, 4, True)])
def test_same_call_through_both_libraries(Sq, S_new, causal, cuda_device):
    """pgqa.flash_attn_with_kvcache takes flash-attn's own argument list: the same keyword
    arguments go to both libraries, each on its own copy of the cache."""
    fa = _fa()
    lens = [1, 300, 4000]
    inp, q, kn, vn = _case(lens, S_new, Sq, 32, 8, seed=71 + Sq)
    d = inp.to(cuda_device)
    kw = dict(cache_seqlens=d.seq_lens, block_table=d.block_table, softmax_scale=inp.scale,
              causal=causal, num_splits=0)
    if S_new:
        kw.update(k=kn.to(cuda_device), v=vn.to(cuda_device))
    qd = q.to(cuda_device)
    k_fa, v_fa = d.k.clone(), d.v.clone()
    try:
        ref = fa(qd, k_fa, v_fa, **kw)
        torch.cuda.synchronize(cuda_device)
    except RuntimeError as e:
        pytest.skip(f"flash_attn_with_kvcache did not run here: {e}")
    out = pgqa.flash_attn_with_kvcache(qd, d.k, d.v, **kw)
    torch.cuda.synchronize(cuda_device)
    if S_new == 0:  # the softmax_lse of the same call, from both libraries
        _, lse_fa = fa(qd, d.k.clone(), d.v.clone(), return_softmax_lse=True, **kw)
        _, lse = pgqa.flash_attn_with_kvcache(qd, d.k, d.v, return_softmax_lse=True, **kw)
        assert lse.shape == lse_fa.shape
        assert torch.allclose(lse, lse_fa.float(), atol=1e-3, rtol=1e-3), \
            f"lse max |diff| {(lse - lse_fa.float()).abs().max().item()}"
    assert out.shape == ref.shape
    assert torch.allclose(out.float(), ref.float(), atol=ATOL, rtol=RTOL), \
        f"max |diff| {(out.float() - ref.float()).abs().max().item()}"
    if S_new:
        assert torch.equal(d.k.view(torch.int16), k_fa.view(torch.int16))
        assert torch.equal(d.v.view(torch.int16), v_fa.view(torch.int16))
