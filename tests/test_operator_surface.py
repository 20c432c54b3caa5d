"""The flash_attn_with_kvcache-style entry point refuses, before touching a device,
every option this library does not implement (CPU only: no kernel is launched)."""
import pytest
import torch

import mx_flash_attn_kernel_opt__b200 as pgqa


def _args(B=2, Sq=1, Hq=32, Hkv=8, P=16, pages=4):
    q = torch.zeros(B, Sq, Hq, 128, dtype=torch.bfloat16)
    k = torch.zeros(pages, P, Hkv, 128, dtype=torch.bfloat16)
    v = torch.zeros_like(k)
    bt = torch.arange(pages, dtype=torch.int32).view(B, pages // B)
    lens = torch.tensor([5, 17], dtype=torch.int32)
    return q, k, v, bt, lens


@pytest.mark.parametrize("option,value", [
    ("rotary_cos", torch.zeros(4, 64)),
    ("cache_batch_idx", torch.zeros(2, dtype=torch.int32)),
    ("cache_leftpad", torch.zeros(2, dtype=torch.int32)),
    ("window_size", (64, 0)),
    ("softcap", 30.0),
    ("alibi_slopes", torch.zeros(32)),
])
def test_unimplemented_options_raise(option, value):
    q, k, v, bt, lens = _args()
    with pytest.raises(NotImplementedError, match="not implemented here"):
        pgqa.flash_attn_with_kvcache(q, k, v, cache_seqlens=lens, block_table=bt,
                                     **{option: value})


def test_non_paged_cache_and_bad_arguments_raise():
    q, k, v, bt, lens = _args()
    with pytest.raises(NotImplementedError, match="block_table=None"):
        pgqa.flash_attn_with_kvcache(q, k, v, cache_seqlens=lens)
    with pytest.raises(ValueError, match=r"\[B, Sq, Hq, D\]"):
        pgqa.flash_attn_with_kvcache(q[:, 0], k, v, cache_seqlens=lens, block_table=bt)
    with pytest.raises(ValueError, match="both k and v"):
        pgqa.flash_attn_with_kvcache(q, k, v, k=torch.zeros(2, 1, 8, 128, dtype=torch.bfloat16),
                                     cache_seqlens=lens, block_table=bt)
    with pytest.raises(ValueError, match="cache_seqlens is required"):
        pgqa.flash_attn_with_kvcache(q, k, v, block_table=bt)
