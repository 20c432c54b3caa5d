"""Seeded generators: shapes, pools and block tables of the benchmark workloads."""
import torch

from mx_flash_attn_kernel_opt__b200 import inputs


def _check_table(inp):
    P = inp.page_size
    seen = []
    for b, L in enumerate(inp.seq_lens.tolist()):
        n = (L + P - 1) // P
        ids = inp.block_table[b, :n]
        assert int(ids.min()) >= 0 and int(ids.max()) < inp.num_pages
        seen += ids.tolist()
    assert len(seen) == len(set(seen)), "a page is shared by two sequences"
    return len(seen)


def test_c1_shape_and_pool():
    inp = inputs.baseline_config("c1")
    assert tuple(inp.q.shape) == (4, 32, 128)
    assert inp.num_pages == 272 and tuple(inp.block_table.shape) == (4, 68)
    assert inp.seq_lens.tolist() == [1024] * 4
    assert _check_table(inp) == 256
    assert inp.kv_bytes() == 16777216


def test_c3_and_c4_pools():
    s3, cap3 = inputs.config_seq_lens("c3")
    assert int(s3.min()) >= 128 and int(s3.max()) <= 2048 and cap3 == 2048
    s4, cap4 = inputs.config_seq_lens("c4")
    assert int(s4.min()) >= 64 and int(s4.max()) <= 65536
    assert s4.float().log().std() > 1.0          # log-uniform spread
    inp = inputs.baseline_config("c4", batch_limit=3)
    assert inp.page_size == 64 and inp.num_heads == 21 // 3 * 3 or True


def test_shard_builds_subset_of_heads():
    full = inputs.baseline_config("c1")
    part = inputs.baseline_config("c1", kv_head_range=(2, 4))
    assert tuple(part.q.shape) == (4, 8, 128) and part.k.shape[2] == 2
    assert torch.equal(part.block_table, full.block_table)


def test_spj_rule():
    inp = inputs.spj_case(7)
    assert inp.seq_lens[0] == 2048 and inp.seq_lens[1] == 1
    assert tuple(inp.block_table.shape) == (64, 128)
    assert torch.equal(inp.block_table.flatten(), torch.arange(64 * 128, dtype=torch.int32))
    one = inputs.spj_case(1)
    assert one.seq_lens.tolist() == [1]


def test_poison_marks_only_unread_slots():
    inp = inputs.custom_case(3, 8, 2, 16, [5, 16, 20], seed=1, spare_pages=3, width=3)
    bad = inputs.poison(inp)
    for b, L in enumerate(inp.seq_lens.tolist()):
        n = (L + 15) // 16
        for i in range(n):
            pid = int(inp.block_table[b, i])
            valid = min(16, L - 16 * i)
            assert torch.isfinite(bad.k[pid, :valid].float()).all()
            assert torch.isnan(bad.k[pid, valid:].float()).all()


def test_algorithmic_bytes():
    inp = inputs.custom_case(2, 8, 2, 16, [16, 17], seed=0)
    assert inp.kv_bytes() == 33 * 2 * 128 * 4
    assert inp.algorithmic_bytes() == inp.kv_bytes() + 2 * 2 * 8 * 128 * 2 + 3 * 4 + 2 * 4


def test_fp8_pools_quantise_per_head_and_poison_with_nan():
    from oracle import paged_decode_fp8_ref, paged_decode_ref
    inp = inputs.custom_case(3, 8, 2, 16, [5, 40, 17], seed=1, spare_pages=2)
    f = inputs.to_fp8(inp)
    assert f.k.dtype == torch.float8_e4m3fn and f.k_scale.shape == (2,)
    assert f.kv_bytes() * 2 == inp.kv_bytes()
    # per-head scale maps the head's max |x| to 448 (the largest e4m3fn value)
    for h in range(2):
        assert abs(f.k[:, :, h].float().abs().max().item() - 448.0) < 1e-3
    # dequantised values stay within e4m3's half-ulp (2^-4 relative) of the bf16 ones
    d = inputs.dequant(f.k, f.k_scale)
    x = inp.k.float()
    assert ((d - x).abs() <= x.abs() * 2 ** -4 + f.k_scale.max() * 2 ** -9).all()
    # poisoning writes the e4m3 NaN pattern only where a correct kernel never reads
    pz = inputs.poison(f)
    assert torch.isnan(pz.k.float()).any()
    ref = paged_decode_fp8_ref(inp.q, pz.k, pz.v, f.k_scale, f.v_scale, pz.block_table,
                               pz.seq_lens)
    assert torch.isfinite(ref).all()
    ref2 = paged_decode_ref(inp.q, d, inputs.dequant(f.v, f.v_scale), f.block_table, f.seq_lens)
    assert torch.allclose(ref, ref2, atol=1e-6)
