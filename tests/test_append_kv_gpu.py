"""GPU parity of the append-KV step and of decode with appended tokens.

The append is index and byte work: the pools after the GPU append must equal the
oracle's bit for bit (compared as raw 16-bit patterns, so NaN poison counts too).  The
decode over the extended sequences must meet the usual parity bar against the oracle
decode of the oracle-appended pools.
"""
import pytest
import torch

import mx_flash_attn_kernel_opt__b200 as pgqa
from mx_flash_attn_kernel_opt__b200 import PgqaError, inputs
from oracle import append_kv_ref, paged_decode_ref
from tests.test_parity_gpu import assert_parity

pytestmark = pytest.mark.gpu


def append_case(lens, S_new, Hq, Hkv, P, seed, Sq=1):
    """Pools and a table that cover L_b + S_new tokens (distinct pages), NaN in every
    slot a correct kernel must not read before the append, seq_lens = L_b."""
    inp = inputs.custom_case(len(lens), Hq, Hkv, P, [L + S_new for L in lens], seed=seed,
                             spare_pages=3)
    inp.seq_lens = torch.tensor(lens, dtype=torch.int32)
    inp = inputs.poison(inp)
    g = torch.Generator().manual_seed(seed + 1)
    B = len(lens)
    kn = torch.randn(B, S_new, Hkv, 128, generator=g).to(torch.bfloat16)
    vn = torch.randn(B, S_new, Hkv, 128, generator=g).to(torch.bfloat16)
    q = torch.randn(B, Sq, Hq, 128, generator=g).to(torch.bfloat16)
    return inp, kn, vn, q


def bits(t):
    return t.contiguous().view(torch.int16).cpu()


@pytest.mark.parametrize("S_new", [1, 3, 16, 37])
@pytest.mark.parametrize("P", [16, 64])
def test_append_matches_oracle_bit_exact(S_new, P, cuda_device):
    lens = [0, 1, 15, 16, P - 1, P, 100, 1000]
    inp, kn, vn, _ = append_case(lens, S_new, 32, 8, P, seed=S_new * 7 + P)
    ek, ev = append_kv_ref(inp.k, inp.v, kn, vn, inp.seq_lens, inp.block_table)
    d = inp.to(cuda_device)
    pgqa.append_kv(kn.to(cuda_device), vn.to(cuda_device), d.k, d.v, d.block_table, d.seq_lens)
    torch.cuda.synchronize(cuda_device)
    pgqa.check_device_error()
    assert torch.equal(bits(d.k), bits(ek))
    assert torch.equal(bits(d.v), bits(ev))


@pytest.mark.parametrize("Sq,S_new,causal", [(1, 1, 0), (4, 4, 1), (4, 4, 0), (3, 5, 1),
                                              (8, 8, 1)])
@pytest.mark.parametrize("Hq,Hkv,P", [(32, 8, 16), (28, 4, 64), (16, 1, 32)])
def test_decode_with_append_vs_oracle(Sq, S_new, causal, Hq, Hkv, P, cuda_device):
    lens = [0, 1, 2, 17, 300, 4000]
    inp, kn, vn, q = append_case(lens, S_new, Hq, Hkv, P, seed=Sq * 13 + S_new + P, Sq=Sq)
    ek, ev = append_kv_ref(inp.k, inp.v, kn, vn, inp.seq_lens, inp.block_table)
    ref = paged_decode_ref(q, ek, ev, inp.block_table, inp.seq_lens + S_new,
                           causal=bool(causal))
    d = inp.to(cuda_device)
    out = pgqa.decode(q.to(cuda_device), d.k, d.v, d.block_table, d.seq_lens,
                      causal=bool(causal), k_new=kn.to(cuda_device), v_new=vn.to(cuda_device))
    torch.cuda.synchronize(cuda_device)
    pgqa.check_device_error()
    assert_parity(out, ref, edge=True, what=f"Sq={Sq} S_new={S_new} causal={causal}")
    assert torch.equal(bits(d.k), bits(ek)) and torch.equal(bits(d.v), bits(ev))


def test_decode_steps_loop(cuda_device):
    """An engine-like loop: each step appends one token per sequence and decodes;
    lengths advance on the host.  Every step must match the oracle."""
    steps, Hq, Hkv, P = 6, 32, 8, 16
    lens0 = [5, 16, 31, 250]
    inp, _, _, _ = append_case(lens0, steps, Hq, Hkv, P, seed=41)
    g = torch.Generator().manual_seed(42)
    d = inp.to(cuda_device)
    k_cpu, v_cpu = inp.k.clone(), inp.v.clone()
    lens = inp.seq_lens.clone()
    for step in range(steps):
        kn = torch.randn(len(lens0), 1, Hkv, 128, generator=g).to(torch.bfloat16)
        vn = torch.randn(len(lens0), 1, Hkv, 128, generator=g).to(torch.bfloat16)
        q = torch.randn(len(lens0), Hq, 128, generator=g).to(torch.bfloat16)
        k_cpu, v_cpu = append_kv_ref(k_cpu, v_cpu, kn, vn, lens, inp.block_table)
        ref = paged_decode_ref(q, k_cpu, v_cpu, inp.block_table, lens + 1)
        out = pgqa.decode(q.to(cuda_device), d.k, d.v, d.block_table, lens.to(cuda_device),
                          k_new=kn.to(cuda_device), v_new=vn.to(cuda_device))
        torch.cuda.synchronize(cuda_device)
        assert_parity(out, ref, edge=True, what=f"step {step}")
        lens = lens + 1
    pgqa.check_device_error()


def test_append_past_capacity_and_bad_page_are_reported(cuda_device):
    inp, kn, vn, _ = append_case([10, 20], 4, 8, 2, 16, seed=3)
    d = inp.to(cuda_device)
    width = d.block_table.shape[1]
    # position past the table capacity
    lens = torch.tensor([width * 16 - 2, 0], dtype=torch.int32, device=cuda_device)
    pgqa.append_kv(kn.to(cuda_device), vn.to(cuda_device), d.k, d.v, d.block_table, lens)
    with pytest.raises(PgqaError) as e:
        pgqa.check_device_error()
    assert e.value.status == 10
    # a page id outside the pool, where sequence 1 (length 20) appends: page 20 // 16
    bt = d.block_table.clone()
    bt[1, 1] = inp.num_pages + 5
    pgqa.append_kv(kn.to(cuda_device), vn.to(cuda_device), d.k, d.v, bt, d.seq_lens)
    with pytest.raises(PgqaError) as e:
        pgqa.check_device_error()
    assert e.value.status == 9
    pgqa.check_device_error()  # cleared
