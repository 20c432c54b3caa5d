"""The tcgen05 / TMEM variant of the decode (csrc/pgqa_tc.cu), selected with PGQA_TC=1.

The e4m3, multi-token and log-sum-exp suites already run on both kernels (fixture
`both_kernels`).  These tests cover what is specific to the variant: the one-token bf16
path forced onto it, bit-identical repeats, units split over many CTAs (records and the
last-arriver merge), and an expired wait, after which the CTA still arrives on the
counters of the units it cuts so that the next call on the same workspace is correct.
"""
import pytest
import torch

import mx_flash_attn_kernel_opt__b200 as pgqa
from mx_flash_attn_kernel_opt__b200 import _lib, inputs
from oracle import paged_decode_fp8_ref, paged_decode_ref
from tests.test_parity_gpu import assert_parity

pytestmark = pytest.mark.gpu


@pytest.fixture(autouse=True)
def tc_on(monkeypatch):
    monkeypatch.setenv("PGQA_TC", "1")


@pytest.mark.parametrize("name", ["c1", "c2", "c3", "c4"])
def test_one_token_bf16_on_the_tensor_core_variant(name, cuda_device):
    inp = inputs.baseline_config(name)
    d = inp.to(cuda_device)
    out = pgqa.decode(d.q, d.k, d.v, d.block_table, d.seq_lens, scale=inp.scale)
    torch.cuda.synchronize()
    pgqa.check_device_error()
    ref = paged_decode_ref(inp.q, inp.k, inp.v, inp.block_table, inp.seq_lens)
    assert_parity(out, ref, what=f"tc {name}")


def test_repeated_calls_bit_identical(cuda_device):
    inp = inputs.to_fp8(inputs.custom_case(3, 32, 8, 16, [5000, 17, 3000], seed=41))
    d = inp.to(cuda_device)
    outs = [pgqa.decode(d.q, d.k, d.v, d.block_table, d.seq_lens, k_scale=d.k_scale,
                        v_scale=d.v_scale) for _ in range(3)]
    torch.cuda.synchronize()
    assert torch.equal(outs[0], outs[1]) and torch.equal(outs[1], outs[2])


def _fresh_ws(inp, dev, Sq=1):
    need = _lib.lib().pgqa_workspace_size_v2(inp.batch, Sq, inp.num_heads, inp.num_heads_k,
                                             128, inp.page_size)
    return torch.zeros(need, dtype=torch.uint8, device=dev)


@pytest.mark.parametrize("kv", ["bf16", "fp8"])
def test_expired_wait_reports_timeout_and_leaves_the_workspace_clean(kv, cuda_device,
                                                                     monkeypatch):
    """CTA 0's first stage waits for 16 bytes nothing sends: its bounded waits expire, the
    call reports PGQA_ERR_DEVICE_TIMEOUT, and the next calls on the same workspace are
    correct.  Two long sequences over 8 KV heads split every unit over several CTAs, so
    CTA 0 cuts the unit that continues into CTA 1."""
    base = inputs.custom_case(2, 32, 8, 16, [6000, 5000], seed=43)
    inp = inputs.to_fp8(base) if kv == "fp8" else base
    d = inp.to(cuda_device)
    ws = _fresh_ws(inp, cuda_device)
    kw = dict(k_scale=d.k_scale, v_scale=d.v_scale) if kv == "fp8" else {}
    monkeypatch.setenv("PGQA_DEBUG_STUCK_BARRIER", "1")
    monkeypatch.setenv("PGQA_WAIT_LIMIT_NS", "20000000")
    pgqa.decode(d.q, d.k, d.v, d.block_table, d.seq_lens, workspace=ws, **kw)
    with pytest.raises(pgqa.PgqaError) as e:
        pgqa.check_device_error(ws)
    assert e.value.status == 8
    monkeypatch.delenv("PGQA_DEBUG_STUCK_BARRIER")
    monkeypatch.delenv("PGQA_WAIT_LIMIT_NS")
    if kv == "fp8":
        ref = paged_decode_fp8_ref(inp.q, inp.k, inp.v, inp.k_scale, inp.v_scale,
                                   inp.block_table, inp.seq_lens)
    else:
        ref = paged_decode_ref(inp.q, inp.k, inp.v, inp.block_table, inp.seq_lens)
    for k in range(2):
        out = pgqa.decode(d.q, d.k, d.v, d.block_table, d.seq_lens, workspace=ws, **kw)
        torch.cuda.synchronize()
        pgqa.check_device_error(ws)
        assert_parity(out, ref, what=f"call {k} after timeout ({kv})")
