"""The device work partition (the analytic split policy), checked on the host.

pgqa_simulate_partition runs the same __host__ __device__ arithmetic the kernel runs
(csrc/pgqa_partition.h).  An independent Python model of the intended split is compared
with it, and the invariants that make the decode correct are checked: every 16-token
chunk belongs to exactly one warp, warps get equal work (+-1 chunk), and each unit
(sequence, KV head, head group) is cut into as many pieces as slices cross it.
"""
import ctypes

import numpy as np
import pytest
import torch

from mx_flash_attn_kernel_opt__b200 import _lib, inputs, make_plan


def simulate(seq_lens, U, cap, plan):
    B = len(seq_lens)
    sl = np.ascontiguousarray(seq_lens, dtype=np.int32)
    ctas = np.zeros(B * U, dtype=np.int32)
    segs = np.zeros(B * U, dtype=np.int32)
    n = _lib.lib().pgqa_simulate_partition(
        sl.ctypes.data_as(ctypes.c_void_p), B, U, cap, ctypes.byref(plan),
        ctas.ctypes.data_as(ctypes.c_void_p), segs.ctypes.data_as(ctypes.c_void_p))
    return n, ctas, segs


def py_model(seq_lens, U, cap, grid, W, minc):
    """Independent restatement: cut the chunk sequence into grid/warp slices."""
    n_b = [-(-min(max(L, 0), cap) // 16) for L in seq_lens]
    units = []  # (begin, end) per unit, b-major
    pos = 0
    for nb in n_b:
        for _ in range(U):
            units.append((pos, pos + nb))
            pos += nb
    T = pos
    if T == 0:
        return 0, [0] * len(units), [0] * len(units), []
    nct = max(1, min(grid, T // (W * minc)))
    # equal units: a multiple of the unit count, if that idles at most 1/32 of the CTAs
    n_units = len(n_b) * U
    if len(set(n_b)) == 1 and n_b[0] > 0 and nct >= n_units:
        aligned = nct // n_units * n_units
        if (nct - aligned) * 32 <= nct:
            nct = aligned
    cta_sl = [(c * T // nct, (c + 1) * T // nct) for c in range(nct)]
    warp_sl = []
    for cs, ce in cta_sl:
        ln = ce - cs
        wa = min(W, ln)
        warp_sl += [(cs + w * ln // wa, cs + (w + 1) * ln // wa) for w in range(wa)]

    def overlaps(sl, u):
        return sum(1 for s, e in sl if s < u[1] and u[0] < e)
    ctas = [overlaps(cta_sl, u) if u[1] > u[0] else 0 for u in units]
    segs = [overlaps(warp_sl, u) if u[1] > u[0] else 0 for u in units]
    return nct, ctas, segs, warp_sl


CASES = [
    ("c1", None), ("c2", None), ("c3", None), ("c4", None),
    ("tiny", [1, 2, 3]), ("zeros", [0, 0, 5, 0]), ("one", [1]),
    ("ragged", [1, 4000, 17, 16, 15, 33, 900, 2]),
]


@pytest.mark.parametrize("name,lens", CASES)
def test_partition_matches_model(name, lens):
    if lens is None:
        cfg = inputs.CONFIGS[name]
        seq, cap = inputs.config_seq_lens(name)
        lens = seq.tolist()
        B, Hq, Hkv, P = cfg["B"], cfg["Hq"], cfg["Hkv"], cfg["P"]
    else:
        B, Hq, Hkv, P = len(lens), 32, 4, 16
        cap = max(max(lens), 1)
    st, plan = make_plan(B, Hq, Hkv, 128, P)
    assert st == 0
    U = plan.units_per_seq
    n, ctas, segs = simulate(lens, U, cap, plan)
    mn, mctas, msegs, warp_sl = py_model(lens, U, cap, plan.grid_ctas, plan.warps_per_cta,
                                         plan.min_chunks_per_warp)
    assert n == mn
    assert ctas.tolist() == mctas
    assert segs.tolist() == msegs
    if warp_sl:
        # exact cover, contiguous, balanced
        assert warp_sl[0][0] == 0
        assert all(a[1] == b[0] for a, b in zip(warp_sl, warp_sl[1:]))
        sizes = [e - s for s, e in warp_sl]
        per_cta = plan.warps_per_cta
        assert min(sizes) >= 1
        assert max(sizes) - min(sizes) <= 2 * (1 + (len(sizes) > per_cta))
    for u, L in enumerate(np.repeat(lens, U)):
        assert (segs[u] == 0) == (L <= 0)
        assert segs[u] >= ctas[u]


def test_long_context_split_count_follows_sm_count():
    # c2: 2 sequences x 8 KV heads of 2048 chunks on 148 CTAs -> ~9-10 CTAs per unit
    seq, cap = inputs.config_seq_lens("c2")
    _, plan = make_plan(2, 64, 8, 128, 16)
    n, ctas, segs = simulate(seq.tolist(), plan.units_per_seq, cap, plan)
    # 16 equal units on 148 SMs: 144 CTAs, every unit on exactly 9 of them
    assert n == 144
    assert set(ctas.tolist()) == {9}
    # every warp slice adds one piece, plus one per unit boundary crossed inside a slice
    assert 144 * plan.warps_per_cta <= segs.sum() <= 144 * plan.warps_per_cta + len(segs)
    # with 4 SMs the same work is split 1-2 ways per unit
    st, small = make_plan(2, 64, 8, 128, 16, num_sms=4, smem_optin=232448)
    n4, ctas4, _ = simulate(seq.tolist(), small.units_per_seq, cap, small)
    assert n4 == 4 and max(ctas4) <= 2


def test_tiny_problem_uses_few_ctas():
    _, plan = make_plan(1, 32, 8, 128, 16)
    n, ctas, segs = simulate([16], plan.units_per_seq, 16, plan)
    assert n == 1 and ctas.tolist() == [1] * 8


def test_seq_lens_clamped_to_capacity():
    _, plan = make_plan(2, 32, 8, 128, 16)
    n, _, segs_a = simulate([10**6, 5], plan.units_per_seq, 64, plan)
    n2, _, segs_b = simulate([64, 5], plan.units_per_seq, 64, plan)
    assert segs_a.tolist() == segs_b.tolist()


def test_equal_units_align_with_cta_slices_only_when_cheap():
    """Equal lengths: CTAs become a multiple of the unit count when that idles at most
    1/32 of them (c1: 32 units -> 128 CTAs, 4 per unit); 80 units would idle 68 of 148,
    so that call keeps 148; ragged lengths are never aligned."""
    _, plan = make_plan(4, 32, 8, 128, 16)
    n, ctas, _ = simulate([1024] * 4, plan.units_per_seq, 1024, plan)
    assert n == 128 and set(ctas.tolist()) == {4}
    _, plan = make_plan(10, 80, 8, 128, 16)
    n, _, _ = simulate([32768] * 10, plan.units_per_seq, 32768, plan)
    assert n == 148
    _, plan = make_plan(2, 64, 8, 128, 16)
    n, _, _ = simulate([32768, 32752], plan.units_per_seq, 32768, plan)
    assert n == 148
