"""The golden vectors come from the reference's Triton operator run under Triton's CPU
interpreter, which tests/golden/gen_golden.py patches so that bf16 (stored there as raw
16-bit patterns) is computed on as numbers.  This test shows the patch is neutral where
it should be and does what it says where it acts, on a small attention-shaped kernel of
this repository's own (a dot, a row max, exp2, a cast to the value type, a second dot):

  * fp32 inputs: the patched interpreter gives bit-identical results to the unpatched
    one (no fp32 operation is touched);
  * bf16 inputs: the patched interpreter matches torch doing the same steps on the CPU
    (bf16 products exact in fp32, fp32 accumulation, bf16 casts rounded to nearest).

It runs in a child process, because TRITON_INTERPRET must be set before triton is
imported and the patch cannot be undone in a process.
"""
import os
import subprocess
import sys
import textwrap

import pytest

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))

CHILD = textwrap.dedent("""
    import os, sys
    os.environ["TRITON_INTERPRET"] = "1"
    sys.path.insert(0, %(golden)r)
    import numpy as np
    import torch
    import triton
    import triton.language as tl

    @triton.jit
    def attn_step(q_ptr, k_ptr, v_ptr, o_ptr, M: tl.constexpr, N: tl.constexpr, D: tl.constexpr):
        om = tl.arange(0, M)
        on = tl.arange(0, N)
        od = tl.arange(0, D)
        q = tl.load(q_ptr + om[:, None] * D + od[None, :])
        k = tl.load(k_ptr + on[:, None] * D + od[None, :])
        v = tl.load(v_ptr + on[:, None] * D + od[None, :])
        s = tl.dot(q, tl.trans(k)) * 0.125
        m = tl.max(s, 1)
        p = tl.exp2(s - m[:, None])
        l = tl.sum(p, 1)
        acc = tl.dot(p.to(v.dtype), v)
        tl.store(o_ptr + om[:, None] * D + od[None, :], acc / l[:, None])

    M, N, D = 16, 32, 64
    g = torch.Generator().manual_seed(3)
    q32, k32, v32 = (torch.randn(r, D, generator=g) for r in (M, N, N))

    def run(q, k, v):
        o = torch.empty(M, D, dtype=torch.float32)
        attn_step[(1,)](q, k, v, o, M, N, D)
        return o

    plain = run(q32, k32, v32)
    import gen_golden
    gen_golden._patch_interpreter_bf16()
    patched = run(q32, k32, v32)
    print("fp32_identical", bool(torch.equal(plain, patched)))

    qb, kb, vb = q32.bfloat16(), k32.bfloat16(), v32.bfloat16()
    got = run(qb, kb, vb)
    s = (qb.float() @ kb.float().T) * 0.125
    p = torch.exp2(s - s.max(1, keepdim=True).values)
    want = (p.bfloat16().float() @ vb.float()) / p.sum(1, keepdim=True)
    err = ((got - want).abs() / want.abs().clamp_min(1e-3)).max().item()
    print("bf16_max_rel_err", err)
""")


def test_interpreter_patch_is_neutral_on_fp32_and_exact_on_bf16():
    pytest.importorskip("triton")
    code = CHILD % {"golden": os.path.join(REPO, "tests", "golden")}
    r = subprocess.run([sys.executable, "-c", code], capture_output=True, text=True, timeout=600,
                       env=dict(os.environ, CUDA_VISIBLE_DEVICES=""))
    assert r.returncode == 0, r.stderr[-3000:]
    lines = dict(l.split(" ", 1) for l in r.stdout.strip().splitlines() if " " in l)
    assert lines.get("fp32_identical") == "True", r.stdout
    assert float(lines["bf16_max_rel_err"]) < 1e-5, r.stdout
