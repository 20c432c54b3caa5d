"""Generates the golden vectors in this directory from the reference's own implementation.

The reference (dddd109/mx_flash_attn_kernel_opt_) ships one implementation of this path
that runs outside MetaX hardware: the Triton operator `run_kernel` of
submission_c500_regions.py:979-1201 (same arguments as the C `run_kernel`).  This script
imports it from a local checkout of the reference and runs it on the CPU under Triton's
interpreter (TRITON_INTERPRET=1).  The interpreter stores bf16 as raw uint16 bit
patterns and would compute on them as integers, so `_patch_interpreter_bf16` first makes
it treat them as numbers (bf16 dots as exact fp32 products with fp32 accumulation, as a
tensor core does; elementwise bf16 arithmetic and fp32 -> bf16 casts rounded to nearest).

Inputs come from mx_flash_attn_kernel_opt__b200.inputs (seeded CPU generators, so the
tests regenerate the same bytes; manifest.json records a sha256 of every input).  Every
row of each output is stored, as bf16 bit patterns.

Cases: the reference's 14-case table (verify_real.py:8-10) with contiguous and permuted
tables, benchmark config c1 whole, reduced-batch slices of c3 (its first 8 sequences)
and c4 (g = 7, P = 64: its shortest, median, 90th-percentile and longest sequences) at
the benchmark's shapes, and a NaN-poisoned pool.

Run (needs the reference checkout; not needed by the tests):
    python tests/golden/gen_golden.py --reference /path/to/reference [cases...]
"""
import argparse
import json
import os
import sys
import time

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(os.path.dirname(HERE))


def _patch_interpreter_bf16():
    """Make Triton's CPU interpreter treat bf16 (stored as raw uint16 bits) as numbers:
    dots as exact fp32 products with fp32 accumulation, elementwise bf16 arithmetic in
    fp32 rounded to nearest-even, fp32 -> bf16 casts rounded to nearest-even, and bf16
    scalar constants (what the GPU lowering of these operations does)."""
    import numpy as np
    import torch
    import triton.language as tl
    import triton.runtime.interpreter as interp

    cls = next(obj for name, obj in vars(interp).items()
               if isinstance(obj, type) and hasattr(obj, "create_dot"))

    def bits_to_f32(bits):
        return (np.asarray(bits).astype(np.uint32) << 16).view(np.float32)

    def f32_to_bits(x):
        t = torch.from_numpy(np.ascontiguousarray(np.asarray(x, dtype=np.float32)))
        return t.to(torch.bfloat16).view(torch.int16).numpy().astype(np.uint16)

    def to_f32(h):
        if h.dtype.scalar == tl.bfloat16:
            return bits_to_f32(h.data)
        return h.data.astype(np.float32)

    orig_dot = cls.create_dot

    def create_dot(self, a, b, d, input_precision, max_num_imprecise_acc):
        if a.dtype.scalar == tl.bfloat16 or b.dtype.scalar == tl.bfloat16:
            prod = np.matmul(to_f32(a), to_f32(b), dtype=np.float32)
            return interp.TensorHandle(prod.astype(d.data.dtype) + d.data, d.dtype.scalar)
        return orig_dot(self, a, b, d, input_precision, max_num_imprecise_acc)

    orig_binary = cls.binary_op

    def binary_op(self, lhs, rhs, op):
        if lhs.dtype.scalar == tl.bfloat16 or rhs.dtype.scalar == tl.bfloat16:
            res = op(to_f32(lhs), to_f32(rhs))
            if res.dtype == np.bool_:
                return interp.TensorHandle(res, tl.int1)
            return interp.TensorHandle(f32_to_bits(res), tl.bfloat16)
        return orig_binary(self, lhs, rhs, op)

    orig_cast = cls.cast_impl

    def cast_impl(self, src, dst_type):
        if src.dtype.scalar == tl.float32 and dst_type.scalar == tl.bfloat16:
            return interp.TensorHandle(f32_to_bits(src.data), tl.bfloat16)
        return orig_cast(self, src, dst_type)

    orig_fp2fp = cls.create_fp_to_fp

    def create_fp_to_fp(self, src, dst_type, rounding_mode):
        if src.dtype.scalar == tl.float32 and dst_type.scalar == tl.bfloat16:
            return interp.TensorHandle(f32_to_bits(src.data), tl.bfloat16)
        if src.dtype.scalar == tl.bfloat16 and dst_type.scalar == tl.float32:
            return interp.TensorHandle(bits_to_f32(src.data), tl.float32)
        return orig_fp2fp(self, src, dst_type, rounding_mode)

    def get_bf16(self, value):
        return interp.TensorHandle(f32_to_bits(np.array([value], dtype=np.float32)),
                                   tl.bfloat16)

    cls.create_dot = create_dot
    cls.binary_op = binary_op
    for name in ("create_fadd", "create_fmul", "create_fdiv", "create_fsub", "create_frem",
                 "create_precise_divf"):
        op = {"create_fadd": np.add, "create_fmul": np.multiply, "create_fdiv": np.divide,
              "create_fsub": np.subtract, "create_frem": np.fmod,
              "create_precise_divf": np.divide}[name]
        setattr(cls, name, (lambda o: (lambda self, l, r: self.binary_op(l, r, o)))(op))
    cls.cast_impl = cast_impl
    cls.create_fp_to_fp = create_fp_to_fp
    cls.get_bf16 = get_bf16


def cases():
    out = []
    for c in range(1, 15):
        out.append({"name": f"spj{c:02d}", "kind": "spj", "case": c, "table": "contiguous"})
    for c in (3, 5, 8, 11):
        out.append({"name": f"spj{c:02d}_perm", "kind": "spj", "case": c, "table": "permuted"})
    out.append({"name": "c1", "kind": "config", "config": "c1"})
    sys.path.insert(0, REPO)
    from mx_flash_attn_kernel_opt__b200 import inputs
    for cfg in ("c3", "c4"):
        out.append({"name": f"{cfg}_slice", "kind": "slice", "config": cfg,
                    "index": inputs.golden_slice_index(cfg)})
    out.append({"name": "spj05_poison", "kind": "spj", "case": 5, "table": "permuted",
                "poison": True})
    return out


def make_inputs(spec):
    sys.path.insert(0, REPO)
    from mx_flash_attn_kernel_opt__b200 import inputs
    if spec["kind"] == "spj":
        inp = inputs.spj_case(spec["case"], table=spec["table"])
    elif spec["kind"] == "slice":
        inp = inputs.golden_slice(spec["config"], spec["index"])
    else:
        inp = inputs.baseline_config(spec["config"])
    if spec.get("poison"):
        inp = inputs.poison(inp)
    return inp


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", required=True)
    ap.add_argument("names", nargs="*")
    args = ap.parse_args()
    os.environ["TRITON_INTERPRET"] = "1"
    import numpy as np
    import torch
    import triton

    _patch_interpreter_bf16()
    sys.path.insert(0, args.reference)
    import submission_c500_regions as ref  # the reference's operator

    man_path = os.path.join(HERE, "manifest.json")
    manifest = json.load(open(man_path)) if os.path.exists(man_path) else {"cases": {}}
    manifest["source"] = ("submission_c500_regions.py:run_kernel (reference), CPU, "
                          f"TRITON_INTERPRET=1, triton {triton.__version__}, "
                          f"torch {torch.__version__}")
    for spec in cases():
        if args.names and spec["name"] not in args.names:
            continue
        inp = make_inputs(spec)
        B, Hq, D = inp.q.shape
        nb, P, Hkv, _ = inp.k.shape
        if nb % B:
            raise SystemExit(f"{spec['name']}: pool not a multiple of B")
        out = torch.zeros(B, 1, Hq, D, dtype=torch.bfloat16)
        t0 = time.time()
        ref.run_kernel(inp.q.view(B, 1, Hq, D), inp.k, inp.v, out, inp.seq_lens,
                       inp.block_table, B, inp.seqlen_k, 1, Hq, Hkv, D, P, nb, 0)
        dt = time.time() - t0
        rows = list(range(B))
        bits = out[rows, 0].contiguous().view(torch.int16).numpy().astype(np.uint16)
        np.savez_compressed(os.path.join(HERE, spec["name"] + ".npz"), rows=np.array(rows),
                            out_bf16_bits=bits)
        manifest["cases"][spec["name"]] = {
            "spec": spec, "digest": inp.digest(), "rows": rows, "shape": [B, Hq, D],
            "seqlen_k": inp.seqlen_k, "seq_lens_head": inp.seq_lens[:8].tolist(),
            "interp_seconds": round(dt, 1)}
        json.dump(manifest, open(man_path, "w"), indent=1, sort_keys=True)
        print(f"{spec['name']}: {dt:.1f}s", flush=True)


if __name__ == "__main__":
    main()
