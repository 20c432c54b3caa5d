"""Generates the golden vectors in this directory from the reference's own implementation.

The reference (dddd109/mx_flash_attn_kernel_opt_) ships one implementation of this path
that runs outside MetaX hardware: the Triton operator `run_kernel` of
submission_c500_regions.py:979-1201 (same arguments as the C `run_kernel`).  This script
imports it from a local checkout of the reference and runs it on the CPU under Triton's
interpreter (TRITON_INTERPRET=1).  The interpreter computes `tl.dot` on raw bf16 bit
patterns as integers, so `_patch_interpreter_bf16_dot` first makes it compute bf16 dots
as exact fp32 products with fp32 accumulation (what a tensor core does).

Inputs come from mx_flash_attn_kernel_opt__b200.inputs (seeded CPU generators, so the
tests regenerate the same bytes; manifest.json records a sha256 of every input).  Only
the first rows of each output are stored, as bf16 bit patterns.

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
ROWS_KEPT = 4


def _patch_interpreter_bf16_dot():
    import numpy as np
    import triton.language as tl
    import triton.runtime.interpreter as interp

    cls = next(obj for name, obj in vars(interp).items()
               if isinstance(obj, type) and hasattr(obj, "create_dot"))
    orig = cls.create_dot

    def to_f32(h):
        if h.dtype.scalar == tl.bfloat16:
            return (h.data.astype(np.uint32) << 16).view(np.float32)
        return h.data.astype(np.float32)

    def create_dot(self, a, b, d, input_precision, max_num_imprecise_acc):
        if a.dtype.scalar == tl.bfloat16 or b.dtype.scalar == tl.bfloat16:
            prod = np.matmul(to_f32(a), to_f32(b), dtype=np.float32)
            return interp.TensorHandle(prod.astype(d.data.dtype) + d.data, d.dtype.scalar)
        return orig(self, a, b, d, input_precision, max_num_imprecise_acc)

    cls.create_dot = create_dot


def cases():
    out = []
    for c in range(1, 15):
        out.append({"name": f"spj{c:02d}", "kind": "spj", "case": c, "table": "contiguous"})
    for c in (3, 5, 8, 11):
        out.append({"name": f"spj{c:02d}_perm", "kind": "spj", "case": c, "table": "permuted"})
    out.append({"name": "c1", "kind": "config", "config": "c1"})
    out.append({"name": "spj05_poison", "kind": "spj", "case": 5, "table": "permuted",
                "poison": True})
    return out


def make_inputs(spec):
    sys.path.insert(0, REPO)
    from mx_flash_attn_kernel_opt__b200 import inputs
    if spec["kind"] == "spj":
        inp = inputs.spj_case(spec["case"], table=spec["table"])
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

    _patch_interpreter_bf16_dot()
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
        rows = list(range(min(B, ROWS_KEPT)))
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
