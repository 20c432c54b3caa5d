"""Helpers to read the golden vectors produced by tests/golden/gen_golden.py."""
import json
import os

import numpy as np
import torch

GOLDEN_DIR = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")
MANIFEST = json.load(open(os.path.join(GOLDEN_DIR, "manifest.json")))
CASES = MANIFEST["cases"]


def make_inputs(spec):
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


def load_rows(name):
    z = np.load(os.path.join(GOLDEN_DIR, name + ".npz"))
    rows = [int(r) for r in z["rows"]]
    bits = torch.from_numpy(z["out_bf16_bits"].astype(np.int16))
    return rows, bits.view(torch.bfloat16)


def is_edge(name):
    spec = CASES[name]["spec"]
    return spec["kind"] == "spj" and spec["case"] in (1, 2, 3)
