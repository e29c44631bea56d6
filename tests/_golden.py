"""Loader for the committed golden fixtures (made by tests/golden/make_golden.py)."""
import glob
import json
import os

import numpy as np
import torch

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


def bf16(a):
    return torch.from_numpy(np.ascontiguousarray(a)).view(torch.bfloat16)


def quant_cases():
    out = []
    for path in sorted(glob.glob(os.path.join(GOLDEN, "quant_*.npz"))):
        z = np.load(path)
        meta = json.loads(str(z["meta"]))
        case = {k: z[k] for k in z.files if k != "meta"}
        for key in ("q", "k", "v", "km"):
            case[key] = bf16(case[key])
        for key in ("q_codes", "k_codes", "q_scale", "k_scale", "v_amax", "v_scale", "v_codes_sage"):
            case[key] = torch.from_numpy(case[key])
        case["meta"] = meta
        out.append(case)
    return out


def kv_schedule():
    with open(os.path.join(GOLDEN, "kv_schedule.json")) as f:
        return json.load(f)
