"""The RoPE restatement (oracle/rope.py) against the reference's own rope_params / causal_rope_freqs /
causal_rope_apply outputs (tests/golden/rope_grid2x4x6.npz, from tests/golden/make_golden.py): bit for
bit, tables and rotated values."""
import os

import numpy as np
import torch

from oracle import rope

GOLD = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", "rope_grid2x4x6.npz")


def _bf16(bits):
    return torch.from_numpy(bits).view(torch.bfloat16)


def test_freqs_table_matches_the_reference():
    g = np.load(GOLD)
    assert torch.equal(rope.freqs_table(128)[:16], torch.from_numpy(g["freqs16"]))


def test_rope_tables_match_the_reference():
    g = np.load(GOLD)
    grid = [tuple(int(v) for v in r) for r in g["grid"]]
    cos, sin = rope.rope_tables(grid, rope.freqs_table(128), start_frame=int(g["start_frame"]))
    assert torch.equal(cos, torch.from_numpy(g["cos"])) and torch.equal(sin, torch.from_numpy(g["sin"]))


def test_rope_apply_matches_the_reference_bit_for_bit():
    g = np.load(GOLD)
    out = rope.rope_apply(_bf16(g["x"]), torch.from_numpy(g["cos"]), torch.from_numpy(g["sin"]))
    assert torch.equal(out.view(torch.int16), torch.from_numpy(g["out"]))
