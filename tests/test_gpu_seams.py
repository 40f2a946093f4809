"""Decode-step and tree-verification seams (ffnmem/infer.py:152-182, drafting/tree.py:165-195) on the
GPU against the reference's fixtures: the memory_step output equals the full forward of the same
positions, and every tree node equals the linear forward along its ancestor path."""

from __future__ import annotations

import numpy as np
import pytest
import torch

from tests.golden import cases
from tests.helpers import assert_fp32_close
from tests.test_gpu_memory import gpu_memory

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda:0")


def T(a, dt=None):
    t = torch.from_numpy(np.ascontiguousarray(a)).to(DEV)
    return t if dt is None else t.to(dt)


def cache_from(lngram, m, g, max_len=64):
    B, L = g["h_prefix"].shape[:2]
    c = lngram.MemoryCache(m, B, max_len)
    c.codes[:, :L] = T(g["codes_prefix"]).to(torch.uint8)
    c.conv_in[:, :L] = T(g["conv_cache"])
    c.length = L
    return c


def test_memory_step_equals_full_forward(lngram, golden):
    g = golden("seams_tiny_multi")
    m = gpu_memory(lngram, "tiny_multi").module
    c = cache_from(lngram, m, g)
    out = lngram.memory_step(m, c, T(g["h_new"]), T(g["codes_new"])).cpu().numpy()
    assert_fp32_close(out, g["step_output"], what="memory_step vs reference memory_step")
    assert_fp32_close(out, g["step_full"], what="memory_step vs full forward")


def test_tree_block_equals_per_path_linear_forward(lngram, golden):
    g = golden("seams_tiny_multi")
    m = gpu_memory(lngram, "tiny_multi").module
    c = cache_from(lngram, m, g)
    out = lngram.tree_memory_block(m, c, T(g["h_new"]), T(g["codes_new"]), cases.TREE_PARENT).cpu().numpy()
    assert_fp32_close(out, g["tree_output"], what="tree block vs reference block")
    assert_fp32_close(out, g["tree_linear"], rtol=1e-4, what="tree block vs per-path linear forward")
    L = g["h_prefix"].shape[1]
    np.testing.assert_array_equal(c.codes[:, L:L + len(cases.TREE_PARENT)].cpu().numpy(), g["codes_new"])


def test_tree_windows_kat(lngram):
    """The reference's ancestor-window KAT (tests/test_live_tree.py:30-41) through the host builders."""
    codes = torch.tensor([0, 10, 20, 30, 40, 50]).view(1, 6, 1)
    hist = torch.tensor([100, 101]).view(1, 2, 1)
    ctx, ok = lngram.tree_ngram_codes(cases.KAT_PARENT, codes, hist, 2)
    assert ctx[0, :, :, 0].tolist() == [[100, 101, 0], [101, 0, 10], [0, 10, 20], [101, 0, 30], [0, 30, 40],
                                        [0, 10, 50]]
    assert ok.all()
