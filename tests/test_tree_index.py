"""Tree-verification index building (``seams.ancestor_table`` / ``tree_slots`` / ``tree_ngram_codes``)
against the oracle's restatement of ``drafting/tree.py:96-127`` and the reference's ancestor-window
KAT (``tests/test_live_tree.py:30-41`` in the reference project).  Plain torch on the CPU."""

from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle import memory as om
from tests.golden import cases


def _random_trees(count: int, seed: int = 0):
    rng = np.random.default_rng([11, seed])
    out = [cases.TREE_PARENT, cases.KAT_PARENT, (-1,), (-1, 0, 1, 2, 3, 4, 5)]
    for _ in range(count):
        n = int(rng.integers(1, 24))
        out.append(tuple([-1] + [int(rng.integers(0, i)) for i in range(1, n)]))
    return out


@pytest.mark.parametrize("parent", _random_trees(24))
def test_tree_slots_match_oracle(lngram, parent):
    for L in (0, 1, 2, 7, 40):
        for back in (0, 1, 2, 3, 9, 12):
            want_idx, want_ok = om.tree_slots(parent, L, back)
            idx, ok = lngram.tree_slots(parent, L, back)
            np.testing.assert_array_equal(ok.numpy(), want_ok)
            np.testing.assert_array_equal(np.where(want_ok, idx.numpy(), 0), np.where(want_ok, want_idx, 0))


def test_ancestor_table_levels(lngram):
    anc, level = lngram.ancestor_table(cases.TREE_PARENT, 3)
    assert level.tolist() == [0, 1, 1, 1, 1, 2, 2, 2, 2, 2, 2, 2, 2, 2, 2, 2]
    assert anc[1].tolist() == list(cases.TREE_PARENT)
    assert (anc[3] == -1).all()


def test_tree_windows_kat(lngram):
    codes = torch.tensor([0, 10, 20, 30, 40, 50]).view(1, 6, 1)
    hist = torch.tensor([100, 101]).view(1, 2, 1)
    ctx, ok = lngram.tree_ngram_codes(cases.KAT_PARENT, codes, hist, 2)
    assert ctx[0, :, :, 0].tolist() == [[100, 101, 0], [101, 0, 10], [0, 10, 20], [101, 0, 30], [0, 30, 40],
                                        [0, 10, 50]]
    assert ok.all()
    ctx, ok = lngram.tree_ngram_codes(cases.KAT_PARENT, codes, None, 2)
    want, want_ok = om.tree_ngram_codes(cases.KAT_PARENT, codes.numpy(), None, 2)
    np.testing.assert_array_equal(ctx.numpy(), want)
    np.testing.assert_array_equal(ok.numpy(), want_ok)
