"""GPU drafter (lng_drafter_*) against the reference drafter's fixtures and the CPU oracle drafter.

The fixtures were written by the reference's RefDrafter (and agreed with its C++ drafter,
``tests/golden/make_golden.py``).  Bars: codes, shortlist ids and drafted tokens exact; logits
within fp32 tolerance; codes computed by the GPU router may differ only at near-zero logits.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle.drafter import OracleDrafter
from tests.golden import cases
from tests.helpers import assert_fp32_close

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda:0")


@pytest.fixture(autouse=True)
def _clear_device_error(lngram):
    lngram._lib.device_error(clear=True)
    yield
    assert lngram._lib.device_error(clear=True) == 0


def make(lngram, case, act=torch.float32):
    config, arrays = cases.draft_bundle(case)
    return lngram.GpuDrafter(lngram.Bundle(config, arrays, {}), act_dtype=act)


@pytest.mark.parametrize("case", ["tiny", "sdb"])
def test_trace_matches_reference(lngram, golden, case):
    g = golden(f"draft_{case}")
    d = make(lngram, case)
    toks = g["tokens"].tolist()
    n = len(toks) if case == "tiny" else 12
    # teacher-forced with the reference's codes: logits over the full vocabulary
    c, ids, lg = d.trace(toks[:n], codes=g["trace_codes"][:n])
    np.testing.assert_array_equal(c, g["trace_codes"][:n])
    assert (ids == np.arange(d.V)).all()
    k = g["trace_top_ids"].shape[1]
    top = np.argsort(-lg, axis=1, kind="stable")[:, :k]
    np.testing.assert_array_equal(np.take_along_axis(ids, top, 1), g["trace_top_ids"][:n])
    assert_fp32_close(np.take_along_axis(lg, top, 1), g["trace_top_logits"][:n], what="top logits")
    if "trace_logits" in g:
        assert_fp32_close(lg, g["trace_logits"][:n], what="full logits")
    # the GPU router's own codes
    c2, _, _ = d.trace(toks[:n])
    assert (c2 != g["trace_codes"][:n]).mean() < 1e-3


@pytest.mark.parametrize("case", ["tiny", "sdb"])
def test_draft_and_hyp_match_reference(lngram, golden, case):
    g = golden(f"draft_{case}")
    d = make(lngram, case)
    toks = g["tokens"].tolist()
    d.commit(toks[: len(toks) // 2])
    out = d.draft(4, last_codes=True)
    assert out.tokens == g["draft_tokens"].tolist()
    np.testing.assert_array_equal(out.topk_ids, g["draft_ids"])
    assert_fp32_close(out.topk_logits, g["draft_logits"], what="draft top-k logits")
    np.testing.assert_array_equal(out.codes, g["draft_codes"])
    hyp = toks[len(toks) // 2: len(toks) // 2 + 3]
    out = d.draft(3, hyp=hyp)
    assert out.tokens == g["hyp_tokens"].tolist()
    np.testing.assert_array_equal(out.codes, g["hyp_codes"])
    np.testing.assert_array_equal(out.topk_ids, g["hyp_ids"])


def test_stateful_api_matches_oracle(lngram):
    """commit / draft / truncate / reset semantics (the reference's tests/test_live_drafter.py:52-103)."""
    config, arrays = cases.draft_bundle("tiny")
    d = make(lngram, "tiny")
    ref = OracleDrafter(config, arrays)
    a = cases.draft_tokens("tiny", 15, seed=5)
    b = cases.draft_tokens("tiny", 7, seed=6)
    for x in (d, ref):
        x.commit(a)
    np.testing.assert_array_equal(d.committed_codes(), ref.committed_codes())
    first = d.draft(3)
    assert first.tokens == ref.draft(3).tokens
    d.draft(5, hyp=b)
    assert d.length == 15 and d.draft(3).tokens == first.tokens   # drafting never mutates the state
    d.commit(b)
    with_b = d.draft(3)
    d.truncate(15)
    np.testing.assert_array_equal(d.committed_codes(), ref.committed_codes())
    assert d.draft(3).tokens == first.tokens
    assert d.draft(3, hyp=b).tokens == with_b.tokens
    np.testing.assert_array_equal(d.draft(3, hyp=b).topk_logits, with_b.topk_logits)
    e = make(lngram, "tiny")                                        # commit in pieces == at once
    for i in range(0, 15, 4):
        e.commit(a[i:i + 4])
    np.testing.assert_array_equal(e.committed_codes(), d.committed_codes())
    codes = np.random.default_rng(1).integers(0, 16, (5, config["routes"]))
    d.commit(a[:5], codes=codes)                                    # target codes override
    ref.commit(a[:5], codes=codes)
    np.testing.assert_array_equal(d.committed_codes()[-5:], codes.astype(np.uint8))
    np.testing.assert_array_equal(d.committed_codes(), ref.committed_codes())
    assert d.draft(2).tokens == ref.draft(2).tokens
    d.reset()
    assert d.length == 0
    with pytest.raises(RuntimeError):
        d.draft(1)
    with pytest.raises(ValueError):
        d.truncate(3)


def test_draft_batch_equals_per_sequence_drafts(lngram):
    d = make(lngram, "tiny")
    prefixes = np.stack([cases.draft_tokens("tiny", 12, seed=20 + s) for s in range(9)])
    got = d.draft_batch(torch.from_numpy(prefixes).to(DEV), 4).cpu().numpy()
    for s in range(9):
        d.reset()
        d.commit(prefixes[s].tolist())
        assert got[s].tolist() == d.draft(4).tokens, s


def test_bf16_drafter_agrees_with_fp32(lngram, golden):
    """SD-B shape with bf16 embedding / tables / folded readout: top-1 agreement with the fp32
    reference drafter's trace and logits within the bf16 bar."""
    g = golden("draft_sdb")
    d = make(lngram, "sdb", act=torch.bfloat16)
    toks = g["tokens"].tolist()[:12]
    _, _, lg = d.trace(toks, codes=g["trace_codes"][:12])
    top1 = lg.argmax(1)
    assert (top1 == g["trace_top_ids"][:12, 0]).mean() >= 0.8
    scale = np.abs(g["trace_top_logits"][:12]).max()
    assert np.abs(lg.max(1) - g["trace_top_logits"][:12, 0]).max() <= 1e-2 * scale
