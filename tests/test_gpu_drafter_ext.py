"""The GPU drafter's SD-C SSM and sketch shortlist, and the extension-class API, against the oracle drafter
(pinned to the reference's RefDrafter and C++ drafter, ``tests/test_oracle_reference_pins.py``) and, where
it was built, the reference's own C++ drafter class (``oracle/_ref``).

Bars: codes, shortlist ids and drafted tokens exact (given the same codes); logits within the fp32
tolerance; the GPU router's own codes may differ only at near-zero logits.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle.drafter import OracleDrafter
from tests.golden import cases
from tests.helpers import BF16_TOL, assert_bf16_close, assert_fp32_close

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda:0")


@pytest.fixture(autouse=True)
def _clear_device_error(lngram):
    lngram._lib.device_error(clear=True)
    yield
    assert lngram._lib.device_error(clear=True) == 0


def bundle(case: str, sketch: bool = False, cap: int = 16, k: int = 4, fallback: bool = True):
    config, arrays = cases.draft_bundle(case)
    if sketch:
        config = dict(config, sketch_k=k, shortlist_cap=cap)
        sk = cases.random_sketch(config, k=k, cap=cap)
        if not fallback:
            sk["fallback"] = np.zeros(0, np.int32)
        arrays = dict(arrays, **sk)
    return config, arrays


def pair(lngram, case, sketch=False, act=torch.float32, **kw):
    config, arrays = bundle(case, sketch, **kw)
    return lngram.GpuDrafter(lngram.Bundle(config, arrays, {}), act_dtype=act), OracleDrafter(config, arrays), config


def _compare_trace(d, ref, toks, full=False):
    c_o, i_o, l_o = ref.trace(toks, full=full)
    c_g, i_g, l_g = d.trace(toks, codes=c_o, full=full)     # the oracle's codes: the same table rows
    np.testing.assert_array_equal(c_g, c_o)
    np.testing.assert_array_equal(i_g, i_o)
    fin = np.isfinite(l_o)
    np.testing.assert_array_equal(np.isfinite(l_g), fin)
    assert_fp32_close(l_g[fin], l_o[fin], what="trace logits")
    c_own, _, _ = d.trace(toks, full=full)                  # the GPU router's own codes
    assert (c_own != c_o).mean() < 1e-2


@pytest.mark.parametrize("case,sketch", [("tiny_ssm", False), ("tiny_ssm", True), ("tiny", True)])
def test_trace_matches_oracle(lngram, case, sketch):
    d, ref, _ = pair(lngram, case, sketch)
    toks = cases.draft_tokens(case, 40, seed=11)
    _compare_trace(d, ref, toks)
    if sketch:
        _compare_trace(d, ref, toks, full=True)


def test_shortlist_without_fallback_reads_the_vocabulary_when_empty(lngram):
    """Positions with no complete n-gram and no fallback list score the whole vocabulary
    (drafter.cpp:539-542): the trace's first columns are ids 0 .. S-1."""
    d, ref, config = pair(lngram, "tiny", sketch=True, fallback=False)
    toks = cases.draft_tokens("tiny", 12, seed=12)
    _compare_trace(d, ref, toks)
    _, ids, _ = d.trace(toks)
    assert ids[0].tolist() == list(range(config["shortlist_cap"]))


@pytest.mark.parametrize("case,sketch", [("tiny_ssm", False), ("tiny_ssm", True), ("tiny", True)])
def test_stateful_drafting_matches_oracle(lngram, case, sketch):
    d, ref, config = pair(lngram, case, sketch)
    a = cases.draft_tokens(case, 21, seed=13)
    b = cases.draft_tokens(case, 5, seed=14)
    for x in (d, ref):
        x.commit(a)
    np.testing.assert_array_equal(d.committed_codes(), ref.committed_codes())
    for hyp in ((), b):
        g, o = d.draft(4, hyp=hyp, last_codes=True), ref.draft(4, hyp=hyp, last_codes=True)
        assert g.tokens == o.tokens
        np.testing.assert_array_equal(g.topk_ids, o.topk_ids)
        np.testing.assert_array_equal(g.codes, o.codes)
        fin = np.isfinite(o.topk_logits)
        assert_fp32_close(g.topk_logits[fin], o.topk_logits[fin], what="draft top-k logits")
    first = d.draft(3).tokens
    d.commit(b)
    ref.commit(b)
    assert d.draft(3).tokens == ref.draft(3).tokens
    d.truncate(21)                                          # exact rollback, SSM state included
    ref.truncate(21)
    assert d.draft(3).tokens == first == ref.draft(3).tokens
    codes = np.random.default_rng(4).integers(0, 16, (3, config["routes"]))
    d.commit(b[:3], codes=codes)                            # target codes override; the SSM still advances
    ref.commit(b[:3], codes=codes)
    np.testing.assert_array_equal(d.committed_codes(), ref.committed_codes())
    assert d.draft(3).tokens == ref.draft(3).tokens


@pytest.mark.parametrize("case,sketch", [("tiny_ssm", False), ("tiny_ssm", True), ("tiny", True)])
def test_draft_batch_equals_per_sequence_drafts(lngram, case, sketch):
    d, _, _ = pair(lngram, case, sketch)
    prefixes = np.stack([cases.draft_tokens(case, 13, seed=30 + s) for s in range(7)])
    got = d.draft_batch(torch.from_numpy(prefixes).to(DEV), 4).cpu().numpy()
    for s in range(7):
        d.reset()
        d.commit(prefixes[s].tolist())
        assert got[s].tolist() == d.draft(4).tokens, s


def test_sdb_ssm_bf16_draft_batch_matches_oracle(lngram):
    """SD-C at the SD-B width in bf16: drafted tokens equal the oracle's argmax along the drafted path,
    or are a near tie within the bf16 bar."""
    config, arrays = bundle("sdb_ssm")
    d = lngram.GpuDrafter(lngram.Bundle(config, arrays, {}), act_dtype=torch.bfloat16)
    ref = OracleDrafter(config, arrays)
    V = int(config["vocab"])
    nseq, plen, gamma = 8, 64, 4
    prefix = np.stack([cases.draft_tokens("sdb_ssm", plen, seed=40 + s) for s in range(nseq)])
    drafted = d.draft_batch(torch.from_numpy(prefix).to(DEV), gamma).cpu().numpy()
    agree = total = 0
    for s in range(nseq):
        toks = prefix[s].tolist() + drafted[s, :gamma - 1].tolist()   # the SSM state runs over the whole prefix
        g_codes, _, g_lg = d.trace(toks)
        _, _, o_lg = ref.trace(toks, codes=g_codes, full=True)
        for g in range(gamma):
            row = o_lg[plen - 1 + g].astype(np.float64)
            assert_bf16_close(g_lg[plen - 1 + g], row, what=f"seq {s} step {g}")
            best = int(np.lexsort((np.arange(V), -row))[0])
            tok = int(drafted[s, g])
            total += 1
            agree += tok == best
            if tok != best:
                assert row[best] - row[tok] <= 2 * BF16_TOL * np.abs(row).max()
    assert agree / total >= 0.75, (agree, total)


def test_extension_class_api(lngram):
    """``Drafter(tensors, numbers, ngrams, threads)`` with the extension's methods and return types,
    against the reference's own C++ class where it was built (else the oracle)."""
    from oracle.build import load_reference_drafter

    config, arrays = bundle("tiny_ssm", sketch=True)
    tensors = {k: torch.from_numpy(np.ascontiguousarray(v)) for k, v in arrays.items()}
    numbers = lngram.drafter.bundle_numbers(config)
    ngrams = [int(n) for n in config["ngrams"]]
    core = lngram.Drafter(tensors, numbers, ngrams, 4)
    toks = cases.draft_tokens("tiny_ssm", 30, seed=15)
    core.commit(toks[:20])
    assert core.length() == 20
    cc = core.committed_codes()
    assert cc.dtype == torch.uint8 and tuple(cc.shape) == (20, config["routes"])
    t, ids, lg, codes = core.draft(4, toks[20:23], 3, True)
    assert t.dtype == torch.int64 and ids.shape == (4, 3) and lg.dtype == torch.float32
    assert codes.dtype == torch.uint8 and codes.shape == (3 + 4, config["routes"])
    oc, oi, ol = core.trace(toks[:10])
    assert oi.shape == (10, config["shortlist_cap"])
    with pytest.raises(RuntimeError):
        core.truncate(99)
    with pytest.raises(RuntimeError):
        lngram.Drafter(tensors, {k: v for k, v in numbers.items() if k != "vocab"}, ngrams)
    ext = load_reference_drafter()
    if ext is None:
        ref = OracleDrafter(config, arrays)
        ref.commit(toks[:20])
        o = ref.draft(4, hyp=toks[20:23], last_codes=True)
        assert t.tolist() == o.tokens
        return
    rtensors = {k: (torch.from_numpy(np.minimum(v.astype(np.int64), 2**31 - 1).astype(np.int32))
                    if v.dtype.kind in "ui" else torch.from_numpy(np.ascontiguousarray(v))) for k, v in arrays.items()}
    rc = ext.Drafter(rtensors, numbers, ngrams, 2)
    rc.commit(toks[:20], None)
    assert torch.equal(rc.committed_codes(), cc)
    rt, rids, rlg, rcodes = rc.draft(4, toks[20:23], 3, True)
    assert torch.equal(rt, t) and torch.equal(rids, ids) and torch.equal(rcodes, codes)
    fin = torch.isfinite(rlg)
    assert_fp32_close(lg[fin].numpy(), rlg[fin].numpy(), rtol=1e-4, what="C++ class logits")
    roc, roi, rol = rc.trace(toks[:10], oc, False)
    assert torch.equal(roi, oi)
    fin = torch.isfinite(rol)
    assert_fp32_close(ol[fin].numpy(), rol[fin].numpy(), rtol=1e-4, what="C++ class trace logits")


@pytest.mark.parametrize("case,sketch", [("tiny_ssm", True), ("tiny", False)])
def test_draft_batch_replays_read_new_prefixes(lngram, case, sketch):
    """Repeated draft_batch calls on the same buffers (the library replays a captured graph of the first
    call's launches) draft from the prefix contents of each call, as fresh per-sequence drafts do."""
    d, _, _ = pair(lngram, case, sketch)
    nseq, plen, gamma = 5, 11, 4
    prefix = torch.empty(nseq, plen, dtype=torch.int64, device=DEV)
    out = torch.empty(nseq, gamma, dtype=torch.int64, device=DEV)
    for it in range(4):
        p = np.stack([cases.draft_tokens(case, plen, seed=100 * it + s) for s in range(nseq)])
        prefix.copy_(torch.from_numpy(p))
        got = d.draft_batch(prefix, gamma, out=out).cpu().numpy()
        for s in range(nseq):
            d.reset()
            d.commit(p[s].tolist())
            assert got[s].tolist() == d.draft(gamma).tokens, (it, s)
    # another shape on the same drafter, then the first again
    short = d.draft_batch(prefix[:3, 4:], 2).cpu().numpy()
    for s in range(3):
        d.reset()
        d.commit(p[s, 4:].tolist())
        assert short[s].tolist() == d.draft(2).tokens, s
    again = d.draft_batch(prefix, gamma, out=out).cpu().numpy()
    assert np.array_equal(again, got)
