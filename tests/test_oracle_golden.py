"""The CPU oracle against the reference's known answers and the committed golden fixtures.

These pin ``oracle/`` (the checker of every GPU parity test) without the reference present:
the fixtures were written by running the reference (``tests/golden/make_golden.py``).
"""

from __future__ import annotations

import numpy as np
import pytest

from oracle import memory as om
from oracle.drafter import OracleDrafter
from tests.golden import cases
from tests.helpers import assert_fp32_close


# --------------------------------------------------------------------------- known answers
def test_v2_suffix_and_digit_order_kat():
    """The reference's address KAT (``tests/test_index_layout.py:28-40``)."""
    codes = np.array([[[3], [5], [7], [9]]])
    a2 = om.aligned_ngram_address(codes, 2, 4)
    a3 = om.aligned_ngram_address(codes, 3, 4)
    assert a2[0, 0, 0] == 3 + 16 * 5
    assert a3[0, 1, 0] == 5 + 16 * 7 + 256 * 9
    p = cases.oracle_params("tiny_multi")
    rng = np.random.default_rng(0)
    tok = om.lookup_route_chunk(rng.integers(0, 16, (1, 6, p.num_routes)), p.tables, p.ngrams, p.bits, 0,
                                p.num_routes)
    assert np.count_nonzero(tok[:, 0]) == 0                    # nothing complete at t = 0
    assert np.count_nonzero(tok[:, 1, :, p.memory_dim:]) == 0  # no 3-gram at t = 1
    assert np.count_nonzero(tok[:, 1, :, :p.memory_dim]) > 0


def test_tree_ancestor_windows_kat(golden):
    """The reference's ancestor-window KAT (``tests/test_live_tree.py:30-41``)."""
    codes = np.array([0, 10, 20, 30, 40, 50]).reshape(1, 6, 1)
    hist = np.array([100, 101]).reshape(1, 2, 1)
    ctx, ok = om.tree_ngram_codes(cases.KAT_PARENT, codes, hist, 2)
    assert ctx[0, :, :, 0].tolist() == [[100, 101, 0], [101, 0, 10], [0, 10, 20], [101, 0, 30], [0, 30, 40],
                                        [0, 10, 50]]
    assert ok.all()
    ctx, ok = om.tree_ngram_codes(cases.KAT_PARENT, codes, None, 2)
    assert ok.tolist() == [[False, False, True], [False, True, True], [True, True, True], [False, True, True],
                           [True, True, True], [True, True, True]]
    g = golden("seams_tiny_multi")
    np.testing.assert_array_equal(om.tree_ngram_codes(cases.KAT_PARENT, codes, hist, 2)[0][0, :, :, 0],
                                  g["kat_ctx_hist"])
    np.testing.assert_array_equal(ctx[0, :, :, 0], g["kat_ctx_nohist"])
    np.testing.assert_array_equal(ok, g["kat_ok_nohist"])


def test_pack_bits_and_zero_tie():
    """``lngram_v2.py:74-89``; a logit of exactly 0 is a 0 bit (``:1017`` uses ``> 0``)."""
    logits = np.array([[[0.5, -1.0, 2.0, 0.0, -0.0, 1e-30, 3.0, -2.0]]], np.float32)
    assert om.quantize_route_logits(logits, 4).tolist() == [[[1 + 4, 2 + 4]]]


# --------------------------------------------------------------------------- memory layer
@pytest.mark.parametrize("case", list(cases.MEMORY_CASES))
def test_memory_oracle_matches_reference(golden, case):
    g = golden(f"memory_{case}")
    c = cases.MEMORY_CASES[case]
    p = cases.oracle_params(case)
    inp = cases.memory_inputs(case)
    if "in_h" in g:
        np.testing.assert_array_equal(inp["h"], g["in_h"])   # the seeded inputs are what the fixture saw
    seg = inp.get("segment_ids")
    valid = inp.get("valid_tokens")
    router_w = cases.memory_params(case)["router.weight"]
    logits = om.route_logits(inp["x"], router_w)
    assert_fp32_close(logits, g["logits"], what="router logits")
    codes = g["codes"].astype(np.int64)                  # readout checks start from identical codes
    np.testing.assert_array_equal(om.quantize_route_logits(g["logits"], p.bits), codes)
    tokens = om.lookup_route_chunk(codes, p.tables, p.ngrams, p.bits, 0, p.num_routes, seg, valid)
    if "tokens" in g:
        np.testing.assert_array_equal(tokens, g["tokens"])
    else:
        for n in p.ngrams:
            np.testing.assert_array_equal(om.row_indices(codes, n, p.bits, 0, p.num_routes), g[f"rows_{n}"])
        np.testing.assert_allclose(tokens.astype(np.float64).sum(-1), g["token_sums"], rtol=1e-6, atol=1e-7)
    q = om.project_query(inp["h"], p)
    assert_fp32_close(q, g["query"], what="query")
    key, value = om.project_memory(tokens, p)
    if "key" in g:
        assert_fp32_close(key, g["key"], what="key")
        assert_fp32_close(value, g["value"], what="value")
    head = om.manual_gqa(q, key, value, p)
    assert_fp32_close(head, g["head"], what="head")
    out = om.memory_forward(inp["h"], codes, p, seg, valid)
    assert_fp32_close(out, g["output"], what="module output")
    wrapper = om.lngram_memory_forward(inp["h"], inp["x"], router_w, p)
    assert_fp32_close(wrapper, g["output_wrapper"], what="LngramMemory output")
    if c.get("stream_chunk"):
        stream = om.memory_forward(inp["h"], codes, p, seg, valid, streaming_chunk=c["stream_chunk"])
        assert_fp32_close(stream, g["output_streaming"], what="streaming output")


def test_decode_and_tree_seams(golden):
    g = golden("seams_tiny_multi")
    p = cases.oracle_params("tiny_multi")
    B, L = g["h_prefix"].shape[:2]
    n = g["h_new"].shape[1]
    hist = p.route_history_length
    ctx = np.concatenate((g["codes_prefix"], g["codes_new"]), 1)[:, max(0, L - hist):]
    lp = (p.conv_weight.shape[-1] - 1) * p.dilation
    conv_hist = g["conv_cache"][:, max(0, L - lp):]
    if conv_hist.shape[1] < lp:
        conv_hist = np.concatenate((np.zeros((B, lp - conv_hist.shape[1], conv_hist.shape[2]), np.float32),
                                    conv_hist), 1)
    out, _ = om.memory_step(g["h_new"], ctx, conv_hist, p)
    assert_fp32_close(out, g["step_output"], what="memory_step")
    assert_fp32_close(out, g["step_full"], what="memory_step vs full forward")
    tree = om.tree_memory_block(g["h_new"], g["codes_new"], cases.TREE_PARENT, g["codes_prefix"][:, L - hist:],
                                g["conv_cache"], L, p)
    assert_fp32_close(tree, g["tree_output"], what="tree block")
    assert_fp32_close(tree, g["tree_linear"], rtol=1e-4, what="tree block vs per-path linear forward")
    ctxw, ok = om.tree_ngram_codes(cases.TREE_PARENT, g["codes_new"], g["codes_prefix"][:, L - hist:], hist)
    np.testing.assert_array_equal(ctxw, g["tree_ctx"])
    np.testing.assert_array_equal(ok, g["tree_valid"])


# --------------------------------------------------------------------------- drafter
@pytest.mark.parametrize("case", ["tiny", "sdb"])
def test_drafter_oracle_matches_reference(golden, case):
    g = golden(f"draft_{case}")
    config, arrays = cases.draft_bundle(case)
    d = OracleDrafter(config, arrays)
    toks = g["tokens"].tolist()
    n = len(toks) if case == "tiny" else 10
    c, ids, lg = d.trace(toks[:n])
    np.testing.assert_array_equal(c, g["trace_codes"][:n])
    k = g["trace_top_ids"].shape[1]
    top = np.argsort(-lg, axis=1, kind="stable")[:, :k]
    np.testing.assert_array_equal(np.take_along_axis(ids, top, 1), g["trace_top_ids"][:n])
    assert_fp32_close(np.take_along_axis(lg, top, 1), g["trace_top_logits"][:n], what="trace logits")
    if "trace_logits" in g:
        assert_fp32_close(lg, g["trace_logits"][:n], what="full trace logits")
    d.reset()
    d.commit(toks[: len(toks) // 2])
    out = d.draft(4, last_codes=True)
    assert out.tokens == g["draft_tokens"].tolist()
    np.testing.assert_array_equal(out.topk_ids, g["draft_ids"])
    assert_fp32_close(out.topk_logits, g["draft_logits"], what="draft logits")
    np.testing.assert_array_equal(out.codes, g["draft_codes"])
    hyp = toks[len(toks) // 2: len(toks) // 2 + 3]
    out = d.draft(3, hyp=hyp)
    assert out.tokens == g["hyp_tokens"].tolist()
    np.testing.assert_array_equal(out.codes, g["hyp_codes"])
    # the reference C++ drafter saw the same codes and agreed with RefDrafter
    assert float(g["cpp_code_mismatch"]) < 1e-3
    np.testing.assert_allclose(g["cpp_trace_top_logits"], g["trace_top_logits"], atol=1e-4)


def test_c_oracle_matches_numpy_oracle():
    """The plain-C addressing oracle (used at the full benchmark sizes) equals the numpy restatement."""
    from oracle.build import load_c_oracle

    lib = load_c_oracle()
    rng = np.random.default_rng(5)
    for (B, T, R, order, bits) in [(3, 40, 4, 2, 4), (2, 64, 184, 3, 4), (2, 24, 3, 4, 5), (32, 2048, 184, 3, 4)]:
        codes = rng.integers(0, 1 << bits, (B, T, R)).astype(np.uint8)
        seg = np.cumsum(rng.random((B, T)) < 0.05, axis=1).astype(np.int64)
        valid = (rng.random((B, T)) > 0.1).astype(np.uint8)
        rows = np.empty((B, T, R), np.int64)
        lib.oracle_row_indices(codes.ctypes.data, B, T, R, order, bits, seg.ctypes.data, valid.ctypes.data,
                               rows.ctypes.data)
        want = np.full((B, T, R), -1, np.int64)
        if T >= order:
            mask = om.valid_mask(order, B, T, seg, valid.astype(bool))
            want[:, order - 1:] = om.row_indices(codes.astype(np.int64), order, bits, 0, R)
            want[~mask] = -1
        np.testing.assert_array_equal(rows, want)
    logits = rng.standard_normal((50, 184 * 4)).astype(np.float32)
    packed = np.empty((50, 184), np.uint8)
    lib.oracle_pack_codes(logits.ctypes.data, 50, 184, 4, packed.ctypes.data)
    np.testing.assert_array_equal(packed, om.quantize_route_logits(logits, 4))


def test_packed_incremental_state_matches_reference_fixture(golden):
    """The packed n-gram suffix after every forward_incremental call (lngram_v2.py:1714-1760)."""
    from tests.golden.make_golden import INCREMENTAL_CALLS

    for case in ("tiny_multi", "scaled_slice"):
        g = golden(f"incremental_{case}")
        c = cases.MEMORY_CASES[case]
        maxn, bits = max(c["ngrams"]), c["bits"]
        codes = g["codes"].astype(np.int64)
        packed, t0, length = None, 0, 0
        for i, n in enumerate(INCREMENTAL_CALLS):
            if n == 1:
                packed = om.advance_packed(packed, codes[:, t0], maxn, bits)
                length = min(length + 1, maxn)
            else:
                ctx = codes[:, max(0, t0 - (maxn - 1)):t0 + n]
                packed = om.pack_suffix(ctx, maxn, bits)
                length = min(ctx.shape[1], maxn) if t0 == 0 else min(length + n, maxn)
            np.testing.assert_array_equal(packed, g[f"packed_{i}"])
            assert length == int(g[f"length_{i}"])
            t0 += n


def test_serving_layout_matches_reference_fixture(golden):
    g = golden("serving_tiny_multi")
    c = cases.MEMORY_CASES["tiny_multi"]
    p = cases.memory_params("tiny_multi")
    for n in c["ngrams"]:
        st = om.serving_table(p[f"tables.ngram_{n}.weight"], c["routes"], n, c["bits"])
        np.testing.assert_array_equal(st[g[f"rows_idx_{n}"]], g[f"rows_{n}"])
    # the serving tokens are the v2 tokens (serving/layout.py:15-17)
    np.testing.assert_array_equal(g["tokens"], g["tokens_v2"])


def test_surrogate_backward_matches_reference_fixture(golden):
    """The training lookup's backward restated (lngram_v2.py:326-447) against the reference's autograd."""
    from tests.golden.make_golden import SURROGATE_CASES

    g = golden("surrogate_backward")
    for i, (case, mode, rs, re) in enumerate(SURROGATE_CASES):
        c = cases.MEMORY_CASES[case]
        p = cases.memory_params(case)
        inp = cases.memory_inputs(case)
        tables = {n: p[f"tables.ngram_{n}.weight"] for n in c["ngrams"]}
        gq, tg = om.surrogate_backward(g[f"c{i}_grad_tokens"], g[f"c{i}_codes"].astype(np.int64), g[f"c{i}_q"],
                                       tables, c["ngrams"], c["bits"], rs, re, 0.7, 1.3, mode == "exact",
                                       inp.get("segment_ids"), inp.get("valid_tokens"))
        want = g[f"c{i}_grad_q"][:, :, rs:re]
        assert_fp32_close(gq, want, rtol=1e-4, what=f"case {i} grad_q")
        assert not g[f"c{i}_grad_q"][:, :, :rs].any() and not g[f"c{i}_grad_q"][:, :, re:].any()
        for n in c["ngrams"]:
            rows = g[f"c{i}_rows_{n}"]
            got = np.stack([tg[n].get(int(r), np.zeros(c["mem_dim"], np.float32)) for r in rows])
            assert_fp32_close(got, g[f"c{i}_grad_table_{n}"], what=f"case {i} table {n} grad")
            assert set(int(r) for r, v in tg[n].items() if np.any(v != 0)) <= set(rows.tolist())


def test_online_counts_oracle_matches_reference(golden):
    """The online-count mixer restated (``oracle.drafter.online_counts_mix``) equals the reference's
    ``OnlineCounts.mix`` bit for bit on the fixture's records (mixed and unmixed rows, deadlines of -1)."""
    from oracle.drafter import online_counts_mix
    from tests.golden.make_golden import ONLINE_CASES

    g = golden("online_counts")
    for i, (orders, bits, kappa) in enumerate(ONLINE_CASES):
        got = online_counts_mix(g[f"c{i}_codes"], g[f"c{i}_x"], orders, bits, int(g[f"c{i}_vocab"]), kappa,
                                g[f"c{i}_p"], g[f"c{i}_win"], g[f"c{i}_real"], g[f"c{i}_deadline"])
        np.testing.assert_array_equal(got, g[f"c{i}_mixed"])
