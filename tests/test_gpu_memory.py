"""GPU parity of the memory path (C ABI on a B200) against the CPU oracle and the reference fixtures.

Bars: codes, row indices and gathered rows bit-exact; fp32 outputs within 1e-5 relative; bf16
outputs within 1e-2 of the fp32 oracle; codes computed from raw inputs may differ only where the
reference logit is within TAU of zero.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle import memory as om
from tests.golden import cases
from tests.helpers import TAU, assert_bf16_close, assert_fp32_close, code_mismatch_ok

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda:0")


def gpu_memory(lngram, case: str, dtype=torch.float32):
    c = cases.MEMORY_CASES[case]
    mem = lngram.LngramMemory(c["d"], {"routes": c["routes"], "mem_dim": c["mem_dim"], "kv_heads": c["kv_heads"],
                                       "q_heads": c["q_heads"], "head_dim": c["head_dim"], "ngrams": list(c["ngrams"]),
                                       "bits_per_route": c["bits"]}, norm_eps=1e-5, device=DEV, dtype=dtype).eval()
    p = cases.memory_params(case)
    state = {("router.weight" if k == "router.weight" else "module." + k): torch.from_numpy(v) for k, v in p.items()}
    mem.load_state_dict(state, strict=True)
    return mem


def T(a, dtype=None):
    t = torch.from_numpy(np.ascontiguousarray(a)).to(DEV)
    return t if dtype is None else t.to(dtype)


@pytest.fixture(autouse=True)
def _clear_device_error(lngram):
    lngram._lib.device_error(clear=True)
    yield
    assert lngram._lib.device_error(clear=True) == 0, "a kernel recorded a device-side error"


# --------------------------------------------------------------------------- a4: pack
def test_quantize_route_logits_bit_exact(lngram):
    rng = np.random.default_rng(0)
    logits = rng.standard_normal((7, 33, 184 * 4)).astype(np.float32)
    logits[rng.random(logits.shape) < 0.05] = 0.0     # ties at zero are a 0 bit
    logits[0, 0, :8] = [-0.0, 0.0, 1e-38, -1e-38, 5, -5, 0, 1]
    m = lngram.RouteNgramMemoryV2(1024, num_routes=184, memory_dim=136, ngrams=(3,), readout_num_heads=16,
                                  readout_num_kv_heads=4, readout_head_dim=64, device=DEV)
    got = m.quantize_route_logits(T(logits)).cpu().numpy()
    np.testing.assert_array_equal(got, om.quantize_route_logits(logits, 4))
    assert got.dtype == np.int32


# --------------------------------------------------------------------------- a3: router
@pytest.mark.parametrize("case", list(cases.MEMORY_CASES))
def test_router_logits_and_codes(lngram, golden, case):
    g = golden(f"memory_{case}")
    mem = gpu_memory(lngram, case)
    x = cases.memory_inputs(case)["x"]
    logits = mem.route_logits(T(x)).cpu().numpy()
    assert_fp32_close(logits, g["logits"], what="router logits")
    codes = mem.route_codes(T(x)).cpu().numpy()
    frac = code_mismatch_ok(codes, g["codes"], g["logits"], cases.MEMORY_CASES[case]["bits"])
    assert frac < 1e-3
    if cases.MEMORY_CASES[case].get("bf16"):   # bf16 router input path
        codes_b = mem.route_codes(T(x, torch.bfloat16)).cpu().numpy()
        code_mismatch_ok(codes_b, g["codes"], g["logits"], cases.MEMORY_CASES[case]["bits"])


# --------------------------------------------------------------------------- a5/a6: lookup
@pytest.mark.parametrize("case", list(cases.MEMORY_CASES))
@pytest.mark.parametrize("code_dtype", [torch.uint8, torch.int32])
def test_lookup_route_chunk_bit_exact(lngram, golden, case, code_dtype):
    g = golden(f"memory_{case}")
    inp = cases.memory_inputs(case)
    p = cases.oracle_params(case)
    mem = gpu_memory(lngram, case).module
    codes = g["codes"].astype(np.int64)
    seg, valid = inp.get("segment_ids"), inp.get("valid_tokens")
    seg_t = None if seg is None else T(seg)
    val_t = None if valid is None else T(valid)
    with torch.no_grad():
        got = mem._lookup_route_chunk(T(codes, code_dtype), None, 0, p.num_routes, seg_t, val_t).cpu().numpy()
    want = om.lookup_route_chunk(codes, p.tables, p.ngrams, p.bits, 0, p.num_routes, seg, valid)
    np.testing.assert_array_equal(got, want)
    if "tokens" in g:
        np.testing.assert_array_equal(got, g["tokens"])
    # a route sub-range and the decode-time target_length view
    r0, r1 = p.num_routes // 3, p.num_routes
    with torch.no_grad():
        sub = mem._lookup_route_chunk(T(codes, code_dtype), None, r0, r1, seg_t, val_t, target_length=5).cpu().numpy()
    np.testing.assert_array_equal(sub, want[:, -5:, r0:r1])


def test_lookup_windows_kat_and_tree(lngram, golden):
    """Windowed lookup == the reference's tree_route_tokens windows (tests/test_live_tree.py KAT)."""
    g = golden("seams_tiny_multi")
    p = cases.oracle_params("tiny_multi")
    mem = gpu_memory(lngram, "tiny_multi").module
    ctx, valid = g["tree_ctx"], g["tree_valid"]
    b, n, w, r = ctx.shape
    seg = np.broadcast_to(valid.astype(np.int32)[None], (b, n, w)).reshape(b * n, w).copy()
    out = torch.empty(b * n, r, p.route_token_dim, device=DEV, dtype=torch.float32)
    codes = T(ctx.reshape(b * n, w, r).astype(np.int32))
    lib = lngram._lib
    lib.check(lib.library().lng_lookup_windows(mem.tables_desc(), codes.data_ptr(), lib.I32, b * n, w,
                                              T(seg).data_ptr(), out.data_ptr(), lib.F32, lib.stream_ptr()))
    want = om.tree_route_tokens(ctx, valid, p).reshape(b * n, r, -1)
    np.testing.assert_array_equal(out.cpu().numpy(), want)


# --------------------------------------------------------------------------- a7/a8: reference pieces
@pytest.mark.parametrize("case", ["tiny", "tiny_multi", "scaled_slice"])
def test_project_and_gqa_pieces(lngram, golden, case):
    g = golden(f"memory_{case}")
    mem = gpu_memory(lngram, case).module
    inp = cases.memory_inputs(case)
    with torch.no_grad():
        q = mem._project_query(T(inp["h"]))
        assert_fp32_close(q.cpu().numpy(), g["query"], what="query")
        k, v = mem._project_memory(T(g["tokens"]))
        assert_fp32_close(k.cpu().numpy(), g["key"], what="key")
        assert_fp32_close(v.cpu().numpy(), g["value"], what="value")
        head = mem._manual_gqa(T(g["query"]), T(g["key"]), T(g["value"]))
        assert_fp32_close(head.cpu().numpy(), g["head"], what="head")
        out = mem._finish(T(g["head"]), T(inp["segment_ids"]) if "segment_ids" in inp else None)
    if "valid_tokens" not in inp:
        assert_fp32_close(out.cpu().numpy(), g["output"], what="_finish")


# --------------------------------------------------------------------------- a11: module forward
@pytest.mark.parametrize("case", list(cases.MEMORY_CASES))
def test_memory_forward_fp32(lngram, golden, case):
    g = golden(f"memory_{case}")
    inp = cases.memory_inputs(case)
    mem = gpu_memory(lngram, case)
    seg = T(inp["segment_ids"]) if "segment_ids" in inp else None
    val = T(inp["valid_tokens"]) if "valid_tokens" in inp else None
    with torch.no_grad():
        out = mem.module(T(inp["h"]), T(g["codes"].astype(np.int32)), segment_ids=seg, valid_tokens=val)
        assert_fp32_close(out.cpu().numpy(), g["output"], what="module forward")
        if "output_streaming" in g:
            assert_fp32_close(out.cpu().numpy(), g["output_streaming"], what="streaming forward")
        if "segment_ids" not in inp and "valid_tokens" not in inp:
            wrapped = mem(T(inp["h"]), T(inp["x"]))
            p = cases.oracle_params(case)
            codes = mem.route_codes(T(inp["x"])).cpu().numpy().astype(np.int64)
            want = om.memory_forward(inp["h"], codes, p)   # same codes as the GPU router chose
            assert_fp32_close(wrapped.cpu().numpy(), want, what="LngramMemory forward")
            if np.array_equal(codes, g["codes"]):
                assert_fp32_close(wrapped.cpu().numpy(), g["output_wrapper"], what="LngramMemory vs reference")


def test_sb_slice_bf16(lngram, golden):
    """SB memory shape in bf16 (tcgen05 GEMMs + tensor-core gather/attention) vs the fp32 reference."""
    g = golden("memory_sb_slice")
    inp = cases.memory_inputs("sb_slice")
    mem = gpu_memory(lngram, "sb_slice", dtype=torch.bfloat16)
    with torch.no_grad():
        out = mem.module(T(inp["h"], torch.bfloat16), T(g["codes"].astype(np.int32))).float().cpu().numpy()
    assert_bf16_close(out, g["output"], what="bf16 forward vs fp32 reference")
    assert_bf16_close(out, g["output_bf16_module"], what="bf16 forward vs reference bf16 module")
    with torch.no_grad():
        tok = mem.module._lookup_route_chunk(T(g["codes"].astype(np.uint8)), None, 0, 184, None, None)
    np.testing.assert_allclose(tok.double().sum(-1).cpu().numpy(), g["token_sums"], rtol=1e-6, atol=1e-6)


# --------------------------------------------------------------------------- full-size properties
def _sb_tables(dtype=torch.bfloat16, rows=184 * 4096, dim=136, seed=2):
    gen = torch.Generator(device=DEV).manual_seed(seed)
    return (torch.randn(rows, dim, device=DEV, generator=gen) * 0.02).to(dtype)


def test_sb_full_size_lookup_rows_exact(lngram):
    """Full SB size (32 x 2048 x 184): gathered rows are exact copies of the addressed rows."""
    from oracle.build import load_c_oracle

    lib_c = load_c_oracle()
    B, Tn, R = 32, 2048, 184
    gen = torch.Generator(device=DEV).manual_seed(0)
    codes = torch.randint(0, 16, (B, Tn, R), device=DEV, dtype=torch.uint8, generator=gen)
    mem = lngram.RouteNgramMemoryV2(1024, num_routes=R, memory_dim=136, ngrams=(3,), readout_num_heads=16,
                                    readout_num_kv_heads=4, readout_head_dim=64, device=DEV, dtype=torch.bfloat16)
    with torch.no_grad():
        mem.tables["ngram_3"].weight.copy_(_sb_tables())
        tok = mem._lookup_route_chunk(codes, None, 0, R, None, None)
    ch = codes.cpu().numpy()
    rows = np.empty((B, Tn, R), np.int64)
    lib_c.oracle_row_indices(ch.ctypes.data, B, Tn, R, 3, 4, None, None, rows.ctypes.data)
    # sampled positions: tokens equal table[row] exactly, zero where invalid
    rng = np.random.default_rng(1)
    bs, ts = rng.integers(0, B, 256), np.concatenate([[0, 1, 2, 2047], rng.integers(0, Tn, 252)])
    table = mem.tables["ngram_3"].weight
    for b, t in zip(bs, ts):
        r = rows[b, t]
        got = tok[b, t]
        if r[0] < 0:
            assert torch.count_nonzero(got) == 0
        else:
            assert torch.equal(got, table[torch.from_numpy(r).to(DEV)])
    # a checksum of checksums over everything
    want_sum = table.double().sum(-1)[torch.from_numpy(np.maximum(rows, 0)).to(DEV)] * torch.from_numpy(rows >= 0).to(DEV)
    torch.testing.assert_close(tok.double().sum(-1), want_sum, rtol=0, atol=1e-9)


def test_sb_full_size_forward_matches_oracle_on_slices(lngram):
    """Full SB forward (bf16); sampled positions match the fp32 oracle run on their causal slices."""
    B, Tn, R, d = 32, 2048, 184, 1024
    mem = lngram.LngramMemory(d, {"routes": R, "mem_dim": 136, "kv_heads": 4, "q_heads": 16, "head_dim": 64,
                                  "ngrams": [3], "bits_per_route": 4}, norm_eps=1e-5, device=DEV,
                              dtype=torch.bfloat16).eval()
    p = cases.memory_params("sb_slice")
    state = {("router.weight" if k == "router.weight" else "module." + k): torch.from_numpy(v) for k, v in p.items()}
    mem.load_state_dict(state, strict=True)
    gen = torch.Generator(device=DEV).manual_seed(1)
    h = torch.randn(B, Tn, d, device=DEV, generator=gen).to(torch.bfloat16)
    hn = (h.float() * torch.rsqrt(h.float().pow(2).mean(-1, keepdim=True) + 1e-5)).to(torch.bfloat16)
    codes = torch.empty(B, Tn, R, device=DEV, dtype=torch.uint8)
    with torch.no_grad():
        out = mem(h, hn, codes_out=codes)
        out2 = mem(h, hn)
    assert torch.equal(out, out2), "forward must be deterministic"
    po = cases.oracle_params("sb_slice", p)
    hc, cc, oc = h.float().cpu().numpy(), codes.cpu().numpy().astype(np.int64), out.float().cpu().numpy()
    rng = np.random.default_rng(2)
    for b, t in zip(rng.integers(0, B, 6), np.concatenate([[0, 5], rng.integers(12, Tn, 4)])):
        s = max(0, t - 15)
        want = om.memory_forward(hc[b:b + 1, s:t + 1], cc[b:b + 1, s:t + 1], po)[0, -1]
        assert_bf16_close(oc[b, t], want, what=f"position ({b}, {t})")


def test_few_positions_match_the_full_batch(lngram):
    """A forward over few positions (the gather splits the routes over block rows and merges the slices;
    the GEMMs split K) gives the rows of the same sequences in a large batch (no splits) within bf16."""
    mem = gpu_memory(lngram, "sb_slice", torch.bfloat16)
    g = torch.Generator(device=DEV).manual_seed(21)
    B, T, d = 96, 16, 1024
    h = torch.randn(B, T, d, device=DEV, generator=g).to(torch.bfloat16)
    hn = lngram.rms_norm(h, torch.ones(d, device=DEV, dtype=torch.bfloat16), 1e-5)
    with torch.no_grad():
        codes = mem.route_codes(hn)                           # the same codes for both (rows identical)
        full = mem.module.forward_codes(h, codes).float()
        for b0, nb in ((0, 1), (5, 2), (40, 4)):               # 16, 32 and 64 positions
            few = mem.module.forward_codes(h[b0:b0 + nb].contiguous(), codes[b0:b0 + nb].contiguous()).float()
            assert_bf16_close(few.cpu().numpy(), full[b0:b0 + nb].cpu().numpy(), what=f"sequences {b0}..{b0 + nb}")


def test_out_of_range_codes_are_flagged_not_read(lngram):
    """A code >= 2^bits is caught by the kernel's own check: the window reads zeros and the
    device error word says so (no out-of-bounds access)."""
    mem = gpu_memory(lngram, "tiny").module
    codes = torch.zeros(1, 8, 8, dtype=torch.int32, device=DEV)
    codes[0, 5, 3] = 200
    with torch.no_grad():
        tok = mem._lookup_route_chunk(codes, None, 0, 8, None, None)
    assert lngram._lib.device_error(clear=True) == 1
    assert torch.count_nonzero(tok[0, 5:8, 3]) == 0
    assert torch.count_nonzero(tok[0, 4, 3]) > 0
