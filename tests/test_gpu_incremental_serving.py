"""The decode / verify seam's remaining parts on the GPU, against the reference's own outputs.

* ``RouteNgramMemoryV2.forward_incremental`` (``lngram_v2.py:1763-1829``): outputs of a prefill, single
  steps and a chunk match the reference's, and the packed n-gram suffix after every call is bit-exact
  (fixtures written by running the reference, ``tests/golden/make_golden.py``).
* ``memory_step(..., route_tokens=)`` (``ffnmem/infer.py:152-182``): the rows a row provider supplies give
  the table path's output; ``decode_memory_step`` with a provider (``infer.py:207-251``).
* The serving layout and the zero-copy row provider (``serving/layout.py``, ``serving/prefetch.py:579-586``):
  the permuted tables equal the reference's, and rows read from mapped host memory equal the v2 lookup.

Bars: integer state and gathered rows bit-exact; fp32 outputs within 1e-5; bf16 within 1e-2.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle import memory as om
from tests.golden import cases
from tests.golden.make_golden import INCREMENTAL_CALLS
from tests.helpers import assert_bf16_close, assert_fp32_close
from tests.test_gpu_memory import gpu_memory

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda:0")


def T(a, dt=None):
    t = torch.from_numpy(np.ascontiguousarray(a)).to(DEV)
    return t if dt is None else t.to(dt)


@pytest.fixture(autouse=True)
def _clear_device_error(lngram):
    lngram._lib.device_error(clear=True)
    yield
    assert lngram._lib.device_error(clear=True) == 0


# --------------------------------------------------------------------------- forward_incremental
@pytest.mark.parametrize("case", ["tiny_multi", "scaled_slice"])
def test_forward_incremental_matches_reference(lngram, golden, case):
    g = golden(f"incremental_{case}")
    m = gpu_memory(lngram, case).module
    h, codes = T(g["in_h"]), T(g["codes"])
    outs, state, t0 = [], None, 0
    for i, n in enumerate(INCREMENTAL_CALLS):
        y, state = m.forward_incremental(h[:, t0:t0 + n], codes[:, t0:t0 + n], state)
        outs.append(y.cpu().numpy())
        np.testing.assert_array_equal(state.packed_route_state.cpu().numpy(), g[f"packed_{i}"])
        assert state.route_state_length == int(g[f"length_{i}"])
        t0 += n
    out = np.concatenate(outs, 1)
    assert_fp32_close(out, g["outputs"], what="incremental outputs vs the reference's")
    assert_fp32_close(out, g["full"], what="incremental outputs vs the full forward")
    np.testing.assert_array_equal(state.route_history.cpu().numpy(), g["route_history"])
    assert_fp32_close(state.conv_history.cpu().numpy(), g["conv_history"], what="conv history")
    # beam reordering
    sel = state.index_select(torch.tensor([1, 0]))
    assert torch.equal(sel.packed_route_state[0], state.packed_route_state[1])


def test_forward_incremental_bf16_sb_matches_oracle(lngram):
    mem = gpu_memory(lngram, "sb_slice", torch.bfloat16)
    m = mem.module
    inp = cases.memory_inputs("sb_slice")
    p = cases.memory_params("sb_slice")
    codes = om.quantize_route_logits(om.route_logits(inp["x"], p["router.weight"]), 4)
    h, cd = T(inp["h"], torch.bfloat16), T(codes.astype(np.uint8))
    outs, state, t0 = [], None, 0
    for n in (16, 1, 1, 1, 8, 1, 1):
        y, state = m.forward_incremental(h[:, t0:t0 + n], cd[:, t0:t0 + n], state)
        outs.append(y.float().cpu().numpy())
        t0 += n
    want = om.memory_forward(inp["h"][:, :t0], codes[:, :t0], cases.oracle_params("sb_slice", p))
    assert_bf16_close(np.concatenate(outs, 1), want, what="bf16 incremental vs the fp32 oracle")


def test_forward_incremental_rejects_training_and_bad_codes(lngram):
    m = gpu_memory(lngram, "tiny_multi").module
    h = torch.zeros(1, 2, 64, device=DEV)
    with pytest.raises(ValueError):
        m.forward_incremental(h, torch.zeros(1, 3, 4, dtype=torch.uint8, device=DEV))
    m.train()
    with pytest.raises(RuntimeError):
        m.forward_incremental(h, torch.zeros(1, 2, 4, dtype=torch.uint8, device=DEV))
    m.eval()


# --------------------------------------------------------------------------- route tokens from a provider
def _cache(lngram, m, g, max_len=64):
    B, L = g["h_prefix"].shape[:2]
    c = lngram.MemoryCache(m, B, max_len)
    c.codes[:, :L] = T(g["codes_prefix"]).to(torch.uint8)
    c.conv_in[:, :L] = T(g["conv_cache"])
    c.length = L
    return c


def test_memory_step_with_supplied_rows_equals_table_path(lngram, golden):
    g = golden("seams_tiny_multi")
    m = gpu_memory(lngram, "tiny_multi").module
    c1, c2 = _cache(lngram, m, g), _cache(lngram, m, g)
    L, n = c1.length, g["codes_new"].shape[1]
    hist = m.route_history_length
    ctx = torch.cat((c1.codes[:, L - hist:L], T(g["codes_new"]).to(torch.uint8)), 1)
    rows = m._lookup_route_chunk(ctx, None, 0, m.num_routes, None, None, target_length=n)
    want = lngram.memory_step(m, c1, T(g["h_new"]), T(g["codes_new"])).cpu().numpy()
    got = lngram.memory_step(m, c2, T(g["h_new"]), T(g["codes_new"]), route_tokens=rows).cpu().numpy()
    assert_fp32_close(got, want, what="memory_step with supplied rows")
    assert_fp32_close(got, g["step_output"], what="memory_step with supplied rows vs the reference")
    assert torch.equal(c1.conv_in, c2.conv_in) or np.allclose(c1.conv_in.cpu().numpy(), c2.conv_in.cpu().numpy(),
                                                              rtol=1e-5, atol=1e-6)


# --------------------------------------------------------------------------- serving layout / zero copy
def test_serving_permutation_matches_reference(lngram, golden):
    g = golden("serving_tiny_multi")
    m = gpu_memory(lngram, "tiny_multi").module
    tabs = lngram.serving.permute_tables(m)
    for n, t in tabs.items():
        np.testing.assert_array_equal(t[T(g[f"rows_idx_{n}"])].cpu().numpy(), g[f"rows_{n}"])
    host = m.tables["ngram_3"].weight.detach().cpu().pin_memory()    # pinned host in, pinned host out
    ph = lngram.serving.permute_table(host, m.num_routes, 3, m.bits_per_route)
    assert not ph.is_cuda and torch.equal(ph, tabs[3].cpu())


@pytest.mark.parametrize("case,dt", [("tiny_multi", torch.float32), ("sb_slice", torch.bfloat16)])
def test_zero_copy_rows_equal_v2_lookup(lngram, golden, case, dt):
    m = gpu_memory(lngram, case, dt).module
    ht = lngram.serving.HostTable.from_module(m)
    assert all(not t.is_cuda and t.is_pinned() for t in ht.tables.values())
    prov = lngram.serving.ZeroCopyGather(ht)
    B, L, n, R = 3, 12, 4, m.num_routes
    gen = torch.Generator(device=DEV).manual_seed(3)
    for L in (0, 1, 12):
        cache = lngram.MemoryCache(m, B, 32)
        cache.codes[:, :L] = torch.randint(0, 16, (B, L, R), device=DEV, generator=gen, dtype=torch.uint8)
        cache.length = L
        new = torch.randint(0, 16, (B, n, R), device=DEV, generator=gen, dtype=torch.uint8)
        rows = prov(0, cache, new)
        hist = m.route_history_length
        ctx = torch.cat((cache.codes[:, max(0, L - hist):L], new), 1)
        want = m._lookup_route_chunk(ctx, None, 0, R, None, None, target_length=n)
        assert torch.equal(rows, want), L
    if case == "tiny_multi":
        g = golden("serving_tiny_multi")
        cache = lngram.MemoryCache(m, 3, 64)
        cache.length = 0
        rows = prov(0, cache, T(g["codes"]))
        np.testing.assert_array_equal(rows.cpu().numpy(), g["tokens"])


def test_decode_step_with_zero_copy_provider(lngram):
    mem = gpu_memory(lngram, "sb_slice", torch.bfloat16)
    m = mem.module
    prov = lngram.serving.ZeroCopyGather({1: lngram.serving.HostTable.from_module(m)})
    inp = cases.memory_inputs("sb_slice")
    h, x = T(inp["h"], torch.bfloat16), T(inp["x"], torch.bfloat16)
    c_tab, c_host = lngram.MemoryCache(m, 1, 64), lngram.MemoryCache(m, 1, 64)
    for t0, n in ((0, 8), (8, 1), (9, 1), (10, 3)):
        a = lngram.decode_memory_step(mem, c_tab, h[:, t0:t0 + n], x[:, t0:t0 + n])
        b = lngram.decode_memory_step(mem, c_host, h[:, t0:t0 + n], x[:, t0:t0 + n], row_provider=prov, pos=1)
        assert_bf16_close(b.float().cpu().numpy(), a.float().cpu().numpy(), what=f"decode step at {t0}")
        c_tab.length += n
        c_host.length += n
    assert prov.rows_read == 13 * 184
