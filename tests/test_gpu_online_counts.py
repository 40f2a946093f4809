"""The acceptance harness's online-count mixer on the GPU (``OnlineCounts``, ``lng_online_counts_mix``)
against the reference's outputs (fixtures written by running ``drafting/drafters.py:117-143``) and the
oracle restatement (pinned to the same fixtures).  Bar: bit-exact (the votes are integer counts and
the mix follows the reference's fp32 operation order)."""

from __future__ import annotations

import ctypes as C

import numpy as np
import pytest
import torch

from oracle.drafter import online_counts_mix
from tests.golden.make_golden import ONLINE_CASES

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda:0")


@pytest.fixture(autouse=True)
def _clear_device_error(lngram):
    lngram._lib.device_error(clear=True)
    yield
    assert lngram._lib.device_error(clear=True) == 0


def T(a):
    return torch.from_numpy(np.ascontiguousarray(a)).to(DEV)


def test_online_counts_match_reference(lngram, golden):
    g = golden("online_counts")
    for i, (orders, bits, kappa) in enumerate(ONLINE_CASES):
        oc = lngram.OnlineCounts(T(g[f"c{i}_codes"]), T(g[f"c{i}_x"]), orders, bits, int(g[f"c{i}_vocab"]), kappa)
        got = oc.mix(T(g[f"c{i}_p"]), T(g[f"c{i}_win"]), T(g[f"c{i}_real"]), T(g[f"c{i}_deadline"]))
        np.testing.assert_array_equal(got.cpu().numpy(), g[f"c{i}_mixed"])


@pytest.mark.parametrize("orders,bits", [((3,), 4), ((1, 2, 3), 2)])
def test_online_counts_sdb_scale_match_oracle(lngram, orders, bits):
    """An SD-B-sized case: 182 routes, a 700-token record with repeated stretches, 64 query windows,
    vocabulary 32,000."""
    rng = np.random.default_rng(8)
    Tn, R, V, N = 700, 182, 32000, 64
    W = max(orders)
    codes = rng.integers(0, 1 << bits, (Tn, R))
    x = rng.integers(0, V, Tn)
    for a, b in ((100, 300), (400, 120), (550, 301)):     # repeats so that pairs share rows
        codes[a:a + 60] = codes[b:b + 60]
        x[a:a + 60] = x[b:b + 60]
    last = rng.integers(0, Tn - 1, N)
    pos = last[:, None] - (W - 1) + np.arange(W)[None]
    real = pos >= 0
    win = codes[np.clip(pos, 0, None)] * real[..., None]
    p = rng.random((N, V)).astype(np.float32)
    p /= p.sum(-1, keepdims=True)
    deadline = last - 1
    want = online_counts_mix(codes, x, orders, bits, V, 0.7, p, win, real, deadline)
    oc = lngram.OnlineCounts(T(codes), T(x), orders, bits, V, 0.7)
    got = oc.mix(T(p), T(win), T(real), T(deadline)).cpu().numpy()
    np.testing.assert_array_equal(got, want)
    assert (np.abs(want - p).max(-1) > 0).sum() > N // 4         # most rows did mix


def test_online_counts_in_place_and_no_pairs(lngram, golden):
    """p and out may be one buffer; a record of one token (no verified pair) leaves p unchanged."""
    lib = lngram._lib
    g = golden("online_counts")
    orders, bits, kappa = ONLINE_CASES[0]
    p = T(g["c0_p"]).float().contiguous()
    codes, x, win = T(g["c0_codes"]), T(g["c0_x"]), T(g["c0_win"])
    real, deadline = T(g["c0_real"]).to(torch.uint8), T(g["c0_deadline"])
    arr = (C.c_int32 * len(orders))(*orders)
    lib.check(lib.library().lng_online_counts_mix(codes.data_ptr(), codes.shape[0], codes.shape[1], arr, len(orders),
                                                  bits, x.data_ptr(), win.data_ptr(), real.data_ptr(), p.shape[0],
                                                  win.shape[1], deadline.data_ptr(), p.data_ptr(), p.shape[1], kappa,
                                                  p.data_ptr(), lib.stream_ptr()))
    np.testing.assert_array_equal(p.cpu().numpy(), g["c0_mixed"])
    oc = lngram.OnlineCounts(codes[:1], x[:1], orders, bits, int(g["c0_vocab"]), kappa)
    p0 = T(g["c0_p"])
    assert torch.equal(oc.mix(p0, win, T(g["c0_real"]), deadline), p0)
