"""Draft logits + fused top-k (lng_logits_topk) against a plain fp32 torch reference.

Ids are exact (ties resolved to the lower id, the reference's order: drafting/cpu/drafter.cpp:547-556);
values within fp32 rounding of h . E[v]."""

from __future__ import annotations

import pytest
import torch

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda:0")


def topk_ref(h, E, k):
    logits = h.double() @ E.double().T
    # (value desc, id asc): stable sort on the negated values keeps ascending ids among ties
    order = torch.sort(-logits, dim=1, stable=True).indices[:, :k]
    return order, logits.gather(1, order).float(), logits.float()


def run_topk(lngram, h, E, k, want_logits=False):
    lib = lngram._lib
    L = lib.library()
    n, d = h.shape
    V = E.shape[0]
    ids = torch.empty(n, k, device=DEV, dtype=torch.int64)
    vals = torch.empty(n, k, device=DEV, dtype=torch.float32)
    logits = torch.empty(n, V, device=DEV, dtype=torch.float32) if want_logits else None
    need = L.lng_logits_topk_scratch_bytes(n, d, V, k)
    scratch = torch.empty(need, device=DEV, dtype=torch.uint8)
    lib.check(L.lng_logits_topk(h.data_ptr(), n, d, E.data_ptr(), lib.dtype_code(E.dtype), V, k, ids.data_ptr(),
                                vals.data_ptr(), None if logits is None else logits.data_ptr(), scratch.data_ptr(),
                                need, lib.stream_ptr()))
    return ids, vals, logits


@pytest.mark.parametrize("n,d,V,k", [(1, 64, 256, 3), (7, 128, 1000, 8), (64, 1024, 32000, 3), (65, 1024, 32000, 1),
                                     (33, 192, 515, 2), (300, 256, 3000, 5)])
@pytest.mark.parametrize("edt", [torch.float32, torch.bfloat16])
def test_logits_topk_matches_fp32_reference(lngram, n, d, V, k, edt):
    g = torch.Generator(device=DEV).manual_seed(n * 31 + V)
    h = torch.randn(n, d, device=DEV, generator=g)
    E = (torch.randn(V, d, device=DEV, generator=g) * 0.02).to(edt)
    ids, vals, logits = run_topk(lngram, h, E, k, want_logits=True)
    want_ids, want_vals, want_logits = topk_ref(h, E.float(), k)
    scale = want_logits.abs().max().item()
    torch.testing.assert_close(logits, want_logits, rtol=1e-5, atol=1e-5 * scale)
    torch.testing.assert_close(vals, want_vals, rtol=1e-5, atol=1e-5 * scale)
    # ids may differ from the float64 order only where two logits are within fp32 rounding
    gap = (want_logits.gather(1, ids) - want_vals).abs().max().item()
    assert gap <= 2e-5 * scale
    assert (ids == want_ids).float().mean().item() > 0.99


@pytest.mark.parametrize("d,edt", [(32, torch.float32), (64, torch.bfloat16)])
def test_logits_topk_ties_prefer_lower_id(lngram, d, edt):
    """Exact ties (CUDA-core kernel for fp32, tensor-core kernel for a bf16 vocabulary)."""
    h = torch.ones(2, d, device=DEV)
    E = torch.zeros(600, d, device=DEV, dtype=edt)
    E[[5, 17, 300, 599]] = 1.0          # four exact ties at the top
    E[[2, 400]] = 0.5
    ids, vals, _ = run_topk(lngram, h, E, 6)
    assert ids[0].tolist() == [5, 17, 300, 599, 2, 400]
    assert vals[0, :4].tolist() == [float(d)] * 4
    # fewer than k candidates: -1 / -inf padding, as the reference pads
    ids, vals, _ = run_topk(lngram, h, E[:3], 5)
    assert ids[0].tolist() == [2, 0, 1, -1, -1]
    assert vals[0, 3].item() == float("-inf")
