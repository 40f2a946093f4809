"""The allocation-free top-k entry point (lng_logits_topk_static) against lng_logits_topk.

Some callers of the draft head cannot allocate device memory at the point where they draft -- code
replayed inside a CUDA graph, or a serving process whose allocator only hands out its own pools --
so the library offers a variant whose scratch lives in a fixed 4 MiB array inside the library.  This
file checks, through the C ABI, that two calls in a row give exactly what the buffer-taking entry
point gives, and that sizes beyond the array are refused with a clear error.  It is collected last
(file name).
"""

from __future__ import annotations

import pytest
import torch

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda:0")


def _with_buffer(lib, h, E, k):
    L = lib.library()
    n, d = h.shape
    V = E.shape[0]
    ids = torch.empty(n, k, device=DEV, dtype=torch.int64)
    vals = torch.empty(n, k, device=DEV, dtype=torch.float32)
    need = L.lng_logits_topk_scratch_bytes(n, d, V, k)
    scratch = torch.empty(need, device=DEV, dtype=torch.uint8)
    lib.check(L.lng_logits_topk(h.data_ptr(), n, d, E.data_ptr(), lib.dtype_code(E.dtype), V, k, ids.data_ptr(),
                                vals.data_ptr(), None, scratch.data_ptr(), need, lib.stream_ptr()))
    return ids, vals


def _static(lib, h, E, k):
    L = lib.library()
    n, d = h.shape
    V = E.shape[0]
    ids = torch.empty(n, k, device=DEV, dtype=torch.int64)
    vals = torch.empty(n, k, device=DEV, dtype=torch.float32)
    lib.check(L.lng_logits_topk_static(h.data_ptr(), n, d, E.data_ptr(), lib.dtype_code(E.dtype), V, k,
                                       ids.data_ptr(), vals.data_ptr(), None, lib.stream_ptr()))
    return ids, vals


def test_static_scratch_topk_matches_buffer_entry_point_twice(lngram):
    lib = lngram._lib
    g = torch.Generator(device=DEV).manual_seed(11)
    E = (torch.randn(32000, 1024, device=DEV, generator=g) * 0.02).to(torch.bfloat16)
    # two calls in a row with different inputs and shapes: the shared array keeps the first call's
    # contents, which must not leak into the second
    for n, k in ((64, 3), (17, 8)):
        h = torch.randn(n, 1024, device=DEV, generator=g)
        got_ids, got_vals = _static(lib, h, E, k)
        want_ids, want_vals = _with_buffer(lib, h, E, k)
        torch.cuda.synchronize()
        assert torch.equal(got_ids, want_ids)
        torch.testing.assert_close(got_vals, want_vals, rtol=1e-5, atol=1e-5 * want_vals.abs().max().item())


def test_static_scratch_rejects_oversized_requests(lngram):
    lib = lngram._lib
    L = lib.library()
    h = torch.zeros(933, 64, device=DEV)
    E = torch.zeros(32000, 64, device=DEV)
    ids = torch.empty(933, 3, device=DEV, dtype=torch.int64)
    vals = torch.empty(933, 3, device=DEV, dtype=torch.float32)
    st = L.lng_logits_topk_static(h.data_ptr(), 933, 64, E.data_ptr(), lib.F32, 32000, 3, ids.data_ptr(),
                                  vals.data_ptr(), None, lib.stream_ptr())
    assert st == lib.ERR_ARGUMENT
    assert b"exceeds the 4 MiB static scratch" in L.lng_last_error()
    # the largest size that fits is accepted
    lib.check(L.lng_logits_topk_static(h.data_ptr(), 932, 64, E.data_ptr(), lib.F32, 32000, 3, ids.data_ptr(),
                                       vals.data_ptr(), None, lib.stream_ptr()))
    torch.cuda.synchronize()


def test_static_scratch_tensor_core_limit_includes_split_rows(lngram):
    """A bf16 vocabulary at d = 1024 takes the tensor-core path, whose split rows share the array:
    394 rows fit at k = 3, V = 32000, 395 do not."""
    lib = lngram._lib
    L = lib.library()
    h = torch.zeros(395, 1024, device=DEV)
    E = torch.zeros(32000, 1024, device=DEV, dtype=torch.bfloat16)
    ids = torch.empty(395, 3, device=DEV, dtype=torch.int64)
    vals = torch.empty(395, 3, device=DEV, dtype=torch.float32)
    st = L.lng_logits_topk_static(h.data_ptr(), 395, 1024, E.data_ptr(), lib.BF16, 32000, 3, ids.data_ptr(),
                                  vals.data_ptr(), None, lib.stream_ptr())
    assert st == lib.ERR_ARGUMENT
    assert b"split rows" in L.lng_last_error()
    lib.check(L.lng_logits_topk_static(h.data_ptr(), 394, 1024, E.data_ptr(), lib.BF16, 32000, 3, ids.data_ptr(),
                                       vals.data_ptr(), None, lib.stream_ptr()))
    torch.cuda.synchronize()
