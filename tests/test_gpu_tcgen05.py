"""tcgen05 GEMM (TMA + TMEM) and the bf16x3 tensor-core router against a plain fp32 torch reference."""

from __future__ import annotations

import numpy as np
import pytest
import torch

from tests.helpers import code_mismatch_ok

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda:0")


@pytest.fixture(autouse=True)
def _clear_device_error(lngram):
    lngram._lib.device_error(clear=True)
    yield
    assert lngram._lib.device_error(clear=True) == 0, "a kernel recorded a device-side error"


def gemm(lngram, a, b, out_dtype, rowscale=None):
    lib = lngram._lib
    m, k = a.shape
    n = b.shape[0]
    c = torch.empty(m, n, device=DEV, dtype=out_dtype)
    lib.check(lib.library().lng_gemm(a.data_ptr(), lib.BF16, a.stride(0), b.data_ptr(), lib.BF16, b.stride(0),
                                     c.data_ptr(), lib.dtype_code(out_dtype), c.stride(0), m, n, k,
                                     None if rowscale is None else rowscale.data_ptr(), 0, lib.stream_ptr()))
    return c


@pytest.mark.parametrize("m,n,k", [(128, 256, 64), (256, 128, 1024), (65536 // 16, 2176, 1024), (300, 1024, 2176),
                                   (129, 136, 72), (1, 16, 16), (777, 520, 200),
                                   # few rows: K split over CTAs, fp32 partials summed by a second kernel
                                   (64, 2176, 1024), (64, 1024, 2176), (1, 2176, 1024), (100, 1000, 512),
                                   # two-SM (cta_group::2) form: 256-row pair tiles, ragged rows / columns
                                   (8192 + 77, 2176, 1024), (8704, 1024, 2176), (9000, 100, 64)])
@pytest.mark.parametrize("out_dtype", [torch.float32, torch.bfloat16])
def test_tc_gemm_matches_fp32_reference(lngram, m, n, k, out_dtype):
    g = torch.Generator(device=DEV).manual_seed(m * 7 + n)
    a = torch.randn(m, k, device=DEV, generator=g).to(torch.bfloat16)
    b = torch.randn(n, k, device=DEV, generator=g).to(torch.bfloat16)
    want = a.float() @ b.float().T
    got = gemm(lngram, a, b, out_dtype).float()
    tol = 1e-5 if out_dtype == torch.float32 else 1e-2
    err = (got - want).abs().max().item()
    assert err <= tol * want.abs().max().item() + 1e-6, (m, n, k, err)


def test_tc_gemm_split_k_rowscale_and_output_stride(lngram):
    """The few-rows form (K split over CTAs) with a row scale and an output row stride above N."""
    lib = lngram._lib
    g = torch.Generator(device=DEV).manual_seed(4)
    m, n, k = 64, 2176, 1024
    a = torch.randn(m, k, device=DEV, generator=g).to(torch.bfloat16)
    b = torch.randn(n, k, device=DEV, generator=g).to(torch.bfloat16)
    rs = torch.rand(m, device=DEV, generator=g) + 0.5
    for out_dtype in (torch.float32, torch.bfloat16):
        c = torch.full((m, n + 64), 7.0, device=DEV, dtype=out_dtype)
        lib.check(lib.library().lng_gemm(a.data_ptr(), lib.BF16, k, b.data_ptr(), lib.BF16, k, c.data_ptr(),
                                         lib.dtype_code(out_dtype), n + 64, m, n, k, rs.data_ptr(), 0,
                                         lib.stream_ptr()))
        want = (a.float() @ b.float().T) * rs[:, None]
        tol = 1e-5 if out_dtype == torch.float32 else 1e-2
        assert (c[:, :n].float() - want).abs().max().item() <= tol * want.abs().max().item()
        assert torch.all(c[:, n:] == 7.0)                    # the row padding is not written


def test_tc_gemm_rowscale_and_strided_operands(lngram):
    g = torch.Generator(device=DEV).manual_seed(3)
    big = torch.randn(512, 1088, device=DEV, generator=g).to(torch.bfloat16)
    a = big[:, :1024]                     # row stride 1088 (multiple of 8)
    b = torch.randn(384, 1024, device=DEV, generator=g).to(torch.bfloat16)
    rs = torch.rand(512, device=DEV, generator=g) + 0.5
    got = gemm(lngram, a, b, torch.float32, rowscale=rs)
    want = (a.float() @ b.float().T) * rs[:, None]
    torch.testing.assert_close(got, want, rtol=1e-5, atol=1e-5 * want.abs().max().item())


@pytest.mark.parametrize("bits,routes,in_dim,n", [(4, 184, 1024, 4099), (5, 184, 1024, 4099), (4, 182, 2048, 4099),
                                                  (4, 8, 128, 4099), (3, 40, 64, 4099),
                                                  # two-SM form (from 8192 rows)
                                                  (4, 184, 1024, 8192 + 5), (5, 184, 1024, 8192 + 300),
                                                  (3, 40, 64, 8192 + 1)])
def test_tc_router_codes_fp32_accurate(lngram, bits, routes, in_dim, n):
    """bf16 inputs x fp32 router weight through the bf16x3 split: codes agree with the fp32 sign
    everywhere the fp32 logit is not within 1e-5 of zero."""
    lib = lngram._lib
    g = torch.Generator(device=DEV).manual_seed(bits * 1000 + routes)
    x = torch.randn(n, in_dim, device=DEV, generator=g).to(torch.bfloat16)
    w = torch.randn(routes * bits, in_dim, device=DEV, generator=g) * 0.02
    split = torch.empty(routes * bits, 3 * in_dim, device=DEV, dtype=torch.bfloat16)
    lib.check(lib.library().lng_router_prepare(w.data_ptr(), routes * bits, in_dim, split.data_ptr(), lib.stream_ptr()))
    recon = split.float().view(routes * bits, 3, in_dim).sum(1)
    assert torch.equal(recon, w), "W1 + W2 + W3 must reproduce the fp32 weight exactly"
    codes = torch.empty(n, routes, device=DEV, dtype=torch.uint8)
    lib.check(lib.library().lng_route_codes_split(x.data_ptr(), n, in_dim, in_dim, split.data_ptr(), routes, bits,
                                                  codes.data_ptr(), lib.stream_ptr()))
    logits = (x.double() @ w.double().T).cpu().numpy()
    want = np.zeros((n, routes), np.int64)
    for j in range(bits):
        want |= (logits[:, j::bits] > 0).astype(np.int64) << j
    frac = code_mismatch_ok(codes.cpu().numpy(), want, logits, bits, tau=1e-5)
    assert frac < 1e-4
