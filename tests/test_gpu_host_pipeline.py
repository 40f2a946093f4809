"""The block RMSNorm that makes the router input (a1, ``ffnmem/model.py:39-48``) and the host-memory
pipelined forward (``LngramMemory.forward_host``).

* ``rms_norm`` rounds the normalised row to x's dtype BEFORE multiplying by the weight, and returns the
  promoted dtype, as the reference's ``xf.type_as(x) * self.weight`` does: checked element-wise
  against that torch expression (bf16 x with an fp32 weight, bf16 x with a bf16 weight, fp32 x),
  exact except for a last-place difference where the row's 1/rms rounds differently.
* ``forward_host`` equals the device forward of the same sequence groups bit for bit, both when the
  router input is copied in and when it is made on the device by ``rms_norm``.
"""

from __future__ import annotations

import pytest
import torch

from tests.golden import cases

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda:0")


def _reference_norm(x: torch.Tensor, w: torch.Tensor, eps: float) -> torch.Tensor:
    """The reference RMSNorm.forward (``ffnmem/model.py:45-48``), evaluated by torch on the CPU."""
    xf = x.float()
    xf = xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + eps)
    return xf.type_as(x) * w


@pytest.mark.parametrize("xdt,wdt", [(torch.bfloat16, torch.float32), (torch.bfloat16, torch.bfloat16),
                                     (torch.float32, torch.float32)])
@pytest.mark.parametrize("d", [1024, 200])
def test_rms_norm_rounds_before_the_weight(lngram, xdt, wdt, d):
    g = torch.Generator().manual_seed(d)
    x = (torch.randn(257, d, generator=g) * 3.0).to(xdt)
    w = (1.0 + 0.3 * torch.randn(d, generator=g)).to(wdt)
    want = _reference_norm(x, w, 1e-5)
    got = lngram.rms_norm(x.to(DEV), w.to(DEV), 1e-5).cpu()
    assert got.dtype == want.dtype == torch.promote_types(xdt, wdt)
    if xdt == torch.bfloat16:
        # the bf16 rounding of the normalised row absorbs the last-bit differences of 1/rms (the sum
        # order of the mean differs from torch's), so nearly every element is bit-identical
        exact = (got == want).float().mean().item()
        assert exact >= 0.99, exact
    # elsewhere off by at most one unit in the last place of the intermediate (x's dtype) rounding,
    # plus a few fp32 units for 1/rms
    ulp = (torch.finfo(xdt).eps + 4 * torch.finfo(torch.float32).eps) * want.float().abs()
    assert ((got.float() - want.float()).abs() <= 1.01 * ulp).all()
    if xdt == torch.bfloat16 and wdt == torch.float32:
        # the rule matters: without the intermediate rounding most values differ
        nocast = x.float() * torch.rsqrt(x.float().pow(2).mean(-1, keepdim=True) + 1e-5) * w
        assert (got == nocast).float().mean().item() < 0.5


def _sb_memory(lngram):
    c = cases.MEMORY_CASES["sb_slice"]
    mem = lngram.LngramMemory(c["d"], {"routes": c["routes"], "mem_dim": c["mem_dim"], "kv_heads": c["kv_heads"],
                                       "q_heads": c["q_heads"], "head_dim": c["head_dim"], "ngrams": list(c["ngrams"]),
                                       "bits_per_route": c["bits"]}, norm_eps=1e-5, device=DEV,
                              dtype=torch.bfloat16).eval()
    p = cases.memory_params("sb_slice")
    state = {("router.weight" if k == "router.weight" else "module." + k): torch.from_numpy(v) for k, v in p.items()}
    mem.load_state_dict(state, strict=True)
    return mem


@pytest.mark.parametrize("groups", [1, 4, 3])
def test_forward_host_equals_device_forward(lngram, groups):
    mem = _sb_memory(lngram)
    B, T, d = 12, 256, 1024
    g = torch.Generator(device=DEV).manual_seed(9)
    h = torch.randn(B, T, d, device=DEV, generator=g).to(torch.bfloat16)
    w = (1.0 + 0.1 * torch.randn(d, device=DEV, generator=g)).to(torch.bfloat16)
    hn = lngram.rms_norm(h, w, 1e-5)
    Bg = B // groups
    with torch.no_grad():
        want = torch.cat([mem(h[i:i + Bg], hn[i:i + Bg]) for i in range(0, B, Bg)]).cpu()
        h_host, hn_host = h.cpu().pin_memory(), hn.cpu().pin_memory()
        got_copied = mem.forward_host(h_host, hn_host, groups=groups)
        got_made = mem.forward_host(h_host, norm_weight=w, norm_eps=1e-5, groups=groups)
        out = torch.empty(B, T, d, dtype=torch.bfloat16).pin_memory()
        mem.forward_host(h_host, norm_weight=w, out=out, groups=groups, synchronize=False)
        h2 = torch.randn(B, T, d, generator=torch.Generator().manual_seed(5)).to(torch.bfloat16).pin_memory()
        out2 = torch.empty(B, T, d, dtype=torch.bfloat16).pin_memory()
        mem.forward_host(h2, norm_weight=w, out=out2, groups=groups, synchronize=False)   # overlaps the first
        mem.wait_host()
        torch.cuda.current_stream().synchronize()
        h2d = h2.to(DEV)
        want2 = torch.cat([mem(h2d[i:i + Bg], lngram.rms_norm(h2d[i:i + Bg], w, 1e-5)) for i in range(0, B, Bg)]).cpu()
    assert torch.equal(out2, want2)
    assert not got_copied.is_cuda
    assert torch.equal(got_copied, want)
    assert torch.equal(got_made, want)
    assert torch.equal(out, want)


def test_forward_host_rejects_ambiguous_router_input(lngram):
    mem = _sb_memory(lngram)
    h = torch.zeros(2, 8, 1024, dtype=torch.bfloat16)
    with pytest.raises(ValueError):
        mem.forward_host(h)
    with pytest.raises(ValueError):
        mem.forward_host(h, h, norm_weight=torch.ones(1024))
