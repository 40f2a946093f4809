"""Pin the oracle to the reference itself (runs only where the reference checkout is present).

1. The reference's stored golden logits (``tests/data/wave1_reference.npz``, written by
   ``tests/test_wave1_unchanged.py`` in the reference) for ``w2_mem_super1`` -- the 24-layer model
   whose layer-1 memory is the SB memory (R = 184) -- are reproduced with THIS ORACLE substituted
   for that memory layer, at the reference's own cross-host tolerance (rtol 1e-4, atol 1e-5).
2. The reference C++ drafter (``oracle/_ref``, built from the reference source) agrees with the
   oracle drafter on the SD-B-shaped bundle, including the sketch shortlist.
"""

from __future__ import annotations

import numpy as np
import pytest

from oracle import memory as om
from oracle.drafter import OracleDrafter
from tests.golden import cases

pytestmark = pytest.mark.reference


def _oracle_params_from_module(m) -> om.MemoryParams:
    t = lambda x: x.detach().float().numpy()  # noqa: E731
    return om.MemoryParams(
        num_routes=m.num_routes, bits=m.bits_per_route, ngrams=tuple(m.ngrams), memory_dim=m.memory_dim,
        num_heads=m.readout_num_heads, num_kv_heads=m.readout_num_kv_heads, head_dim=m.readout_head_dim,
        eps=m.readout_query_norm.eps, tables={n: t(m.tables[f"ngram_{n}"].weight) for n in m.ngrams},
        q_norm=t(m.readout_query_norm.weight), mem_norm=t(m.readout_memory_norm.weight),
        q_proj=t(m.readout_q_proj.weight), kv_proj=t(m.readout_kv_proj.weight), o_proj=t(m.readout_o_proj.weight),
        conv_norm=t(m.short_conv.norm.weight), conv_weight=t(m.short_conv.conv.weight),
        conv_bias=None if m.short_conv.conv.bias is None else t(m.short_conv.conv.bias),
        conv_dilation=m.short_conv.dilation, sink_active_mass=m.sink_initial_active_mass)


@pytest.mark.slow
def test_wave1_golden_logits_with_oracle_memory(reference_path):
    import torch

    from ffnmem.config import load_config
    from ffnmem.model import Transformer

    data = np.load(reference_path / "tests" / "data" / "wave1_reference.npz")
    cfg = load_config(reference_path / "configs" / "w2_mem_super1.yaml", ["model.seq_len=64"])["model"]
    torch.manual_seed(0)
    model = Transformer(cfg)
    torch.manual_seed(1)
    for b in model.blocks:
        if b.memory is not None:
            torch.nn.init.normal_(b.memory.module.readout_o_proj.weight, std=0.02)
    model.eval()
    swapped = []
    for b in model.blocks:
        if b.memory is None:
            continue
        mem = b.memory
        p = _oracle_params_from_module(mem.module)
        w = mem.router.weight.detach().float().numpy()

        def forward(h, h_norm, router_in=None, _p=p, _w=w):
            out = om.lngram_memory_forward(h.detach().float().numpy(), h_norm.detach().float().numpy(), _w, _p)
            return torch.from_numpy(out).to(h.dtype)

        mem.forward = forward
        swapped.append(p.num_routes)
    assert swapped == [184]
    x = torch.randint(0, 32768, (1, 64), generator=torch.Generator().manual_seed(7))
    with torch.no_grad():
        got = model(x)[..., :256].numpy()
    np.testing.assert_allclose(got, data["w2_mem_super1"], rtol=1e-4, atol=1e-5)


def test_reference_cpp_drafter_agrees_with_oracle_shortlist(reference_path):
    from oracle.build import build_reference_drafter, load_reference_drafter

    build_reference_drafter(reference_path)
    ext = load_reference_drafter()
    if ext is None:
        pytest.skip("reference C++ drafter not built")
    import drafting.cpu_drafter as cd
    from drafting.export_drafter import Bundle

    cd._EXT = ext
    config, arrays = cases.draft_bundle("tiny")
    sk = cases.random_sketch(config, cap=16)
    config = dict(config, sketch_k=4, shortlist_cap=16)
    arrays = dict(arrays, **sk)
    toks = cases.draft_tokens("tiny", 80, seed=3)
    cpp = cd.CppDrafter(Bundle(config, arrays, {}), threads=2)
    ref = cd.RefDrafter(Bundle(config, arrays, {}))
    ora = OracleDrafter(config, arrays)
    c_ref, i_ref, l_ref = ref.trace(toks)
    c_o, i_o, l_o = ora.trace(toks)
    np.testing.assert_array_equal(c_o, c_ref)
    np.testing.assert_array_equal(i_o, i_ref)
    fin = np.isfinite(l_ref)
    np.testing.assert_array_equal(fin, np.isfinite(l_o))
    np.testing.assert_allclose(l_o[fin], l_ref[fin], rtol=1e-5, atol=1e-5)
    _, i_c, l_c = cpp.trace(toks, codes=c_ref)
    np.testing.assert_array_equal(i_c, i_o)
    np.testing.assert_allclose(l_c[fin], l_o[fin], atol=1e-4)
    for d in (cpp, ora):
        d.commit(toks[:30])
    a, b = cpp.draft(4, hyp=toks[30:33], last_codes=True), ora.draft(4, hyp=toks[30:33], last_codes=True)
    assert a.tokens == b.tokens
    np.testing.assert_array_equal(a.topk_ids, b.topk_ids)
    np.testing.assert_array_equal(a.codes, b.codes)


@pytest.mark.parametrize("sketch", [False, True])
def test_reference_drafters_agree_with_oracle_ssm(reference_path, sketch):
    """SD-C bundles (the SSM read by the router and the query), with and without a sketch shortlist:
    the reference's RefDrafter and its C++ drafter against the oracle drafter."""
    from oracle.build import build_reference_drafter, load_reference_drafter

    build_reference_drafter(reference_path)
    ext = load_reference_drafter()
    if ext is None:
        pytest.skip("reference C++ drafter not built")
    import drafting.cpu_drafter as cd
    from drafting.export_drafter import Bundle

    cd._EXT = ext
    config, arrays = cases.draft_bundle("tiny_ssm")
    if sketch:
        config = dict(config, sketch_k=4, shortlist_cap=16)
        arrays = dict(arrays, **cases.random_sketch(config, cap=16))
    toks = cases.draft_tokens("tiny_ssm", 60, seed=8)
    ref = cd.RefDrafter(Bundle(config, arrays, {}))
    cpp = cd.CppDrafter(Bundle(config, arrays, {}), threads=2)
    ora = OracleDrafter(config, arrays)
    c_ref, i_ref, l_ref = ref.trace(toks)
    c_o, i_o, l_o = ora.trace(toks)
    np.testing.assert_array_equal(c_o, c_ref)
    np.testing.assert_array_equal(i_o, i_ref)
    fin = np.isfinite(l_ref)
    np.testing.assert_array_equal(fin, np.isfinite(l_o))
    np.testing.assert_allclose(l_o[fin], l_ref[fin], rtol=1e-5, atol=1e-5)
    _, i_c, l_c = cpp.trace(toks, codes=c_ref)
    np.testing.assert_array_equal(i_c, i_o)
    np.testing.assert_allclose(l_c[fin], l_o[fin], atol=1e-4)
    for d in (cpp, ora):
        d.commit(toks[:25])
    a, b = cpp.draft(4, hyp=toks[25:28], last_codes=True), ora.draft(4, hyp=toks[25:28], last_codes=True)
    assert a.tokens == b.tokens
    np.testing.assert_array_equal(a.topk_ids, b.topk_ids)
    np.testing.assert_array_equal(a.codes, b.codes)
