"""CPU checks of the C-ABI boundary: the library loads, exports every symbol that
``include/lngram_b200.h`` declares, the ctypes table matches the header, and the product path
refuses to run without a B200 (there is no CPU fallback)."""

from __future__ import annotations

import re
import subprocess
from pathlib import Path

import pytest
import torch

REPO = Path(__file__).resolve().parents[1]
HEADER = REPO / "include" / "lngram_b200.h"


def header_functions() -> set[str]:
    text = HEADER.read_text()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return set(re.findall(r"\b(lng_[a-z0-9_]+)\s*\(", text))


def test_header_declares_the_path():
    names = header_functions()
    for required in ("lng_quantize_route_logits", "lng_route_codes", "lng_lookup_route_chunk", "lng_route_attend",
                     "lng_memory_forward", "lng_fold_readout", "lng_gemm", "lng_logits_topk", "lng_drafter_create",
                     "lng_drafter_draft", "lng_drafter_trace", "lng_sink_gqa", "lng_conv_window"):
        assert required in names


def test_library_exports_every_declared_symbol(lngram):
    lib_path = lngram._lib.LIB_PATH
    if not lib_path.exists():
        pytest.skip("library not built (run __graft_entry__.build())")
    out = subprocess.run(["nm", "-D", "--defined-only", str(lib_path)], capture_output=True, text=True, check=True)
    exported = set(re.findall(r"\sT\s+(lng_\w+)", out.stdout))
    missing = header_functions() - exported
    assert not missing, f"declared but not exported: {sorted(missing)}"
    lib = lngram._lib.library(require_device=False)
    assert lib.lng_abi_version() == 1


def test_ctypes_table_matches_header(lngram):
    assert set(lngram._lib.SIGNATURES) == header_functions()


@pytest.mark.skipif(torch.cuda.is_available(), reason="checks the no-GPU refusal")
def test_no_cpu_fallback(lngram):
    if not lngram._lib.LIB_PATH.exists():
        pytest.skip("library not built")
    with pytest.raises(RuntimeError, match="CUDA"):
        lngram._lib.library(require_device=True)
    m = lngram.RouteNgramMemoryV2(64, num_routes=4, memory_dim=16, ngrams=(2, 3), readout_num_heads=4,
                                  readout_num_kv_heads=2, readout_head_dim=16).eval()
    with torch.no_grad(), pytest.raises(RuntimeError):
        m(torch.zeros(1, 4, 64), torch.zeros(1, 4, 4, dtype=torch.int32))


def test_reference_validation_errors(lngram):
    """Constructor errors mirror the reference's ValueErrors (lngram_v2.py:878-933)."""
    with pytest.raises(ValueError):
        lngram.RouteNgramMemoryV2(64, bits_per_route=17)
    with pytest.raises(ValueError):
        lngram.RouteNgramMemoryV2(64, readout_num_heads=3, readout_num_kv_heads=2, readout_head_dim=16)
    with pytest.raises(ValueError):
        lngram.RouteNgramMemoryV2(64, readout_num_heads=4, readout_num_kv_heads=2, readout_head_dim=8)
    m = lngram.RouteNgramMemoryV2(64, num_routes=4, memory_dim=16, ngrams=(3, 2, 3), readout_num_heads=4,
                                  readout_num_kv_heads=2, readout_head_dim=16)
    assert m.ngrams == (2, 3) and m.route_token_dim == 32
    assert abs(m.readout_sink_logit - __import__("math").log(4)) < 1e-12
    with pytest.raises(ValueError):
        m(torch.zeros(1, 4, 32), torch.zeros(1, 4, 4))


def test_state_dict_names_match_reference_module(lngram):
    """A reference state_dict loads unchanged: same parameter names and shapes."""
    m = lngram.RouteNgramMemoryV2(64, num_routes=4, memory_dim=16, ngrams=(2, 3), readout_num_heads=4,
                                  readout_num_kv_heads=2, readout_head_dim=16)
    from tests.golden import cases

    names = set(cases.memory_params("tiny_multi")) - {"router.weight"}
    assert set(m.state_dict()) == names
    for k, v in cases.memory_params("tiny_multi").items():
        if k in m.state_dict():
            assert tuple(m.state_dict()[k].shape) == v.shape, k
