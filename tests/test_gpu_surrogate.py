"""The training-mode lookup on the GPU (``RouteNgramMemoryV2._lookup_route_chunk`` with gradients): the
route-logit gradient of the q surrogate (``lngram_v2.py:326-447``, approximate and exact modes) and the
tables' row gradient match the reference's autograd (fixture written by running the reference,
``tests/golden/make_golden.py``), with route chunks, packed segments and padding masks."""

from __future__ import annotations

import numpy as np
import pytest
import torch

from tests.golden import cases
from tests.golden.make_golden import SURROGATE_CASES
from tests.helpers import assert_fp32_close
from tests.test_gpu_memory import gpu_memory

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda:0")


@pytest.mark.parametrize("i", range(len(SURROGATE_CASES)))
def test_training_lookup_backward_matches_reference(lngram, golden, i):
    case, mode, rs, re = SURROGATE_CASES[i]
    g = golden("surrogate_backward")
    mem = gpu_memory(lngram, case)
    m = mem.module
    m.q_surrogate_mode, m.q_surrogate_temperature, m.q_surrogate_scale = mode, 0.7, 1.3
    m.train()
    inp = cases.memory_inputs(case)
    seg = None if "segment_ids" not in inp else torch.from_numpy(inp["segment_ids"]).to(DEV)
    val = None if "valid_tokens" not in inp else torch.from_numpy(inp["valid_tokens"]).to(DEV)
    codes = torch.from_numpy(g[f"c{i}_codes"]).to(DEV)
    q = torch.from_numpy(g[f"c{i}_q"]).to(DEV).requires_grad_(True)
    for t in m.tables.values():
        t.weight.grad = None
    tok = m._lookup_route_chunk(codes, q, rs, re, seg, val)
    (tok * torch.from_numpy(g[f"c{i}_grad_tokens"]).to(DEV)).sum().backward()
    m.eval()
    assert_fp32_close(q.grad.cpu().numpy(), g[f"c{i}_grad_q"], rtol=1e-4, what="surrogate grad_q")
    c = cases.MEMORY_CASES[case]
    for n in c["ngrams"]:
        gw = m.tables[f"ngram_{n}"].weight.grad.cpu().numpy()
        rows = g[f"c{i}_rows_{n}"]
        assert_fp32_close(gw[rows], g[f"c{i}_grad_table_{n}"], what=f"table {n} row gradient")
        other = np.ones(gw.shape[0], bool)
        other[rows] = False
        assert not gw[other].any()


def test_surrogate_off_leaves_q_without_gradient_and_cache_is_rejected(lngram):
    m = gpu_memory(lngram, "tiny_multi").module
    m.train()
    codes = torch.randint(0, 16, (1, 8, 4), device=DEV, dtype=torch.uint8)
    q = torch.randn(1, 8, 4, 4, device=DEV, requires_grad=True)
    with pytest.raises(RuntimeError):
        m._lookup_route_chunk(codes, q, 0, 4, None, None, target_length=2)
    m.q_surrogate_enable = False
    tok = m._lookup_route_chunk(codes, q, 0, 4, None, None)
    tok.sum().backward()
    assert q.grad is None
    assert m.tables["ngram_3"].weight.grad is not None
    m.q_surrogate_enable = True
    m.eval()
