"""The torch-CPU port (``oracle/torch_port.py``, the timed CPU baseline of ``bench.py``) computes
what the numpy oracle computes, and what the reference's own forward computes where the reference
checkout is present."""

from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle import memory as om
from oracle import torch_port as tp
from tests.golden import cases
from tests.helpers import assert_fp32_close


@pytest.mark.parametrize("case", ["sb_slice", "tiny_multi", "scaled_slice"])
def test_forward_matches_numpy_oracle(case):
    c = cases.MEMORY_CASES[case]
    params = cases.memory_params(case)
    inp = cases.memory_inputs(case)
    if "segment_ids" in inp or "valid_tokens" in inp:
        inp = {k: inp[k] for k in ("h", "x")}
    p = tp.from_state(params, c)
    got = tp.lngram_forward(torch.from_numpy(inp["h"]), torch.from_numpy(inp["x"]), p).numpy()
    want = om.lngram_memory_forward(inp["h"], inp["x"], params["router.weight"], cases.oracle_params(case, params))
    assert_fp32_close(got, want, what=f"{case} forward")


@pytest.mark.parametrize("case", ["tiny_multi", "sb_slice"])
def test_tree_block_matches_numpy_oracle(case):
    c = cases.MEMORY_CASES[case]
    params = cases.memory_params(case)
    po = cases.oracle_params(case, params)
    p = tp.from_state(params, c)
    parent = cases.TREE_PARENT
    rng = np.random.default_rng(3)
    n, d, R = len(parent), c["d"], c["routes"]
    hist = max(c["ngrams"]) - 1
    lp = 3 * max(c["ngrams"])
    h = rng.standard_normal((2, n, d)).astype(np.float32)
    x = om.rms_norm(h, None, 1e-5)
    codes = om.quantize_route_logits(om.route_logits(x, params["router.weight"]), c["bits"])
    history = rng.integers(0, 1 << c["bits"], (2, hist, R))
    conv = rng.standard_normal((2, lp, d)).astype(np.float32)
    want = om.tree_memory_block(h, codes, parent, history, conv, lp, po)
    got = tp.tree_block(torch.from_numpy(h), torch.from_numpy(x), parent, torch.from_numpy(history),
                        torch.from_numpy(conv), p).numpy()
    assert_fp32_close(got, want, what=f"{case} tree block")


@pytest.mark.reference
def test_forward_matches_reference_forward(reference_path):
    from ffnmem.memory.wrapper import LngramMemory

    c = cases.MEMORY_CASES["sb_slice"]
    params = cases.memory_params("sb_slice")
    inp = cases.memory_inputs("sb_slice")
    mem = LngramMemory(c["d"], {"routes": c["routes"], "mem_dim": c["mem_dim"], "kv_heads": c["kv_heads"],
                                "q_heads": c["q_heads"], "head_dim": c["head_dim"], "ngrams": list(c["ngrams"]),
                                "bits_per_route": c["bits"]}, norm_eps=1e-5).eval()
    state = {("router.weight" if k == "router.weight" else "module." + k): torch.from_numpy(v)
             for k, v in params.items()}
    mem.load_state_dict(state, strict=True)
    with torch.no_grad():
        want = mem(torch.from_numpy(inp["h"]), torch.from_numpy(inp["x"])).numpy()
    got = tp.lngram_forward(torch.from_numpy(inp["h"]), torch.from_numpy(inp["x"]), tp.from_state(params, c)).numpy()
    assert_fp32_close(got, want, what="torch port vs reference forward")
