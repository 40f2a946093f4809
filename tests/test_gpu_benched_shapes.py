"""Parity at the shapes ``bench.py`` times, not only at small cases.

* SD-B drafting: ``GpuDrafter.draft_batch`` in bf16 over 64 sequences x 1024-token prefixes, gamma = 4,
  182 routes, vocabulary 32,000, against the oracle drafter (``drafting/cpu_drafter.py:76-289``)
  teacher-forced along the drafted path.  A drafted token may differ from the oracle's argmax only
  where the oracle's own logits put it within the bf16 bar of the best one (a near tie).
* Tree verification: ``tree_memory_block`` at the SB layer (184 routes, 136 dims, bf16) over 64
  sequences x the 16-node tree after 1,024 cached positions, against the oracle's tree block
  (``drafting/tree.py:178-195``) and the per-path linear ``memory_step`` (``ffnmem/infer.py:152-182``)
  on sampled sequences.
* The scaled table: 184 routes x 2**20 rows x 136 bf16 dims (52.5 GB, byte offsets past 2**32), 5-bit
  codes, order 4.  Gathered rows are the C oracle's addresses bit-exactly; forward outputs at sampled
  positions match the oracle run on their causal slices.

Bars (``tests/helpers.py``): integer work exact, bf16 outputs within 1e-2 of the fp32 oracle.
"""

from __future__ import annotations

import math

import numpy as np
import pytest
import torch

from oracle import drafter as od
from oracle import memory as om
from tests.golden import cases
from tests.helpers import BF16_TOL, assert_bf16_close

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda:0")


@pytest.fixture(autouse=True)
def _clear_device_error(lngram):
    lngram._lib.device_error(clear=True)
    yield
    assert lngram._lib.device_error(clear=True) == 0, "a kernel recorded a device-side error"


# --------------------------------------------------------------------------- SD-B draft_batch
def test_sdb_draft_batch_bf16_matches_oracle_drafter(lngram):
    config, arrays = cases.draft_bundle("sdb")
    nseq, plen, gamma = 64, 1024, 4
    V = int(config["vocab"])
    d = lngram.GpuDrafter(lngram.Bundle(config, arrays, {}), act_dtype=torch.bfloat16)
    ref = od.OracleDrafter(config, arrays)
    gen = torch.Generator(device=DEV).manual_seed(300)
    prefix = torch.randint(0, V, (nseq, plen), device=DEV, generator=gen)
    drafted = d.draft_batch(prefix, gamma).cpu().numpy()
    assert drafted.shape == (nseq, gamma) and ((drafted >= 0) & (drafted < V)).all()
    pre = prefix.cpu().numpy()
    maxn = max(config["ngrams"])
    # windows of the drafts reach back maxn - 1 positions and a position's code reads its own and the
    # previous token, so the last maxn + 1 prefix tokens determine every draft (position 0 of this
    # teacher-forced trace uses the start vector, and its code is never read by those windows)
    tail = maxn + 1
    agree = total = 0
    code_flips = []
    for s in range(nseq):
        toks = pre[s, -tail:].tolist() + drafted[s, :gamma - 1].tolist()
        g_codes, _, g_lg = d.trace(toks)
        o_codes, _, _ = ref.trace(toks, full=True)
        code_flips.append(float((g_codes[1:] != o_codes[1:]).mean()))
        # the oracle on the GPU's codes, so that both read the same table rows
        _, _, o_lg = ref.trace(toks, codes=g_codes, full=True)
        for g in range(gamma):
            row = o_lg[tail - 1 + g].astype(np.float64)
            scale = float(np.abs(row).max())
            assert_bf16_close(g_lg[tail - 1 + g], row, what=f"seq {s} step {g} logits")
            best = int(np.lexsort((np.arange(V), -row))[0])
            tok = int(drafted[s, g])
            total += 1
            if tok == best:
                agree += 1
            else:
                margin = row[best] - row[tok]
                assert margin <= 2 * BF16_TOL * scale, (
                    f"seq {s} step {g}: drafted {tok}, oracle {best}, margin {margin:.3e} > bf16 bar")
    assert max(code_flips) < 1e-3, f"router code flips {max(code_flips):.2e}"
    assert agree / total >= 0.9, f"only {agree}/{total} drafted tokens equal the oracle's argmax"


# --------------------------------------------------------------------------- tree verification at SB
def _sb_memory(lngram):
    c = cases.MEMORY_CASES["sb_slice"]
    mem = lngram.LngramMemory(c["d"], {"routes": c["routes"], "mem_dim": c["mem_dim"], "kv_heads": c["kv_heads"],
                                       "q_heads": c["q_heads"], "head_dim": c["head_dim"], "ngrams": list(c["ngrams"]),
                                       "bits_per_route": c["bits"]}, norm_eps=1e-5, device=DEV,
                              dtype=torch.bfloat16).eval()
    p = cases.memory_params("sb_slice")
    state = {("router.weight" if k == "router.weight" else "module." + k): torch.from_numpy(v) for k, v in p.items()}
    mem.load_state_dict(state, strict=True)
    return mem, cases.oracle_params("sb_slice", p)


def test_sb_tree_block_bf16_matches_oracle(lngram):
    mem, po = _sb_memory(lngram)
    m = mem.module
    parent = cases.TREE_PARENT
    B, L, n, d, R = 64, 1024, len(parent), 1024, 184
    gen = torch.Generator(device=DEV).manual_seed(401)
    cache = lngram.MemoryCache(m, B, L + n)
    cache.codes[:, :L] = torch.randint(0, 16, (B, L, R), device=DEV, generator=gen, dtype=torch.uint8)
    cache.conv_in[:, :L] = torch.randn(B, L, d, device=DEV, generator=gen).to(torch.bfloat16)
    cache.length = L
    h = torch.randn(B, n, d, device=DEV, generator=gen).to(torch.bfloat16)
    codes = torch.randint(0, 16, (B, n, R), device=DEV, generator=gen, dtype=torch.uint8)
    with torch.no_grad():
        out = lngram.tree_memory_block(m, cache, h, codes, parent).float().cpu().numpy()
    np.testing.assert_array_equal(cache.codes[:, L:L + n].cpu().numpy(), codes.cpu().numpy())
    hist = m.route_history_length
    lp = (m.short_conv.kernel_size - 1) * m.short_conv.dilation
    hc, cc = h.float().cpu().numpy(), codes.cpu().numpy().astype(np.int64)
    ch = cache.codes[:, L - hist:L].cpu().numpy().astype(np.int64)
    conv = cache.conv_in[:, L - lp:L].float().cpu().numpy()
    for b in (0, 17, 63):
        # the block: only the last `lp` cached conv inputs and `hist` cached codes are read
        want = om.tree_memory_block(hc[b:b + 1], cc[b:b + 1], parent, ch[b:b + 1], conv[b:b + 1], lp, po)[0]
        assert_bf16_close(out[b], want, what=f"tree block, sequence {b}")
        # every node equals the linear decode step along its ancestor path
        for i in (0, 3, 7, 15):
            path = om.tree_path(parent, i)
            ctx = np.concatenate((ch[b:b + 1], cc[b:b + 1, path]), 1)
            lin, _ = om.memory_step(hc[b:b + 1, path], ctx, conv[b:b + 1], po)
            assert_bf16_close(out[b, i], lin[0, -1], what=f"node {i} of sequence {b} vs its linear path")


# --------------------------------------------------------------------------- scaled table (2**20 rows)
class _DeviceRows:
    """A read-only view of a device table for the oracle: ``rows[idx]`` fetches only those rows."""

    def __init__(self, weight: torch.Tensor):
        self.weight = weight.detach()
        self.shape = tuple(weight.shape)

    def __getitem__(self, idx):
        idx = np.asarray(idx)
        got = self.weight[torch.from_numpy(idx.reshape(-1)).to(DEV)].float().cpu().numpy()
        return got.reshape(*idx.shape, self.shape[1])


def test_scaled_table_full_rows_forward_and_addresses(lngram):
    from oracle.build import load_c_oracle

    R, bits, order, md, d = 184, 5, 4, 136, 1024
    span = (1 << bits) ** order                                         # 2**20 rows per route
    B, Tn = 2, 4096
    mem = lngram.LngramMemory(d, {"routes": R, "mem_dim": md, "kv_heads": 4, "q_heads": 16, "head_dim": 64,
                                  "ngrams": [order], "bits_per_route": bits, "table_init_std_scale": 0.0},
                              norm_eps=1e-5, device=DEV, dtype=torch.bfloat16).eval()
    m = mem.module
    w = m.tables[f"ngram_{order}"].weight
    assert w.numel() * w.element_size() > (1 << 32)
    with torch.no_grad():
        for r in range(R):
            g = torch.Generator(device=DEV).manual_seed(7919 + r)
            w[r * span:(r + 1) * span].copy_((torch.randn(span, md, device=DEV, generator=g) * 0.02).to(torch.bfloat16))
        p = cases.memory_params("sb_slice")   # readout weights of the SB shape (same d / heads / Dt)
        for k in ("readout_query_norm.weight", "readout_memory_norm.weight", "readout_q_proj.weight",
                  "readout_kv_proj.weight", "readout_o_proj.weight", "short_conv.norm.weight",
                  "short_conv.conv.weight"):
            mod, attr = k.rsplit(".", 1)
            getattr(m.get_submodule(mod), attr).copy_(torch.from_numpy(p[k]))
        gr = torch.Generator(device=DEV).manual_seed(3)
        mem.router.weight.copy_(torch.randn(R * bits, d, device=DEV, generator=gr) * 0.02)
    gen = torch.Generator(device=DEV).manual_seed(5)
    h = torch.randn(B, Tn, d, device=DEV, generator=gen).to(torch.bfloat16)
    hn = (h.float() * torch.rsqrt(h.float().pow(2).mean(-1, keepdim=True) + 1e-5)).to(torch.bfloat16)
    codes = torch.empty(B, Tn, R, device=DEV, dtype=torch.uint8)
    with torch.no_grad():
        out = mem(h, hn, codes_out=codes)
        tok = m._lookup_route_chunk(codes, None, 0, R, None, None)
    cc = codes.cpu().numpy()
    assert cc.max() < (1 << bits)
    # addresses: the C oracle's rows, gathered rows exact (routes beyond 2**32 bytes included)
    lib_c = load_c_oracle()
    rows = np.empty((B, Tn, R), np.int64)
    lib_c.oracle_row_indices(np.ascontiguousarray(cc).ctypes.data, B, Tn, R, order, bits, None, None,
                             rows.ctypes.data)
    assert rows.max() >= (R - 1) * span
    rng = np.random.default_rng(6)
    for b, t in zip(rng.integers(0, B, 64), np.concatenate([[0, 1, 2, 3, Tn - 1], rng.integers(0, Tn, 59)])):
        r = rows[b, t]
        if r[0] < 0:
            assert torch.count_nonzero(tok[b, t]) == 0
        else:
            assert torch.equal(tok[b, t], w[torch.from_numpy(r).to(DEV)])
    del tok
    # codes from the fp32 router agree with the oracle's away from zero logits
    xs = hn[:, :64].float().cpu().numpy()
    lg = om.route_logits(xs, mem.router.weight.detach().float().cpu().numpy())
    want_codes = om.quantize_route_logits(lg, bits)
    flips = (want_codes != cc[:, :64]).mean()
    assert flips < 1e-3, flips
    # outputs at sampled positions: the oracle on the causal slice, with the same codes and tables
    po = om.MemoryParams(num_routes=R, bits=bits, ngrams=(order,), memory_dim=md, num_heads=16, num_kv_heads=4,
                         head_dim=64, eps=1e-5, tables={order: _DeviceRows(w)},
                         q_norm=p["readout_query_norm.weight"], mem_norm=p["readout_memory_norm.weight"],
                         q_proj=p["readout_q_proj.weight"], kv_proj=p["readout_kv_proj.weight"],
                         o_proj=p["readout_o_proj.weight"], conv_norm=p["short_conv.norm.weight"],
                         conv_weight=p["short_conv.conv.weight"])
    reach = order - 1 + (m.short_conv.kernel_size - 1) * m.short_conv.dilation   # 3 + 12 positions back
    hc, oc = h.float().cpu().numpy(), out.float().cpu().numpy()
    for b, t in zip((0, 1, 0, 1, 0), (0, 7, 300, 2047, Tn - 1)):
        s = max(0, t - reach)
        want = om.memory_forward(hc[b:b + 1, s:t + 1], cc[b:b + 1, s:t + 1].astype(np.int64), po)[0, -1]
        assert_bf16_close(oc[b, t], want, what=f"scaled forward at ({b}, {t})")
    del mem, m, w
    torch.cuda.empty_cache()
    assert math.isfinite(float(np.abs(oc).max()))
