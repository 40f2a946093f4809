"""Write the golden fixtures of this folder by running the REFERENCE implementation.

    python tests/golden/make_golden.py [--reference /path/to/lngram-decode]

Needs the reference checkout (imported read-only from ``--reference``) and, for the C++
drafter fixture, ``oracle/_ref`` built by ``python oracle/build.py``.  Inputs come from
``cases.py`` (seeded numpy); each ``.npz`` stores small inputs and the reference's outputs.
The fixtures are committed; the tests replay them without the reference present.
"""

from __future__ import annotations

import argparse
import os
import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
REPO = HERE.parents[1]
sys.path.insert(0, str(REPO))

from tests.golden import cases  # noqa: E402


def _t(a, dtype=None):
    import torch

    t = torch.from_numpy(np.ascontiguousarray(a))
    return t if dtype is None else t.to(dtype)


def reference_memory(case: str):
    """A reference ``LngramMemory`` (``ffnmem/memory/wrapper.py:50``) loaded with ``cases`` weights."""
    import torch
    from ffnmem.memory.wrapper import LngramMemory

    c = cases.MEMORY_CASES[case]
    cfg = {"routes": c["routes"], "mem_dim": c["mem_dim"], "kv_heads": c["kv_heads"], "q_heads": c["q_heads"],
           "head_dim": c["head_dim"], "ngrams": list(c["ngrams"]), "bits_per_route": c["bits"],
           "execution_mode": "full"}
    mem = LngramMemory(c["d"], cfg, init_std=0.02, norm_eps=1e-5).eval()
    p = cases.memory_params(case)
    state = {("router.weight" if k == "router.weight" else "module." + k): _t(v) for k, v in p.items()}
    mem.load_state_dict(state, strict=True)
    return mem


def write_memory_case(case: str) -> None:
    import torch

    c = cases.MEMORY_CASES[case]
    mem = reference_memory(case)
    m = mem.module
    inp = cases.memory_inputs(case)
    h, x = _t(inp["h"]), _t(inp["x"])
    seg = _t(inp["segment_ids"]) if "segment_ids" in inp else None
    valid = _t(inp["valid_tokens"]) if "valid_tokens" in inp else None
    out = {}
    with torch.no_grad():
        logits = mem.route_logits(x)
        codes = m.quantize_route_logits(logits)
        out["logits"] = logits.numpy()
        out["codes"] = codes.numpy().astype(np.uint8)
        out["output_wrapper"] = mem(h, x).numpy()                        # LngramMemory.forward
        tokens = m._lookup_route_chunk(codes, None, 0, m.num_routes, seg, valid)
        q = m._project_query(h)
        key, value = m._project_memory(tokens)
        head = m._manual_gqa(q, key, value)
        out["output"] = m(h, codes, segment_ids=seg, valid_tokens=valid).numpy()
        out["head"] = head.numpy()
        out["query"] = q.numpy()
        big = tokens.numel() > 500_000
        if big:
            # Row indices (bit-exact addressing) and per-token sums stand in for the 3.3 MB tokens.
            from ffnmem.memory.lngram_v2 import _aligned_ngram_address

            for n in m.ngrams:
                a = _aligned_ngram_address(codes.to(torch.int64), n, m.bits_per_route)
                out[f"rows_{n}"] = (a + torch.arange(m.num_routes).view(1, 1, -1) * (m.alphabet_size ** n)).numpy()
            out["token_sums"] = tokens.double().sum(-1).numpy()
            out["key_sums"] = key.double().sum(-1).numpy()
        else:
            out["tokens"] = tokens.numpy()
            out["key"] = key.numpy()
            out["value"] = value.numpy()
        if c.get("stream_chunk"):
            m.execution_mode = "streaming"
            m.stream_route_chunk_size = int(c["stream_chunk"])
            out["output_streaming"] = m(h, codes, segment_ids=seg, valid_tokens=valid).numpy()
            m.execution_mode = "full"
        if c.get("bf16"):
            mb = m.to(torch.bfloat16)
            out["output_bf16_module"] = mb(h.to(torch.bfloat16), codes).float().numpy()
    for k in ("ids", "segment_ids", "valid_tokens"):
        if k in inp:
            out["in_" + k] = inp[k]
    if inp["h"].size <= 200_000:
        out["in_h"] = inp["h"]
        out["in_x"] = inp["x"]
    np.savez_compressed(HERE / f"memory_{case}.npz", **out)
    print(f"memory_{case}.npz", {k: v.shape for k, v in out.items()})


def write_seams() -> None:
    """Decode seam (``ffnmem/infer.py:152-182``) and tree block (``drafting/tree.py:178-195``) on the
    ``tiny_multi`` memory, each against the linear full forward of the same positions."""
    import torch
    from drafting.tree import tree_ngram_codes, tree_path, tree_route_tokens, tree_slots

    case = "tiny_multi"
    mem = reference_memory(case)
    m = mem.module
    B, L, n = 2, 11, len(cases.TREE_PARENT)
    s = cases.seam_inputs(case, B, L, n)
    hp, hn, cp, cn = (_t(s[k]) for k in ("h_prefix", "h_new", "codes_prefix", "codes_new"))
    out = {k: v for k, v in s.items()}
    hist = m.route_history_length
    lp = m.short_conv.left_padding
    with torch.no_grad():
        # decode seam: prefix then n new positions == full forward over L + n
        full = m(torch.cat((hp, hn), 1), torch.cat((cp, cn), 1))
        out["step_full"] = full[:, L:].numpy()
        # reference memory_step semantics on the context window [L-hist, L+n)
        ctx = torch.cat((cp, cn), 1)[:, max(0, L - hist):]
        tokens = m._lookup_route_chunk(ctx, None, 0, m.num_routes, None, None, target_length=n)
        key, value = m._project_memory(tokens)
        head = m._manual_gqa(m._project_query(hn), key, value)
        mixed = m.readout_o_proj(head.reshape(B, n, -1))
        pre = m.readout_o_proj(m._manual_gqa(m._project_query(hp), *m._project_memory(
            m._lookup_route_chunk(cp, None, 0, m.num_routes, None, None))).reshape(B, L, -1))
        conv_cache = m.short_conv.norm(pre)
        window = torch.cat((conv_cache, m.short_conv.norm(mixed)), 1)[:, max(0, L - lp):]
        if window.shape[1] < lp + n:
            window = torch.nn.functional.pad(window, (0, 0, lp + n - window.shape[1], 0))
        conv_out = m.short_conv.act(m.short_conv.conv(window.transpose(1, 2))).transpose(1, 2)
        out["step_output"] = (mixed + conv_out).numpy()
        out["conv_cache"] = conv_cache.numpy()
        # tree block, nodes = TREE_PARENT; reference pieces composed as in tree.py:178-195
        parent = cases.TREE_PARENT
        ctxw, valid = tree_ngram_codes(parent, cn, cp[:, max(0, L - hist):L], hist)
        rt = tree_route_tokens(m, ctxw, valid)
        key, value = m._project_memory(rt)
        head = m._manual_gqa(m._project_query(hn), key, value)
        mixed = m.readout_o_proj(head.reshape(B, n, -1))
        ci = torch.cat((conv_cache, m.short_conv.norm(mixed)), 1)
        idx, ok = tree_slots(parent, L, lp)
        window = ci[:, idx] * ok[None, :, :, None].to(ci.dtype)
        conv_out = m.short_conv.act(m.short_conv.conv(window.reshape(B * n, lp + 1, -1).transpose(1, 2)))
        out["tree_output"] = (mixed + conv_out.transpose(1, 2).reshape(B, n, -1)).numpy()
        out["tree_ctx"] = ctxw.numpy()
        out["tree_valid"] = valid.numpy()
        # linearised per-path reference: full forward over prefix + path, last position
        lin = []
        for i in range(n):
            path = tree_path(parent, i)
            seq_h = torch.cat((hp, hn[:, path]), 1)
            seq_c = torch.cat((cp, cn[:, path]), 1)
            lin.append(m(seq_h, seq_c)[:, -1])
        out["tree_linear"] = torch.stack(lin, 1).numpy()
        # the reference's own ancestor-window KAT (tests/test_live_tree.py:30-41)
        kc = torch.tensor([0, 10, 20, 30, 40, 50]).view(1, 6, 1)
        kh = torch.tensor([100, 101]).view(1, 2, 1)
        kctx, kok = tree_ngram_codes(cases.KAT_PARENT, kc, kh, 2)
        out["kat_ctx_hist"] = kctx[0, :, :, 0].numpy()
        kctx, kok = tree_ngram_codes(cases.KAT_PARENT, kc, None, 2)
        out["kat_ctx_nohist"] = kctx[0, :, :, 0].numpy()
        out["kat_ok_nohist"] = kok.numpy()
    np.savez_compressed(HERE / "seams_tiny_multi.npz", **out)
    print("seams_tiny_multi.npz", {k: v.shape for k, v in out.items()})


def write_draft_case(case: str, n_trace: int, with_cpp: bool) -> None:
    from drafting.cpu_drafter import RefDrafter
    from drafting.export_drafter import Bundle

    config, arrays = cases.draft_bundle(case)
    toks = cases.draft_tokens(case, n_trace)
    out = {}
    ref = RefDrafter(Bundle(config, arrays, {}))
    c, ids, lg = ref.trace(toks)
    out["trace_codes"] = c
    k = 8
    top = np.argsort(-lg, axis=1, kind="stable")[:, :k]
    out["trace_top_ids"] = np.take_along_axis(ids, top, 1)
    out["trace_top_logits"] = np.take_along_axis(lg, top, 1)
    out["trace_logit_sums"] = lg.astype(np.float64).sum(1)
    if lg.size <= 400_000:
        out["trace_logits"] = lg
    prefix = toks[: n_trace // 2]
    ref.reset()
    ref.commit(prefix)
    d = ref.draft(4, last_codes=True)
    out["draft_tokens"], out["draft_ids"], out["draft_logits"], out["draft_codes"] = (
        np.asarray(d.tokens), d.topk_ids, d.topk_logits, d.codes)
    hyp = toks[n_trace // 2: n_trace // 2 + 3]
    d = ref.draft(3, hyp=hyp)
    out["hyp_tokens"], out["hyp_ids"], out["hyp_logits"], out["hyp_codes"] = (
        np.asarray(d.tokens), d.topk_ids, d.topk_logits, d.codes)
    if with_cpp:
        sys.path.insert(0, str(REPO))
        from oracle.build import load_reference_drafter

        ext = load_reference_drafter()
        if ext is not None:
            from drafting.cpu_drafter import CppDrafter
            import drafting.cpu_drafter as cd

            cd._EXT = ext
            cpp = CppDrafter(Bundle(config, arrays, {}), threads=os.cpu_count() or 1)
            cc, cids, clg = cpp.trace(toks, codes=c)
            out["cpp_trace_top_logits"] = np.take_along_axis(clg, top, 1)
            cc2, _, _ = cpp.trace(toks)
            out["cpp_code_mismatch"] = np.asarray((cc2 != c).mean())
    out["tokens"] = np.asarray(toks)
    np.savez_compressed(HERE / f"draft_{case}.npz", **out)
    print(f"draft_{case}.npz", {k: np.shape(v) for k, v in out.items()})


INCREMENTAL_CALLS = (10, 1, 1, 1, 1, 1, 3, 1, 1)   # positions per forward_incremental call (a prefill, steps, a chunk)


def write_incremental(case: str) -> None:
    """``RouteNgramMemoryV2.forward_incremental`` (``lngram_v2.py:1763-1829``): a prefill, single steps and a
    multi-position chunk, with the state after every call, and the full forward of the same positions."""
    import torch

    mem = reference_memory(case)
    m = mem.module
    inp = cases.memory_inputs(case)
    T = sum(INCREMENTAL_CALLS)
    h = _t(inp["h"][:, :T])
    with torch.no_grad():
        codes = m.quantize_route_logits(mem.route_logits(_t(inp["x"][:, :T])))
        outs, state, t0 = [], None, 0
        out = {"codes": codes.numpy().astype(np.uint8), "in_h": inp["h"][:, :T]}
        for i, n in enumerate(INCREMENTAL_CALLS):
            y, state = m.forward_incremental(h[:, t0:t0 + n], codes[:, t0:t0 + n], state)
            outs.append(y.numpy())
            out[f"packed_{i}"] = state.packed_route_state.numpy()
            out[f"length_{i}"] = np.asarray(state.route_state_length)
            t0 += n
        out["outputs"] = np.concatenate(outs, 1)
        out["route_history"] = state.route_history.numpy()
        out["conv_history"] = state.conv_history.numpy()
        out["full"] = m(h, codes).numpy()
    np.savez_compressed(HERE / f"incremental_{case}.npz", **out)
    print(f"incremental_{case}.npz", {k: np.shape(v) for k, v in out.items()})


def write_serving(case: str) -> None:
    """The serving row layout (``serving/layout.py``): sampled rows of ``permute_tables`` and the route
    tokens ``serving_route_tokens`` reads from it, next to the v2 lookup's."""
    import torch
    from serving.layout import permute_tables, serving_route_tokens

    mem = reference_memory(case)
    m = mem.module
    inp = cases.memory_inputs(case)
    with torch.no_grad():
        codes = m.quantize_route_logits(mem.route_logits(_t(inp["x"])))
        tabs = permute_tables(m)
        out = {"codes": codes.numpy().astype(np.uint8)}
        rng = np.random.default_rng(17)
        for n, t in tabs.items():
            idx = np.sort(rng.choice(t.shape[0], size=min(512, t.shape[0]), replace=False))
            out[f"rows_idx_{n}"] = idx
            out[f"rows_{n}"] = t[torch.from_numpy(idx)].numpy()
        out["tokens"] = serving_route_tokens(tabs, codes, m.ngrams, m.bits_per_route).numpy()
        out["tokens_v2"] = m._lookup_route_chunk(codes, None, 0, m.num_routes, None, None).numpy()
    np.savez_compressed(HERE / f"serving_{case}.npz", **out)
    print(f"serving_{case}.npz", {k: np.shape(v) for k, v in out.items()})


SURROGATE_CASES = (("tiny_multi", "approximate", 1, 3), ("tiny_multi", "exact", 0, 4), ("scaled_slice", "approximate", 0, 3),
                   ("scaled_slice", "exact", 1, 2))


def write_surrogate() -> None:
    """The training-mode lookup's backward (``lngram_v2.py:1047-1113`` with ``_LngramSurrogate``,
    ``:326-447``): q_logits.grad and the tables' row gradients for a seeded token gradient."""
    import torch

    out = {}
    for i, (case, mode, rs, re) in enumerate(SURROGATE_CASES):
        mem = reference_memory(case)
        m = mem.module
        m.q_surrogate_mode = mode
        m.q_surrogate_temperature = 0.7
        m.q_surrogate_scale = 1.3
        m.train()
        inp = cases.memory_inputs(case)
        seg = _t(inp["segment_ids"]) if "segment_ids" in inp else None
        valid = _t(inp["valid_tokens"]) if "valid_tokens" in inp else None
        with torch.no_grad():
            logits = mem.route_logits(_t(inp["x"]))
            codes = m.quantize_route_logits(logits)
        b, t = codes.shape[:2]
        q = logits.view(b, t, m.num_routes, m.bits_per_route).clone().requires_grad_(True)
        tok = m._lookup_route_chunk(codes, q, rs, re, seg, valid)
        gen = torch.Generator().manual_seed(50 + i)
        g = torch.randn(tok.shape, generator=gen)
        (tok * g).sum().backward()
        out[f"c{i}_grad_tokens"] = g.numpy()
        out[f"c{i}_codes"] = codes.numpy().astype(np.uint8)
        out[f"c{i}_q"] = q.detach().numpy()
        out[f"c{i}_grad_q"] = q.grad.numpy()
        for n in m.ngrams:
            gw = m.tables[f"ngram_{n}"].weight.grad
            rows = torch.nonzero(gw.abs().sum(-1) > 0).view(-1)
            out[f"c{i}_rows_{n}"] = rows.numpy()
            out[f"c{i}_grad_table_{n}"] = gw[rows].numpy()
    np.savez_compressed(HERE / "surrogate_backward.npz", **out)
    print("surrogate_backward.npz", {k: np.shape(v) for k, v in out.items()})


ONLINE_CASES = (((3,), 4, 1.0), ((1, 2), 2, 0.5))   # (orders, bits, kappa)


def online_inputs(i: int, orders, bits: int) -> dict:
    """Seeded inputs of an online-counts case: a record's codes [T, R] and tokens [T] with repeated
    stretches (so in-context n-grams recur), windows [N, W, R] of it with leading non-real slots, the
    verified-pair deadlines and a distribution p [N, V]."""
    rng = np.random.default_rng(70 + i)
    T, R, V, N = 48, 6, 50, 9
    W = max(orders)
    codes = rng.integers(0, 1 << bits, (T, R))
    x = rng.integers(0, V, T)
    codes[20:30] = codes[5:15]                      # a repeated stretch of codes and tokens
    x[20:30] = x[5:15]
    last = rng.integers(0, T - 1, N)
    last[0] = 0
    pos = last[:, None] - (W - 1) + np.arange(W)[None]
    real = pos >= 0
    win = codes[np.clip(pos, 0, None)] * real[..., None]
    p = rng.random((N, V)).astype(np.float32)
    p /= p.sum(-1, keepdims=True)
    return {"codes": codes.astype(np.int64), "x": x.astype(np.int64), "win": win.astype(np.int64), "real": real,
            "deadline": (last - 1).astype(np.int64), "p": p, "vocab": V}


def write_online() -> None:
    """The online-count mixer of the acceptance harness (``drafting/drafters.py:117-143``) on seeded
    records: the mixed distribution for each case."""
    import torch
    from drafting.drafters import OnlineCounts

    out = {}
    for i, (orders, bits, kappa) in enumerate(ONLINE_CASES):
        inp = online_inputs(i, orders, bits)
        oc = OnlineCounts(_t(inp["codes"]), _t(inp["x"]), orders, bits, inp["vocab"], kappa)
        mixed = oc.mix(_t(inp["p"]), _t(inp["win"]), _t(inp["real"]), _t(inp["deadline"]))
        for k, v in inp.items():
            out[f"c{i}_{k}"] = np.asarray(v)
        out[f"c{i}_mixed"] = mixed.numpy()
    np.savez_compressed(HERE / "online_counts.npz", **out)
    print("online_counts.npz", {k: np.shape(v) for k, v in out.items()})


def main(argv=None) -> None:
    ap = argparse.ArgumentParser(description=__doc__)
    ap.add_argument("--reference", default=os.environ.get("LNGRAM_REFERENCE") or str(HERE.parents[2] / "reference"))
    ap.add_argument("--only", nargs="*", default=None)
    args = ap.parse_args(argv)
    sys.path.insert(0, args.reference)
    import torch

    torch.set_num_threads(max(1, os.cpu_count() or 1))
    todo = args.only or ["memory", "seams", "draft", "incremental", "serving", "surrogate", "online"]
    if "memory" in todo:
        for case in cases.MEMORY_CASES:
            write_memory_case(case)
    if "seams" in todo:
        write_seams()
    if "draft" in todo:
        write_draft_case("tiny", 60, with_cpp=True)
        write_draft_case("sdb", 24, with_cpp=True)
    if "incremental" in todo:
        write_incremental("tiny_multi")
        write_incremental("scaled_slice")
    if "serving" in todo:
        write_serving("tiny_multi")
    if "surrogate" in todo:
        write_surrogate()
    if "online" in todo:
        write_online()


if __name__ == "__main__":
    main()
