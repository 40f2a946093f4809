"""Seeded synthetic inputs shared by the golden-fixture writer and the tests.

Everything is generated with ``numpy.random.default_rng`` (PCG64: identical on every host),
so the fixtures in this folder store only small inputs and the reference's outputs; the
large arrays (tables, embeddings) are regenerated from the seeds at test time.  Seed
convention: 0 token ids, 1 hidden states, 2 tables, 3 router, 4 projections,
5 norms / conv / start vectors.  Generated in fp32 and, for bf16 cases, rounded to
bf16-representable values (round to nearest even), as the reference initialises in fp32
and casts (``ffnmem/memory/lngram_v2.py:20-33``).

Parameter dictionaries use the reference's ``state_dict`` names
(``RouteNgramMemoryV2``: ``tables.ngram_<n>.weight``, ``readout_*``, ``short_conv.*``),
so the same dictionary loads into the reference module, the oracle and the CUDA module.
"""

from __future__ import annotations

import math

import numpy as np

F32 = np.float32


def bf16_round(x: np.ndarray) -> np.ndarray:
    """Round fp32 values to the nearest bf16-representable value (ties to even)."""
    u = np.ascontiguousarray(x, dtype=F32).view(np.uint32).astype(np.uint64)
    u = (u + 0x7FFF + ((u >> 16) & 1)) & 0xFFFF0000
    return u.astype(np.uint32).view(F32)


def _normal(seed: int, shape, std: float, stream: int = 0) -> np.ndarray:
    rng = np.random.default_rng([seed, stream])
    return (rng.standard_normal(size=shape, dtype=F32) * F32(std)).astype(F32)


# --------------------------------------------------------------------------- memory layer
MEMORY_CASES = {
    # The tiny_cpu configuration: router fed by E[x] directly; R=8, 4 bits, n=3, 32 dims.
    "tiny": dict(d=128, routes=8, bits=4, ngrams=(3,), mem_dim=32, q_heads=4, kv_heads=2, head_dim=32,
                 B=2, T=64, vocab=32000, router="embedding", bf16=False),
    # The reference's own tiny memory (configs/tiny_cpu.yaml): orders (2, 3), with packed
    # segments and left padding, and the streaming route-chunk mode.
    "tiny_multi": dict(d=64, routes=4, bits=4, ngrams=(2, 3), mem_dim=16, q_heads=4, kv_heads=2, head_dim=16,
                       B=3, T=40, router="hidden", bf16=False, segments=True, valid=True, stream_chunk=3),
    # SB memory shape on a short slice, bf16-valued data.
    "sb_slice": dict(d=1024, routes=184, bits=4, ngrams=(3,), mem_dim=136, q_heads=16, kv_heads=4, head_dim=64,
                     B=1, T=48, router="hidden", bf16=True, o_std=0.006),
    # Scaled-table addressing: 5-bit codes, 4-gram windows, 2**20 rows per route.
    "scaled_slice": dict(d=64, routes=3, bits=5, ngrams=(4,), mem_dim=8, q_heads=4, kv_heads=2, head_dim=16,
                         B=2, T=24, router="hidden", bf16=False),
}


def memory_params(case: str) -> dict:
    """State-dict-named fp32 arrays for ``RouteNgramMemoryV2`` plus ``router.weight``."""
    c = MEMORY_CASES[case]
    rnd = bf16_round if c.get("bf16") else (lambda a: a)
    d, r, bits, md = c["d"], c["routes"], c["bits"], c["mem_dim"]
    qh, kv, hd = c["q_heads"], c["kv_heads"], c["head_dim"]
    dt = len(c["ngrams"]) * md
    p = {}
    for i, n in enumerate(c["ngrams"]):
        p[f"tables.ngram_{n}.weight"] = rnd(_normal(2, (r * (1 << bits) ** n, md), 0.02, stream=i))
    p["readout_query_norm.weight"] = rnd(1.0 + _normal(5, (d,), 0.1, 0))
    p["readout_memory_norm.weight"] = rnd(1.0 + _normal(5, (dt,), 0.1, 1))
    p["readout_q_proj.weight"] = rnd(_normal(4, (qh * hd, d), 0.02, 0))
    p["readout_kv_proj.weight"] = rnd(_normal(4, (2 * kv * hd, dt), 0.02, 1))
    p["readout_o_proj.weight"] = rnd(_normal(4, (d, qh * hd), c.get("o_std", 0.05), 2))
    p["short_conv.norm.weight"] = rnd(1.0 + _normal(5, (d,), 0.1, 2))
    p["short_conv.conv.weight"] = rnd(_normal(5, (d, 1, 4), 0.2, 3))
    if c["router"] == "embedding":
        p["router.weight"] = _normal(3, (r * bits, d), (1.0 / math.sqrt(r * bits)) / 2)
    else:
        p["router.weight"] = _normal(3, (r * bits, d), 0.02)
    return p


def memory_inputs(case: str) -> dict:
    """h [B,T,d], the router input x [B,T,d] and optional segment_ids / valid_tokens."""
    c = MEMORY_CASES[case]
    b, t, d = c["B"], c["T"], c["d"]
    out = {}
    if c["router"] == "embedding":
        ids = np.random.default_rng([0, 0]).integers(0, c["vocab"], size=(b, t))
        rows = _normal(1, (c["vocab"], d), 0.02)
        out["ids"] = ids
        out["h"] = rows[ids]
        out["x"] = out["h"]
    else:
        h = _normal(1, (b, t, d), 1.0)
        if c.get("bf16"):
            h = bf16_round(h)
        ms = np.mean(h.astype(F32) ** 2, -1, keepdims=True, dtype=F32)
        x = (h / np.sqrt(ms + F32(1e-5))).astype(F32)
        out["h"] = h
        out["x"] = bf16_round(x) if c.get("bf16") else x
    if c.get("segments"):
        seg = np.zeros((b, t), np.int64)
        seg[0, 13:] = 1
        seg[0, 27:] = 2
        seg[2, 5:] = 1
        out["segment_ids"] = seg
    if c.get("valid"):
        valid = np.ones((b, t), bool)
        valid[1, :7] = False       # left padding
        valid[2, 33:] = False      # right padding
        out["valid_tokens"] = valid
    return out


def oracle_params(case: str, params: dict | None = None):
    """The oracle's ``MemoryParams`` view of ``memory_params(case)``."""
    from oracle.memory import MemoryParams

    c = MEMORY_CASES[case]
    p = memory_params(case) if params is None else params
    return MemoryParams(
        num_routes=c["routes"], bits=c["bits"], ngrams=tuple(c["ngrams"]), memory_dim=c["mem_dim"],
        num_heads=c["q_heads"], num_kv_heads=c["kv_heads"], head_dim=c["head_dim"], eps=1e-5,
        tables={n: p[f"tables.ngram_{n}.weight"] for n in c["ngrams"]},
        q_norm=p["readout_query_norm.weight"], mem_norm=p["readout_memory_norm.weight"],
        q_proj=p["readout_q_proj.weight"], kv_proj=p["readout_kv_proj.weight"], o_proj=p["readout_o_proj.weight"],
        conv_norm=p["short_conv.norm.weight"], conv_weight=p["short_conv.conv.weight"])


# --------------------------------------------------------------------------- drafter bundles
DRAFT_CASES = {
    # SD-B shape: embed2 router over 182 routes, full-vocab scoring.
    "sdb": dict(d=1024, vocab=32000, routes=182, bits=4, ngrams=(3,), mem_dim=136, kv_heads=4, head_dim=64,
                q_heads=4, table_dtype="fp32", bf16=True, w_o_std=0.02),
    # Reference-sized tiny drafter (configs/tiny_cpu_sd.yaml with embed2): orders (2, 3), fp16 tables.
    "tiny": dict(d=64, vocab=256, routes=4, bits=4, ngrams=(2, 3), mem_dim=16, kv_heads=2, head_dim=16,
                 q_heads=2, table_dtype="fp16", bf16=False, w_o_std=0.2),
    # SD-C: the tiny drafter with a 16-state diagonal SSM read by the router and the query.
    "tiny_ssm": dict(d=64, vocab=256, routes=4, bits=4, ngrams=(2, 3), mem_dim=16, kv_heads=2, head_dim=16,
                     q_heads=2, table_dtype="fp16", bf16=False, w_o_std=0.2, ssm=16),
    # SD-C at the SD-B width (bf16-valued data): 64 states, router and query reading them.
    "sdb_ssm": dict(d=1024, vocab=32000, routes=182, bits=4, ngrams=(3,), mem_dim=136, kv_heads=4, head_dim=64,
                    q_heads=4, table_dtype="fp32", bf16=True, w_o_std=0.02, ssm=64),
}


def draft_bundle(case: str) -> tuple[dict, dict]:
    """(config, arrays) in the reference bundle layout (``drafting/export_drafter.py:25-34``,
    ``bundle_config`` ``:211-214``)."""
    c = DRAFT_CASES[case]
    rnd = bf16_round if c.get("bf16") else (lambda a: a)
    d, v, r, bits, md = c["d"], c["vocab"], c["routes"], c["bits"], c["mem_dim"]
    kv, hd, qh = c["kv_heads"], c["head_dim"], c["q_heads"]
    dt = len(c["ngrams"]) * md
    a = {"embedding": rnd(_normal(1, (v, d), 0.02, 7))}
    tdt = np.float16 if c["table_dtype"] == "fp16" else np.float32
    for i, n in enumerate(c["ngrams"]):
        a[f"table_{n}"] = rnd(_normal(2, (r * (1 << bits) ** n, md), 0.02, 10 + i)).astype(tdt)
    a["mem_norm"] = rnd(1.0 + _normal(5, (dt,), 0.1, 10))
    a["kv_proj"] = rnd(_normal(4, (2 * kv * hd, dt), 0.02, 10))
    n_ssm = int(c.get("ssm", 0))
    a["router"] = _normal(3, (r * bits, 2 * d + n_ssm), 0.02, 10)
    a["router_prev_norm"] = rnd(1.0 + _normal(5, (d,), 0.1, 11))
    a["router_cur_norm"] = rnd(1.0 + _normal(5, (d,), 0.1, 12))
    a["router_start"] = rnd(_normal(5, (d,), 0.02, 13))
    a["q_norm"] = rnd(1.0 + _normal(5, (d,), 0.1, 14))
    a["w_q"] = rnd(_normal(4, (qh * hd, d), 0.02, 11))
    a["w_o"] = rnd(_normal(4, (d, qh * hd), c["w_o_std"], 12))
    a["out_norm"] = rnd(1.0 + _normal(5, (d,), 0.1, 15))
    if n_ssm:
        # ffnmem/memory/ssm.py:23-35: W_in N(0, 0.02), decays geometrically spaced in 1 - a between
        # 0.5 and 0.001; the bundle stores a = sigmoid(theta) (drafting/export_drafter.py:30)
        a["ssm_norm"] = rnd(1.0 + _normal(5, (d,), 0.1, 16))
        a["ssm_w_in"] = rnd(_normal(4, (n_ssm, d), 0.02 if d > 64 else 0.2, 13))
        one_minus = np.exp(np.linspace(math.log(0.5), math.log(0.001), n_ssm)).astype(F32)
        a["ssm_decay"] = (F32(1.0) - one_minus).astype(F32)
        a["w_sq"] = rnd(_normal(4, (qh * hd, n_ssm), 0.02 if d > 64 else 0.2, 14))
    eps = 1e-5
    config = dict(kind="sd_c" if n_ssm else "sd_b", router_kind="embed2_ssm" if n_ssm else "embed2", d_model=d,
                  vocab=v, routes=r, bits=bits, ngrams=list(c["ngrams"]), mem_dim=md, kv_heads=kv, head_dim=hd,
                  q_heads=qh, ssm_dim=n_ssm, query_ssm=bool(n_ssm), norm_eps=eps, ssm_eps=eps, router_eps=eps, draft_eps=eps, mem_eps=eps,
                  softmax_scale=hd ** -0.5, sink_logit=math.log(r * 0.5 / 0.5), sketch_k=0, shortlist_cap=0,
                  table_dtype=c["table_dtype"], layer=1, groups=qh // kv, route_token_dim=dt)
    return config, a


def draft_tokens(case: str, n: int, seed: int = 0) -> list:
    return [int(x) for x in np.random.default_rng([0, seed]).integers(0, DRAFT_CASES[case]["vocab"], size=n)]


def random_sketch(config: dict, k: int = 4, seed: int = 0, empty_frac: float = 0.3, cap: int = 16) -> dict:
    """Sketch arrays (``drafting/sketches.py:1-30``: uint16 ids, uint32 counts per table row)
    plus the ``fallback`` list (``export_drafter.py:217-226``), as in the reference tests'
    ``random_sketch`` (``tests/test_live_export.py:47-58``)."""
    rng = np.random.default_rng([9, seed])
    out = {}
    tot = np.zeros(config["vocab"], np.float64)
    for n in config["ngrams"]:
        rows = config["routes"] * (1 << config["bits"]) ** n
        ids = rng.integers(0, config["vocab"], (rows, k)).astype(np.uint16)
        cnt = rng.integers(1, 50, (rows, k))
        cnt[rng.random(cnt.shape) < empty_frac] = 0
        out[f"sketch_ids_{n}"] = ids
        out[f"sketch_counts_{n}"] = cnt.astype(np.uint32)
    low = min(config["ngrams"])
    ids = out[f"sketch_ids_{low}"].astype(np.int64).ravel()
    tot = np.bincount(ids, weights=out[f"sketch_counts_{low}"].astype(np.float64).ravel(), minlength=config["vocab"])
    nz = np.flatnonzero(tot > 0)
    nz = nz[np.lexsort((nz, -tot[nz]))]
    out["fallback"] = nz[:cap].astype(np.int32)
    return out


# --------------------------------------------------------------------------- tree / decode seams
# Default tree parent array: root + 4 children + 11 grandchildren.
TREE_PARENT = (-1, 0, 0, 0, 0, 1, 1, 1, 2, 2, 2, 3, 3, 3, 4, 4)
# The reference's tree KAT (``tests/test_live_tree.py:15``).
KAT_PARENT = (-1, 0, 1, 0, 3, 1)


def seam_inputs(case: str, B: int, L: int, n: int, seed: int = 0) -> dict:
    """Prefix hidden states/codes [B, L] and new/node hidden states/codes [B, n] for the decode
    and tree seams (codes drawn uniformly, so every table row is reachable)."""
    c = MEMORY_CASES[case]
    rng = np.random.default_rng([6, seed])
    a = 1 << c["bits"]
    h = _normal(1, (B, L + n, c["d"]), 1.0, 20 + seed)
    if c.get("bf16"):
        h = bf16_round(h)
    codes = rng.integers(0, a, size=(B, L + n, c["routes"]))
    return dict(h_prefix=h[:, :L], h_new=h[:, L:], codes_prefix=codes[:, :L], codes_new=codes[:, L:])
