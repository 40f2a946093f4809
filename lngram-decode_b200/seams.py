"""The memory layer's decode and tree-verification seams on the lngram_b200 kernels.

* ``memory_step`` -- ``ffnmem/infer.py:152-182``: the memory output of n new positions after L
  cached ones: codes over the context [history + new], the fused gather + sink attention on the
  last n positions, the folded output map, and the short conv over the cached normalised outputs.
* ``decode_memory_step`` -- the memory block of ``decode_step(..., row_provider=)``
  (``ffnmem/infer.py:207-251``): rows from a row provider (e.g. ``serving.ZeroCopyGather``) replace the
  table lookup.
* ``tree_memory_block`` -- the memory part of ``tree_verify_step`` (``drafting/tree.py:165-195``):
  every node's n-gram window and conv window follow its ancestors, then the cached positions.
* ``tree_slots`` / ``tree_ngram_codes`` -- the node windows of ``drafting/tree.py:96-127``, built from a
  device-side ancestor table (``ancestor_table``).

``MemoryCache`` holds the memory part of the reference's ``DecodeState`` (``ffnmem/infer.py:65-112``):
codes [B, max_len, R] and conv inputs [B, max_len, d], indexed by absolute position.
"""

from __future__ import annotations

import torch
from torch import Tensor

from . import _lib
from ._lib import check, ptr, stream_ptr


class MemoryCache:
    def __init__(self, m, batch: int, max_len: int, device=None, dtype=None):
        device = device or m.readout_q_proj.weight.device
        dtype = dtype or m.readout_q_proj.weight.dtype
        self.batch, self.max_len, self.length = int(batch), int(max_len), 0
        self.codes = torch.zeros(batch, max_len, m.num_routes, dtype=torch.uint8, device=device)
        self.conv_in = torch.zeros(batch, max_len, m.hidden_size, dtype=dtype, device=device)

    def truncate(self, length: int) -> None:
        if not 0 <= length <= self.length:
            raise ValueError(f"cannot truncate to {length} (length {self.length})")
        self.length = length


_ANCESTORS: dict = {}


def ancestor_table(parent, depth: int, device=None) -> tuple[Tensor, Tensor]:
    """(anc, level) of a draft tree: anc[j, i] = the j-th ancestor of node i (anc[0] = i, -1 above
    the root) for j <= depth, and level[i] = the node's distance from the root.  Built on the device
    by repeated gathers through the parent array (one gather per level), not per node, and kept per
    (parent array, depth, device): a decode loop verifies the same tree shape step after step."""
    key = (tuple(int(x) for x in parent), int(depth), str(device))
    hit = _ANCESTORS.get(key)
    if hit is not None:
        return hit
    res = _ancestor_table(key[0], depth, device)
    if len(_ANCESTORS) > 64:
        _ANCESTORS.clear()
    _ANCESTORS[key] = res
    return res


def _ancestor_table(parent, depth: int, device) -> tuple[Tensor, Tensor]:
    par = torch.as_tensor(parent, dtype=torch.long, device=device)
    n = par.numel()
    cur = torch.arange(n, dtype=torch.long, device=device)
    rows = [cur]
    for _ in range(max(depth, n - 1)):     # a path is at most n nodes long
        cur = torch.where(cur >= 0, par[cur.clamp_min(0)], cur)
        rows.append(cur)
    chain = torch.stack(rows)                                         # [max(depth, n - 1) + 1, n]
    level = (chain >= 0).sum(0) - 1
    anc = chain[:depth + 1]
    return anc, level


def tree_slots(parent, L: int, back: int, device=None) -> tuple[Tensor, Tensor]:
    """Slots [n, back + 1] (oldest first) of every node and its ``back`` predecessors: first the
    node's ancestors (node a sits at slot L + a), then, past the root, the cached positions L - 1,
    L - 2, ...; ``ok`` is False for slots before position 0.  The reading order of the reference's
    ``drafting/tree.py:96-127`` (a node's window follows its ancestor path, then the history)."""
    anc, level = ancestor_table(parent, back, device)
    j = torch.arange(back + 1, device=anc.device)[:, None]            # steps back from the node
    # j <= level: ancestor j of the node; beyond the root: cached position L - (j - level)
    slot = torch.where(j <= level[None], L + anc, L - (j - level[None]))
    ok = slot >= 0
    return slot.clamp_min(0).flip(0).t().contiguous(), ok.flip(0).t().contiguous()


def tree_ngram_codes(parent, codes: Tensor, history: Tensor | None = None, hist: int = 2) -> tuple[Tensor, Tensor]:
    """Code windows [B, n, hist+1, R] of the tree nodes ``codes`` [B, n, R] after ``history``
    [B, h, R] (zeros where a slot precedes position 0), and the slot validity [n, hist+1]."""
    h = 0 if history is None else history.shape[1]
    seq = codes if history is None else torch.cat((history.to(codes.dtype), codes), 1)
    idx, ok = tree_slots(parent, h, hist, codes.device)
    return seq[:, idx] * ok[None, :, :, None].to(codes.dtype), ok


def _readout_rows(m, h: Tensor, tokens: Tensor) -> Tensor:
    """The readout over caller-supplied route tokens [B, n, R, Dt] (no table lookup)."""
    lib = _lib.library()
    f = m.folded()
    act = m._act()
    h = h.to(act).contiguous()
    M = h.numel() // m.hidden_size
    qd = m.readout_num_heads * m.route_token_dim
    rs = torch.empty(M, device=h.device, dtype=torch.float32)
    check(lib.lng_rms_rows(ptr(h), _lib.dtype_code(act), M, m.hidden_size, m.eps, ptr(rs), stream_ptr()), "rms")
    tdt = m.tables[f"ngram_{m.ngrams[0]}"].weight.dtype
    tokens = tokens.to(device=h.device, dtype=tdt).contiguous()
    if tuple(tokens.shape[-2:]) != (m.num_routes, m.route_token_dim) or tokens.numel() != M * m.num_routes * m.route_token_dim:
        raise ValueError(f"route_tokens must be [B, n, {m.num_routes}, {m.route_token_dim}]")
    qa = m._linear(h.view(M, -1), f["w_qk"])
    u = torch.empty(M, qd, device=h.device, dtype=act)
    check(lib.lng_route_attend_rows(ptr(tokens), _lib.dtype_code(tdt), M, m.num_routes, m.route_token_dim,
                                    m.readout_num_heads, m.eps, m.readout_sink_logit, ptr(qa), ptr(rs), ptr(u),
                                    _lib.dtype_code(act), stream_ptr()), "route_attend_rows")
    return m._linear(u, f["w_vo"])


def _readout(m, h: Tensor, tables, codes, cdt, B, T, window, seg, target_length):
    """qa = h . w_qk^T, qscale = 1/rms(h), fused attention, mixed = u . w_vo^T."""
    lib = _lib.library()
    f = m.folded()
    act = m._act()
    h = h.to(act).contiguous()
    M = h.numel() // m.hidden_size
    qd = m.readout_num_heads * m.route_token_dim
    rs = torch.empty(M, device=h.device, dtype=torch.float32)
    check(lib.lng_rms_rows(ptr(h), _lib.dtype_code(act), M, m.hidden_size, m.eps, ptr(rs), stream_ptr()), "rms")
    qa = m._linear(h.view(M, -1), f["w_qk"])
    u = torch.empty(M, qd, device=h.device, dtype=act)
    check(lib.lng_route_attend(tables, ptr(codes), cdt, B, T, window, None, None, ptr(seg), target_length, 0,
                               m.num_routes, m.readout_num_heads, m.eps, m.readout_sink_logit, ptr(qa), ptr(rs),
                               ptr(u), _lib.dtype_code(act), 0, None, None, stream_ptr()), "route_attend")
    return m._linear(u, f["w_vo"])


def _conv(m, mixed: Tensor, cache: MemoryCache, new_slot: Tensor, slot: Tensor) -> Tensor:
    out = torch.empty_like(mixed)
    check(_lib.library().lng_conv_window(m.readout_desc(), ptr(mixed), mixed.shape[0], ptr(cache.conv_in),
                                         ptr(new_slot), ptr(slot), ptr(out), stream_ptr()), "conv_window")
    return out


def _conv_lags(k: int, dil: int, device) -> Tensor:
    """Tap lags (k - 1 - tap) * dil, made on the device (a tensor built from a Python list would be a
    host-to-device copy on every decode step)."""
    return (k - 1 - torch.arange(k, device=device)) * dil


@torch.no_grad()
def memory_step(m, cache: MemoryCache, h: Tensor, codes_new: Tensor, route_codes_ctx: Tensor | None = None,
                route_tokens: Tensor | None = None) -> Tensor:
    """``ffnmem/infer.py:152-182``: output [B, n, d] for n new positions after ``cache.length``.  The new
    codes and conv inputs are written into the cache; ``cache.length`` is left to the caller (the
    reference's ``decode_step`` advances it after all layers).  ``route_tokens`` [B, n, R, Dt] (optional):
    rows supplied by the caller (host-RAM serving, a row provider); the table lookup is skipped."""
    B, n, d = h.shape
    L = cache.length
    if L + n > cache.max_len:
        raise ValueError(f"cache full: {L} + {n} > {cache.max_len}")
    cache.codes[:, L:L + n] = codes_new.to(torch.uint8)
    if route_tokens is not None:
        mixed = _readout_rows(m, h, route_tokens)
    else:
        hist = m.route_history_length
        ctx = cache.codes[:, max(0, L - hist):L + n] if route_codes_ctx is None else route_codes_ctx.to(torch.uint8)
        ctx = ctx.contiguous()
        mixed = _readout(m, h, m.tables_desc(), ctx, _lib.U8, B, ctx.shape[1], 0, None, n)
    k, dil = m.short_conv.kernel_size, m.short_conv.dilation
    dev = h.device
    pos = L + torch.arange(n, device=dev)
    base = (torch.arange(B, device=dev) * cache.max_len)[:, None]
    new_slot = (base + pos[None, :]).reshape(-1).contiguous()
    lags = _conv_lags(k, dil, dev)
    src = pos[:, None] - lags[None, :]                                    # [n, k]
    slot = torch.where(src[None] >= 0, base[:, :, None] + src[None], torch.full_like(src[None], -1))
    out = _conv(m, mixed, cache, new_slot, slot.reshape(B * n, k).contiguous())
    return out.view(B, n, d)


_TREE_PLANS: dict = {}


def _tree_plan(parent, L: int, B: int, max_len: int, hist: int, k: int, dil: int, device) -> dict:
    """Index tensors of one tree shape after L cached positions (built once, kept on the device):
    the n-gram window slots / validity of every node and the conv slots in the flat cache."""
    key = (tuple(int(x) for x in parent), L, B, max_len, hist, k, dil, str(device))
    plan = _TREE_PLANS.get(key)
    if plan is not None:
        return plan
    n = len(parent)
    h0 = min(L, hist)
    gidx, gok = tree_slots(parent, h0, hist, device)                      # slots into [history(h0) | nodes]
    lp = (k - 1) * dil
    idx, ok = tree_slots(parent, L, lp, device)
    taps = torch.arange(k, device=device) * dil                           # window columns the taps read
    tslot = torch.where(ok[:, taps], idx[:, taps], torch.full_like(idx[:, taps], -1))  # [n, k]
    base = (torch.arange(B, device=device) * max_len)[:, None, None]
    slot = torch.where(tslot[None] >= 0, base + tslot[None], torch.full_like(tslot[None], -1))
    new_slot = (torch.arange(B, device=device) * max_len)[:, None] + L + torch.arange(n, device=device)[None]
    plan = {"h0": h0, "gidx": gidx, "gok": gok[None, :, :, None].to(torch.uint8),
            "gok_nw": gok.to(torch.uint8).contiguous(),
            "seg": gok.to(torch.int32)[None].expand(B, n, hist + 1).reshape(B * n, hist + 1).contiguous(),
            "slot": slot.reshape(B * n, k).contiguous(), "new_slot": new_slot.reshape(-1).contiguous()}
    if len(_TREE_PLANS) > 64:
        _TREE_PLANS.clear()
    _TREE_PLANS[key] = plan
    return plan


@torch.no_grad()
def tree_memory_block(m, cache: MemoryCache, h: Tensor, codes: Tensor, parent) -> Tensor:
    """``drafting/tree.py:178-195``: memory output [B, n, d] of tree nodes ``codes`` [B, n, R] placed
    after ``cache.length``; writes the nodes' codes and conv inputs at L .. L+n-1 in node order."""
    B, n, d = h.shape
    L = cache.length
    if L + n > cache.max_len:
        raise ValueError(f"cache full: {L} + {n} > {cache.max_len}")
    if len(parent) != n:
        raise ValueError(f"parent has {len(parent)} nodes, h has {n}")
    hist = m.route_history_length
    k, dil = m.short_conv.kernel_size, m.short_conv.dilation
    plan = _tree_plan(parent, L, B, cache.max_len, hist, k, dil, h.device)
    codes = codes.to(device=h.device, dtype=torch.uint8).contiguous()
    h = h.to(m._act()).contiguous()
    W = hist + 1
    # one library call: node windows (+ the nodes' codes into the cache), readout, conv window
    tables, ro = m.tables_desc(), m.readout_desc()
    lib = _lib.library()
    ws = torch.empty(lib.lng_tree_workspace_bytes(tables, ro, B, n, W), device=h.device, dtype=torch.uint8)
    out = torch.empty(B, n, d, device=h.device, dtype=h.dtype)
    check(lib.lng_tree_memory_block(tables, ro, B, n, W, L, plan["h0"], cache.max_len, ptr(h), ptr(codes),
                                    ptr(cache.codes), ptr(cache.conv_in), ptr(plan["gidx"]), ptr(plan["gok_nw"]),
                                    ptr(plan["seg"]), ptr(plan["slot"]), ptr(plan["new_slot"]), ptr(out), ptr(ws),
                                    ws.numel(), stream_ptr()), "tree memory block")
    return out


@torch.no_grad()
def decode_memory_step(mem, cache: MemoryCache, h: Tensor, h_norm: Tensor, row_provider=None, pos: int = 0,
                       router_in: Tensor | None = None) -> Tensor:
    """The memory block of ``decode_step`` (``ffnmem/infer.py:207-251``, lines 230-240): the router's codes
    of the n new positions, then ``row_provider(pos, cache, codes_new) -> route tokens [B, n, R, Dt] | None``
    -- called after the codes are known and before they are written to the cache (``cache.length`` is
    still L), as the reference calls it -- and ``memory_step`` on those rows (or on the tables when it
    returns None or there is no provider).  ``mem`` is an ``LngramMemory``; the caller advances
    ``cache.length`` after the step, as ``decode_step`` does after all layers."""
    x = h_norm if mem.router_input == "hidden" else router_in
    if x is None:
        raise ValueError(f"router_input={mem.router_input} needs router_in")
    codes = mem.route_codes(x)
    rows = None if row_provider is None else row_provider(pos, cache, codes)
    return memory_step(mem.module, cache, h, codes, route_tokens=rows)
