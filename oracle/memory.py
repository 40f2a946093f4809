"""numpy restatement of the Lngram v2 memory path (test oracle; see ``oracle/__init__.py``).

Arrays are float32 (bf16-valued data is passed already upcast) and integer
codes are int64.  Shapes follow the reference: B batch, T time, R routes,
``bits`` bits per route, A = 2**bits, n-gram orders ``ngrams``, ``mem_dim``
per order, Dt = len(ngrams) * mem_dim, readout heads QH = KV * G, head dim HD.
Citations are ``path:line`` inside the reference project.
"""

from __future__ import annotations

import math
from dataclasses import dataclass, field

import numpy as np

F32 = np.float32


# --------------------------------------------------------------------------- router
def route_logits(x: np.ndarray, w: np.ndarray) -> np.ndarray:
    """fp32 linear router, ``ffnmem/memory/wrapper.py:98-101`` (autocast off, both operands fp32)."""
    return (x.astype(F32) @ w.astype(F32).T).astype(F32)


def pack_bits_to_route_codes(bits: np.ndarray, bits_per_route: int) -> np.ndarray:
    """``ffnmem/memory/lngram_v2.py:74-89``: code[r] = sum_j bit[r*bits + j] << j (int)."""
    *lead, channels = bits.shape
    if bits_per_route <= 0 or bits_per_route > 30 or channels % bits_per_route:
        raise ValueError("channels must be divisible by bits_per_route in [1, 30]")
    routes = channels // bits_per_route
    grouped = bits.reshape(*lead, routes, bits_per_route).astype(np.int64)
    weights = np.left_shift(np.int64(1), np.arange(bits_per_route, dtype=np.int64))
    return (grouped * weights).sum(-1).astype(np.int64)


def quantize_route_logits(logits: np.ndarray, bits_per_route: int) -> np.ndarray:
    """``lngram_v2.py:1012-1017``: bit = logit > 0 (0 is a 0 bit), then pack."""
    return pack_bits_to_route_codes(logits > 0, bits_per_route)


def rms_norm(x: np.ndarray, w: np.ndarray | None, eps: float) -> np.ndarray:
    """RMSNorm in fp32: ``lngram_v2.py:37-53`` (F.rms_norm) and ``ffnmem/model.py:39-48``
    (identical for fp32 inputs): x * rsqrt(mean(x^2) + eps) * w."""
    xf = x.astype(F32)
    ms = np.mean(np.square(xf, dtype=F32), axis=-1, keepdims=True, dtype=F32)
    out = xf * (F32(1.0) / np.sqrt(ms + F32(eps))).astype(F32)
    if w is not None:
        out = out * w.astype(F32)
    return out.astype(F32)


def token_router_features(emb: np.ndarray, prev_w: np.ndarray, cur_w: np.ndarray, start: np.ndarray,
                          eps: float) -> np.ndarray:
    """``ffnmem/memory/router.py:50-59`` (``embed2``): concat(RMSNorm(E[x[t-1]] or start),
    RMSNorm(E[x[t]])) for emb [B, T, d] -> [B, T, 2d]."""
    b = emb.shape[0]
    prev = np.concatenate((np.broadcast_to(start.astype(F32), (b, 1, emb.shape[-1])), emb[:, :-1]), axis=1)
    return np.concatenate((rms_norm(prev, prev_w, eps), rms_norm(emb, cur_w, eps)), axis=-1)


# --------------------------------------------------------------------------- addressing
def aligned_ngram_address(codes: np.ndarray, order: int, bits: int) -> np.ndarray:
    """``lngram_v2.py:314-325``: addresses [B, T-order+1, R] of every complete window,
    oldest code least significant: sum_k c[t-order+1+k] << (k * bits)."""
    b, t, r = codes.shape
    valid_length = t - order + 1
    if valid_length <= 0:
        return np.zeros((b, 0, r), np.int64)
    address = codes[:, :valid_length, :].astype(np.int64).copy()
    for exp in range(1, order):
        address |= codes[:, exp:exp + valid_length, :].astype(np.int64) << (exp * bits)
    return address


def valid_mask(order: int, batch: int, time: int, segment_ids: np.ndarray | None,
               valid_tokens: np.ndarray | None) -> np.ndarray:
    """``lngram_v2.py:1027-1045``: window ending at t is valid iff t >= order-1, the window's
    first and last positions share a segment, and the LAST position is a valid token."""
    valid = np.zeros((batch, time), bool)
    if time < order:
        return valid
    suffix = np.ones((batch, time - order + 1), bool)
    if segment_ids is not None:
        suffix &= segment_ids[:, : time - order + 1] == segment_ids[:, order - 1:]
    if valid_tokens is not None:
        suffix &= valid_tokens[:, order - 1:].astype(bool)
    valid[:, order - 1:] = suffix
    return valid


def row_indices(codes: np.ndarray, order: int, bits: int, route_start: int, route_end: int) -> np.ndarray:
    """Global table rows [B, T-order+1, R'] of ``lngram_v2.py:1075-1084``:
    row = r * A**order + address (route offsets ``:1075-1083``)."""
    address = aligned_ngram_address(codes[:, :, route_start:route_end], order, bits)
    offsets = np.arange(route_start, route_end, dtype=np.int64) * ((1 << bits) ** order)
    return address + offsets.reshape(1, 1, -1)


def lookup_route_chunk(codes: np.ndarray, tables: dict, ngrams, bits: int, route_start: int, route_end: int,
                       segment_ids: np.ndarray | None = None, valid_tokens: np.ndarray | None = None,
                       target_length: int | None = None) -> np.ndarray:
    """``lngram_v2.py:1047-1113``: route tokens [B, T', R', Dt] -- per order, gather the rows of
    every complete window, left-pad order-1 zero rows, zero invalid windows, concatenate orders
    on the feature axis; ``target_length`` keeps the last positions (``:1108-1109``)."""
    b, t, _ = codes.shape
    rp = route_end - route_start
    memories = []
    for order in ngrams:
        table = tables[order]
        mem_dim = table.shape[1]
        mask = valid_mask(order, b, t, segment_ids, valid_tokens)
        if t - order + 1 <= 0:
            memory = np.zeros((b, t, rp, mem_dim), F32)
        else:
            rows = row_indices(codes, order, bits, route_start, route_end)
            values = table[rows].astype(F32)
            memory = np.concatenate((np.zeros((b, order - 1, rp, mem_dim), F32), values), axis=1)
            memory = memory * mask[:, :, None, None].astype(F32)
        if target_length is not None:
            memory = memory[:, -int(target_length):]
        memories.append(memory)
    return np.concatenate(memories, axis=-1)


# --------------------------------------------------------------------------- readout
@dataclass
class MemoryParams:
    """Parameters of ``RouteNgramMemoryV2`` (``lngram_v2.py:830-1010``) as fp32 numpy arrays."""

    num_routes: int
    bits: int
    ngrams: tuple
    memory_dim: int
    num_heads: int
    num_kv_heads: int
    head_dim: int
    eps: float
    tables: dict                      # order -> [R * A**order, memory_dim]
    q_norm: np.ndarray                # readout_query_norm.weight [d]
    mem_norm: np.ndarray              # readout_memory_norm.weight [Dt]
    q_proj: np.ndarray                # [QH*HD, d]
    kv_proj: np.ndarray               # [2*KV*HD, Dt] keys first, then values
    o_proj: np.ndarray                # [d, QH*HD]
    conv_norm: np.ndarray             # short_conv.norm.weight [d]
    conv_weight: np.ndarray           # short_conv.conv.weight [d, 1, k]
    conv_bias: np.ndarray | None = None
    conv_dilation: int | None = None  # default max(ngrams) (``:1000``)
    sink_active_mass: float = 0.5
    extra: dict = field(default_factory=dict)

    @property
    def groups(self) -> int:
        return self.num_heads // self.num_kv_heads

    @property
    def route_token_dim(self) -> int:
        return len(self.ngrams) * self.memory_dim

    @property
    def softmax_scale(self) -> float:
        return self.head_dim ** -0.5

    @property
    def sink_logit(self) -> float:
        """``lngram_v2.py:1865-1875``: b0 = log(R * (1 - mass) / mass)."""
        m = self.sink_active_mass
        return math.log(self.num_routes * (1.0 - m) / m)

    @property
    def dilation(self) -> int:
        return max(self.ngrams) if self.conv_dilation is None else int(self.conv_dilation)

    @property
    def route_history_length(self) -> int:
        return max(self.ngrams) - 1


def project_query(h: np.ndarray, p: MemoryParams) -> np.ndarray:
    """``lngram_v2.py:1115-1118``: q = q_proj(RMSNorm(h)) viewed [B, T, QH, HD]."""
    b, t, _ = h.shape
    q = rms_norm(h, p.q_norm, p.eps) @ p.q_proj.T
    return q.astype(F32).reshape(b, t, p.num_heads, p.head_dim)


def project_memory(tokens: np.ndarray, p: MemoryParams) -> tuple[np.ndarray, np.ndarray]:
    """``lngram_v2.py:1120-1131``: RMSNorm(Dt) then kv_proj; K, V [B, T, KV, R, HD]."""
    kv = (rms_norm(tokens, p.mem_norm, p.eps) @ p.kv_proj.T).astype(F32)
    inner = p.num_kv_heads * p.head_dim
    key, value = kv[..., :inner], kv[..., inner:]
    b, t, r, _ = key.shape
    key = key.reshape(b, t, r, p.num_kv_heads, p.head_dim).transpose(0, 1, 3, 2, 4)
    value = value.reshape(b, t, r, p.num_kv_heads, p.head_dim).transpose(0, 1, 3, 2, 4)
    return key, value


def real_route_probabilities(scores: np.ndarray, sink_logit: float) -> np.ndarray:
    """``lngram_v2.py:1877-1885``: exp(s - m) / (sum exp(s - m) + exp(b0 - m)), m = max(max s, b0)."""
    s = scores.astype(F32)
    m = np.maximum(s.max(-1, keepdims=True), F32(sink_logit))
    ex = np.exp(s - m).astype(F32)
    den = ex.sum(-1, keepdims=True, dtype=F32) + np.exp(F32(sink_logit) - m).astype(F32)
    return (ex / den).astype(F32)


def manual_gqa(query: np.ndarray, key: np.ndarray, value: np.ndarray, p: MemoryParams) -> np.ndarray:
    """``lngram_v2.py:1899-1920``: grouped scores * HD^-0.5, sink probabilities, P @ V."""
    b, t = query.shape[:2]
    grouped = query.reshape(b, t, p.num_kv_heads, p.groups, p.head_dim)
    scores = np.matmul(grouped, np.swapaxes(key, -1, -2)).astype(F32) * F32(p.softmax_scale)
    probs = real_route_probabilities(scores, p.sink_logit)
    out = np.matmul(probs, value).astype(F32)
    return out.reshape(b, t, p.num_heads, p.head_dim)


def streaming_partial(query: np.ndarray, key: np.ndarray, value: np.ndarray, p: MemoryParams,
                      state: tuple | None = None) -> tuple:
    """One route chunk of ``_streaming_update`` (``lngram_v2.py:1922-1942``), seeded as in
    ``:1992-1997`` (max = b0, sum = 1, value = 0) when ``state`` is None.  Returns
    (running_max, running_sum, running_value) with shapes [B,T,KV,G], [B,T,KV,G], [B,T,KV,G,HD]."""
    b, t = query.shape[:2]
    grouped = query.reshape(b, t, p.num_kv_heads, p.groups, p.head_dim)
    scores = np.matmul(grouped, np.swapaxes(key, -1, -2)).astype(F32) * F32(p.softmax_scale)
    if state is None:
        shape = (b, t, p.num_kv_heads, p.groups)
        state = (np.full(shape, p.sink_logit, F32), np.ones(shape, F32),
                 np.zeros(shape + (p.head_dim,), F32))
    run_max, run_sum, run_val = state
    new_max = np.maximum(run_max, scores.max(-1))
    old_scale = np.exp(run_max - new_max).astype(F32)
    ex = np.exp(scores - new_max[..., None]).astype(F32)
    new_sum = run_sum * old_scale + ex.sum(-1, dtype=F32)
    new_val = run_val * old_scale[..., None] + np.matmul(ex, value).astype(F32)
    return new_max.astype(F32), new_sum.astype(F32), new_val.astype(F32)


def streaming_finish(state: tuple, p: MemoryParams) -> np.ndarray:
    """``lngram_v2.py:2066-2070``: value / max(sum, tiny) -> [B, T, QH, HD]."""
    _, run_sum, run_val = state
    b, t = run_sum.shape[:2]
    out = run_val / np.maximum(run_sum, np.finfo(np.float32).tiny)[..., None]
    return out.astype(F32).reshape(b, t, p.num_heads, p.head_dim)


def depthwise_causal_conv(values: np.ndarray, p: MemoryParams, segment_ids: np.ndarray | None = None) -> np.ndarray:
    """``lngram_v2.py:207-286``: SiLU(depthwise causal conv(RMSNorm(values))) with zero left
    padding (k-1)*dilation; taps are stored oldest -> newest; with ``segment_ids`` a tap is
    dropped when its position is in another segment (``:251-271``)."""
    b, t, c = values.shape
    x = rms_norm(values, p.conv_norm, p.eps)
    k = p.conv_weight.shape[-1]
    dil = p.dilation
    out = np.zeros((b, t, c), F32)
    for tap in range(k):
        lag = (k - 1 - tap) * dil
        w = p.conv_weight[:, 0, tap].astype(F32)
        if lag == 0:
            shifted = x
            ok = np.ones((b, t, 1), F32)
        else:
            shifted = np.zeros_like(x)
            if lag < t:
                shifted[:, lag:] = x[:, :-lag]
            ok = np.zeros((b, t, 1), F32)
            if lag < t:
                if segment_ids is None:
                    ok[:, lag:] = 1.0
                else:
                    ok[:, lag:, 0] = (segment_ids[:, lag:] == segment_ids[:, :-lag]).astype(F32)
        out = out + shifted * ok * w
    if p.conv_bias is not None:
        out = out + p.conv_bias.astype(F32)
    return silu(out)


def silu(x: np.ndarray) -> np.ndarray:
    return (x / (F32(1.0) + np.exp(-x))).astype(F32)


def finish(head: np.ndarray, p: MemoryParams, segment_ids: np.ndarray | None = None) -> np.ndarray:
    """``lngram_v2.py:1354-1359``: mixed = o_proj(head); mixed + short_conv(mixed)."""
    b, t = head.shape[:2]
    mixed = (head.reshape(b, t, -1) @ p.o_proj.T).astype(F32)
    return (mixed + depthwise_causal_conv(mixed, p, segment_ids)).astype(F32)


def memory_forward(h: np.ndarray, codes: np.ndarray, p: MemoryParams, segment_ids: np.ndarray | None = None,
                   valid_tokens: np.ndarray | None = None, streaming_chunk: int | None = None) -> np.ndarray:
    """``RouteNgramMemoryV2.forward`` (``lngram_v2.py:1361-1407``), full mode or (with
    ``streaming_chunk``) the streaming route-chunk mode of ``:1944-2070``."""
    query = project_query(h, p)
    if streaming_chunk:
        state = None
        for start in range(0, p.num_routes, streaming_chunk):
            end = min(p.num_routes, start + streaming_chunk)
            tokens = lookup_route_chunk(codes, p.tables, p.ngrams, p.bits, start, end, segment_ids, valid_tokens)
            key, value = project_memory(tokens, p)
            state = streaming_partial(query, key, value, p, state)
        head = streaming_finish(state, p)
    else:
        tokens = lookup_route_chunk(codes, p.tables, p.ngrams, p.bits, 0, p.num_routes, segment_ids, valid_tokens)
        key, value = project_memory(tokens, p)
        head = manual_gqa(query, key, value, p)
    out = finish(head, p, segment_ids)
    if valid_tokens is not None:
        out = out * valid_tokens[..., None].astype(F32)
    return out


def lngram_memory_forward(h: np.ndarray, router_x: np.ndarray, router_w: np.ndarray, p: MemoryParams) -> np.ndarray:
    """``LngramMemory.forward`` in eval mode (``ffnmem/memory/wrapper.py:103-125``): fp32 router
    on ``router_x`` (h_norm, or router_in for token routers), sign codes, module forward."""
    codes = quantize_route_logits(route_logits(router_x, router_w), p.bits)
    return memory_forward(h, codes, p)


# --------------------------------------------------------------------------- draft head
def lookup_rows_at(codes: np.ndarray, b_idx: np.ndarray, t_idx: np.ndarray, p: MemoryParams) -> np.ndarray:
    """``ffnmem/memory/draft.py:26-47``: route tokens [N, R, Dt] of the n-grams ending at
    (b_idx[i], t_idx[i]); window slots before t = 0 form their own segment (zero rows)."""
    hist = p.route_history_length
    offs = np.arange(hist + 1)
    win_t = t_idx[:, None] - hist + offs[None, :]
    real = win_t >= 0
    win_t = np.maximum(win_t, 0)
    win_codes = codes[b_idx[:, None], win_t] * real[..., None].astype(codes.dtype)
    seg = real.astype(np.int64)
    tokens = lookup_route_chunk(win_codes, p.tables, p.ngrams, p.bits, 0, p.num_routes, seg, None)
    return tokens[:, -1]


@dataclass
class DraftParams:
    """``DraftReadout`` (``ffnmem/memory/draft.py:50-71``) weights + the tied embedding."""

    q_heads: int
    head_dim: int
    eps: float
    q_norm: np.ndarray   # [d]
    w_q: np.ndarray      # [q_heads*HD, d]
    w_o: np.ndarray      # [d, q_heads*HD]
    out_norm: np.ndarray  # [d]


def draft_hidden(emb_cur: np.ndarray, route_tokens: np.ndarray, mp: MemoryParams, dp: DraftParams) -> np.ndarray:
    """``ffnmem/memory/draft.py:73-86``: q = W_q RMSNorm(e); shared memory norm + KV
    projection; sink attention over routes; W_o -> RMSNorm.  emb_cur [N, d], tokens [N, R, Dt]."""
    n = emb_cur.shape[0]
    q = rms_norm(emb_cur, dp.q_norm, dp.eps) @ dp.w_q.T
    key, value = project_memory(route_tokens[:, None], mp)
    key, value = key[:, 0], value[:, 0]
    groups = dp.q_heads // mp.num_kv_heads
    q = q.astype(F32).reshape(n, mp.num_kv_heads, groups, dp.head_dim)
    scores = np.matmul(q, np.swapaxes(key, -1, -2)).astype(F32) * F32(mp.softmax_scale)
    probs = real_route_probabilities(scores, mp.sink_logit)
    out = np.matmul(probs, value).astype(F32).reshape(n, dp.q_heads * dp.head_dim)
    return rms_norm(out @ dp.w_o.T, dp.out_norm, dp.eps)


def draft_logits(emb_cur: np.ndarray, route_tokens: np.ndarray, embedding: np.ndarray, mp: MemoryParams,
                 dp: DraftParams) -> np.ndarray:
    """``draft.py:88-91`` + ``ffnmem/model.py:237-250``: logits = hidden @ E^T."""
    return (draft_hidden(emb_cur, route_tokens, mp, dp) @ embedding.astype(F32).T).astype(F32)


# --------------------------------------------------------------------------- decode / tree seams
def memory_step(h_new: np.ndarray, codes_ctx: np.ndarray, conv_hist: np.ndarray, p: MemoryParams) -> tuple:
    """``ffnmem/infer.py:152-182`` for one memory block: route tokens over the code context
    (history then new, ``target_length`` = new), readout, o_proj, conv over the cached
    normalised conv inputs.  ``conv_hist`` [B, lp, d] holds RMSNorm(mixed) of the previous
    ``lp`` positions (zeros before the sequence start).  Returns (output, new conv inputs)."""
    b, n, _ = h_new.shape
    tokens = lookup_route_chunk(codes_ctx, p.tables, p.ngrams, p.bits, 0, p.num_routes, None, None, target_length=n)
    key, value = project_memory(tokens, p)
    head = manual_gqa(project_query(h_new, p), key, value, p)
    mixed = (head.reshape(b, n, -1) @ p.o_proj.T).astype(F32)
    conv_in = rms_norm(mixed, p.conv_norm, p.eps)
    window = np.concatenate((conv_hist.astype(F32), conv_in), axis=1)
    conv_out = conv_window(window, p)[:, -n:]
    return (mixed + conv_out).astype(F32), conv_in


def conv_window(window: np.ndarray, p: MemoryParams) -> np.ndarray:
    """Valid (unpadded) depthwise conv + SiLU over already-normalised inputs: output t uses
    window[t + tap*dil] (taps oldest -> newest), the ``conv.conv(window)`` of ``infer.py:180`` and
    ``tree.py:192``; returns [B, W - (k-1)*dil, d]."""
    k = p.conv_weight.shape[-1]
    dil = p.dilation
    lp = (k - 1) * dil
    b, w, c = window.shape
    out = np.zeros((b, w - lp, c), F32)
    for tap in range(k):
        out = out + window[:, tap * dil: tap * dil + w - lp] * p.conv_weight[:, 0, tap].astype(F32)
    if p.conv_bias is not None:
        out = out + p.conv_bias.astype(F32)
    return silu(out)


def tree_path(parent, i: int) -> list:
    """``drafting/tree.py:78-84``: root .. i."""
    out = []
    while i >= 0:
        out.append(i)
        i = parent[i]
    return out[::-1]


def tree_slots(parent, L: int, back: int) -> tuple[np.ndarray, np.ndarray]:
    """``drafting/tree.py:96-111``: per node the ``back`` predecessors along its ancestors then
    the L cached positions (oldest first); slot L + a = node a.  (idx, ok) [n, back+1]."""
    n = len(parent)
    idx = np.zeros((n, back + 1), np.int64)
    ok = np.zeros((n, back + 1), bool)
    for i in range(n):
        path = tree_path(parent, i)
        for j in range(back + 1):
            if j < len(path):
                s = L + path[len(path) - 1 - j]
            else:
                s = L - (j - len(path) + 1)
            if s >= 0:
                idx[i, back - j], ok[i, back - j] = s, True
    return idx, ok


def tree_ngram_codes(parent, codes: np.ndarray, history: np.ndarray | None, hist: int) -> tuple:
    """``drafting/tree.py:114-127``: code windows [B, n, hist+1, R] along ancestors, then history."""
    h = 0 if history is None else history.shape[1]
    allc = codes if history is None else np.concatenate((history.astype(codes.dtype), codes), 1)
    idx, ok = tree_slots(parent, h, hist)
    ctx = allc[:, np.maximum(idx, 0)] * ok[None, :, :, None].astype(codes.dtype)
    return ctx, ok


def tree_route_tokens(ctx: np.ndarray, valid: np.ndarray, p: MemoryParams) -> np.ndarray:
    """``drafting/tree.py:130-136``: v2 lookup over each window with validity as segments."""
    b, n, w, r = ctx.shape
    seg = np.broadcast_to(valid.astype(np.int64)[None], (b, n, w)).reshape(b * n, w)
    rt = lookup_route_chunk(ctx.reshape(b * n, w, r), p.tables, p.ngrams, p.bits, 0, p.num_routes, seg, None)
    return rt[:, -1].reshape(b, n, r, -1)


def tree_memory_block(h: np.ndarray, codes: np.ndarray, parent, code_history: np.ndarray,
                      conv_cache: np.ndarray, L: int, p: MemoryParams) -> np.ndarray:
    """The memory block of ``tree_verify_step`` (``drafting/tree.py:178-195``).

    h [B, n, d] node inputs; codes [B, n, R] node codes; code_history [B, <=hist, R] codes of the
    positions just before the root; conv_cache [B, L, d] cached normalised conv inputs of the
    L positions before the root.  Returns mixed + conv over each node's ancestor window."""
    b, n, _ = h.shape
    ctx, valid = tree_ngram_codes(parent, codes, code_history, p.route_history_length)
    rt = tree_route_tokens(ctx, valid, p)
    key, value = project_memory(rt, p)
    head = manual_gqa(project_query(h, p), key, value, p)
    mixed = (head.reshape(b, n, -1) @ p.o_proj.T).astype(F32)
    ci = np.concatenate((conv_cache.astype(F32), rms_norm(mixed, p.conv_norm, p.eps)), axis=1)
    lp = (p.conv_weight.shape[-1] - 1) * p.dilation
    idx, ok = tree_slots(parent, L, lp)
    window = ci[:, idx] * ok[None, :, :, None].astype(F32)          # [B, n, lp+1, d]
    conv_out = conv_window(window.reshape(b * n, lp + 1, -1), p).reshape(b, n, -1)
    return (mixed + conv_out).astype(F32)


# --------------------------------------------------------------------------- incremental state / serving layout
def pack_suffix(codes: np.ndarray, maxn: int, bits: int) -> np.ndarray:
    """``lngram_v2.py:1714-1726`` (_pack_suffix): the last min(T, maxn) codes of [B, T, R] packed into
    int32 [B, R], the newest in digit maxn - 1."""
    t = codes.shape[1]
    keep = min(t, maxn)
    out = np.zeros((codes.shape[0], codes.shape[2]), np.int64)
    for off in range(keep):
        out |= codes[:, t - keep + off].astype(np.int64) << ((maxn - keep + off) * bits)
    return out.astype(np.int32)


def advance_packed(packed: np.ndarray | None, current: np.ndarray, maxn: int, bits: int) -> np.ndarray:
    """``lngram_v2.py:1728-1740`` (_advance_packed): shift down one digit, the new codes in the top digit."""
    p = np.zeros(current.shape, np.int64) if packed is None else packed.astype(np.int64)
    return ((p >> bits) | (current.astype(np.int64) << ((maxn - 1) * bits))).astype(np.int32)


def reverse_digits(n_digits: int, bits: int) -> np.ndarray:
    """``serving/layout.py:26-34``: j -> j with its n base-2^bits digits reversed."""
    j = np.arange((1 << bits) ** n_digits, dtype=np.int64)
    out = np.zeros_like(j)
    for k in range(n_digits):
        out |= ((j >> (k * bits)) & ((1 << bits) - 1)) << ((n_digits - 1 - k) * bits)
    return out


def serving_table(table: np.ndarray, routes: int, order: int, bits: int) -> np.ndarray:
    """``serving/layout.py:37-42`` (permute_table): row j of each route block = v2 row reverse_digits(j)."""
    block = (1 << bits) ** order
    return table.reshape(routes, block, -1)[:, reverse_digits(order, bits)].reshape(table.shape)


def surrogate_backward(grad_tokens: np.ndarray, codes: np.ndarray, q: np.ndarray, tables: dict, ngrams, bits: int,
                       route_start: int, route_end: int, temperature: float, scale: float, exact: bool,
                       segment_ids: np.ndarray | None = None, valid_tokens: np.ndarray | None = None):
    """Backward of the training lookup (``lngram_v2.py:1047-1113``) through ``_LngramSurrogate``
    (``:359-447``), per order: the rows' gradient into the table (dict order -> {row: grad}) and the
    route-logit gradient [B, T, R', bits] (approximate: one-bit counterfactuals; exact: the alphabet)."""
    b, t, _ = codes.shape
    rp = route_end - route_start
    A = 1 << bits
    md = next(iter(tables.values())).shape[1]
    p = (1.0 / (1.0 + np.exp(-temperature * q[:, :, route_start:route_end].astype(F32)))).astype(F32)
    grad_q = np.zeros((b, t, rp, bits), F32)
    tgrad = {}
    for oi, order in enumerate(ngrams):
        vl = t - order + 1
        tgrad[order] = {}
        if vl <= 0:
            continue
        g = grad_tokens[..., oi * md:(oi + 1) * md].astype(F32)
        mask = valid_mask(order, b, t, segment_ids, valid_tokens)
        gv = g[:, order - 1:] * mask[:, order - 1:, None, None]
        idx = row_indices(codes, order, bits, route_start, route_end)        # [B, VL, R']
        table = tables[order].astype(F32)
        for bb, ii, rr in zip(*np.nonzero(mask[:, order - 1:, None].repeat(rp, 2))):
            row = int(idx[bb, ii, rr])
            tgrad[order][row] = tgrad[order].get(row, 0) + gv[bb, ii, rr]
        if temperature == 0.0 or scale == 0.0:
            continue
        gq = np.zeros_like(grad_q)
        cur = (table[idx] * gv).sum(-1)
        for e in range(order):
            if exact:
                src = codes[:, e:e + vl, route_start:route_end].astype(np.int64)
                sp = p[:, e:e + vl]
                base = idx - src * (A ** e)
                for c in range(A):
                    d = (table[base + c * (A ** e)] * gv).sum(-1)
                    cb = np.array([(c >> j) & 1 for j in range(bits)], F32)
                    cp = np.where(cb.astype(bool), sp, 1.0 - sp).prod(-1)
                    gq[:, e:e + vl] += (cp[..., None] * (cb - sp) * d[..., None]) * F32(scale * temperature)
            else:
                for j in range(bits):
                    m = 1 << (e * bits + j)
                    fd = (table[idx ^ m] * gv).sum(-1)
                    sign = np.where((idx & m) != 0, -1.0, 1.0).astype(F32)
                    gq[:, e:e + vl, :, j] += (fd - cur) * sign
        if not exact:
            gq = gq * (F32(scale * temperature) * p * (1.0 - p))
        grad_q += gq
    return grad_q, tgrad
