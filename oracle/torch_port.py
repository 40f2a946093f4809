"""torch-CPU restatement of the reference memory-layer forward (TEST / CPU-BASELINE INFRASTRUCTURE).

The reference's inference path is a sequence of PyTorch CPU operators; this module restates the
same algorithm with the same operator kinds (``F.linear`` GEMMs, an ``F.embedding`` row gather,
batched ``matmul`` attention, a grouped ``conv1d``) so that ``bench.py``'s CPU arm runs at the
speed of the reference's own forward on the host cores, which the numpy restatement
(``oracle/memory.py``) does not.  The numpy restatement stays the parity oracle; this port is
checked against it (``tests/test_torch_port.py``) and, where the reference checkout exists, against
the reference forward itself.

Steps and the reference lines they restate:

* router: fp32 ``x . W^T`` and the sign pack (``ffnmem/memory/wrapper.py:98-101``,
  ``ffnmem/memory/lngram_v2.py:74-89``, ``:1012-1017``);
* query: ``q_proj(RMSNorm(h))`` (``lngram_v2.py:1115-1118``);
* route tokens: rows ``r * A^n + sum_k c[t-n+1+k] << (k*bits)`` of every complete window, ``n - 1``
  leading zero rows, orders concatenated (``:314-325``, ``:1047-1113``);
* keys / values: ``kv_proj(RMSNorm(tokens))`` (``:1120-1131``);
* sink attention: ``exp(s - m) / (sum exp(s - m) + exp(b0 - m))``, ``m = max(max s, b0)``
  (``:1877-1920``);
* finish: ``o_proj``, then ``+ SiLU(depthwise causal conv(RMSNorm(.)))`` (``:207-286``,
  ``:1354-1359``).

Only ``tests/`` and ``bench.py``'s CPU arms import this module.
"""

from __future__ import annotations

import math
from dataclasses import dataclass

import torch
import torch.nn.functional as F
from torch import Tensor


@dataclass
class PortParams:
    num_routes: int
    bits: int
    ngrams: tuple
    memory_dim: int
    num_heads: int
    num_kv_heads: int
    head_dim: int
    eps: float
    tables: dict          # order -> [R * A**order, memory_dim] (fp32)
    q_norm: Tensor
    mem_norm: Tensor
    q_proj: Tensor
    kv_proj: Tensor
    o_proj: Tensor
    conv_norm: Tensor
    conv_weight: Tensor   # [d, 1, k]
    router: Tensor        # [R * bits, d]
    sink_active_mass: float = 0.5

    @property
    def sink_logit(self) -> float:
        m = self.sink_active_mass
        return math.log(self.num_routes * (1.0 - m) / m)

    @property
    def dilation(self) -> int:
        return max(self.ngrams)


def from_state(params: dict, cfg: dict, eps: float = 1e-5) -> PortParams:
    """PortParams from state-dict-named fp32 numpy arrays (``tests/golden/cases.memory_params``)."""
    t = {k: torch.from_numpy(v).float() for k, v in params.items()}
    return PortParams(num_routes=cfg["routes"], bits=cfg["bits"], ngrams=tuple(cfg["ngrams"]),
                      memory_dim=cfg["mem_dim"], num_heads=cfg["q_heads"], num_kv_heads=cfg["kv_heads"],
                      head_dim=cfg["head_dim"], eps=eps,
                      tables={n: t[f"tables.ngram_{n}.weight"] for n in cfg["ngrams"]},
                      q_norm=t["readout_query_norm.weight"], mem_norm=t["readout_memory_norm.weight"],
                      q_proj=t["readout_q_proj.weight"], kv_proj=t["readout_kv_proj.weight"],
                      o_proj=t["readout_o_proj.weight"], conv_norm=t["short_conv.norm.weight"],
                      conv_weight=t["short_conv.conv.weight"], router=t["router.weight"])


def _rms(x: Tensor, w: Tensor, eps: float) -> Tensor:
    return x * torch.rsqrt(x.pow(2).mean(-1, keepdim=True) + eps) * w


def route_codes(x: Tensor, p: PortParams) -> Tensor:
    bits = (F.linear(x.float(), p.router) > 0).view(*x.shape[:-1], p.num_routes, p.bits)
    weights = torch.tensor([1 << j for j in range(p.bits)], dtype=torch.int64)
    return (bits.to(torch.int64) * weights).sum(-1)


def route_tokens(codes: Tensor, p: PortParams, target_length: int | None = None) -> Tensor:
    """[B, T', R, Dt] for codes [B, T, R] (no segments / valid-token masks: the benchmark inputs)."""
    b, t, r = codes.shape
    parts = []
    for n in p.ngrams:
        span = 1 << (p.bits * n)
        out = torch.zeros(b, t, r, p.memory_dim)
        if t >= n:
            addr = codes[:, :t - n + 1].clone()
            for k in range(1, n):
                addr |= codes[:, k:t - n + 1 + k] << (k * p.bits)
            rows = addr + torch.arange(r, dtype=torch.int64) * span
            out[:, n - 1:] = F.embedding(rows, p.tables[n])
        parts.append(out if target_length is None else out[:, -target_length:])
    return torch.cat(parts, -1)


def readout(h: Tensor, tokens: Tensor, p: PortParams) -> Tensor:
    """Head output [B, T, QH*HD] of the sink attention over the route tokens."""
    b, t, _ = h.shape
    g = p.num_heads // p.num_kv_heads
    q = F.linear(_rms(h, p.q_norm, p.eps), p.q_proj).view(b, t, p.num_kv_heads, g, p.head_dim)
    kv = F.linear(_rms(tokens, p.mem_norm, p.eps), p.kv_proj)
    inner = p.num_kv_heads * p.head_dim
    r = tokens.shape[2]
    key = kv[..., :inner].reshape(b, t, r, p.num_kv_heads, p.head_dim).transpose(2, 3)
    value = kv[..., inner:].reshape(b, t, r, p.num_kv_heads, p.head_dim).transpose(2, 3)
    scores = torch.matmul(q, key.transpose(-1, -2)) * (p.head_dim ** -0.5)
    sink = torch.tensor(p.sink_logit)
    m = torch.maximum(scores.amax(-1, keepdim=True), sink)
    ex = torch.exp(scores - m)
    probs = ex / (ex.sum(-1, keepdim=True) + torch.exp(sink - m))
    return torch.matmul(probs, value).reshape(b, t, p.num_heads * p.head_dim)


def conv_finish(mixed: Tensor, p: PortParams) -> Tensor:
    k = p.conv_weight.shape[-1]
    lp = (k - 1) * p.dilation
    x = _rms(mixed, p.conv_norm, p.eps).transpose(1, 2)
    y = F.conv1d(F.pad(x, (lp, 0)), p.conv_weight, dilation=p.dilation, groups=x.shape[1])
    return mixed + F.silu(y).transpose(1, 2)


@torch.no_grad()
def lngram_forward(h: Tensor, x: Tensor, p: PortParams) -> Tensor:
    """``LngramMemory.forward(h, h_norm=x)`` in eval mode, fp32."""
    h = h.float()
    codes = route_codes(x, p)
    mixed = F.linear(readout(h, route_tokens(codes, p), p), p.o_proj)
    return conv_finish(mixed, p)


@torch.no_grad()
def tree_block(h: Tensor, x: Tensor, parent, code_history: Tensor, conv_cache: Tensor, p: PortParams) -> Tensor:
    """The memory block of ``drafting/tree.py:178-195`` for one batch of trees: node codes from the
    router, each node's n-gram window and conv window along its ancestors then the cached
    positions (``code_history`` [B, H, R], ``conv_cache`` [B, lp, d] of normalised conv inputs)."""
    h = h.float()
    b, n, _ = h.shape
    codes = route_codes(x, p)
    hist = max(p.ngrams) - 1
    k = p.conv_weight.shape[-1]
    lp = (k - 1) * p.dilation
    back = max(hist, lp)
    # ancestor slots: a[j, i] = j-th ancestor of node i (-1 above the root), level = depth
    par = torch.tensor([int(v) for v in parent])
    chain = [torch.arange(n)]
    for _ in range(max(back, n - 1)):
        c = chain[-1]
        chain.append(torch.where(c >= 0, par[c.clamp_min(0)], c))
    chain = torch.stack(chain)
    level = (chain >= 0).sum(0) - 1

    def slots(L: int, depth: int):
        j = torch.arange(depth + 1)[:, None]
        s = torch.where(j <= level[None], L + chain[:depth + 1], L - (j - level[None]))
        return s.clamp_min(0).flip(0).t(), (s >= 0).flip(0).t()

    H = code_history.shape[1]
    gi, gok = slots(H, hist)
    allc = torch.cat((code_history.long(), codes), 1)
    ctx = allc[:, gi] * gok[None, :, :, None]                              # [B, n, hist + 1, R]
    toks = []
    for order in p.ngrams:
        span = 1 << (p.bits * order)
        addr = torch.zeros(b, n, p.num_routes, dtype=torch.int64)
        for kk in range(order):
            addr |= ctx[:, :, hist + 1 - order + kk] << (kk * p.bits)
        ok = gok[:, hist + 1 - order:].all(-1)                             # [n]
        rows = addr + torch.arange(p.num_routes, dtype=torch.int64) * span
        toks.append(F.embedding(rows, p.tables[order]) * ok[None, :, None, None])
    mixed = F.linear(readout(h, torch.cat(toks, -1), p), p.o_proj)
    ci = torch.cat((conv_cache.float(), _rms(mixed, p.conv_norm, p.eps)), 1)
    ci_idx, ci_ok = slots(conv_cache.shape[1], lp)
    taps = torch.arange(k) * p.dilation
    win = ci[:, ci_idx[:, taps]] * ci_ok[:, taps][None, :, :, None]       # [B, n, k, d]
    y = (win * p.conv_weight[:, 0, :].t()[None, None]).sum(2)
    return mixed + F.silu(y)
