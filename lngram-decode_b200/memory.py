"""Drop-in mirrors of the reference memory modules, running on the lngram_b200 CUDA library.

``RouteNgramMemoryV2`` keeps the constructor arguments, parameter names (so a reference
``state_dict`` loads unchanged), methods and error behaviour of the reference's
``ffnmem/memory/lngram_v2.py:830-1407`` for inference; ``LngramMemory`` mirrors the wrapper of
``ffnmem/memory/wrapper.py:50-125`` (router in fp32, sign codes, module forward).

Every method dispatches to the C ABI (``include/lngram_b200.h``) on the tensors' CUDA device and
current stream.  There is no CPU path: CPU tensors raise.  Training: ``_lookup_route_chunk`` carries
the reference's backward (the tables' row gradient and the q surrogate of ``lngram_v2.py:326-447``);
the readout (``forward``, ``_project_*``, ``_manual_gqa``) is inference-only and raises in training mode.
"""

from __future__ import annotations

import math
from dataclasses import dataclass
from typing import Optional, Sequence

import torch
from torch import Tensor, nn

from . import _lib
from ._lib import check, ptr, stream_ptr

WRAPPER_KEYS = ("routes", "mem_dim", "kv_heads", "q_heads", "head_dim", "router_init_std", "rank1", "router_input",
                "token_router")
# Appendix E recipe of the reference wrapper (ffnmem/memory/wrapper.py:37-47)
APPENDIX_E = dict(bits_per_route=4, ngrams=(2, 3), table_init_std_scale=1.0, output_proj_init_std_scale=0.0,
                  conv_zero_init=True, conv_kernel_size=4, q_surrogate_enable=True, q_surrogate_mode="approximate",
                  sink_initial_active_mass=0.5)


class _Norm(nn.Module):
    """Parameter holder with the reference RMSNorm's name (``lngram_v2.py:37-53``)."""

    def __init__(self, size: int, eps: float, device=None, dtype=None):
        super().__init__()
        self.hidden_size = int(size)
        self.eps = float(eps)
        self.weight = nn.Parameter(torch.ones(size, device=device, dtype=dtype))


class _ShortConv(nn.Module):
    """Parameter holder of ``DepthwiseCausalConv`` (``lngram_v2.py:207-248``)."""

    def __init__(self, d: int, k: int, dilation: int, eps: float, bias: bool, zero_init: bool, device=None, dtype=None):
        super().__init__()
        self.hidden_size, self.kernel_size, self.dilation = int(d), int(k), int(dilation)
        self.left_padding = (self.kernel_size - 1) * self.dilation
        self.norm = _Norm(d, eps, device=device, dtype=dtype)
        self.conv = nn.Conv1d(d, d, kernel_size=k, dilation=dilation, groups=d, bias=bias, device=device, dtype=dtype)
        if zero_init:
            nn.init.zeros_(self.conv.weight)
            if self.conv.bias is not None:
                nn.init.zeros_(self.conv.bias)


def _normal_(w: Tensor, std: float) -> None:
    """fp32 init then cast (``lngram_v2.py:20-33``)."""
    with torch.no_grad():
        if std == 0.0:
            w.zero_()
        else:
            w.copy_(torch.empty_like(w, dtype=torch.float32).normal_(0.0, std).to(w.dtype))


def _cuda(t: Tensor, what: str) -> Tensor:
    if not t.is_cuda:
        raise RuntimeError(f"{what} must be a CUDA tensor: lngram_b200 has no CPU path")
    return t


def rms_norm(x: Tensor, weight: Tensor | None, eps: float) -> Tensor:
    """The model block's RMSNorm (``ffnmem/model.py:39-48``), e.g. the ``attn_norm`` whose output is the
    memory router's input (``ffnmem/model.py:114``): the row is normalised in fp32, rounded to x's dtype,
    then multiplied by ``weight``; the result has the promoted dtype of x and the weight, as in torch."""
    x = _cuda(x, "x").contiguous()
    if weight is not None:
        weight = weight.detach().to(x.device).contiguous()
        if weight.dtype not in (torch.float32, torch.bfloat16):
            weight = weight.float()
    out_dt = x.dtype if weight is None else torch.promote_types(x.dtype, weight.dtype)
    d = x.shape[-1]
    y = torch.empty(x.shape, device=x.device, dtype=out_dt)
    with _lib.on_device(x.device):
        check(_lib.library().lng_rms_norm_model(ptr(x), _lib.dtype_code(x.dtype), x.numel() // d, d, ptr(weight),
                                                _lib.dtype_code(weight.dtype) if weight is not None else 0,
                                                float(eps), ptr(y), _lib.dtype_code(out_dt), stream_ptr()),
              "rms_norm")
    return y


@dataclass
class LngramIncrementalState:
    """The side state of ``forward_incremental`` that travels with an attention KV cache
    (``lngram_v2.py:187-204``): the last max_order - 1 route codes [B, H, R], the packed n-gram suffix
    [B, R] int32 (newest code in the top digit), how many positions it holds, and the conv history
    [B, d, left_padding] of normalised outputs."""

    route_history: Optional[Tensor] = None
    packed_route_state: Optional[Tensor] = None
    route_state_length: int = 0
    conv_history: Optional[Tensor] = None

    def index_select(self, indices: Tensor) -> "LngramIncrementalState":
        """The rows ``indices`` of every tensor (beam reordering), as the reference's ``index_select``."""
        def select(value: Optional[Tensor]) -> Optional[Tensor]:
            return None if value is None else value.index_select(0, indices.to(value.device))

        return LngramIncrementalState(select(self.route_history), select(self.packed_route_state),
                                      int(self.route_state_length), select(self.conv_history))


class _TrainLookup(torch.autograd.Function):
    """Route tokens of the lookup kernel with the reference's backward (``lng_lookup_backward``): the
    gathered rows' gradient into each order table and, when ``q_logits`` is given, the surrogate's
    route-logit gradient (``lngram_v2.py:326-447``)."""

    @staticmethod
    def forward(ctx, module, codes, q_logits, route_start, route_end, seg, val, *tables):
        with torch.no_grad():
            tokens = module._lookup_tokens(codes, route_start, route_end, seg, val, None)
        ctx.module, ctx.rs, ctx.re = module, route_start, route_end
        ctx.has = (q_logits is not None, seg is not None, val is not None)
        empty = codes.new_empty(0)
        ctx.save_for_backward(codes, q_logits if q_logits is not None else empty, seg if seg is not None else empty,
                              val if val is not None else empty)
        return tokens

    @staticmethod
    def backward(ctx, grad):
        codes, q, seg, val = ctx.saved_tensors
        has_q, has_seg, has_val = ctx.has
        m = ctx.module
        b, t, _ = codes.shape
        rs, re = ctx.rs, ctx.re
        grad = grad.contiguous()
        tables = [m.tables[f"ngram_{n}"].weight for n in m.ngrams]
        need = ctx.needs_input_grad[7:]
        gtabs = [torch.zeros(w.shape, device=w.device, dtype=torch.float32) if nd else None
                 for w, nd in zip(tables, need)]
        arr = (_lib.C.c_void_p * _lib.MAX_ORDERS)(*([ptr(g) for g in gtabs] + [None] * (_lib.MAX_ORDERS - len(gtabs))))
        grad_q = q32 = gq = None
        if has_q and ctx.needs_input_grad[2]:
            q32 = q.float().contiguous()
            gq = torch.empty(b, t, re - rs, m.bits_per_route, device=q.device, dtype=torch.float32)
        with _lib.on_device(grad.device):
            check(_lib.library().lng_lookup_backward(
                m.tables_desc(with_ss=False), ptr(codes), _lib.U8 if codes.dtype == torch.uint8 else _lib.I32, b, t,
                rs, re, ptr(seg) if has_seg else None, ptr(val) if has_val else None, ptr(grad),
                _lib.dtype_code(grad.dtype), ptr(q32), q.shape[2] if q32 is not None else 0,
                m.q_surrogate_temperature, m.q_surrogate_scale, int(m.q_surrogate_mode == "exact"), ptr(gq), arr,
                stream_ptr()), "lookup backward")
        if gq is not None:
            grad_q = torch.zeros(q.shape, device=q.device, dtype=torch.float32)
            grad_q[:, :, rs:re] = gq
            grad_q = grad_q.to(q.dtype)
        tgrads = [None if g is None else g.to(w.dtype) for g, w in zip(gtabs, tables)]
        return (None, None, grad_q, None, None, None, None, *tgrads)


class RouteNgramMemoryV2(nn.Module):
    """Inference drop-in for the reference ``RouteNgramMemoryV2`` (sink readout v2)."""

    def __init__(self, hidden_size: int, bits_per_route: int = 4, num_routes: int = 16, memory_dim: int = 128,
                 ngrams: Sequence[int] = (2, 3), initializer_range: float = 0.02, table_init_std_scale: float = 0.0,
                 output_proj_init_std_scale: float = 1.0, readout_q_proj_init_std_scale: float = 1.0,
                 readout_kv_proj_init_std_scale: float = 1.0, readout_num_heads: int = 16,
                 readout_num_kv_heads: int = 2, readout_head_dim: int = 128, readout_attention_dropout: float = 0.0,
                 rmsnorm_eps: float = 1e-6, normalization: str = "RMSNorm", conv_kernel_size: int = 4,
                 conv_dilation: Optional[int] = None, conv_bias: bool = False, conv_zero_init: bool = True,
                 execution_mode: str = "full", auto_max_kv_mb: float = 384.0, stream_route_chunk_size: int = 64,
                 readout_checkpoint_streaming: bool = False, q_surrogate_enable: bool = True,
                 q_surrogate_mode: str = "approximate", q_surrogate_temperature: float = 1.0,
                 q_surrogate_scale: float = 1.0, dropout: float = 0.0, sink_initial_active_mass: float = 0.5,
                 device=None, dtype=None):
        super().__init__()
        # validation mirrors lngram_v2.py:878-933 (ValueError)
        self.hidden_size, self.bits_per_route = int(hidden_size), int(bits_per_route)
        self.num_routes, self.memory_dim = int(num_routes), int(memory_dim)
        if self.hidden_size <= 0:
            raise ValueError("hidden_size must be positive")
        if not 1 <= self.bits_per_route <= 16:
            raise ValueError("bits_per_route must be in [1, 16]")
        if self.num_routes <= 0 or self.memory_dim <= 0:
            raise ValueError("num_routes and memory_dim must be positive")
        if str(normalization).lower().replace("_", "") != "rmsnorm":
            raise ValueError("lngram_b200 implements the RMSNorm readout normalisation")
        if int(conv_kernel_size) <= 0 or (conv_dilation is not None and int(conv_dilation) <= 0):
            raise ValueError("conv_kernel_size / conv_dilation must be positive")
        self.ngrams = tuple(sorted({int(v) for v in ngrams}))
        if not self.ngrams or min(self.ngrams) < 1 or len(self.ngrams) > _lib.MAX_ORDERS:
            raise ValueError(f"invalid n-gram orders: {self.ngrams}")
        self.max_ngram_order = max(self.ngrams)
        self.route_history_length = self.max_ngram_order - 1
        self.alphabet_size = 1 << self.bits_per_route
        self.route_logits_dim = self.num_routes * self.bits_per_route
        self.route_token_dim = len(self.ngrams) * self.memory_dim
        self.readout_num_heads, self.readout_num_kv_heads = int(readout_num_heads), int(readout_num_kv_heads)
        self.readout_head_dim = int(readout_head_dim)
        if self.readout_num_heads % self.readout_num_kv_heads:
            raise ValueError("readout_num_heads must be divisible by readout_num_kv_heads")
        if self.readout_num_heads * self.readout_head_dim != self.hidden_size:
            raise ValueError("LNGram GQA must preserve the full query width: readout_num_heads * readout_head_dim "
                             f"must equal hidden_size; got {self.readout_num_heads} * {self.readout_head_dim} != "
                             f"{self.hidden_size}")
        self.readout_groups = self.readout_num_heads // self.readout_num_kv_heads
        self.readout_inner_dim = self.readout_num_heads * self.readout_head_dim
        self.readout_kv_inner_dim = self.readout_num_kv_heads * self.readout_head_dim
        self.softmax_scale = self.readout_head_dim ** -0.5
        self.execution_mode = str(execution_mode).lower()
        if self.execution_mode not in {"full", "streaming", "auto"}:
            raise ValueError("execution_mode must be full, streaming, or auto")
        self.stream_route_chunk_size = int(stream_route_chunk_size)
        if float(q_surrogate_temperature) < 0.0:
            raise ValueError("q_surrogate_temperature must be non-negative")
        self.q_surrogate_enable = bool(q_surrogate_enable)
        self.q_surrogate_mode = str(q_surrogate_mode).lower()
        if self.q_surrogate_mode not in {"exact", "approximate"}:
            raise ValueError("q_surrogate_mode must be exact or approximate")
        self.q_surrogate_temperature = float(q_surrogate_temperature)
        self.q_surrogate_scale = float(q_surrogate_scale)
        mass = float(sink_initial_active_mass)
        if not math.isfinite(mass) or not 0.0 < mass < 1.0:
            raise ValueError("sink_initial_active_mass must be finite and in (0, 1)")
        self.sink_initial_active_mass = mass
        self.readout_sink_logit = math.log(self.num_routes * (1.0 - mass) / mass)
        max_rows = max(self.num_routes * self.alphabet_size ** n for n in self.ngrams)
        self.index_dtype = torch.int32 if max_rows - 1 <= torch.iinfo(torch.int32).max else torch.long
        eps = float(rmsnorm_eps)
        self.tables = nn.ModuleDict()
        for n in self.ngrams:
            t = nn.Embedding(self.num_routes * self.alphabet_size ** n, self.memory_dim, device=device, dtype=dtype)
            _normal_(t.weight, initializer_range * table_init_std_scale)
            self.tables[f"ngram_{n}"] = t
        self.readout_query_norm = _Norm(hidden_size, eps, device, dtype)
        self.readout_memory_norm = _Norm(self.route_token_dim, eps, device, dtype)
        self.readout_q_proj = nn.Linear(hidden_size, self.readout_inner_dim, bias=False, device=device, dtype=dtype)
        self.readout_kv_proj = nn.Linear(self.route_token_dim, 2 * self.readout_kv_inner_dim, bias=False,
                                         device=device, dtype=dtype)
        self.readout_o_proj = nn.Linear(self.readout_inner_dim, hidden_size, bias=False, device=device, dtype=dtype)
        _normal_(self.readout_q_proj.weight, initializer_range * readout_q_proj_init_std_scale)
        _normal_(self.readout_kv_proj.weight, initializer_range * readout_kv_proj_init_std_scale)
        _normal_(self.readout_o_proj.weight, initializer_range * output_proj_init_std_scale)
        dil = max(self.ngrams) if conv_dilation is None else int(conv_dilation)
        self.short_conv = _ShortConv(hidden_size, int(conv_kernel_size), dil, eps, bool(conv_bias),
                                     bool(conv_zero_init), device, dtype)
        self._fold_key = None
        self._fold = None

    # ------------------------------------------------------------------ descriptors
    @property
    def eps(self) -> float:
        return self.readout_query_norm.eps

    def _act(self) -> torch.dtype:
        dt = self.readout_q_proj.weight.dtype
        if dt not in (torch.float32, torch.bfloat16):
            raise ValueError("lngram_b200 runs the readout in fp32 or bf16")
        return dt

    def row_sumsq(self) -> dict:
        """Per-row sums of squares of every order table (fp32; cached per table version), read by the
        fused readout instead of recomputing each gathered row's RMS."""
        ws = [self.tables[f"ngram_{n}"].weight for n in self.ngrams]
        key = tuple((w.data_ptr(), w._version, w.dtype, str(w.device)) for w in ws)
        if getattr(self, "_ss_key", None) == key:
            return self._ss
        ss = {n: torch.empty(w.shape[0], device=w.device, dtype=torch.float32) for n, w in zip(self.ngrams, ws)}
        desc = self.tables_desc(with_ss=False)
        arr = (_lib.C.c_void_p * _lib.MAX_ORDERS)(*([ss[n].data_ptr() for n in self.ngrams] +
                                                    [None] * (_lib.MAX_ORDERS - len(self.ngrams))))
        with _lib.on_device(ws[0].device):
            check(_lib.library().lng_table_row_ss(desc, arr, stream_ptr()), "table row sums of squares")
        self._ss, self._ss_key = ss, key
        return ss

    def tables_desc(self, route_tables: dict | None = None, with_ss: bool = True) -> _lib.Tables:
        tabs = route_tables or {n: self.tables[f"ngram_{n}"].weight for n in self.ngrams}
        ss = self.row_sumsq() if (with_ss and route_tables is None) else None
        t = _lib.Tables()
        if ss is not None:
            for i, n in enumerate(self.ngrams):
                t.row_ss[i] = ss[n].data_ptr()
        t.n_orders = len(self.ngrams)
        dts = set()
        for i, n in enumerate(self.ngrams):
            w = _cuda(tabs[n], "table")
            if not w.is_contiguous():
                raise ValueError("tables must be contiguous")
            t.orders[i] = n
            t.tables[i] = w.data_ptr()
            dts.add(w.dtype)
        if len(dts) != 1:
            raise ValueError("all order tables must share a dtype")
        t.table_dtype = _lib.dtype_code(dts.pop())
        t.bits = self.bits_per_route
        t.num_routes = self.num_routes
        t.memory_dim = self.memory_dim
        return t

    def _guard(self) -> None:
        if self.training and torch.is_grad_enabled():
            raise RuntimeError("lngram_b200 implements the inference forward; the training surrogate "
                               "(lngram_v2.py:328-465) stays on the reference path")

    def folded(self) -> dict:
        """w_qk / w_vo of the folded readout (recomputed when any readout parameter changes)."""
        params = (self.readout_query_norm.weight, self.readout_q_proj.weight, self.readout_memory_norm.weight,
                  self.readout_kv_proj.weight, self.readout_o_proj.weight)
        key = tuple((p.data_ptr(), p._version, p.dtype, str(p.device)) for p in params)
        if self._fold_key == key:
            return self._fold
        act = self._act()
        dev = _cuda(self.readout_q_proj.weight, "readout weights").device
        lib = _lib.library()
        f32 = [p.detach().float().contiguous() for p in params]
        qh, dt, d = self.readout_num_heads, self.route_token_dim, self.hidden_size
        w_qk = torch.empty(qh * dt, d, device=dev, dtype=act)
        w_vo = torch.empty(d, qh * dt, device=dev, dtype=act)
        with _lib.on_device(dev):
            check(lib.lng_fold_readout(d, dt, qh, self.readout_num_kv_heads, self.readout_head_dim, ptr(f32[0]),
                                       ptr(f32[1]), ptr(f32[2]), ptr(f32[3]), ptr(f32[4]), ptr(w_qk), ptr(w_vo),
                                       _lib.dtype_code(act), stream_ptr()), "fold readout")
        conv_w = self.short_conv.conv.weight.detach().float().reshape(d, -1).contiguous()
        conv_b = None if self.short_conv.conv.bias is None else self.short_conv.conv.bias.detach().float().contiguous()
        self._fold = dict(w_qk=w_qk, w_vo=w_vo, conv_norm=self.short_conv.norm.weight.detach().float().contiguous(),
                          conv_w=conv_w, conv_b=conv_b)
        self._fold_key = key
        return self._fold

    def readout_desc(self, router_w: Tensor | None = None, router_w_split: Tensor | None = None) -> _lib.Readout:
        f = self.folded()
        r = _lib.Readout()
        r.hidden = self.hidden_size
        r.num_heads, r.num_kv_heads, r.head_dim = self.readout_num_heads, self.readout_num_kv_heads, self.readout_head_dim
        r.eps = self.eps
        r.sink_logit = self.readout_sink_logit
        r.conv_kernel, r.conv_dilation = self.short_conv.kernel_size, self.short_conv.dilation
        r.act_dtype = _lib.dtype_code(self._act())
        r.w_qk, r.w_vo = ptr(f["w_qk"]), ptr(f["w_vo"])
        r.conv_norm, r.conv_weight = ptr(f["conv_norm"]), ptr(f["conv_w"])
        r.conv_bias = ptr(f["conv_b"])
        if router_w is not None:
            r.router_w = ptr(router_w)
            r.router_in_dim = router_w.shape[1]
        r.router_w_split = ptr(router_w_split)
        return r

    # ------------------------------------------------------------------ reference methods
    def quantize_route_logits(self, q_logits: Tensor) -> Tensor:
        """``lngram_v2.py:1012-1017`` -> int32 codes [..., R] (bit-exact)."""
        if q_logits.shape[-1] != self.route_logits_dim:
            raise ValueError(f"route logits dim={q_logits.shape[-1]}, expected {self.route_logits_dim}")
        x = _cuda(q_logits, "q_logits").float().contiguous()
        out = torch.empty(*x.shape[:-1], self.num_routes, device=x.device, dtype=torch.int32)
        n = x.numel() // self.route_logits_dim
        with _lib.on_device(x.device):
            check(_lib.library().lng_quantize_route_logits(ptr(x), n, self.num_routes, self.bits_per_route, ptr(out),
                                                           _lib.I32, stream_ptr()), "quantize_route_logits")
        return out

    def _codes(self, codes: Tensor) -> tuple[Tensor, int]:
        codes = _cuda(codes, "route codes")
        if codes.dtype == torch.uint8:
            return codes.contiguous(), _lib.U8
        return codes.to(torch.int32).contiguous(), _lib.I32

    def _use_surrogate(self, q_logits: Optional[Tensor]) -> bool:
        """``lngram_v2.py:1019-1025``."""
        return bool(self.q_surrogate_enable and self.training and torch.is_grad_enabled() and q_logits is not None)

    def _lookup_route_chunk(self, route_codes: Tensor, q_logits_btrm: Optional[Tensor], route_start: int,
                            route_end: int, segment_ids: Optional[Tensor], valid_tokens: Optional[Tensor],
                            target_length: Optional[int] = None) -> Tensor:
        """``lngram_v2.py:1047-1113``: route tokens [B, T', R', Dt] in the table dtype (exact copies).  In
        training mode with gradients enabled the tokens carry the backward of the reference: the rows'
        gradient into the order tables and, with ``q_logits_btrm`` [B, T, R, bits] and the surrogate
        enabled, its route-logit gradient (``_LngramSurrogate``, ``:326-447``)."""
        if self.training and torch.is_grad_enabled():
            use_sur = self._use_surrogate(q_logits_btrm)
            if use_sur and target_length is not None:
                raise RuntimeError("cached inference cannot use surrogate gradients")
            codes, _ = self._codes(route_codes)
            seg = None if segment_ids is None else segment_ids.to(device=codes.device, dtype=torch.int64).contiguous()
            val = None if valid_tokens is None else valid_tokens.to(device=codes.device, dtype=torch.bool).contiguous()
            tables = [self.tables[f"ngram_{n}"].weight for n in self.ngrams]
            tokens = _TrainLookup.apply(self, codes, q_logits_btrm if use_sur else None, int(route_start),
                                        int(route_end), seg, val, *tables)
            return tokens if target_length is None else tokens[:, -int(target_length):]
        return self._lookup_tokens(route_codes, route_start, route_end, segment_ids, valid_tokens, target_length)

    def _lookup_tokens(self, route_codes: Tensor, route_start: int, route_end: int, segment_ids: Optional[Tensor],
                       valid_tokens: Optional[Tensor], target_length: Optional[int] = None) -> Tensor:
        b, t, _ = route_codes.shape
        codes, cdt = self._codes(route_codes)
        tout = t if target_length is None else min(int(target_length), t)
        w = self.tables[f"ngram_{self.ngrams[0]}"].weight
        out = torch.empty(b, tout, route_end - route_start, self.route_token_dim, device=codes.device, dtype=w.dtype)
        seg = None if segment_ids is None else segment_ids.to(device=codes.device, dtype=torch.int64).contiguous()
        val = None if valid_tokens is None else valid_tokens.to(device=codes.device, dtype=torch.bool).contiguous()
        desc = self.tables_desc()
        with _lib.on_device(codes.device):
            check(_lib.library().lng_lookup_route_chunk(desc, ptr(codes), cdt, b, t, int(route_start), int(route_end),
                                                        ptr(seg), ptr(val), int(tout) if target_length is not None else 0,
                                                        ptr(out), _lib.dtype_code(out.dtype), stream_ptr()),
                  "_lookup_route_chunk")
        return out

    def _linear(self, x: Tensor, w: Tensor, out_dtype: torch.dtype | None = None) -> Tensor:
        """y = x . w^T through lng_gemm (tcgen05 for bf16 x bf16, CUDA cores otherwise)."""
        x = x.contiguous()
        w = w.contiguous()
        k = x.shape[-1]
        m = x.numel() // k
        n = w.shape[0]
        out = torch.empty(*x.shape[:-1], n, device=x.device, dtype=out_dtype or x.dtype)
        with _lib.on_device(x.device):
            check(_lib.library().lng_gemm(ptr(x), _lib.dtype_code(x.dtype), k, ptr(w), _lib.dtype_code(w.dtype), k,
                                          ptr(out), _lib.dtype_code(out.dtype), n, m, n, k, None, 0, stream_ptr()),
                  "gemm")
        return out

    def _rms_norm(self, x: Tensor, w: Tensor) -> Tensor:
        x = x.contiguous()
        d = x.shape[-1]
        wf = w.detach().float().contiguous()
        out = torch.empty_like(x)
        with _lib.on_device(x.device):
            check(_lib.library().lng_rms_norm(ptr(x), _lib.dtype_code(x.dtype), x.numel() // d, d, ptr(wf), self.eps,
                                              ptr(out), _lib.dtype_code(out.dtype), stream_ptr()), "rms_norm")
        return out

    def _project_query(self, hidden_states: Tensor) -> Tensor:
        """``lngram_v2.py:1115-1118``: q_proj(RMSNorm(h)) -> [B, T, QH, HD]."""
        self._guard()
        b, t, _ = hidden_states.shape
        h = _cuda(hidden_states, "hidden_states")
        q = self._linear(self._rms_norm(h, self.readout_query_norm.weight), self.readout_q_proj.weight)
        return q.view(b, t, self.readout_num_heads, self.readout_head_dim)

    def _project_memory(self, route_tokens: Tensor) -> tuple[Tensor, Tensor]:
        """``lngram_v2.py:1120-1131``: RMSNorm(Dt) + kv_proj -> K, V [B, T, KV, R, HD]."""
        self._guard()
        rt = _cuda(route_tokens, "route_tokens")
        kv = self._linear(self._rms_norm(rt, self.readout_memory_norm.weight), self.readout_kv_proj.weight)
        key, value = kv.split(self.readout_kv_inner_dim, dim=-1)
        b, t, r, _ = key.shape
        shape = (b, t, r, self.readout_num_kv_heads, self.readout_head_dim)
        return key.reshape(shape).permute(0, 1, 3, 2, 4), value.reshape(shape).permute(0, 1, 3, 2, 4)

    def _real_route_probabilities(self, scores: Tensor) -> Tensor:
        """``lngram_v2.py:1877-1885`` (elementwise; kept for API completeness)."""
        scores = scores.float()
        sink = scores.new_tensor(self.readout_sink_logit)
        m = torch.maximum(scores.amax(dim=-1, keepdim=True), sink)
        ex = torch.exp(scores - m)
        return ex / (ex.sum(dim=-1, keepdim=True) + torch.exp(sink - m))

    def _manual_gqa(self, query: Tensor, key: Tensor, value: Tensor) -> Tensor:
        """``lngram_v2.py:1899-1920`` with explicit K/V: sink attention over routes."""
        self._guard()
        b, t = query.shape[:2]
        q = _cuda(query, "query").contiguous()
        k, v = key.contiguous(), value.contiguous()
        r = k.shape[-2]
        out = torch.empty(b, t, self.readout_num_heads, self.readout_head_dim, device=q.device, dtype=q.dtype)
        with _lib.on_device(q.device):
            check(_lib.library().lng_sink_gqa(ptr(q), ptr(k), ptr(v), _lib.dtype_code(q.dtype), b * t,
                                              self.readout_num_kv_heads, self.readout_groups, r, self.readout_head_dim,
                                              self.readout_sink_logit, ptr(out), stream_ptr()), "_manual_gqa")
        return out

    def _finish(self, head_output: Tensor, segment_ids: Optional[Tensor]) -> Tensor:
        """``lngram_v2.py:1354-1359``: o_proj then + SiLU(conv(RMSNorm(.)))."""
        self._guard()
        b, t = head_output.shape[:2]
        mixed = self._linear(head_output.reshape(b, t, self.readout_inner_dim), self.readout_o_proj.weight)
        return self._conv_finish(mixed, segment_ids, None)

    def _conv_finish(self, mixed: Tensor, segment_ids: Optional[Tensor], valid_tokens: Optional[Tensor]) -> Tensor:
        b, t, _ = mixed.shape
        out = torch.empty_like(mixed)
        seg = None if segment_ids is None else segment_ids.to(device=mixed.device, dtype=torch.int64).contiguous()
        val = None if valid_tokens is None else valid_tokens.to(device=mixed.device, dtype=torch.bool).contiguous()
        desc = self.readout_desc()
        with _lib.on_device(mixed.device):
            check(_lib.library().lng_conv_finish(desc, ptr(mixed.contiguous()), b, t, ptr(seg), ptr(val), ptr(out),
                                                 None, stream_ptr()), "conv finish")
        return out

    def forward(self, hidden_states: Tensor, route_codes_btr: Tensor, q_logits: Optional[Tensor] = None,
                segment_ids: Optional[Tensor] = None, valid_tokens: Optional[Tensor] = None) -> Tensor:
        """``lngram_v2.py:1361-1407`` (full and streaming modes compute the same function)."""
        if hidden_states.dim() != 3:
            raise ValueError("hidden_states must be [B,T,H]")
        b, t, hidden = hidden_states.shape
        if hidden != self.hidden_size:
            raise ValueError(f"hidden size={hidden}, expected {self.hidden_size}")
        if tuple(route_codes_btr.shape) != (b, t, self.num_routes):
            raise ValueError("route_codes_btr has an incompatible shape")
        if q_logits is not None and tuple(q_logits.shape) != (b, t, self.route_logits_dim):
            raise ValueError(f"q_logits shape={tuple(q_logits.shape)}, expected {(b, t, self.route_logits_dim)}")
        self._guard()
        return self.forward_codes(hidden_states, route_codes_btr, segment_ids, valid_tokens)

    @torch.no_grad()
    def forward_incremental(self, hidden_states: Tensor, route_codes_btr: Tensor,
                            state: Optional[LngramIncrementalState] = None) -> tuple[Tensor, LngramIncrementalState]:
        """``lngram_v2.py:1763-1829``: the exact prompt / decode forward of T new positions after ``state``.
        T = 1 reads the rows through the packed suffix (``_advance_packed`` / ``_lookup_packed``: a code
        window whose valid slots are the state's length); T > 1 looks up the context [history, codes]
        and packs its suffix (``_pack_suffix``).  The conv runs over [conv history, new normalised
        outputs].  Returns (output [B, T, d], the new state)."""
        if self.training:
            raise RuntimeError("forward_incremental is inference-only; call eval() first")
        from .seams import _readout

        if state is None:
            state = LngramIncrementalState()
        b, t, _ = hidden_states.shape
        if tuple(route_codes_btr.shape) != (b, t, self.num_routes):
            raise ValueError("incremental route code shape mismatch")
        h = _cuda(hidden_states, "hidden_states")
        dev = h.device
        act = self._act()
        h = h.to(act).contiguous()
        R, bits, maxn = self.num_routes, self.bits_per_route, self.max_ngram_order
        cdt = torch.uint8 if bits <= 8 else torch.int32
        cc = _lib.U8 if bits <= 8 else _lib.I32
        codes = route_codes_btr.to(device=dev, dtype=cdt).contiguous()
        ctx = codes if state.route_history is None else torch.cat(
            (state.route_history.to(device=dev, dtype=cdt), codes), 1).contiguous()
        lib = _lib.library()
        s = stream_ptr()
        packed = torch.empty(b, R, dtype=torch.int32, device=dev)
        with _lib.on_device(dev):
            if t == 1:
                pin = (torch.zeros(b, R, dtype=torch.int32, device=dev) if state.packed_route_state is None
                       else state.packed_route_state.to(device=dev, dtype=torch.int32).contiguous())
                window = torch.empty(b, maxn, R, dtype=torch.uint8, device=dev)
                check(lib.lng_packed_suffix(ptr(codes), cc, b, 1, R, bits, maxn, ptr(pin), ptr(packed), ptr(window), s),
                      "advance packed state")
                length = min(int(state.route_state_length) + 1, maxn)
                seg = (torch.arange(maxn, device=dev) >= maxn - length).to(torch.int32).expand(b, maxn).contiguous()
                mixed = _readout(self, h, self.tables_desc(), window, _lib.U8, b, 0, maxn, seg, 0)
            else:
                mixed = _readout(self, h, self.tables_desc(), ctx, cc, b, ctx.shape[1], 0, None, t)
                check(lib.lng_packed_suffix(ptr(ctx), cc, b, ctx.shape[1], R, bits, maxn, None, ptr(packed), None, s),
                      "pack suffix")
                length = min(int(state.route_state_length) + t, maxn)
                if state.route_state_length == 0 and state.route_history is None:
                    length = min(ctx.shape[1], maxn)
            conv = self.short_conv
            lp, k, dil, d = conv.left_padding, conv.kernel_size, conv.dilation, self.hidden_size
            cache = torch.zeros(b, lp + t, d, dtype=act, device=dev)
            if state.conv_history is not None and lp:
                cache[:, :lp] = state.conv_history.to(device=dev, dtype=act).transpose(1, 2)
            base = torch.arange(b, device=dev) * (lp + t)
            pos = lp + torch.arange(t, device=dev)
            new_slot = (base[:, None] + pos[None]).reshape(-1).contiguous()
            lags = (k - 1 - torch.arange(k, device=dev)) * dil     # made on the device: no host copy
            slot = (base[:, None, None] + pos[None, :, None] - lags[None, None, :]).reshape(b * t, k).contiguous()
            out = torch.empty(b * t, d, dtype=act, device=dev)
            check(lib.lng_conv_window(self.readout_desc(), ptr(mixed), b * t, ptr(cache), ptr(new_slot), ptr(slot),
                                      ptr(out), s), "conv window")
        hist = self.route_history_length
        new_state = LngramIncrementalState(
            route_history=ctx[:, ctx.shape[1] - hist:].contiguous() if hist else ctx[:, :0],
            packed_route_state=packed, route_state_length=int(length),
            conv_history=cache[:, cache.shape[1] - lp:].transpose(1, 2).contiguous() if lp else cache[:, :0].transpose(1, 2))
        return out.view(b, t, d), new_state

    def forward_codes(self, h: Tensor, codes: Optional[Tensor], segment_ids=None, valid_tokens=None, router_x=None,
                      router_w=None, codes_out: Optional[Tensor] = None, out: Optional[Tensor] = None,
                      workspace: Optional[Tensor] = None, router_w_split: Optional[Tensor] = None) -> Tensor:
        """One ``lng_memory_forward`` call: codes (given, or from the fp32 router on ``router_x``),
        folded query GEMM, fused gather + sink attention, folded output GEMM, conv finish."""
        h = _cuda(h, "hidden_states")
        act = self._act()
        if h.dtype != act:
            h = h.to(act)
        h = h.contiguous()
        b, t, _ = h.shape
        desc_t = self.tables_desc()
        desc_r = self.readout_desc(router_w, router_w_split)
        lib = _lib.library()
        cptr, cdt = None, 0
        if codes is not None:
            codes, cdt = self._codes(codes)
            cptr = ptr(codes)
        xptr, xdt = None, 0
        if router_x is not None:
            router_x = _cuda(router_x, "router input")
            if router_x.dtype not in (torch.float32, torch.bfloat16):
                router_x = router_x.float()
            router_x = router_x.contiguous()
            xptr, xdt = ptr(router_x), _lib.dtype_code(router_x.dtype)
        seg = None if segment_ids is None else segment_ids.to(device=h.device, dtype=torch.int64).contiguous()
        val = None if valid_tokens is None else valid_tokens.to(device=h.device, dtype=torch.bool).contiguous()
        if out is None:
            out = torch.empty_like(h)
        need = lib.lng_memory_workspace_bytes(desc_t, desc_r, b * t)
        if workspace is None or workspace.numel() < need:
            workspace = torch.empty(need, device=h.device, dtype=torch.uint8)
        with _lib.on_device(h.device):
            check(lib.lng_memory_forward(desc_t, desc_r, b, t, ptr(h), xptr, xdt, cptr, cdt, ptr(seg), ptr(val),
                                         ptr(out), ptr(codes_out), ptr(workspace), workspace.numel(), stream_ptr()),
                  "memory forward")
        return out


class LngramMemory(nn.Module):
    """Inference drop-in for the reference wrapper ``ffnmem/memory/wrapper.py:50-125``: owns the
    router ``d_in -> R*bits`` (evaluated in fp32), quantises, runs the module."""

    def __init__(self, d_model: int, mem_cfg: dict, init_std: float = 0.02, norm_eps: float = 1e-5, ssm_dim: int = 0,
                 device=None, dtype=None):
        super().__init__()
        cfg = dict(APPENDIX_E)
        cfg.update({k: v for k, v in mem_cfg.items() if k not in WRAPPER_KEYS})
        self.routes = int(mem_cfg["routes"])
        self.bits = int(cfg["bits_per_route"])
        head_dim = int(mem_cfg.get("head_dim", 64))
        q_heads = int(mem_cfg.get("q_heads", d_model // head_dim))
        if "ngrams" in cfg:
            cfg["ngrams"] = tuple(int(n) for n in cfg["ngrams"])
        for k in ("q_surrogate_enable", "q_surrogate_mode"):
            cfg.pop(k, None)
        self.module = RouteNgramMemoryV2(hidden_size=d_model, num_routes=self.routes, memory_dim=int(mem_cfg["mem_dim"]),
                                         readout_num_heads=q_heads, readout_num_kv_heads=int(mem_cfg.get("kv_heads", 4)),
                                         readout_head_dim=head_dim, initializer_range=init_std, rmsnorm_eps=norm_eps,
                                         device=device, dtype=dtype, **cfg)
        self.router_input = str(mem_cfg.get("router_input", "hidden"))
        if self.router_input not in ("hidden", "embed2"):
            raise ValueError(f"router_input {self.router_input!r} is not supported by lngram_b200 (hidden, embed2)")
        in_dim = d_model if self.router_input == "hidden" else 2 * d_model
        self.router = nn.Linear(in_dim, self.routes * self.bits, bias=False, device=device, dtype=torch.float32)
        nn.init.normal_(self.router.weight, mean=0.0, std=float(mem_cfg.get("router_init_std", init_std)))
        if (mem_cfg.get("token_router") or {}).get("enabled", False) or mem_cfg.get("rank1"):
            raise ValueError("token_router (SD-A) and rank1 are not part of the lngram_b200 inference path")

    def route_logits(self, h_norm: Tensor) -> Tensor:
        """fp32 router logits (``wrapper.py:98-101``), materialised only on request."""
        x = _cuda(h_norm, "router input")
        x = x.contiguous() if x.dtype in (torch.float32, torch.bfloat16) else x.float().contiguous()
        w = self.router.weight.detach().float().contiguous()
        n = x.numel() // x.shape[-1]
        logits = torch.empty(*x.shape[:-1], w.shape[0], device=x.device, dtype=torch.float32)
        codes = torch.empty(*x.shape[:-1], self.routes, device=x.device, dtype=torch.uint8)
        with _lib.on_device(x.device):
            check(_lib.library().lng_route_codes(ptr(x), _lib.dtype_code(x.dtype), n, x.shape[-1], x.shape[-1], ptr(w),
                                                 self.routes, self.bits, ptr(codes), _lib.U8, ptr(logits), stream_ptr()),
                  "route_logits")
        return logits

    def router_split(self) -> Tensor | None:
        """The router weight as bf16 parts W1 | W2 | W3 for the tensor-core router (cached per weight
        version); None when the shape does not suit it (bits > 6 or in_dim % 64 != 0)."""
        w = self.router.weight
        if self.bits > 6 or w.shape[1] % 64 != 0 or not w.is_cuda:
            return None
        key = (w.data_ptr(), w._version, str(w.device))
        if getattr(self, "_split_key", None) == key:
            return self._split
        wf = w.detach().float().contiguous()
        split = torch.empty(wf.shape[0], 3 * wf.shape[1], device=wf.device, dtype=torch.bfloat16)
        with _lib.on_device(wf.device):
            check(_lib.library().lng_router_prepare(ptr(wf), wf.shape[0], wf.shape[1], ptr(split), stream_ptr()),
                  "router_prepare")
        self._split, self._split_key = split, key
        return split

    def route_codes(self, x: Tensor) -> Tensor:
        """Codes [.., R] (uint8) of the fp32 router without materialising its logits (tensor cores
        for bf16 inputs, CUDA cores for fp32 inputs)."""
        x = _cuda(x, "router input")
        x = x.contiguous() if x.dtype in (torch.float32, torch.bfloat16) else x.float().contiguous()
        n = x.numel() // x.shape[-1]
        codes = torch.empty(*x.shape[:-1], self.routes, device=x.device, dtype=torch.uint8)
        split = self.router_split() if x.dtype == torch.bfloat16 else None
        lib = _lib.library()
        with _lib.on_device(x.device):
            if split is not None:
                check(lib.lng_route_codes_split(ptr(x), n, x.shape[-1], x.shape[-1], ptr(split), self.routes,
                                                self.bits, ptr(codes), stream_ptr()), "route_codes")
            else:
                w = self.router.weight.detach().float().contiguous()
                check(lib.lng_route_codes(ptr(x), _lib.dtype_code(x.dtype), n, x.shape[-1], x.shape[-1], ptr(w),
                                          self.routes, self.bits, ptr(codes), _lib.U8, None, stream_ptr()),
                      "route_codes")
        return codes

    def forward_host(self, h: Tensor, h_norm: Tensor | None = None, *, norm_weight: Tensor | None = None,
                     norm_eps: float = 1e-5, out: Tensor | None = None, groups: int = 4,
                     synchronize: bool = True) -> Tensor:
        """``forward`` for a batch held in host memory: h [B, T, d] (pinned CPU for overlap) -> out
        [B, T, d] on the CPU.  The router input is ``h_norm`` as given (copied in as well) or, with
        ``norm_weight``, made on the device from h by the block's RMSNorm (``rms_norm``, the
        reference's ``attn_norm`` at ``ffnmem/model.py:114``), so only h crosses PCIe.

        The batch is split into ``groups`` groups of whole sequences that flow through three CUDA
        streams -- copy in, forward, copy out -- with two device buffers per stream, so the copy of
        group g + 1 in, the forward of group g and the copy of group g - 1 out run at the same time
        (PCIe is full duplex).  The forward follows the caller's pending work on the current stream; the
        copies in of ``h`` wait only for their device buffers.  ``synchronize=True`` returns once ``out``
        is written.  ``synchronize=False`` returns with the copies out in flight and leaves the current
        stream unordered after them, so a next call's copies in and forwards overlap this call's last
        forward and copies out; call ``wait_host()`` (orders the current stream after the last copy out)
        or ``torch.cuda.synchronize()`` before reading ``out``, and do not rewrite ``h`` before then."""
        if self.training and torch.is_grad_enabled():
            raise RuntimeError("lngram_b200 implements the inference forward only")
        if self.router_input != "hidden":
            raise ValueError("forward_host supports the hidden-state router (router_input='hidden')")
        if (h_norm is None) == (norm_weight is None):
            raise ValueError("give exactly one of h_norm (copied in) or norm_weight (made on the device)")
        if h.dim() != 3 or h.is_cuda:
            raise ValueError("h must be a host tensor [B, T, d]")
        B, T, d = h.shape
        groups = max(1, min(int(groups), B))
        while B % groups:
            groups -= 1
        Bg = B // groups
        dev = self.router.weight.device
        act = self.module._act()
        if out is None:
            out = torch.empty(B, T, d, dtype=act, pin_memory=True)
        w = None if norm_weight is None else norm_weight.detach().to(dev)
        hn_dtype = (h.dtype if h_norm is None and w is None else
                    (h_norm.dtype if h_norm is not None else torch.promote_types(act, w.dtype)))
        key = (Bg, T, d, h.dtype, hn_dtype, str(dev))
        st = getattr(self, "_host_pipe", None)
        if st is None or st["key"] != key:
            mk = lambda dt: [torch.empty(Bg, T, d, device=dev, dtype=dt) for _ in range(2)]  # noqa: E731
            desc_t, desc_r = self.module.tables_desc(), self.module.readout_desc(self.router.weight)
            need = _lib.library().lng_memory_workspace_bytes(desc_t, desc_r, Bg * T)
            st = {"key": key, "h": mk(h.dtype), "hn": mk(hn_dtype), "out": mk(act),
                  "ws": torch.empty(need, device=dev, dtype=torch.uint8),
                  "streams": [torch.cuda.Stream(dev) for _ in range(3)]}
            self._host_pipe = st
        s_in, s_comp, s_out = st["streams"]
        cur = torch.cuda.current_stream(dev)
        # the forward reads the module's parameters: it follows the caller's pending work; the copies in
        # only wait for the buffer slot they overwrite to be free (events kept across calls, so one
        # call's copies in overlap the previous call's last forward and copies out)
        start = torch.cuda.Event()
        start.record(cur)
        s_comp.wait_event(start)
        last_comp, last_out = st.setdefault("last_comp", [None, None]), st.setdefault("last_out", [None, None])
        ev_out = None
        for g in range(groups):
            k = g % 2
            rows = slice(g * Bg, (g + 1) * Bg)
            if last_comp[k] is not None:
                s_in.wait_event(last_comp[k])        # slot k's inputs were read by an earlier group
            with torch.cuda.stream(s_in):
                st["h"][k].copy_(h[rows], non_blocking=True)
                if h_norm is not None:
                    st["hn"][k].copy_(h_norm[rows], non_blocking=True)
                ev_in = torch.cuda.Event()
                ev_in.record(s_in)
            s_comp.wait_event(ev_in)
            if last_out[k] is not None:
                s_comp.wait_event(last_out[k])       # slot k's output was copied out by an earlier group
            with torch.cuda.stream(s_comp):
                hd = st["h"][k]
                if w is not None:
                    hn = st["hn"][k]
                    check(_lib.library().lng_rms_norm_model(ptr(hd), _lib.dtype_code(hd.dtype), Bg * T, d, ptr(w),
                                                            _lib.dtype_code(w.dtype), float(norm_eps), ptr(hn),
                                                            _lib.dtype_code(hn.dtype), stream_ptr()), "rms_norm")
                self.forward(hd, st["hn"][k], out=st["out"][k], workspace=st["ws"])
                ev_comp = torch.cuda.Event()
                ev_comp.record(s_comp)
            last_comp[k] = ev_comp
            s_out.wait_event(ev_comp)
            with torch.cuda.stream(s_out):
                out[rows].copy_(st["out"][k], non_blocking=True)
                ev_out = torch.cuda.Event()
                ev_out.record(s_out)
            last_out[k] = ev_out
        st["tail"] = ev_out                          # copies out run in order on s_out: the last covers all
        if synchronize:
            cur.wait_event(ev_out)
            ev_out.synchronize()
        return out

    def wait_host(self) -> None:
        """Order the current stream after the last copy out of ``forward_host`` (no-op before the first)."""
        st = getattr(self, "_host_pipe", None)
        if st is not None and st.get("tail") is not None:
            torch.cuda.current_stream(st["h"][0].device).wait_event(st["tail"])

    def forward(self, h: Tensor, h_norm: Tensor, router_in: Tensor | None = None, *, codes_out: Tensor | None = None,
                out: Tensor | None = None, workspace: Tensor | None = None) -> Tensor:
        """``wrapper.py:103-125`` (eval): one fused C call from router input to memory output."""
        if self.training and torch.is_grad_enabled():
            raise RuntimeError("lngram_b200 implements the inference forward only")
        if self.router_input == "hidden":
            x = h_norm
        else:
            if router_in is None:
                raise ValueError(f"router_input={self.router_input} needs router_in from the model")
            x = router_in
        w = self.router.weight.detach()
        if w.dtype != torch.float32 or not w.is_contiguous():
            w = w.float().contiguous()
        split = self.router_split() if x.dtype == torch.bfloat16 else None
        return self.module.forward_codes(h, None, router_x=x, router_w=w, codes_out=codes_out, out=out,
                                         workspace=workspace, router_w_split=split)
