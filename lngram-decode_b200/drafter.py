"""GPU drafters with the reference drafter's two Python-facing APIs, over the C ABI's ``lng_drafter_*``.

* ``Drafter(tensors, numbers, ngrams, threads=1)`` -- the class the reference's C++ extension exports
  (``drafting/cpu/drafter.cpp:582-595``): the same constructor (bundle tensors by name, numbers by name,
  the n-gram orders, a thread count that results never depend on), the methods ``reset / length /
  truncate / committed_codes / commit / draft / trace`` with the same arguments, defaults and torch
  return types, and ``RuntimeError`` where the C++ class raises.  Code that holds ``ext.Drafter`` --
  ``CppDrafter._core`` (``drafting/cpu_drafter.py:327-389``), ``cpu_drafter.bench / check`` -- can hold
  this object instead.
* ``GpuDrafter(bundle)`` -- the ``RefDrafter`` / ``CppDrafter`` wrapper API (``drafting/cpu_drafter.py:
  76-389``) over a ``Drafter`` core, plus ``draft_batch`` for many independent sequences at once (the
  reference API is batch-1).

Bundles: embed2 routers with full-vocabulary scoring, the SD-C SSM (``router_kind`` ``embed2_ssm``
and / or ``query_ssm``) and sketch shortlists (``sketch_k`` > 0, ``shortlist_cap`` > 0), as the C++
drafter.  ``act_dtype=torch.float32`` (default) computes in fp32 like the reference drafter;
``torch.bfloat16`` keeps the embedding, tables and folded readout in bf16 (tensor cores).

    d = GpuDrafter(bundle)              # bundle path, lngram_b200 Bundle, or the reference's Bundle
    d.commit(prompt_tokens)             # verified tokens (optionally with the target's codes)
    out = d.draft(4)                    # out.tokens, out.topk_ids [4, k], out.topk_logits, out.codes
    d.truncate(n)                       # exact rollback
"""

from __future__ import annotations

import ctypes as C
from dataclasses import dataclass

import numpy as np
import torch

from . import _lib
from .bundle import Bundle, as_bundle

_NP_DT = {np.dtype(np.float32): _lib.F32, np.dtype(np.float16): _lib.F16, np.dtype(np.int32): _lib.I32}
_INT_NUMBERS = ("d_model", "vocab", "routes", "bits", "mem_dim", "kv_heads", "head_dim", "q_heads", "ssm_dim",
                "sketch_k", "shortlist_cap")
_FLOAT_NUMBERS = ("router_eps", "draft_eps", "mem_eps", "ssm_eps", "softmax_scale", "sink_logit")


def _raise(status: int, what: str) -> None:
    """A failed call as the C++ class reports it: RuntimeError (TORCH_CHECK / std::runtime_error)."""
    if status == _lib.OK:
        return
    msg = (_lib.library(require_device=False).lng_last_error() or b"").decode(errors="replace")
    raise RuntimeError(f"{what}: {msg}")


def _as_array(a) -> np.ndarray:
    """A bundle tensor as a C-contiguous numpy array of a dtype the C ABI takes: fp32 / fp16 kept, bf16 and
    other floats as fp32, integers (uint16 sketch ids, uint32 counts) as int32 clamped at 2^31 - 1
    (``drafting/export_drafter.py`` ``Bundle.tensors``)."""
    if isinstance(a, torch.Tensor):
        a = a.detach().cpu()
        a = a.float() if a.dtype == torch.bfloat16 else a
        a = a.numpy()
    a = np.asarray(a)
    if a.dtype.kind in "ui" and a.dtype != np.int32:
        a = np.minimum(a.astype(np.int64), np.iinfo(np.int32).max).astype(np.int32)
    elif a.dtype not in _NP_DT:
        a = a.astype(np.float32)
    return np.ascontiguousarray(a)


class Drafter:
    """``ext.Drafter`` (``drafting/cpu/drafter.cpp:582-595``) on the GPU.  ``threads`` is accepted for the
    signature; the per-token work runs on the device.  Every call holds the object's own lock in C."""

    def __init__(self, tensors: dict, numbers: dict, ngrams, threads: int = 1, *,
                 act_dtype: torch.dtype = torch.float32, device: torch.device | str | None = None):
        for k in _INT_NUMBERS + _FLOAT_NUMBERS + ("router_ssm", "query_ssm"):
            if k not in numbers:
                raise RuntimeError(f"missing number: {k}")
        self.device = torch.device(device) if device is not None else torch.device("cuda", torch.cuda.current_device())
        self.R = int(numbers["routes"])
        self.V = int(numbers["vocab"])
        self.cap = int(numbers["shortlist_cap"])
        self.K = int(numbers["sketch_k"])
        self.threads = int(threads)
        nums = _lib.DrafterNumbers()
        for k in _INT_NUMBERS:
            setattr(nums, k, int(numbers[k]))
        for k in _FLOAT_NUMBERS:
            setattr(nums, k, float(numbers[k]))
        nums.router_ssm = int(float(numbers["router_ssm"]) != 0.0)
        nums.query_ssm = int(float(numbers["query_ssm"]) != 0.0)
        orders = [int(n) for n in ngrams]
        if not 1 <= len(orders) <= _lib.MAX_ORDERS:
            raise RuntimeError(f"ngrams must hold 1 .. {_lib.MAX_ORDERS} orders")
        nums.n_orders = len(orders)
        for i, n in enumerate(orders):
            nums.orders[i] = n
        self._keep = []
        arr = (_lib.Array * len(tensors))()
        for i, (name, t) in enumerate(tensors.items()):
            a = _as_array(t)
            self._keep.append(a)
            arr[i].name = name.encode()
            arr[i].data_host = a.ctypes.data
            arr[i].dtype = _NP_DT[a.dtype]
            arr[i].ndim = a.ndim
            for j, s in enumerate(a.shape[:4]):
                arr[i].shape[j] = s
        handle = C.c_void_p()
        lib = _lib.library()
        with _lib.on_device(self.device):
            _raise(lib.lng_drafter_create(C.byref(nums), arr, len(tensors), _lib.dtype_code(act_dtype),
                                          C.byref(handle)), "Drafter")
        self._keep = None  # the library holds device copies
        self._h = handle

    def __del__(self):
        h = getattr(self, "_h", None)
        if h is not None and h.value:
            try:
                _lib.library(require_device=False).lng_drafter_destroy(h)
            except Exception:
                pass
            self._h = None

    # ------------------------------------------------------------------ the extension's methods
    def reset(self) -> None:
        _raise(_lib.library().lng_drafter_reset(self._h), "reset")

    def length(self) -> int:
        return int(_lib.library().lng_drafter_length(self._h))

    def truncate(self, n: int) -> None:
        _raise(_lib.library().lng_drafter_truncate(self._h, int(n)), "truncate")

    def committed_codes(self) -> torch.Tensor:
        out = np.zeros((self.length(), self.R), np.uint8)
        _raise(_lib.library().lng_drafter_committed_codes(self._h, out.ctypes.data), "committed_codes")
        return torch.from_numpy(out)

    def commit(self, tokens, codes: torch.Tensor | None = None) -> None:
        toks = np.ascontiguousarray(np.asarray([int(x) for x in tokens], np.int64))
        cp = None
        if codes is not None:
            cc = np.ascontiguousarray(np.asarray(torch.as_tensor(codes).to(torch.int32)))
            if cc.ndim != 2 or cc.shape != (len(toks), self.R):
                raise RuntimeError("codes must be [n, R]")
            cp = cc.ctypes.data
        with _lib.on_device(self.device):
            _raise(_lib.library().lng_drafter_commit(self._h, toks.ctypes.data, len(toks), cp), "commit")

    def draft(self, gamma: int, hyp, topk: int = 3, last_codes: bool = False):
        """(tokens int64 [gamma], top-k ids int64 [gamma, topk] (-1 padded), top-k logits float32
        [gamma, topk] (-inf padded), codes uint8 [len(hyp) + advanced drafts, R])."""
        gamma, k = int(gamma), int(topk)
        if gamma < 0 or k < 1:
            raise RuntimeError("need gamma >= 0 and topk >= 1")
        hypa = np.ascontiguousarray(np.asarray([int(x) for x in hyp], np.int64))
        toks = np.zeros(max(gamma, 1), np.int64)
        ids = np.full((max(gamma, 1), k), -1, np.int64)
        lg = np.full((max(gamma, 1), k), -np.inf, np.float32)
        n_codes = len(hypa) + (gamma if last_codes else max(gamma - 1, 0))
        codes = np.zeros((max(n_codes, 1), self.R), np.uint8)
        with _lib.on_device(self.device):
            _raise(_lib.library().lng_drafter_draft(self._h, gamma, hypa.ctypes.data if len(hypa) else None, len(hypa),
                                                    k, int(bool(last_codes)), toks.ctypes.data, ids.ctypes.data,
                                                    lg.ctypes.data, codes.ctypes.data), "draft")
        return (torch.from_numpy(toks[:gamma]), torch.from_numpy(ids[:gamma]), torch.from_numpy(lg[:gamma]),
                torch.from_numpy(codes[:n_codes]))

    def trace_columns(self, full: bool) -> int:
        """Columns S of ``trace``: the vocabulary, or ``shortlist_cap`` with a sketch (drafter.cpp:333-334)."""
        return self.V if (full or self.cap <= 0 or self.K <= 0) else self.cap

    def trace(self, tokens, codes: torch.Tensor | None = None, full: bool = False):
        """Teacher-forced pass from an empty state: (codes uint8 [T, R], ids int64 [T, S], logits float32
        [T, S]) with S = ``trace_columns(full)``."""
        toks = np.ascontiguousarray(np.asarray([int(x) for x in tokens], np.int64))
        T = len(toks)
        S = self.trace_columns(full)
        cp = None
        if codes is not None:
            cc = np.ascontiguousarray(np.asarray(torch.as_tensor(codes).to(torch.int32)))
            if cc.ndim != 2 or cc.shape != (T, self.R):
                raise RuntimeError("codes must be [T, R]")
            cp = cc.ctypes.data
        oc = np.zeros((T, self.R), np.uint8)
        oi = np.full((T, S), -1, np.int64)
        ol = np.full((T, S), -np.inf, np.float32)
        if T:
            with _lib.on_device(self.device):
                _raise(_lib.library().lng_drafter_trace(self._h, toks.ctypes.data, T, cp, int(bool(full)), S,
                                                        oc.ctypes.data, oi.ctypes.data, ol.ctypes.data), "trace")
        return torch.from_numpy(oc), torch.from_numpy(oi), torch.from_numpy(ol)

    # ------------------------------------------------------------------ beyond the extension
    def draft_batch(self, prefix: torch.Tensor, gamma: int, out: torch.Tensor | None = None) -> torch.Tensor:
        """Greedy drafts for independent sequences: prefix [nseq, plen] int64 (device) -> [nseq, gamma]
        (the drafter's own committed state is not used or changed)."""
        if prefix.dim() != 2:
            raise ValueError("prefix must be [nseq, plen]")
        prefix = prefix.to(device=self.device, dtype=torch.int64).contiguous()
        nseq, plen = prefix.shape
        if out is None:
            out = torch.empty(nseq, gamma, device=self.device, dtype=torch.int64)
        with _lib.on_device(self.device):
            _lib.check(_lib.library().lng_drafter_draft_batch(self._h, prefix.data_ptr(), nseq, plen, int(gamma),
                                                              out.data_ptr(), _lib.stream_ptr()), "draft_batch")
        return out


def bundle_numbers(config: dict, shortlist_cap: int | None = None) -> dict:
    """The ``numbers`` dictionary ``CppDrafter`` passes to the extension (``drafting/cpu_drafter.py:343-350``)."""
    c = config
    cap = int(c.get("shortlist_cap", 0) if shortlist_cap is None else shortlist_cap)
    num = {k: float(c[k]) for k in ("d_model", "vocab", "routes", "bits", "mem_dim", "kv_heads", "head_dim",
                                    "q_heads", "ssm_dim", "sketch_k", "norm_eps", "ssm_eps", "router_eps",
                                    "draft_eps", "mem_eps", "softmax_scale", "sink_logit")}
    num["shortlist_cap"] = float(cap)
    num["router_ssm"] = float(c["router_kind"] == "embed2_ssm")
    num["query_ssm"] = float(bool(c.get("query_ssm", False)))
    return num


@dataclass
class DraftOut:
    tokens: list
    topk_ids: np.ndarray     # int64 [gamma, k] (-1 = fewer candidates)
    topk_logits: np.ndarray  # float32 [gamma, k]
    codes: np.ndarray        # uint8 [len(hyp) + advanced drafts, R]

    @property
    def runner_up(self) -> int:
        return int(self.topk_ids[0, 1]) if self.topk_ids.shape[1] > 1 else -1


class GpuDrafter:
    """Same API as the reference's RefDrafter / CppDrafter; every step runs on the GPU (``Drafter`` core)."""

    name = "b200"

    def __init__(self, bundle: Bundle | str, topk: int = 3, shortlist_cap: int | None = None, threads: int = 1,
                 act_dtype: torch.dtype = torch.float32, device: torch.device | str | None = None):
        b = as_bundle(bundle)
        c = self.cfg = dict(b.config)
        self.topk = int(topk)
        self.R = int(c["routes"])
        self.V = int(c["vocab"])
        self._core = Drafter(b.arrays, bundle_numbers(c, shortlist_cap), [int(n) for n in c["ngrams"]], threads,
                             act_dtype=act_dtype, device=device)
        self.device = self._core.device
        self._tokens: list = []

    # ------------------------------------------------------------------ state
    @property
    def length(self) -> int:
        return self._core.length()

    @property
    def tokens(self) -> list:
        return list(self._tokens)

    def committed_codes(self) -> np.ndarray:
        return self._core.committed_codes().numpy()

    def reset(self) -> None:
        self._core.reset()
        self._tokens = []

    def truncate(self, length: int) -> None:
        if not 0 <= length <= self.length:
            raise ValueError(f"cannot truncate to {length} (length {self.length})")
        self._core.truncate(int(length))
        del self._tokens[length:]

    def commit(self, tokens, codes=None) -> None:
        toks = [int(x) for x in tokens]
        if codes is not None and np.asarray(codes).shape != (len(toks), self.R):
            raise ValueError("codes must be [n, R]")
        ct = None if codes is None else torch.as_tensor(np.asarray(codes), dtype=torch.int32)
        self._core.commit(toks, ct)
        self._tokens.extend(toks)

    # ------------------------------------------------------------------ drafting
    def draft(self, gamma: int, hyp=(), topk: int | None = None, last_codes: bool = False) -> DraftOut:
        toks, ids, lg, codes = self._core.draft(int(gamma), [int(x) for x in hyp], int(topk or self.topk),
                                                bool(last_codes))
        return DraftOut([int(x) for x in toks.tolist()], ids.numpy(), lg.numpy(), codes.numpy().astype(np.uint8))

    def trace(self, tokens, codes=None, full: bool = False):
        """Teacher-forced pass from an empty state: codes [T, R], ids [T, S], logits [T, S] (S = the
        vocabulary, or shortlist_cap with a sketch unless ``full``)."""
        ct = None if codes is None else torch.as_tensor(np.asarray(codes), dtype=torch.int32)
        c, i, lg = self._core.trace([int(x) for x in tokens], ct, bool(full))
        return c.numpy().astype(np.uint8), i.numpy(), lg.numpy()

    def draft_batch(self, prefix: torch.Tensor, gamma: int, out: torch.Tensor | None = None) -> torch.Tensor:
        """Greedy drafts for independent sequences: prefix [nseq, plen] int64 (device) -> [nseq, gamma]."""
        return self._core.draft_batch(prefix, gamma, out)


def make_drafter(bundle, impl: str = "b200", **kw):
    """``impl``: only ``b200`` here; the reference's ``make_drafter`` gains a branch that calls this."""
    if impl != "b200":
        raise ValueError(f"unknown drafter impl {impl!r}")
    return GpuDrafter(bundle, **kw)


class OnlineCounts:
    """``drafting/drafters.py:117-143``: in-context (order, route, row) -> next-token counts from one
    record's verified pairs, mixed into a drafter's distribution on the GPU (``lng_online_counts_mix``:
    the same fp32 results as the reference).  ``codes`` [T, R] and ``x`` [T] are the record's codes and
    tokens; ``route_chunk`` is accepted for the reference's signature (the kernel compares every route
    at once)."""

    def __init__(self, codes: torch.Tensor, x: torch.Tensor, orders, bits: int, vocab: int, kappa: float = 1.0,
                 route_chunk: int = 32):
        if codes.dim() != 2 or x.dim() != 1 or codes.shape[0] != x.shape[0]:
            raise ValueError("codes must be [T, R] and x [T]")
        self.codes = codes.to(torch.int64).contiguous()
        self.x = x.to(device=self.codes.device, dtype=torch.int64).contiguous()
        self.nxt = self.x[1:]
        self.orders, self.bits, self.vocab, self.kappa, self.rc = tuple(int(n) for n in orders), int(bits), \
            int(vocab), float(kappa), int(route_chunk)
        self.routes = self.codes.shape[1]
        self._orders = (C.c_int32 * len(self.orders))(*self.orders)

    def mix(self, p: torch.Tensor, win: torch.Tensor, real: torch.Tensor, deadline: torch.Tensor) -> torch.Tensor:
        """p [N, V]; only pairs t <= deadline[j] (token t+1 verified for row j) count."""
        dev = self.codes.device
        if not dev.type == "cuda":
            raise RuntimeError("OnlineCounts runs on the GPU: give it device tensors")
        n_rows, W = win.shape[0], win.shape[1]
        p = p.to(device=dev, dtype=torch.float32).contiguous()
        win = win.to(device=dev, dtype=torch.int64).contiguous()
        real = real.to(device=dev, dtype=torch.uint8).contiguous()
        deadline = deadline.to(device=dev, dtype=torch.int64).reshape(n_rows).contiguous()
        out = torch.empty_like(p)
        with _lib.on_device(dev):
            _lib.check(_lib.library().lng_online_counts_mix(
                self.codes.data_ptr(), self.codes.shape[0], self.routes, self._orders, len(self.orders), self.bits,
                self.x.data_ptr(), win.data_ptr(), real.data_ptr(), n_rows, W, deadline.data_ptr(), p.data_ptr(),
                p.shape[1], self.kappa, out.data_ptr(), _lib.stream_ptr()), "online counts")
        return out

