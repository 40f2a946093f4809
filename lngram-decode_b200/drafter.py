"""GPU drafter with the API of the reference's ``RefDrafter`` / ``CppDrafter``
(``drafting/cpu_drafter.py:76-389``) over the C ABI's ``lng_drafter_*`` (``drafting/cpu/drafter.cpp``).

    d = GpuDrafter(bundle)              # bundle path, lngram_b200 Bundle, or the reference's Bundle
    d.commit(prompt_tokens)             # verified tokens (optionally with the target's codes)
    out = d.draft(4)                    # out.tokens, out.topk_ids [4, k], out.topk_logits, out.codes
    d.truncate(n)                       # exact rollback

``act_dtype=torch.float32`` (default) computes in fp32 like the reference drafter;
``torch.bfloat16`` keeps the embedding, tables and folded readout in bf16 (tensor cores).
``draft_batch`` drafts for many independent sequences at once (the reference API is batch-1).
"""

from __future__ import annotations

import ctypes as C
from dataclasses import dataclass

import numpy as np
import torch

from . import _lib
from ._lib import check
from .bundle import Bundle, as_bundle

_NP_DT = {np.dtype(np.float32): _lib.F32, np.dtype(np.float16): _lib.F16, np.dtype(np.int32): _lib.I32}


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
    """Same API as the reference's RefDrafter / CppDrafter; every step runs on the GPU."""

    name = "b200"

    def __init__(self, bundle: Bundle | str, topk: int = 3, shortlist_cap: int | None = None, threads: int = 1,
                 act_dtype: torch.dtype = torch.float32, device: torch.device | str | None = None):
        b = as_bundle(bundle)
        c = self.cfg = dict(b.config)
        self.topk = int(topk)
        self.R = int(c["routes"])
        self.V = int(c["vocab"])
        self.device = torch.device(device) if device is not None else torch.device("cuda", torch.cuda.current_device())
        cap = int(c.get("shortlist_cap", 0) if shortlist_cap is None else shortlist_cap)
        nums = _lib.DrafterNumbers()
        for k in ("d_model", "vocab", "routes", "bits", "mem_dim", "kv_heads", "head_dim", "q_heads", "ssm_dim",
                  "sketch_k"):
            setattr(nums, k, int(c[k]))
        nums.shortlist_cap = cap
        for k in ("router_eps", "draft_eps", "mem_eps", "ssm_eps", "softmax_scale", "sink_logit"):
            setattr(nums, k, float(c[k]))
        nums.router_ssm = int(c["router_kind"] == "embed2_ssm")
        nums.query_ssm = int(bool(c.get("query_ssm", False)))
        ngrams = [int(n) for n in c["ngrams"]]
        nums.n_orders = len(ngrams)
        for i, n in enumerate(ngrams):
            nums.orders[i] = n
        keep = []
        arr = (_lib.Array * len(b.arrays))()
        for i, (name, a) in enumerate(b.arrays.items()):
            a = np.ascontiguousarray(a)
            if a.dtype not in _NP_DT:
                a = np.ascontiguousarray(a.astype(np.int32 if a.dtype.kind in "ui" else np.float32))
            keep.append(a)
            arr[i].name = name.encode()
            arr[i].data_host = a.ctypes.data
            arr[i].dtype = _NP_DT[a.dtype]
            arr[i].ndim = a.ndim
            for j, s in enumerate(a.shape[:4]):
                arr[i].shape[j] = s
        handle = C.c_void_p()
        lib = _lib.library()
        with torch.cuda.device(self.device):
            check(lib.lng_drafter_create(C.byref(nums), arr, len(b.arrays), _lib.dtype_code(act_dtype),
                                         C.byref(handle)), "drafter create")
        self._h = handle
        self._tokens: list = []

    def __del__(self):
        h = getattr(self, "_h", None)
        if h is not None and h.value:
            try:
                _lib.library(require_device=False).lng_drafter_destroy(h)
            except Exception:
                pass
            self._h = None

    # ------------------------------------------------------------------ state
    @property
    def length(self) -> int:
        return int(_lib.library().lng_drafter_length(self._h))

    @property
    def tokens(self) -> list:
        return list(self._tokens)

    def committed_codes(self) -> np.ndarray:
        out = np.zeros((self.length, self.R), np.uint8)
        check(_lib.library().lng_drafter_committed_codes(self._h, out.ctypes.data), "committed_codes")
        return out

    def reset(self) -> None:
        check(_lib.library().lng_drafter_reset(self._h), "reset")
        self._tokens = []

    def truncate(self, length: int) -> None:
        if not 0 <= length <= self.length:
            raise ValueError(f"cannot truncate to {length} (length {self.length})")
        check(_lib.library().lng_drafter_truncate(self._h, int(length)), "truncate")
        del self._tokens[length:]

    def commit(self, tokens, codes=None) -> None:
        toks = np.ascontiguousarray(np.asarray([int(x) for x in tokens], np.int64))
        cp = None
        if codes is not None:
            cc = np.ascontiguousarray(np.asarray(codes).astype(np.int32))
            if cc.shape != (len(toks), self.R):
                raise ValueError("codes must be [n, R]")
            cp = cc.ctypes.data
        with torch.cuda.device(self.device):
            check(_lib.library().lng_drafter_commit(self._h, toks.ctypes.data, len(toks), cp), "commit")
        self._tokens.extend(int(x) for x in toks)

    # ------------------------------------------------------------------ drafting
    def draft(self, gamma: int, hyp=(), topk: int | None = None, last_codes: bool = False) -> DraftOut:
        k = int(topk or self.topk)
        hypa = np.ascontiguousarray(np.asarray([int(x) for x in hyp], np.int64))
        toks = np.zeros(max(gamma, 1), np.int64)
        ids = np.full((max(gamma, 1), k), -1, np.int64)
        lg = np.full((max(gamma, 1), k), -np.inf, np.float32)
        n_codes = len(hypa) + (gamma if last_codes else max(gamma - 1, 0))
        codes = np.zeros((max(n_codes, 1), self.R), np.uint8)
        with torch.cuda.device(self.device):
            check(_lib.library().lng_drafter_draft(self._h, int(gamma), hypa.ctypes.data if len(hypa) else None,
                                                   len(hypa), k, int(bool(last_codes)), toks.ctypes.data,
                                                   ids.ctypes.data, lg.ctypes.data, codes.ctypes.data), "draft")
        return DraftOut([int(x) for x in toks[:gamma]], ids[:gamma], lg[:gamma], codes[:n_codes])

    def trace(self, tokens, codes=None, full: bool = False):
        """Teacher-forced pass from an empty state (full vocabulary): codes [T, R], ids [T, V], logits [T, V]."""
        toks = np.ascontiguousarray(np.asarray([int(x) for x in tokens], np.int64))
        T = len(toks)
        cp = None
        if codes is not None:
            cc = np.ascontiguousarray(np.asarray(codes).astype(np.int32))
            cp = cc.ctypes.data
        oc = np.zeros((T, self.R), np.uint8)
        oi = np.zeros((T, self.V), np.int64)
        ol = np.zeros((T, self.V), np.float32)
        with torch.cuda.device(self.device):
            check(_lib.library().lng_drafter_trace(self._h, toks.ctypes.data, T, cp, int(bool(full)), self.V,
                                                   oc.ctypes.data, oi.ctypes.data, ol.ctypes.data), "trace")
        return oc, oi, ol

    def draft_batch(self, prefix: torch.Tensor, gamma: int, out: torch.Tensor | None = None) -> torch.Tensor:
        """Greedy drafts for independent sequences: prefix [nseq, plen] int64 (device) -> [nseq, gamma]."""
        if prefix.dim() != 2:
            raise ValueError("prefix must be [nseq, plen]")
        prefix = prefix.to(device=self.device, dtype=torch.int64).contiguous()
        nseq, plen = prefix.shape
        if out is None:
            out = torch.empty(nseq, gamma, device=self.device, dtype=torch.int64)
        with torch.cuda.device(self.device):
            check(_lib.library().lng_drafter_draft_batch(self._h, prefix.data_ptr(), nseq, plen, int(gamma),
                                                         out.data_ptr(), _lib.stream_ptr()), "draft_batch")
        return out


def make_drafter(bundle, impl: str = "b200", **kw):
    """``impl``: only ``b200`` here; the reference's ``make_drafter`` gains a branch that calls this."""
    if impl != "b200":
        raise ValueError(f"unknown drafter impl {impl!r}")
    return GpuDrafter(bundle, **kw)
