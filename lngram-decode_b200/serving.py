"""Serving memory tables from host RAM on the GPU (the reference's ``serving/``), zero-copy.

* ``permute_table`` / ``permute_tables`` -- the serving row layout of ``serving/layout.py:26-52``: within
  each route's block the n-gram address is stored with the CURRENT code least significant, so the rows a
  next step may read are contiguous.  Runs on the GPU (``lng_serving_permute``) for device tensors and
  for pinned host tensors (read and written through their mapped addresses).
* ``HostTable`` -- one memory layer's serving-layout tables in pinned host memory, mapped into the
  device address space (``lng_host_map``): tables larger than HBM stay in host RAM.
* ``ZeroCopyGather`` -- a ``decode_step`` row provider (``ffnmem/infer.py:207-251``,
  ``row_provider(pos, state, codes_new) -> route tokens [B, n, R, Dt]``) whose kernel reads each needed
  row straight from the mapped host tables across PCIe (``lng_lookup_serving_rows``): the transfer mode
  the reference leaves as ``NotImplementedError`` (``serving/prefetch.py:579-586``).

The rows equal the v2 lookup's (``serving/layout.py:70-84``; the zero rows of n-grams that start before
position 0 included), so ``seams.memory_step(..., route_tokens=rows)`` gives the table path's output.
"""

from __future__ import annotations

import ctypes as C

import torch
from torch import Tensor

from . import _lib
from ._lib import check, ptr, stream_ptr


def _device_address(t: Tensor) -> int:
    """A pointer kernels can use for ``t``: its own for device tensors, the mapped one for pinned host."""
    if t.is_cuda:
        return t.data_ptr()
    if not t.is_pinned():
        raise ValueError("host tables must be in pinned memory (Tensor.pin_memory())")
    dev = C.c_void_p()
    check(_lib.library().lng_host_map(t.data_ptr(), t.numel() * t.element_size(), C.byref(dev)), "host map")
    return dev.value


def permute_table(weight: Tensor, routes: int, order: int, bits: int) -> Tensor:
    """v2 table [R * A^order, D] -> the serving layout (``serving/layout.py:37-42``): row j of a route
    block holds the v2 row ``reverse_digits(j)``.  Device tensors stay on their device; pinned host
    tensors give a pinned host result (the GPU reads and writes them over PCIe)."""
    w = weight.detach().contiguous()
    if w.shape[0] != routes * (1 << bits) ** order:
        raise ValueError("weight rows must be routes * 2**(bits * order)")
    out = torch.empty_like(w) if w.is_cuda else torch.empty(w.shape, dtype=w.dtype, pin_memory=True)
    if not w.is_cuda and not w.is_pinned():
        w = w.pin_memory()
    dev = w.device if w.is_cuda else torch.device("cuda", torch.cuda.current_device())
    with _lib.on_device(dev):
        check(_lib.library().lng_serving_permute(_device_address(w), _device_address(out), _lib.dtype_code(w.dtype),
                                                 routes, order, bits, w.shape[1], stream_ptr()), "serving permute")
        if not w.is_cuda:
            torch.cuda.current_stream().synchronize()
    return out


def permute_tables(module) -> dict:
    """Serving-layout copies of every order's table of a ``RouteNgramMemoryV2`` (``serving/layout.py:45-52``)."""
    return {n: permute_table(module.tables[f"ngram_{n}"].weight, module.num_routes, n, module.bits_per_route)
            for n in module.ngrams}


class HostTable:
    """One memory layer's tables in the serving layout, held in pinned host memory and mapped for the GPU."""

    def __init__(self, tables: dict, routes: int, ngrams, bits: int):
        self.ngrams = tuple(int(n) for n in ngrams)
        self.routes, self.bits = int(routes), int(bits)
        self.tables = {}
        for n in self.ngrams:
            t = tables[n]
            if t.is_cuda:
                t = t.cpu()
            self.tables[n] = t.contiguous() if t.is_pinned() else t.contiguous().pin_memory()
        dims = {t.shape[1] for t in self.tables.values()}
        dts = {t.dtype for t in self.tables.values()}
        if len(dims) != 1 or len(dts) != 1:
            raise ValueError("all orders must share the row width and dtype")
        self.dim = dims.pop()
        self.dtype = dts.pop()
        self._addr = {n: _device_address(t) for n, t in self.tables.items()}

    @classmethod
    def from_module(cls, module) -> "HostTable":
        """The serving-layout copy of a ``RouteNgramMemoryV2``'s tables, permuted on the GPU and moved to host."""
        return cls({n: t.cpu() for n, t in permute_tables(module).items()}, module.num_routes, module.ngrams,
                   module.bits_per_route)

    @property
    def nbytes(self) -> int:
        return sum(t.numel() * t.element_size() for t in self.tables.values())

    def descriptor(self) -> _lib.Tables:
        t = _lib.Tables()
        t.n_orders = len(self.ngrams)
        for i, n in enumerate(self.ngrams):
            t.orders[i] = n
            t.tables[i] = self._addr[n]
        t.table_dtype = _lib.dtype_code(self.dtype)
        t.bits = self.bits
        t.num_routes = self.routes
        t.memory_dim = self.dim
        return t


class ZeroCopyGather:
    """Row provider reading route tokens straight from host RAM: ``provider(pos, state, codes_new)`` with
    ``state.codes`` the cached codes ([B, max_len, R] of this layer, or a dict by layer position as the
    reference's ``DecodeState``) and ``state.length`` the cached length.  ``host`` is a ``HostTable`` or a
    dict {layer position: HostTable}."""

    def __init__(self, host, device: torch.device | str | None = None):
        self.host = host
        self.device = torch.device(device) if device is not None else torch.device("cuda", torch.cuda.current_device())
        self.rows_read = 0

    def _table(self, pos: int) -> HostTable:
        return self.host[pos] if isinstance(self.host, dict) else self.host

    def __call__(self, pos: int, state, codes_new: Tensor) -> Tensor:
        ht = self._table(pos)
        codes_all = state.codes[pos] if isinstance(state.codes, dict) else state.codes
        L = int(state.length)
        b, n, r = codes_new.shape
        hist = max(ht.ngrams) - 1
        h0 = min(L, hist)
        ctx = torch.cat((codes_all[:, L - h0:L].to(self.device, torch.uint8),
                         codes_new.to(self.device, torch.uint8)), 1).contiguous()
        out = torch.empty(b, n, r, len(ht.ngrams) * ht.dim, device=self.device, dtype=ht.dtype)
        with _lib.on_device(self.device):
            check(_lib.library().lng_lookup_serving_rows(ht.descriptor(), ptr(ctx), _lib.U8, b, h0 + n, n, ptr(out),
                                                         stream_ptr()), "zero-copy gather")
        self.rows_read += b * n * r * len(ht.ngrams)
        return out
