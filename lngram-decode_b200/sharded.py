"""Route-sharded memory layer across GPUs (one process per GPU, NCCL over NVLink).

Each rank holds the table rows of a contiguous block of routes [r0, r1) and the router rows of those
routes.  A forward over positions [B, T] (hidden states replicated on every rank):

1. codes of the local routes (the router's rows r0*bits .. r1*bits);
2. the folded query (replicated) and the fused gather + sink attention over the local routes in
   partial mode: the online-softmax state (m, l, u) of the shard, the sink seeded on rank 0 only;
   for 16-bit tables and bf16 activations the kernel writes (u, l) directly as one bf16 pack
   [M, QH, Dt + 1], every shard offset by the sink logit b0;
3. ``all_reduce(MAX)`` of m, then each rank rescales (l, u) by exp(m_local - m_glob) -- for
   kernel-written packs only the rows whose offset differs from the maximum;
4. ``reduce_scatter(SUM)`` of the packed buffer (bf16 for bf16 layers) by whole-sequence blocks
   (B / world sequences per rank), so the short conv needs no halo;
5. on the local block: u / l, the folded output map, the conv finish -> out [B / world, T, d].

Steps 3-5 are the exact decomposition of the reference's streaming readout over route chunks
(``ffnmem/memory/lngram_v2.py:1944-2070``: running max, rescaled sums, final division) with one
chunk per rank.  The two collectives are the only data-path communication.
"""

from __future__ import annotations

import math

import torch
import torch.distributed as dist
from torch import Tensor

from . import _lib
from ._lib import check, ptr, stream_ptr
from .memory import LngramMemory


def route_bounds(routes: int, world: int) -> list[tuple[int, int]]:
    """Contiguous route blocks, the first ``routes % world`` ranks one route larger."""
    base, extra = divmod(routes, world)
    out, start = [], 0
    for r in range(world):
        n = base + (1 if r < extra else 0)
        out.append((start, start + n))
        start += n
    return out


class GridPlace:
    """A rank's place in a route x data grid of ``world`` ranks: ``route_shards`` consecutive ranks hold the
    route blocks of one layer copy and process the same block of sequences; the ``data_shards`` such groups
    split the batch by whole sequences (data parallel, no exchange between groups)."""

    def __init__(self, rank: int, world: int, route_shards: int, group=None, group_m=None):
        self.route_index, self.route_shards = rank % route_shards, route_shards
        self.data_index, self.data_shards = rank // route_shards, world // route_shards
        self.group, self.group_m = group, group_m


def route_data_grid(world: int, route_shards: int, rank: int) -> GridPlace:
    """This rank's ``GridPlace`` and the communicators of its route group (one for the state exchange,
    one for the max all-reduce, so the two do not queue behind each other).  Collective: every rank
    creates every group, in the same order, as torch.distributed requires."""
    if route_shards < 1 or world % route_shards:
        raise ValueError(f"route_shards={route_shards} must divide the world size {world}")
    groups = []
    for d in range(world // route_shards):
        ranks = list(range(d * route_shards, (d + 1) * route_shards))
        groups.append((dist.new_group(ranks), dist.new_group(ranks)) if route_shards > 1 else (None, None))
    g, gm = groups[rank // route_shards]
    return GridPlace(rank, world, route_shards, g, gm)


def all_reduce_max(t: Tensor, group=None) -> Tensor:
    if dist.is_initialized() and dist.get_world_size(group) > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX, group=group)
    return t


def reduce_scatter_rows(t: Tensor, group=None) -> Tensor:
    """SUM over ranks of ``t`` [N, ...]; rank r receives rows r*N/world .. (r+1)*N/world."""
    world = dist.get_world_size(group) if dist.is_initialized() else 1
    if world == 1:
        return t
    if t.shape[0] % world:
        raise ValueError("rows must split evenly across ranks")
    out = torch.empty((t.shape[0] // world,) + tuple(t.shape[1:]), device=t.device, dtype=t.dtype)
    dist.reduce_scatter_tensor(out, t.contiguous(), op=dist.ReduceOp.SUM, group=group)
    return out


class RouteShardedMemory:
    """One rank's share of a route-sharded ``LngramMemory``."""

    def __init__(self, full: LngramMemory, rank: int, world: int, group=None, routes_total: int | None = None,
                 group_m=None):
        """``full`` holds every route (its rows of this rank are sliced out), or -- with
        ``routes_total`` -- only this rank's block of routes already (its sink logit must then be the
        whole layer's, log(routes_total (1 - mass) / mass)).  ``rank`` / ``world`` are the position and
        size of the route group ``group`` (the default group when None); ``group_m`` is a second
        communicator over the same ranks for the max all-reduce (``route_data_grid`` makes both; without
        it one is created here, collectively over ``group``'s ranks)."""
        m = full.module
        self.rank, self.world, self.group = int(rank), int(world), group
        self.R_total = int(routes_total) if routes_total is not None else m.num_routes
        self.bounds = route_bounds(self.R_total, world)
        self.r0, self.r1 = self.bounds[rank]
        self.full = full
        dev = m.readout_q_proj.weight.device
        pre_sliced = routes_total is not None
        if pre_sliced and m.num_routes != self.r1 - self.r0:
            raise ValueError(f"the local module holds {m.num_routes} routes, rank {rank} owns {self.r1 - self.r0}")
        # the rank's rows of every order table (route-major layout: contiguous) and of the router
        self.tables = {}
        for n in m.ngrams:
            span = m.alphabet_size ** n
            w = m.tables[f"ngram_{n}"].weight.detach()
            self.tables[n] = w if pre_sliced else w[self.r0 * span:self.r1 * span].contiguous()
        rw = full.router.weight.detach()
        self.router_w = (rw if pre_sliced else rw[self.r0 * full.bits:self.r1 * full.bits]).float().contiguous()
        self.router_split = None
        if full.bits <= 6 and self.router_w.shape[1] % 64 == 0:
            self.router_split = torch.empty(self.router_w.shape[0], 3 * self.router_w.shape[1], device=dev,
                                            dtype=torch.bfloat16)
            check(_lib.library().lng_router_prepare(ptr(self.router_w), self.router_w.shape[0], self.router_w.shape[1],
                                                    ptr(self.router_split), stream_ptr()), "router split")
        self.pack_dtype = torch.bfloat16 if m._act() == torch.bfloat16 else torch.float32
        # 16-bit tables + bf16 activations: the attention kernel writes the bf16 pack itself
        self.packed = self.pack_dtype == torch.bfloat16 and self.tables[m.ngrams[0]].dtype in (torch.bfloat16,
                                                                                              torch.float16)
        # b0 = log(R (1 - mass) / mass) of the whole layer (the local module's own is of its R_local)
        mass = m.sink_initial_active_mass
        self.sink_logit = math.log(self.R_total * (1.0 - mass) / mass)
        # the max all-reduce runs on its own communicator, so it does not queue behind the previous
        # group's reduce-scatter (collectives of one communicator run in order on one stream);
        # created collectively, so every rank constructs its shard at the same point
        self.group_m = group_m
        if group_m is None and world > 1 and dist.is_initialized() and dist.get_world_size(group) > 1:
            ranks = dist.get_process_group_ranks(group) if group is not None else list(range(dist.get_world_size()))
            self.group_m = dist.new_group(ranks)
        self.ss = {}
        self.dev = dev

    def _tables_desc(self):
        m = self.full.module
        t = _lib.Tables()
        t.n_orders = len(m.ngrams)
        for i, n in enumerate(m.ngrams):
            t.orders[i] = n
            t.tables[i] = self.tables[n].data_ptr()
        t.table_dtype = _lib.dtype_code(self.tables[m.ngrams[0]].dtype)
        t.bits = m.bits_per_route
        t.num_routes = self.r1 - self.r0
        t.memory_dim = m.memory_dim
        if not self.ss:
            desc = t
            self.ss = {n: torch.empty(self.tables[n].shape[0], device=self.dev, dtype=torch.float32) for n in m.ngrams}
            arr = (_lib.C.c_void_p * _lib.MAX_ORDERS)(*([self.ss[n].data_ptr() for n in m.ngrams] +
                                                        [None] * (_lib.MAX_ORDERS - len(m.ngrams))))
            check(_lib.library().lng_table_row_ss(desc, arr, stream_ptr()), "row sums of squares")
        for i, n in enumerate(m.ngrams):
            t.row_ss[i] = self.ss[n].data_ptr()
        return t

    @torch.no_grad()
    def forward(self, h: Tensor, router_x: Tensor, chunks: int = 1) -> Tensor:
        """h, router_x [B, T, *] (the same on every rank) -> this rank's B / world sequences.

        With ``chunks`` > 1 the batch is processed in that many groups of whole sequences, pipelined:
        a group's max all-reduce (on its own communicator) runs while the next group is gathered, its
        reduce-scatter while the group after that is gathered; the rank then returns the r-th block of
        every group, in group order (chunks = 1: the r-th block of B)."""
        B, T, d = h.shape
        if B % (self.world * chunks):
            raise ValueError("the batch must split into whole sequences per rank and chunk")
        Bc = B // chunks
        multi = self.world > 1 and dist.is_initialized()
        gm = self.group_m if self.group_m is not None else self.group
        outs, staged, pending = [], None, None
        for c in range(chunks + 1):
            cur = None
            if c < chunks:  # gather group c; start its max all-reduce
                hc, xc = h[c * Bc:(c + 1) * Bc], router_x[c * Bc:(c + 1) * Bc]
                state = self.partial_packed(hc, xc) if self.packed else self.partial(hc, xc)
                mglob = state[0].clone()
                work_m = dist.all_reduce(mglob, op=dist.ReduceOp.MAX, group=gm, async_op=True) if multi else None
                cur = (state, mglob, work_m)
            if staged is not None:  # group c - 1: rescale to the global offsets, start its reduce-scatter
                state, mglob, work_m = staged
                if work_m is not None:
                    work_m.wait()  # the current stream waits for the maximum
                if self.packed:
                    mloc, pack = state
                    self.rescale(mloc, mglob, pack)
                else:
                    mloc, lloc, u = state
                    pack = self.pack(mloc, mglob, lloc, u)
                pack = pack.view(Bc * T, -1)
                if multi:
                    mine = torch.empty((Bc * T // self.world, pack.shape[1]), device=pack.device, dtype=pack.dtype)
                    work = dist.reduce_scatter_tensor(mine, pack, op=dist.ReduceOp.SUM, group=self.group,
                                                      async_op=True)
                else:
                    mine, work = pack, None
                if pending is not None:
                    outs.append(self._finish_pending(pending, T))
                pending = (work, mine, pack)  # the pack stays referenced until its reduction is done
            staged = cur
        outs.append(self._finish_pending(pending, T))
        return outs[0] if len(outs) == 1 else torch.cat(outs, 0)

    def _finish_pending(self, pending, T: int) -> Tensor:
        work, mine, _pack = pending
        if work is not None:
            work.wait()  # the current stream waits for the reduction
        return self.finish(mine, mine.shape[0] // T, T)

    def pack(self, mloc: Tensor, mglob: Tensor, lloc: Tensor, u: Tensor) -> Tensor:
        """(u, l) * exp(m_local - m_glob) packed [M, QH, Dt + 1] for the SUM reduction, in the pack
        dtype (bf16 for bf16 layers: half the bytes on NVLink; fp32 otherwise)."""
        M, QH, Dt = u.shape
        pack = torch.empty(M, QH, Dt + 1, device=u.device, dtype=self.pack_dtype)
        check(_lib.library().lng_attend_pack(ptr(mloc), ptr(mglob), ptr(lloc), ptr(u), M, QH, Dt, ptr(pack),
                                             _lib.dtype_code(self.pack_dtype), stream_ptr()), "pack")
        return pack

    def finish(self, packed: Tensor, Bb: int, T: int) -> Tensor:
        """Summed packed states of Bb whole sequences -> memory output [Bb, T, d]."""
        m = self.full.module
        act = m._act()
        QH, Dt = m.readout_num_heads, m.route_token_dim
        Mb = packed.shape[0]
        ub = torch.empty(Mb, QH * Dt, device=packed.device, dtype=act)
        packed = packed.contiguous()
        check(_lib.library().lng_attend_unpack(ptr(packed), _lib.dtype_code(packed.dtype), Mb, QH, Dt, ptr(ub),
                                               _lib.dtype_code(act), stream_ptr()), "unpack")
        mixed = m._linear(ub, m.folded()["w_vo"])
        return m._conv_finish(mixed.view(Bb, T, m.hidden_size), None, None)

    def rescale(self, mloc: Tensor, mglob: Tensor, pack: Tensor) -> None:
        """Rows of a kernel-written pack whose offset differs from the global maximum, rescaled in place."""
        M, QH, Dt1 = pack.shape
        check(_lib.library().lng_attend_pack_rescale(ptr(mloc), ptr(mglob), M, QH, Dt1 - 1, ptr(pack),
                                                     _lib.dtype_code(pack.dtype), stream_ptr()), "pack rescale")

    @torch.no_grad()
    def partial_packed(self, h: Tensor, router_x: Tensor) -> tuple[Tensor, Tensor]:
        """This rank's state as the bf16 pack [B*T, QH, Dt + 1] = (u, l) and m [B*T, QH], written by the
        attention kernel (partial mode 3 with the sink on rank 0, 4 elsewhere)."""
        m = self.full.module
        codes, qa, rs, (B, T, M) = self._query(h, router_x)
        Dt, QH = m.route_token_dim, m.readout_num_heads
        mloc = torch.empty(M, QH, device=h.device, dtype=torch.float32)
        pack = torch.empty(M, QH, Dt + 1, device=h.device, dtype=torch.bfloat16)
        check(_lib.library().lng_route_attend(self._tables_desc(), ptr(codes), _lib.U8, B, T, 0, None, None, None, 0, 0,
                                              self.r1 - self.r0, QH, m.eps, self.sink_logit, ptr(qa), ptr(rs),
                                              ptr(pack), _lib.BF16, 3 if self.rank == 0 else 4, ptr(mloc), None,
                                              stream_ptr()), "route_attend packed")
        return mloc, pack

    def _query(self, h: Tensor, router_x: Tensor):
        """Codes of the local routes, 1/rms(h) and the folded query, shared by both state forms."""
        m = self.full.module
        lib = _lib.library()
        s = stream_ptr()
        act = m._act()
        B, T, d = h.shape
        M = B * T
        Rl = self.r1 - self.r0
        h = h.to(act).contiguous()
        x = router_x.contiguous() if router_x.dtype in (torch.float32, torch.bfloat16) else router_x.float()
        codes = torch.empty(B, T, Rl, device=h.device, dtype=torch.uint8)
        if x.dtype == torch.bfloat16 and self.router_split is not None:
            check(lib.lng_route_codes_split(ptr(x), M, x.shape[-1], x.shape[-1], ptr(self.router_split), Rl,
                                            m.bits_per_route, ptr(codes), s), "route codes (tensor cores)")
        else:
            check(lib.lng_route_codes(ptr(x), _lib.dtype_code(x.dtype), M, x.shape[-1], x.shape[-1],
                                      ptr(self.router_w), Rl, m.bits_per_route, ptr(codes), _lib.U8, None, s),
                  "route codes")
        f = m.folded()
        rs = torch.empty(M, device=h.device, dtype=torch.float32)
        check(lib.lng_rms_rows(ptr(h), _lib.dtype_code(act), M, d, m.eps, ptr(rs), s), "rms")
        tdt = self.tables[m.ngrams[0]].dtype
        qa = m._linear(h.view(M, d), f["w_qk"].to(tdt) if f["w_qk"].dtype != tdt else f["w_qk"])
        return codes, qa, rs, (B, T, M)

    @torch.no_grad()
    def partial(self, h: Tensor, router_x: Tensor) -> tuple[Tensor, Tensor, Tensor]:
        """This rank's online-softmax state over its routes: m, l [B*T, QH] and u [B*T, QH, Dt] (fp32)."""
        m = self.full.module
        codes, qa, rs, (B, T, M) = self._query(h, router_x)
        Dt, QH = m.route_token_dim, m.readout_num_heads
        mloc = torch.empty(M, QH, device=h.device, dtype=torch.float32)
        lloc = torch.empty_like(mloc)
        u = torch.empty(M, QH, Dt, device=h.device, dtype=torch.float32)
        # sink: b0 = log(R_total (1 - mass) / mass) of the whole layer, seeded on rank 0 only
        check(_lib.library().lng_route_attend(self._tables_desc(), ptr(codes), _lib.U8, B, T, 0, None, None, None, 0, 0,
                                              self.r1 - self.r0, QH, m.eps, self.sink_logit, ptr(qa), ptr(rs), ptr(u),
                                              _lib.F32, 1 if self.rank == 0 else 2, ptr(mloc), ptr(lloc),
                                              stream_ptr()), "route_attend partial")
        return mloc, lloc, u
