"""The group pipeline of ``RouteShardedMemory.forward`` on CPU ranks (gloo, world size 2).

``forward(h, x, chunks=k)`` gathers group c + 1 while group c's max all-reduce is in flight, and
rescales and reduce-scatters group c only after that (a one-group lag), then returns the rank's
block of every group in group order.  Here the rank's device steps (``partial``, ``pack``,
``finish``) are replaced by the oracle's arithmetic for its routes, so the test runs the real
``forward`` -- its collectives, its lag and its output order -- without a GPU, and checks the result
against the oracle's unsharded readout (``_streaming_gqa`` with one route chunk per rank,
``ffnmem/memory/lngram_v2.py:1944-2070``) for every chunk count that divides the batch.
"""

from __future__ import annotations

import os
import socket
import sys
from pathlib import Path

import numpy as np
import torch
import torch.multiprocessing as mp

REPO = Path(__file__).resolve().parents[1]


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank: int, world: int, port: int, out_dir: str) -> None:
    sys.path.insert(0, str(REPO))
    import torch.distributed as dist

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from __graft_entry__ import load_package
        from oracle import memory as om
        from tests.golden import cases

        sharded = load_package().sharded
        case = "tiny_multi"
        p = cases.oracle_params(case)
        w_router = cases.memory_params(case)["router.weight"]
        inp = cases.memory_inputs(case)
        # four whole sequences: two per rank at chunks = 1, one per rank and group at chunks = 2
        h_all = np.ascontiguousarray(np.concatenate((inp["h"][:2], inp["h"][:2, ::-1]), 0))
        x_all = np.ascontiguousarray(np.concatenate((inp["x"][:2], inp["x"][:2, ::-1]), 0))
        B, T = h_all.shape[:2]
        QH, HD = p.num_heads, p.head_dim
        r0, r1 = sharded.route_bounds(p.num_routes, world)[rank]

        shard = sharded.RouteShardedMemory.__new__(sharded.RouteShardedMemory)
        shard.rank, shard.world, shard.group, shard.group_m, shard.packed = rank, world, None, None, False

        def partial(hc, xc):
            h, x = hc.numpy(), xc.numpy()
            codes = om.quantize_route_logits(om.route_logits(x, w_router), p.bits)
            query = om.project_query(h, p)
            key, value = om.project_memory(om.lookup_route_chunk(codes, p.tables, p.ngrams, p.bits, r0, r1), p)
            shape = (h.shape[0], T, p.num_kv_heads, p.groups)
            seed = None if rank == 0 else (np.full(shape, -np.inf, np.float32), np.zeros(shape, np.float32),
                                           np.zeros(shape + (HD,), np.float32))
            m, l, o = om.streaming_partial(query, key, value, p, seed)
            M = h.shape[0] * T
            return (torch.from_numpy(m.reshape(M, QH).copy()), torch.from_numpy(l.reshape(M, QH).copy()),
                    torch.from_numpy(o.reshape(M, QH, HD).copy()))

        def pack(mloc, mglob, lloc, u):
            s = torch.exp(mloc - mglob)
            return torch.cat((u * s.unsqueeze(-1), (lloc * s).unsqueeze(-1)), dim=-1)

        def finish(mine, Bb, T_):
            v = mine.view(Bb * T_, QH, HD + 1)
            return (v[..., :HD] / v[..., HD:]).reshape(Bb, T_, QH * HD)

        shard.partial, shard.pack, shard.finish = partial, pack, finish
        h_t, x_t = torch.from_numpy(h_all), torch.from_numpy(x_all)
        full = om.manual_gqa(om.project_query(h_all, p), *om.project_memory(om.lookup_route_chunk(
            om.quantize_route_logits(om.route_logits(x_all, w_router), p.bits), p.tables, p.ngrams, p.bits, 0,
            p.num_routes), p), p).reshape(B, T, QH * HD)
        res = {}
        for chunks in (1, 2):
            got = shard.forward(h_t, x_t, chunks=chunks).numpy()
            Bc = B // chunks
            per = Bc // world
            # the rank's block of every group, in group order
            rows = [s for c in range(chunks) for s in range(c * Bc + rank * per, c * Bc + (rank + 1) * per)]
            res[f"got{chunks}"], res[f"want{chunks}"] = got, full[rows]
        np.savez(os.path.join(out_dir, f"rank{rank}.npz"), **res)
    finally:
        dist.destroy_process_group()


def test_two_rank_group_pipeline(tmp_path):
    port = _free_port()
    mp.start_processes(_rank_main, args=(2, port, str(tmp_path)), nprocs=2, start_method="spawn")
    for r in range(2):
        z = np.load(tmp_path / f"rank{r}.npz")
        for chunks in (1, 2):
            got, want = z[f"got{chunks}"], z[f"want{chunks}"]
            assert got.shape == want.shape
            scale = np.abs(want).max()
            np.testing.assert_allclose(got, want, rtol=1e-5, atol=1e-5 * scale)
