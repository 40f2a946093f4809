"""Route-sharded combine on CPU ranks (gloo, world size 2): the collective choreography of
``lngram-decode_b200/sharded.py`` (``all_reduce_max``, ``reduce_scatter_rows`` by whole-sequence
blocks) applied to oracle partial states of each rank's routes reproduces the oracle's unsharded
readout (``_streaming_gqa`` with one route chunk per rank, ``ffnmem/memory/lngram_v2.py:1944-2070``).
The per-rank arithmetic here is the oracle's; the GPU kernels for it are tested in
``tests/test_gpu_sharded.py``."""

from __future__ import annotations

import os
import socket
import sys
from pathlib import Path

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

REPO = Path(__file__).resolve().parents[1]


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank: int, world: int, port: int, out_dir: str, route_shards: int = 0) -> None:
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
        inp = cases.memory_inputs(case)
        rs = route_shards or world
        place = sharded.route_data_grid(world, rs, rank)
        group, group_m = place.group, place.group_m
        # two sequences per route group (one block per rank of the group): the data block of this group
        h_all = np.concatenate((inp["h"][:2], inp["h"][:2, ::-1]), 0)[:2 * place.data_shards]
        x_all = np.concatenate((inp["x"][:2], inp["x"][:2, ::-1]), 0)[:2 * place.data_shards]
        codes_all = om.quantize_route_logits(om.route_logits(x_all, cases.memory_params(case)["router.weight"]), p.bits)
        blk = slice(2 * place.data_index, 2 * place.data_index + 2)
        h, codes = np.ascontiguousarray(h_all[blk]), codes_all[blk]
        B, T = h.shape[:2]
        rank_g = place.route_index
        r0, r1 = sharded.route_bounds(p.num_routes, rs)[rank_g]
        query = om.project_query(h, p)
        key, value = om.project_memory(om.lookup_route_chunk(codes, p.tables, p.ngrams, p.bits, r0, r1), p)
        shape = (B, T, p.num_kv_heads, p.groups)
        seed = None if rank_g == 0 else (np.full(shape, -np.inf, np.float32), np.zeros(shape, np.float32),
                                         np.zeros(shape + (p.head_dim,), np.float32))
        m, l, o = om.streaming_partial(query, key, value, p, seed)
        QH, HD = p.num_heads, p.head_dim
        m_t = torch.from_numpy(m.reshape(B * T, QH).copy())
        m_g = sharded.all_reduce_max(m_t.clone(), group_m)
        s = torch.exp(m_t - m_g).unsqueeze(-1)
        pack = torch.cat((torch.from_numpy(o.reshape(B * T, QH, HD)) * s,
                          torch.from_numpy(l.reshape(B * T, QH, 1)) * s), dim=-1)
        mine = sharded.reduce_scatter_rows(pack.reshape(B * T, -1), group).view(-1, QH, HD + 1)
        head = (mine[..., :HD] / mine[..., HD:]).numpy()
        full = om.manual_gqa(query, *om.project_memory(
            om.lookup_route_chunk(codes, p.tables, p.ngrams, p.bits, 0, p.num_routes), p), p)
        want = full.reshape(B * T, QH, HD)[rank_g * (B * T // rs):(rank_g + 1) * (B * T // rs)]
        np.save(os.path.join(out_dir, f"rank{rank}.npy"), np.stack([head, want]))
    finally:
        dist.destroy_process_group()


def test_two_rank_route_sharded_combine(tmp_path):
    port = _free_port()
    mp.start_processes(_rank_main, args=(2, port, str(tmp_path)), nprocs=2, start_method="spawn")
    for r in range(2):
        got, want = np.load(tmp_path / f"rank{r}.npy")
        scale = np.abs(want).max()
        np.testing.assert_allclose(got, want, rtol=1e-5, atol=1e-5 * scale)


def test_four_rank_route_by_data_grid(tmp_path):
    """2 route shards x 2 data blocks: each pair exchanges only within itself (its own communicators)."""
    port = _free_port()
    mp.start_processes(_rank_main, args=(4, port, str(tmp_path), 2), nprocs=4, start_method="spawn")
    for r in range(4):
        got, want = np.load(tmp_path / f"rank{r}.npy")
        scale = np.abs(want).max()
        np.testing.assert_allclose(got, want, rtol=1e-5, atol=1e-5 * scale)


def test_route_bounds_cover_all_routes():
    from __graft_entry__ import load_package

    sharded = load_package().sharded
    for R, P in [(184, 8), (184, 3), (4, 4), (5, 2), (23, 8)]:
        b = sharded.route_bounds(R, P)
        assert b[0][0] == 0 and b[-1][1] == R and all(x[1] == y[0] for x, y in zip(b, b[1:]))
        assert max(e - s for s, e in b) - min(e - s for s, e in b) <= 1
