"""Route-sharded memory forward on the GPU.

* Shards emulated on one GPU: each shard's partial state from the fused kernel (sink on shard 0
  only), combined through the pack / unpack kernels, equals the unsharded forward (fp32: 1e-5;
  bf16 SB shape: 1e-2).
* Two GPUs (skipped with fewer): one process per GPU over NCCL; every rank's block of sequences
  equals the single-GPU forward of those sequences, also with two overlapped sequence groups.
"""

from __future__ import annotations

import os
import socket
import sys
from pathlib import Path

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

from tests.golden import cases
from tests.helpers import assert_bf16_close, assert_fp32_close
from tests.test_gpu_memory import gpu_memory

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda:0")
REPO = Path(__file__).resolve().parents[1]


def emulate(lngram, mem, h, x, world):
    shards = [lngram.RouteShardedMemory(mem, r, world) for r in range(world)]
    parts = [s.partial(h, x) for s in shards]
    mg = parts[0][0].clone()
    for p in parts[1:]:
        mg = torch.maximum(mg, p[0])
    total = sum(s.pack(p[0], mg, p[1], p[2]) for s, p in zip(shards, parts))
    B, T = h.shape[:2]
    return shards[0].finish(total.view(B * T, -1), B, T)


@pytest.mark.parametrize("world", [2, 3])
def test_emulated_shards_equal_full_forward_fp32(lngram, world):
    case = "tiny_multi"
    mem = gpu_memory(lngram, case)
    inp = cases.memory_inputs(case)
    h = torch.from_numpy(inp["h"]).to(DEV)
    x = torch.from_numpy(inp["x"]).to(DEV)
    with torch.no_grad():
        want = mem(h, x).cpu().numpy()
        got = emulate(lngram, mem, h, x, world).cpu().numpy()
    assert_fp32_close(got, want, what=f"{world} emulated route shards")


def test_emulated_shards_sb_shape_bf16(lngram, golden):
    g = golden("memory_sb_slice")
    mem = gpu_memory(lngram, "sb_slice", dtype=torch.bfloat16)
    inp = cases.memory_inputs("sb_slice")
    h = torch.from_numpy(inp["h"]).to(DEV).to(torch.bfloat16)
    x = torch.from_numpy(inp["x"]).to(DEV)
    with torch.no_grad():
        got = emulate(lngram, mem, h, x, 8).float().cpu().numpy()
    assert_bf16_close(got, g["output_wrapper"], what="8 emulated shards vs reference")


def test_emulated_packed_shards_sb_shape_bf16(lngram, golden):
    """Kernel-written bf16 packs (partial modes 3 / 4), rescaled to the global maximum and summed."""
    g = golden("memory_sb_slice")
    mem = gpu_memory(lngram, "sb_slice", dtype=torch.bfloat16)
    inp = cases.memory_inputs("sb_slice")
    h = torch.from_numpy(inp["h"]).to(DEV).to(torch.bfloat16)
    x = torch.from_numpy(inp["x"]).to(DEV)
    shards = [lngram.RouteShardedMemory(mem, r, 8) for r in range(8)]
    assert all(s.packed for s in shards)
    with torch.no_grad():
        parts = [s.partial_packed(h, x) for s in shards]
        mg = parts[0][0].clone()
        for q in parts[1:]:
            mg = torch.maximum(mg, q[0])
        for s, q in zip(shards, parts):
            s.rescale(q[0], mg, q[1])
        total = sum(q[1].float() for q in parts).to(torch.bfloat16)
        B, T = h.shape[:2]
        got = shards[0].finish(total.view(B * T, -1), B, T).float().cpu().numpy()
    assert_bf16_close(got, g["output_wrapper"], what="8 emulated packed shards vs reference")


def local_shard(lngram, case: str, rank: int, world: int, dtype=torch.float32):
    """A memory holding only the routes of ``rank`` (tables and router rows sliced from the case's
    parameters, readout weights whole), wrapped as a pre-sliced route shard."""
    c = cases.MEMORY_CASES[case]
    R = c["routes"]
    r0, r1 = lngram.sharded.route_bounds(R, world)[rank]
    p = cases.memory_params(case)
    state = {}
    for k, v in p.items():
        if k.startswith("tables.ngram_"):
            span = (1 << c["bits"]) ** int(k.split("_")[1].split(".")[0])
            v = v[r0 * span:r1 * span]
        elif k == "router.weight":
            v = v[r0 * c["bits"]:r1 * c["bits"]]
        state[k if k == "router.weight" else "module." + k] = torch.from_numpy(np.ascontiguousarray(v))
    mem = lngram.LngramMemory(c["d"], {"routes": r1 - r0, "mem_dim": c["mem_dim"], "kv_heads": c["kv_heads"],
                                       "q_heads": c["q_heads"], "head_dim": c["head_dim"], "ngrams": list(c["ngrams"]),
                                       "bits_per_route": c["bits"]}, norm_eps=1e-5, device=DEV, dtype=dtype).eval()
    mem.load_state_dict(state, strict=True)
    return lngram.RouteShardedMemory(mem, rank, world, routes_total=R)


@pytest.mark.parametrize("case,world", [("tiny_multi", 3), ("scaled_slice", 2)])
def test_pre_sliced_shards_equal_full_forward(lngram, case, world):
    mem = gpu_memory(lngram, case)
    inp = cases.memory_inputs(case)
    h = torch.from_numpy(inp["h"]).to(DEV)
    x = torch.from_numpy(inp["x"]).to(DEV)
    shards = [local_shard(lngram, case, r, world) for r in range(world)]
    with torch.no_grad():
        want = mem(h, x).cpu().numpy()
        parts = [s.partial(h, x) for s in shards]
        mg = parts[0][0].clone()
        for q in parts[1:]:
            mg = torch.maximum(mg, q[0])
        total = sum(s.pack(q[0], mg, q[1], q[2]) for s, q in zip(shards, parts))
        B, T = h.shape[:2]
        got = shards[0].finish(total.view(B * T, -1), B, T).cpu().numpy()
    assert_fp32_close(got, want, what=f"{world} pre-sliced route shards ({case})")


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank: int, world: int, port: int, out_dir: str) -> None:
    import datetime

    sys.path.insert(0, str(REPO))
    import torch.distributed as dist

    torch.cuda.set_device(rank)
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                            device_id=torch.device("cuda", rank))
    try:
        from __graft_entry__ import load_package
        from tests.test_gpu_memory import gpu_memory as make

        lngram = load_package()
        global DEV
        DEV = torch.device("cuda", rank)
        import tests.test_gpu_memory as tgm

        tgm.DEV = DEV
        mem = make(lngram, "tiny")
        inp = cases.memory_inputs("tiny")
        h = torch.from_numpy(inp["h"]).to(DEV)
        x = torch.from_numpy(inp["x"]).to(DEV)
        shard = lngram.RouteShardedMemory(mem, rank, world)
        with torch.no_grad():
            out = shard.forward(h, x)
            full = mem(h, x)
            # two overlapped sequence groups over 4 sequences: rank r gets sequence r of each group
            h4 = torch.cat((h, h.flip(1)), 0)
            x4 = torch.cat((x, x.flip(1)), 0)
            out4 = shard.forward(h4, x4, chunks=2)
            full4 = mem(h4, x4)
        torch.cuda.synchronize()
        B = h.shape[0]
        blk = slice(rank * B // world, (rank + 1) * B // world)
        np.save(os.path.join(out_dir, f"rank{rank}.npy"), np.stack([out.cpu().numpy(), full[blk].cpu().numpy()]))
        np.save(os.path.join(out_dir, f"rank{rank}_chunks.npy"),
                np.stack([out4.cpu().numpy(), full4[[rank, 2 + rank]].cpu().numpy()]))
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_two_gpu_route_sharded_forward(tmp_path):
    port = _free_port()
    mp.start_processes(_rank_main, args=(2, port, str(tmp_path)), nprocs=2, start_method="spawn")
    for r in range(2):
        got, want = np.load(tmp_path / f"rank{r}.npy")
        assert_fp32_close(got, want, what=f"rank {r} block")
        got, want = np.load(tmp_path / f"rank{r}_chunks.npy")
        assert_fp32_close(got, want, what=f"rank {r} blocks of two overlapped groups")
