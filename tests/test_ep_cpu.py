"""Expert parallelism, host side (no GPU): the placement, the shard ranges,
the workspace of pulsar_moe_layer_ep, and the communicator id travelling
over a 2-rank gloo group."""
import ctypes
import os

import pytest


def test_shards_partition_the_experts():
    from pulsar_b200.ep import shard
    for E, world in ((128, 1), (128, 2), (128, 8), (256, 8), (32, 4)):
        ranges = [shard(E, world, r) for r in range(world)]
        assert ranges[0][0] == 0 and ranges[-1][1] == E
        assert all(a[1] == b[0] for a, b in zip(ranges, ranges[1:]))
        assert all(hi - lo == E // world for lo, hi in ranges)


def test_snake_order_balances_popularity():
    from pulsar_b200.ep import shard, snake_order, zipf_popularity
    E, world = 128, 8
    pop = zipf_popularity(E, 1.2, 2003)
    order = snake_order(pop, world)
    assert sorted(order) == list(range(E))  # a permutation
    loads = [sum(pop[order[p]] for p in range(*shard(E, world, r))) for r in range(world)]
    naive = [sum(pop[p] for p in range(*shard(E, world, r))) for r in range(world)]
    # each rank holds exactly one of the eight most popular experts
    top = sorted(range(E), key=lambda e: -pop[e])[:world]
    for r in range(world):
        lo, hi = shard(E, world, r)
        assert sum(1 for p in range(lo, hi) if order[p] in top) == 1
    assert max(loads) / min(loads) < max(naive) / min(naive)


def test_ep_workspace_extends_the_gathered_layout():
    import pulsar_b200
    from pulsar_b200 import LayerDesc
    L = pulsar_b200.lib()
    d = LayerDesc()  # C4 shapes
    d.n_embd, d.n_ff, d.n_expert, d.n_used, d.quant, d.router_mode = 4096, 1536, 128, 8, 0, 1
    d.row_bytes_gu, d.row_bytes_down = 16 * 84, 6 * 84
    d.gate = d.up = d.down = d.router_w = 1
    d.expert_lo, d.expert_hi = 16, 32
    for world, T in ((2, 32), (8, 32), (8, 256)):
        one = L.pulsar_moe_layer_workspace(ctypes.byref(d), world * T)
        ep = L.pulsar_moe_layer_ep_workspace(ctypes.byref(d), world, T)
        assert ep >= one + world * T * 4096 * 4  # + the per-token sums ahead of the reduce-scatter
        assert ep - one < world * T * 4096 * 4 + 512
    assert L.pulsar_moe_layer_ep_workspace(ctypes.byref(d), 0, 32) == 0
    # world > 1 without a communicator is refused before any device work
    assert L.pulsar_moe_layer_ep(ctypes.byref(d), None, 0, 2, 1, 1, None, 4, 1, 1 << 30, None) == 0
    d.expert_hi = 0  # every rank must name its experts
    assert L.pulsar_moe_layer_ep(ctypes.byref(d), 1, 0, 2, 1, 1, None, 4, 1, 1 << 30, None) == 0


def _id_worker(rank, world, port, q):
    import torch.distributed as dist

    import pulsar_b200
    os.environ["MASTER_ADDR"], os.environ["MASTER_PORT"] = "127.0.0.1", str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    from pulsar_b200.ep import share_unique_id
    uid = share_unique_id(rank, None, device="cpu")
    q.put((rank, bytes(uid)))
    dist.destroy_process_group()


def test_unique_id_reaches_every_rank_gloo():
    """rank 0's NCCL id, broadcast over a world-size-2 gloo group, arrives
    byte-identical on rank 1 (the step before each rank's pulsar_ep_comm_init)"""
    import socket

    import torch.multiprocessing as mp
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_id_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    got = dict(q.get(timeout=120) for _ in range(2))
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    assert got[0] == got[1] and len(got[0]) == 128 and any(got[0])
