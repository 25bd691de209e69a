"""Expert parallelism across the GPUs of one box: placement and the NCCL
communicator of pulsar_moe_layer_ep.

The reference spreads a model's experts over tiers (GPU, CPU lane, NVMe
stream) and gathers the results (crates/engine/src/lib.rs:8395-8450,
8620-8638).  With every expert resident in HBM, the B200 build shards the
experts over the GPUs instead: rank r owns a contiguous range of expert
slots, and a load-time placement (snake order over expert popularity)
decides which logical expert sits in which slot, so the hot experts of a
Zipf-skewed router spread over the ranks.
"""
from __future__ import annotations

import ctypes

import torch

from ._lib import check, lib


def shard(n_expert: int, world: int, rank: int) -> tuple[int, int]:
    """expert slots [lo, hi) of rank `rank` (even split)"""
    return rank * n_expert // world, (rank + 1) * n_expert // world


def snake_order(popularity, world: int) -> list[int]:
    """Placement: slot -> logical expert.  Experts sorted by popularity
    (descending, ties by id) are dealt to the ranks in snake order (0..N-1,
    N-1..0, ...); rank r's experts then fill its slot range in that order.
    Every rank gets the same number of experts and a near-equal share of
    the popular ones."""
    E = len(popularity)
    assert E % world == 0, "experts must split evenly over the ranks"
    ranked = sorted(range(E), key=lambda e: (-float(popularity[e]), e))
    per = [[] for _ in range(world)]
    for i, e in enumerate(ranked):
        rnd, pos = divmod(i, world)
        per[pos if rnd % 2 == 0 else world - 1 - pos].append(e)
    return [e for r in range(world) for e in per[r]]


def zipf_popularity(n_expert: int, s: float, seed: int):
    """expected popularity order of make_layer's Zipf router bias (rank 1 =
    most popular): the bias is a decreasing function of the seeded rank"""
    g = torch.Generator().manual_seed(seed)
    rank = torch.randperm(n_expert, generator=g).to(torch.float64) + 1.0
    return (rank.pow(-s)).tolist()


def share_unique_id(rank: int, group=None, device=None) -> bytes:
    """rank 0's 128-byte NCCL id (pulsar_ep_unique_id), broadcast to every
    rank of a torch.distributed group (gloo: host tensors; nccl: device)"""
    import torch.distributed as dist
    uid = (ctypes.c_uint8 * 128)()
    if rank == 0:
        check(lib().pulsar_ep_unique_id(ctypes.cast(uid, ctypes.c_void_p)), "ep_unique_id")
    t = torch.tensor(list(bytes(uid)), dtype=torch.uint8)
    if dist.get_backend(group) == "nccl":
        t = t.to(device if device is not None else torch.device("cuda", torch.cuda.current_device()))
    dist.broadcast(t, src=0, group=group)
    return bytes(t.cpu().tolist())


class EpComm:
    """The NCCL communicator of one rank for pulsar_moe_layer_ep, created
    through the library (same NCCL as its collectives).  The 128-byte id
    travels from rank 0 over an existing torch.distributed group."""

    def __init__(self, rank: int, world: int, group=None, device=None):
        self.rank, self.world = rank, world
        raw = share_unique_id(rank, group, device)
        uid = (ctypes.c_uint8 * 128).from_buffer_copy(raw)
        h = ctypes.c_void_p()
        check(lib().pulsar_ep_comm_init(ctypes.byref(h), ctypes.cast(uid, ctypes.c_void_p), world, rank),
              "ep_comm_init")
        self.handle = h.value

    def destroy(self):
        if self.handle:
            lib().pulsar_ep_comm_destroy(self.handle)
            self.handle = None
