"""pulsar_moe_layer_ep on 2 GPUs (skipped with fewer): each rank builds the
same host-encoded layer, computes only its expert range, routes its own
tokens, and gets back residual + moe(x) for its tokens through the NCCL
dispatch / combine; every rank's result is checked against the CPU oracle
of the full layer.  Ranks are child processes, one per GPU, NVLS off."""
import os
import socket

import numpy as np
import pytest

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

TOL = 1e-3
CASES = {  # name: (HostLayer kwargs, tokens per rank)
    "q4k-shared": (dict(H=512, F=512, E=32, k=8, quant=2, router_mode=0, zipf=(1.1, "select"), shared=(2, 512)), 9),
    "q2k-softmax": (dict(H=1024, F=512, E=16, k=8, quant=0, router_mode=1, zipf=(1.2, "logit")), 32),
    "q2k-tensor-cores": (dict(H=512, F=512, E=8, k=2, quant=0, router_mode=1), 400),
}


def _worker(rank, world, port, name, q):
    try:
        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
        import sys
        sys.path.insert(0, os.path.dirname(os.path.abspath(__file__)))
        import torch.distributed as dist

        from helpers import HostLayer, rel_l2
        from pulsar_b200.ep import EpComm, shard
        torch.cuda.set_device(rank)
        dist.init_process_group("gloo", rank=rank, world_size=world)
        kw, T = CASES[name]
        L = HostLayer(seed=61, **kw)
        rng = np.random.default_rng(700 + rank)
        x = rng.normal(0, 1, (T, L.H)).astype(np.float32)
        resid = rng.normal(0, 1, (T, L.H)).astype(np.float32)
        _, sel, w = L.oracle_route(x)
        ref = L.oracle_ffn(x, sel, w) + resid
        dl = L.to_device()
        dl.expert_lo, dl.expert_hi = shard(L.E, world, rank)
        comm = EpComm(rank, world)
        ws = torch.zeros(dl.ep_workspace_bytes(world, T), dtype=torch.uint8, device="cuda")
        out = torch.zeros((T, L.H), dtype=torch.float32, device="cuda")
        errs = []
        for rep in range(2):  # the second call reuses the workspace
            dl.forward_ep(comm, torch.from_numpy(x).cuda(), out, ws, residual=torch.from_numpy(resid).cuda())
            torch.cuda.synchronize()
            errs.append(rel_l2(out.cpu().numpy() - resid, ref - resid))
        v = dl.ws_view(ws, T * world)
        err_word = int(ws[v.err - ws.data_ptr():v.err - ws.data_ptr() + 4].view(torch.int32).item())
        q.put((rank, errs, err_word, None))
        dist.barrier()
        comm.destroy()
        dist.destroy_process_group()
    except Exception as e:  # report instead of hanging the parent
        import traceback
        q.put((rank, None, None, traceback.format_exc()))


@pytest.mark.parametrize("name", list(CASES))
def test_ep_two_gpus_vs_oracle(oracle, name):
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    import torch.multiprocessing as mp
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, name, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = [q.get(timeout=300) for _ in range(2)]
    for p in procs:
        p.join(timeout=120)
    for rank, errs, err_word, tb in res:
        assert tb is None, tb
        print(name, "rank", rank, "rel_l2", errs)
        assert err_word == 0
        assert max(errs) < TOL, (rank, errs)
