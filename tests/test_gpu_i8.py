"""Routed Q2_K experts on the tcgen05 integer tensor cores (pm_tci8.cuh).

Both paths form every dot in the CPU lane's arithmetic - the integer
super-block sums exactly, the f32 terms in super-block order - so the
integer tensor-core path and the dp4a engine (PULSAR_LAYER_NO_I8) must give
the same output bit for bit, and the mid rows must equal the oracle's (but
for the glu exponential's rare 1-3 ulp differences).  Token counts cover one
token, partial 16- and 32-token tiles, tiles split across an expert (33,
300 tokens) and 128-row blocks of both passes."""
import numpy as np
import pytest

from helpers import HostLayer, reader, rel_l2

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

CASES = [  # (H, F, E, k, T); under 192 tokens per expert the dp4a engine takes every expert when the
    # integer path is off (above it the fp16 tiles would, which are not exact)
    (1024, 512, 16, 8, 1), (1024, 512, 16, 8, 5), (1024, 512, 16, 8, 33), (512, 768, 8, 2, 150),
    (4096, 1536, 8, 4, 20), (512, 768, 8, 2, 700)]


@pytest.mark.parametrize("H,F,E,k,T", CASES, ids=[f"H{c[0]}-F{c[1]}-E{c[2]}-k{c[3]}-T{c[4]}" for c in CASES])
def test_i8_equals_dp4a_and_oracle(oracle, H, F, E, k, T):
    L = HostLayer(H=H, F=F, E=E, k=k, quant=0, seed=71, router_mode=1, zipf=(1.2, "logit"))
    x = np.random.default_rng(T).normal(0, 1, (T, H)).astype(np.float32)
    _, sel, w = L.oracle_route(x)
    ref, ref_mid = L.oracle_ffn(x, sel, w, return_mid=True)
    dl = L.to_device()
    xd = torch.from_numpy(x).cuda()
    outs, mids = [], []
    for flags in (2, 1):  # integer tensor cores (PULSAR_LAYER_FORCE_I8), then the dp4a engine (NO_I8)
        dl.desc().path_flags = flags
        ws = torch.zeros(dl.workspace_bytes(T), dtype=torch.uint8, device="cuda")
        out = torch.zeros((T, H), dtype=torch.float32, device="cuda")
        dl.forward(xd, out, ws)
        torch.cuda.synchronize()
        v = dl.ws_view(ws, T)
        rd = reader(ws)
        n = rd(v.n_items, 8, np.uint32)
        assert rd(v.err, 1, np.uint32)[0] == 0
        if flags == 2:
            assert n[7] > 0 and n[2] == 0, "routed experts expected on the integer tensor cores"
        mids.append(rd(v.mid, T * v.n_slot * v.f_max, np.float32).reshape(T, v.n_slot, v.f_max)[:, :k, :F])
        outs.append(out.cpu().numpy())
    if T * k / E < 150:  # both paths exact: identical bits
        assert np.array_equal(mids[0].view(np.uint32), mids[1].view(np.uint32)), "mid: integer MMA vs dp4a"
        assert np.array_equal(outs[0].view(np.uint32), outs[1].view(np.uint32)), "out: integer MMA vs dp4a"
    ulp = np.abs(mids[0].view(np.int32).astype(np.int64) - ref_mid[:, :, :F].view(np.int32).astype(np.int64))
    assert ulp.max() <= 4 and np.count_nonzero(ulp) <= max(3, ulp.size // 1000), (int(ulp.max()), np.count_nonzero(ulp))
    assert rel_l2(outs[0], ref) < 1e-3
