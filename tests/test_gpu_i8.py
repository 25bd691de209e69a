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


def _planes_ref(slab: np.ndarray, n_mat: int, rows: int, cols: int) -> np.ndarray:
    """the tile-plane image restated from the GGUF Q2_K bytes (include/pulsar_moe.h,
    pulsar_repack_q2k_tiles): per (matrix, 128-row block, super-block) qs as [4 x 16 B][128 rows],
    then the rows' 16 scale bytes, then their d, dmin"""
    nsb = cols // 256
    b = slab[:n_mat * rows * nsb * 84].reshape(n_mat, rows // 128, 128, nsb, 84).transpose(0, 1, 3, 2, 4)
    qs = b[..., 16:80].reshape(n_mat, rows // 128, nsb, 128, 4, 16).transpose(0, 1, 2, 4, 3, 5)
    parts = [qs.reshape(n_mat, rows // 128, nsb, -1), b[..., 0:16].reshape(n_mat, rows // 128, nsb, -1),
             b[..., 80:84].reshape(n_mat, rows // 128, nsb, -1)]
    return np.concatenate(parts, axis=-1).reshape(-1)


@pytest.mark.parametrize("H,F,E", [(512, 768, 3), (4096, 1536, 2)])
def test_tile_planes_regroup_the_gguf_bytes(oracle, H, F, E):
    L = HostLayer(H=H, F=F, E=E, k=1, quant=0, seed=5, router_mode=1)
    dl = L.to_device()
    torch.cuda.synchronize()
    for slab, tiles, rows, cols in ((dl.gate, dl.gate_tiles, F, H), (dl.up, dl.up_tiles, F, H),
                                    (dl.down, dl.down_tiles, H, F)):
        got = tiles.cpu().numpy()
        want = _planes_ref(slab.cpu().numpy(), E, rows, cols)
        assert got.size == want.size and np.array_equal(got, want)


def test_no_tile_images_keeps_q2k_off_the_integer_path(oracle):
    L = HostLayer(H=1024, F=512, E=16, k=8, quant=0, seed=72, router_mode=1)
    T = 40
    x = np.random.default_rng(3).normal(0, 1, (T, 1024)).astype(np.float32)
    _, sel, w = L.oracle_route(x)
    ref = L.oracle_ffn(x, sel, w)
    dl = L.to_device()
    dl.gate_tiles = dl.up_tiles = dl.down_tiles = None
    dl._desc = None
    dl.desc().path_flags = 2  # asks for the integer passes, which need the images
    ws = torch.zeros(dl.workspace_bytes(T), dtype=torch.uint8, device="cuda")
    out = torch.zeros((T, 1024), dtype=torch.float32, device="cuda")
    dl.forward(torch.from_numpy(x).cuda(), out, ws)
    torch.cuda.synchronize()
    v = dl.ws_view(ws, T)
    assert reader(ws)(v.n_items, 8, np.uint32)[7] == 0
    assert rel_l2(out.cpu().numpy(), ref) < 1e-3
