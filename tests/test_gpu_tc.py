"""Large batches: experts with >= 192 tokens (and the shared expert) run on
the tcgen05 tensor-core tiles (fp16 hi + lo split operands, fp32
accumulation) in every supported block format; the rest on the dp4a engine.  Outputs and mid rows must
match the CPU oracle within the expert-FFN tolerance."""
import numpy as np
import pytest

from helpers import HostLayer, rel_l2

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

TOL = 1e-3


def _ws(ws, base, ptr, n, dt):
    off = ptr - base
    return ws[off:off + n * np.dtype(dt).itemsize].view(dt)


CASES = [  # (routed format, shared (format, F) or None, T)
    (2, None, 300), (2, (2, 512), 300), (2, None, 512), (2, (2, 512), 512),
    (0, None, 300), (1, None, 300), (10, None, 300), (12, None, 300), (1, (10, 512), 300)]


@pytest.mark.parametrize("quant,shared,T", CASES, ids=[f"q{q}-sh{s}-T{t}" for q, s, t in CASES])
def test_tensor_core_tiles(oracle, quant, shared, T):
    L = HostLayer(H=512, F=512, E=8, k=2, quant=quant, seed=11, router_mode=0, zipf=(1.1, "select"), shared=shared)
    x = np.random.default_rng(5).normal(0, 1, (T, L.H)).astype(np.float32)
    _, sel, w = L.oracle_route(x)
    ref, ref_mid = L.oracle_ffn(x, sel, w, return_mid=True)
    dl = L.to_device()
    wst = torch.zeros(dl.workspace_bytes(T), dtype=torch.uint8, device="cuda")
    out = torch.zeros((T, L.H), dtype=torch.float32, device="cuda")
    dl.forward(torch.from_numpy(x).cuda(), out, wst)
    torch.cuda.synchronize()
    v = dl.ws_view(wst, T)
    ws, base = wst.cpu().numpy(), wst.data_ptr()
    n = _ws(ws, base, v.n_items, 6, np.uint32)
    assert n[4] > 0, "no tensor-core tiles at this batch"
    ns = v.n_slot
    mid = _ws(ws, base, v.mid, T * ns * v.f_max, np.float32).reshape(T * ns, v.f_max)[:, :ref_mid.shape[-1]]
    rm = ref_mid.reshape(T * ns, -1)
    got = out.cpu().numpy()
    print(quant, shared, T, "tiles", int(n[4]), "splits", int(n[5]), "out", rel_l2(got, ref),
          "mid", rel_l2(mid, rm))
    assert rel_l2(mid, rm) < TOL
    assert rel_l2(got, ref) < TOL


def test_tensor_core_c3_structure(oracle):
    """C3's structure on the tensor-core path: H 2880 (11.25 q8_K blocks, a
    zero-padded tail), MXFP4, gate/up/down and router biases, softmax
    routing, swiglu_oai; F reduced to 640 (a 128-value tail block in the
    q8_K mid rows) so the oracle finishes in seconds."""
    T = 448  # every expert gets 211-245 tokens: all on the tensor-core path
    L = HostLayer(H=2880, F=640, E=4, k=2, quant=12, seed=23, router_mode=1, act_op=2, biases=True)
    x = np.random.default_rng(9).normal(0, 1, (T, L.H)).astype(np.float32)
    _, sel, w = L.oracle_route(x)
    ref = L.oracle_ffn(x, sel, w)
    dl = L.to_device()
    wst = torch.zeros(dl.workspace_bytes(T), dtype=torch.uint8, device="cuda")
    out = torch.zeros((T, L.H), dtype=torch.float32, device="cuda")
    dl.forward(torch.from_numpy(x).cuda(), out, wst)
    torch.cuda.synchronize()
    v = dl.ws_view(wst, T)
    n = _ws(wst.cpu().numpy(), wst.data_ptr(), v.n_items, 6, np.uint32)
    assert n[4] > 0, "no tensor-core tiles at this batch"
    assert rel_l2(out.cpu().numpy(), ref) < TOL
