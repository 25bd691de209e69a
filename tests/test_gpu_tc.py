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
    dl.desc().path_flags = 1  # PULSAR_LAYER_NO_I8: Q2_K experts on the fp16 tiles too
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


IMG_CASES = [2, 0, 1, 10, 12]  # Q4_K, Q2_K, IQ2_XXS, Q8_0, MXFP4


@pytest.mark.parametrize("quant", IMG_CASES, ids=[f"q{q}" for q in IMG_CASES])
def test_tensor_core_weight_images(oracle, quant):
    """The dequantized weights the tensor cores multiply: every down-pass
    image pair (fp16 hi + lo, 128 rows x 64 K) of every tensor-core expert
    against the oracle's f32 dequant of the same blocks.  hi + lo equals the
    f32 weight to |w - (hi + lo)| <= 2^-22 |w| + 2^-25 (hi = fp16(w), lo =
    fp16(w - hi); the 2^-25 term is half the fp16 subnormal spacing of lo);
    MXFP4 weights are exact in fp16: hi == w and no lo image is written."""
    from helpers import reader, sw128_unswizzle, tc_images
    T = 512  # about 256 tokens per expert: every expert on the tensor-core path
    L = HostLayer(H=512, F=512, E=4, k=2, quant=quant, seed=31, router_mode=0)
    x = np.random.default_rng(6).normal(0, 1, (T, L.H)).astype(np.float32)
    dl = L.to_device()
    dl.desc().path_flags = 1  # PULSAR_LAYER_NO_I8: Q2_K experts on the fp16 tiles too
    wst = torch.zeros(dl.workspace_bytes(T), dtype=torch.uint8, device="cuda")
    out = torch.zeros((T, L.H), dtype=torch.float32, device="cuda")
    dl.forward(torch.from_numpy(x).cuda(), out, wst)
    torch.cuda.synchronize()
    v = dl.ws_view(wst, T)
    rd = reader(wst)
    items = tc_images(rd, v)
    assert items and len(items) <= v.tc_slots
    item_expert = rd(v.item_expert, max(items) + 1, np.uint32)
    H, F = L.H, L.F
    nch, pairs_per_slot = F // 64, v.tc_slot_bytes // (2 * 16384)
    worst = 0.0
    for o, item in enumerate(items):
        e = int(item_expert[item])
        down = L.down[e]
        deq = np.stack([oracle.dequant(quant, down[r * L.rb_dn:(r + 1) * L.rb_dn], F) for r in range(H)])
        for rt in range(H // 128):
            for c in range(nch):
                pi = rt * nch + c
                pair = rd(v.tc_img + o * v.tc_slot_bytes + pi * 2 * 16384, 2 * 16384, np.uint8)
                hi = sw128_unswizzle(pair[:16384]).astype(np.float32)
                has_lo = rd(v.tc_lo + o * pairs_per_slot + pi, 1, np.uint8)[0]
                lo = sw128_unswizzle(pair[16384:]).astype(np.float32) if has_lo else np.zeros_like(hi)
                wv = deq[128 * rt:128 * rt + 128, 64 * c:64 * c + 64]
                if quant == 12:
                    assert not has_lo and np.array_equal(hi, wv), (e, rt, c)
                    continue
                d = np.abs(wv.astype(np.float64) - (hi.astype(np.float64) + lo))
                bound = np.abs(wv.astype(np.float64)) * 2.0 ** -22 + 2.0 ** -25
                worst = max(worst, float(np.max(d / bound)))
                assert np.all(d <= bound), (e, rt, c, float(np.max(d)))
    print(f"quant {quant}: {len(items)} experts, worst |w - (hi + lo)| / bound {worst:.3f}")
