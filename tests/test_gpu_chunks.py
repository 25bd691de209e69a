"""Work units of <= 8 tokens: layers whose experts serve more tokens than
one unit holds (chunked work list), with and without a shared expert."""
import numpy as np
import pytest

from helpers import HostLayer, rel_l2

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

TC_MIN = 192  # experts with at least this many tokens take the tensor-core path (moe_layer.cu PM_TC_MIN)


@pytest.mark.parametrize("T", [8, 9, 16, 17])
@pytest.mark.parametrize("shared", [None, (2, 512)])
def test_token_chunks(oracle, T, shared):
    L = HostLayer(H=512, F=512, E=32, k=8, quant=2, seed=4, router_mode=0, zipf=(1.1, "select"), shared=shared)
    x = np.random.default_rng(9).normal(0, 1, (T, L.H)).astype(np.float32)
    _, sel, w = L.oracle_route(x)
    ref = L.oracle_ffn(x, sel, w)
    dl = L.to_device()
    ws = torch.zeros(dl.workspace_bytes(T), dtype=torch.uint8, device="cuda")
    out = torch.zeros((T, L.H), dtype=torch.float32, device="cuda")
    dl.forward(torch.from_numpy(x).cuda(), out, ws)
    torch.cuda.synchronize()
    got = out.cpu().numpy()
    per_tok = [round(rel_l2(got[t], ref[t]), 5) for t in range(T)]
    print(T, shared is not None, per_tok)
    assert rel_l2(got, ref) < 1e-3, per_tok


def _ws(ws, base, ptr, n, dt):
    off = ptr - base
    return ws[off:off + n * np.dtype(dt).itemsize].view(dt)


@pytest.mark.parametrize("rep", range(3))
def test_work_list_and_stages(oracle, rep):
    """CSR, work list, mid rows and down partials of one layer call"""
    T = 17
    L = HostLayer(H=512, F=512, E=32, k=8, quant=2, seed=4, router_mode=0, zipf=(1.1, "select"))
    x = np.random.default_rng(9).normal(0, 1, (T, L.H)).astype(np.float32)
    _, sel, w = L.oracle_route(x)
    dl = L.to_device()
    wst = torch.zeros(dl.workspace_bytes(T), dtype=torch.uint8, device="cuda")
    out = torch.zeros((T, L.H), dtype=torch.float32, device="cuda")
    dl.forward(torch.from_numpy(x).cuda(), out, wst)
    torch.cuda.synchronize()
    v = dl.ws_view(wst, T)
    ws, base = wst.cpu().numpy(), wst.data_ptr()
    n = _ws(ws, base, v.n_items, 6, np.uint32)
    ie = _ws(ws, base, v.item_expert, n[0], np.uint32)
    st = _ws(ws, base, v.item_start, n[0] + 1, np.uint32)
    pairs = _ws(ws, base, v.pairs, st[-1], np.uint32)
    wi = _ws(ws, base, v.work_item, n[2], np.uint32)
    w0 = _ws(ws, base, v.work_t0, n[2], np.uint32)
    k, ns = L.k, v.n_slot
    # every routed (t, s) exactly once, under its expert
    want = sorted((int(sel[t, s]), t * ns + s) for t in range(T) for s in range(k))
    got = sorted((int(ie[i]), int(p)) for i in range(n[0]) for p in pairs[st[i]:st[i + 1]])
    assert got == want, "CSR mismatch"
    # items of >= TC_MIN tokens go to tensor-core tiles of 64 tokens (Q4_K),
    # the rest to work units of 8; together they cover every item once
    tc = _ws(ws, base, v.tc_tile, 2 * n[4], np.uint32).reshape(-1, 2)
    size = {i: int(st[i + 1] - st[i]) for i in range(n[0])}
    tc_items = {int(i) for i in tc[:, 0]}
    assert tc_items == {i for i in range(n[0]) if size[i] >= TC_MIN}, "tensor-core item choice"
    assert sorted(map(tuple, tc.tolist())) == sorted((i, c) for i in tc_items for c in range(0, size[i], 64))
    units = sorted(zip(wi.tolist(), w0.tolist()))
    exp_units = sorted((i, c) for i in range(n[0]) if i not in tc_items for c in range(0, size[i], 8))
    assert units == exp_units, "work list mismatch"
    mid = _ws(ws, base, v.mid, T * ns * v.f_max, np.float32).reshape(T * ns, v.f_max)
    ref, ref_mid = L.oracle_ffn(x, sel, w, return_mid=True)
    bad_mid = [p for p in range(T * ns) if rel_l2(mid[p], ref_mid.reshape(T * ns, -1)[p]) > 1e-3]
    part = _ws(ws, base, v.partial, T * ns * L.H, np.float32).reshape(T * ns, L.H)
    zero_part = [p for p in range(T * ns) if not part[p].any()]
    got_out = out.cpu().numpy()
    bad_tok = [t for t in range(T) if rel_l2(got_out[t], ref[t]) > 1e-3]
    print("rep", rep, "bad_mid", bad_mid, "zero_partial", zero_part, "bad_tok", bad_tok)
    assert not bad_mid and not zero_part and not bad_tok
