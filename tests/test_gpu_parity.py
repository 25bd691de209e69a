"""GPU parity: the sm_100a kernels (through the C ABI) against the CPU oracle.

Bit-exact: q8_K bytes, router logits, top-k indices and route weights,
encoder bytes.  Expert-FFN outputs: relative L2 <= 1e-3 (north-star
tolerance) and the reference selftest bound max|d| <= 1e-3 * max(|ref|, 1)
(crates/kernels/cuda/pulsar_kernels.cu:6318-6319).
"""
import numpy as np
import pytest

from helpers import FMT, HostLayer, ref_close, rel_l2

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

TOL = 1e-3


@pytest.fixture(scope="module")
def pb():
    import pulsar_b200
    pulsar_b200.lib()
    return pulsar_b200


def dev(a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def host(t):
    torch.cuda.synchronize()
    return t.cpu().numpy()


@pytest.mark.parametrize("n,rows", [(2048, 3), (2880, 2), (704, 5), (7168, 1), (256, 64)])
def test_q8k_bitexact(oracle, pb, n, rows):
    from pulsar_b200 import ops
    rng = np.random.default_rng(n + rows)
    x = rng.normal(0, 1, (rows, n)).astype(np.float32)
    x[0, :17] = 0.0
    if rows > 1:
        x[1] = 0.0  # all-zero row
    out = torch.zeros(ops.q8k_bytes(n, rows), dtype=torch.uint8, device="cuda")
    ops.quantize_q8_k(out, dev(x), n, rows)
    assert np.array_equal(host(out), oracle.quantize_q8k(x).reshape(-1))


@pytest.mark.parametrize("E,H,T", [(128, 2048, 1), (256, 2048, 9), (32, 2880, 5), (256, 7168, 3), (896, 300, 2)])
def test_router_logits_bitexact(oracle, pb, E, H, T):
    from pulsar_b200 import ops
    rng = np.random.default_rng(E * H + T)
    W = rng.normal(0, 0.02, (E, H)).astype(np.float32)
    x = rng.normal(0, 1, (T, H)).astype(np.float32)
    out = torch.zeros((T, E), dtype=torch.float32, device="cuda")
    ops.matmul_f32(out, dev(W), dev(x), H, E, T)
    assert np.array_equal(host(out).view(np.uint32), oracle.router_logits(W, x).view(np.uint32))


@pytest.mark.parametrize("E,k,T,mode,G,TG", [(128, 8, 7, 1, 0, 0), (256, 8, 33, 0, 0, 0), (64, 4, 5, 0, 0, 0),
                                            (256, 8, 64, 0, 8, 4), (32, 4, 11, 1, 0, 0), (896, 16, 3, 0, 0, 0)])
def test_router_select_bitexact(oracle, pb, E, k, T, mode, G, TG):
    from pulsar_b200 import ops
    rng = np.random.default_rng(E + k + T)
    logits = (rng.normal(0, 2, (T, E))).astype(np.float32)
    logits[0, 3] = logits[0, 5]  # a tie: lower index wins
    bias = rng.normal(0, 0.2, E).astype(np.float32)
    sel_ref, w_ref = oracle.router_select(logits, bias, k, 1.7, mode, n_group=G, topk_group=TG)
    sel = torch.zeros((T, k), dtype=torch.int32, device="cuda")
    w = torch.zeros((T, k), dtype=torch.float32, device="cuda")
    if G:
        # group-limited selection goes through the fused router entry
        W = rng.normal(0, 0.02, (E, 64)).astype(np.float32)
        x = rng.normal(0, 1, (T, 64)).astype(np.float32)
        lg_ref = oracle.router_logits(W, x)
        sel_ref, w_ref = oracle.router_select(lg_ref, bias, k, 1.7, mode, n_group=G, topk_group=TG)
        lg = torch.zeros((T, E), dtype=torch.float32, device="cuda")
        ops.router_logits_select(sel, w, lg, dev(x), dev(W), None, dev(bias), 64, E, k, 1.7, T, mode, G, TG)
    else:
        ops.router_select(sel, w, dev(logits), dev(bias), E, k, 1.7, T, mode)
    assert np.array_equal(host(sel), sel_ref)
    assert np.array_equal(host(w).view(np.uint32), w_ref.view(np.uint32))


@pytest.mark.parametrize("fmt,n", [("Q4_K", 2048), ("Q2_K", 4096), ("Q8_0", 2880), ("MXFP4", 2880),
                                   ("IQ2_XXS", 2048)])
def test_gpu_encoders_bitexact(oracle, pb, fmt, n):
    from pulsar_b200 import ops
    q = FMT[fmt]
    rows = 24 if fmt == "IQ2_XXS" else 64
    rng = np.random.default_rng(q * 7 + n)
    x = rng.normal(0, 0.02, (rows, n)).astype(np.float32)
    x[1, :64] = 0.0
    qw = np.ones(n, np.float32) if fmt == "IQ2_XXS" else None
    rb = pb.row_bytes(q, n)
    out = torch.zeros(rows * rb, dtype=torch.uint8, device="cuda")
    ops.quantize_rows(out, dev(x), q, qw=None if qw is None else dev(qw))
    ref = oracle.quantize(q, x, qw).reshape(-1)
    got = host(out)
    bad = np.nonzero(got != ref)[0]
    assert bad.size == 0, f"{bad.size} bytes differ, first at {bad[:5]}"


CASES = [  # (fmt, H, F, E, k, T, act, biases)
    ("Q4_K", 512, 512, 8, 4, 3, 0, False),
    ("Q2_K", 1024, 512, 8, 4, 2, 0, False),
    ("IQ2_XXS", 512, 256, 8, 4, 3, 0, False),
    ("MXFP4", 704, 704, 8, 4, 3, 2, True),
    ("Q8_0", 704, 512, 8, 4, 2, 0, False),
]


def _ptr_records(L, dl, sel, T, k, null_slot=None):
    recs = []
    for t in range(T):
        for s in range(k):
            e = int(sel[t, s])
            if (t, s) == null_slot:
                recs.append(None)
                continue
            g, u, d = dl.expert_rows(e)
            r = dict(gate=g, up=u, down=d)
            if L.gate_b is not None:
                r.update(gate_b=dl.gate_b[e], up_b=dl.up_b[e], down_b=dl.down_b[e])
            recs.append(r)
    return recs


@pytest.mark.parametrize("case", CASES, ids=[c[0] for c in CASES])
def test_abi_pair_down_vs_oracle(oracle, pb, case):
    """pulsar_moe_pair_swiglu -> pulsar_quantize_q8_K -> pulsar_moe_down
    (+ down_bias), the engine's plain decode sequence (elib:8489-8506)."""
    from pulsar_b200 import ops
    fmt, H, F, E, k, T, act, biases = case
    q = FMT[fmt]
    L = HostLayer(H, F, E, k, q, seed=hash(case) % 1000, act_op=act, biases=biases)
    rng = np.random.default_rng(1)
    x = rng.normal(0, 1, (T, H)).astype(np.float32)
    _, sel, w = L.oracle_route(x)
    dl = L.to_device()
    null = (0, 1)  # one NULL slot (cu:6220)
    ptrs = ops.expert_ptrs_tensor(_ptr_records(L, dl, sel, T, k, null), "cuda")
    xq = torch.zeros(ops.q8k_bytes(H, T), dtype=torch.uint8, device="cuda")
    ops.quantize_q8_k(xq, dev(x), H, T)
    mid = torch.zeros((T, k, F), dtype=torch.float32, device="cuda")
    wd = dev(w)
    ops.moe_pair_swiglu(mid, ptrs, wd, xq, H, F, k, T, L.rb_gu, q, act)
    midq = torch.zeros(ops.q8k_bytes(F, T * k), dtype=torch.uint8, device="cuda")
    ops.quantize_q8_k(midq, mid, F, T * k)
    out = torch.zeros((T, H), dtype=torch.float32, device="cuda")
    ops.moe_down(out, ptrs, midq, F, H, k, T, L.rb_dn, q)
    if biases:
        ops.moe_down_bias(out, ptrs, wd, H, k, T)
    # oracle with the same NULL slot
    wref = w.copy()
    sel_n = sel.copy()
    sel_n[null] = -1
    ref, ref_mid = L.oracle_ffn(x, sel_n, wref, return_mid=True)
    g_mid = host(mid)
    assert float(np.abs(g_mid[null]).max()) == 0.0
    assert rel_l2(g_mid, ref_mid[:, :k, :F]) < TOL
    # q8_K of the GPU mids equals the oracle quantizer on the same values
    assert np.array_equal(host(midq), oracle.quantize_q8k(g_mid.reshape(T * k, F)).reshape(-1))
    got = host(out)
    assert rel_l2(got, ref) < TOL and ref_close(got, ref)
    assert pb.abi_error() == 0


@pytest.mark.parametrize("case", CASES[:3], ids=[c[0] for c in CASES[:3]])
def test_abi_grouped_vs_plain(oracle, pb, case):
    """grouped CSR entry points (elib:8356-8390 build) vs the oracle"""
    from pulsar_b200 import ops
    fmt, H, F, E, k, T, act, biases = case
    q = FMT[fmt]
    T = 19
    L = HostLayer(H, F, E, k, q, seed=5, act_op=act)
    rng = np.random.default_rng(2)
    x = rng.normal(0, 1, (T, H)).astype(np.float32)
    _, sel, w = L.oracle_route(x)
    dl = L.to_device()
    groups = {}
    for t in range(T):
        for s in range(k):
            groups.setdefault(int(sel[t, s]), []).append((t << 4) | s)
    gexp = list(groups)
    gptrs = ops.expert_ptrs_tensor([dict(zip(("gate", "up", "down"), dl.expert_rows(e))) for e in gexp], "cuda")
    starts = np.cumsum([0] + [len(groups[e]) for e in gexp]).astype(np.uint32)
    pairs = np.concatenate([np.array(groups[e], np.uint32) for e in gexp])
    xq = torch.zeros(ops.q8k_bytes(H, T), dtype=torch.uint8, device="cuda")
    ops.quantize_q8_k(xq, dev(x), H, T)
    mid = torch.zeros((T, k, F), dtype=torch.float32, device="cuda")
    ops.moe_pair_swiglu_grouped(mid, gptrs, dev(starts), dev(pairs), dev(w), xq, H, F, k, len(gexp), L.rb_gu, q, act)
    midq = torch.zeros(ops.q8k_bytes(F, T * k), dtype=torch.uint8, device="cuda")
    ops.quantize_q8_k(midq, mid, F, T * k)
    partial = torch.zeros((T, k, H), dtype=torch.float32, device="cuda")
    ops.moe_down_grouped(partial, gptrs, dev(starts), dev(pairs), midq, F, H, k, len(gexp), L.rb_dn, q)
    out = torch.zeros((T, H), dtype=torch.float32, device="cuda")
    ops.moe_slot_sum(out, partial, H, k, T)
    ref = L.oracle_ffn(x, sel, w)
    got = host(out)
    assert rel_l2(got, ref) < TOL and ref_close(got, ref)


LAYER_CASES = [  # (name, kwargs, T)
    ("C1-like", dict(H=512, F=768, E=16, k=8, quant=2, router_mode=1, zipf=(1.1, "logit")), 1),
    ("C1-like-T5", dict(H=512, F=768, E=16, k=8, quant=2, router_mode=1, zipf=(1.1, "logit")), 5),
    ("C2-like", dict(H=512, F=512, E=32, k=8, quant=2, router_mode=0, zipf=(1.1, "select"), shared=(2, 512)), 8),
    ("C3-like", dict(H=704, F=704, E=8, k=4, quant=12, router_mode=1, act_op=2, biases=True), 3),
    ("C4-like", dict(H=1024, F=512, E=16, k=8, quant=0, router_mode=1, zipf=(1.2, "logit")), 32),
    ("C5-like", dict(H=512, F=512, E=32, k=8, quant=1, router_mode=0, n_group=8, topk_group=4,
                     zipf=(1.1, "select"), shared=(10, 512)), 6),
]


@pytest.mark.parametrize("name,kw,T", LAYER_CASES, ids=[c[0] for c in LAYER_CASES])
def test_fused_layer_vs_oracle(oracle, pb, name, kw, T):
    L = HostLayer(seed=11, **kw)
    rng = np.random.default_rng(3)
    x = rng.normal(0, 1, (T, L.H)).astype(np.float32)
    resid = rng.normal(0, 1, (T, L.H)).astype(np.float32)
    lg, sel, w = L.oracle_route(x)
    ref = L.oracle_ffn(x, sel, w) + resid
    dl = L.to_device()
    ws = torch.zeros(dl.workspace_bytes(T), dtype=torch.uint8, device="cuda")
    out = torch.zeros((T, L.H), dtype=torch.float32, device="cuda")
    dl.forward(dev(x), out, ws, residual=dev(resid))
    got = host(out)
    v = dl.ws_view(ws, T)
    n_slot = v.n_slot
    # pull the workspace views back through torch (as raw bytes)
    base = ws.data_ptr()
    wsh = host(ws)

    def view(p, n, dt):
        off = p - base
        return wsh[off:off + n * np.dtype(dt).itemsize].view(dt)

    assert np.array_equal(view(v.logits, T * L.E, np.float32).reshape(T, L.E).view(np.uint32), lg.view(np.uint32))
    g_sel = view(v.selected, T * n_slot, np.int32).reshape(T, n_slot)
    g_w = view(v.weights, T * n_slot, np.float32).reshape(T, n_slot)
    assert np.array_equal(g_sel[:, :L.k], sel)
    assert np.array_equal(g_w[:, :L.k].view(np.uint32), w.view(np.uint32))
    xq_ref = oracle.quantize_q8k(x).reshape(-1)
    assert np.array_equal(view(v.xq, xq_ref.size, np.uint8), xq_ref)
    assert view(v.err, 1, np.uint32)[0] == 0
    assert rel_l2(got - resid, ref - resid) < TOL, name
    assert ref_close(got - resid, ref - resid)


def test_fused_layer_expert_shards_sum(oracle, pb):
    """expert-parallel shards [lo, hi) computed separately sum to the full
    layer, and each shard equals the oracle restricted to its experts"""
    L = HostLayer(H=512, F=512, E=32, k=8, quant=2, seed=4, router_mode=0, zipf=(1.1, "select"), shared=(2, 512))
    T = 9
    x = np.random.default_rng(9).normal(0, 1, (T, L.H)).astype(np.float32)
    _, sel, w = L.oracle_route(x)
    dl = L.to_device()
    ws = torch.zeros(dl.workspace_bytes(T), dtype=torch.uint8, device="cuda")
    full = torch.zeros((T, L.H), dtype=torch.float32, device="cuda")
    dl.forward(dev(x), full, ws)
    assert rel_l2(host(full), L.oracle_ffn(x, sel, w)) < TOL
    acc = np.zeros((T, L.H), np.float64)
    for lo, hi in ((0, 8), (8, 16), (16, 32)):
        dl.expert_lo, dl.expert_hi, dl._desc = lo, hi, None
        part = torch.zeros((T, L.H), dtype=torch.float32, device="cuda")
        dl.forward(dev(x), part, ws)
        got = host(part)
        ref = L.oracle_ffn(x, sel, w, lo=lo, hi=hi, with_shared=(lo == 0))
        assert rel_l2(got, ref) < TOL, (lo, hi, rel_l2(got, ref))
        acc += got
    assert rel_l2(acc, host(full)) < 1e-5
