"""Known-answer tests that pin the CPU oracle to the reference's own tests.

Each test restates one reference test with its seed and threshold:
  crates/quant/src/cpu_dot.rs:825-1097   dots vs an f64 dequant reference
  crates/quant/src/lib.rs:1052-1104      encoder round trips (rel RMSE)
  crates/quant/src/iq.rs:451-551         iq2_xxs tables + round trip
  crates/kernels/cuda/pulsar_kernels.cu:1140-1291  router selftest shapes
plus the IQ2_XXS grid and sign table pinned to the reference's CUDA tables
(tests/golden/iq2_tables.json, made by tests/golden/make_golden.py).
"""
import hashlib
import json
import math
import os

import numpy as np
import pytest

from rng import GqaRand, Lcg, lcg_random_row, xorshift_rows

GOLDEN = os.path.join(os.path.dirname(__file__), "golden")


def f16(b0, b1):
    return float(np.frombuffer(bytes([b0, b1]), np.float16)[0])


def k4_scale_min(j, q):
    if j < 4:
        return q[j] & 63, q[j + 4] & 63
    return (q[j + 4] & 15) | ((q[j - 4] >> 6) << 4), (q[j + 4] >> 4) | ((q[j] >> 6) << 4)


def f64_act(xq_bytes, n, orc):
    d, qs, _ = orc.q8k_fields(xq_bytes)
    return (d[:, None].astype(np.float64) * qs.astype(np.float64)).reshape(-1)[:n]


def test_iq2xxs_dot_matches_dequant(oracle):
    # cpu_dot.rs:825-851 dot_matches_dequant_reference (seed 42, n 2048)
    n = 2048
    st = Lcg(42)
    src = st.take(n)
    act = st.take(n)
    row = oracle.quantize(oracle.IQ2_XXS, src, np.ones(n, np.float32))[0]
    xq = oracle.quantize_q8k(act)[0]
    got = oracle.vec_dot(oracle.IQ2_XXS, row, xq, n)
    deq = oracle.dequant(oracle.IQ2_XXS, row, n).astype(np.float64)
    ref = float(np.sum(deq * f64_act(xq, n, oracle)))
    assert abs(got - ref) / max(abs(ref), 1e-6) < 1e-4
    true_dot = float(np.dot(src.astype(np.float64), act.astype(np.float64)))
    assert np.sign(ref) == np.sign(true_dot) or abs(true_dot) < 1.0


def _random_row(seed, n, block, scale_bytes):
    st = Lcg(seed)
    nb = n // 256
    row = lcg_random_row(st, nb * block)
    for ib in range(nb):
        for off in scale_bytes:
            row[ib * block + off] &= 0x3B
    act = st.take(n)
    return row, act


def test_q2k_dot_matches_dequant(oracle):
    # cpu_dot.rs:889-915 (seed 99, n 5120)
    n = 5120
    row, act = _random_row(99, n, 84, (81, 83))
    xq = oracle.quantize_q8k(act)[0]
    got = oracle.vec_dot(oracle.Q2_K, row, xq, n)
    a = f64_act(xq, n, oracle)
    ref = 0.0
    for ib in range(n // 256):
        b = row[ib * 84:(ib + 1) * 84]
        xd, xmin = f16(b[80], b[81]), f16(b[82], b[83])
        for c in range(16):
            k, js, half = c // 8, (c % 8) // 2, c % 2
            for i in range(16):
                q = (int(b[16 + 32 * k + 16 * half + i]) >> (2 * js)) & 3
                v = xd * (b[c] & 15) * q - xmin * (b[c] >> 4)
                ref += v * a[ib * 256 + 16 * c + i]
    assert abs(got - ref) / max(abs(ref), 1e-6) < 1e-4


def test_q4k_dot_matches_dequant(oracle):
    # cpu_dot.rs:957-995 (seed 424242, n 5120)
    n = 5120
    row, act = _random_row(424242, n, 144, (1, 3))
    xq = oracle.quantize_q8k(act)[0]
    got = oracle.vec_dot(oracle.Q4_K, row, xq, n)
    a = f64_act(xq, n, oracle)
    ref = 0.0
    for ib in range(n // 256):
        b = row[ib * 144:(ib + 1) * 144]
        xd, xmin = f16(b[0], b[1]), f16(b[2], b[3])
        sc = b[4:16]
        for j in range(4):
            sc1, m1 = k4_scale_min(2 * j, sc)
            sc2, m2 = k4_scale_min(2 * j + 1, sc)
            for i in range(32):
                v = int(b[16 + 32 * j + i])
                ref += (xd * sc1 * (v & 15) - xmin * m1) * a[ib * 256 + 64 * j + i]
                ref += (xd * sc2 * (v >> 4) - xmin * m2) * a[ib * 256 + 64 * j + 32 + i]
    assert abs(got - ref) / max(abs(ref), 1e-6) < 1e-4


@pytest.mark.parametrize("quant", ["MXFP4", "Q8_0"])
def test_block_format_dots_match_dequant(oracle, quant):
    # the reference GPU math of cu:2053 / cu:2174 vs an f64 dequant, n = 2880
    # (a partial tail super-block, the config-3 width)
    q = getattr(oracle, quant)
    n = 2880
    st = Lcg(2024)
    src = st.take(n) * np.float32(0.05)
    act = st.take(n)
    row = oracle.quantize(q, src)[0]
    xq = oracle.quantize_q8k(act)[0]
    got = oracle.vec_dot(q, row, xq, n)
    ref = float(np.sum(oracle.dequant(q, row, n).astype(np.float64) * f64_act(xq, n, oracle)))
    assert abs(got - ref) / max(abs(ref), 1e-6) < 1e-4


def _rel_rmse(x, y):
    x = x.astype(np.float64)
    y = y.astype(np.float64)
    return math.sqrt(np.mean((x - y) ** 2)) / math.sqrt(np.mean(x ** 2))


@pytest.mark.parametrize("quant,thr", [("Q8_0", 0.01), ("Q2_K", 0.30), ("Q4_K", 0.08)])
def test_encoder_roundtrip(oracle, quant, thr):
    # crates/quant/src/lib.rs:1052-1104 check() with rand_rows(QK_K*8, 42)
    q = getattr(oracle, quant)
    x = xorshift_rows(256 * 8, 42)
    enc = oracle.quantize(q, x)[0]
    assert enc.size == oracle.row_bytes(q, x.size)
    dec = oracle.dequant(q, enc, x.size)
    assert _rel_rmse(x, dec) < thr


def test_iq2xxs_roundtrip(oracle):
    # crates/quant/src/iq.rs:525-550 (xorshift seed 7, uniform imatrix)
    x = xorshift_rows(256 * 8, 7)
    enc = oracle.quantize(oracle.IQ2_XXS, x, np.ones_like(x))[0]
    assert enc.size == 8 * 66
    rel = _rel_rmse(x, oracle.dequant(oracle.IQ2_XXS, enc, x.size))
    assert rel < 0.6 and rel < 0.9


def test_mxfp4_roundtrip(oracle):
    # BASELINE-defined encoder: e2m1 with an E8M0 scale per 32 values.
    # Expected rel RMSE on gaussian-like rows sits near 0.1.
    x = xorshift_rows(256 * 8, 42)
    enc = oracle.quantize(oracle.MXFP4, x)[0]
    assert enc.size == 8 * 8 * 17
    assert _rel_rmse(x, oracle.dequant(oracle.MXFP4, enc, x.size)) < 0.15
    z = oracle.quantize(oracle.MXFP4, np.zeros(64, np.float32))[0]
    assert not z.any()


def test_q8k_quantizer_semantics(oracle):
    # cpu_dot.rs:26-50: d = amax/127, q = round-half-away(x*127/amax), i32 bsums
    x = xorshift_rows(512, 3)
    x[5] = -x[np.argmax(np.abs(x))] * 2  # a negative max
    b = oracle.quantize_q8k(x)[0]
    d, qs, bs = oracle.q8k_fields(b)
    for blk in range(2):
        v = x[blk * 256:(blk + 1) * 256]
        amax = np.float32(np.max(np.abs(v)))
        assert d[blk] == np.float32(amax / np.float32(127.0))
        inv = np.float32(np.float32(127.0) / amax)
        prod = (v * inv).astype(np.float32)
        q = np.clip(np.sign(prod) * np.floor(np.abs(prod) + np.float32(0.5)), -127, 127)
        assert np.array_equal(qs[blk].astype(np.int32), q.astype(np.int32))
        assert np.array_equal(bs[blk], qs[blk].astype(np.int32).reshape(16, 16).sum(1))
    # zero block and zero-padded tail (704 = 2.75 blocks)
    x = np.zeros(704, np.float32)
    x[:600] = xorshift_rows(600, 5)
    b = oracle.quantize_q8k(x)[0]
    d, qs, bs = oracle.q8k_fields(b)
    assert qs.shape == (3, 256) and not qs[2, 192:].any()
    b0 = oracle.quantize_q8k(np.zeros(256, np.float32))[0]
    assert not b0.any()


def test_iq2_tables_match_reference_cuda_tables(oracle):
    # iq.rs:478-501 reads the CUDA grid; here it is pinned by digest
    g = json.load(open(os.path.join(GOLDEN, "iq2_tables.json")))
    grid = b"".join(int(oracle.lib().orc_iq2xxs_grid(i)).to_bytes(8, "little") for i in range(256))
    assert hashlib.sha256(grid).hexdigest() == g["iq2xxs_grid_sha256"]
    ks = bytes(i | ((bin(i).count("1") & 1) << 7) for i in range(128))
    assert hashlib.sha256(ks).hexdigest() == g["ksigns_iq2xs_sha256"]


def test_expf_is_faithful(oracle):
    rng = np.random.default_rng(0)
    xs = np.concatenate([rng.uniform(-100, 88, 20000), rng.uniform(-5, 5, 20000),
                         np.array([0.0, -0.0, 1.0, -1.0, 88.7, -103.9])]).astype(np.float32)
    for x in xs:
        got = np.float32(oracle.lib().orc_expf(float(x)))
        ref = math.exp(float(x))
        if ref < 1.2e-38:  # subnormal range: absolute check
            assert abs(float(got) - ref) <= 1.5e-45
            continue
        ulp = float(np.spacing(np.float32(ref)))
        assert abs(float(got) - ref) <= 1.0 * ulp, (x, got, ref)  # faithful


def _reference_router_host(logits, bias, k, scale, softmax):
    """The reference selftest's host reference (cu:1156-1180): full softmax
    over all experts (or sigmoid), top-k by prob + bias, renormalize."""
    T, E = logits.shape
    sel = np.zeros((T, k), np.int32)
    w = np.zeros((T, k), np.float64)
    for t in range(T):
        lg = logits[t].astype(np.float64)
        if softmax:
            p = np.exp(lg - lg.max())
            p /= p.sum()
        else:
            p = 1.0 / (1.0 + np.exp(-lg))
        score = p + bias.astype(np.float64)
        for j in range(k):
            b = int(np.argmax(score))
            sel[t, j] = b
            w[t, j] = p[b]
            score[b] = -np.inf
        w[t] = w[t] / max(w[t].sum(), 6.103515625e-5) * scale
    return sel, w


@pytest.mark.parametrize("E,k,scale,T,softmax", [
    (64, 8, 2.5, 7, 0), (256, 8, 1.0, 5, 0), (96, 6, 1.5, 1, 0), (128, 8, 1.0, 6, 1),
    (384, 8, 1.0, 3, 1), (896, 16, 1.0, 3, 0), (896, 16, 1.0, 2, 1)])
def test_router_select_matches_reference_selftest(oracle, E, k, scale, T, softmax):
    # pulsar_router_selftest shapes (cu:1276-1290), idx exact, |w| <= 1e-5
    r = GqaRand()
    logits = np.array([r.next() * np.float32(4.0) for _ in range(T * E)], np.float32).reshape(T, E)
    bias = np.array([0.0 if softmax else r.next() for _ in range(E)], np.float32)
    sel, w = oracle.router_select(logits, bias, k, scale, softmax)
    rsel, rw = _reference_router_host(logits, bias, k, scale, softmax)
    assert np.array_equal(sel, rsel)
    assert np.max(np.abs(w - rw)) <= 1e-5


def test_router_sink_mode(oracle):
    # mode 2 (cu:1182-1266 router_sink_selftest_one): 256 routed + 2 shared, k 6
    r = GqaRand(99)
    E, S, k, T, scale = 256, 2, 6, 5, 8.0
    logits = np.array([r.next() * np.float32(4.0) for _ in range(T * (E + S))], np.float32).reshape(T, E + S)
    bias = np.array([r.next() for _ in range(E)], np.float32)
    sel, w = oracle.router_select(logits, bias, k, scale, 2, n_shexp=S)
    for t in range(T):
        score = 1.0 / (1.0 + np.exp(-logits[t, :E].astype(np.float64))) + bias
        top = []
        for _ in range(k):
            b = int(np.argmax(score))
            top.append(b)
            score[b] = -np.inf
        assert list(sel[t, :k]) == top and list(sel[t, k:]) == [E, E + 1]
        raw = np.concatenate([logits[t, top], logits[t, E:]]).astype(np.float64)
        ls = -np.log1p(np.exp(-raw))
        ref = np.exp(ls - ls.max())
        ref = ref / ref.sum() * scale
        assert np.max(np.abs(w[t] - ref)) <= 1e-5


def test_router_group_limited(oracle):
    # DeepSeek-V3 group-limited top-k (no reference counterpart): brute force
    rng = np.random.default_rng(11)
    T, E, k, G, TG = 9, 256, 8, 8, 4
    logits = rng.normal(0, 2, (T, E)).astype(np.float32)
    bias = rng.normal(0, 0.1, E).astype(np.float32)
    sel, w = oracle.router_select(logits, bias, k, 2.5, 0, n_group=G, topk_group=TG)
    for t in range(T):
        p = np.array([oracle.lib().orc_sigmoid(float(v)) for v in logits[t]], np.float32)
        score = (p + bias).astype(np.float32)
        gs = [float(np.float32(np.sort(score[g * 32:(g + 1) * 32])[-1] + np.sort(score[g * 32:(g + 1) * 32])[-2]))
              for g in range(G)]
        keep = sorted(range(G), key=lambda g: (-gs[g], g))[:TG]
        cand = [(-float(score[e]), e) for e in range(E) if e // 32 in keep]
        top = [e for _, e in sorted(cand)[:k]]
        assert list(sel[t]) == top
        pw = p[top]
        ref = pw / max(np.float32(pw.sum()), 6.103515625e-5) * 2.5
        assert np.max(np.abs(w[t] - ref)) <= 1e-6


def test_router_logits_fixed_order(oracle):
    rng = np.random.default_rng(5)
    E, H, T = 32, 2880, 3
    W = rng.normal(0, 0.02, (E, H)).astype(np.float32)
    x = rng.normal(0, 1, (T, H)).astype(np.float32)
    lg = oracle.router_logits(W, x)
    ref = (x.astype(np.float64) @ W.astype(np.float64).T)
    assert np.max(np.abs(lg - ref)) < 1e-5
