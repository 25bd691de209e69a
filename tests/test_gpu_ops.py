"""The standalone reference entry points around the expert path, through
the C ABI on the GPU: pulsar_add_bias_rows (cu:3631), pulsar_swiglu
(cu:6551), pulsar_add (cu:6754) and pulsar_rms_norm (cu:6494).  add and the
bias rows are one f32 add per element (bit-exact against numpy); swiglu
against the oracle's glu (this library's exp vs glibc expf: rel 2e-6);
rms_norm against a binary64 numpy reference (rel 2e-6)."""
import numpy as np
import pytest

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def ops():
    import pulsar_b200
    from pulsar_b200 import ops as o
    pulsar_b200.lib()
    return o


def dev(a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def test_add_bias_rows(ops):
    rng = np.random.default_rng(1)
    x = rng.normal(0, 1, (37, 2880)).astype(np.float32)
    b = rng.normal(0, 0.01, 2880).astype(np.float32)
    xd = dev(x)
    ops.add_bias_rows(xd, dev(b), 2880, 37)
    assert np.array_equal(xd.cpu().numpy(), x + b[None])


def test_add(ops):
    rng = np.random.default_rng(2)
    a, b = (rng.normal(0, 1, 100_003).astype(np.float32) for _ in range(2))
    out = torch.zeros(100_003, dtype=torch.float32, device="cuda")
    ops.add(out, dev(a), dev(b), 100_003)
    assert np.array_equal(out.cpu().numpy(), a + b)


@pytest.mark.parametrize("act,clamp,weight", [(0, 0.0, 1.0), (0, 0.0, 0.37), (2, 7.0, 1.0), (2, 7.0, 0.5)])
def test_swiglu(ops, oracle, act, clamp, weight):
    n = 4099
    rng = np.random.default_rng(3 + act)
    g = rng.normal(0, 4, n).astype(np.float32)
    u = rng.normal(0, 4, n).astype(np.float32)
    out = torch.zeros(n, dtype=torch.float32, device="cuda")
    ops.swiglu(out, dev(g), dev(u), n, clamp=clamp, weight=weight, act_op=act)
    gc, uc = g, u
    if clamp > 1e-6:
        gc = np.minimum(g, np.float32(clamp))
        uc = np.clip(u, np.float32(-clamp), np.float32(clamp))
    L = oracle.lib()
    ref = np.array([L.orc_glu(float(a), float(b), act) for a, b in zip(gc, uc)], np.float32) * np.float32(weight)
    got = out.cpu().numpy()
    assert np.allclose(got, ref, rtol=2e-6, atol=1e-30), float(np.max(np.abs(got - ref)))


@pytest.mark.parametrize("n,rows,with_w", [(2048, 9, False), (2880, 5, True), (7168, 3, True)])
def test_rms_norm(ops, n, rows, with_w):
    rng = np.random.default_rng(n)
    x = rng.normal(0, 3, (rows, n)).astype(np.float32)
    w = rng.normal(1, 0.1, n).astype(np.float32) if with_w else None
    import pulsar_b200
    from pulsar_b200._lib import check, ptr
    out = torch.zeros((rows, n), dtype=torch.float32, device="cuda")
    xd, wd = dev(x), None if w is None else dev(w)
    check(pulsar_b200.lib().pulsar_rms_norm(ptr(out), ptr(xd), ptr(wd), n, rows, 1e-6), "rms_norm")
    torch.cuda.synchronize()
    x64 = x.astype(np.float64)
    ref = x64 / np.sqrt(np.mean(x64 ** 2, axis=1, keepdims=True) + 1e-6)
    if w is not None:
        ref = ref * w.astype(np.float64)[None]
    assert np.allclose(out.cpu().numpy(), ref, rtol=2e-6, atol=1e-7)
