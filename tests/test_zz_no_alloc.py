"""pulsar_moe_layer_noalloc: the layer for callers that cannot allocate.

Some callers of this library own no device allocator: a plugin running
inside a host process that hands out all device memory from its own pool,
or code that must not call cudaMalloc (and synchronise the device) while it
runs.  pulsar_moe_layer_noalloc serves them from a fixed scratch array inside
the library.  This test calls it through the C ABI twice in a row (the array
keeps the previous call's contents) and checks each result against
pulsar_moe_layer with a caller-owned workspace, within the tolerance the
other layer tests use.  The file is collected last on purpose.
"""
import ctypes

import numpy as np
import pytest

from helpers import HostLayer, rel_l2

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

TOL = 1e-3


def test_noalloc_matches_workspace_layer_twice():
    import pulsar_b200
    from pulsar_b200._lib import LayerDesc, ptr

    lib = pulsar_b200.lib()
    lib.pulsar_moe_layer_noalloc.argtypes = [ctypes.POINTER(LayerDesc), ctypes.c_void_p, ctypes.c_void_p,
                                             ctypes.c_void_p, ctypes.c_uint32, ctypes.c_void_p]
    lib.pulsar_moe_layer_noalloc.restype = ctypes.c_int
    L = HostLayer(H=512, F=512, E=32, k=8, quant=2, seed=21, router_mode=0, zipf=(1.1, "select"), shared=(2, 512))
    dl = L.to_device()
    T = 11
    ws = torch.zeros(dl.workspace_bytes(T), dtype=torch.uint8, device="cuda")
    stream = torch.cuda.current_stream().cuda_stream
    for call in range(2):
        x = torch.from_numpy(np.random.default_rng(100 + call).normal(0, 1, (T, L.H)).astype(np.float32)).cuda()
        resid = torch.from_numpy(np.random.default_rng(200 + call).normal(0, 1, (T, L.H)).astype(np.float32)).cuda()
        want = torch.zeros((T, L.H), dtype=torch.float32, device="cuda")
        dl.forward(x, want, ws, residual=resid)
        got = torch.full((T, L.H), float("nan"), dtype=torch.float32, device="cuda")
        ok = lib.pulsar_moe_layer_noalloc(ctypes.byref(dl.desc()), ptr(got), ptr(x), ptr(resid), T, stream)
        assert ok == 1, f"call {call} returned 0"
        torch.cuda.synchronize()
        g, w = got.cpu().numpy(), want.cpu().numpy()
        assert np.isfinite(g).all()
        assert rel_l2(g - resid.cpu().numpy(), w - resid.cpu().numpy()) < TOL, f"call {call}"


def test_noalloc_rejects_oversize():
    import pulsar_b200
    from pulsar_b200._lib import LayerDesc

    lib = pulsar_b200.lib()
    lib.pulsar_moe_layer_noalloc.argtypes = [ctypes.POINTER(LayerDesc), ctypes.c_void_p, ctypes.c_void_p,
                                             ctypes.c_void_p, ctypes.c_uint32, ctypes.c_void_p]
    L = HostLayer(H=512, F=512, E=32, k=8, quant=2, seed=21, router_mode=0)
    dl = L.to_device()
    T = 4096  # workspace far above the built-in 32 MiB
    assert dl.workspace_bytes(T) > (32 << 20)
    out = torch.zeros((1, L.H), dtype=torch.float32, device="cuda")
    assert lib.pulsar_moe_layer_noalloc(ctypes.byref(dl.desc()), out.data_ptr(), out.data_ptr(), None, T, None) == 0
