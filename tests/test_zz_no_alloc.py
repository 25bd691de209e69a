"""pulsar_moe_layer_noalloc: the layer for callers that cannot allocate.

Some callers of this library own no device allocator: a plugin running
inside a host process that hands out all device memory from its own pool,
or code that must not call cudaMalloc (and synchronise the device) while it
runs.  pulsar_moe_layer_noalloc serves them from a fixed scratch array inside
the library.  This test calls it through the C ABI several times in a row -
the array keeps each call's contents, and the calls change batch size and
descriptor (shared expert on and off, a larger call that dirties more of the
array in between) - and checks every result against pulsar_moe_layer with a
caller-owned workspace and against the CPU oracle, within the tolerance the
other layer tests use.  The call's error word is read through
pulsar_moe_layer_ws_view with a NULL workspace.  The file is collected last
on purpose.
"""
import ctypes

import numpy as np
import pytest

from helpers import HostLayer, rel_l2

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

TOL = 1e-3


def _bind():
    import pulsar_b200
    from pulsar_b200._lib import LayerDesc, WsView
    lib = pulsar_b200.lib()
    lib.pulsar_moe_layer_noalloc.argtypes = [ctypes.POINTER(LayerDesc), ctypes.c_void_p, ctypes.c_void_p,
                                             ctypes.c_void_p, ctypes.c_uint32, ctypes.c_void_p]
    lib.pulsar_moe_layer_noalloc.restype = ctypes.c_int
    lib.pulsar_moe_layer_ws_view.argtypes = [ctypes.POINTER(LayerDesc), ctypes.c_uint32, ctypes.c_void_p,
                                             ctypes.POINTER(WsView)]
    lib.cudaMemcpy.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_size_t, ctypes.c_int]
    lib.cudaMemcpy.restype = ctypes.c_int
    return lib, WsView


def test_noalloc_matches_workspace_layer_and_oracle():
    from pulsar_b200._lib import ptr

    lib, WsView = _bind()
    shared = HostLayer(H=512, F=512, E=32, k=8, quant=2, seed=21, router_mode=0, zipf=(1.1, "select"),
                       shared=(2, 512))
    plain = HostLayer(H=512, F=512, E=16, k=4, quant=0, seed=22, router_mode=1, zipf=(1.2, "logit"))
    layers = {"shared": (shared, shared.to_device()), "plain": (plain, plain.to_device())}
    stream = torch.cuda.current_stream().cuda_stream
    # (layer, tokens): repeated calls, a large one (more of the array written) between small ones
    calls = [("shared", 11), ("shared", 11), ("plain", 3), ("shared", 64), ("plain", 1), ("shared", 5)]
    for i, (name, T) in enumerate(calls):
        H, dl = layers[name]
        rng = np.random.default_rng(100 + i)
        x_h = rng.normal(0, 1, (T, H.H)).astype(np.float32)
        r_h = rng.normal(0, 1, (T, H.H)).astype(np.float32)
        _, sel, w = H.oracle_route(x_h)
        ref = H.oracle_ffn(x_h, sel, w)
        x, resid = torch.from_numpy(x_h).cuda(), torch.from_numpy(r_h).cuda()
        ws = torch.zeros(dl.workspace_bytes(T), dtype=torch.uint8, device="cuda")
        want = torch.zeros((T, H.H), dtype=torch.float32, device="cuda")
        dl.forward(x, want, ws, residual=resid)
        got = torch.full((T, H.H), float("nan"), dtype=torch.float32, device="cuda")
        ok = lib.pulsar_moe_layer_noalloc(ctypes.byref(dl.desc()), ptr(got), ptr(x), ptr(resid), T, stream)
        assert ok == 1, f"call {i} returned 0"
        torch.cuda.synchronize()
        v = WsView()
        assert lib.pulsar_moe_layer_ws_view(ctypes.byref(dl.desc()), T, None, ctypes.byref(v)) == 1
        err = np.zeros(1, np.uint32)
        assert lib.cudaMemcpy(err.ctypes.data, v.err, 4, 2) == 0  # cudaMemcpyDeviceToHost
        assert err[0] == 0, f"call {i}: error word {err[0]}"
        g, wnt = got.cpu().numpy() - r_h, want.cpu().numpy() - r_h
        assert np.isfinite(g).all()
        assert rel_l2(g, wnt) < TOL, f"call {i} vs pulsar_moe_layer"
        assert rel_l2(g, ref) < TOL, f"call {i} vs oracle"


def test_noalloc_rejects_oversize():
    lib, _ = _bind()
    L = HostLayer(H=512, F=512, E=32, k=8, quant=2, seed=21, router_mode=0)
    dl = L.to_device()
    T = 4096  # workspace far above the built-in 32 MiB
    assert dl.workspace_bytes(T) > (32 << 20)
    out = torch.zeros((1, L.H), dtype=torch.float32, device="cuda")
    assert lib.pulsar_moe_layer_noalloc(ctypes.byref(dl.desc()), out.data_ptr(), out.data_ptr(), None, T, None) == 0
