"""Shared test helpers: host-built layers (oracle encoders) mirrored on the
device, and the oracle's full-layer reference computation."""
from __future__ import annotations

import numpy as np

import oracle as orc

FMT = {"Q2_K": 0, "IQ2_XXS": 1, "Q4_K": 2, "Q8_0": 10, "MXFP4": 12}


def rel_l2(a, b) -> float:
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30))


def ref_close(got, ref, rel=1e-3):
    """the reference selftest criterion: max |d| <= rel * max(max|ref|, 1)"""
    got = np.asarray(got, np.float64)
    ref = np.asarray(ref, np.float64)
    return float(np.max(np.abs(got - ref))) <= rel * max(float(np.max(np.abs(ref))), 1.0)


class HostLayer:
    """A layer built on the host with the oracle encoders (numpy bytes)."""

    def __init__(self, H, F, E, k, quant, seed, router_mode=1, act_op=0, n_group=0, topk_group=0,
                 weight_scale=1.0, shared=None, biases=False, zipf=None, std=0.02):
        rng = np.random.default_rng(seed)
        self.H, self.F, self.E, self.k, self.quant = H, F, E, k, quant
        self.router_mode, self.act_op = router_mode, act_op
        self.n_group, self.topk_group, self.weight_scale = n_group, topk_group, weight_scale
        qw = np.ones(H, np.float32) if quant == 1 else None
        qwf = np.ones(F, np.float32) if quant == 1 else None
        self.rb_gu, self.rb_dn = orc.row_bytes(quant, H), orc.row_bytes(quant, F)
        self.gate = orc.quantize(quant, rng.normal(0, std, (E * F, H)).astype(np.float32), qw).reshape(E, F * self.rb_gu)
        self.up = orc.quantize(quant, rng.normal(0, std, (E * F, H)).astype(np.float32), qw).reshape(E, F * self.rb_gu)
        self.down = orc.quantize(quant, rng.normal(0, std, (E * H, F)).astype(np.float32), qwf).reshape(E, H * self.rb_dn)
        self.router_w = rng.normal(0, std, (E, H)).astype(np.float32)
        self.logit_b = None
        self.select_b = None
        if zipf is not None:
            s, kind = zipf
            rank = rng.permutation(E).astype(np.float64) + 1.0
            if kind == "select":
                self.select_b = (rank ** -s).astype(np.float32)
            else:
                self.logit_b = (-s * np.log(rank)).astype(np.float32)
        self.gate_b = self.up_b = self.down_b = None
        if biases:
            self.gate_b = rng.normal(0, 0.01, (E, F)).astype(np.float32)
            self.up_b = rng.normal(0, 0.01, (E, F)).astype(np.float32)
            self.down_b = rng.normal(0, 0.01, (E, H)).astype(np.float32)
            lb = rng.normal(0, 0.01, E).astype(np.float32)
            self.logit_b = lb if self.logit_b is None else (self.logit_b + lb).astype(np.float32)
        self.shared = None
        if shared is not None:
            sq, Fs = shared
            qs = np.ones(H, np.float32) if sq == 1 else None
            qsf = np.ones(Fs, np.float32) if sq == 1 else None
            self.shared = dict(
                quant=sq, F=Fs, rb_gu=orc.row_bytes(sq, H), rb_dn=orc.row_bytes(sq, Fs),
                gate=orc.quantize(sq, rng.normal(0, std, (Fs, H)).astype(np.float32), qs).reshape(-1),
                up=orc.quantize(sq, rng.normal(0, std, (Fs, H)).astype(np.float32), qs).reshape(-1),
                down=orc.quantize(sq, rng.normal(0, std, (H, Fs)).astype(np.float32), qsf).reshape(-1))

    # ------------------------------------------------------------ oracle
    def oracle_route(self, x):
        lg = orc.router_logits(self.router_w, x, self.logit_b)
        sel, w = orc.router_select(lg, self.select_b, self.k, self.weight_scale, self.router_mode,
                                   n_group=self.n_group, topk_group=self.topk_group)
        return lg, sel, w

    def oracle_ffn(self, x, sel, w, lo=0, hi=None, with_shared=True, return_mid=False):
        hi = self.E if hi is None else hi
        T = x.shape[0]
        ns = 1 if (self.shared is not None and with_shared) else 0
        slots, ws = [], np.zeros((T, self.k + ns), np.float32)
        for t in range(T):
            row = []
            for s in range(self.k):
                e = int(sel[t, s])
                ws[t, s] = w[t, s]
                if lo <= e < hi:
                    d = dict(gate=self.gate[e], up=self.up[e], down=self.down[e])
                    if self.gate_b is not None:
                        d.update(gate_b=self.gate_b[e], up_b=self.up_b[e], down_b=self.down_b[e])
                    row.append(d)
                else:
                    row.append(None)
            if ns:
                ws[t, self.k] = 1.0
                row.append(dict(gate=self.shared["gate"], up=self.shared["up"], down=self.shared["down"]))
            slots.append(row)
        sh = None
        if ns:
            s = self.shared
            sh = (s["F"], s["quant"], s["rb_gu"], s["rb_dn"])
        return orc.moe_ffn(x, slots, ws, self.H, self.k, (self.F, self.quant, self.rb_gu, self.rb_dn), sh,
                           act_op=self.act_op, return_mid=return_mid)

    # ------------------------------------------------------------ device
    def to_device(self):
        import torch
        from pulsar_b200 import LayerSpec, MoeLayer

        dev = torch.device("cuda")

        def up_(a, slack=True):
            a = np.ascontiguousarray(a)
            if a.dtype != np.uint8:  # f32 tensors keep their shape ([E][F] bias rows)
                return torch.from_numpy(a.copy()).to(dev)
            t = torch.from_numpy(a.reshape(-1).copy())
            if slack:
                t = torch.cat([t, torch.zeros(256, dtype=torch.uint8)])
            return t.to(dev)

        spec = LayerSpec(n_embd=self.H, n_ff=self.F, n_expert=self.E, n_used=self.k, quant=self.quant,
                         act_op=self.act_op, router_mode=self.router_mode, n_group=self.n_group,
                         topk_group=self.topk_group, weight_scale=self.weight_scale,
                         shared_quant=None if self.shared is None else self.shared["quant"],
                         shared_n_ff=0 if self.shared is None else self.shared["F"])
        L = MoeLayer(spec=spec, gate=up_(self.gate), up=up_(self.up), down=up_(self.down),
                     router_w=up_(self.router_w))
        L.router_logit_b = None if self.logit_b is None else up_(self.logit_b)
        L.router_select_b = None if self.select_b is None else up_(self.select_b)
        if self.gate_b is not None:
            L.gate_b, L.up_b, L.down_b = up_(self.gate_b), up_(self.up_b), up_(self.down_b)
        if self.shared is not None:
            L.shared_gate, L.shared_up, L.shared_down = (up_(self.shared[n]) for n in ("gate", "up", "down"))
        L.build_tiles()
        return L


class DeviceMirror:
    """The oracle's view of a layer built on the device (make_layer: GPU
    block encoders, byte-identical to the crates/quant encoders): router
    weights, biases and the slabs of the experts a batch selects are copied
    to the host on demand, so true-size layers (GBs of experts) are checked
    against the oracle without encoding them on the CPU."""

    def __init__(self, layer):
        s = layer.spec
        self.dl, self.spec = layer, s
        self.H, self.F, self.E, self.k, self.quant = s.n_embd, s.n_ff, s.n_expert, s.n_used, s.quant
        self.router_mode, self.act_op = s.router_mode, s.act_op
        self.n_group, self.topk_group, self.weight_scale = s.n_group, s.topk_group, s.weight_scale
        self.rb_gu, self.rb_dn = layer.rb_gu, layer.rb_down

        def h(t):
            return None if t is None else t.detach().cpu().numpy()

        self.router_w = h(layer.router_w)
        self.logit_b, self.select_b = h(layer.router_logit_b), h(layer.router_select_b)
        self.gate_b, self.up_b, self.down_b = h(layer.gate_b), h(layer.up_b), h(layer.down_b)
        self.shared = None
        self.shared_gate_w = None
        if s.shared_quant is not None:
            sq, Fs = s.shared_quant, s.shared_n_ff
            self.shared = dict(quant=sq, F=Fs, rb_gu=orc.row_bytes(sq, self.H), rb_dn=orc.row_bytes(sq, Fs))
            self.shared_gate_w = h(layer.shared_gate_w)
            for n, t, rows, rb in (("gate", layer.shared_gate, Fs, self.shared["rb_gu"]),
                                   ("up", layer.shared_up, Fs, self.shared["rb_gu"]),
                                   ("down", layer.shared_down, self.H, self.shared["rb_dn"])):
                self.shared[n] = t[:rows * rb].cpu().numpy()
        self._exp = {}

    def expert(self, e: int):
        if e not in self._exp:
            g, u, d = self.dl.expert_rows(e)
            self._exp[e] = tuple(t.cpu().numpy() for t in (g, u, d))
        return self._exp[e]

    def oracle_route(self, x):
        lg = orc.router_logits(self.router_w, x, self.logit_b)
        sel, w = orc.router_select(lg, self.select_b, self.k, self.weight_scale, self.router_mode,
                                   n_group=self.n_group, topk_group=self.topk_group)
        return lg, sel, w

    def oracle_ffn(self, x, sel, w, with_shared=True, return_mid=False):
        T = x.shape[0]
        ns = 1 if (self.shared is not None and with_shared) else 0
        slots, ws = [], np.zeros((T, self.k + ns), np.float32)
        for t in range(T):
            row = []
            for s in range(self.k):
                e = int(sel[t, s])
                ws[t, s] = w[t, s]
                g, u, d = self.expert(e)
                dd = dict(gate=g, up=u, down=d)
                if self.gate_b is not None:
                    dd.update(gate_b=self.gate_b[e], up_b=self.up_b[e], down_b=self.down_b[e])
                row.append(dd)
            if ns:
                ws[t, self.k] = 1.0
                row.append(dict(gate=self.shared["gate"], up=self.shared["up"], down=self.shared["down"]))
            slots.append(row)
        sh = None
        if ns:
            s = self.shared
            sh = (s["F"], s["quant"], s["rb_gu"], s["rb_dn"])
        if ns and self.shared_gate_w is not None:
            # qwen35 (real/qwen35.rs:2160-2169): moe_out + sigmoid(gate_w . x) * shared_out
            routed = orc.moe_ffn(x, [r[:self.k] for r in slots], np.ascontiguousarray(ws[:, :self.k]), self.H,
                                 self.k, (self.F, self.quant, self.rb_gu, self.rb_dn), None, act_op=self.act_op,
                                 return_mid=return_mid)
            mid = None
            if return_mid:
                routed, mid = routed
            shared = orc.moe_ffn(x, [r[self.k:] for r in slots], np.ascontiguousarray(ws[:, self.k:]), self.H, 0,
                                 (self.F, self.quant, self.rb_gu, self.rb_dn), sh, act_op=self.act_op)
            s_ = orc.router_logits(self.shared_gate_w[None, :], x)[:, 0]
            g = (np.float32(1.0) / (np.float32(1.0) + np.exp(-s_).astype(np.float32))).astype(np.float32)
            out = (routed + shared * g[:, None]).astype(np.float32)
            return (out, mid) if return_mid else out
        return orc.moe_ffn(x, slots, ws, self.H, self.k, (self.F, self.quant, self.rb_gu, self.rb_dn), sh,
                           act_op=self.act_op, return_mid=return_mid)


def reader(ws):
    """rd(device pointer, n, dtype): n elements of a workspace region, copied to the host"""
    base = ws.data_ptr()

    def rd(p, n, dt):
        nb = n * np.dtype(dt).itemsize
        return ws[p - base:p - base + nb].cpu().numpy().view(dt)
    return rd


def tc_images(rd, v):
    """The items (CSR expert entries) of the tensor-core experts of the last
    layer call, in ordinal order: image slot o of the last wave holds the
    last pass's (down) images of items[o].  Ordinals are dense over the
    tiles' items in tile order (the first tile of an item has t0 0).
    rd(pointer, n, dtype) reads device memory."""
    n = rd(v.n_items, 7, np.uint32)
    tiles = rd(v.tc_tile, 2 * int(n[4]), np.uint32).reshape(-1, 2)
    items = [int(it) for it, t0 in tiles if t0 == 0]
    return items


def sw128_unswizzle(img: np.ndarray) -> np.ndarray:
    """128 x 64 fp16 K-major tile in the 128-byte swizzle -> [128][64] fp16"""
    b = img.reshape(16, 8, 8, 16)  # atom, row in atom, 16-byte chunk position, bytes
    out = np.zeros((128, 64), np.float16)
    for r in range(128):
        for j in range(8):
            out[r, 8 * j:8 * j + 8] = b[r >> 3, r & 7, j ^ (r & 7)].view(np.float16)
    return out
