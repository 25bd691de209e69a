"""MoE layers on the device: weights, descriptor, the one-call forward.

MoeLayer holds one routed-expert FFN layer the way the reference engine
holds it (expert slabs per tensor, slab e at base + e * rows * row_bytes,
crates/engine/src/lib.rs:576-592; router weight as f32, elib:2884-2921),
builds the pulsar_moe_layer_desc and runs the layer through
pulsar_moe_layer (router -> q8_K -> gate/up + glu -> q8_K -> down ->
combine, all on the GPU).  make_layer() creates seeded synthetic layers:
f32 N(0, std) weights generated on the device and quantized with the GPU
block encoders (byte-identical to the crates/quant encoders).
"""
from __future__ import annotations

import ctypes
import math
from dataclasses import dataclass, field

import torch

from ._lib import QUANT_Q2_K, LayerDesc, WsView, check, lib, ptr, row_bytes
from .ops import quantize_rows

SLAB_SLACK = 256  # tail slack after every slab (crates/engine/src/lib.rs:594-600)


@dataclass
class LayerSpec:
    n_embd: int
    n_ff: int
    n_expert: int
    n_used: int
    quant: int
    act_op: int = 0
    router_mode: int = 1          # 0 sigmoid + selection bias, 1 softmax
    n_group: int = 0
    topk_group: int = 0
    weight_scale: float = 1.0
    zipf_s: float = 0.0           # router bias skew (0 = none)
    zipf_kind: str = "logit"      # "logit" (added to logits) or "select" (selection score only)
    shared_quant: int | None = None
    shared_n_ff: int = 0
    biases: bool = False          # per-expert gate/up/down biases + router logit bias
    router_q8_0: bool = False     # router weights stored as Q8_0 and used as their exact f32 dequant
    shared_gate: bool = False     # qwen35 sigmoid gate on the shared expert's output (a [n_embd] vector)
    weight_std: float = 0.02
    bias_std: float = 0.01


@dataclass
class MoeLayer:
    spec: LayerSpec
    gate: torch.Tensor
    up: torch.Tensor
    down: torch.Tensor
    router_w: torch.Tensor
    router_logit_b: torch.Tensor | None = None
    router_select_b: torch.Tensor | None = None
    gate_b: torch.Tensor | None = None
    up_b: torch.Tensor | None = None
    down_b: torch.Tensor | None = None
    shared_gate: torch.Tensor | None = None
    shared_up: torch.Tensor | None = None
    shared_down: torch.Tensor | None = None
    shared_gate_w: torch.Tensor | None = None
    expert_lo: int = 0
    expert_hi: int = 0
    slab_lo: int = 0              # first expert held in the routed slabs (shards hold [slab_lo, expert_hi))
    # Q2_K tile-plane images of gate / up / down (pulsar_repack_q2k_tiles), for the integer tensor-core passes
    gate_tiles: torch.Tensor | None = None
    up_tiles: torch.Tensor | None = None
    down_tiles: torch.Tensor | None = None
    _desc: LayerDesc | None = field(default=None, repr=False)

    # ---------------------------------------------------------- geometry
    @property
    def rb_gu(self) -> int:
        return row_bytes(self.spec.quant, self.spec.n_embd)

    @property
    def rb_down(self) -> int:
        return row_bytes(self.spec.quant, self.spec.n_ff)

    def weight_bytes_per_expert(self) -> int:
        s = self.spec
        return 2 * s.n_ff * self.rb_gu + s.n_embd * self.rb_down

    def shared_bytes(self) -> int:
        s = self.spec
        if s.shared_quant is None:
            return 0
        return (2 * s.shared_n_ff * row_bytes(s.shared_quant, s.n_embd)
                + s.n_embd * row_bytes(s.shared_quant, s.shared_n_ff))

    # -------------------------------------------------------------- desc
    def desc(self) -> LayerDesc:
        if self._desc is not None:
            return self._desc
        s = self.spec
        d = LayerDesc()
        d.n_embd, d.n_ff, d.n_expert, d.n_used = s.n_embd, s.n_ff, s.n_expert, s.n_used
        d.quant, d.act_op, d.router_mode = s.quant, s.act_op, s.router_mode
        d.n_group, d.topk_group, d.weight_scale = s.n_group, s.topk_group, s.weight_scale
        d.row_bytes_gu, d.row_bytes_down = self.rb_gu, self.rb_down
        d.expert_stride_gu = s.n_ff * self.rb_gu
        d.expert_stride_down = s.n_embd * self.rb_down
        # slab e sits at base + e * stride: a shard's base is its first slab less slab_lo strides
        # (never dereferenced for experts outside the shard)
        d.gate = ptr(self.gate) - self.slab_lo * d.expert_stride_gu
        d.up = ptr(self.up) - self.slab_lo * d.expert_stride_gu
        d.down = ptr(self.down) - self.slab_lo * d.expert_stride_down
        d.gate_b, d.up_b, d.down_b = ptr(self.gate_b), ptr(self.up_b), ptr(self.down_b)
        d.router_w = ptr(self.router_w)
        d.router_logit_b, d.router_select_b = ptr(self.router_logit_b), ptr(self.router_select_b)
        if s.shared_quant is not None:
            d.n_shared, d.shared_quant, d.shared_n_ff = 1, s.shared_quant, s.shared_n_ff
            d.shared_row_bytes_gu = row_bytes(s.shared_quant, s.n_embd)
            d.shared_row_bytes_down = row_bytes(s.shared_quant, s.shared_n_ff)
            d.shared_gate, d.shared_up, d.shared_down = ptr(self.shared_gate), ptr(self.shared_up), ptr(self.shared_down)
            d.shared_gate_w = ptr(self.shared_gate_w)
        d.expert_lo, d.expert_hi = self.expert_lo, self.expert_hi
        if self.gate_tiles is not None:
            d.gate_tiles = ptr(self.gate_tiles) - self.slab_lo * d.expert_stride_gu
            d.up_tiles = ptr(self.up_tiles) - self.slab_lo * d.expert_stride_gu
            d.down_tiles = ptr(self.down_tiles) - self.slab_lo * d.expert_stride_down
        self._desc = d
        return d

    def build_tiles(self) -> bool:
        """Load-time repack of Q2_K routed slabs into tile planes (the device
        image the integer tensor-core passes stream; the GGUF slabs stay).
        False (nothing built) for other formats or shapes the planes do not
        cover (rows % 128, columns % 256)."""
        s = self.spec
        if s.quant != QUANT_Q2_K or s.n_ff % 256 or s.n_embd % 256:
            return False
        n = (self.expert_hi or s.n_expert) - self.slab_lo
        st = torch.cuda.current_stream().cuda_stream
        out = []
        for slab, rows, cols, rb in ((self.gate, s.n_ff, s.n_embd, self.rb_gu), (self.up, s.n_ff, s.n_embd, self.rb_gu),
                                     (self.down, s.n_embd, s.n_ff, self.rb_down)):
            t = torch.empty(n * rows * rb, dtype=torch.uint8, device=slab.device)
            check(lib().pulsar_repack_q2k_tiles(ptr(t), ptr(slab), n, rows, cols, rb, rows * rb, st),
                  "repack_q2k_tiles")
            out.append(t)
        self.gate_tiles, self.up_tiles, self.down_tiles = out
        self._desc = None
        return True

    def workspace_bytes(self, max_tok: int) -> int:
        n = int(lib().pulsar_moe_layer_workspace(ctypes.byref(self.desc()), max_tok))
        if n == 0:
            raise ValueError("layer descriptor rejected by pulsar_moe_layer_workspace")
        return n

    def forward(self, x: torch.Tensor, out: torch.Tensor, ws: torch.Tensor, residual: torch.Tensor | None = None,
                stream: torch.cuda.Stream | None = None) -> torch.Tensor:
        """out = residual + moe(x) (or moe(x)); x, out f32 [T][H] on the device."""
        T = x.shape[0]
        st = torch.cuda.current_stream() if stream is None else stream
        check(lib().pulsar_moe_layer(ctypes.byref(self.desc()), ptr(out), ptr(x), ptr(residual), T, ptr(ws),
                                     ws.numel(), st.cuda_stream), "moe_layer")
        return out

    def ep_workspace_bytes(self, world: int, max_tok: int) -> int:
        n = int(lib().pulsar_moe_layer_ep_workspace(ctypes.byref(self.desc()), world, max_tok))
        if n == 0:
            raise ValueError("layer descriptor rejected by pulsar_moe_layer_ep_workspace")
        return n

    def forward_ep(self, comm, x: torch.Tensor, out: torch.Tensor, ws: torch.Tensor,
                   residual: torch.Tensor | None = None, stream: torch.cuda.Stream | None = None) -> torch.Tensor:
        """expert-parallel layer (pulsar_moe_layer_ep): x, out, residual hold
        this rank's tokens; comm is an ep.EpComm"""
        T = x.shape[0]
        st = torch.cuda.current_stream() if stream is None else stream
        check(lib().pulsar_moe_layer_ep(ctypes.byref(self.desc()), comm.handle, comm.rank, comm.world, ptr(out),
                                        ptr(x), ptr(residual), T, ptr(ws), ws.numel(), st.cuda_stream),
              "moe_layer_ep")
        return out

    def ws_view(self, ws: torch.Tensor, n_tok: int) -> WsView:
        v = WsView()
        check(lib().pulsar_moe_layer_ws_view(ctypes.byref(self.desc()), n_tok, ptr(ws), ctypes.byref(v)), "ws_view")
        return v

    def expert_rows(self, e: int):
        """(gate, up, down) byte views of expert e (device tensors)."""
        s = self.spec
        e -= self.slab_lo
        g = self.gate[e * s.n_ff * self.rb_gu:(e + 1) * s.n_ff * self.rb_gu]
        u = self.up[e * s.n_ff * self.rb_gu:(e + 1) * s.n_ff * self.rb_gu]
        d = self.down[e * s.n_embd * self.rb_down:(e + 1) * s.n_embd * self.rb_down]
        return g, u, d


# ------------------------------------------------------------------ builders

def zipf_bias(n_expert: int, s: float, kind: str, seed: int) -> torch.Tensor:
    """Zipf(s) expert skew: a seeded permutation gives each expert a rank
    r = 1..E; selection-score bias r^-s (sigmoid routers) or logit bias
    -s ln r (softmax routers)."""
    g = torch.Generator().manual_seed(seed)
    rank = torch.randperm(n_expert, generator=g).to(torch.float64) + 1.0
    if kind == "select":
        return rank.pow(-s).to(torch.float32)
    return (-s * torch.log(rank)).to(torch.float32)


def _quantized(rows: int, n: int, quant: int, std: float, gen: torch.Generator, device, chunk_rows: int = 1 << 16,
               qw: torch.Tensor | None = None) -> torch.Tensor:
    """rows x n f32 N(0, std) generated on the device, encoded to `quant`."""
    rb = row_bytes(quant, n)
    out = torch.empty(rows * rb + SLAB_SLACK, dtype=torch.uint8, device=device)
    out[rows * rb:].zero_()
    for r0 in range(0, rows, chunk_rows):
        r1 = min(rows, r0 + chunk_rows)
        x = torch.randn((r1 - r0, n), generator=gen, device=device, dtype=torch.float32) * std
        quantize_rows(out[r0 * rb:r1 * rb], x.contiguous(), quant, qw=qw)
    return out


def q8_0_roundtrip(w: torch.Tensor) -> torch.Tensor:
    """rows of f32 -> Q8_0 blocks (GPU encoder, crates/quant q8_0) -> their f32
    dequant d * q, exact in f32: the engine stores the router as Q8_0 and
    uploads it dequantized (crates/engine/src/lib.rs:2884-2921)"""
    from ._lib import QUANT_Q8_0
    rows, n = w.shape
    rb = row_bytes(QUANT_Q8_0, n)
    q = torch.empty(rows * rb, dtype=torch.uint8, device=w.device)
    quantize_rows(q, w, QUANT_Q8_0)
    blk = q.view(rows, n // 32, 34)
    d = blk[:, :, 0:2].contiguous().view(torch.float16).to(torch.float32)
    v = blk[:, :, 2:].contiguous().view(torch.int8).to(torch.float32)
    return (d * v).reshape(rows, n).contiguous()


def _expert_slabs(spec: LayerSpec, seed: int, lo: int, hi: int, dev, order=None):
    """gate, up, down slabs of expert slots [lo, hi): slot p holds logical
    expert order[p] (identity without order), whose matrix m comes from its
    own generator stream, so a shard holds the same bytes as the full layer
    does for those experts."""
    s = spec
    qw = torch.ones(s.n_embd, device=dev) if s.quant == 1 else None
    qw_f = torch.ones(s.n_ff, device=dev) if s.quant == 1 else None
    out = []
    for m, (rows, n, q) in enumerate(((s.n_ff, s.n_embd, qw), (s.n_ff, s.n_embd, qw), (s.n_embd, s.n_ff, qw_f))):
        rb = row_bytes(s.quant, n)
        slab = torch.empty((hi - lo) * rows * rb + SLAB_SLACK, dtype=torch.uint8, device=dev)
        slab[(hi - lo) * rows * rb:].zero_()
        for e in range(lo, hi):
            le = int(order[e]) if order is not None else e
            g = torch.Generator(device=dev).manual_seed(seed * 1_000_003 + 7 * le + m)
            x = torch.randn((rows, n), generator=g, device=dev, dtype=torch.float32) * s.weight_std
            o = (e - lo) * rows * rb
            quantize_rows(slab[o:o + rows * rb], x, s.quant, qw=q)
        out.append(slab)
    return out


def make_layer(spec: LayerSpec, seed: int, device="cuda", lo: int = 0, hi: int = 0, order=None) -> MoeLayer:
    """Seeded synthetic layer: every tensor from its own generator stream.
    lo, hi (hi 0 = all): build the routed slabs of experts [lo, hi) only -
    an expert-parallel shard; the layer then computes those experts only.
    order: expert placement - slot p holds logical expert order[p] (router
    rows, biases and slabs permuted alike, so the layer computes the same
    function; ep.snake_order balances popular experts over the shards)."""
    dev = torch.device(device)
    s = spec
    hi = hi or s.n_expert

    def gen(k: int) -> torch.Generator:
        return torch.Generator(device=dev).manual_seed(seed * 1000 + k)

    gate, up, down = _expert_slabs(s, seed, lo, hi, dev, order)
    router_w = torch.randn((s.n_expert, s.n_embd), generator=gen(4), device=dev) * s.weight_std
    if s.router_q8_0:
        router_w = q8_0_roundtrip(router_w.contiguous())
    perm = None if order is None else torch.as_tensor(list(order), dtype=torch.long, device=dev)
    if perm is not None:
        router_w = router_w[perm]
    layer = MoeLayer(spec=s, gate=gate, up=up, down=down, router_w=router_w.contiguous(), slab_lo=lo)
    if (lo, hi) != (0, s.n_expert):
        layer.expert_lo, layer.expert_hi = lo, hi
    if s.zipf_s > 0:
        b = zipf_bias(s.n_expert, s.zipf_s, s.zipf_kind, seed).to(dev)
        if perm is not None:
            b = b[perm].contiguous()
        if s.zipf_kind == "select":
            layer.router_select_b = b
        else:
            layer.router_logit_b = b
    if s.biases:
        def bias(shape, k):
            t = torch.randn(shape, generator=gen(k), device=dev) * s.bias_std
            return (t if perm is None else t[perm]).contiguous()
        layer.gate_b = bias((s.n_expert, s.n_ff), 5)
        layer.up_b = bias((s.n_expert, s.n_ff), 6)
        layer.down_b = bias((s.n_expert, s.n_embd), 7)
        rb = bias((s.n_expert,), 8)
        layer.router_logit_b = rb if layer.router_logit_b is None else (layer.router_logit_b + rb).contiguous()
    if s.shared_quant is not None:
        sq = s.shared_quant
        qs = torch.ones(s.n_embd, device=dev) if sq == 1 else None
        qsf = torch.ones(s.shared_n_ff, device=dev) if sq == 1 else None
        layer.shared_gate = _quantized(s.shared_n_ff, s.n_embd, sq, s.weight_std, gen(9), dev, qw=qs)
        layer.shared_up = _quantized(s.shared_n_ff, s.n_embd, sq, s.weight_std, gen(10), dev, qw=qs)
        layer.shared_down = _quantized(s.n_embd, s.shared_n_ff, sq, s.weight_std, gen(11), dev, qw=qsf)
        if s.shared_gate:
            layer.shared_gate_w = (torch.randn((s.n_embd,), generator=gen(12), device=dev) * s.weight_std).contiguous()
    layer.build_tiles()
    return layer


def seeded_hidden(n_tok: int, n_embd: int, seed: int, device="cuda") -> torch.Tensor:
    g = torch.Generator(device=device).manual_seed(seed)
    return torch.randn((n_tok, n_embd), generator=g, device=device, dtype=torch.float32)
