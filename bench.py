"""MoE-layer tokens/s on B200: BASELINE config 2.

Workload: the shared-expert MoE stack of config 2 - 40 layers of hidden
2048, 256 routed experts (sigmoid top-8, Zipf(1.1) selection bias) plus one
always-on shared expert, expert intermediate 512, all Q4_K.  Weights are
seeded f32 N(0, 0.02) generated on the device and encoded with the GPU Q4_K
encoder (byte-identical to crates/quant quantize_row_q4_k); hidden rows are
fresh seeded N(0, 1) per step.  A step is one decode batch of T tokens
through the 40-layer stack (layer l+1 reads layer l's output: the residual
add is fused into the combine).  The stack's expert bytes read per step
(hundreds of MB to GB) exceed the 126 MB L2, so no flush is needed.

value     tokens/s with inputs resident in HBM: K replays of a captured CUDA
          graph of the step, CUDA events on the launching stream, max over ranks.
e2e       the same through the public API each step: pinned host x -> device,
          the stack, device -> pinned host of the final hidden rows.
roofline  the dominant kernel (the stream-K gate/up pass, pm_layer_sk_kernel
          <.., 2, 0>): algorithmic bytes per launch (distinct routed experts x
          gate+up bytes + shared gate+up + q8_K activations) / its CUDA-event
          duration, vs the measured HBM copy bandwidth; traffic from ncu.
cpu_baseline  the C restatement of the reference CPU expert lane (oracle/,
          all host threads) on a bounded sample of the same stack.

N > 1 (torchrun): expert parallel, weak scaling.  Each rank owns its own T
tokens and E/N experts; per layer the ranks all-gather the hidden rows,
compute their experts for every token and reduce-scatter the outputs back to
the token owners (NCCL).  --impl reference times the CPU lane alone.
"""
from __future__ import annotations

import argparse
import datetime
import faulthandler
import json
import os
import subprocess
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)
faulthandler.enable()

import numpy as np  # noqa: E402
import torch  # noqa: E402

CFG = dict(name="C2", n_embd=2048, n_ff=512, n_expert=256, n_used=8, layers=40, zipf=1.1, batches=(1, 8, 64))
METRIC = "MoE-layer tokens/s and % of HBM/tensor roofline at 1/2/4/8 B200"
# DRAM bytes (read + write) per gate/up launch over the launch's algorithmic bytes, from one
# ncu capture of this workload (profiles/pm_layer_sk_kernel_c2_b64.md: 228.4 + 13.2 MB
# against 221.2 MB); the reported traffic scales it to this run's launch.
TRAFFIC_RATIO = (228.40 + 13.16) / 221.2
TRAFFIC_NOTE = ("ncu dram__bytes_read.sum + dram__bytes_write.sum of pm_layer_sk_kernel gate/up (config 2, "
                "batch 64) / algorithmic bytes, times this run's algorithmic bytes per launch")
UNIT = "tokens/s"


def log(*a):
    print(*a, file=sys.stderr, flush=True)


class ClockSampler:
    """nvidia-smi clock / throttle samples during the timed region."""

    def __init__(self, gpu: int):
        self.gpu, self.proc, self.lines = gpu, None, []

    def __enter__(self):
        q = ("clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,clocks_event_reasons.hw_slowdown,"
             "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
             "clocks_event_reasons.sw_power_cap")
        try:
            self.proc = subprocess.Popen(["nvidia-smi", "-i", str(self.gpu), f"--query-gpu={q}",
                                          "--format=csv,noheader,nounits", "-lms", "100"],
                                         stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            threading.Thread(target=self._read, daemon=True).start()
            t0 = time.time()  # nvidia-smi takes a moment to start: wait for its first sample
            while not self.lines and time.time() - t0 < 5.0 and self.proc.poll() is None:
                time.sleep(0.02)
        except FileNotFoundError:
            self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def __exit__(self, *a):
        if self.proc:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except Exception:
                self.proc.kill()

    def summary(self):
        sm, mx, reasons = [], 0.0, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            f = [x.strip() for x in ln.split(",")]
            if len(f) < 8:
                continue
            try:
                sm.append(float(f[0]))
                mx = max(mx, float(f[1]))
            except ValueError:
                continue
            for n, v in zip(names, f[4:8]):
                if v.lower() == "active":
                    reasons.add(n)
        return {"sm_mhz": float(np.median(sm)) if sm else None, "sm_max_mhz": mx or None,
                "reasons": sorted(reasons), "samples": len(sm)}


def measured_peak_hbm():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        return float(json.load(open(p))["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


def build_stack(layers: int, lo: int, hi: int, dev):
    from pulsar_b200 import QUANT_Q4_K, LayerSpec, make_layer
    spec = LayerSpec(n_embd=CFG["n_embd"], n_ff=CFG["n_ff"], n_expert=CFG["n_expert"], n_used=CFG["n_used"],
                     quant=QUANT_Q4_K, router_mode=0, zipf_s=CFG["zipf"], zipf_kind="select",
                     shared_quant=QUANT_Q4_K, shared_n_ff=CFG["n_ff"])
    stack = []
    for l in range(layers):
        L = make_layer(spec, seed=2000 + l, device=dev)
        L.expert_lo, L.expert_hi = lo, hi
        stack.append(L)
    torch.cuda.synchronize()
    return stack


class Runner:
    """Static buffers and the captured CUDA graph of one decode step."""

    def __init__(self, stack, T: int, world: int, group=None):
        self.stack, self.T, self.world, self.group = stack, T, world, group
        H = CFG["n_embd"]
        dev = torch.device("cuda")
        self.Tg = T * world  # tokens each rank computes its experts for
        self.x = torch.zeros((T, H), dtype=torch.float32, device=dev)
        self.h = [torch.zeros((self.Tg, H), dtype=torch.float32, device=dev) for _ in range(2)]
        self.part = torch.zeros((self.Tg, H), dtype=torch.float32, device=dev)
        self.rs = torch.zeros((T, H), dtype=torch.float32, device=dev)
        self.r = [torch.zeros((T, H), dtype=torch.float32, device=dev) for _ in range(2)]
        self.ws = torch.zeros(max(L.workspace_bytes(self.Tg) for L in stack), dtype=torch.uint8, device=dev)
        self.cur = torch.zeros((T, H), dtype=torch.float32, device=dev)
        self.xn = torch.zeros((self.Tg, H), dtype=torch.float32, device=dev)
        self.graph = None
        self.stream = torch.cuda.Stream()

    def step_body(self):
        """x -> per layer: x + moe(rms_norm(x)) -> cur (this rank's rows)"""
        from pulsar_b200 import ops
        cur = self.x
        for L in self.stack:
            if self.world == 1:
                nxt = self.h[0] if cur is not self.h[0] else self.h[1]
                ops.rms_norm(self.xn, cur)
                L.forward(self.xn, nxt, self.ws, residual=cur)
                cur = nxt
            else:
                import torch.distributed as dist
                dist.all_gather_into_tensor(self.h[0], cur, group=self.group)
                ops.rms_norm(self.xn, self.h[0])
                L.forward(self.xn, self.part, self.ws)
                dist.reduce_scatter_tensor(self.rs, self.part, group=self.group)
                nxt = self.r[0] if cur is not self.r[0] else self.r[1]
                torch.add(self.rs, cur, out=nxt)
                cur = nxt
        self.cur.copy_(cur)

    def capture(self):
        with torch.cuda.stream(self.stream):
            for _ in range(2):
                self.step_body()
        torch.cuda.synchronize()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=self.stream):
            self.step_body()
        torch.cuda.synchronize()
        self.graph = g

    def run(self, x_dev):
        with torch.cuda.stream(self.stream):
            self.x.copy_(x_dev, non_blocking=True)
            self.graph.replay()


def launches_per_layer(T: int) -> int:
    """kernels one layer step launches for a layer call over T tokens (all ranks' tokens under
    expert parallelism): rms_norm, router (+ q8_K of x), selection, gate/up, down, combine, and
    when an expert can reach 192 tokens the tensor-core passes - per pass (gate/up, down) the
    token-image pack plus one expand + one gemm (the workloads here fit one expert wave) - and
    the tensor-core mid kernel"""
    return 6 + (7 if T >= 192 else 0)


def max_over_ranks(ms: float, world: int) -> float:
    if world == 1:
        return ms
    import torch.distributed as dist
    t = torch.tensor([ms], device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def barrier(world):
    if world > 1:
        import torch.distributed as dist
        dist.barrier()


def timed(runner: Runner, xs, steps: int, warmup: int, world: int):
    st = runner.stream
    for i in range(warmup):
        runner.run(xs[i % len(xs)])
    torch.cuda.synchronize()
    barrier(world)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(st)
    for i in range(steps):
        runner.run(xs[(warmup + i) % len(xs)])
    e1.record(st)
    torch.cuda.synchronize()
    return max_over_ranks(e0.elapsed_time(e1), world) / steps


def timed_e2e(runner: Runner, xs_host, steps: int, warmup: int, world: int):
    """public-API loop: pinned host x -> device -> stack -> pinned host out"""
    st = runner.stream
    out_h = torch.empty(runner.cur.shape, dtype=torch.float32).pin_memory()

    def one(i):
        with torch.cuda.stream(st):
            runner.x.copy_(xs_host[i % len(xs_host)], non_blocking=True)
            runner.graph.replay()
            out_h.copy_(runner.cur, non_blocking=True)

    for i in range(warmup):
        one(i)
    torch.cuda.synchronize()
    barrier(world)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(st)
    for i in range(steps):
        one(warmup + i)
    e1.record(st)
    torch.cuda.synchronize()
    nbytes = runner.cur.numel() * 4
    return max_over_ranks(e0.elapsed_time(e1), world) / steps, nbytes, nbytes


def profile_stages(runner: Runner, x_dev):
    """Per-kernel CUDA-event times of one eager step (events recorded by
    pulsar_moe_layer_profiled on the launching stream), and the distinct
    experts each layer touched (read from the workspace)."""
    import ctypes

    from pulsar_b200 import lib
    from pulsar_b200._lib import check, ptr
    from pulsar_b200 import ops
    st = runner.stream
    stage_ms = np.zeros(5)
    gu_bytes = layer_bytes = 0.0
    H, F = CFG["n_embd"], CFG["n_ff"]
    runner.x.copy_(x_dev)
    torch.cuda.synchronize()
    cur = runner.x
    for L in runner.stack:
        nxt = runner.h[0] if cur is not runner.h[0] else runner.h[1]
        with torch.cuda.stream(st):
            ops.rms_norm(runner.xn, cur)
        evs = [torch.cuda.Event(enable_timing=True) for _ in range(6)]
        for e in evs:
            e.record(st)  # creates the event handle
        torch.cuda.synchronize()
        arr = (ctypes.c_void_p * 6)(*[e.cuda_event for e in evs])
        check(lib().pulsar_moe_layer_profiled(ctypes.byref(L.desc()), ptr(nxt), ptr(runner.xn), ptr(cur), runner.T,
                                              ptr(runner.ws), runner.ws.numel(), st.cuda_stream, arr),
              "moe_layer_profiled")
        torch.cuda.synchronize()
        for i in range(5):
            stage_ms[i] += evs[i].elapsed_time(evs[i + 1])
        v = L.ws_view(runner.ws, runner.T)
        n_routed = int(runner.ws.view(torch.int32)[(v.n_items - runner.ws.data_ptr()) // 4 + 1].item())
        act = runner.T * ((H + 255) // 256) * 292
        gu_bytes += (n_routed + 1) * 2 * F * L.rb_gu + act
        layer_bytes += ((n_routed + 1) * L.weight_bytes_per_expert() + L.router_w.numel() * 4
                        + runner.T * H * 8)
        cur = nxt
    n = len(runner.stack)
    return stage_ms / n, gu_bytes / n, layer_bytes / n


def cpu_baseline(stack, T: int, x0: np.ndarray, threads: int, budget_s: float = 15.0):
    """The oracle lane (C restatement of the reference CPU expert lane) over
    the first layers of the same stack on all host threads, extrapolated to
    the 40-layer step.  Returns (tokens/s, layers sampled)."""
    import oracle as orc
    H, E, F, k = CFG["n_embd"], CFG["n_expert"], CFG["n_ff"], CFG["n_used"]
    t_total, done = 0.0, 0
    x = x0.astype(np.float32).copy()
    for L in stack:
        gate, up, down = (t.cpu().numpy() for t in (L.gate, L.up, L.down))
        sg, su, sd = (t.cpu().numpy() for t in (L.shared_gate, L.shared_up, L.shared_down))
        rw = L.router_w.cpu().numpy()
        sb = L.router_select_b.cpu().numpy()
        rg, rd = L.rb_gu, L.rb_down
        if not np.isfinite(x).all():
            raise RuntimeError(f"cpu baseline: non-finite hidden rows entering layer {done}")
        t0 = time.perf_counter()
        xn = (x / np.sqrt(np.mean(x.astype(np.float64) ** 2, axis=1, keepdims=True) + 1e-6)).astype(np.float32)
        lg = orc.router_logits(rw, xn)
        sel, w = orc.router_select(lg, sb, k, 1.0, 0)
        slots, ws = [], np.zeros((T, k + 1), np.float32)
        for t in range(T):
            row = []
            for s in range(k):
                e = int(sel[t, s])
                ws[t, s] = w[t, s]
                row.append(dict(gate=gate[e * F * rg:(e + 1) * F * rg], up=up[e * F * rg:(e + 1) * F * rg],
                                down=down[e * H * rd:(e + 1) * H * rd]))
            ws[t, k] = 1.0
            row.append(dict(gate=sg, up=su, down=sd))
            slots.append(row)
        out = orc.moe_ffn(xn, slots, ws, H, k, (F, 2, rg, rd), (F, 2, rg, rd), n_threads=threads)
        x = (x + out).astype(np.float32)
        t_total += time.perf_counter() - t0
        done += 1
        if t_total > budget_s:
            break
    step_s = t_total / done * CFG["layers"]
    return T / step_s, done


def measured_peak_tensor():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        return float(json.load(open(p))["bf16_tflops"]), "measured (cuBLAS bf16 burst)"
    return 1590.0, "fallback"


def prefill_c3(args):
    """C3 prefill: one layer of H 2880, 32 MXFP4 experts (softmax top-4, F 2880,
    biases, swiglu_oai) at T = 2048 tokens, one GPU.  Every expert sees
    about 256 tokens, so the routed FFN runs on the tcgen05 tiles.  The
    roofline is the tensor pipe: algorithmic FLOPs 2 T k 3 H F + 2 T E H per
    step over the step's CUDA-event time against the measured bf16 dense
    peak.  The tiles issue two fp16 MMAs per product here (weights hi x
    tokens hi + lo; the weight lo images of MXFP4 are zero, so their MMA is
    skipped), reported beside it as issued FLOPs."""
    from pulsar_b200 import lib, make_layer
    from pulsar_b200.configs import CONFIGS
    lib()
    if int(os.environ.get("WORLD_SIZE", "1")) > 1 and int(os.environ.get("RANK", "0")) != 0:
        return
    dev = torch.device("cuda", int(os.environ.get("LOCAL_RANK", "0")))
    torch.cuda.set_device(dev)
    spec = CONFIGS["C3"]["spec"]
    T, H, F, E, k = 2048, spec.n_embd, spec.n_ff, spec.n_expert, spec.n_used
    L = make_layer(spec, seed=3000, device=dev)
    ws = torch.zeros(L.workspace_bytes(T), dtype=torch.uint8, device=dev)
    g = torch.Generator(device=dev)
    xs = []
    for i in range(8):
        g.manual_seed(3_000_000 + i)
        xs.append(torch.randn((T, H), generator=g, device=dev))
    x = torch.zeros((T, H), dtype=torch.float32, device=dev)
    out = torch.zeros_like(x)
    st = torch.cuda.Stream()
    with torch.cuda.stream(st):
        for _ in range(2):
            L.forward(x, out, ws, stream=st)
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=st):
        L.forward(x, out, ws, stream=st)
    torch.cuda.synchronize()

    def one(i, host=None, out_h=None):
        with torch.cuda.stream(st):
            x.copy_(host[i % len(host)] if host is not None else xs[i % len(xs)], non_blocking=True)
            graph.replay()
            if out_h is not None:
                out_h.copy_(out, non_blocking=True)

    def time_loop(**kw):
        for i in range(args.warmup):
            one(i, **kw)
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(st)
        for i in range(args.steps):
            one(args.warmup + i, **kw)
        e1.record(st)
        torch.cuda.synchronize()
        return e0.elapsed_time(e1) / args.steps

    with ClockSampler(dev.index) as clk:
        ms = time_loop()
    host = [t.cpu().pin_memory() for t in xs]
    out_h = torch.empty((T, H), dtype=torch.float32).pin_memory()
    e2e_ms = time_loop(host=host, out_h=out_h)
    v = L.ws_view(ws, T)
    n = ws.view(torch.int32)[(v.n_items - ws.data_ptr()) // 4:(v.n_items - ws.data_ptr()) // 4 + 6].cpu().tolist()
    flops = 2.0 * T * k * 3 * H * F + 2.0 * T * E * H
    issued = 2 * 2.0 * T * k * 3 * H * F  # wh xh + wh xl: MXFP4 weights are exact in fp16 (zero lo images)
    peak, peak_kind = measured_peak_tensor()
    ach = flops / (ms / 1e3) / 1e12
    cfg = {"workload": "C3 prefill, one layer (BASELINE configs[2] shapes)", "n_embd": H, "n_ff": F,
           "n_expert": E, "n_used": k, "quant": "MXFP4", "router": "softmax top-4, router + expert biases",
           "act": "swiglu_oai", "tokens": T, "parallelism": "single",
           "l2": "32 experts x 13.2 MB = 423 MB of weights per step exceed the 126 MB L2 (no flush)"}
    print(json.dumps({
        "metric": METRIC, "value": T / (ms / 1e3), "unit": UNIT, "n_gpus": 1, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": "fp16 hi+lo split operands (tcgen05 kind::f16), f32 accumulate", "data": "synthetic (seeded)",
        "config": cfg,
        "e2e": {"value": T / (e2e_ms / 1e3), "unit": UNIT, "h2d_bytes_per_step": T * H * 4,
                "d2h_bytes_per_step": T * H * 4},
        "gpu_launches": (launches_per_layer(T) - 1) * args.steps, "clocks": clk.summary(),
        "roofline": {"bound": "tensor", "achieved": ach, "peak": peak, "unit": "TFLOP/s", "frac": ach / peak,
                     "peak_kind": peak_kind, "traffic": None, "algorithmic_flops_per_step": flops,
                     "issued_mma_flops_per_step": issued, "issued_tflops": issued / (ms / 1e3) / 1e12,
                     "scope": "whole layer step (router, selection, tensor-core tiles, mid, combine)"},
        "tc_tiles": n[4], "tc_splits": n[5], "cpu_baseline": None}), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--batch", type=int, default=64, help="decode batch per rank of the headline value")
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--layers", type=int, default=CFG["layers"])
    ap.add_argument("--no-cpu", action="store_true", help="skip the CPU baseline leg")
    ap.add_argument("--no-profile", action="store_true", help="skip the per-kernel roofline leg")
    ap.add_argument("--all-batches", action="store_true", help="also time decode batches 1 and 8")
    ap.add_argument("--workload", default="c2-decode", choices=["c2-decode", "c3-prefill"],
                    help="c3-prefill: one C3 layer at T 2048 on the tensor-core path (a secondary line)")
    args = ap.parse_args()
    if args.workload == "c3-prefill":
        return prefill_c3(args)
    CFG["layers"] = args.layers
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    T = args.batch
    config = {"workload": "C2 shared-expert MoE stack, decode (BASELINE configs[1])", "layers": CFG["layers"],
              "n_embd": CFG["n_embd"], "n_expert": CFG["n_expert"], "n_used": CFG["n_used"], "n_shared": 1,
              "n_ff": CFG["n_ff"], "quant": "Q4_K", "router": "sigmoid top-8, Zipf(1.1) selection bias",
              "batch_per_rank": T, "global_batch": T * world,
              "parallelism": f"ep{world}" if world > 1 else "single",
              "l2": "per-step expert bytes exceed the 126 MB L2 (no flush)"}

    if args.impl == "reference":
        if rank != 0:
            return
        import oracle as orc
        orc.build()
        if not torch.cuda.is_available():
            print(json.dumps({"impl": "reference", "unavailable": "the seeded weights are built on the GPU box"}))
            return
        dev = torch.device("cuda", local)
        torch.cuda.set_device(dev)
        threads = os.cpu_count() or 1
        stack = build_stack(min(CFG["layers"], 4), 0, 0, dev)
        vals, nl = [], 0
        for i in range(args.warmup + args.steps):
            x0 = np.random.default_rng(10_000 + i).normal(0, 1, (T, CFG["n_embd"])).astype(np.float32)
            v, nl = cpu_baseline(stack, T, x0, threads, budget_s=2.0)
            if i >= args.warmup:
                vals.append(v)
        val = float(np.mean(vals))
        print(json.dumps({
            "impl": "reference", "metric": METRIC, "value": val, "unit": UNIT, "higher_is_better": True,
            "n_gpus": world, "steps": args.steps, "warmup": args.warmup, "ms_per_step": T / val * 1e3,
            "dtype": "int8 dots, f32", "data": "synthetic (seeded)", "config": config, "scaling": "weak",
            "vs_baseline": None,
            "cpu_baseline": {"value": val, "unit": UNIT, "cores": threads, "kind": "port",
                             "sample": f"oracle CPU lane on {nl} of {CFG['layers']} layers per step, extrapolated"},
            "e2e": {"value": val, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}))
        return

    import pulsar_b200
    pulsar_b200.lib()
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    group = None
    if world > 1:
        import torch.distributed as dist
        dist.init_process_group("nccl", device_id=dev, timeout=datetime.timedelta(seconds=300))
        group = dist.group.WORLD
    E = CFG["n_expert"]
    lo, hi = (rank * E // world, (rank + 1) * E // world) if world > 1 else (0, 0)
    t0 = time.time()
    stack = build_stack(CFG["layers"], lo, hi, dev)
    log(f"[rank {rank}] built {CFG['layers']} layers in {time.time() - t0:.1f}s "
        f"({sum(L.gate.numel() + L.up.numel() + L.down.numel() for L in stack) / 1e9:.1f} GB)")

    def inputs(Tb, n):
        g = torch.Generator(device=dev)
        xs = []
        for i in range(n):
            g.manual_seed(1_000_000 * (rank + 1) + 7919 * Tb + i)
            xs.append(torch.randn((Tb, CFG["n_embd"]), generator=g, device=dev))
        return xs

    results, head = {}, None
    batches = sorted(set([T] + (list(CFG["batches"]) if args.all_batches else [])))
    for Tb in batches:
        runner = Runner(stack, Tb, world, group)
        runner.capture()
        xs = inputs(Tb, min(args.steps + args.warmup, 32))
        with ClockSampler(local) as clk:
            ms = timed(runner, xs, args.steps, args.warmup, world)
        clocks = clk.summary()
        xs_host = [x.cpu().pin_memory() for x in xs]
        e2e_ms, h2d, d2h = timed_e2e(runner, xs_host, args.steps, args.warmup, world)
        tok = Tb * world
        results[Tb] = {"tokens_per_s": tok / (ms / 1e3), "ms_per_step": ms,
                       "e2e_tokens_per_s": tok / (e2e_ms / 1e3), "e2e_ms_per_step": e2e_ms}
        if Tb == T:
            head = (runner, xs, ms, e2e_ms, h2d, d2h, clocks)
        log(f"[rank {rank}] T={Tb}: {ms:.3f} ms/step, {tok / (ms / 1e3):.0f} tok/s, e2e {e2e_ms:.3f} ms")

    runner, xs, ms, e2e_ms, h2d, d2h, clocks = head
    line = None
    if rank == 0:
        roof = None
        if world == 1 and not args.no_profile:
            peak, peak_kind = measured_peak_hbm()
            st_ms, gu_bytes, layer_bytes = profile_stages(runner, xs[0])
            gu_ms = float(st_ms[3])
            ach = gu_bytes / (gu_ms / 1e3) / 1e9
            layer_ms = float(st_ms.sum())
            roof = {"bound": "hbm", "kernel": "pm_layer_sk_kernel gate/up (dp4a stream-K: gate + up + glu -> mid)",
                    "achieved": ach, "peak": peak, "unit": "GB/s", "frac": ach / peak, "peak_kind": peak_kind,
                    "traffic": TRAFFIC_RATIO * gu_bytes, "traffic_note": TRAFFIC_NOTE,
                    "algorithmic_bytes_per_launch": gu_bytes, "launch_ms": gu_ms,
                    "stage_ms": dict(zip(["router_logits+q8k_x", "(fused)", "select_csr", "gate_up", "down_combine"],
                                         map(float, st_ms))),
                    "layer": {"algorithmic_bytes": layer_bytes, "eager_ms": layer_ms,
                              "eager_gbs": layer_bytes / (layer_ms / 1e3) / 1e9,
                              "graph_ms": ms / CFG["layers"],
                              "graph_gbs": layer_bytes / (ms / CFG["layers"] / 1e3) / 1e9,
                              "graph_frac": layer_bytes / (ms / CFG["layers"] / 1e3) / 1e9 / peak}}
            log(f"[rank 0] roofline {json.dumps(roof)}")
        cpu = None
        if world == 1 and not args.no_cpu:
            import oracle as orc
            orc.build()
            threads = os.cpu_count() or 1
            v, nl = cpu_baseline(stack, T, xs[0].cpu().numpy(), threads)
            cpu = {"value": v, "unit": UNIT, "cores": threads, "kind": "port",
                   "sample": f"oracle CPU lane (C restatement of crates/engine cpu_tier::Lane) on {nl} of "
                             f"{CFG['layers']} layers, batch {T}, extrapolated to the 40-layer step"}
        tok = T * world
        line = {"metric": METRIC, "value": tok / (ms / 1e3), "unit": UNIT, "n_gpus": world, "steps": args.steps,
                "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True, "scaling": "weak",
                "vs_baseline": None, "dtype": "int8 dp4a dots, f32 accumulate", "data": "synthetic (seeded)",
                "config": config,
                "e2e": {"value": tok / (e2e_ms / 1e3), "unit": UNIT, "h2d_bytes_per_step": h2d,
                        "d2h_bytes_per_step": d2h},
                "gpu_launches": launches_per_layer(T * world) * CFG["layers"] * args.steps, "clocks": clocks, "roofline": roof,
                "cpu_baseline": cpu, "per_batch": {str(k): v for k, v in results.items()}}
    if line is not None:
        print(json.dumps(line), flush=True)
    if world > 1:
        # Skip destroy_process_group: tearing down NCCL communicators that live
        # CUDA graphs still reference can block indefinitely.  All device work is
        # complete here; every rank leaves after one bounded barrier.
        import torch.distributed as dist
        torch.cuda.synchronize()
        threading.Timer(60.0, os._exit, args=(0,)).start()  # bound the barrier below
        try:
            dist.barrier(device_ids=[local])
            torch.cuda.synchronize()
        finally:
            sys.stdout.flush()
            sys.stderr.flush()
            os._exit(0)


if __name__ == "__main__":
    main()
