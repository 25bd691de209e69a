"""MoE-layer tokens/s on B200 for the BASELINE configurations.

Default workload (--workload c4-decode): BASELINE configs[3], the largest
configuration that fits one GPU - a stack of 94 MoE layers of hidden 4096,
128 routed experts (softmax top-8, Zipf(1.2) logit bias), expert
intermediate 1536, Q2_K experts (74.5 GB), router weights Q8_0 used as their
exact f32 dequant.  Weights are seeded f32 N(0, 0.02) generated on the
device and encoded with the GPU block encoders (byte-identical to
crates/quant); hidden rows are fresh seeded N(0, 1) per step.  A step is one
decode batch of T tokens through the whole stack (layer l+1 reads layer l's
output: x + moe(rms_norm(x)), the residual add fused into the layer's
combine).  The stack's expert bytes read per step exceed the 126 MB L2, so
no flush is needed.  Decode batches 1, 32 and 256; the headline is T = 256
(the routed experts then run on the tcgen05 integer tensor cores).

Other workloads: c2-decode (configs[1], 40 layers, T 1/8/64), c1-decode
(configs[0]: one layer, T = 1, four weight copies rotated so L2 cannot hold
them), c3-prefill (configs[2], one layer at T = 2048 on the tensor cores).

value     tokens/s with inputs resident in HBM: K replays of a captured CUDA
          graph of the step, CUDA events on the launching stream, max over ranks.
e2e       the same through the public API each step: pinned host x -> device,
          the stack, device -> pinned host of the final hidden rows.
roofline  the dominant kernel, the gate/up pass (pm_tci8_kernel<Q2_K, 2> on
          the integer tensor cores when the batch has >= 1 routed token per expert
          on average, else the stream-K dp4a pm_layer_sk_kernel<.., 2, 0>):
          algorithmic bytes per launch (distinct routed experts x gate+up
          bytes + shared gate+up + q8_K activations) / its CUDA-event duration
          on the launching stream, vs the measured HBM copy bandwidth.
cpu_baseline  the C restatement of the reference CPU expert lane (oracle/,
          all host threads) on a bounded sample of the same workload.

N > 1 (torchrun): expert parallel, weak scaling, through the library's
pulsar_moe_layer_ep.  Each rank owns its own T tokens and E/N expert slots
(experts placed in snake order over their Zipf popularity); per layer every
rank routes its own tokens, the q8_K rows / ids / weights are all-gathered,
each rank runs its experts for every token that chose them (and the shared
expert for its own tokens), and the sums are reduce-scattered back to the
token owners - NCCL collectives on the layer's stream, inside the graph.

--impl reference times the reference's CPU expert lane (the oracle port)
alone, on rank 0, with weights built by the oracle's own encoders.
"""
from __future__ import annotations

import argparse
import datetime
import faulthandler
import json
import os
import platform
import subprocess
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)
faulthandler.enable()

import numpy as np  # noqa: E402
import torch  # noqa: E402

METRIC = "MoE-layer tokens/s and % of HBM/tensor roofline at 1/2/4/8 B200"
UNIT = "tokens/s"
WORKLOADS = {
    "c4-decode": dict(cfg="C4", layers=94, batches=(1, 32, 256), batch=256, copies=1,
                      label="C4 Q2_K expert stack, decode (BASELINE configs[3])"),
    "c2-decode": dict(cfg="C2", layers=40, batches=(1, 8, 64), batch=64, copies=1,
                      label="C2 shared-expert MoE stack, decode (BASELINE configs[1])"),
    "c1-decode": dict(cfg="C1", layers=1, batches=(1,), batch=1, copies=4,
                      label="C1 single MoE layer, decode T=1 (BASELINE configs[0])"),
}
# DRAM bytes (read + write) per gate/up launch over the launch's algorithmic bytes, from one
# ncu capture per workload (committed summaries under profiles/); the reported traffic scales
# it to this run's launch.  None where no capture of that workload exists.
TRAFFIC_RATIO = {"c2-decode": (228.40 + 13.16) / 221.2, "c4-decode": (387.09 + 16.27) / 398.9}


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


def measured_peak(key: str, fallback: float):
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        return float(json.load(open(p))[key]), "measured"
    return fallback, "fallback"


def cpu_info():
    model = platform.processor() or ""
    try:
        for ln in open("/proc/cpuinfo"):
            if ln.startswith("model name"):
                model = ln.split(":", 1)[1].strip()
                break
    except OSError:
        pass
    n = os.cpu_count() or 1
    return model, n


def spec_of(wl: dict):
    from pulsar_b200.configs import CONFIGS
    return CONFIGS[wl["cfg"]]["spec"]


def config_dict(wl: dict, spec, T: int, world: int):
    q = {0: "Q2_K", 1: "IQ2_XXS", 2: "Q4_K", 10: "Q8_0", 12: "MXFP4"}
    router = ("sigmoid" if spec.router_mode == 0 else "softmax") + f" top-{spec.n_used}"
    if spec.zipf_s:
        router += f", Zipf({spec.zipf_s}) {'selection' if spec.zipf_kind == 'select' else 'logit'} bias"
    if spec.router_q8_0:
        router += ", router weights Q8_0 (exact f32 dequant)"
    c = {"workload": wl["label"], "layers": wl["layers"], "n_embd": spec.n_embd, "n_expert": spec.n_expert,
         "n_used": spec.n_used, "n_shared": 1 if spec.shared_quant is not None else 0, "n_ff": spec.n_ff,
         "quant": q[spec.quant], "router": router, "batch_per_rank": T, "global_batch": T * world,
         "parallelism": f"ep{world}" if world > 1 else "single",
         "l2": "per-step expert bytes exceed the 126 MB L2 (no flush)"}
    if wl["copies"] > 1:
        c["l2"] = (f"{wl['copies']} weight copies of the layer rotated step by step "
                   f"({wl['copies']} x the layer's bytes > 4 x the 126 MB L2; no flush)")
    return c


def build_stack(wl: dict, world: int, rank: int, dev):
    """the workload's layers on this rank: all experts at N = 1; under
    expert parallelism only this rank's expert slots, with the experts
    placed in snake order over their Zipf popularity"""
    from pulsar_b200 import make_layer
    from pulsar_b200.ep import shard, snake_order, zipf_popularity
    spec = spec_of(wl)
    stack = []
    n = wl["layers"] * wl["copies"]
    for l in range(n):
        seed = 2000 + l
        if world == 1:
            L = make_layer(spec, seed=seed, device=dev)
        else:
            lo, hi = shard(spec.n_expert, world, rank)
            order = snake_order(zipf_popularity(spec.n_expert, spec.zipf_s or 1.0, seed), world)
            L = make_layer(spec, seed=seed, device=dev, lo=lo, hi=hi, order=order)
        stack.append(L)
    torch.cuda.synchronize()
    return stack


class Runner:
    """Static buffers and the captured CUDA graph of one step.  A step runs
    `per_step` passes of T tokens; each pass is x + moe(rms_norm(x)) through
    `layers` consecutive layers of the stack (copies > 1: pass i uses weight
    copy i, so one replay is `copies` decode steps on different weights)."""

    def __init__(self, stack, wl, T: int, world: int, comm=None):
        self.stack, self.wl, self.T, self.world, self.comm = stack, wl, T, world, comm
        self.copies = wl["copies"]
        H = stack[0].spec.n_embd
        dev = torch.device("cuda")
        self.x = torch.zeros((self.copies, T, H), dtype=torch.float32, device=dev)
        self.h = [torch.zeros((T, H), dtype=torch.float32, device=dev) for _ in range(2)]
        nbytes = max((L.workspace_bytes(T) if world == 1 else L.ep_workspace_bytes(world, T)) for L in stack)
        self.ws = torch.zeros(nbytes, dtype=torch.uint8, device=dev)
        self.cur = torch.zeros((self.copies, T, H), dtype=torch.float32, device=dev)
        self.xn = torch.zeros((T, H), dtype=torch.float32, device=dev)
        self.graph = None
        self.stream = torch.cuda.Stream()

    def step_body(self):
        from pulsar_b200 import ops
        nl = self.wl["layers"]
        for c in range(self.copies):
            cur = self.x[c]
            for L in self.stack[c * nl:(c + 1) * nl]:
                nxt = self.h[0] if cur is not self.h[0] else self.h[1]
                ops.rms_norm(self.xn, cur)
                if self.world == 1:
                    L.forward(self.xn, nxt, self.ws, residual=cur)
                else:  # pulsar_moe_layer_ep: route own tokens, NCCL dispatch / combine inside the call
                    L.forward_ep(self.comm, self.xn, nxt, self.ws, residual=cur)
                cur = nxt
            self.cur[c].copy_(cur)

    def capture(self, x_dev):
        """warm-up passes on real hidden states (a zero input would route every
        token to the same experts), then the graph capture"""
        with torch.cuda.stream(self.stream):
            self.x.copy_(x_dev)
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


def i8_on(spec, T: int, world: int = 1) -> bool:
    """routed Q2_K experts on the integer tensor-core passes (the library's rule: at least one
    routed token per expert on average, over every rank's tokens)"""
    return spec.quant == 0 and T * world * spec.n_used >= spec.n_expert


def launches_per_layer(T: int, world: int = 1, tc_fmt: bool = True, i8: bool = False) -> int:
    """this library's kernels one layer step launches for a layer call over T tokens per rank:
    rms_norm, router (+ q8_K of x), selection (two launches under expert parallelism: top-k, then
    the CSR after the dispatch), the dp4a gate/up and down passes, combine; with the integer
    tensor-core passes on, their gate/up, mid q8_K and down kernels; otherwise, when an expert
    can reach 192 tokens (counted over every rank's tokens), the fp16 tensor-core passes - per
    pass (gate/up, down) the token-image pack plus one expand + one gemm (these workloads fit one
    expert wave) - and the tensor-core mid kernel.  NCCL's own kernels are not counted."""
    n = 6 + (1 if world > 1 else 0)
    if i8:
        return n + 3
    return n + (7 if T * world >= 192 and tc_fmt else 0)


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

    from pulsar_b200 import lib, ops, row_bytes
    from pulsar_b200._lib import check, ptr
    st = runner.stream
    stage_ms = np.zeros(5)
    gu_bytes = layer_bytes = 0.0
    spec = runner.stack[0].spec
    H, F = spec.n_embd, spec.n_ff
    runner.x.copy_(x_dev)
    torch.cuda.synchronize()
    n_calls, tiles = 0, 0
    for c in range(runner.copies):
        cur = runner.x[c]
        nl = runner.wl["layers"]
        for L in runner.stack[c * nl:(c + 1) * nl]:
            nxt = runner.h[0] if cur is not runner.h[0] else runner.h[1]
            with torch.cuda.stream(st):
                ops.rms_norm(runner.xn, cur)
            evs = [torch.cuda.Event(enable_timing=True) for _ in range(6)]
            for e in evs:
                e.record(st)  # creates the event handle
            torch.cuda.synchronize()
            arr = (ctypes.c_void_p * 6)(*[e.cuda_event for e in evs])
            check(lib().pulsar_moe_layer_profiled(ctypes.byref(L.desc()), ptr(nxt), ptr(runner.xn), ptr(cur),
                                                  runner.T, ptr(runner.ws), runner.ws.numel(), st.cuda_stream, arr),
                  "moe_layer_profiled")
            torch.cuda.synchronize()
            for i in range(5):
                stage_ms[i] += evs[i].elapsed_time(evs[i + 1])
            v = L.ws_view(runner.ws, runner.T)
            base = (v.n_items - runner.ws.data_ptr()) // 4
            n = runner.ws.view(torch.int32)[base:base + 6].cpu().tolist()
            n_routed, tiles = int(n[1]), tiles + int(n[4])
            ns = 1 if spec.shared_quant is not None else 0
            act = runner.T * ((H + 255) // 256) * 292
            sh_gu = 2 * spec.shared_n_ff * row_bytes(spec.shared_quant, H) if ns else 0
            gu_bytes += n_routed * 2 * F * L.rb_gu + sh_gu + act
            layer_bytes += (n_routed * L.weight_bytes_per_expert() + L.shared_bytes() + L.router_w.numel() * 4
                            + runner.T * H * 8)
            cur = nxt
            n_calls += 1
    return stage_ms / n_calls, gu_bytes / n_calls, layer_bytes / n_calls, tiles / n_calls


# ---------------------------------------------------------------- CPU lane

class RefStack:
    """The workload's stack for the CPU lane, built with the oracle's own
    encoders (no product code): `distinct` expert weight sets encoded on the
    host and tiled over the E expert slots of one layer (the lane reads each
    slot from its own address, as it would distinct experts: the slab is far
    larger than any CPU cache), and per layer its own router weights and
    Zipf bias, so routing differs layer by layer.  Layer l of the stack uses
    the shared slab with router l."""

    def __init__(self, wl: dict, n_router_layers: int, distinct: int = 8, seed: int = 90_000):
        import oracle as orc
        spec = spec_of(wl)
        self.spec = spec
        s = spec
        H, F, E = s.n_embd, s.n_ff, s.n_expert
        rng = np.random.default_rng(seed)
        q = s.quant
        qw = np.ones(H, np.float32) if q == 1 else None
        qwf = np.ones(F, np.float32) if q == 1 else None
        self.rb_gu, self.rb_dn = orc.row_bytes(q, H), orc.row_bytes(q, F)
        from concurrent.futures import ThreadPoolExecutor

        def enc(rows, n, qq, ww):
            x = rng.normal(0, s.weight_std, (rows, n)).astype(np.float32)
            parts = np.array_split(np.arange(rows), min(rows, os.cpu_count() or 1))
            with ThreadPoolExecutor(len(parts)) as ex:  # the oracle encoders release the GIL (ctypes)
                out = list(ex.map(lambda ix: orc.quantize(qq, x[ix[0]:ix[-1] + 1], ww), parts))
            return np.concatenate(out, axis=0).reshape(-1)
        d = min(distinct, E)
        g = [enc(F, H, q, qw) for _ in range(d)]
        u = [enc(F, H, q, qw) for _ in range(d)]
        dn = [enc(H, F, q, qwf) for _ in range(d)]
        self.gate = np.stack([g[e % d] for e in range(E)])
        self.up = np.stack([u[e % d] for e in range(E)])
        self.down = np.stack([dn[e % d] for e in range(E)])
        self.shared = None
        if s.shared_quant is not None:
            sq, Fs = s.shared_quant, s.shared_n_ff
            self.shared = dict(quant=sq, F=Fs, rb_gu=orc.row_bytes(sq, H), rb_dn=orc.row_bytes(sq, Fs),
                               gate=enc(Fs, H, sq, None), up=enc(Fs, H, sq, None), down=enc(H, Fs, sq, None))
        self.routers = []
        for l in range(n_router_layers):
            w = rng.normal(0, s.weight_std, (E, H)).astype(np.float32)
            if s.router_q8_0:
                w = np.stack([orc.dequant(10, r, H) for r in orc.quantize(10, w)])
            lb = sb = None
            if s.zipf_s:
                rank = rng.permutation(E).astype(np.float64) + 1.0
                if s.zipf_kind == "select":
                    sb = (rank ** -s.zipf_s).astype(np.float32)
                else:
                    lb = (-s.zipf_s * np.log(rank)).astype(np.float32)
            self.routers.append((w, lb, sb))

    def layer(self, l, x, threads):
        """x + moe(rms_norm(x)) through layer l on the CPU lane"""
        import oracle as orc
        s = self.spec
        H, k = s.n_embd, s.n_used
        w_r, lb, sb = self.routers[l % len(self.routers)]
        xn = (x / np.sqrt(np.mean(x.astype(np.float64) ** 2, axis=1, keepdims=True) + 1e-6)).astype(np.float32)
        lg = orc.router_logits(w_r, xn, lb)
        sel, w = orc.router_select(lg, sb, k, s.weight_scale, s.router_mode, n_group=s.n_group,
                                   topk_group=s.topk_group)
        T = x.shape[0]
        ns = 1 if self.shared is not None else 0
        slots, ws = [], np.zeros((T, k + ns), np.float32)
        for t in range(T):
            row = []
            for j in range(k):
                e = int(sel[t, j])
                ws[t, j] = w[t, j]
                row.append(dict(gate=self.gate[e], up=self.up[e], down=self.down[e]))
            if ns:
                ws[t, k] = 1.0
                row.append(dict(gate=self.shared["gate"], up=self.shared["up"], down=self.shared["down"]))
            slots.append(row)
        sh = None
        if ns:
            sh = (self.shared["F"], self.shared["quant"], self.shared["rb_gu"], self.shared["rb_dn"])
        out = orc.moe_ffn(xn, slots, ws, H, k, (s.n_ff, s.quant, self.rb_gu, self.rb_dn), sh, act_op=s.act_op,
                          n_threads=threads)
        return (x + out).astype(np.float32)


def cpu_lane_sample(ref: RefStack, wl: dict, T: int, x0: np.ndarray, threads: int, budget_s: float):
    """Run the CPU lane through consecutive layers of the stack until the
    budget is spent (at least one layer).  Returns (seconds, layers run)."""
    x = x0.astype(np.float32).copy()
    t0 = time.perf_counter()
    nl = 0
    while True:
        x = ref.layer(nl, x, threads)
        nl += 1
        if nl >= wl["layers"] * wl["copies"] or time.perf_counter() - t0 >= budget_s:
            break
    return time.perf_counter() - t0, nl


def reference_arm(args, wl, T, world, rank):
    """--impl reference: the reference's CPU expert lane (the oracle port of
    crates/engine cpu_tier::Lane) on all host threads, rank 0 only.  A step is
    a bounded sample: T tokens through as many consecutive layers of the
    stack as fit the per-step budget; value = tokens/s of the whole stack
    (T / (per-layer time x layers)), ms_per_step = the sample's measured time."""
    if rank != 0:
        return
    import oracle as orc
    orc.build()
    spec = spec_of(wl)
    model, ncpu = cpu_info()
    threads = ncpu
    t0 = time.time()
    ref = RefStack(wl, n_router_layers=8)
    log(f"[reference] oracle-encoded stack in {time.time() - t0:.1f}s")
    n_layers = wl["layers"] * wl["copies"]
    per_tok_layer, samples, layers_run = [], [], []
    rng = np.random.default_rng(10_000)
    budget = float(os.environ.get("PULSAR_REF_STEP_S", "3.0"))
    for i in range(args.warmup + args.steps):
        x0 = rng.normal(0, 1, (T, spec.n_embd)).astype(np.float32)
        sec, nl = cpu_lane_sample(ref, wl, T, x0, threads, budget if i >= args.warmup else 0.0)
        if i >= args.warmup:
            samples.append(sec)
            layers_run.append(nl)
            per_tok_layer.append(sec / nl)
    layer_s = float(np.sum(samples) / np.sum(layers_run))
    val = T * wl["copies"] / (layer_s * n_layers)
    ms = float(np.mean(samples)) * 1e3
    nl_mean = float(np.mean(layers_run))
    print(json.dumps({
        "impl": "reference", "metric": METRIC, "value": val, "unit": UNIT, "higher_is_better": True,
        "n_gpus": world, "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms,
        "dtype": "int8 dots, f32", "data": "synthetic (seeded)", "config": config_dict(wl, spec, T, 1),
        "scaling": "weak", "vs_baseline": None,
        "cpu_baseline": {"value": val, "unit": UNIT, "cores": threads, "kind": "port", "cpu": model,
                         "sample": f"each step: {T} tokens through {nl_mean:.1f} of the {n_layers} layers "
                                   f"(measured {ms:.0f} ms); value = T / (per-layer time x {n_layers})"},
        "e2e": {"value": val, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}), flush=True)


def cpu_baseline_leg(wl, T, x0, budget_s=15.0):
    """cpu_baseline of the GPU line: the same CPU lane as the reference arm,
    at the reference default thread count (cores / 2 - 2, crates/engine/src/
    lib.rs:1893-1896) and on all host threads."""
    model, ncpu = cpu_info()
    ref = RefStack(wl, n_router_layers=8)
    n_layers = wl["layers"] * wl["copies"]
    res = {}
    for threads in sorted({max(1, ncpu // 2 - 2), ncpu}):
        sec, nl = cpu_lane_sample(ref, wl, T, x0, threads, budget_s / 2)
        res[threads] = T * wl["copies"] / (sec / nl * n_layers)
    best = max(res, key=res.get)
    return {"value": res[best], "unit": UNIT, "cores": best, "kind": "port", "cpu": model,
            "by_threads": {str(k): v for k, v in res.items()},
            "sample": f"oracle CPU lane (C restatement of crates/engine cpu_tier::Lane), batch {T}, "
                      f"oracle-encoded weights, consecutive layers for ~{budget_s / 2:.0f} s per thread "
                      f"count, per-layer time x {n_layers} layers"}


# ------------------------------------------------------------- C3 prefill

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
    peak, peak_kind = measured_peak("bf16_tflops", 1590.0)
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
                     "peak_kind": peak_kind + " (cuBLAS bf16 burst)", "traffic": None,
                     "algorithmic_flops_per_step": flops,
                     "issued_mma_flops_per_step": issued, "issued_tflops": issued / (ms / 1e3) / 1e12,
                     "scope": "whole layer step (router, selection, tensor-core tiles, mid, combine)"},
        "tc_tiles": n[4], "tc_splits": n[5], "cpu_baseline": None}), flush=True)


# -------------------------------------------------------------------- main

def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--workload", default="c4-decode", choices=sorted(WORKLOADS) + ["c3-prefill"])
    ap.add_argument("--batch", type=int, default=0, help="decode batch per rank of the headline value "
                                                         "(0 = the workload's default)")
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--layers", type=int, default=0, help="override the stack depth (diagnostics only)")
    ap.add_argument("--no-cpu", action="store_true", help="skip the CPU baseline leg")
    ap.add_argument("--no-profile", action="store_true", help="skip the per-kernel roofline leg")
    ap.add_argument("--all-batches", action="store_true", help="also time the workload's other decode batches")
    ap.add_argument("--path-flags", type=int, default=0, help="layer descriptor path_flags (diagnostics only: "
                    "1 keeps routed Q2_K off the integer tensor cores, 2 forces them on)")
    args = ap.parse_args()
    if args.workload == "c3-prefill":
        return prefill_c3(args)
    wl = dict(WORKLOADS[args.workload])
    if args.layers:
        wl["layers"] = args.layers
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    T = args.batch or wl["batch"]
    spec = spec_of(wl)
    config = config_dict(wl, spec, T, world)

    if args.impl == "reference":
        return reference_arm(args, wl, T, world, rank)

    import pulsar_b200
    pulsar_b200.lib()
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    comm = None
    if world > 1:
        import torch.distributed as dist

        from pulsar_b200.ep import EpComm
        dist.init_process_group("nccl", device_id=dev, timeout=datetime.timedelta(seconds=300))
        comm = EpComm(rank, world, device=dev)
    H = spec.n_embd
    t0 = time.time()
    stack = build_stack(wl, world, rank, dev)
    for L in stack:
        L.desc().path_flags = args.path_flags
    log(f"[rank {rank}] built {len(stack)} layers in {time.time() - t0:.1f}s "
        f"({sum(L.gate.numel() + L.up.numel() + L.down.numel() for L in stack) / 1e9:.1f} GB)")

    def inputs(Tb, n):
        g = torch.Generator(device=dev)
        xs = []
        for i in range(n):
            g.manual_seed(1_000_000 * (rank + 1) + 7919 * Tb + i)
            xs.append(torch.randn((wl["copies"], Tb, H), generator=g, device=dev))
        return xs

    results, head = {}, None
    batches = sorted(set([T] + (list(wl["batches"]) if args.all_batches else [])))
    tok_per_step = lambda Tb: Tb * world * wl["copies"]  # noqa: E731
    for Tb in batches:
        runner = Runner(stack, wl, Tb, world, comm)
        xs = inputs(Tb, min(args.steps + args.warmup, 16))
        runner.capture(xs[0])
        with ClockSampler(local) as clk:
            ms = timed(runner, xs, args.steps, args.warmup, world)
        clocks = clk.summary()
        xs_host = [x.cpu().pin_memory() for x in xs]
        e2e_ms, h2d, d2h = timed_e2e(runner, xs_host, args.steps, args.warmup, world)
        tok = tok_per_step(Tb)
        results[Tb] = {"tokens_per_s": tok / (ms / 1e3), "ms_per_step": ms,
                       "e2e_tokens_per_s": tok / (e2e_ms / 1e3), "e2e_ms_per_step": e2e_ms}
        if Tb == T:
            head = (runner, xs, ms, e2e_ms, h2d, d2h, clocks)
        else:
            del runner
        log(f"[rank {rank}] T={Tb}: {ms:.3f} ms/step, {tok / (ms / 1e3):.0f} tok/s, e2e {e2e_ms:.3f} ms")

    runner, xs, ms, e2e_ms, h2d, d2h, clocks = head
    line = None
    if rank == 0:
        roof = None
        n_layer_calls = wl["layers"] * wl["copies"]
        if world == 1 and not args.no_profile:
            peak, peak_kind = measured_peak("hbm_gbs", 6650.0)
            st_ms, gu_bytes, layer_bytes, tiles = profile_stages(runner, xs[0])
            gu_ms = float(st_ms[3])
            ach = gu_bytes / (gu_ms / 1e3) / 1e9
            layer_ms = float(st_ms.sum())
            graph_layer_ms = ms / n_layer_calls
            ratio = TRAFFIC_RATIO.get(args.workload)
            i8 = i8_on(spec, T)
            kname = ("pm_tci8_kernel<Q2_K, 2> gate/up (tcgen05 kind::i8, glu -> mid)" if i8 else
                     "pm_layer_sk_kernel gate/up (dp4a stream-K: gate + up + glu -> mid)")
            roof = {"bound": "hbm", "kernel": kname,
                    "achieved": ach, "peak": peak, "unit": "GB/s", "frac": ach / peak,
                    "peak_kind": peak_kind + " (STREAM-style copy)",
                    "traffic": ratio * gu_bytes if ratio else None,
                    "traffic_note": ("ncu dram__bytes_read.sum + dram__bytes_write.sum of the gate/up launch over "
                                     "its algorithmic bytes, times this run's algorithmic bytes per launch")
                    if ratio else "no ncu capture of this workload",
                    "algorithmic_bytes_per_launch": gu_bytes, "launch_ms": gu_ms, "tc_tiles_per_layer": tiles,
                    "stage_ms": dict(zip(["router_logits+q8k_x", "(fused)", "select_csr", "gate_up",
                                          "down_combine"], map(float, st_ms))),
                    "layer": {"algorithmic_bytes": layer_bytes, "eager_ms": layer_ms,
                              "eager_gbs": layer_bytes / (layer_ms / 1e3) / 1e9,
                              "graph_ms": graph_layer_ms,
                              "graph_gbs": layer_bytes / (graph_layer_ms / 1e3) / 1e9,
                              "graph_frac": layer_bytes / (graph_layer_ms / 1e3) / 1e9 / peak}}
            log(f"[rank 0] roofline {json.dumps(roof)}")
        cpu = None
        if world == 1 and not args.no_cpu:
            import oracle as orc
            orc.build()
            cpu = cpu_baseline_leg(wl, T, xs[0][0].cpu().numpy())
        tok = tok_per_step(T)
        if world > 1:
            config["placement"] = "experts in snake order over Zipf popularity, E/N contiguous slots per rank"
        line = {"metric": METRIC, "value": tok / (ms / 1e3), "unit": UNIT, "n_gpus": world, "steps": args.steps,
                "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True, "scaling": "weak",
                "vs_baseline": None, "dtype": ("int8 x int8 -> s32 on tcgen05 kind::i8, f32 terms" if i8_on(spec, T, world)
                                                    else "int8 dp4a dots, f32 accumulate"), "data": "synthetic (seeded)",
                "config": config,
                "e2e": {"value": tok / (e2e_ms / 1e3), "unit": UNIT, "h2d_bytes_per_step": h2d,
                        "d2h_bytes_per_step": d2h},
                "gpu_launches": launches_per_layer(T, world, i8=i8_on(spec, T, world)) * n_layer_calls * args.steps, "clocks": clocks,
                "roofline": roof, "cpu_baseline": cpu, "per_batch": {str(k): v for k, v in results.items()}}
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
