#!/usr/bin/env python
"""Benchmark of the B200-native tensor-parallel linear path.

Metric: fused TP GEMM + all-reduce microseconds per layer,
decode shapes of config 2 (hidden 4096, intermediate 12288, 32 q / 8 kv heads,
head_dim 128: qkv 4096->6144, o 4096->4096, gate_up 4096->24576,
down 12288->4096, no bias, bf16), tokens per step 1/8/32/128/256, TP = the
number of GPUs. Synthetic data: weights ~N(0, 0.02), activations ~N(0, 1),
seed 0, random-init weights (no checkpoint exists here).

One step = the linear path of L distinct decoder layers in the order of
LlamaDecoderLayer.forward (models/llama.py:77-86), built from this repo's
public layer classes: qkv_proj (column GEMM) -> o_proj fused with the
all-reduce and post_attention_layernorm -> gate_up_proj (column GEMM) on that
norm's output -> down_proj fused with the all-reduce and the next layer's
input_layernorm. With one GPU there is no all-reduce, and each row-parallel
layer runs as the column GEMM followed by the fused_add_rmsnorm kernel
(`config.row_path`). Attention and silu_and_mul are outside the step; their
outputs are fixed synthetic activations. The gated MLP's front half
(gate_up_proj + silu_and_mul, fused by pgb_gate_up_silu) is timed beside the
step under `config.mlp_front_us`, and the attention block's front (qkv_proj +
RoPE + KV-cache store, fused by pgb_qkv_rope_store) under
`config.attn_front_us`. On one GPU, `config.full_layer_us` times the whole decoder layer
minus the attention itself (all four fused kernels through the public API) against the
reference's own unfused calls on the same weights. L is chosen so the step's weights
exceed 3x the 126 MB L2, so every layer streams its weights from HBM (no L2
flush is needed). The step is captured once in a CUDA graph (as the
reference's decode graphs, engine/graph.py:100-142) and replayed.

Headline `value`: microseconds per layer at T = 256 (lower is better), the
batch of the end-to-end config. Every decode T is reported under
`config.per_tokens`.

    python bench.py [--gpus N --steps K --warmup W] [--impl reference]
"""

from __future__ import annotations

import argparse
import importlib
import json
import math
import os
import statistics
import subprocess
import sys
import time
from pathlib import Path

import torch

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

H, I, NQ, NKV, HD = 4096, 12288, 32, 8, 128
QKV = (NQ + 2 * NKV) * HD  # 6144
EPS = 1e-6
TOKENS = (1, 8, 32, 128, 256)
HEADLINE_T = 256
L2_BYTES = 126 * 2**20
GATE_UP_T256_TP1_DRAM_BYTES = 207_560_960  # 203.54 MB read + 4.02 MB written (ncu, one launch)


def load_peaks() -> dict:
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return {"hbm_gbs": d["hbm_gbs"], "bf16_tflops": d["bf16_tflops"], "src": "measured"}
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "src": "fallback"}


NVLINK_GBS = 770.0  # measured peer copy per direction on this pool


# ---------------------------------------------------------------- roofline --


def op_costs(T: int, n: int) -> dict:
    """Algorithmic HBM bytes, FLOPs and NVLink bytes per GPU for each op.

    Column GEMM: HBM 2(N_l K + T K + T N_l), FLOPs 2 T K N_l.
    Row fused: HBM 2(N K_l + T K_l + T N) + 2(2 T N) + 2 N (weights, x, out,
    residual read + write, norm weight); NVLink 2(n-1)/n T N 2 bytes per
    direction (P2P reduce-scatter + all-gather formula).
    """
    def col(K, N):
        return {"hbm": 2.0 * (N * K + T * K + T * N), "flops": 2.0 * T * K * N, "nvl": 0.0}

    def row(K, N):
        return {"hbm": 2.0 * (N * K + T * K + T * N) + 2.0 * 2 * T * N + 2.0 * N,
                "flops": 2.0 * T * K * N,
                "nvl": (2.0 * (n - 1) / n * T * N * 2) if n > 1 else 0.0}

    return {"qkv": col(H, QKV // n), "o": row(H // n, H), "gate_up": col(H, 2 * I // n),
            "down": row(I // n, H)}


def roofline_us(T: int, n: int, peaks: dict) -> float:
    tot = 0.0
    for c in op_costs(T, n).values():
        tot += max(c["hbm"] / (peaks["hbm_gbs"] * 1e9), c["flops"] / (peaks["bf16_tflops"] * 1e12),
                   c["nvl"] / (NVLINK_GBS * 1e9))
    return tot * 1e6


# ------------------------------------------------------------------ clocks --


class ClockSampler:
    """nvidia-smi clocks and throttle reasons sampled during the timed region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, device_index: int):
        self.idx = device_index
        self.proc = None
        self.lines: list[str] = []

    def start(self):
        import tempfile

        self._f = tempfile.NamedTemporaryFile("w+", suffix=".csv", delete=False)
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.idx), f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "100"], stdout=self._f, stderr=subprocess.DEVNULL, text=True)
            time.sleep(0.3)  # first sample before the timed region
        except (OSError, FileNotFoundError):
            self.proc = None

    def stop(self) -> dict:
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        self._f.flush()
        self._f.close()
        with open(self._f.name) as fh:
            self.lines = [ln.strip() for ln in fh if ln.strip()]
        os.unlink(self._f.name)
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            parts = [p.strip() for p in ln.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                mx = float(parts[2])
            except ValueError:
                continue
            for nm, v in zip(names, parts[5:9]):
                if v.lower().startswith("active"):
                    reasons.add(nm)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": mx,
                "reasons": sorted(reasons), "samples": len(sm)}


# ------------------------------------------------------------- our arm ----


class Step:
    """L decoder layers of the linear path, built from the public layer classes."""

    def __init__(self, pgb_layers, T: int, n: int, rank: int, layers: list, dev):
        self.L = pgb_layers
        self.layers = layers
        g = torch.Generator(device=dev).manual_seed(1000 + T * 8 + rank)
        self.h = torch.randn(T, H, device=dev, generator=g).bfloat16()
        self.a = torch.randn(T, H // n, device=dev, generator=g).bfloat16()
        self.m = torch.randn(T, I // n, device=dev, generator=g).bfloat16()
        self.res0 = torch.randn(T, H, device=dev, generator=g).bfloat16()
        self.residual = self.res0.clone()
        self.out = None

    def run(self):
        L = self.L
        L.reset_fusion_context()
        L._CTX.residual = self.residual  # as returned by the first input_layernorm
        h = self.h
        for lay in self.layers:
            lay["qkv"].forward(h)
            x1 = lay["o"].forward(self.a)
            x1, _ = lay["ln1"].forward(x1, self.residual)
            lay["gate_up"].forward(x1)
            x2 = lay["down"].forward(self.m)
            x2, _ = lay["ln2"].forward(x2, self.residual)
            h = x2
        self.out = h
        return h


def build_layers(pgb_layers, n: int, rank: int, n_layers: int, dev):
    L = pgb_layers
    layers = []
    for li in range(n_layers):
        g = torch.Generator(device=dev).manual_seed(li * 131 + rank)

        def w(rows, cols):
            return (torch.randn(rows, cols, device=dev, generator=g) * 0.02).bfloat16()

        qkv = L.LinearColParallelPartitioned(H, HD, [(NQ, False), (NKV, True), (NKV, True)], has_bias=False)
        qkv.weight = w(*qkv.weight.shape)
        o = L.LinearRowParallel(NQ * HD, H, has_bias=False)
        o.weight = w(*o.weight.shape)
        gu = L.LinearColParallelMerged(H, [I, I], has_bias=False)
        gu.weight = w(*gu.weight.shape)
        down = L.LinearRowParallel(I, H, has_bias=False)
        down.weight = w(*down.weight.shape)
        ln1 = L.RMSNormFused(H, EPS)
        ln1.weight = torch.ones(H, device=dev).bfloat16()
        ln2 = L.RMSNormFused(H, EPS)
        ln2.weight = torch.ones(H, device=dev).bfloat16()
        o.link_norm(ln1)
        down.link_norm(ln2)
        layers.append({"qkv": qkv, "o": o, "gate_up": gu, "down": down, "ln1": ln1, "ln2": ln2})
    return layers


def time_graph(graph, stream, steps, warmup, barrier):
    for _ in range(warmup):
        graph.replay()
    torch.cuda.synchronize()
    barrier()
    torch.cuda.synchronize()
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(steps):
        graph.replay()
    e1.record(stream)
    torch.cuda.synchronize()
    barrier()
    torch.cuda.synchronize()
    return e0.elapsed_time(e1)  # ms


def capture(fn, stream):
    fn()  # eager warm-up: allocates workspaces outside capture
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.stream(stream):
        with torch.cuda.graph(g, stream=stream):
            fn()
    torch.cuda.synchronize()
    return g


def run_ours(args) -> dict | None:
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    n = world
    if args.gpus != world:
        raise SystemExit(f"--gpus {args.gpus} but WORLD_SIZE={world}")
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    import torch.distributed as dist

    if world > 1:
        dist.init_process_group("gloo", rank=rank, world_size=world)
        barrier = dist.barrier
    else:
        barrier = lambda: None  # noqa: E731

    pgb = importlib.import_module("pico-sglang_b200")
    D = importlib.import_module("pico-sglang_b200.distributed")
    L = importlib.import_module("pico-sglang_b200.layers")
    D.set_tp_info(D.DistributedInfo(rank, world))
    if world > 1:
        D.enable_pgb_distributed(D.get_tp_info(), dist.group.WORLD, 64 << 20)
    else:
        D.local_comm(64 << 20)

    peaks = load_peaks()
    bytes_per_layer = 2.0 * (QKV * H + H * H + 2 * I * H + H * I) / n
    n_layers = args.layers or max(1, math.ceil(3 * L2_BYTES / bytes_per_layer))
    layers = build_layers(L, n, rank, n_layers, dev)
    stream = torch.cuda.Stream(dev)

    per_t = {}
    graphs = {}
    steps_obj = {}
    for T in args.tokens:
        st = Step(L, T, n, rank, layers, dev)
        with torch.cuda.stream(stream):
            g = capture(st.run, stream)
        graphs[T] = g
        steps_obj[T] = st
        clocks = ClockSampler(local) if T == HEADLINE_T else None
        if clocks:
            clocks.start()
        with torch.cuda.stream(stream):
            ms = time_graph(g, stream, args.steps, args.warmup, barrier)
        ck = clocks.stop() if clocks else None
        ms_t = torch.tensor([ms])
        if world > 1:
            dist.all_reduce(ms_t, op=dist.ReduceOp.MAX)
        us_layer = ms_t.item() * 1000.0 / args.steps / n_layers
        roof = roofline_us(T, n, peaks)
        per_t[T] = {"us_per_layer": round(us_layer, 3), "tok_per_s_per_layer": round(T / (us_layer * 1e-6), 1),
                    "roofline_us": round(roof, 3), "frac_of_roofline": round(roof / us_layer, 4)}
        if ck:
            per_t[T]["clocks"] = ck

    # Dominant kernel: gate_up column GEMM (52% of a layer's weight bytes), at
    # the headline T, one launch per layer (distinct weights), CUDA events.
    T = HEADLINE_T if HEADLINE_T in args.tokens else args.tokens[-1]
    st = steps_obj[T]
    x1 = torch.randn(T, H, device=dev).bfloat16()

    def gate_up_only():
        for lay in layers:
            lay["gate_up"].forward(x1)

    with torch.cuda.stream(stream):
        g_gu = capture(gate_up_only, stream)
        ms_gu = time_graph(g_gu, stream, args.steps, args.warmup, barrier)
    gu_us = ms_gu * 1000.0 / args.steps / n_layers
    gu_bytes = op_costs(T, n)["gate_up"]["hbm"]
    achieved = gu_bytes / (gu_us * 1e-6) / 1e9

    # Per-op breakdown at the headline T (each op alone over the L layers).
    breakdown = {}
    res = st.residual

    def only(name):
        def f():
            L.reset_fusion_context()
            for lay in layers:
                if name == "qkv":
                    lay["qkv"].forward(st.h)
                elif name == "o":
                    L._CTX.residual = res
                    lay["o"].forward(st.a)
                elif name == "down":
                    L._CTX.residual = res
                    lay["down"].forward(st.m)
        return f

    for name in ("qkv", "o", "down"):
        with torch.cuda.stream(stream):
            gg = capture(only(name), stream)
            ms_op = time_graph(gg, stream, args.steps, args.warmup, barrier)
        breakdown[name] = round(ms_op * 1000.0 / args.steps / n_layers, 3)
        del gg
    breakdown["gate_up"] = round(gu_us, 3)
    mlp_front = mlp_front_timings(args, pgb, layers, x1, stream, barrier, n_layers) if args.extras else None
    attn_front = (attn_front_timings(args, pgb, L, layers, st.h, stream, barrier, n_layers, n, dev)
                  if args.extras else None)

    # End to end through the public API: pinned host inputs copied in, the
    # captured layer stack replayed, the output and residual copied out.
    hbuf = {k: torch.empty_like(v, device="cpu").pin_memory() for k, v in
            (("h", st.h), ("a", st.a), ("m", st.m), ("r", st.res0))}
    for k, v in (("h", st.h), ("a", st.a), ("m", st.m), ("r", st.res0)):
        hbuf[k].copy_(v)
    out_h = torch.empty((T, H), dtype=torch.bfloat16).pin_memory()
    res_h = torch.empty((T, H), dtype=torch.bfloat16).pin_memory()
    g = graphs[T]
    h2d = sum(t.numel() * t.element_size() for t in hbuf.values())
    d2h = out_h.numel() * 2 + res_h.numel() * 2

    def e2e_step():
        st.h.copy_(hbuf["h"], non_blocking=True)
        st.a.copy_(hbuf["a"], non_blocking=True)
        st.m.copy_(hbuf["m"], non_blocking=True)
        st.residual.copy_(hbuf["r"], non_blocking=True)
        g.replay()
        out_h.copy_(st.out, non_blocking=True)
        res_h.copy_(st.residual, non_blocking=True)

    with torch.cuda.stream(stream):
        for _ in range(args.warmup):
            e2e_step()
        torch.cuda.synchronize()
        barrier()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(args.steps):
            e2e_step()
        e1.record(stream)
        torch.cuda.synchronize()
        barrier()
    ms_e = torch.tensor([e0.elapsed_time(e1)])
    if world > 1:
        dist.all_reduce(ms_e, op=dist.ReduceOp.MAX)
    e2e_us = ms_e.item() * 1000.0 / args.steps / n_layers

    lib = library_path_baseline(args, n, rank, world, dev, stream, barrier, T) if args.library_baseline else None
    lib_small = None
    if args.library_baseline and 1 in args.tokens and T != 1:
        lib_small = library_path_baseline(args, n, rank, world, dev, stream, barrier, 1)
    full = None
    if world == 1 and args.extras:
        full = {str(t): full_layer_timings(args, pgb, L, layers, dev, stream, barrier, n_layers, t)
                for t in sorted({1, T} & set(args.tokens) | {T})}

    result = None
    if rank == 0:
        head = per_t[T]
        cpu = cpu_baseline(T) if (world == 1 and not args.no_cpu_baseline) else None
        # One rank: o_proj and down_proj each run as the column GEMM + the norm
        # kernel (pgb_comm_set_one_rank_path); more ranks: one fused kernel each.
        launches = (4 if world > 1 else 6) * n_layers * args.steps
        result = {
            "metric": "fused TP GEMM+allreduce+RMSNorm us/layer (decode, config 2)",
            "value": head["us_per_layer"],
            "unit": "us/layer",
            "n_gpus": n,
            "steps": args.steps,
            "warmup": args.warmup,
            "ms_per_step": round(head["us_per_layer"] * n_layers / 1000.0, 5),
            "higher_is_better": False,
            "scaling": "strong",
            "vs_baseline": None,
            "dtype": "bf16",
            "data": "synthetic (random-init weights ~N(0,0.02), activations ~N(0,1), seed 0)",
            "config": {
                "workload": f"config 2 decode layer, T={T} tokens, TP={n}",
                "hidden": H, "intermediate": I, "q_heads": NQ, "kv_heads": NKV, "head_dim": HD,
                "tokens": T, "tp": n, "layers_per_step": n_layers,
                "row_path": ("fused GEMM + all-reduce + residual-add + RMSNorm kernel" if n > 1 else
                             "one rank: column GEMM then the fused_add_rmsnorm kernel (no all-reduce)"),
                "l2": f"inputs larger than L2: {n_layers} distinct layers, "
                      f"{bytes_per_layer * n_layers / 2**20:.0f} MiB of weights per GPU per step",
                "graph": "step captured in one CUDA graph and replayed",
                "per_tokens": {str(k): v for k, v in per_t.items()},
                "op_breakdown_us": breakdown,
                "mlp_front_us": mlp_front,
                "attn_front_us": attn_front,
                "layer_roofline_us": head["roofline_us"],
                "layer_frac_of_roofline": head["frac_of_roofline"],
            },
            "tok_per_s_per_layer": head["tok_per_s_per_layer"],
            "roofline": {
                "kernel": "col_gemm_kernel (gate_up_proj, swap-AB tcgen05)",
                "bound": "hbm",
                "achieved": round(achieved, 1),
                "peak": peaks["hbm_gbs"],
                "unit": "GB/s",
                "frac": round(achieved / peaks["hbm_gbs"], 4),
                "peak_src": peaks["src"] + " (burst copy bandwidth)",
                # DRAM read + write bytes of one gate_up launch at T=256, TP=1, from the
                # ncu capture summarised in profiles/col_gemm_gate_up_T256.md.
                "traffic": GATE_UP_T256_TP1_DRAM_BYTES if (n == 1 and T == 256) else None,
                "algorithmic_bytes_per_launch": gu_bytes,
                "avg_launch_us": round(gu_us, 3),
            },
            "e2e": {"value": round(e2e_us, 3), "unit": "us/layer", "h2d_bytes_per_step": h2d,
                    "d2h_bytes_per_step": d2h,
                    "how": "pinned H2D of the step inputs + graph replay of the public-layer stack + D2H of "
                           "output and residual, per step; divided by layers per step"},
            "gpu_launches": launches,
            "clocks": per_t[T].get("clocks"),
        }
        if cpu:
            result["cpu_baseline"] = cpu
        if lib:
            result["library_baseline"] = lib
        if lib_small:
            result["library_baseline_T1"] = lib_small
        if full:
            result["config"]["full_layer_us"] = full
    if world > 1:
        D.destroy_distributed()
        dist.destroy_process_group()
    return result


def mlp_front_timings(args, pgb, layers, x1, stream, barrier, n_layers) -> dict:
    """The gated MLP's front half, gate_up_proj then silu_and_mul
    (python/picosgl/layers/mlp.py:43-46), per layer at the headline T, three ways:
    the fused kernel, this library's GEMM then its standalone activation, and
    the reference's own calls (F.linear + flashinfer.silu_and_mul). Each is
    captured over the L distinct layers and replayed like the step."""
    import torch.nn.functional as F

    ways = {
        "fused_gate_up_silu": lambda lay: pgb.gate_up_silu(x1, lay["gate_up"].weight),
        "col_gemm_then_silu_and_mul": lambda lay: pgb.silu_and_mul(pgb.col_gemm(x1, lay["gate_up"].weight)),
    }
    if args.library_baseline:
        try:
            import flashinfer

            ways["F.linear_then_flashinfer_silu_and_mul"] = (
                lambda lay: flashinfer.silu_and_mul(F.linear(x1, lay["gate_up"].weight)))
        except Exception:  # pragma: no cover - flashinfer missing
            pass
    out = {"tokens": int(x1.shape[0])}
    for name, fn in ways.items():
        def f(fn=fn):
            for lay in layers:
                fn(lay)

        with torch.cuda.stream(stream):
            gg = capture(f, stream)
            ms = time_graph(gg, stream, args.steps, args.warmup, barrier)
        ms_t = torch.tensor([ms])
        if dist_is_initialized():
            torch.distributed.all_reduce(ms_t, op=torch.distributed.ReduceOp.MAX)
        out[name] = round(ms_t.item() * 1000.0 / args.steps / n_layers, 3)
        del gg
    return out


def attn_front_timings(args, pgb, L, layers, h, stream, barrier, n_layers, n, dev) -> dict:
    """The attention block's front, qkv_proj + RoPE + KV-cache store
    (RotaryAttention.proj, python/picosgl/layers/attention.py:94-117, then
    store_kv), per layer at the headline T, three ways: the fused kernel, this
    library's GEMM then its standalone RoPE + store, and the reference's calls
    (F.linear + flashinfer.apply_rope_with_cos_sin_cache_inplace + an index
    store). Positions are random below 4096 (RoPE theta 1e6, config 5); each
    layer writes its own [4096, kv heads, 128] caches at random slots."""
    import torch.nn.functional as F

    T = h.shape[0]
    nq, nkv = NQ // n, max(NKV // n, 1)
    table = L.get_rope(HD, HD, 4096, 1e6, None).cache_on(dev)
    g = torch.Generator(device=dev).manual_seed(11)
    pos = torch.randint(0, 4096, (T,), generator=g, device=dev, dtype=torch.int32)
    loc = torch.randperm(4096, generator=g, device=dev)[:T].to(torch.int32)
    caches = [(torch.zeros(4096, nkv, HD, device=dev, dtype=torch.bfloat16),
               torch.zeros(4096, nkv, HD, device=dev, dtype=torch.bfloat16)) for _ in layers]

    def fused(lay, kc, vc):
        pgb.ops.qkv_rope_store(h, lay["qkv"].weight, pos, loc, table, nq, nkv, HD, kc, vc)

    def unfused(lay, kc, vc):
        pgb.ops.rope_store(pgb.col_gemm(h, lay["qkv"].weight), pos, loc, table, nq, nkv, HD, kc, vc)

    ways = {"fused_qkv_rope_store": fused, "col_gemm_then_rope_store": unfused}
    if args.library_baseline:
        try:
            import flashinfer

            rope = flashinfer.apply_rope_with_cos_sin_cache_inplace
            loc64 = loc.long()

            def library(lay, kc, vc):
                # The split views go to flashinfer strided, as RotaryEmbedding.forward
                # reshapes them without a copy (python/picosgl/layers/rotary.py:40-45).
                qkv = F.linear(h, lay["qkv"].weight)
                q, k, v = qkv.split([nq * HD, nkv * HD, nkv * HD], dim=-1)
                rope(pos, q, k, HD, table, is_neox=True)
                kc[loc64] = k.view(T, nkv, HD)
                vc[loc64] = v.view(T, nkv, HD)

            ways["F.linear_flashinfer_rope_index_store"] = library
        except Exception:  # pragma: no cover - flashinfer missing
            pass
    out = {"tokens": int(T), "q_heads": nq, "kv_heads": nkv}
    for name, fn in ways.items():
        def f(fn=fn):
            for lay, (kc, vc) in zip(layers, caches):
                fn(lay, kc, vc)

        with torch.cuda.stream(stream):
            gg = capture(f, stream)
            ms = time_graph(gg, stream, args.steps, args.warmup, barrier)
        ms_t = torch.tensor([ms])
        if dist_is_initialized():
            torch.distributed.all_reduce(ms_t, op=torch.distributed.ReduceOp.MAX)
        out[name] = round(ms_t.item() * 1000.0 / args.steps / n_layers, 3)
        del gg
    return out


def full_layer_timings(args, pgb, L, layers, dev, stream, barrier, n_layers, T) -> dict:
    """A decoder layer without the attention itself, one GPU, per layer, two ways on the same
    weights. This library's public API: qkv_rope_store (qkv_proj + RoPE + KV store), o_proj
    linked to post_attention_layernorm (GEMM + residual add + RMSNorm in one kernel),
    gate_up_silu, down_proj linked to the next input_layernorm. The reference's own calls
    (python/picosgl/layers/attention.py:94-123, mlp.py:43-48, norm.py:73-75): F.linear, the
    FlashInfer RoPE on the strided split, an index store into the cache, F.linear +
    fused_add_rmsnorm, F.linear + silu_and_mul, F.linear + fused_add_rmsnorm. The attention
    output is a fixed synthetic [T, H] tensor in both."""
    import torch.nn.functional as F

    g = torch.Generator(device=dev).manual_seed(21 + T)
    h = torch.randn(T, H, device=dev, generator=g).bfloat16()
    a = torch.randn(T, H, device=dev, generator=g).bfloat16()
    res = torch.randn(T, H, device=dev, generator=g).bfloat16()
    table = L.get_rope(HD, HD, 4096, 1e6, None).cache_on(dev)
    pos = torch.randint(0, 4096, (T,), generator=g, device=dev, dtype=torch.int32)
    loc = torch.randperm(4096, generator=g, device=dev)[:T].to(torch.int32)
    loc64 = loc.long()
    caches = [(torch.zeros(4096, NKV, HD, device=dev, dtype=torch.bfloat16),
               torch.zeros(4096, NKV, HD, device=dev, dtype=torch.bfloat16)) for _ in layers]

    def ours():
        L.reset_fusion_context()
        L._CTX.residual = res
        x = h
        for lay, (kc, vc) in zip(layers, caches):
            pgb.ops.qkv_rope_store(x, lay["qkv"].weight, pos, loc, table, NQ, NKV, HD, kc, vc)
            x1 = lay["o"].forward(a)
            x1, _ = lay["ln1"].forward(x1, res)
            m = pgb.gate_up_silu(x1, lay["gate_up"].weight)
            x2 = lay["down"].forward(m)
            x, _ = lay["ln2"].forward(x2, res)

    ways = {"ours": ours}
    try:
        import flashinfer

        ln = torch.ones(H, device=dev).bfloat16()

        def library():
            x = h
            for lay, (kc, vc) in zip(layers, caches):
                qkv = F.linear(x, lay["qkv"].weight)
                q, k, v = qkv.split([NQ * HD, NKV * HD, NKV * HD], dim=-1)
                flashinfer.apply_rope_with_cos_sin_cache_inplace(pos, q, k, HD, table, is_neox=True)
                kc[loc64] = k.view(T, NKV, HD)
                vc[loc64] = v.view(T, NKV, HD)
                y = F.linear(a, lay["o"].weight)
                flashinfer.fused_add_rmsnorm(y, res, ln, EPS)
                m = flashinfer.silu_and_mul(F.linear(y, lay["gate_up"].weight))
                x = F.linear(m, lay["down"].weight)
                flashinfer.fused_add_rmsnorm(x, res, ln, EPS)

        if args.library_baseline:
            ways["library"] = library
    except Exception:  # pragma: no cover - flashinfer missing
        pass
    out = {"tokens": int(T)}
    for name, fn in ways.items():
        with torch.cuda.stream(stream):
            gg = capture(fn, stream)
            ms = time_graph(gg, stream, args.steps, args.warmup, barrier)
        out[name] = round(ms * 1000.0 / args.steps / n_layers, 3)
        del gg
    return out


def dist_is_initialized() -> bool:
    return torch.distributed.is_available() and torch.distributed.is_initialized()


def library_path_baseline(args, n, rank, world, dev, stream, barrier, T) -> dict:
    """The reference's own unfused calls on the same box: F.linear (cuBLAS),
    torch.distributed NCCL all_reduce for TP > 1 (stand-in for pynccl), and
    flashinfer.fused_add_rmsnorm, captured in a CUDA graph."""
    try:
        import flashinfer

        fa = flashinfer.fused_add_rmsnorm
        kind = "flashinfer.fused_add_rmsnorm"
    except Exception:  # pragma: no cover - flashinfer missing
        fa = None
        kind = "torch restatement of fused_add_rmsnorm"
    import torch.distributed as dist
    import torch.nn.functional as F

    grp = None
    if world > 1:
        grp = dist.new_group(backend="nccl")
    bytes_per_layer = 2.0 * (QKV * H + H * H + 2 * I * H + H * I) / n
    n_layers = args.layers or max(1, math.ceil(3 * L2_BYTES / bytes_per_layer))
    g = torch.Generator(device=dev).manual_seed(7 + rank)

    def w(r, c):
        return (torch.randn(r, c, device=dev, generator=g) * 0.02).bfloat16()

    layers = [{"qkv": w(QKV // n, H), "o": w(H, H // n), "gu": w(2 * I // n, H), "down": w(H, I // n)}
              for _ in range(n_layers)]
    ln = torch.ones(H, device=dev).bfloat16()
    h = torch.randn(T, H, device=dev, generator=g).bfloat16()
    a = torch.randn(T, H // n, device=dev, generator=g).bfloat16()
    m = torch.randn(T, I // n, device=dev, generator=g).bfloat16()
    res = torch.randn(T, H, device=dev, generator=g).bfloat16()

    def addnorm(x, r):
        if fa is not None:
            fa(x, r, ln, EPS)
        else:
            s = x.float() + r.float()
            r.copy_(s.bfloat16())
            x.copy_((s * torch.rsqrt(s.pow(2).mean(-1, keepdim=True) + EPS) * ln.float()).bfloat16())
        return x

    def step():
        x = h
        for lay in layers:
            F.linear(x, lay["qkv"])
            y = F.linear(a, lay["o"])
            if grp is not None:
                dist.all_reduce(y, group=grp)
            x1 = addnorm(y, res)
            F.linear(x1, lay["gu"])
            y2 = F.linear(m, lay["down"])
            if grp is not None:
                dist.all_reduce(y2, group=grp)
            x = addnorm(y2, res)

    with torch.cuda.stream(stream):
        gr = capture(step, stream)
        ms = time_graph(gr, stream, args.steps, args.warmup, barrier)
    ms_t = torch.tensor([ms])
    if world > 1:
        dist.all_reduce(ms_t, op=dist.ReduceOp.MAX)
    del gr
    if grp is not None:
        dist.destroy_process_group(grp)
    return {"us_per_layer": round(ms_t.item() * 1000.0 / args.steps / n_layers, 3), "tokens": T,
            "path": f"F.linear (cuBLAS) + {'torch NCCL all_reduce (pynccl stand-in) + ' if n > 1 else ''}{kind}",
            "graph": True}


# ----------------------------------------------------------- CPU baseline --


def _cpu_sample(T: int, budget_s: float):
    """The CPU oracle (numpy restatement of the reference path) on one layer
    of the bench config at TP=1, f32 BLAS accumulation, repeated until the
    time budget is spent. Returns (us per layer, reps, threads)."""
    import numpy as np

    import oracle

    rng = np.random.default_rng(0)
    f32 = np.float32
    wts = {
        "qkv": (rng.standard_normal((QKV, H), dtype=f32) * 0.02),
        "o": (rng.standard_normal((H, H), dtype=f32) * 0.02),
        "gate_up": (rng.standard_normal((2 * I, H), dtype=f32) * 0.02),
        "down": (rng.standard_normal((H, I), dtype=f32) * 0.02),
        "ln1": np.ones(H, f32),
        "ln2": np.ones(H, f32),
    }
    wts = {k: oracle.round_to(v, "bf16") for k, v in wts.items()}
    h = oracle.round_to(rng.standard_normal((T, H), dtype=f32), "bf16")
    a = oracle.round_to(rng.standard_normal((T, H), dtype=f32), "bf16")
    m = oracle.round_to(rng.standard_normal((T, I), dtype=f32), "bf16")
    r = oracle.round_to(rng.standard_normal((T, H), dtype=f32), "bf16")
    oracle.tp_layer_step(h, a, m, r, wts, EPS, n=1, dtype="bf16", accum="f32")  # warm
    reps, t0 = 0, time.perf_counter()
    while True:
        oracle.tp_layer_step(h, a, m, r, wts, EPS, n=1, dtype="bf16", accum="f32")
        reps += 1
        el = time.perf_counter() - t0
        if el >= budget_s or reps >= 50:
            break
    try:
        from threadpoolctl import threadpool_info

        threads = max((i.get("num_threads", 1) for i in threadpool_info()), default=os.cpu_count())
    except Exception:
        threads = os.cpu_count()
    return el / reps * 1e6, reps, threads


def cpu_baseline(T: int, budget_s: float = 10.0) -> dict:
    us, reps, threads = _cpu_sample(T, budget_s)
    return {"value": round(us, 1), "unit": "us/layer", "cores": threads, "kind": "port",
            "sample": f"{reps} passes of one config-2 layer at T={T}, TP=1 on the host "
                      f"(numpy oracle, f32 BLAS), {os.cpu_count()} host cores visible"}


def run_reference(args) -> dict | None:
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return None
    T = HEADLINE_T if HEADLINE_T in args.tokens else args.tokens[-1]
    vals = []
    threads = None
    reps_tot = 0
    for _ in range(args.warmup):
        _cpu_sample(T, 0.0)
    for _ in range(args.steps):
        us, reps, threads = _cpu_sample(T, 2.0)
        vals.append(us)
        reps_tot += reps
    us = statistics.median(vals)
    return {
        "impl": "reference",
        "metric": "fused TP GEMM+allreduce+RMSNorm us/layer (decode, config 2)",
        "value": round(us, 1),
        "unit": "us/layer",
        "n_gpus": args.gpus,
        "steps": args.steps,
        "warmup": args.warmup,
        "higher_is_better": False,
        "scaling": "strong",
        "vs_baseline": None,
        "dtype": "bf16",
        "data": "synthetic",
        "config": {"workload": f"config 2 decode layer, T={T} tokens, TP={args.gpus}", "tokens": T},
        "cpu_baseline": {"value": round(us, 1), "unit": "us/layer", "cores": threads, "kind": "port",
                         "sample": f"{reps_tot} passes of one layer at T={T} (numpy oracle of the reference "
                                   f"path, f32 BLAS) on the host; the reference's Python package cannot "
                                   f"run on this box, so its restatement in oracle/ is timed"},
        "e2e": {"value": round(us, 1), "unit": "us/layer", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="pgb", choices=["pgb", "reference"])
    ap.add_argument("--tokens", default=",".join(map(str, TOKENS)))
    ap.add_argument("--layers", type=int, default=0)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-library-baseline", dest="library_baseline", action="store_false")
    ap.add_argument("--no-extras", dest="extras", action="store_false",
                    help="skip the side measurements (MLP / attention fronts, full layer); the step is unchanged")
    args = ap.parse_args()
    args.tokens = [int(t) for t in args.tokens.split(",")]
    if args.warmup < 3:
        args.warmup = 3
    res = run_reference(args) if args.impl == "reference" else run_ours(args)
    if res is not None:
        print(json.dumps(res), flush=True)


if __name__ == "__main__":
    main()
