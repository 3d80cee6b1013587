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
outputs are fixed synthetic activations. L is chosen so the step's weights
exceed 3x the 126 MB L2, so every layer streams its weights from HBM (no L2
flush is needed). The step is captured once in a CUDA graph (as the
reference's decode graphs, engine/graph.py:100-142) and replayed.

Before anything is timed, `parity` runs the fused row-parallel op (o_proj and
down_proj shapes of config 2 at T = 1 and 256, and of config 4 at T = 64) at
TP = N through the public API and compares it with the full-width f32
restatement of the reference sequence (per-rank bf16 partials, their sum
rounded to bf16, residual add, RMSNorm): every element within
max(2e-2 * RMS, 2 bf16 ulp + the effect of one bf16 rounding flip of each
rank's partial and of the reduced sum), and every rank holding bit-identical
results.
A failed check makes the process exit 1 after printing the line.

Beside the headline, the same run records (all per layer, CUDA events on the
launching stream, max over ranks):
  library_baseline      the reference's own unfused calls on this box: F.linear
                        (cuBLAS), torch NCCL all_reduce for TP > 1 (stand-in
                        for pynccl), flashinfer.fused_add_rmsnorm; per op too
  config.full_layer_us  the decoder layer minus the attention itself, through
                        the public API (fused fronts, real chain), against the
                        reference's calls on the same weights
  config.decode_36_layers  a 36-layer stack of that chain at T = 256 (config 5's
                        depth), tokens/s of the linear path
  config.prefill        config 3 (T = 8192) per op and per layer, fraction of
                        the tensor roofline
  config.config4        config 4 shapes (hidden 5120) at decode T = 64 and
                        prefill T = 4096
  config.nvlink         peer bandwidth measured here (NCCL send/recv ring) and
                        the NVLink GB/s of each fused row-parallel op

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
from dataclasses import dataclass
from datetime import timedelta
from pathlib import Path

import torch

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

EPS = 1e-6
TOKENS = (1, 8, 32, 128, 256)
HEADLINE_T = 256
PREFILL_T = 8192
L2_BYTES = 126 * 2**20
# DRAM read + write bytes of one gate_up launch (T=256, TP=1) of the single-CTA
# column kernel, from the ncu capture in profiles/col_gemm_gate_up_T256.md. The
# bench line reports it as `traffic` only when that kernel runs the shape.
GATE_UP_T256_TP1_DRAM_BYTES = 207_560_960  # 203.54 MB read + 4.02 MB written (ncu, one launch)
NVLINK_FALLBACK_GBS = 770.0  # peer copy per direction measured on this pool (profiling recipe)


@dataclass(frozen=True)
class Shape:
    """A dense decoder's linear shapes (BASELINE configs 2/3/5 and 4)."""

    name: str
    H: int
    I: int
    NQ: int
    NKV: int
    HD: int

    @property
    def QKV(self) -> int:
        return (self.NQ + 2 * self.NKV) * self.HD

    def local(self, n: int) -> dict:
        nkv = max(self.NKV // n, 1)
        return {"qkv": ((self.NQ // n + 2 * nkv) * self.HD, self.H), "o": (self.H, self.NQ * self.HD // n),
                "gate_up": (2 * self.I // n, self.H), "down": (self.H, self.I // n), "nq": self.NQ // n,
                "nkv": nkv}

    def layer_weight_bytes(self, n: int) -> float:
        loc = self.local(n)
        return 2.0 * sum(loc[k][0] * loc[k][1] for k in ("qkv", "o", "gate_up", "down"))


CFG2 = Shape("config 2", 4096, 12288, 32, 8, 128)
CFG4 = Shape("config 4", 5120, 25600, 64, 8, 128)


def gemm_kernel_name(T: int, N: int, K: int, sms: int = 148) -> str:
    """The column kernel the library's planner picks for y[T, N] = x . W^T (K
    inner): the CTA-pair kernels (prefill or 256-token decode tiles) or the
    single-CTA kernel."""
    try:
        import ctypes
        lib = importlib.import_module("pico-sglang_b200._lib").load()
        buf = ctypes.create_string_buffer(512)
        if lib.pgb_describe_plan(T, N, K, sms, 0, 1, buf, 512) != 0:
            return "col_gemm_kernel"
        desc = buf.value.decode()
    except Exception:  # the label only; never fail the bench line over it
        return "col_gemm_kernel"
    if "pair=1" in desc:
        return "col_gemm_pair_swap_kernel" if "swap=1" in desc else "col_gemm_pair_kernel"
    return "col_gemm_kernel"


def load_peaks() -> dict:
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return {"hbm_gbs": d["hbm_gbs"], "bf16_tflops": d["bf16_tflops"],
                "bf16_tflops_sustained": d.get("bf16_tflops_sustained", d["bf16_tflops"]), "src": "measured"}
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0, "src": "fallback"}


# ---------------------------------------------------------------- roofline --


def op_costs(T: int, n: int, cfg: Shape = CFG2) -> dict:
    """Algorithmic HBM bytes, FLOPs and NVLink bytes per GPU for each op.

    Column GEMM: HBM 2(N_l K + T K + T N_l), FLOPs 2 T K N_l.
    Row fused: HBM 2(N K_l + T K_l + T N) + 2(2 T N) + 2 N (weights, x, out,
    residual read + write, norm weight); NVLink 2(n-1)/n T N 2 bytes per
    direction (P2P reduce-scatter + all-gather formula).
    """
    loc = cfg.local(n)

    def col(N, K):
        return {"hbm": 2.0 * (N * K + T * K + T * N), "flops": 2.0 * T * K * N, "nvl": 0.0}

    def row(N, K):
        return {"hbm": 2.0 * (N * K + T * K + T * N) + 2.0 * 2 * T * N + 2.0 * N,
                "flops": 2.0 * T * K * N,
                "nvl": (2.0 * (n - 1) / n * T * N * 2) if n > 1 else 0.0}

    return {"qkv": col(*loc["qkv"]), "o": row(*loc["o"]), "gate_up": col(*loc["gate_up"]),
            "down": row(*loc["down"])}


def op_roofline_us(c: dict, peaks: dict, nvl_gbs: float, tflops: float | None = None) -> float:
    tf = tflops or peaks["bf16_tflops"]
    return max(c["hbm"] / (peaks["hbm_gbs"] * 1e9), c["flops"] / (tf * 1e12),
               c["nvl"] / (nvl_gbs * 1e9)) * 1e6


def roofline_us(T: int, n: int, peaks: dict, nvl_gbs: float, cfg: Shape = CFG2, tflops: float | None = None) -> float:
    return sum(op_roofline_us(c, peaks, nvl_gbs, tflops) for c in op_costs(T, n, cfg).values())


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


# ------------------------------------------------------------- harness ----


class Ctx:
    """Process-wide bench state: ranks, device, stream, groups."""

    def __init__(self, args):
        self.args = args
        self.world = int(os.environ.get("WORLD_SIZE", "1"))
        self.rank = int(os.environ.get("RANK", "0"))
        self.local = int(os.environ.get("LOCAL_RANK", "0"))
        self.n = self.world
        if args.gpus != self.world:
            raise SystemExit(f"--gpus {args.gpus} but WORLD_SIZE={self.world}")
        torch.cuda.set_device(self.local)
        self.dev = torch.device("cuda", self.local)
        import torch.distributed as dist

        self.dist = dist
        self.nccl = None
        if self.world > 1:
            dist.init_process_group("gloo", rank=self.rank, world_size=self.world, timeout=timedelta(seconds=300))
        self.stream = torch.cuda.Stream(self.dev)

    def barrier(self):
        if self.world > 1:
            self.dist.barrier()

    def nccl_group(self):
        """NCCL group of the library baseline (the reference's pynccl stand-in)."""
        if self.world > 1 and self.nccl is None:
            self.nccl = self.dist.new_group(backend="nccl", timeout=timedelta(seconds=300))
        return self.nccl

    def max_over_ranks(self, v: float) -> float:
        t = torch.tensor([v], dtype=torch.float64)
        if self.world > 1:
            self.dist.all_reduce(t, op=self.dist.ReduceOp.MAX)
        return t.item()

    def all_true(self, ok: bool) -> bool:
        t = torch.tensor([1 if ok else 0], dtype=torch.int64)
        if self.world > 1:
            self.dist.all_reduce(t, op=self.dist.ReduceOp.MIN)
        return bool(t.item())


def time_graph(ctx: Ctx, graph, steps: int, warmup: int) -> float:
    """ms for `steps` replays, CUDA events on the bench stream, max over ranks."""
    stream = ctx.stream
    with torch.cuda.stream(stream):
        for _ in range(warmup):
            graph.replay()
        torch.cuda.synchronize()
        ctx.barrier()
        torch.cuda.synchronize()
        e0 = torch.cuda.Event(enable_timing=True)
        e1 = torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(steps):
            graph.replay()
        e1.record(stream)
        torch.cuda.synchronize()
        ctx.barrier()
        torch.cuda.synchronize()
    return ctx.max_over_ranks(e0.elapsed_time(e1))


def capture(ctx: Ctx, fn):
    # Inputs are made on the default stream: let that work finish before the
    # bench stream touches them (the caching allocator hands out blocks that
    # pending default-stream work may still write).
    torch.cuda.synchronize()
    with torch.cuda.stream(ctx.stream):
        fn()  # eager warm-up: allocates workspaces (and NCCL state) outside capture
        torch.cuda.synchronize()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=ctx.stream):
            fn()
    torch.cuda.synchronize()
    return g


def time_fn_us(ctx: Ctx, fn, reps: int, steps: int | None = None, warmup: int | None = None) -> float:
    """Per-repetition microseconds of fn (fn runs `reps` units per call)."""
    steps = steps or ctx.args.steps
    warmup = warmup or ctx.args.warmup
    g = capture(ctx, fn)
    ms = time_graph(ctx, g, steps, warmup)
    del g
    return ms * 1000.0 / steps / reps


def rand_w(g, rows, cols, dev):
    return (torch.randn(rows, cols, device=dev, generator=g) * 0.02).bfloat16()


def build_layers(ctx: Ctx, L, cfg: Shape, n_layers: int, seed0: int = 0):
    """n_layers decoder layers of the public layer classes, TP-sharded for this rank."""
    layers = []
    dev = ctx.dev
    for li in range(n_layers):
        g = torch.Generator(device=dev).manual_seed(seed0 + li * 131 + ctx.rank)
        qkv = L.LinearColParallelPartitioned(cfg.H, cfg.HD, [(cfg.NQ, False), (cfg.NKV, True), (cfg.NKV, True)],
                                             has_bias=False)
        qkv.weight = rand_w(g, *qkv.weight.shape, dev)
        o = L.LinearRowParallel(cfg.NQ * cfg.HD, cfg.H, has_bias=False)
        o.weight = rand_w(g, *o.weight.shape, dev)
        gu = L.LinearColParallelMerged(cfg.H, [cfg.I, cfg.I], has_bias=False)
        gu.weight = rand_w(g, *gu.weight.shape, dev)
        down = L.LinearRowParallel(cfg.I, cfg.H, has_bias=False)
        down.weight = rand_w(g, *down.weight.shape, dev)
        ln1 = L.RMSNormFused(cfg.H, EPS)
        ln1.weight = torch.ones(cfg.H, device=dev).bfloat16()
        ln2 = L.RMSNormFused(cfg.H, EPS)
        ln2.weight = torch.ones(cfg.H, device=dev).bfloat16()
        o.link_norm(ln1)
        down.link_norm(ln2)
        layers.append({"qkv": qkv, "o": o, "gate_up": gu, "down": down, "ln1": ln1, "ln2": ln2})
    return layers


def n_layers_for(cfg: Shape, n: int, override: int = 0) -> int:
    return override or max(1, math.ceil(3 * L2_BYTES / cfg.layer_weight_bytes(n)))


class Step:
    """L decoder layers of the linear path, built from the public layer classes."""

    def __init__(self, ctx: Ctx, L, T: int, layers: list, cfg: Shape = CFG2):
        self.L = L
        self.layers = layers
        n, dev = ctx.n, ctx.dev
        g = torch.Generator(device=dev).manual_seed(1000 + T * 8 + ctx.rank)
        self.h = torch.randn(T, cfg.H, device=dev, generator=g).bfloat16()
        self.a = torch.randn(T, cfg.NQ * cfg.HD // n, device=dev, generator=g).bfloat16()
        self.m = torch.randn(T, cfg.I // n, device=dev, generator=g).bfloat16()
        self.res0 = torch.randn(T, cfg.H, device=dev, generator=g).bfloat16()
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


# ------------------------------------------------------------- parity -----


def _ulp(t):
    return torch.exp2(torch.floor(torch.log2(t.float().abs().clamp_min(1e-30))) - 7)


def _within(a, ref, tol=2e-2, ulps=2, extra=None):
    """|a - ref| <= max(tol * RMS(ref), ulps * ulp(ref) + extra) elementwise;
    returns (ok, worst / bound, max|diff| / RMS)."""
    ref = ref.float()
    rms = ref.pow(2).mean().sqrt().item()
    d = (a.float() - ref).abs()
    u = ulps * _ulp(ref) + (extra if extra is not None else 0.0)
    worst = (d / torch.maximum(torch.full_like(d, tol * rms), u)).max().item()
    return worst <= 1.0, worst, d.max().item() / max(rms, 1e-30)


def parity_check(ctx: Ctx, pgb, comm) -> dict:
    """The fused row-parallel op at TP = N against the full-width f32
    restatement of the reference sequence (LinearRowParallel.forward ->
    all_reduce -> fused_add_rmsnorm, python/picosgl/layers/linear.py:90-97,
    csrc/src/pynccl.cu:95-137, layers/norm.py:73-75). Every rank builds the
    same full-width inputs, runs its K-slice, and checks the result; the
    ranks' outputs are then compared bit for bit."""
    torch.backends.cuda.matmul.allow_tf32 = False
    n, rank, dev = ctx.n, ctx.rank, ctx.dev
    cases = []
    for cfg, T, op in ((CFG2, 1, "o"), (CFG2, 256, "o"), (CFG2, 1, "down"), (CFG2, 256, "down"),
                       (CFG4, 64, "o"), (CFG4, 64, "down")):
        H = cfg.H
        Kf = cfg.NQ * cfg.HD if op == "o" else cfg.I
        g = torch.Generator(device=dev).manual_seed(500 + T + Kf + H)
        x = torch.randn(T, Kf, device=dev, generator=g).bfloat16()
        w = rand_w(g, H, Kf, dev)
        r = torch.randn(T, H, device=dev, generator=g).bfloat16()
        nw = (1.0 + 0.1 * torch.randn(H, device=dev, generator=g)).bfloat16()
        k = Kf // n
        xl = x[:, rank * k:(rank + 1) * k].contiguous()
        wl = w[:, rank * k:(rank + 1) * k].contiguous()
        rr = r.clone()
        o = pgb.ops.row_gemm_allreduce_addnorm(comm, xl, wl, rr, nw, EPS)
        comm.check_status()
        parts = [(x[:, i * k:(i + 1) * k].float() @ w[:, i * k:(i + 1) * k].float().t()).bfloat16()
                 for i in range(n)]
        y = torch.stack([p.float() for p in parts]).sum(0).bfloat16()
        s = y.float() + r.float()
        ref_r = s.bfloat16()
        # The reference's output is materialised in bf16 (FlashInfer writes the
        # normalised row in the input dtype).
        rcp = torch.rsqrt(s.pow(2).mean(-1, keepdim=True) + EPS)
        ref = (s * rcp * nw.float()).bfloat16()
        # Two correct implementations may round each rank's bf16 partial and
        # the bf16 sum to neighbouring values (different summation orders):
        # allow one such flip per partial and in the sum, carried through the
        # residual add and the norm.
        dy = _ulp(y) + sum(_ulp(p_) for p_ in parts)
        ok_o, worst_o, d_o = _within(o, ref, extra=rcp * nw.float().abs() * dy)
        ok_r, worst_r, d_r = _within(rr, ref_r, extra=dy)
        same = True
        if n > 1:
            mine = torch.cat([o.reshape(-1), rr.reshape(-1)]).view(torch.uint8).cpu()
            got = [torch.empty_like(mine) for _ in range(n)]
            ctx.dist.all_gather(got, mine)
            same = all(torch.equal(got[0], t) for t in got[1:])
        cases.append({"case": f"{cfg.name} {op}_proj T={T} K_local={k} N={H}",
                      "max_abs_diff_over_rms": round(max(d_o, d_r), 5),
                      "worst_over_bound": round(max(worst_o, worst_r), 4),
                      "ranks_identical": same, "ok": bool(ok_o and ok_r and same)})
    ok = ctx.all_true(all(c["ok"] for c in cases))
    return {"ok": ok, "bar": "max(2e-2 x RMS, 2 bf16 ulp + one bf16 rounding flip of each rank partial and of "
                              "the reduced sum carried through the norm) per element vs the full-width f32 "
                              "restatement; all ranks bit-identical",
            "max_abs_diff_over_rms": max(c["max_abs_diff_over_rms"] for c in cases), "cases": cases}


# ----------------------------------------------------- library baseline ---


def _addnorm_fn():
    try:
        import flashinfer

        return flashinfer.fused_add_rmsnorm, "flashinfer.fused_add_rmsnorm"
    except Exception:  # pragma: no cover - flashinfer missing

        def fa(x, r, w, eps):
            s = x.float() + r.float()
            r.copy_(s.bfloat16())
            x.copy_((s * torch.rsqrt(s.pow(2).mean(-1, keepdim=True) + eps) * w.float()).bfloat16())

        return fa, "torch restatement of fused_add_rmsnorm"


def library_baseline(ctx: Ctx, cfg: Shape, T: int, n_layers: int, per_op: bool) -> dict:
    """The reference's own unfused calls on the same box: F.linear (cuBLAS),
    torch.distributed NCCL all_reduce for TP > 1 (stand-in for pynccl), and
    flashinfer.fused_add_rmsnorm, captured in a CUDA graph. Same step as ours
    (synthetic attention output and activation)."""
    import torch.nn.functional as F

    fa, kind = _addnorm_fn()
    grp = ctx.nccl_group()
    dist = ctx.dist
    n, dev = ctx.n, ctx.dev
    loc = cfg.local(n)
    g = torch.Generator(device=dev).manual_seed(7 + ctx.rank)
    layers = [{k: rand_w(g, *loc[k], dev) for k in ("qkv", "o", "gate_up", "down")} for _ in range(n_layers)]
    ln = torch.ones(cfg.H, device=dev).bfloat16()
    h = torch.randn(T, cfg.H, device=dev, generator=g).bfloat16()
    a = torch.randn(T, loc["o"][1], device=dev, generator=g).bfloat16()
    m = torch.randn(T, loc["down"][1], device=dev, generator=g).bfloat16()
    res = torch.randn(T, cfg.H, device=dev, generator=g).bfloat16()

    def row(x, w):
        y = F.linear(x, w)
        if grp is not None:
            dist.all_reduce(y, group=grp)
        fa(y, res, ln, EPS)
        return y

    def step():
        x = h
        for lay in layers:
            F.linear(x, lay["qkv"])
            x1 = row(a, lay["o"])
            F.linear(x1, lay["gate_up"])
            x = row(m, lay["down"])

    out = {"us_per_layer": round(time_fn_us(ctx, step, n_layers), 3), "tokens": T,
           "path": f"F.linear (cuBLAS) + {'torch NCCL all_reduce (pynccl stand-in) + ' if n > 1 else ''}{kind}",
           "graph": True}
    if per_op:
        ops = {"qkv": lambda lay: F.linear(h, lay["qkv"]), "o": lambda lay: row(a, lay["o"]),
               "gate_up": lambda lay: F.linear(h, lay["gate_up"]), "down": lambda lay: row(m, lay["down"])}
        out["op_us"] = {}
        for name, fn in ops.items():
            out["op_us"][name] = round(time_fn_us(ctx, lambda fn=fn: [fn(lay) for lay in layers], n_layers), 3)
        if grp is not None:
            yb = torch.empty(T, cfg.H, device=dev, dtype=torch.bfloat16)
            out["op_us"]["nccl_all_reduce_alone"] = round(
                time_fn_us(ctx, lambda: [dist.all_reduce(yb, group=grp) for _ in range(n_layers)], n_layers), 3)
    return out


# -------------------------------------------------------- side timings ----


def full_chain(ctx: Ctx, pgb, L, layers, cfg: Shape, T: int, seed: int, library: bool):
    """The decoder layer minus the attention itself, per layer, as a callable.
    Ours (public API): qkv_rope_store (qkv_proj + RoPE + KV store), o_proj
    linked to post_attention_layernorm (GEMM + all-reduce + residual add +
    RMSNorm in one kernel), gate_up_silu, down_proj linked to the next
    input_layernorm. Library: the reference's calls
    (python/picosgl/layers/attention.py:94-123, mlp.py:43-48, norm.py:73-75):
    F.linear, the FlashInfer RoPE on the strided split, an index store into the
    cache, F.linear + all_reduce + fused_add_rmsnorm, F.linear +
    silu_and_mul, F.linear + all_reduce + fused_add_rmsnorm. The attention
    output is a fixed synthetic tensor in both."""
    import torch.nn.functional as F

    n, dev = ctx.n, ctx.dev
    loc = cfg.local(n)
    nq, nkv = loc["nq"], loc["nkv"]
    g = torch.Generator(device=dev).manual_seed(seed + T + ctx.rank)
    h = torch.randn(T, cfg.H, device=dev, generator=g).bfloat16()
    a = torch.randn(T, nq * cfg.HD, device=dev, generator=g).bfloat16()
    res = torch.randn(T, cfg.H, device=dev, generator=g).bfloat16()
    table = L.get_rope(cfg.HD, cfg.HD, 4096, 1e6, None).cache_on(dev)
    pos = torch.randint(0, 4096, (T,), generator=g, device=dev, dtype=torch.int32)
    rows = max(4096, T)
    loc_i = torch.randperm(rows, generator=g, device=dev)[:T].to(torch.int32)
    loc64 = loc_i.long()
    caches = [(torch.zeros(rows, nkv, cfg.HD, device=dev, dtype=torch.bfloat16),
               torch.zeros(rows, nkv, cfg.HD, device=dev, dtype=torch.bfloat16)) for _ in layers]
    if not library:
        def ours():
            L.reset_fusion_context()
            L._CTX.residual = res
            x = h
            for lay, (kc, vc) in zip(layers, caches):
                pgb.ops.qkv_rope_store(x, lay["qkv"].weight, pos, loc_i, table, nq, nkv, cfg.HD, kc, vc)
                x1 = lay["o"].forward(a)
                x1, _ = lay["ln1"].forward(x1, res)
                mm = pgb.gate_up_silu(x1, lay["gate_up"].weight)
                x2 = lay["down"].forward(mm)
                x, _ = lay["ln2"].forward(x2, res)
        return ours

    import flashinfer

    fa = flashinfer.fused_add_rmsnorm
    grp = ctx.nccl_group()
    ln = torch.ones(cfg.H, device=dev).bfloat16()

    def lib():
        x = h
        for lay, (kc, vc) in zip(layers, caches):
            qkv = F.linear(x, lay["qkv"].weight)
            q, k, v = qkv.split([nq * cfg.HD, nkv * cfg.HD, nkv * cfg.HD], dim=-1)
            flashinfer.apply_rope_with_cos_sin_cache_inplace(pos, q, k, cfg.HD, table, is_neox=True)
            kc[loc64] = k.view(T, nkv, cfg.HD)
            vc[loc64] = v.view(T, nkv, cfg.HD)
            y = F.linear(a, lay["o"].weight)
            if grp is not None:
                ctx.dist.all_reduce(y, group=grp)
            fa(y, res, ln, EPS)
            mm = flashinfer.silu_and_mul(F.linear(y, lay["gate_up"].weight))
            x = F.linear(mm, lay["down"].weight)
            if grp is not None:
                ctx.dist.all_reduce(x, group=grp)
            fa(x, res, ln, EPS)
    return lib


def full_layer_timings(ctx: Ctx, pgb, L, layers, cfg: Shape, T: int) -> dict:
    out = {"tokens": int(T)}
    out["ours"] = round(time_fn_us(ctx, full_chain(ctx, pgb, L, layers, cfg, T, 21, False), len(layers)), 3)
    if ctx.args.library_baseline:
        try:
            out["library"] = round(time_fn_us(ctx, full_chain(ctx, pgb, L, layers, cfg, T, 21, True), len(layers)), 3)
        except ImportError:  # pragma: no cover - flashinfer missing
            pass
    return out


def decode_stack(ctx: Ctx, pgb, L, peaks: dict, nvl: float, n_layers: int = 36, T: int = HEADLINE_T) -> dict:
    """Config 5's depth: 36 distinct layers of the chain above at T = 256 in one
    CUDA graph, tokens/s of the linear path (attention, embedding and LM head
    are not in it), ours and the reference's calls."""
    layers = build_layers(ctx, L, CFG2, n_layers, seed0=90000)
    roof = n_layers * roofline_us(T, ctx.n, peaks, nvl)
    res = {"layers": n_layers, "tokens_per_step": T, "scope": "linear path only (no attention, embedding, LM head)"}
    for name, lib in (("ours", False), ("library", True)):
        if lib and not ctx.args.library_baseline:
            continue
        try:
            us = time_fn_us(ctx, full_chain(ctx, pgb, L, layers, CFG2, T, 33, lib), 1,
                            steps=max(5, ctx.args.steps // 2))
        except ImportError:  # pragma: no cover - flashinfer missing
            continue
        res[name] = {"us_per_step": round(us, 2), "tok_per_s": round(T / (us * 1e-6), 1),
                     "frac_of_linear_roofline": round(roof / us, 4)}
    res["roofline_us_per_step"] = round(roof, 2)
    del layers
    torch.cuda.empty_cache()
    return res


def linear_step_timings(ctx: Ctx, L, cfg: Shape, T: int, n_layers: int, peaks: dict, nvl: float,
                        tflops: float | None = None) -> dict:
    """The bench step (linear path) at another shape / token count, plus each
    op alone, with the roofline."""
    layers = build_layers(ctx, L, cfg, n_layers, seed0=7000 + T)
    st = Step(ctx, L, T, layers, cfg)
    us = time_fn_us(ctx, st.run, n_layers)
    roof = roofline_us(T, ctx.n, peaks, nvl, cfg, tflops)
    out = {"tokens": T, "tp": ctx.n, "layers_per_step": n_layers, "us_per_layer": round(us, 3),
           "roofline_us": round(roof, 3), "frac_of_roofline": round(roof / us, 4)}
    out["op_us"] = op_breakdown(ctx, L, layers, st, cfg, T, peaks, nvl, tflops)
    del layers, st
    torch.cuda.empty_cache()
    return out


def op_breakdown(ctx: Ctx, L, layers, st: Step, cfg: Shape, T: int, peaks: dict, nvl: float,
                 tflops: float | None = None) -> dict:
    res = st.residual
    costs = op_costs(T, ctx.n, cfg)
    x1 = st.h

    def only(name):
        def f():
            L.reset_fusion_context()
            for lay in layers:
                if name == "qkv":
                    lay["qkv"].forward(st.h)
                elif name == "gate_up":
                    lay["gate_up"].forward(x1)
                elif name == "o":
                    L._CTX.residual = res
                    lay["o"].forward(st.a)
                else:
                    L._CTX.residual = res
                    lay["down"].forward(st.m)
        return f

    out = {}
    for name in ("qkv", "o", "gate_up", "down"):
        us = time_fn_us(ctx, only(name), len(layers))
        c = costs[name]
        rec = {"us": round(us, 3), "roofline_us": round(op_roofline_us(c, peaks, nvl, tflops), 3),
               "hbm_gbs": round(c["hbm"] / (us * 1e-6) / 1e9, 1)}
        if c["flops"] / (us * 1e-6) > 1e13:
            rec["tflops"] = round(c["flops"] / (us * 1e-6) / 1e12, 1)
        if c["nvl"] > 0:
            rec["nvlink_gbs"] = round(c["nvl"] / (us * 1e-6) / 1e9, 1)
        out[name] = rec
    return out


def measure_nvlink(ctx: Ctx, nbytes: int = 256 << 20) -> float | None:
    """Per-direction peer bandwidth on this box: every rank sends nbytes to
    rank + 1 and receives from rank - 1 at once (NCCL send/recv over NVLink),
    CUDA events, max time over ranks. Used as the NVLink roofline denominator."""
    if ctx.world < 2:
        return None
    grp = ctx.nccl_group()
    dist = ctx.dist
    src = torch.empty(nbytes // 2, dtype=torch.bfloat16, device=ctx.dev).fill_(1)
    dst = torch.empty_like(src)
    nxt, prv = (ctx.rank + 1) % ctx.n, (ctx.rank - 1) % ctx.n

    def once():
        ops = [dist.P2POp(dist.isend, src, nxt, grp), dist.P2POp(dist.irecv, dst, prv, grp)]
        for r in dist.batch_isend_irecv(ops):
            r.wait()

    torch.cuda.synchronize()
    with torch.cuda.stream(ctx.stream):
        for _ in range(3):
            once()
        torch.cuda.synchronize()
        ctx.barrier()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(ctx.stream)
        reps = 10
        for _ in range(reps):
            once()
        e1.record(ctx.stream)
        torch.cuda.synchronize()
    ms = ctx.max_over_ranks(e0.elapsed_time(e1)) / reps
    del src, dst
    return nbytes / (ms * 1e-3) / 1e9


def mlp_front_timings(ctx: Ctx, pgb, layers, x1) -> dict:
    """The gated MLP's front half, gate_up_proj then silu_and_mul
    (python/picosgl/layers/mlp.py:43-46), per layer at the headline T, three ways:
    the fused kernel, this library's GEMM then its standalone activation, and
    the reference's own calls (F.linear + flashinfer.silu_and_mul)."""
    import torch.nn.functional as F

    ways = {
        "fused_gate_up_silu": lambda lay: pgb.gate_up_silu(x1, lay["gate_up"].weight),
        "col_gemm_then_silu_and_mul": lambda lay: pgb.silu_and_mul(pgb.col_gemm(x1, lay["gate_up"].weight)),
    }
    if ctx.args.library_baseline:
        try:
            import flashinfer

            ways["F.linear_then_flashinfer_silu_and_mul"] = (
                lambda lay: flashinfer.silu_and_mul(F.linear(x1, lay["gate_up"].weight)))
        except Exception:  # pragma: no cover - flashinfer missing
            pass
    out = {"tokens": int(x1.shape[0])}
    for name, fn in ways.items():
        out[name] = round(time_fn_us(ctx, lambda fn=fn: [fn(lay) for lay in layers], len(layers)), 3)
    return out


def attn_front_timings(ctx: Ctx, pgb, L, layers, h) -> dict:
    """The attention block's front, qkv_proj + RoPE + KV-cache store
    (RotaryAttention.proj, python/picosgl/layers/attention.py:94-117, then
    store_kv), per layer at the headline T, three ways: the fused kernel, this
    library's GEMM then its standalone RoPE + store, and the reference's calls
    (F.linear + flashinfer.apply_rope_with_cos_sin_cache_inplace + an index
    store). Positions are random below 4096 (RoPE theta 1e6, config 5); each
    layer writes its own [4096, kv heads, 128] caches at random slots."""
    import torch.nn.functional as F

    cfg, n, dev = CFG2, ctx.n, ctx.dev
    T = h.shape[0]
    nq, nkv, HD = cfg.local(n)["nq"], cfg.local(n)["nkv"], cfg.HD
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
    if ctx.args.library_baseline:
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
        out[name] = round(time_fn_us(ctx, lambda fn=fn: [fn(lay, kc, vc) for lay, (kc, vc) in zip(layers, caches)],
                                     len(layers)), 3)
    return out


# ------------------------------------------------------------- our arm ----


def run_ours(args) -> tuple[dict | None, bool]:
    ctx = Ctx(args)
    n, rank, world, dev = ctx.n, ctx.rank, ctx.world, ctx.dev
    pgb = importlib.import_module("pico-sglang_b200")
    D = importlib.import_module("pico-sglang_b200.distributed")
    L = importlib.import_module("pico-sglang_b200.layers")
    D.set_tp_info(D.DistributedInfo(rank, world))
    if world > 1:
        comm = D.enable_pgb_distributed(D.get_tp_info(), ctx.dist.group.WORLD, 64 << 20)
    else:
        comm = D.local_comm(64 << 20)

    peaks = load_peaks()
    parity = parity_check(ctx, pgb, comm)
    nvl_measured = measure_nvlink(ctx) if world > 1 else None
    nvl = nvl_measured or NVLINK_FALLBACK_GBS

    n_layers = n_layers_for(CFG2, n, args.layers)
    layers = build_layers(ctx, L, CFG2, n_layers)

    per_t = {}
    graphs = {}
    steps_obj = {}
    for T in args.tokens:
        st = Step(ctx, L, T, layers)
        g = capture(ctx, st.run)
        graphs[T] = g
        steps_obj[T] = st
        clocks = ClockSampler(ctx.local) if T == HEADLINE_T else None
        if clocks:
            clocks.start()
        ms = time_graph(ctx, g, args.steps, args.warmup)
        ck = clocks.stop() if clocks else None
        us_layer = ms * 1000.0 / args.steps / n_layers
        roof = roofline_us(T, n, peaks, nvl)
        per_t[T] = {"us_per_layer": round(us_layer, 3), "tok_per_s_per_layer": round(T / (us_layer * 1e-6), 1),
                    "roofline_us": round(roof, 3), "frac_of_roofline": round(roof / us_layer, 4)}
        if ck:
            per_t[T]["clocks"] = ck

    # Dominant kernel: gate_up column GEMM (52% of a layer's weight bytes), at
    # the headline T, one launch per layer (distinct weights), CUDA events.
    T = HEADLINE_T if HEADLINE_T in args.tokens else args.tokens[-1]
    st = steps_obj[T]
    breakdown = op_breakdown(ctx, L, layers, st, CFG2, T, peaks, nvl)
    gu_us = breakdown["gate_up"]["us"]
    gu_bytes = op_costs(T, n)["gate_up"]["hbm"]
    gu_kernel = gemm_kernel_name(T, 2 * CFG2.I // n, CFG2.H, torch.cuda.get_device_properties(dev).multi_processor_count)
    achieved = gu_bytes / (gu_us * 1e-6) / 1e9

    # End to end through the public API: pinned host inputs copied in, the
    # captured layer stack replayed, the output and residual copied out.
    hbuf = {k: torch.empty_like(v, device="cpu").pin_memory() for k, v in
            (("h", st.h), ("a", st.a), ("m", st.m), ("r", st.res0))}
    for k, v in (("h", st.h), ("a", st.a), ("m", st.m), ("r", st.res0)):
        hbuf[k].copy_(v)
    out_h = torch.empty(tuple(st.h.shape), dtype=torch.bfloat16).pin_memory()
    res_h = torch.empty(tuple(st.h.shape), dtype=torch.bfloat16).pin_memory()
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

    with torch.cuda.stream(ctx.stream):
        for _ in range(args.warmup):
            e2e_step()
        torch.cuda.synchronize()
        ctx.barrier()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(ctx.stream)
        for _ in range(args.steps):
            e2e_step()
        e1.record(ctx.stream)
        torch.cuda.synchronize()
        ctx.barrier()
    e2e_us = ctx.max_over_ranks(e0.elapsed_time(e1)) * 1000.0 / args.steps / n_layers
    for gg in graphs.values():
        del gg
    graphs.clear()

    lib = lib_small = None
    if args.library_baseline:
        lib = library_baseline(ctx, CFG2, T, n_layers, per_op=True)
        if 1 in args.tokens and T != 1:
            lib_small = library_baseline(ctx, CFG2, 1, n_layers, per_op=False)

    extras = {}
    if args.extras:
        x1 = torch.randn(T, CFG2.H, device=dev).bfloat16()
        extras["mlp_front_us"] = mlp_front_timings(ctx, pgb, layers, x1)
        extras["attn_front_us"] = attn_front_timings(ctx, pgb, L, layers, st.h)
        extras["full_layer_us"] = {str(t): full_layer_timings(ctx, pgb, L, layers, CFG2, t)
                                   for t in sorted({1, T} & set(args.tokens) | {T})}
    del layers, steps_obj
    torch.cuda.empty_cache()
    if args.extras:
        extras["decode_36_layers"] = decode_stack(ctx, pgb, L, peaks, nvl)
        tf_s = peaks["bf16_tflops_sustained"]
        pre = linear_step_timings(ctx, L, CFG2, PREFILL_T, 2, peaks, nvl, tflops=tf_s)
        pre["roofline_peak"] = f"bf16 sustained {tf_s} TFLOP/s ({peaks['src']}), HBM {peaks['hbm_gbs']} GB/s, " \
                               f"NVLink {nvl:.0f} GB/s"
        if args.library_baseline:
            pre["library"] = library_baseline(ctx, CFG2, PREFILL_T, 2, per_op=True)
        extras["prefill"] = pre
        c4 = {}
        for t4, nl in ((64, n_layers_for(CFG4, n)), (4096, 2)):
            rec = linear_step_timings(ctx, L, CFG4, t4, nl, peaks, nvl, tflops=(tf_s if t4 > 256 else None))
            if args.library_baseline:
                rec["library"] = library_baseline(ctx, CFG4, t4, nl, per_op=False)
            c4[str(t4)] = rec
        extras["config4"] = c4

    result = None
    if rank == 0:
        head = per_t[T]
        cpu = cpu_baseline(T) if (world == 1 and not args.no_cpu_baseline) else None
        cpu1 = cpu_baseline_config1() if (world == 1 and not args.no_cpu_baseline) else None
        # One rank: o_proj and down_proj each run as the column GEMM + the norm
        # kernel (pgb_comm_set_one_rank_path); more ranks: one fused kernel each.
        launches = (4 if world > 1 else 6) * n_layers * args.steps
        nvl_info = {"peer_gbs_measured": round(nvl_measured, 1) if nvl_measured else None,
                    "peer_gbs_used": round(nvl, 1),
                    "how": ("NCCL send/recv ring of 256 MiB per rank, all ranks at once, CUDA events, max over "
                            "ranks" if nvl_measured else
                            "one GPU: no NVLink; 770 GB/s per direction is the pool's measured peer copy"),
                    "o_fused_gbs": breakdown["o"].get("nvlink_gbs"),
                    "down_fused_gbs": breakdown["down"].get("nvlink_gbs"),
                    "formula": "2(n-1)/n * T * H * 2 bytes per direction (P2P reduce-scatter + all-gather)"}
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
            "parity": parity,
            "config": {
                "workload": f"config 2 decode layer, T={T} tokens, TP={n}",
                "hidden": CFG2.H, "intermediate": CFG2.I, "q_heads": CFG2.NQ, "kv_heads": CFG2.NKV,
                "head_dim": CFG2.HD, "tokens": T, "tp": n, "layers_per_step": n_layers,
                "row_path": ("fused GEMM + all-reduce + residual-add + RMSNorm kernel" if n > 1 else
                             "one rank: column GEMM then the fused_add_rmsnorm kernel (no all-reduce)"),
                "l2": f"inputs larger than L2: {n_layers} distinct layers, "
                      f"{CFG2.layer_weight_bytes(n) * n_layers / 2**20:.0f} MiB of weights per GPU per step",
                "graph": "step captured in one CUDA graph and replayed",
                "per_tokens": {str(k): v for k, v in per_t.items()},
                "op_breakdown_us": breakdown,
                "layer_roofline_us": head["roofline_us"],
                "layer_frac_of_roofline": head["frac_of_roofline"],
                "nvlink": nvl_info,
                **extras,
            },
            "tok_per_s_per_layer": head["tok_per_s_per_layer"],
            "roofline": {
                "kernel": f"{gu_kernel} (gate_up_proj, swap-AB tcgen05)",
                "bound": "hbm",
                "achieved": round(achieved, 1),
                "peak": peaks["hbm_gbs"],
                "unit": "GB/s",
                "frac": round(achieved / peaks["hbm_gbs"], 4),
                "peak_src": peaks["src"] + " (burst copy bandwidth)",
                # DRAM read + write bytes of one launch from an ncu capture of this
                # kernel on this shape, where one exists (see GATE_UP_T256_TP1_DRAM_BYTES).
                "traffic": GATE_UP_T256_TP1_DRAM_BYTES if (n == 1 and T == 256 and gu_kernel == "col_gemm_kernel")
                else None,
                "traffic_single_cta_kernel": GATE_UP_T256_TP1_DRAM_BYTES if (n == 1 and T == 256) else None,
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
        if cpu1:
            result["cpu_baseline_config1"] = cpu1
        if lib:
            result["library_baseline"] = lib
        if lib_small:
            result["library_baseline_T1"] = lib_small
    ok = parity["ok"]
    if world > 1:
        D.destroy_distributed()
        if ctx.nccl is not None:
            ctx.dist.destroy_process_group(ctx.nccl)
        ctx.dist.destroy_process_group()
    return result, ok


# ----------------------------------------------------------- CPU baseline --


def _cpu_sample(T: int, budget_s: float):
    """The CPU oracle (numpy restatement of the reference path) on one layer
    of the bench config at TP=1, f32 BLAS accumulation, repeated until the
    time budget is spent. Returns (us per layer, reps, threads)."""
    import numpy as np

    import oracle

    H, I, QKV = CFG2.H, CFG2.I, CFG2.QKV
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


def _config1_rank(rank: int, port: int, threads: int, budget_s: float, q) -> None:
    """One rank of BASELINE config 1 on the CPU: the oracle's restatement of
    LinearRowParallel.forward on this rank's K-half, the sum all-reduce over a
    gloo group of two processes, then fused_add_rmsnorm, all in f32."""
    try:
        from threadpoolctl import threadpool_limits

        threadpool_limits(threads)
    except Exception:
        pass
    import numpy as np
    import torch.distributed as dist

    import oracle

    # Under torchrun this process inherits the elastic agent's store setting,
    # which would make both ranks clients of a store nobody serves: the pair
    # below has its own rendezvous.
    os.environ.pop("TORCHELASTIC_USE_AGENT_STORE", None)
    torch.set_num_threads(threads)
    dist.init_process_group("gloo", rank=rank, world_size=2, init_method=f"tcp://127.0.0.1:{port}",
                            timeout=timedelta(seconds=120))
    gen = torch.Generator().manual_seed(0)
    x = torch.randn(64, 4096, generator=gen)
    w = torch.randn(4096, 4096, generator=gen) * 0.02
    res0 = torch.randn(64, 4096, generator=gen)
    nw = np.ones(4096, np.float32)
    xl = x[:, rank * 2048:(rank + 1) * 2048].numpy()
    wl = w[:, rank * 2048:(rank + 1) * 2048].numpy()

    def layer():
        y = torch.from_numpy(oracle.linear(xl, wl, dtype="f32", accum="f32"))
        dist.all_reduce(y)
        return oracle.fused_add_rmsnorm(y.numpy(), res0.numpy(), nw, EPS, dtype="f32")

    layer()
    dist.barrier()
    reps, t0 = 0, time.perf_counter()
    while True:
        layer()
        reps += 1
        flag = torch.tensor([1 if (time.perf_counter() - t0) >= budget_s or reps >= 2000 else 0])
        dist.all_reduce(flag, op=dist.ReduceOp.MAX)
        if flag.item():
            break
    el = time.perf_counter() - t0
    dist.destroy_process_group()
    q.put((rank, el / reps * 1e6, reps))


def cpu_baseline_config1(budget_s: float = 5.0) -> dict | None:
    """BASELINE config 1 as written: world_size 2 over gloo, fp32, x [64, 4096]
    split to [64, 2048] per rank, W [4096, 4096] split along K, residual add +
    RMSNorm (weight ones, eps 1e-6), seed 0; the reference's Python package is
    not on this box, so the oracle's restatement runs in two spawned processes
    with the host's cores split between them."""
    import multiprocessing as mp

    cores = os.cpu_count() or 2
    threads = max(1, cores // 2)
    port = 29000 + (os.getpid() % 900)
    ctxm = mp.get_context("spawn")
    q = ctxm.Queue()
    procs = [ctxm.Process(target=_config1_rank, args=(r, port, threads, budget_s, q)) for r in range(2)]
    for p in procs:
        p.start()
    got = {}
    try:
        for _ in range(2):
            r, us, reps = q.get(timeout=180)
            got[r] = (us, reps)
    except Exception:
        return None
    finally:
        for p in procs:
            p.join(timeout=30)
            if p.is_alive():
                p.kill()
    us = max(v[0] for v in got.values())
    return {"value": round(us, 1), "unit": "us/layer", "cores": 2 * threads, "kind": "port",
            "threads_per_rank": threads, "host_cores": cores,
            "sample": f"{got[0][1]} passes of BASELINE config 1 (LinearRowParallel + gloo all_reduce + "
                      f"fused_add_rmsnorm, fp32, world_size 2, x[64,4096], W[4096,4096]) in two processes, "
                      f"oracle restatement"}


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
    cfg1 = cpu_baseline_config1() if not args.no_cpu_baseline else None
    out = {
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
        "config": {"workload": f"config 2 decode layer, T={T} tokens, TP={args.gpus}",
                   "hidden": CFG2.H, "intermediate": CFG2.I, "q_heads": CFG2.NQ, "kv_heads": CFG2.NKV,
                   "head_dim": CFG2.HD, "tokens": T, "tp": args.gpus},
        "cpu_baseline": {"value": round(us, 1), "unit": "us/layer", "cores": threads, "kind": "port",
                         "sample": f"{reps_tot} passes of one layer at T={T} (numpy oracle of the reference "
                                   f"path, f32 BLAS) on the host; the reference's Python package cannot "
                                   f"run on this box, so its restatement in oracle/ is timed"},
        "e2e": {"value": round(us, 1), "unit": "us/layer", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    if cfg1:
        out["cpu_baseline_config1"] = cfg1
    return out


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
                    help="skip the side measurements (fronts, full layer, 36-layer stack, prefill, config 4); "
                         "the step is unchanged")
    args = ap.parse_args()
    args.tokens = [int(t) for t in args.tokens.split(",")]
    if args.warmup < 3:
        args.warmup = 3
    if args.impl == "reference":
        res, ok = run_reference(args), True
    else:
        res, ok = run_ours(args)
    if res is not None:
        print(json.dumps(res), flush=True)
    if not ok:
        sys.stderr.write("parity check failed (see the line's `parity` object)\n")
        sys.exit(1)


if __name__ == "__main__":
    main()
