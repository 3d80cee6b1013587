"""Multi-GPU communicator and fused row-parallel kernel, one process per GPU.

Mirrors the reference's communicator test (tests/distributed/test_pynccl.py):
spawned ranks, a gloo CPU group for bootstrap, the same known answers
(ones reduced four times = tp^4; rank values = n(n-1)/2 with rank 0
lagging 1 s; half zeros / half ones -> {0, tp}; all_gather of the rank id).
Then the fused GEMM + all-reduce + residual-add + RMSNorm at TP = n against
the full-width f32 restatement, one-shot and two-shot sizes, CUDA-graph
replay, and a bounded timeout when a peer never joins.

Needs at least 2 GPUs; ranks never share a GPU (kernels that wait on one
another must run on different devices).
"""

from __future__ import annotations

import os
import sys
import time
import traceback
from datetime import timedelta
from pathlib import Path

import pytest
import torch

pytestmark = pytest.mark.gpu

ROOT = Path(__file__).resolve().parent.parent
EPS = 1e-6


def _ngpus() -> int:
    return torch.cuda.device_count() if torch.cuda.is_available() else 0


def _ulp(t):
    mant = {torch.bfloat16: 7, torch.float16: 10, torch.float32: 23}[t.dtype]
    return torch.exp2(torch.floor(torch.log2(t.float().abs().clamp_min(1e-30))) - mant)


def _within(a, ref, tol=2e-2, ulps=2, extra=None):
    """|a - ref| <= max(tol * RMS(ref), ulps * ulp(ref) + extra) elementwise.

    The reference rounds each rank's partial to bf16 (F.linear), rounds the
    reduced sum again (all_reduce in bf16), then rounds residual and output:
    two roundings precede every compared value, so two-ulp flips between two
    correct implementations are expected at large magnitudes. `extra` adds
    the effect of one rounding flip of each partial and of the reduced sum
    carried through the residual add and the norm (summation orders differ;
    the NVLink switch rounds its f32 sum on its own).
    """
    rms = ref.float().pow(2).mean().sqrt().item()
    d = (a.float() - ref.float()).abs()
    u = ulps * _ulp(ref) + (extra if extra is not None else 0.0)
    worst = (d / torch.maximum(torch.full_like(d, tol * rms), u)).max().item()
    return worst <= 1.0, f"max|diff|={d.max().item():.4g} rms={rms:.4g} worst/bound={worst:.3g}"


def _no_worse_than_reference(mine, ref_path, exact):
    """Error of this kernel against the unrounded f64 result is at most the
    reference algorithm's own error, plus a quarter of it or half an output
    ulp at the largest magnitude, whichever is larger: the sums run in other
    orders (the NVLink switch picks its own), so one element's rounding can
    land one step away from the reference's."""
    em = (mine.double() - exact).abs().max().item()
    er = (ref_path.double() - exact).abs().max().item()
    half_ulp = 0.5 * _ulp(exact.abs().max().reshape(1).to(mine.dtype)).item()
    return em <= max(1.25 * er, er + half_ulp) + 1e-6, f"err_mine={em:.4g} err_reference={er:.4g}"


def _worker(rank: int, world: int, port: int, case: str, q):
    try:
        sys.path.insert(0, str(ROOT))
        import importlib

        import torch.distributed as dist

        torch.cuda.set_device(rank)
        dist.init_process_group("gloo", rank=rank, world_size=world,
                                init_method=f"tcp://127.0.0.1:{port}", timeout=timedelta(seconds=120))
        pgb = importlib.import_module("pico-sglang_b200")
        D = importlib.import_module("pico-sglang_b200.distributed")
        # The fused case also binds an NVLink multicast region where the
        # devices support it; the timeout case keeps it off (a rank that
        # leaves while its memory is bound to a multicast object is not a
        # failure to provoke).
        comm = D.init_comm(tp_rank=rank, tp_size=world, tp_cpu_group=dist.group.WORLD,
                           max_size_bytes=64 << 20, nvls=(case == "fused"))
        dev = torch.device("cuda", rank)
        out = {}
        if case == "known_answers":
            K = 512
            dtype = torch.float16
            f = lambda x: comm.all_reduce(x, "sum")  # noqa: E731
            x = torch.ones(8192 * K, dtype=dtype, device=dev)
            for _ in range(4):
                f(x)
            out["pow"] = bool(torch.all(x == world ** 4).item())
            x = torch.full((8192 * K,), rank, dtype=dtype, device=dev)
            if rank == 0:
                torch.cuda.synchronize()
                time.sleep(1)
            f(x)
            out["lag"] = bool(torch.all(x == world * (world - 1) // 2).item())
            x = torch.cat([torch.zeros(8192 * K // 2, dtype=dtype, device=dev),
                           torch.ones(8192 * K // 2, dtype=dtype, device=dev)])
            f(x)
            out["half"] = bool(torch.all(x[: 8192 * K // 2] == 0).item() and torch.all(x[8192 * K // 2:] == world).item())
            for dt in (torch.bfloat16, torch.float32):
                for n in (1, 7, 1000, 12345):
                    x = torch.full((n,), float(rank + 1), dtype=dt, device=dev)
                    f(x)
                    out[f"small_{dt}_{n}"] = bool(torch.all(x == world * (world + 1) / 2).item())
            src = torch.full((K,), rank, dtype=dtype, device=dev)
            dst = torch.empty((K * world,), dtype=dtype, device=dev)
            comm.all_gather(dst, src)
            exp = torch.arange(world, dtype=dtype, device=dev).repeat_interleave(K)
            out["gather"] = bool(torch.equal(dst, exp))
            # 16-byte vector path (above) and element path (7 elements)
            for cnt, dt in ((7, torch.bfloat16), (1000, torch.float32), (3 << 20, torch.bfloat16)):
                src = torch.full((cnt,), rank + 1, dtype=dt, device=dev)
                dst = torch.empty((cnt * world,), dtype=dt, device=dev)
                comm.all_gather(dst, src)
                exp = torch.arange(1, world + 1, dtype=dt, device=dev).repeat_interleave(cnt)
                out[f"gather_{cnt}_{dt}"] = bool(torch.equal(dst, exp))
            # a large payload in chunks through the vector path: 96 MiB > the 64 MiB buffer
            x = torch.full((48 << 20,), float(rank + 1), dtype=torch.bfloat16, device=dev)
            f(x)
            out["chunked"] = bool(torch.all(x == world * (world + 1) / 2).item())
            comm.check_status()
        elif case == "fused":
            # Decode shapes under every exchange mode of the multi-rank row op
            # (per-piece one-shot / two-shot, the cost model's pick, and the
            # grid-barrier kernel), then a prefill shape and a ragged one.
            import ctypes

            sup = ctypes.c_int(0)
            pgb._lib.call("pgb_comm_nvls_supported", comm.handle, ctypes.byref(sup))
            out["nvls_bound_where_supported"] = (comm.nvls == bool(sup.value), f"supported={sup.value} bound={comm.nvls}")
            modes = ("auto", "oneshot", "twoshot", "barrier") + (("nvls",) if comm.nvls else ())
            runs = [(mode, shp) for mode in modes
                    for shp in ((1, 4096, 4096), (8, 4096, 12288), (64, 4096, 4096), (256, 4096, 12288),
                                (64, 5120, 25600))]
            # A prefill batch: the default mode runs it as the pair-tile GEMM + all-reduce
            # + norm, the barrier mode on the fused kernel.
            runs += [("auto", (1000, 4096, 2048)), ("barrier", (1000, 4096, 2048)), ("auto", (3, 200, 256)),
                     ("twoshot", (3, 200, 256))]
            if comm.nvls:
                runs += [("nvls", (3, 200, 256))]
            for mode, (T, H, K) in runs:
                comm.set_exchange_mode(mode)
                g = torch.Generator(device=dev).manual_seed(T + H + K)
                x = torch.randn(T, K, device=dev, generator=g).bfloat16()
                w = (torch.randn(H, K, device=dev, generator=g) * 0.02).bfloat16()
                r = torch.randn(T, H, device=dev, generator=g).bfloat16()
                nw = (1.0 + 0.1 * torch.randn(H, device=dev, generator=g)).bfloat16()
                k = K // world
                xl = x[:, rank * k:(rank + 1) * k].contiguous()
                wl = w[:, rank * k:(rank + 1) * k].contiguous()
                # Reference: per-rank bf16 partials (F.linear), summed, rounded, add-norm.
                parts = [(x[:, i * k:(i + 1) * k].float() @ w[:, i * k:(i + 1) * k].float().t()).bfloat16()
                         for i in range(world)]
                y = torch.stack([p.float() for p in parts]).sum(0).bfloat16()
                s = y.float() + r.float()
                ref_r = s.bfloat16()
                rcp = torch.rsqrt(s.pow(2).mean(-1, keepdim=True) + EPS)
                ref = (s * rcp * nw.float()).bfloat16()
                dparts = sum(_ulp(p) for p in parts)
                dy = _ulp(y) + dparts
                ye = x.double() @ w.double().t()
                se = ye + r.double()
                exact = se * torch.rsqrt(se.pow(2).mean(-1, keepdim=True) + EPS) * nw.double()
                rr = r.clone()
                o = pgb.ops.row_gemm_allreduce_addnorm(comm, xl, wl, rr, nw, EPS)
                yy = pgb.ops.row_gemm_allreduce_addnorm(comm, xl, wl, None, None, EPS)
                comm.check_status()
                tag = f"{mode}_{T}_{H}_{K}"
                out[f"out_{tag}"] = _within(o, ref, extra=rcp * nw.float().abs() * dy)
                out[f"res_{tag}"] = _within(rr, ref_r, extra=dy)
                out[f"y_{tag}"] = _within(yy, y, extra=dparts)
                out[f"exact_out_{tag}"] = _no_worse_than_reference(o, ref, exact)
                out[f"exact_res_{tag}"] = _no_worse_than_reference(rr, ref_r, se)
                # Every rank must hold the identical result (replicated residual
                # stream): gather every rank's tensors and compare them bit for bit.
                mine = torch.cat([o.reshape(-1), rr.reshape(-1), yy.reshape(-1)]).view(torch.uint8).cpu()
                gathered = [torch.empty_like(mine) for _ in range(world)]
                dist.all_gather(gathered, mine)
                same = all(torch.equal(gathered[0], t) for t in gathered[1:])
                out[f"same_{tag}"] = (same, "tensors differ between ranks")
            comm.set_exchange_mode("auto")
            # f32 check mode: IEEE f32 GEMM + all-reduce + add/RMSNorm, 1e-5 relative
            T, H, K = 8, 4096, 4096
            g = torch.Generator(device=dev).manual_seed(17)
            xf = torch.randn(T, K, device=dev, generator=g)
            wf = torch.randn(H, K, device=dev, generator=g) * 0.02
            rf = torch.randn(T, H, device=dev, generator=g)
            nwf = torch.rand(H, device=dev, generator=g) + 0.5
            k0, k1 = rank * K // world, (rank + 1) * K // world
            rr32 = rf.clone()
            o32 = pgb.ops.row_gemm_allreduce_addnorm(comm, xf[:, k0:k1].contiguous(), wf[:, k0:k1].contiguous(),
                                                     rr32, nwf, EPS)
            torch.cuda.synchronize()
            s64 = xf.double() @ wf.double().t() + rf.double()
            ref64 = s64 * torch.rsqrt(s64.pow(2).mean(-1, keepdim=True) + EPS) * nwf.double()
            rms = ref64.pow(2).mean().sqrt().item()
            e_out = (o32.double() - ref64).abs().max().item() / rms
            e_res = (rr32.double() - s64).abs().max().item() / s64.pow(2).mean().sqrt().item()
            out["f32_check"] = (e_out <= 1e-5 and e_res <= 1e-5, f"rel err out {e_out:.3g} residual {e_res:.3g}")
            # graph replay
            T, H, K = 16, 4096, 4096
            g = torch.Generator(device=dev).manual_seed(5)
            x = torch.randn(T, K // world, device=dev, generator=g).bfloat16()
            w = (torch.randn(H, K // world, device=dev, generator=g) * 0.02).bfloat16()
            r = torch.randn(T, H, device=dev, generator=g).bfloat16()
            nw = torch.ones(H, device=dev).bfloat16()
            rr = r.clone()
            o = torch.empty_like(r)
            pgb.ops.row_gemm_allreduce_addnorm(comm, x, w, rr, nw, EPS, out=o)
            torch.cuda.synchronize()
            first = o.clone()
            s = torch.cuda.Stream()
            graph = torch.cuda.CUDAGraph()
            with torch.cuda.stream(s), torch.cuda.graph(graph, stream=s):
                pgb.ops.row_gemm_allreduce_addnorm(comm, x, w, rr, nw, EPS, out=o)
            same = True
            for _ in range(3):
                rr.copy_(r)
                torch.cuda.synchronize()
                dist.barrier()
                graph.replay()
                torch.cuda.synchronize()
                same &= bool(torch.equal(o, first))
            comm.check_status()
            del graph
            out["graph"] = (same, "")
        elif case == "timeout":
            comm.set_timeout(0.3)
            x = torch.ones(4096, dtype=torch.bfloat16, device=dev)
            raised = False
            if rank == 0:
                comm.all_reduce(x, "sum")  # rank 1 never joins
                try:
                    comm.check_status()
                except pgb.PGBTimeout:
                    raised = True
            torch.cuda.synchronize()
            out["raised"] = raised if rank == 0 else True
        dist.barrier()
        comm.close()
        dist.destroy_process_group()
        q.put((rank, out, None))
    except Exception:
        q.put((rank, None, traceback.format_exc()))


def _run(world: int, case: str):
    import torch.multiprocessing as mp

    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = 29700 + (os.getpid() % 200)
    procs = [ctx.Process(target=_worker, args=(r, world, port, case, q)) for r in range(world)]
    for p in procs:
        p.start()
    results = {}
    try:
        for _ in range(world):
            rank, out, err = q.get(timeout=300)
            assert err is None, f"rank {rank} failed:\n{err}"
            results[rank] = out
    finally:
        for p in procs:
            p.join(timeout=60)
            if p.is_alive():
                p.kill()
    return results


def _worlds():
    n = _ngpus()
    return [w for w in (2, 4, 8) if w <= n] or [2]


@pytest.mark.parametrize("world", _worlds())
def test_known_answers(world):
    if _ngpus() < world:
        pytest.skip(f"needs {world} GPUs")
    res = _run(world, "known_answers")
    for rank, out in res.items():
        bad = [k for k, v in out.items() if not v]
        assert not bad, f"rank {rank}: {bad}"


@pytest.mark.parametrize("world", _worlds())
def test_fused_row_parallel_tp(world):
    if _ngpus() < world:
        pytest.skip(f"needs {world} GPUs")
    res = _run(world, "fused")
    for rank, out in res.items():
        bad = {k: v[1] for k, v in out.items() if not v[0]}
        assert not bad, f"rank {rank}: {bad}"


def test_peer_timeout_is_reported_not_hung():
    if _ngpus() < 2:
        pytest.skip("needs 2 GPUs")
    res = _run(2, "timeout")
    assert res[0]["raised"], "rank 0 did not see a timeout"
