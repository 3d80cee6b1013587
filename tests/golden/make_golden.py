"""Generate the golden fixtures in this directory from the reference itself.

Runs only where the reference's Python sources are present: it imports them
read-only from the directory that PICOSGL_SRC names (the reference project's
`python/` directory). The fixtures it writes are committed, so the tests never
need the reference.

    PICOSGL_SRC=<reference checkout>/python python tests/golden/make_golden.py

What it records:
  cfg1.npz   BASELINE config 1 (CPU plumbing): the reference's
             LinearRowParallel (python/picosgl/layers/linear.py:76-97) at
             world_size 2 over a gloo process group plugged into
             DistributedCommunicator.impl (the pattern of
             tests/mtp/test_tp2_numeric.py:72-88), f32, weights sharded by the
             reference's own _shard_tensor (models/weight.py:41-78). Inputs
             are regenerated from torch.manual_seed(0) in the order
             x, W, residual (documented in the `meta` entry), so only
             outputs are stored. The RMSNorm step runs FlashInfer on a GPU
             in the reference; here it is a torch restatement of the same
             kernel (norm.cuh:387-470), stored separately as `out_restated`.
  tp_small.npz  bf16 and f32 row-parallel results at TP 1/2/4 and the
             column-parallel merged / partitioned shards (with kv-head
             replication) produced by the reference's layers and loader.
  mlp_small.npz  the reference's GatedMLP (python/picosgl/layers/mlp.py:17-48)
             at TP 1/2, bf16 and f32: the gate_up tensor its forward hands to
             act_fn and the activation's output. act_fn is silu_and_mul,
             which runs FlashInfer on a GPU in the reference; here it is a
             torch restatement of FlashInfer's act_and_mul kernel
             (include/flashinfer/activation.cuh, silu from
             flashinfer/jit/activation.py), checked against
             torch.nn.functional.silu before it is used.
  layer_shapes.json  state-dict keys and shard shapes of the reference's
             GatedMLP and RotaryAttention (config 2, TP 1/2/4/8, and a qwen-style
             bias + kv-replication case), so the mirrors' drop-in shapes are
             checked without the reference.
  rope_small.npz  the reference's RoPE cos/sin tables (get_rope,
             python/picosgl/layers/rotary.py:63-151) for default, partial
             (rotary_dim < head_dim), llama3 and yarn scaling. Applying them
             needs FlashInfer on a GPU (rotary.py:48-59), so only the tables
             are recorded here.
"""

from __future__ import annotations

import os
import sys
from pathlib import Path

import numpy as np
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

HERE = Path(__file__).resolve().parent
REF = os.environ.get("PICOSGL_SRC", "")


def _ref_imports():
    if not REF:
        raise SystemExit("set PICOSGL_SRC to the reference project's python/ directory")
    if REF not in sys.path:
        sys.path.insert(0, REF)
    import picosgl.distributed.info as info  # noqa: F401
    from picosgl.distributed import DistributedInfo, set_tp_info
    from picosgl.distributed.impl import DistributedCommunicator, DistributedImpl
    from picosgl.layers.linear import (
        LinearColParallelMerged,
        LinearColParallelPartitioned,
        LinearRowParallel,
    )
    from picosgl.models.weight import _shard_tensor

    return (info, DistributedInfo, set_tp_info, DistributedCommunicator, DistributedImpl,
            LinearRowParallel, LinearColParallelMerged, LinearColParallelPartitioned, _shard_tensor)


def _reset_tp(info, DistributedInfo, set_tp_info, rank, size):
    info._TP_INFO = None
    set_tp_info(DistributedInfo(rank=rank, size=size))


def _torch_fused_add_rmsnorm(x, residual, w, eps):
    """Restatement of FlashInfer FusedAddRMSNormKernel (norm.cuh:387-470) in torch."""
    s = x.float() + residual.float()
    res = s.to(x.dtype)
    rcp = torch.rsqrt(s.pow(2).mean(-1, keepdim=True) + eps)
    return (s * rcp * w.float()).to(x.dtype), res


def cfg1_inputs():
    torch.manual_seed(0)
    x = torch.randn(64, 4096)
    W = torch.randn(4096, 4096) * 0.02
    residual = torch.randn(64, 4096)
    return x, W, residual


def _cfg1_worker(rank, world, port, q):
    (info, DistributedInfo, set_tp_info, DistributedCommunicator, DistributedImpl,
     LinearRowParallel, _, _, _shard_tensor) = _ref_imports()
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)

    class GlooImpl(DistributedImpl):
        def all_reduce(self, x):
            dist.all_reduce(x)
            return x

        def all_gather(self, x):
            out = [torch.empty_like(x) for _ in range(world)]
            dist.all_gather(out, x)
            return torch.cat(out, 0)

    _reset_tp(info, DistributedInfo, set_tp_info, rank, world)
    x, W, residual = cfg1_inputs()
    layer = LinearRowParallel(4096, 4096, has_bias=False)
    layer.weight = _shard_tensor("model.layers.0.self_attn.o_proj.weight", W, rank, world, 8)
    DistributedCommunicator.impl = GlooImpl()
    y = layer.forward(x.chunk(world, dim=1)[rank].contiguous())
    out, res = _torch_fused_add_rmsnorm(y.clone(), residual.clone(), torch.ones(4096), 1e-6)
    if rank == 0:
        q.put((y.numpy().copy(), out.numpy().copy(), res.numpy().copy()))
    dist.barrier()
    dist.destroy_process_group()


def make_cfg1():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = 29611
    procs = [ctx.Process(target=_cfg1_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    y, out, res = q.get(timeout=600)
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0, "cfg1 worker failed"
    np.savez_compressed(
        HERE / "cfg1.npz",
        y=y,
        out_restated=out,
        residual_out=res,
        meta=np.array(
            "torch.manual_seed(0); x=randn(64,4096); W=randn(4096,4096)*0.02; "
            "residual=randn(64,4096); f32; world_size=2 gloo; eps=1e-6; norm weight ones"
        ),
    )


def make_tp_small():
    (info, DistributedInfo, set_tp_info, DistributedCommunicator, DistributedImpl,
     LinearRowParallel, LinearColParallelMerged, LinearColParallelPartitioned,
     _shard_tensor) = _ref_imports()

    class RecordingImpl(DistributedImpl):
        """Returns the row-parallel partial unchanged, as tests/mtp/test_tp2_numeric.py:72-88."""

        def __init__(self):
            self.records = []

        def all_reduce(self, x):
            self.records.append(x.detach().clone())
            return x

        def all_gather(self, x):
            raise AssertionError("not used")

    g = torch.Generator().manual_seed(42)
    H, I, T = 256, 512, 8
    nq, nkv, hd = 8, 2, 32
    data = {}
    x_h = torch.randn(T, H, generator=g)
    x_i = torch.randn(T, I, generator=g)
    w_down = torch.randn(H, I, generator=g) * 0.02
    w_gate = torch.randn(I, H, generator=g) * 0.02
    w_up = torch.randn(I, H, generator=g) * 0.02
    wq = torch.randn(nq * hd, H, generator=g) * 0.02
    wk = torch.randn(nkv * hd, H, generator=g) * 0.02
    wv = torch.randn(nkv * hd, H, generator=g) * 0.02
    for k, v in dict(x_h=x_h, x_i=x_i, w_down=w_down, w_gate=w_gate, w_up=w_up, wq=wq, wk=wk,
                     wv=wv).items():
        data[k] = v.numpy()
    for dt_name, dt in (("f32", torch.float32), ("bf16", torch.bfloat16)):
        for n in (1, 2, 4):
            for r in range(n):
                _reset_tp(info, DistributedInfo, set_tp_info, r, n)
                rec = RecordingImpl()
                DistributedCommunicator.impl = rec
                down = LinearRowParallel(I, H, has_bias=False)
                down.weight = _shard_tensor("m.down_proj.weight", w_down, r, n, nkv).to(dt)
                p = down.forward(x_i.chunk(n, 1)[r].contiguous().to(dt))
                assert len(rec.records) == (1 if n > 1 else 0)
                data[f"row_{dt_name}_tp{n}_r{r}"] = p.float().numpy()

                gu = LinearColParallelMerged(H, [I, I], has_bias=False)
                parts = [_shard_tensor("m.gate_proj.weight", w_gate, r, n, nkv),
                         _shard_tensor("m.up_proj.weight", w_up, r, n, nkv)]
                gu.weight = torch.cat(parts, 0).to(dt)
                assert tuple(gu.weight.shape) == (2 * I // n, H)
                if dt_name == "f32":
                    data[f"gateup_w_tp{n}_r{r}"] = gu.weight.numpy()
                data[f"gateup_{dt_name}_tp{n}_r{r}"] = gu.forward(x_h.to(dt)).float().numpy()

                qkv = LinearColParallelPartitioned(H, hd, [(nq, False), (nkv, True), (nkv, True)],
                                                   has_bias=False)
                parts = [_shard_tensor("a.q_proj.weight", wq, r, n, nkv),
                         _shard_tensor("a.k_proj.weight", wk, r, n, nkv),
                         _shard_tensor("a.v_proj.weight", wv, r, n, nkv)]
                w_local = torch.cat(parts, 0)
                assert tuple(w_local.shape) == tuple(qkv.weight.shape), (w_local.shape, qkv.weight.shape)
                qkv.weight = w_local.to(dt)
                if dt_name == "f32":
                    data[f"qkv_w_tp{n}_r{r}"] = qkv.weight.numpy()
                data[f"qkv_{dt_name}_tp{n}_r{r}"] = qkv.forward(x_h.to(dt)).float().numpy()
    data["meta"] = np.array(f"H={H} I={I} T={T} nq={nq} nkv={nkv} hd={hd} seed=42")
    np.savez_compressed(HERE / "tp_small.npz", **data)


def _torch_silu_and_mul(gate_up):
    """Restatement of FlashInfer's act_and_mul kernel with silu: g / (1 + exp(-g)) * u in f32,
    cast once to the input dtype."""
    i = gate_up.shape[-1] // 2
    g, u = gate_up[..., :i].float(), gate_up[..., i:].float()
    return (g / (1.0 + torch.exp(-g)) * u).to(gate_up.dtype)


def make_mlp_small():
    (info, DistributedInfo, set_tp_info, DistributedCommunicator, DistributedImpl,
     _, _, _, _shard_tensor) = _ref_imports()
    from picosgl.layers.mlp import GatedMLP

    class PassImpl(DistributedImpl):
        def all_reduce(self, x):
            return x

        def all_gather(self, x):
            raise AssertionError("not used")

    g = torch.Generator().manual_seed(77)
    H, I, T = 128, 192, 6
    x = torch.randn(T, H, generator=g)
    w_gate = torch.randn(I, H, generator=g) * 0.2
    w_up = torch.randn(I, H, generator=g) * 0.1
    w_down = torch.randn(H, I, generator=g) * 0.05
    data = dict(x=x.numpy(), w_gate=w_gate.numpy(), w_up=w_up.numpy())
    probe = torch.linspace(-30, 30, 2001)
    ref = torch.nn.functional.silu(probe)
    got = _torch_silu_and_mul(torch.cat([probe, torch.ones_like(probe)])[None])[0]
    assert torch.allclose(got, ref, rtol=1e-6, atol=1e-7)
    DistributedCommunicator.impl = PassImpl()
    for dt_name, dt in (("f32", torch.float32), ("bf16", torch.bfloat16)):
        for n in (1, 2):
            for r in range(n):
                _reset_tp(info, DistributedInfo, set_tp_info, r, n)
                mlp = GatedMLP(H, I, "silu")
                mlp.gate_up_proj.weight = torch.cat(
                    [_shard_tensor("m.gate_proj.weight", w_gate, r, n, 1),
                     _shard_tensor("m.up_proj.weight", w_up, r, n, 1)], 0).to(dt)
                mlp.down_proj.weight = _shard_tensor("m.down_proj.weight", w_down, r, n, 1).to(dt)
                seen = {}

                def act(gate_up, out=None, seen=seen):
                    seen["gate_up"] = gate_up.clone()
                    seen["act"] = _torch_silu_and_mul(gate_up)
                    return seen["act"]

                mlp.act_fn = act
                mlp.forward(x.to(dt))
                data[f"gateup_{dt_name}_tp{n}_r{r}"] = seen["gate_up"].float().numpy()
                data[f"act_{dt_name}_tp{n}_r{r}"] = seen["act"].float().numpy()
    data["meta"] = np.array(f"H={H} I={I} T={T} seed=77 gate*0.2 up*0.1 down*0.05")
    np.savez_compressed(HERE / "mlp_small.npz", **data)


ROPE_CASES = {
    "default_hd128": (128, 128, 96, 1e6, None),
    "partial_hd128_rd64": (128, 64, 96, 1e4, None),
    "default_hd64": (64, 64, 96, 1e4, None),
    "llama3": (128, 128, 96, 5e5, (("rope_type", "llama3"), ("factor", 8.0), ("low_freq_factor", 1.0),
                                   ("high_freq_factor", 4.0), ("original_max_position_embeddings", 64))),
    "yarn": (128, 128, 96, 1e6, (("rope_type", "yarn"), ("factor", 4.0),
                                 ("original_max_position_embeddings", 64))),
}


def make_rope_small():
    _ref_imports()
    from picosgl.layers.rotary import get_rope

    data = {}
    for name, (hd, rd, max_pos, base, scaling) in ROPE_CASES.items():
        data[name] = get_rope(hd, rd, max_pos, base, scaling)._cos_sin_cache.numpy().copy()
    data["meta"] = np.array(repr(ROPE_CASES))
    np.savez_compressed(HERE / "rope_small.npz", **data)


LAYER_CASES = {
    "config2": dict(hidden=4096, inter=12288, head_dim=128, nq=32, nkv=8, bias=False),
    "bias_kv2": dict(hidden=2048, inter=5632, head_dim=64, nq=16, nkv=2, bias=True),
}


def make_layer_shapes():
    import json

    (info, DistributedInfo, set_tp_info, _, _, _, _, _, _) = _ref_imports()
    from picosgl.layers.attention import RotaryAttention
    from picosgl.layers.mlp import GatedMLP

    out = {}
    for name, c in LAYER_CASES.items():
        for n in (1, 2, 4, 8):
            _reset_tp(info, DistributedInfo, set_tp_info, 0, n)
            attn = RotaryAttention(c["hidden"], c["head_dim"], c["nq"], c["nkv"], 0, c["head_dim"], 256, 1e6, None,
                                   has_attn_bias=c["bias"])
            mlp = GatedMLP(c["hidden"], c["inter"], "silu")
            out[f"{name}_tp{n}"] = {
                "attn": {k: list(v.shape) for k, v in attn.state_dict().items()},
                "mlp": {k: list(v.shape) for k, v in mlp.state_dict().items()},
                "attn_local_heads": [attn.num_qo_heads, attn.num_kv_heads],
            }
    (HERE / "layer_shapes.json").write_text(json.dumps({"cases": LAYER_CASES, "shapes": out}, indent=1))


if __name__ == "__main__":
    torch.set_num_threads(4)
    make_tp_small()
    make_mlp_small()
    make_rope_small()
    make_layer_shapes()
    make_cfg1()
    print("wrote", sorted(p.name for p in HERE.glob("*.npz")))
