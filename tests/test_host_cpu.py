"""Host-side logic on the CPU: communicator bootstrap over a gloo group of
two ranks, layer shard sizes, and the row-parallel -> RMSNorm fusion wiring.
The device calls are replaced by torch CPU restatements, so no GPU is used."""

from __future__ import annotations

import importlib
import os
import sys
import traceback
from datetime import timedelta
from pathlib import Path

import numpy as np
import pytest
import torch

ROOT = Path(__file__).resolve().parent.parent
GOLD = ROOT / "tests" / "golden"


# --------------------------------------------------- bootstrap over gloo --


def _boot_worker(rank, world, port, q):
    try:
        sys.path.insert(0, str(ROOT))
        import torch.distributed as dist

        D = importlib.import_module("pico-sglang_b200.distributed")
        seen = {}

        class FakeComm:
            def __init__(self, r, w, max_bytes, uid, device=None):
                seen["uid"] = bytes(uid)
                seen["ctor"] = (r, w, max_bytes)
                self.world_size = w

            def export_handle(self):
                return bytes([rank]) * 64

            def open_peers(self, handles):
                seen["handles"] = [h[0] for h in handles]

        D.PGBCommunicator = FakeComm
        D.create_uid = lambda: bytes(range(128))
        dist.init_process_group("gloo", rank=rank, world_size=world,
                                init_method=f"tcp://127.0.0.1:{port}", timeout=timedelta(seconds=60))
        D.init_comm(tp_rank=rank, tp_size=world, tp_cpu_group=dist.group.WORLD, max_size_bytes=123)
        dist.destroy_process_group()
        q.put((rank, seen, None))
    except Exception:
        q.put((rank, None, traceback.format_exc()))


def test_init_comm_bootstrap_gloo_two_ranks():
    import torch.multiprocessing as mp

    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    world, port = 2, 29500 + os.getpid() % 300
    ps = [ctx.Process(target=_boot_worker, args=(r, world, port, q)) for r in range(world)]
    for p in ps:
        p.start()
    got = {}
    for _ in range(world):
        rank, seen, err = q.get(timeout=120)
        assert err is None, err
        got[rank] = seen
    for p in ps:
        p.join(timeout=30)
    # Rank 0's uid reached every rank; handles arrive in rank order.
    assert got[0]["uid"] == got[1]["uid"] == bytes(range(128))
    for r in range(world):
        assert got[r]["ctor"] == (r, world, 123)
        assert got[r]["handles"] == [0, 1]


# ------------------------------------------------------ layer mirrors ----


@pytest.mark.parametrize("n", [1, 2, 4, 8])
def test_layer_shard_sizes_match_reference_formulas(pgb, n):
    D = importlib.import_module("pico-sglang_b200.distributed")
    L = importlib.import_module("pico-sglang_b200.layers")
    H, I, nq, nkv, hd = 4096, 12288, 32, 8, 128
    with D.tp_override(D.DistributedInfo(0, n)):
        qkv = L.LinearColParallelPartitioned(H, hd, [(nq, False), (nkv, True), (nkv, True)], False)
        gu = L.LinearColParallelMerged(H, [I, I], False)
        o = L.LinearRowParallel(nq * hd, H, False)
        down = L.LinearRowParallel(I, H, False)
    assert tuple(qkv.weight.shape) == ((nq // n + 2 * max(nkv // n, 1)) * hd, H)
    assert tuple(gu.weight.shape) == (2 * I // n, H)
    assert tuple(o.weight.shape) == (H, nq * hd // n)
    assert tuple(down.weight.shape) == (H, I // n)
    assert set(o.state_dict()) == {"weight"} and o.bias is None


def test_partitioned_kv_replication_matches_golden_shapes(pgb):
    gold = np.load(GOLD / "tp_small.npz")
    D = importlib.import_module("pico-sglang_b200.distributed")
    L = importlib.import_module("pico-sglang_b200.layers")
    for n in (1, 2, 4):
        with D.tp_override(D.DistributedInfo(0, n)):
            qkv = L.LinearColParallelPartitioned(256, 32, [(8, False), (2, True), (2, True)], False)
        assert tuple(qkv.weight.shape) == gold[f"qkv_w_tp{n}_r0"].shape


# ---------------------------------------------------- fusion wiring ------


class _Recorder:
    """CPU restatements of the libpgb ops, recording every call."""

    def __init__(self):
        self.calls = []

    def col_gemm(self, x, w, bias=None, out=None):
        self.calls.append("col")
        y = (x.float() @ w.float().t()).to(x.dtype)
        return y

    def row_gemm_allreduce_addnorm(self, comm, x, w, residual, norm_w, eps, out=None, bias=None):
        self.calls.append("row_fused" if norm_w is not None else "row")
        y = (x.float() @ w.float().t()).to(x.dtype)
        if norm_w is None:
            return y
        s = y.float() + residual.float()
        residual.copy_(s.to(x.dtype))
        return (s * torch.rsqrt(s.pow(2).mean(-1, keepdim=True) + eps) * norm_w.float()).to(x.dtype)

    def fused_add_rmsnorm(self, x, residual, w, eps):
        self.calls.append("addnorm")
        s = x.float() + residual.float()
        residual.copy_(s.to(x.dtype))
        x.copy_((s * torch.rsqrt(s.pow(2).mean(-1, keepdim=True) + eps) * w.float()).to(x.dtype))

    def rmsnorm(self, x, w, eps, out=None):
        self.calls.append("rmsnorm")
        return (x.float() * torch.rsqrt(x.float().pow(2).mean(-1, keepdim=True) + eps) * w.float()).to(x.dtype)


class _Obj:
    pass


def _decoder(L, n_layers, H, I, g):
    layers = []
    for _ in range(n_layers):
        lay = _Obj()
        lay.input_layernorm = L.RMSNormFused(H, 1e-6)
        lay.post_attention_layernorm = L.RMSNormFused(H, 1e-6)
        lay.self_attn = _Obj()
        lay.self_attn.o_proj = L.LinearRowParallel(H, H, False)
        lay.mlp = _Obj()
        lay.mlp.down_proj = L.LinearRowParallel(I, H, False)
        for op in (lay.self_attn.o_proj, lay.mlp.down_proj):
            op.weight = torch.randn(op.weight.shape, generator=g) * 0.05
        for nm in (lay.input_layernorm, lay.post_attention_layernorm):
            nm.weight = 1 + 0.1 * torch.randn(H, generator=g)
        layers.append(lay)
    final = L.RMSNormFused(H, 1e-6)
    final.weight = torch.ones(H)
    return layers, final


def _forward(layers, final, x, a_list, m_list):
    """models/llama.py:77-86 and :103-108 with attention / act replaced by fixed inputs."""
    residual = None
    for lay, a, m in zip(layers, a_list, m_list):
        x, residual = lay.input_layernorm.forward(x, residual)
        x = lay.self_attn.o_proj.forward(a + 0 * x[:, : a.shape[1]].sum())
        x, residual = lay.post_attention_layernorm.forward(x, residual)
        x = lay.mlp.down_proj.forward(m + 0 * x[:, : 1].sum())
    x, _ = final.forward(x, residual)
    return x


def test_linked_row_layers_fuse_and_match_unfused(pgb, monkeypatch):
    D = importlib.import_module("pico-sglang_b200.distributed")
    L = importlib.import_module("pico-sglang_b200.layers")
    rec = _Recorder()
    for name in ("col_gemm", "row_gemm_allreduce_addnorm", "fused_add_rmsnorm", "rmsnorm"):
        monkeypatch.setattr(L.ops, name, getattr(rec, name))
    monkeypatch.setattr(L, "local_comm", lambda *a, **k: object())
    g = torch.Generator().manual_seed(0)
    H, I, T = 64, 128, 5
    with D.tp_override(D.DistributedInfo(0, 1)):
        layers, final = _decoder(L, 3, H, I, g)
    x = torch.randn(T, H, generator=g)
    a_list = [torch.randn(T, H, generator=g) for _ in layers]
    m_list = [torch.randn(T, I, generator=g) for _ in layers]

    L.reset_fusion_context()
    ref = _forward(layers, final, x.clone(), a_list, m_list)
    unfused_calls = list(rec.calls)
    assert "row_fused" not in unfused_calls

    assert L.link_fused_norms(layers, final) == 2 * len(layers)
    rec.calls.clear()
    L.reset_fusion_context()
    out = _forward(layers, final, x.clone(), a_list, m_list)
    # First input_layernorm is a plain rmsnorm; every other norm is fused into
    # the row-parallel layer that produces its input.
    assert rec.calls == ["rmsnorm"] + ["row_fused"] * (2 * len(layers))
    torch.testing.assert_close(out, ref, rtol=1e-5, atol=1e-5)


def test_attention_and_mlp_mirrors_match_reference_shapes():
    """RotaryAttention / GatedMLP mirrors: the reference's state-dict keys and
    shard shapes at TP 1/2/4/8 (kv-head replication and attention bias
    included), recorded from the reference by tests/golden/make_golden.py."""
    import json

    L = importlib.import_module("pico-sglang_b200.layers")
    D = importlib.import_module("pico-sglang_b200.distributed")
    gold = json.loads((Path(__file__).resolve().parent / "golden" / "layer_shapes.json").read_text())
    for name, c in gold["cases"].items():
        for n in (1, 2, 4, 8):
            ref = gold["shapes"][f"{name}_tp{n}"]
            with D.tp_override(D.DistributedInfo(0, n)):
                attn = L.RotaryAttention(c["hidden"], c["head_dim"], c["nq"], c["nkv"], 0, c["head_dim"], 256, 1e6,
                                         None, has_attn_bias=c["bias"])
                mlp = L.GatedMLP(c["hidden"], c["inter"], "silu")
            assert {k: list(v.shape) for k, v in attn.state_dict().items()} == ref["attn"], (name, n)
            assert {k: list(v.shape) for k, v in mlp.state_dict().items()} == ref["mlp"], (name, n)
            assert [attn.num_qo_heads, attn.num_kv_heads] == ref["attn_local_heads"]


def test_gated_mlp_and_attention_refuse_unfused_variants():
    L = importlib.import_module("pico-sglang_b200.layers")
    D = importlib.import_module("pico-sglang_b200.distributed")
    with D.tp_override(D.DistributedInfo(0, 1)):
        with pytest.raises(NotImplementedError):
            L.GatedMLP(64, 128, "gelu")
        with pytest.raises(ValueError):
            L.GatedMLP(64, 128, "relu")
        with pytest.raises(NotImplementedError):
            L.RotaryAttention(256, 64, 4, 1, 0, 64, 32, 1e4, None, qk_norm_eps=1e-6)
