"""Pin the CPU oracle (oracle/) before trusting it.

1. Against golden vectors produced by the reference's own Python layers
   (tests/golden/make_golden.py): BASELINE config 1 at world_size 2 over
   gloo, and TP 1/2/4 shards of the row- and column-parallel layers.
2. Against the known answers of the reference communicator test
   (tests/distributed/test_pynccl.py:95-148).
3. Against properties of RMSNorm the reference relies on.
"""

from __future__ import annotations

from pathlib import Path

import numpy as np
import pytest
import torch

import oracle

GOLD = Path(__file__).resolve().parent / "golden"


@pytest.fixture(scope="module")
def tp_small():
    return dict(np.load(GOLD / "tp_small.npz"))


def test_round_to_bf16_matches_torch():
    g = torch.Generator().manual_seed(3)
    a = torch.randn(10000, generator=g) * 100
    a[:5] = torch.tensor([0.0, -0.0, 1e-40, 3.0e38, float("inf")])
    ref = a.to(torch.bfloat16).float().numpy()
    got = oracle.round_to(a.numpy(), "bf16")
    assert np.array_equal(got, ref)
    ref16 = a.clamp(-6e4, 6e4).half().float().numpy()
    assert np.array_equal(oracle.round_to(a.clamp(-6e4, 6e4).numpy(), "f16"), ref16)


def test_cfg1_row_parallel_matches_reference_gloo():
    """Config 1: reference LinearRowParallel, world_size 2, gloo all_reduce, f32."""
    gold = np.load(GOLD / "cfg1.npz")
    torch.manual_seed(0)
    x = torch.randn(64, 4096).numpy()
    W = (torch.randn(4096, 4096) * 0.02).numpy()
    residual = torch.randn(64, 4096).numpy()
    out, res, y = oracle.row_parallel_addnorm(x, W, residual, np.ones(4096, np.float32), 1e-6, n=2,
                                              dtype="f32")
    rel = np.abs(y - gold["y"]).max() / np.abs(gold["y"]).max()
    assert rel < 1e-5, rel
    rel = np.abs(out - gold["out_restated"]).max() / np.abs(gold["out_restated"]).max()
    assert rel < 1e-5, rel
    assert np.abs(res - gold["residual_out"]).max() / np.abs(gold["residual_out"]).max() < 1e-5


@pytest.mark.parametrize("n", [1, 2, 4])
def test_row_parallel_partials_match_reference(tp_small, n):
    x = tp_small["x_i"]
    w = tp_small["w_down"]
    for r in range(n):
        w_r, x_r = oracle.row_shard(w, x, r, n)
        got32 = oracle.linear(x_r, w_r, dtype="f32")
        ref32 = tp_small[f"row_f32_tp{n}_r{r}"]
        assert np.abs(got32 - ref32).max() <= 1e-5 * np.abs(ref32).max()
        xb, wb = oracle.round_to(x_r, "bf16"), oracle.round_to(w_r, "bf16")
        gotb = oracle.linear(xb, wb, dtype="bf16")
        refb = tp_small[f"row_bf16_tp{n}_r{r}"]
        # Both round one f32-class accumulation to bf16: at most one ulp apart.
        assert np.abs(gotb - refb).max() <= 2 ** -7 * np.abs(refb).max()
    # TP partial sums reproduce TP=1 (tests/mtp/test_tp2_numeric.py:175-188 bar: 1e-3).
    full = tp_small["row_f32_tp1_r0"]
    summed = oracle.all_reduce_sum([tp_small[f"row_f32_tp{n}_r{r}"] for r in range(n)], "f32")
    err = np.abs(summed - full).max()
    assert err < 1e-3 and err / np.abs(full).max() < 1e-3


@pytest.mark.parametrize("n", [1, 2, 4])
def test_column_parallel_shards_match_reference_loader(tp_small, n):
    for r in range(n):
        w_gu = oracle.col_shard_merged([tp_small["w_gate"], tp_small["w_up"]], r, n)
        assert np.array_equal(w_gu, tp_small[f"gateup_w_tp{n}_r{r}"])
        w_qkv = oracle.col_shard_partitioned(tp_small["wq"], tp_small["wk"], tp_small["wv"],
                                             num_kv_heads=2, rank=r, n=n)
        assert np.array_equal(w_qkv, tp_small[f"qkv_w_tp{n}_r{r}"])
        y = oracle.linear(tp_small["x_h"], w_gu, dtype="f32")
        ref = tp_small[f"gateup_f32_tp{n}_r{r}"]
        assert np.abs(y - ref).max() <= 1e-5 * np.abs(ref).max()
        y = oracle.linear(tp_small["x_h"], w_qkv, dtype="f32")
        ref = tp_small[f"qkv_f32_tp{n}_r{r}"]
        assert np.abs(y - ref).max() <= 1e-5 * np.abs(ref).max()


@pytest.mark.parametrize("tp", [2, 4, 8])
def test_all_reduce_known_answers(tp):
    """tests/distributed/test_pynccl.py:95-134, restated for the oracle."""
    K = 512
    x = np.ones(8192 * K // 64, np.float32)
    for _ in range(4):
        x = oracle.all_reduce_sum([x] * tp, "f16")
    assert np.all(x == tp ** 4)
    x = oracle.all_reduce_sum([np.full(1024, r, np.float32) for r in range(tp)], "f16")
    assert np.all(x == tp * (tp - 1) // 2)
    half = np.concatenate([np.zeros(512, np.float32), np.ones(512, np.float32)])
    x = oracle.all_reduce_sum([half] * tp, "f16")
    assert np.all(x[:512] == 0) and np.all(x[512:] == tp)


def test_fused_add_rmsnorm_properties():
    g = np.random.default_rng(5)
    x = g.standard_normal((16, 512)).astype(np.float32)
    r = g.standard_normal((16, 512)).astype(np.float32)
    w = np.ones(512, np.float32)
    out, res = oracle.fused_add_rmsnorm(x, r, w, 1e-6, "f32")
    np.testing.assert_allclose(res, x + r, rtol=0, atol=0)
    np.testing.assert_allclose(np.sqrt((out.astype(np.float64) ** 2).mean(-1)), 1.0, rtol=1e-5)
    # Scale invariance of RMSNorm (eps negligible).
    out2, _ = oracle.fused_add_rmsnorm(4 * x, 4 * r, w, 1e-12, "f32")
    np.testing.assert_allclose(out2, out, rtol=1e-5, atol=1e-6)
    # bf16 mode: residual is the rounded f32 sum; the norm uses the unrounded sum.
    outb, resb = oracle.fused_add_rmsnorm(oracle.round_to(x, "bf16"), oracle.round_to(r, "bf16"),
                                          w, 1e-6, "bf16")
    s = oracle.round_to(x, "bf16") + oracle.round_to(r, "bf16")
    assert np.array_equal(resb, oracle.round_to(s, "bf16"))
    # rmsnorm without residual
    o = oracle.rmsnorm(x, w, 1e-6, "f32")
    np.testing.assert_allclose(np.sqrt((o.astype(np.float64) ** 2).mean(-1)), 1.0, rtol=1e-5)


def test_tp_layer_step_sharded_equals_unsharded():
    """Row-parallel sums over n ranks reproduce the TP=1 layer (f32 mode)."""
    g = np.random.default_rng(9)
    H, I, T = 128, 256, 4
    wts = {
        "qkv": g.standard_normal((192, H)).astype(np.float32) * 0.02,
        "o": g.standard_normal((H, H)).astype(np.float32) * 0.02,
        "gate_up": g.standard_normal((2 * I, H)).astype(np.float32) * 0.02,
        "down": g.standard_normal((H, I)).astype(np.float32) * 0.02,
        "ln1": np.ones(H, np.float32),
        "ln2": np.ones(H, np.float32),
    }
    h, a = (g.standard_normal((T, H)).astype(np.float32) for _ in range(2))
    m = g.standard_normal((T, I)).astype(np.float32)
    res = g.standard_normal((T, H)).astype(np.float32)
    one = oracle.tp_layer_step(h, a, m, res, wts, 1e-6, n=1, dtype="f32")
    four = oracle.tp_layer_step(h, a, m, res, wts, 1e-6, n=4, rank=2, dtype="f32")
    for k in ("x1", "r1", "x2", "r2"):
        np.testing.assert_allclose(four[k], one[k], rtol=1e-5, atol=1e-5)


@pytest.fixture(scope="module")
def mlp_small():
    return dict(np.load(GOLD / "mlp_small.npz"))


@pytest.mark.parametrize("n", [1, 2])
@pytest.mark.parametrize("dt", ["f32", "bf16"])
def test_gated_mlp_activation_matches_reference(mlp_small, n, dt):
    """The reference GatedMLP's gate_up (its merged shards) and its act_fn
    output (mlp.py:43-46), recorded by tests/golden/make_golden.py."""
    for r in range(n):
        w_gu = oracle.col_shard_merged([mlp_small["w_gate"], mlp_small["w_up"]], r, n)
        gu_ref = mlp_small[f"gateup_{dt}_tp{n}_r{r}"]
        gu = oracle.linear(oracle.round_to(mlp_small["x"], dt), oracle.round_to(w_gu, dt), dtype=dt)
        if dt == "f32":
            assert np.abs(gu - gu_ref).max() <= 1e-5 * np.abs(gu_ref).max()
        else:
            # torch's CPU bf16 matmul rounds an f32 accumulation: at most one ulp apart.
            ulp = 2.0 ** (np.floor(np.log2(np.maximum(np.abs(gu_ref), 1e-30))) - 7)
            assert np.all(np.abs(gu - gu_ref) <= ulp)
        act = oracle.silu_and_mul(gu_ref, dt)
        act_ref = mlp_small[f"act_{dt}_tp{n}_r{r}"]
        assert act.shape == (gu_ref.shape[0], gu_ref.shape[1] // 2)
        if dt == "f32":
            assert np.abs(act - act_ref).max() <= 1e-6 * np.abs(act_ref).max()
        else:
            ulp = 2.0 ** (np.floor(np.log2(np.maximum(np.abs(act_ref), 1e-30))) - 7)
            assert np.all(np.abs(act - act_ref) <= ulp)
            assert np.mean(act != act_ref) < 0.01


def test_silu_and_mul_against_torch_silu():
    """Independent pin: torch.nn.functional.silu times the up half, and the
    limits silu(0) = 0, silu(x) -> x for large x, -> 0 for very negative x."""
    x = np.linspace(-90, 90, 4001, dtype=np.float32)
    gu = np.concatenate([x, np.ones_like(x)])[None]
    got = oracle.silu_and_mul(gu, "f32")[0]
    ref = torch.nn.functional.silu(torch.from_numpy(x)).numpy()
    assert np.allclose(got, ref, rtol=2e-6, atol=1e-30)
    edge = oracle.silu_and_mul(np.array([[0.0, 50.0, -200.0, 2.0, 3.0, 4.0]], np.float32), "f32")[0]
    assert edge[0] == 0.0 and abs(edge[1] - 150.0) < 1e-4 and edge[2] == 0.0


def test_gate_up_silu_ragged_and_empty():
    rng = np.random.default_rng(5)
    x = rng.standard_normal((3, 24)).astype(np.float32)
    w = (rng.standard_normal((2 * 5, 24)) * 0.1).astype(np.float32)
    y = oracle.gate_up_silu(x, w, dtype="f32")
    gu = x.astype(np.float64) @ w.T.astype(np.float64)
    ref = gu[:, :5] / (1 + np.exp(-gu[:, :5])) * gu[:, 5:]
    assert np.allclose(y, ref, rtol=1e-5, atol=1e-6)
    assert oracle.gate_up_silu(x[:0], w, dtype="bf16").shape == (0, 5)


@pytest.fixture(scope="module")
def rope_small():
    return dict(np.load(GOLD / "rope_small.npz"))


ROPE_CASES = {
    "default_hd128": (128, 128, 96, 1e6, None),
    "partial_hd128_rd64": (128, 64, 96, 1e4, None),
    "default_hd64": (64, 64, 96, 1e4, None),
    "llama3": (128, 128, 96, 5e5, (("rope_type", "llama3"), ("factor", 8.0), ("low_freq_factor", 1.0),
                                   ("high_freq_factor", 4.0), ("original_max_position_embeddings", 64))),
    "yarn": (128, 128, 96, 1e6, (("rope_type", "yarn"), ("factor", 4.0),
                                 ("original_max_position_embeddings", 64))),
}


@pytest.mark.parametrize("name", sorted(ROPE_CASES))
def test_rope_table_matches_reference(rope_small, name):
    """The layer mirror's cos/sin table (what the kernels read) is bit-identical
    to the reference's get_rope table (python/picosgl/layers/rotary.py:63-151)."""
    import importlib

    L = importlib.import_module("pico-sglang_b200.layers")
    hd, rd, mp, base, sc = ROPE_CASES[name]
    assert np.array_equal(L.get_rope(hd, rd, mp, base, sc)._cos_sin_cache.numpy(), rope_small[name])


def test_rope_oracle_properties(rope_small):
    """NeoX RoPE: position 0 is the identity; each (i, i + rd/2) pair keeps its
    norm; dims from rd on are untouched; rotating by p then reading the pair
    as a complex number equals multiplying by exp(i * angle) (f32 tolerance)."""
    table = rope_small["partial_hd128_rd64"]
    hd, rd = 128, 64
    rng = np.random.default_rng(3)
    x = rng.standard_normal((5, 2 * hd)).astype(np.float32)
    pos = np.array([0, 1, 7, 50, 95])
    y = oracle.apply_rope_neox(x, pos, table, hd, "f32")
    assert np.array_equal(y[0], x[0])
    xh, yh = x.reshape(5, 2, hd), y.reshape(5, 2, hd)
    assert np.array_equal(yh[..., rd:], xh[..., rd:])
    n_in = xh[..., : rd // 2] ** 2 + xh[..., rd // 2: rd] ** 2
    n_out = yh[..., : rd // 2] ** 2 + yh[..., rd // 2: rd] ** 2
    assert np.allclose(n_in, n_out, rtol=1e-5, atol=1e-6)
    z = (xh[..., : rd // 2] + 1j * xh[..., rd // 2: rd]).astype(np.complex128)
    ang = np.arctan2(table[pos, rd // 2:], table[pos, : rd // 2])[:, None, :]
    zr = z * np.exp(1j * ang)
    assert np.allclose(yh[..., : rd // 2], zr.real, atol=2e-5) and np.allclose(yh[..., rd // 2: rd], zr.imag, atol=2e-5)


def test_qkv_rope_store_oracle_scatters_rows():
    rng = np.random.default_rng(4)
    T, K, nq, nkv, hd = 3, 32, 2, 1, 64
    x = rng.standard_normal((T, K)).astype(np.float32)
    w = (rng.standard_normal(((nq + 2 * nkv) * hd, K)) * 0.1).astype(np.float32)
    table = np.concatenate([np.ones((8, 32)), np.zeros((8, 32))], 1).astype(np.float32)  # identity rotation
    kc = np.full((10, nkv, hd), 7.0, np.float32)
    vc = np.full((10, nkv, hd), 7.0, np.float32)
    q, kc2, vc2 = oracle.qkv_rope_store(x, w, None, [1, 2, 3], [9, 0, 4], table, nq, nkv, hd, kc, vc, "f32")
    qkv = oracle.linear(x, w, dtype="f32")
    assert np.array_equal(q, qkv[:, : nq * hd])
    assert np.array_equal(kc2[[9, 0, 4]].reshape(T, -1), qkv[:, nq * hd: (nq + nkv) * hd])
    assert np.array_equal(vc2[[9, 0, 4]].reshape(T, -1), qkv[:, (nq + nkv) * hd:])
    untouched = [i for i in range(10) if i not in (9, 0, 4)]
    assert np.all(kc2[untouched] == 7.0) and np.all(vc2[untouched] == 7.0)
