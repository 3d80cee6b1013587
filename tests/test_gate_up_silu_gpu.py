"""gate_up_proj GEMM with silu_and_mul in its epilogue, and the standalone activation.

The reference's GatedMLP.forward (python/picosgl/layers/mlp.py:43-48) runs
gate_up_proj (F.linear into a [T, 2I] bf16 tensor) and then silu_and_mul
(python/picosgl/layers/activation.py:9-12 -> flashinfer.silu_and_mul).
pgb_gate_up_silu does both in one kernel. Checked against
  - the CPU oracle (oracle.gate_up_silu) at sizes it finishes in seconds,
  - a plain torch f32 restatement over cuBLAS's bf16 gate_up at model sizes,
  - the reference's own library calls (F.linear + flashinfer.silu_and_mul).
Tolerance. The activation is computed from gate_up rounded to bf16, as the
reference materialises it; two GEMMs that sum in different orders round some
gate_up values to neighbouring bf16 numbers, and silu(g) * u turns one such
flip into |silu'(g) u| ulp(g) or |silu(g)| ulp(u) of output (several output
ulps where |u| is large). The bound per element is therefore
max(2e-2 * RMS, 1 output ulp) -- the bf16 bar of the column-GEMM tests --
plus the effect of one bf16 ulp in g and in u, evaluated on the reference's
own gate_up. The f32 check mode holds 1e-5 relative to RMS against float64.
"""

from __future__ import annotations

import importlib

import pytest
import torch

import oracle

pytestmark = pytest.mark.gpu


def _check(y, ref, tol=2e-2):
    """|y - ref| <= max(tol * RMS(ref), 1 ulp of the output dtype at ref)."""
    mant = {torch.bfloat16: 7, torch.float16: 10}[y.dtype]
    ref = ref.float()
    rms = ref.pow(2).mean().sqrt().item()
    d = (y.float() - ref).abs()
    u = _ulp(ref, mant, y.dtype)
    worst = (d / torch.maximum(torch.full_like(d, tol * rms), u)).max().item()
    assert worst <= 1.0, f"max|diff|={d.max().item():.4g} rms={rms:.4g} worst/bound={worst:.3g}"


def _ulp(a, mant, dtype):
    """Spacing of `dtype` at |a|, with a mant-bit mantissa; at least the
    subnormal spacing (fp16 outputs below 6.1e-5 are subnormal)."""
    sub = torch.finfo(dtype).tiny * 2.0 ** -mant
    return torch.exp2(torch.floor(torch.log2(a.abs().clamp_min(1e-30))) - mant).clamp_min(sub)


def _check_act(y, gu, tol=2e-2):
    """y against silu(g) * u of the rounded gate_up gu [T, 2I] (see module docstring)."""
    mant = {torch.bfloat16: 7, torch.float16: 10}[y.dtype]
    gu = gu.double()
    i = gu.shape[1] // 2
    g, u = gu[:, :i], gu[:, i:]
    sg = torch.sigmoid(g)
    ref = g * sg * u
    flip = (sg * (1 + g * (1 - sg)) * u).abs() * _ulp(g, mant, y.dtype) + (g * sg).abs() * _ulp(u, mant, y.dtype)
    rms = ref.pow(2).mean().sqrt().item()
    d = (y.double() - ref).abs()
    bound = torch.maximum(torch.full_like(d, tol * rms), _ulp(ref, mant, y.dtype)) + flip
    worst = (d / bound).max().item()
    assert worst <= 1.0, f"max|diff|={d.max().item():.4g} rms={rms:.4g} worst/bound={worst:.3g}"


def _inputs(T, I, K, dev, seed, bias=False, dtype=torch.bfloat16):
    g = torch.Generator(device=dev).manual_seed(seed)
    x = torch.randn(T, K, device=dev, generator=g).to(dtype)
    w = (torch.randn(2 * I, K, device=dev, generator=g) * 0.02).to(dtype)
    b = (torch.randn(2 * I, device=dev, generator=g) * 0.5).to(dtype) if bias else None
    return x, w, b


def _torch_ref(x, w, b=None):
    """bf16 gate_up from cuBLAS (the reference's F.linear), then silu * up in f32."""
    gu = torch.nn.functional.linear(x, w, b)
    i = gu.shape[-1] // 2
    g, u = gu[:, :i].float(), gu[:, i:].float()
    return g / (1.0 + torch.exp(-g)) * u


def _gate_up(x, w, b=None):
    return torch.nn.functional.linear(x, w, b)


# Oracle-sized shapes: decode (swap tiles, split tails), ragged tokens,
# tails in I (not a multiple of 64 / 128) and in K, prefill orientation.
ORACLE_SHAPES = [
    (1, 64, 256, False),
    (5, 200, 136, True),
    (32, 384, 512, False),
    (33, 520, 1000, True),
    (100, 256, 1024, False),
    (256, 1024, 512, False),
    (300, 264, 256, True),
    (1000, 512, 1000, False),
]


@pytest.mark.parametrize("T,I,K,bias", ORACLE_SHAPES)
def test_gate_up_silu_matches_oracle(pgb, cuda_device, T, I, K, bias):
    x, w, b = _inputs(T, I, K, cuda_device, 5000 + T + I + K, bias)
    y = pgb.gate_up_silu(x, w, b)
    torch.cuda.synchronize()
    xn, wn = x.float().cpu().numpy(), w.float().cpu().numpy()
    bn = None if b is None else b.float().cpu().numpy()
    gu = oracle.linear(xn, wn, bn, "bf16")
    ref = oracle.silu_and_mul(gu, "bf16")
    _check_act(y.cpu(), torch.from_numpy(gu))
    # Most outputs agree with the oracle's to the last bit.
    assert (y.cpu().float() != torch.from_numpy(ref)).float().mean().item() < 0.05


# Config-2 shapes (hidden 4096, intermediate 12288) at TP 1/2/4/8, decode and prefill.
MODEL_SHAPES = [
    (1, 12288, 4096),
    (8, 12288, 4096),
    (32, 1536, 4096),
    (64, 6144, 4096),
    (128, 12288, 4096),
    (256, 12288, 4096),
    (256, 3072, 4096),
    (2048, 12288, 4096),
]


@pytest.mark.parametrize("T,I,K", MODEL_SHAPES)
def test_gate_up_silu_matches_f32_restatement(pgb, cuda_device, T, I, K):
    x, w, _ = _inputs(T, I, K, cuda_device, 6000 + T + I)
    y = pgb.gate_up_silu(x, w)
    torch.cuda.synchronize()
    _check_act(y, _gate_up(x, w))


def test_gate_up_silu_fp16(pgb, cuda_device):
    x, w, b = _inputs(48, 1024, 2048, cuda_device, 61, bias=True, dtype=torch.float16)
    y = pgb.gate_up_silu(x, w, b)
    torch.cuda.synchronize()
    _check_act(y, _gate_up(x, w, b))


def test_gate_up_silu_matches_reference_library_path(pgb, cuda_device):
    """F.linear (cuBLAS) + flashinfer.silu_and_mul: the reference's own calls."""
    flashinfer = pytest.importorskip("flashinfer")
    for T in (1, 32, 256, 1024):
        x, w, _ = _inputs(T, 12288, 4096, cuda_device, 7000 + T)
        gu = torch.nn.functional.linear(x, w)
        ref = flashinfer.silu_and_mul(gu)
        y = pgb.gate_up_silu(x, w)
        torch.cuda.synchronize()
        _check_act(y, gu)
        _check_act(ref, gu)  # the library path meets the same bound
        assert (y != ref).float().mean().item() < 0.05


def test_silu_and_mul_matches_flashinfer(pgb, cuda_device):
    """Standalone activation against flashinfer.silu_and_mul on the same input:
    the same f32 steps, so at most one-ulp differences from its division."""
    flashinfer = pytest.importorskip("flashinfer")
    g = torch.Generator(device=cuda_device).manual_seed(8)
    for T, I in ((1, 12288), (37, 1000), (256, 12288), (5, 13)):
        x = (torch.randn(T, 2 * I, device=cuda_device, generator=g) * 4).bfloat16()
        if (2 * I * 2) % 16:
            ref = _torch_silu_mul_ref(x)
        else:
            ref = flashinfer.silu_and_mul(x)
        y = pgb.silu_and_mul(x)
        torch.cuda.synchronize()
        mism = (y != ref).float().mean().item()
        _check(y, ref.float(), tol=0.0)
        assert mism < 1e-3, f"T={T} I={I}: {mism:.2%} of elements differ"


def _torch_silu_mul_ref(x):
    i = x.shape[-1] // 2
    g, u = x[..., :i].float(), x[..., i:].float()
    return (g / (1.0 + torch.exp(-g)) * u).to(x.dtype)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16, torch.float32])
def test_silu_and_mul_dtypes_and_ragged(pgb, cuda_device, dtype):
    g = torch.Generator(device=cuda_device).manual_seed(9)
    for T, I in ((3, 7), (64, 1024), (1, 4)):
        x = (torch.randn(T, 2 * I, device=cuda_device, generator=g) * 3).to(dtype)
        y = pgb.silu_and_mul(x)
        torch.cuda.synchronize()
        ref = _torch_silu_mul_ref(x.float())
        if dtype == torch.float32:
            assert (y - ref).abs().max().item() <= 1e-6 * max(ref.abs().max().item(), 1.0)
        else:
            _check(y, ref, tol=0.0)


@pytest.mark.parametrize("T", [1, 64, 300])
def test_gate_up_silu_f32_check_mode(pgb, cuda_device, T):
    """f32 check mode against float64. The 1e-5 bar is the GEMM's: gate_up
    within 1e-5 * RMS(gate_up), carried through the activation, i.e.
    |diff| <= 1e-5 * RMS(gate_up) * (|silu'(g) u| + |silu(g)|) + 1e-5 * RMS(out).
    (A bound of 1e-5 * RMS(out) alone does not hold for the product of two
    GEMM outputs: where |g| and |u| are several RMS, each input's error is
    multiplied by the other.)"""
    g = torch.Generator(device=cuda_device).manual_seed(40 + T)
    I, K = 1024, 2048
    x = torch.randn(T, K, device=cuda_device, generator=g)
    w = torch.randn(2 * I, K, device=cuda_device, generator=g) * 0.03
    b = torch.randn(2 * I, device=cuda_device, generator=g) * 0.3
    y = pgb.gate_up_silu(x, w, b)
    torch.cuda.synchronize()
    gu = x.double() @ w.double().t() + b.double()
    gg, uu = gu[:, :I], gu[:, I:]
    sg = torch.sigmoid(gg)
    ref = gg * sg * uu
    rms = ref.pow(2).mean().sqrt().item()
    rms_gu = gu.pow(2).mean().sqrt().item()
    bound = 1e-5 * rms_gu * ((sg * (1 + gg * (1 - sg)) * uu).abs() + (gg * sg).abs()) + 1e-5 * rms
    worst = ((y.double() - ref).abs() / bound).max().item()
    assert worst <= 1.0, f"worst/bound={worst:.3g}"
    # The f32 path borrows the shared workspace; the 16-bit kernels after it
    # still find their counters zeroed.
    xb, wb, _ = _inputs(256, 12288, 4096, cuda_device, 41)
    yb = pgb.gate_up_silu(xb, wb)
    torch.cuda.synchronize()
    _check_act(yb, _gate_up(xb, wb))


def test_gate_up_silu_repeatable_and_empty(pgb, cuda_device):
    x, w, _ = _inputs(200, 12288, 4096, cuda_device, 11)
    outs = [pgb.gate_up_silu(x, w) for _ in range(3)]
    torch.cuda.synchronize()
    assert all(torch.equal(o, outs[0]) for o in outs[1:])
    e = pgb.gate_up_silu(x[:0], w)
    assert e.shape == (0, 12288)


def test_gate_up_silu_rejects_bad_width(pgb, cuda_device):
    x, w, _ = _inputs(4, 12, 256, cuda_device, 12)  # I = 12 is not a multiple of 8
    with pytest.raises(pgb.PGBError, match="multiples of 8"):
        pgb.gate_up_silu(x, w)


def test_gated_mlp_layer_matches_reference_composition(pgb, cuda_device):
    """GatedMLP mirror (mlp.py:17-48) at TP 1: fused gate_up + activation, then
    down_proj, against F.linear -> silu_and_mul restatement -> F.linear."""
    D = importlib.import_module("pico-sglang_b200.distributed")
    L = importlib.import_module("pico-sglang_b200.layers")
    H, I, T = 4096, 12288, 16
    with D.tp_override(D.DistributedInfo(0, 1)):
        mlp = L.GatedMLP(H, I, "silu")
    g = torch.Generator(device=cuda_device).manual_seed(13)
    mlp.gate_up_proj.weight = (torch.randn(2 * I, H, device=cuda_device, generator=g) * 0.02).bfloat16()
    mlp.down_proj.weight = (torch.randn(H, I, device=cuda_device, generator=g) * 0.02).bfloat16()
    x = torch.randn(2, T // 2, H, device=cuda_device, generator=g).bfloat16()
    L.reset_fusion_context()
    y = mlp.forward(x)
    torch.cuda.synchronize()
    act = _torch_ref(x.reshape(T, H), mlp.gate_up_proj.weight).bfloat16()
    ref = act.float() @ mlp.down_proj.weight.float().t()
    assert y.shape == (2, T // 2, H)
    _check(y.reshape(T, H), ref)
    # The unfused route (act_fn replaced) gives the same activation input.
    mlp.act_fn = pgb.silu_and_mul
    y2 = mlp.forward(x)
    torch.cuda.synchronize()
    _check(y2.reshape(T, H), ref)
    assert set(mlp.state_dict()) == {"gate_up_proj.weight", "down_proj.weight"}
