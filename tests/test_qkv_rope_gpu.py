"""qkv_proj GEMM with RoPE and the KV-cache store in its epilogue (and the standalone RoPE + store).

Reference sequence: RotaryAttention.proj (python/picosgl/layers/attention.py:94-117):
qkv_proj (F.linear, bf16) -> split -> flashinfer.apply_rope_with_cos_sin_cache_inplace
(rotary.py:53-59, NeoX) -> the backend's store_kv (cache/kv/mha_pool.py:45-56):
k_cache[out_loc] = k, v_cache[out_loc] = v.

Checked against
  - the CPU oracle (oracle.qkv_rope_store) at sizes it finishes in seconds;
  - this library's unfused pair (col_gemm, then rope_store): bit-identical, as
    both round the same accumulators and use the same RoPE arithmetic;
  - the reference's own calls (cuBLAS F.linear + flashinfer RoPE + index store).
Tolerance. RoPE reads qkv rounded to bf16; two GEMMs that sum in different
orders round some of those values to neighbouring bf16 numbers, and an output
dim then moves by up to one ulp of its own input plus one ulp of its partner
(|cos|, |sin| <= 1). The bound per element is max(2e-2 * RMS, 1 output ulp)
plus those two ulps, evaluated on the reference's own qkv. Slots not in
out_loc must keep their previous contents exactly.
"""

from __future__ import annotations

import importlib

import pytest
import torch

import oracle

pytestmark = pytest.mark.gpu

MAX_POS = 4096
SENTINEL = 3.0


def _ulp(a, mant=7):
    return torch.exp2(torch.floor(torch.log2(a.abs().clamp_min(1e-30))) - mant).clamp_min(
        torch.finfo(torch.bfloat16).tiny * 2.0 ** -mant)


def _own_partner(heads, rd):
    """For rotated outputs: the input dim itself and its NeoX partner (zero
    for unrotated dims). heads: [T, H, hd]."""
    half = rd // 2
    partner = torch.zeros_like(heads)
    partner[..., :half] = heads[..., half:rd]
    partner[..., half:rd] = heads[..., :half]
    return heads, partner


def _check(y, ref, own, partner, tol=2e-2):
    ref, y = ref.double(), y.double()
    rms = ref.pow(2).mean().sqrt().item()
    d = (y - ref).abs()
    bound = torch.maximum(torch.full_like(d, tol * rms), _ulp(ref)) + _ulp(own.double()) + _ulp(partner.double())
    worst = (d / bound).max().item()
    assert worst <= 1.0, f"max|diff|={d.max().item():.4g} rms={rms:.4g} worst/bound={worst:.3g}"


def _case(T, K, nq, nkv, hd, rd, dev, seed, bias=False, idx=torch.int32, dtype=torch.bfloat16):
    L = importlib.import_module("pico-sglang_b200.layers")
    g = torch.Generator(device=dev).manual_seed(seed)
    N = (nq + 2 * nkv) * hd
    x = torch.randn(T, K, device=dev, generator=g).to(dtype)
    w = (torch.randn(N, K, device=dev, generator=g) * 0.02).to(dtype)
    b = (torch.randn(N, device=dev, generator=g) * 0.5).to(dtype) if bias else None
    table = L.get_rope(hd, rd, MAX_POS, 1e6, None).cache_on(dev)
    pos = torch.randint(0, MAX_POS, (T,), generator=g, device=dev).to(idx)
    rows = 2 * T + 16
    loc = torch.randperm(rows, generator=g, device=dev)[:T].to(idx)
    kc = torch.full((rows, nkv, hd), SENTINEL, dtype=dtype, device=dev)
    vc = torch.full((rows, nkv, hd), SENTINEL, dtype=dtype, device=dev)
    return dict(x=x, w=w, b=b, table=table, pos=pos, loc=loc, kc=kc, vc=vc, nq=nq, nkv=nkv, hd=hd, rd=rd)


def _fused(pgb, c):
    return pgb.ops.qkv_rope_store(c["x"], c["w"], c["pos"], c["loc"], c["table"], c["nq"], c["nkv"], c["hd"],
                                  c["kc"], c["vc"], bias=c["b"])


def _compare(c, q, kc, vc, qkv_ref, q_ref, kc_ref, vc_ref):
    """q / cache rows against references; qkv_ref is the reference's rounded qkv."""
    T, nq, nkv, hd, rd = q.shape[0], c["nq"], c["nkv"], c["hd"], c["rd"]
    loc = c["loc"].long().cpu()
    qh = qkv_ref[:, : nq * hd].reshape(T, nq, hd)
    kh = qkv_ref[:, nq * hd:(nq + nkv) * hd].reshape(T, nkv, hd)
    vh = qkv_ref[:, (nq + nkv) * hd:].reshape(T, nkv, hd)
    _check(q.cpu().reshape(T, nq, hd), q_ref.reshape(T, nq, hd), *_own_partner(qh, rd))
    _check(kc.cpu()[loc], kc_ref[loc], *_own_partner(kh, rd))
    _check(vc.cpu()[loc], vc_ref[loc], vh, torch.zeros_like(vh))
    keep = torch.ones(kc.shape[0], dtype=torch.bool)
    keep[loc] = False
    assert torch.all(kc.cpu()[keep] == SENTINEL) and torch.all(vc.cpu()[keep] == SENTINEL)


# (T, K, nq, nkv, hd, rd, bias, index dtype): decode tiles of 32/64/256 tokens with split
# tails, ragged token counts, head_dim 64, partial rotary, bias, int64 indices, prefill.
ORACLE_CASES = [
    (1, 256, 4, 1, 128, 128, False, torch.int32),
    (7, 512, 8, 2, 128, 128, True, torch.int32),
    (33, 256, 8, 4, 64, 64, False, torch.int64),
    (100, 512, 4, 2, 128, 64, True, torch.int32),
    (256, 384, 8, 1, 128, 128, False, torch.int64),
    (300, 256, 4, 2, 64, 64, True, torch.int32),
    (520, 512, 8, 2, 128, 128, False, torch.int32),
    # head_dim 256 and 512 (rotary.py:49 accepts them): GEMM, then the standalone rotation
    (5, 512, 4, 1, 256, 256, True, torch.int32),
    (64, 256, 2, 1, 256, 128, False, torch.int64),
    (300, 512, 2, 1, 512, 512, False, torch.int32),
]


@pytest.mark.parametrize("T,K,nq,nkv,hd,rd,bias,idx", ORACLE_CASES)
def test_qkv_rope_store_matches_oracle(pgb, cuda_device, T, K, nq, nkv, hd, rd, bias, idx):
    c = _case(T, K, nq, nkv, hd, rd, cuda_device, 900 + T + hd, bias, idx)
    q = _fused(pgb, c)
    torch.cuda.synchronize()
    assert pgb.ops.rope_index_error(cuda_device) == 0
    f = lambda t: t.float().cpu().numpy()  # noqa: E731
    xn, wn = f(c["x"]), f(c["w"])
    bn = None if c["b"] is None else f(c["b"])
    qkv = oracle.linear(xn, wn, bn, "bf16")
    q_ref, kc_ref, vc_ref = oracle.qkv_rope_store(xn, wn, bn, c["pos"].cpu().numpy(), c["loc"].cpu().numpy(),
                                                  f(c["table"]), nq, nkv, hd, f(c["kc"]), f(c["vc"]), "bf16")
    _compare(c, q, c["kc"], c["vc"], torch.from_numpy(qkv), torch.from_numpy(q_ref), torch.from_numpy(kc_ref),
             torch.from_numpy(vc_ref))
    assert (q.cpu().float() != torch.from_numpy(q_ref)).float().mean().item() < 0.05


# Config-2 shapes (32 q / 8 kv heads of 128, hidden 4096) at TP 1/2/8, decode and prefill.
MODEL_CASES = [(1, 32, 8), (32, 32, 8), (256, 32, 8), (64, 16, 4), (256, 4, 1), (2048, 32, 8)]


@pytest.mark.parametrize("T,nq,nkv", MODEL_CASES)
def test_fused_equals_unfused_pair(pgb, cuda_device, T, nq, nkv):
    """col_gemm then rope_store gives the same bits as the fused kernel."""
    c = _case(T, 4096, nq, nkv, 128, 128, cuda_device, 1000 + T + nq)
    q = _fused(pgb, c)
    kc2, vc2 = torch.full_like(c["kc"], SENTINEL), torch.full_like(c["vc"], SENTINEL)
    qkv = pgb.col_gemm(c["x"], c["w"])
    q2 = pgb.ops.rope_store(qkv, c["pos"], c["loc"], c["table"], nq, nkv, 128, kc2, vc2)
    torch.cuda.synchronize()
    assert torch.equal(q, q2)
    assert torch.equal(c["kc"], kc2) and torch.equal(c["vc"], vc2)


@pytest.mark.parametrize("T", [1, 32, 256, 1024])
def test_matches_reference_library_path(pgb, cuda_device, T):
    """cuBLAS F.linear + flashinfer.apply_rope_with_cos_sin_cache_inplace + the index store."""
    flashinfer = pytest.importorskip("flashinfer")
    nq, nkv, hd = 32, 8, 128
    c = _case(T, 4096, nq, nkv, hd, hd, cuda_device, 2000 + T)
    qkv = torch.nn.functional.linear(c["x"], c["w"])
    # clone, not contiguous: a one-row slice is already "contiguous" and would
    # let flashinfer rotate qkv itself in place.
    q_ref = qkv[:, : nq * hd].clone()
    k_ref = qkv[:, nq * hd:(nq + nkv) * hd].clone()
    v_ref = qkv[:, (nq + nkv) * hd:].clone()
    flashinfer.apply_rope_with_cos_sin_cache_inplace(c["pos"], q_ref, k_ref, hd, c["table"], is_neox=True)
    kc_ref, vc_ref = c["kc"].clone(), c["vc"].clone()
    kc_ref[c["loc"].long()] = k_ref.view(T, nkv, hd)
    vc_ref[c["loc"].long()] = v_ref.view(T, nkv, hd)
    q = _fused(pgb, c)
    torch.cuda.synchronize()
    _compare(c, q, c["kc"], c["vc"], qkv.float().cpu(), q_ref.float().cpu(), kc_ref.float().cpu(),
             vc_ref.float().cpu())


def test_standalone_rope_store_matches_flashinfer(pgb, cuda_device):
    """Same materialised qkv through flashinfer's RoPE and through rope_store:
    the same f32 steps, so at most rare one-ulp differences."""
    flashinfer = pytest.importorskip("flashinfer")
    for T, nq, nkv, hd, rd in ((1, 32, 8, 128, 128), (77, 8, 2, 64, 64), (256, 32, 8, 128, 64)):
        c = _case(T, 256, nq, nkv, hd, rd, cuda_device, 3000 + T)
        qkv = (torch.randn(T, (nq + 2 * nkv) * hd, device=cuda_device) * 2).bfloat16()
        q_ref = qkv[:, : nq * hd].clone()  # clone: flashinfer rotates in place
        k_ref = qkv[:, nq * hd:(nq + nkv) * hd].clone()
        flashinfer.apply_rope_with_cos_sin_cache_inplace(c["pos"], q_ref, k_ref, hd, c["table"], is_neox=True)
        q = pgb.ops.rope_store(qkv, c["pos"], c["loc"], c["table"], nq, nkv, hd, c["kc"], c["vc"])
        torch.cuda.synchronize()
        q_in = qkv[:, : nq * hd].float().cpu().reshape(T, nq, hd)
        _check(q.cpu().reshape(T, nq, hd), q_ref.float().cpu().reshape(T, nq, hd), *_own_partner(q_in, rd), tol=0.0)
        k_got = c["kc"][c["loc"].long()].reshape(T, -1)
        assert (q != q_ref).float().mean().item() < 1e-2
        assert (k_got != k_ref).float().mean().item() < 1e-2
        assert torch.equal(c["vc"][c["loc"].long()].reshape(T, -1), qkv[:, (nq + nkv) * hd:])


@pytest.mark.parametrize("T", [1, 64, 300])
def test_qkv_rope_store_f32_check_mode(pgb, cuda_device, T):
    """f32: |diff| <= 1.5e-5 * RMS(qkv) against float64 (the GEMM's 1e-5 bar
    through a rotation, |cos| + |sin| <= sqrt 2)."""
    nq, nkv, hd = 4, 2, 128
    c = _case(T, 1024, nq, nkv, hd, hd, cuda_device, 4000 + T, bias=True, dtype=torch.float32)
    q = _fused(pgb, c)
    torch.cuda.synchronize()
    assert pgb.ops.rope_index_error(cuda_device) == 0
    qkv = c["x"].double() @ c["w"].double().t() + c["b"].double()
    table = c["table"].double()
    rows = table[c["pos"].long()]
    cs, sn = rows[:, None, : hd // 2], rows[:, None, hd // 2:]

    def rot(h):
        a, b = h[..., : hd // 2], h[..., hd // 2:]
        return torch.cat([a * cs - b * sn, b * cs + a * sn], -1)

    q_ref = rot(qkv[:, : nq * hd].reshape(T, nq, hd))
    k_ref = rot(qkv[:, nq * hd:(nq + nkv) * hd].reshape(T, nkv, hd))
    v_ref = qkv[:, (nq + nkv) * hd:].reshape(T, nkv, hd)
    bar = 1.5e-5 * qkv.pow(2).mean().sqrt().item()
    loc = c["loc"].long()
    assert (q.double().reshape(T, nq, hd) - q_ref).abs().max().item() <= bar
    assert (c["kc"][loc].double() - k_ref).abs().max().item() <= bar
    assert (c["vc"][loc].double() - v_ref).abs().max().item() <= bar


def test_out_of_range_indices_skip_the_token(pgb, cuda_device):
    """A position >= max_position or a slot >= cache rows: that token writes
    nothing (its q row keeps its old contents, no cache row changes) and the
    index-error word reads 5; the other tokens are exact. The kernels check
    both indices before any load or store that uses them."""
    T, nq, nkv, hd = 40, 8, 2, 128
    c = _case(T, 512, nq, nkv, hd, hd, cuda_device, 5000)
    c["pos"][3] = MAX_POS
    c["loc"][7] = c["kc"].shape[0]
    pgb.ops.rope_index_error(cuda_device, reset=True)
    q = torch.full((T, nq * hd), SENTINEL, dtype=torch.bfloat16, device=cuda_device)
    pgb.ops.qkv_rope_store(c["x"], c["w"], c["pos"], c["loc"], c["table"], nq, nkv, hd, c["kc"], c["vc"], q_out=q)
    torch.cuda.synchronize()
    assert pgb.ops.rope_index_error(cuda_device, reset=True) == 5
    assert pgb.ops.rope_index_error(cuda_device) == 0
    assert torch.all(q[3] == SENTINEL) and torch.all(q[7] == SENTINEL)
    good = [t for t in range(T) if t not in (3, 7)]
    kc2, vc2 = torch.full_like(c["kc"], SENTINEL), torch.full_like(c["vc"], SENTINEL)
    sub = torch.tensor(good, device=cuda_device)
    q2 = pgb.ops.rope_store(pgb.col_gemm(c["x"], c["w"])[sub].contiguous(), c["pos"][sub].contiguous(),
                            c["loc"][sub].contiguous(), c["table"], nq, nkv, hd, kc2, vc2)
    torch.cuda.synchronize()
    assert torch.equal(q[sub], q2)
    assert torch.equal(c["kc"], kc2) and torch.equal(c["vc"], vc2)
    # The split-tile kernels that share the workspace are unaffected.
    x = torch.randn(1, 4096, device=cuda_device).bfloat16()
    w = (torch.randn(24576, 4096, device=cuda_device) * 0.02).bfloat16()
    y = pgb.col_gemm(x, w)
    ref = x.float() @ w.float().t()
    assert (y.float() - ref).abs().max().item() <= 2e-2 * ref.pow(2).mean().sqrt().item() + 0.02


def test_rotary_attention_mirror_proj_store(pgb, cuda_device):
    """RotaryAttention mirror (attention.py:46-117) at TP 1: proj_store gives
    the fused result, with the reference's weight names."""
    D = importlib.import_module("pico-sglang_b200.distributed")
    L = importlib.import_module("pico-sglang_b200.layers")
    with D.tp_override(D.DistributedInfo(0, 1)):
        attn = L.RotaryAttention(4096, 128, 32, 8, 0, 128, MAX_POS, 1e6, None)
    assert set(attn.state_dict()) == {"qkv_proj.weight", "o_proj.weight"}
    c = _case(16, 4096, 32, 8, 128, 128, cuda_device, 6000)
    attn.qkv_proj.weight = c["w"]
    q = attn.proj_store(c["x"].view(2, 8, 4096), c["pos"].view(2, 8), c["loc"].view(2, 8), c["kc"], c["vc"])
    assert q.shape == (2, 8, 32, 128)
    kc2, vc2 = torch.full_like(c["kc"], SENTINEL), torch.full_like(c["vc"], SENTINEL)
    q2 = pgb.ops.qkv_rope_store(c["x"], c["w"], c["pos"], c["loc"], c["table"], 32, 8, 128, kc2, vc2)
    torch.cuda.synchronize()
    assert torch.equal(q.reshape(16, -1), q2) and torch.equal(c["kc"], kc2)


def test_empty_and_bad_shapes(pgb, cuda_device):
    c = _case(4, 256, 4, 1, 128, 128, cuda_device, 7000)
    q = pgb.ops.qkv_rope_store(c["x"][:0], c["w"], c["pos"][:0], c["loc"][:0], c["table"], 4, 1, 128, c["kc"],
                               c["vc"])
    assert q.shape == (0, 512)
    c96 = _case(4, 256, 4, 1, 128, 128, cuda_device, 7001)
    L = importlib.import_module("pico-sglang_b200.layers")
    t96 = L.get_rope(128, 96, 64, 1e4, None).cache_on(cuda_device)
    with pytest.raises(pgb.PGBError, match="rotary_dim"):
        pgb.ops.qkv_rope_store(c96["x"], c96["w"], c96["pos"] % 64, c96["loc"], t96, 4, 1, 128, c96["kc"], c96["vc"])
