"""Column-parallel GEMM (qkv_proj / gate_up_proj) on the tcgen05 kernel.

Compared with a plain torch f32 restatement of F.linear
(python/picosgl/layers/linear.py:23-27): y = bf16(x_f32 @ w_f32^T + b).
Tolerance: max |diff| <= 2e-2 * RMS(reference) (the bf16 bar of the
north-star parity rule); in practice both round an f32 accumulation once,
so differences are a few bf16 ulps.
"""

from __future__ import annotations

import pytest
import torch

pytestmark = pytest.mark.gpu


def _ref(x, w, b=None):
    y = x.float() @ w.float().t()
    if b is not None:
        y = y + b.float()
    return y


def _check(y, ref, tol=2e-2):
    """|y - ref| <= max(tol * RMS(ref), 1 ulp of the output dtype at ref)."""
    mant = {torch.bfloat16: 7, torch.float16: 10}[y.dtype]
    rms = ref.pow(2).mean().sqrt().item()
    d = (y.float() - ref).abs()
    u = torch.exp2(torch.floor(torch.log2(ref.abs().clamp_min(1e-30))) - mant)
    worst = (d / torch.maximum(torch.full_like(d, tol * rms), u)).max().item()
    assert worst <= 1.0, f"max|diff|={d.max().item():.4g} rms={rms:.4g} worst/bound={worst:.3g}"


SHAPES = [
    # (T, N, K): decode TP=1/8 qkv, gate_up; ragged tokens; tails in N and K
    (1, 6144, 4096),
    (8, 6144, 4096),
    (1, 24576, 4096),  # gate_up: a full wave of whole tiles, then a split tail
    (256, 24576, 4096),
    (32, 768, 4096),
    (33, 3072, 4096),
    (64, 1280, 5120),
    (100, 512, 1024),
    (128, 6144, 4096),
    (200, 200, 136),
    (256, 3072, 4096),
    (257, 512, 512),
    (1000, 1024, 1000),
    (2048, 6144, 4096),
    # config 3 prefill (8192 tokens): qkv_proj and gate_up_proj at TP=1
    (8192, 6144, 4096),
    (8192, 24576, 4096),
    # config 4 (hidden 5120) shards at TP=8: qkv 10240/8, gate_up 51200/8; T=64 and 4096
    (64, 1280, 5120),
    (64, 6400, 5120),
    (4096, 6400, 5120),
]


@pytest.mark.parametrize("T,N,K", SHAPES)
@pytest.mark.parametrize("dtype", [torch.bfloat16])
def test_col_gemm_matches_f32(pgb, cuda_device, T, N, K, dtype):
    g = torch.Generator(device=cuda_device).manual_seed(1234 + T + N + K)
    x = torch.randn(T, K, device=cuda_device, generator=g).to(dtype)
    w = (torch.randn(N, K, device=cuda_device, generator=g) * 0.02).to(dtype)
    y = pgb.col_gemm(x, w)
    torch.cuda.synchronize()
    _check(y, _ref(x, w))


def test_col_gemm_fp16_and_bias(pgb, cuda_device):
    """fp16 with a bias on each kernel: single-CTA decode (T = 4), the decode
    CTA-pair kernel (T = 200) and the prefill CTA-pair kernel (T = 300)."""
    g = torch.Generator(device=cuda_device).manual_seed(7)
    for T in (4, 200, 300):
        x = torch.randn(T, 512, device=cuda_device, generator=g).half()
        w = (torch.randn(1024, 512, device=cuda_device, generator=g) * 0.02).half()
        b = torch.randn(1024, device=cuda_device, generator=g).half()
        y = pgb.col_gemm(x, w, b)
        torch.cuda.synchronize()
        _check(y, _ref(x, w, b))


def test_col_gemm_repeatable_and_workspace_clean(pgb, cuda_device):
    """Split-K counters are reset by the kernel: repeated calls agree bit for bit."""
    g = torch.Generator(device=cuda_device).manual_seed(11)
    x = torch.randn(8, 4096, device=cuda_device, generator=g).bfloat16()
    w = (torch.randn(4096, 4096, device=cuda_device, generator=g) * 0.02).bfloat16()
    y0 = pgb.col_gemm(x, w)
    for _ in range(5):
        y1 = pgb.col_gemm(x, w)
        torch.cuda.synchronize()
        assert torch.equal(y0, y1)


def test_col_gemm_rejects_bad_shapes(pgb, cuda_device):
    x = torch.randn(4, 12, device=cuda_device).bfloat16()
    w = torch.randn(16, 12, device=cuda_device).bfloat16()
    with pytest.raises(pgb.PGBError, match="multiples of 8"):
        pgb.col_gemm(x, w)


def test_col_gemm_shapes_share_one_workspace(pgb, cuda_device):
    """Calls of different shapes on one workspace, through the C ABI. The
    first plans few split tiles (a small counter set) and leaves f32 partials
    in its exchange area; the later ones plan more split tiles, so with a
    plan-sized counter region their counters would lie where those partials
    are. The counter region is fixed, so every call is exact."""
    import ctypes

    lib = pgb._lib.load()
    shapes = [(32, 768, 4096), (1, 24576, 4096), (33, 3072, 4096), (128, 24576, 4096), (32, 768, 4096)]
    need = max(lib.pgb_col_gemm_workspace_size(T, N, K) for T, N, K in shapes)
    ws = torch.zeros(need, dtype=torch.uint8, device=cuda_device)
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    for i, (T, N, K) in enumerate(shapes):
        g = torch.Generator(device=cuda_device).manual_seed(300 + i)
        x = torch.randn(T, K, device=cuda_device, generator=g).bfloat16()
        w = (torch.randn(N, K, device=cuda_device, generator=g) * 0.02).bfloat16()
        y = torch.empty(T, N, dtype=torch.bfloat16, device=cuda_device)
        rc = lib.pgb_col_gemm(x.data_ptr(), w.data_ptr(), None, y.data_ptr(), T, N, K, 1, ws.data_ptr(),
                              ctypes.c_size_t(need), stream)
        assert rc == 0, lib.pgb_last_error()
        torch.cuda.synchronize()
        _check(y, _ref(x, w))
    head = ws[:256 + 8192]
    assert int(head.count_nonzero().item()) == 0, "status word and counters are left zeroed"


# Decode shards of config 2 (hidden 4096, intermediate 12288, 32 q / 8 kv heads
# of 128) at TP = 1, 2, 4, 8: qkv, o, gate_up and down.
_DECODE_NK = sorted({(n, k) for tp in (1, 2, 4, 8) for n, k in (
    (6144 // tp, 4096), (4096, 4096 // tp), (24576 // tp, 4096), (4096, 12288 // tp))})


def test_col_gemm_decode_sequence_writes_every_element(pgb, cuda_device):
    """Every decode shard at T = 1, 64, 128, 256, one after another on one
    stream and one workspace (each plan leaves its own split partials behind
    for the next), eagerly and as CUDA-graph replays. The output is filled
    with NaN first: an element that no CTA stores, or a split tile summed
    from a stale partial, fails the comparison."""
    stream = torch.cuda.Stream(cuda_device)
    cases = [(T, n, k) for T in (256, 1, 128, 64) for n, k in _DECODE_NK]
    g = torch.Generator(device=cuda_device).manual_seed(77)
    xs = {(T, k): torch.randn(T, k, device=cuda_device, generator=g).bfloat16() for T, _, k in cases}
    ws = {(n, k): (torch.randn(n, k, device=cuda_device, generator=g) * 0.02).bfloat16() for _, n, k in cases}
    ys = {c: torch.empty(c[0], c[1], device=cuda_device, dtype=torch.bfloat16) for c in cases}
    torch.cuda.synchronize()
    with torch.cuda.stream(stream):
        for c in cases:  # eager, and sizes the shared workspace before capture
            ys[c].fill_(float("nan"))
            pgb.col_gemm(xs[(c[0], c[2])], ws[(c[1], c[2])], out=ys[c])
        stream.synchronize()
        for c in cases:
            _check(ys[c], _ref(xs[(c[0], c[2])], ws[(c[1], c[2])]))
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=stream):
            for c in cases:
                ys[c].fill_(float("nan"))
                pgb.col_gemm(xs[(c[0], c[2])], ws[(c[1], c[2])], out=ys[c])
        for _ in range(3):
            graph.replay()
        stream.synchronize()
    for c in cases:
        _check(ys[c], _ref(xs[(c[0], c[2])], ws[(c[1], c[2])]))
    del graph
