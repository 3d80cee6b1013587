"""f32 check mode: column GEMM and the fused row op in IEEE f32.

The north-star bound for the f32 check mode is 1e-5 relative: here
max |diff| <= 1e-5 * RMS(reference), with the reference computed in float64
from the same f32 inputs (the exact value the f32 path rounds). The fused op
follows F.linear -> all_reduce -> fused_add_rmsnorm
(python/picosgl/layers/linear.py:90-97, norm.py:73-75) at f32.
"""

from __future__ import annotations

import importlib

import pytest
import torch

pytestmark = pytest.mark.gpu

REL = 1e-5


def _rel_err(y, ref):
    ref = ref.double()
    rms = ref.pow(2).mean().sqrt().item()
    return (y.double() - ref).abs().max().item() / rms


@pytest.mark.parametrize("T,N,K", [(1, 6144, 4096), (33, 3072, 4096), (256, 1000, 1000), (1000, 1024, 1000)])
def test_col_gemm_f32(pgb, cuda_device, T, N, K):
    g = torch.Generator(device=cuda_device).manual_seed(99 + T + N)
    x = torch.randn(T, K, device=cuda_device, generator=g)
    w = torch.randn(N, K, device=cuda_device, generator=g) * 0.02
    b = torch.randn(N, device=cuda_device, generator=g)
    y = pgb.col_gemm(x, w, b)
    torch.cuda.synchronize()
    ref = x.double() @ w.double().t() + b.double()
    assert _rel_err(y, ref) <= REL


@pytest.mark.parametrize("T", [1, 64, 300])
def test_row_fused_f32_tp1(pgb, cuda_device, T):
    D = importlib.import_module("pico-sglang_b200.distributed")
    comm = D.PGBCommunicator(0, 1, 64 << 20, D.create_uid(), 0)
    try:
        H, K = 4096, 4096
        g = torch.Generator(device=cuda_device).manual_seed(7 + T)
        x = torch.randn(T, K, device=cuda_device, generator=g)
        w = torch.randn(H, K, device=cuda_device, generator=g) * 0.02
        r = torch.randn(T, H, device=cuda_device, generator=g)
        nw = torch.rand(H, device=cuda_device, generator=g) + 0.5
        r0 = r.clone()
        out = pgb.row_gemm_allreduce_addnorm(comm, x, w, r, nw, 1e-6)
        torch.cuda.synchronize()
        s = x.double() @ w.double().t() + r0.double()
        ref = s * torch.rsqrt(s.pow(2).mean(-1, keepdim=True) + 1e-6) * nw.double()
        assert _rel_err(r, s) <= REL
        assert _rel_err(out, ref) <= REL
    finally:
        comm.close()
