"""The C-ABI library on the CPU: it loads, exports what include/pgb.h
declares, and rejects bad arguments with a status + message (no GPU calls)."""

from __future__ import annotations

import ctypes
import re
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parent.parent


def header_symbols() -> set[str]:
    text = (ROOT / "include" / "pgb.h").read_text()
    return set(re.findall(r"PGB_API\s+[\w\s\*]+?\b(pgb_\w+)\s*\(", text))


def test_library_exports_every_declared_symbol(pgb):
    lib = pgb._lib.load()
    declared = header_symbols()
    assert len(declared) >= 18
    for name in declared:
        assert hasattr(lib, name), f"{name} declared in include/pgb.h but not exported"
    # The ctypes signature table covers exactly the header.
    assert set(pgb._lib.declared_symbols()) == declared


def test_version_and_uid(pgb):
    lib = pgb._lib.load()
    assert lib.pgb_version() == 100
    a = (ctypes.c_uint8 * 128)()
    b = (ctypes.c_uint8 * 128)()
    assert lib.pgb_create_uid(a) == 0 and lib.pgb_create_uid(b) == 0
    assert bytes(a) != bytes(b)


def _last_error(lib) -> str:
    return lib.pgb_last_error().decode()


@pytest.mark.parametrize("rank,world", [(0, 0), (2, 2), (-1, 4), (0, 9)])
def test_comm_create_rejects_bad_ranks(pgb, rank, world):
    lib = pgb._lib.load()
    uid = (ctypes.c_uint8 * 128)()
    out = ctypes.c_void_p()
    rc = lib.pgb_comm_create(rank, world, 1 << 20, uid, 0, ctypes.byref(out))
    assert rc == pgb._lib.PGB_ERR_INVALID
    assert "comm_create" in _last_error(lib)
    assert out.value is None


def test_gemm_rejects_bad_arguments_before_touching_the_device(pgb):
    lib = pgb._lib.load()
    rc = lib.pgb_col_gemm(1, 1, None, 1, 4, 16, 12, pgb._lib.PGB_BF16, 1, 1 << 20, None)
    assert rc == pgb._lib.PGB_ERR_INVALID and "multiples of 8" in _last_error(lib)
    rc = lib.pgb_col_gemm(1, 1, None, 1, 4, 16, 16, 7, 1, 1 << 20, None)  # no such dtype
    assert rc == pgb._lib.PGB_ERR_UNSUPPORTED
    rc = lib.pgb_col_gemm(1, 1, None, 1, -1, 16, 16, pgb._lib.PGB_BF16, 1, 1 << 20, None)
    assert rc == pgb._lib.PGB_ERR_INVALID
    rc = lib.pgb_row_gemm_allreduce_addnorm(None, 1, 1, None, 1, 1, 1e-6, 1, 4, 16, 16, 1, None)
    assert rc == pgb._lib.PGB_ERR_INVALID and "null communicator" in _last_error(lib)
    rc = lib.pgb_fused_add_rmsnorm(16, 16, 16, 1e-6, 4, 12, pgb._lib.PGB_BF16, None)
    assert rc == pgb._lib.PGB_ERR_INVALID
    rc = lib.pgb_all_reduce(None, 1, 4, pgb._lib.PGB_BF16, 0, None)
    assert rc == pgb._lib.PGB_ERR_INVALID


def test_errors_surface_as_python_exceptions(pgb):
    with pytest.raises(pgb.PGBError, match="null communicator"):
        pgb._lib.call("pgb_row_gemm_allreduce_addnorm", None, 1, 1, None, 1, 1, 1e-6, 1, 4, 16, 16, 1, None)


def test_workspace_size_is_deterministic(pgb):
    lib = pgb._lib.load()
    a = lib.pgb_col_gemm_workspace_size(8, 6144, 4096)
    assert a == lib.pgb_col_gemm_workspace_size(8, 6144, 4096) and a >= 256
    assert lib.pgb_col_gemm_workspace_size(0, 1, 1) == 256


SHAPE_SWEEP = [
    (T, N, K)
    for T in (1, 3, 8, 32, 33, 64, 128, 200, 256, 257, 1000, 8192)
    for N, K in ((6144, 4096), (24576, 4096), (4096, 512), (4096, 12288), (768, 4096), (3072, 4096),
                 (200, 136), (128, 64), (5120, 25600), (10240, 5120))
]


@pytest.mark.parametrize("sms", [148, 132, 7])
def test_work_decomposition_covers_every_k_block_once(pgb, sms):
    """Every planned GEMM (column: round-robin + stream-K; row-parallel: all
    stream-K, launched on every SM; with and without cluster split-K) covers
    each (tile, k-block) exactly once with consistent contributor counts and
    slab indices."""
    lib = pgb._lib.load()
    bad = []
    for T, N, K in SHAPE_SWEEP:
        for all_sk, grid in ((0, 0), (1, sms)):
            for clusters in (0, 1):
                if lib.pgb_check_work_plan(T, N, K, sms, all_sk, grid, clusters) != 0:
                    bad.append((T, N, K, all_sk, clusters, lib.pgb_last_error().decode()))
    assert not bad, bad[:5]


def test_fused_epilogue_entry_points_reject_bad_arguments_before_the_device(pgb):
    """gate_up + silu, qkv + RoPE + store and the standalone kernels check their
    arguments on the host and return a status; nothing here needs a GPU."""
    lib = pgb._lib.load()
    L = pgb._lib
    ws = ctypes.c_size_t(1 << 20)
    # gate_up_silu: I not a multiple of 8, an unknown dtype, T == 0 (nothing to do)
    rc = lib.pgb_gate_up_silu(1, 1, None, 1, 4, 12, 256, L.PGB_BF16, 1, ws, None)
    assert rc == L.PGB_ERR_INVALID and "multiples of 8" in _last_error(lib)
    assert lib.pgb_gate_up_silu(1, 1, None, 1, 4, 16, 256, 9, 1, ws, None) == L.PGB_ERR_UNSUPPORTED
    assert lib.pgb_gate_up_silu(1, 1, None, 1, 0, 16, 256, L.PGB_BF16, 1, ws, None) == L.PGB_OK
    assert lib.pgb_gate_up_silu(None, 1, None, 1, 4, 16, 256, L.PGB_BF16, 1, ws, None) == L.PGB_ERR_INVALID
    # silu_and_mul: bad width, null pointers, empty input
    assert lib.pgb_silu_and_mul(1, 1, 4, 0, L.PGB_BF16, None) == L.PGB_ERR_INVALID
    assert lib.pgb_silu_and_mul(None, 1, 4, 8, L.PGB_BF16, None) == L.PGB_ERR_INVALID
    assert lib.pgb_silu_and_mul(1, 1, 0, 8, L.PGB_BF16, None) == L.PGB_OK

    def qkv(hd=128, rd=128, idx=L.PGB_I32, T=4, rows=64):
        return lib.pgb_qkv_rope_store(16, 16, None, T, 256, 4, 1, hd, rd, 16, 16, idx, 16, 64, 16, 16, 16, rows,
                                      L.PGB_BF16, 16, ws, None)

    assert qkv(hd=96) == L.PGB_ERR_UNSUPPORTED and "head_dim" in _last_error(lib)
    assert qkv(rd=32) == L.PGB_ERR_UNSUPPORTED and "rotary_dim" in _last_error(lib)
    assert qkv(rd=192) == L.PGB_ERR_UNSUPPORTED
    assert qkv(idx=7) == L.PGB_ERR_INVALID and "index dtype" in _last_error(lib)
    assert qkv(rows=1 << 40) == L.PGB_ERR_INVALID  # slots beyond int32
    assert qkv(T=0) == L.PGB_OK
    rc = lib.pgb_qkv_rope_store(16, 16, None, 4, 256, 4, 1, 128, 128, 16, 16, L.PGB_I32, 16, 64, 24, 16, 16, 64,
                                L.PGB_BF16, 16, ws, None)
    assert rc == L.PGB_ERR_INVALID and "16-byte aligned" in _last_error(lib)
    rc = lib.pgb_rope_store(16, 4, 4, 1, 128, 128, 16, 16, L.PGB_I32, 16, 64, 16, 16, 16, 64, L.PGB_BF16, None, None)
    assert rc == L.PGB_ERR_INVALID and "null" in _last_error(lib)
    # workspace sizes: the gated op plans the [T, 2I] GEMM; f32 adds its intermediate
    assert lib.pgb_gate_up_silu_workspace_size(8, 12288, 4096, L.PGB_BF16) == \
        lib.pgb_col_gemm_workspace_size(8, 24576, 4096)
    assert lib.pgb_qkv_rope_store_workspace_size(8, 32, 8, 128, 4096, L.PGB_BF16) == \
        lib.pgb_col_gemm_workspace_size(8, 6144, 4096)
    assert lib.pgb_gate_up_silu_workspace_size(3, 16, 32, L.PGB_F32) == 256 + 8192 + 3 * 32 * 4
    assert lib.pgb_comm_set_one_rank_path(None, 1) == L.PGB_ERR_INVALID


def test_torch_ops_have_no_cpu_fallback(pgb):
    """The new ops refuse CPU tensors loudly instead of computing on the host."""
    import torch

    x = torch.zeros(2, 64, dtype=torch.bfloat16)
    with pytest.raises(ValueError, match="CUDA"):
        pgb.gate_up_silu(x, torch.zeros(32, 64, dtype=torch.bfloat16))
    with pytest.raises(ValueError, match="CUDA"):
        pgb.silu_and_mul(x)
    with pytest.raises(ValueError, match="CUDA"):
        pgb.ops.qkv_rope_store(x, torch.zeros(3 * 128, 64, dtype=torch.bfloat16), torch.zeros(2, dtype=torch.int32),
                               torch.zeros(2, dtype=torch.int32), torch.zeros(8, 128), 1, 1, 128,
                               torch.zeros(4, 1, 128, dtype=torch.bfloat16), torch.zeros(4, 1, 128, dtype=torch.bfloat16))


def test_rope_store_rejects_mixed_dtypes_before_launch(pgb):
    """rope_store computes in qkv's element type end to end, so caches or a q
    buffer of another type would be written past their rows: refused."""
    import torch

    qkv = torch.zeros(2, 3 * 128, dtype=torch.float32)
    idx = torch.zeros(2, dtype=torch.int32)
    table = torch.zeros(8, 128)
    kc = torch.zeros(4, 1, 128, dtype=torch.bfloat16)
    with pytest.raises(TypeError, match="k_cache"):
        pgb.ops.rope_store(qkv, idx, idx, table, 1, 1, 128, kc, kc.float())
    with pytest.raises(TypeError, match="q_out"):
        pgb.ops.rope_store(qkv, idx, idx, table, 1, 1, 128, kc.float(), kc.float(),
                           q_out=torch.zeros(2, 128, dtype=torch.bfloat16))
    with pytest.raises(TypeError, match="status"):
        pgb.ops.rope_store(qkv, idx, idx, table, 1, 1, 128, kc.float(), kc.float(),
                           status=torch.zeros(1, dtype=torch.int64))


def _plan(lib, T, N, K, sms=148, fused_row=0):
    import ctypes

    buf = ctypes.create_string_buffer(512)
    assert lib.pgb_describe_plan(T, N, K, sms, fused_row, 1, buf, 512) == 0
    return dict(kv.split("=") for kv in buf.value.decode().split())


def test_cta_pair_plans(pgb):
    """Column kernels run prefill shapes (T > 256) and 129-256-token decode
    batches on CTA pairs; shorter batches and the row-parallel kernels keep
    single-CTA tiles; the pair decompositions cover every k-block once."""
    lib = pgb._lib.load()
    p = _plan(lib, 8192, 24576, 4096)
    assert (p["swap"], p["pair"]) == ("0", "1")
    p = _plan(lib, 256, 24576, 4096)
    assert (p["swap"], p["pair"], p["bn"]) == ("1", "1", "256")
    assert int(p["grid"]) <= 148 // 2  # pairs
    for T in (1, 8, 64, 128):
        assert _plan(lib, T, 4096, 4096)["pair"] == "0"
    assert _plan(lib, 256, 4096, 4096, fused_row=1)["pair"] == "0"
    for sms in (148, 132, 100):
        for T in (129, 200, 256):
            for N, K in ((512, 256), (768, 4096), (3072, 4096), (4096, 12288), (24576, 4096), (12800, 5120)):
                assert lib.pgb_check_work_plan(T, N, K, sms, 0, 0, 1) == 0, (T, N, K, sms, lib.pgb_last_error())
