"""CPU oracle for the tensor-parallel linear path -- TEST INFRASTRUCTURE ONLY.

This package restates, in numpy, what the reference (dakingffo/pico-sglang)
computes on the path the CUDA library replaces: the column-parallel and
row-parallel linears, the gated MLP's silu_and_mul on the gate_up output,
RoPE on the q and k heads with the KV-cache store,
the sum all-reduce that follows a row-parallel linear, and the residual-add
+ RMSNorm that consumes it.

It is the checker, never the product. Only tests/, __graft_entry__.smoke()
and bench.py's CPU-baseline leg (and its --impl reference arm) may import
it. The library under pico-sglang_b200/ never imports it and has no CPU
fallback.

Pinning: tests/test_oracle.py checks this restatement against golden
vectors produced by running the reference's own Python layers on the CPU
(tests/golden/make_golden.py, which imports the reference read-only), and
against the known answers of the reference's communicator test
(tests/distributed/test_pynccl.py:95-148). The RMSNorm half is a restatement
of FlashInfer's FusedAddRMSNormKernel (flashinfer/data/include/flashinfer/
norm.cuh:387-470, a third-party dependency the reference calls at
python/picosgl/layers/norm.py:74); no reference test exercises it, so on the
CPU it is pinned to that published kernel only, and the GPU tests pin it to
the installed flashinfer.fused_add_rmsnorm itself. silu_and_mul restates
flashinfer's act_and_mul kernel the same way; it is pinned on the CPU to the
reference's GatedMLP run with that restatement as its act_fn (mlp_small.npz)
and to torch.nn.functional.silu, and on the GPU to flashinfer.silu_and_mul.
apply_rope_neox restates flashinfer's rope kernel; its cos/sin table comes
from the reference's own get_rope (rope_small.npz), the rotation is pinned to
its defining properties on the CPU and to flashinfer's
apply_rope_with_cos_sin_cache_inplace on the GPU.
"""

from .tp_linear import (  # noqa: F401
    all_reduce_sum,
    apply_rope_neox,
    col_shard_merged,
    col_shard_partitioned,
    fused_add_rmsnorm,
    gate_up_silu,
    linear,
    qkv_rope_store,
    rmsnorm,
    round_to,
    row_parallel_addnorm,
    row_shard,
    silu_and_mul,
    store_kv,
    tp_layer_step,
)
