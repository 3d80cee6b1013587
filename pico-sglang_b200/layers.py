"""Drop-in mirrors of the reference's TP linear layers and fused RMSNorm.

Constructor signatures, attribute names (``weight`` / ``bias``, found by the
loader through BaseOP.state_dict, python/picosgl/layers/base.py:14-59) and
local shard sizes are those of python/picosgl/layers/linear.py:11-97 and
norm.py:56-75; ``forward`` runs the libpgb kernels.

Fusing a row-parallel layer with the norm that consumes it. The reference's
decoder layer (models/llama.py:77-86) calls, in order,
``x, residual = input_layernorm(x, residual)`` -> attention ... ``o_proj(x)``
-> ``x, residual = post_attention_layernorm(x, residual)`` -> mlp ...
``down_proj(x)`` -> the next layer's ``input_layernorm`` (or the final
``norm``). ``link_norm`` ties a row-parallel layer to its consumer. Every
RMSNormFused.forward records the residual it returns; a linked
LinearRowParallel.forward then runs GEMM + all-reduce + residual-add + norm
in one kernel on that residual (in place) and returns the normalised output,
remembered as already normalised for that norm and residual. The consumer's
forward recognises it and returns ``(x, residual)`` unchanged. The model
code does not change, the stream order is the same, and CUDA-graph capture
records the same single kernel.
"""

from __future__ import annotations

import functools
import math
import threading

import torch

from . import ops
from .distributed import DistributedCommunicator, get_tp_info, local_comm


def div_even(a: int, b: int, allow_replicate: bool = False) -> int:
    """a / b for an exact split across b ranks (the contract of utils/misc.py:20-26).

    With allow_replicate, fewer items than ranks (kv heads under a wide TP
    group) give 1 item per rank, each replicated on b / a ranks."""
    if allow_replicate and a < b:
        if b % a:
            raise AssertionError(f"{b} ranks cannot replicate {a} kv heads evenly")
        return 1
    q, rem = divmod(a, b)
    if rem:
        raise AssertionError(f"{a} does not split evenly over {b} ranks")
    return q


def _public_attrs(obj):
    return [(k, v) for k, v in vars(obj).items() if not k.startswith("_")]


class BaseOP:
    """Loader contract of layers/base.py:14-59: every public tensor attribute is
    a parameter named by its attribute path ("mlp.down_proj.weight"); nested
    BaseOPs contribute their own under their attribute name."""

    def state_dict(self, *, prefix: str = "", result: dict | None = None) -> dict:
        out = {} if result is None else result
        for name, val in _public_attrs(self):
            path = name if not prefix else prefix + "." + name
            if isinstance(val, BaseOP):
                val.state_dict(prefix=path, result=out)
            elif isinstance(val, torch.Tensor):
                out[path] = val
        return out

    def load_state_dict(self, state_dict: dict, *, prefix: str = "", _internal: bool = False) -> None:
        for name, val in _public_attrs(self):
            path = name if not prefix else prefix + "." + name
            if isinstance(val, BaseOP):
                val.load_state_dict(state_dict, prefix=path, _internal=True)
            elif isinstance(val, torch.Tensor):
                new = state_dict.pop(path)
                if tuple(new.shape) != tuple(val.shape):
                    raise AssertionError(f"{path}: checkpoint shape {tuple(new.shape)}, layer {tuple(val.shape)}")
                setattr(self, name, new.to(val.dtype))
        if state_dict and not _internal:
            raise RuntimeError(f"Unexpected keys in state_dict: {sorted(state_dict)}")


class _FuseContext(threading.local):
    def __init__(self) -> None:
        self.residual: torch.Tensor | None = None
        self.fused: tuple | None = None  # (out, norm, residual) produced by a linked row layer


_CTX = _FuseContext()


def reset_fusion_context() -> None:
    _CTX.residual = None
    _CTX.fused = None


def _flat2d(x: torch.Tensor) -> torch.Tensor:
    return x.reshape(-1, x.shape[-1]) if x.dim() != 2 else x


class LinearTPImpl(BaseOP):
    """layers/linear.py:11-27, forward on the tcgen05 column GEMM."""

    def __init__(self, input_size: int, output_size: int, has_bias: bool):
        self.weight = torch.empty(output_size, input_size)
        self.bias = torch.empty(output_size) if has_bias else None

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        x2 = _flat2d(x).contiguous()
        y = ops.col_gemm(x2, self.weight, self.bias)
        return y.view(*x.shape[:-1], y.shape[-1])


class LinearReplicated(LinearTPImpl):
    pass


class LinearColParallelMerged(LinearTPImpl):
    """linear.py:45-56 (gate_up_proj): local rows [gate/n; up/n]."""

    def __init__(self, input_size: int, output_sizes: list[int], has_bias: bool):
        tp = get_tp_info()
        super().__init__(input_size, sum(div_even(s, tp.size) for s in output_sizes), has_bias)


class LinearColParallelPartitioned(LinearTPImpl):
    """linear.py:59-73 (qkv_proj): per-head shards with kv replication."""

    def __init__(self, input_size: int, partition_size: int, partitions: list[tuple[int, bool]],
                 has_bias: bool):
        tp = get_tp_info()
        parts = [div_even(p, tp.size, rep) for p, rep in partitions]
        super().__init__(input_size, sum(parts) * partition_size, has_bias)


class LinearRowParallel(LinearTPImpl):
    """linear.py:76-97: K-sharded GEMM followed by the sum all-reduce.

    Unlinked, forward returns the reduced output (fused GEMM + all-reduce for
    TP > 1, the plain GEMM for TP = 1). Linked to its consuming RMSNormFused,
    forward also applies the residual-add + RMSNorm (module docstring).
    """

    def __init__(self, input_size: int, output_size: int, has_bias: bool):
        tp = get_tp_info()
        self._tp_size = tp.size
        self._norm: RMSNormFused | None = None
        super().__init__(div_even(input_size, tp.size), output_size, has_bias)

    def link_norm(self, norm: "RMSNormFused | None") -> None:
        self._norm = norm

    def _comm(self):
        c = DistributedCommunicator.comm
        if c is None:
            if self._tp_size > 1:
                raise RuntimeError("TP > 1 needs enable_pgb_distributed() before forward")
            c = local_comm()
        return c

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        x2 = _flat2d(x).contiguous()
        T = x2.shape[0]
        N = self.weight.shape[0]
        res = _CTX.residual
        norm = self._norm
        if norm is not None and res is not None and res.shape == (T, N) and res.dtype == x2.dtype:
            out = ops.row_gemm_allreduce_addnorm(self._comm(), x2, self.weight, res, norm.weight, norm.eps,
                                                 bias=self.bias)
            if x.dim() != 2:
                out = out.view(*x.shape[:-1], N)
            _CTX.fused = (out, norm, res)  # the exact object handed to the consumer
            return out
        if self._tp_size == 1:
            y = ops.col_gemm(x2, self.weight, self.bias)
        else:
            y = ops.row_gemm_allreduce_addnorm(self._comm(), x2, self.weight, None, None, 0.0, bias=self.bias)
        return y.view(*x.shape[:-1], N)


def silu_and_mul(x: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
    """layers/activation.py:9-12: silu(x[..., :I]) * x[..., I:] on the libpgb kernel."""
    return ops.silu_and_mul(x, out=out)


class GatedMLP(BaseOP):
    """layers/mlp.py:17-48 with the activation fused into gate_up_proj.

    Same attributes (``gate_up_proj``, ``act_fn``, ``down_proj``) and shards.
    While ``act_fn`` is this module's silu_and_mul, forward runs gate_up_proj
    and the activation as one kernel (the [T, 2I] gate_up tensor is never
    stored), then down_proj; an act_fn set to anything else runs unfused, in
    the reference's order.
    """

    def __init__(self, hidden_size: int, intermediate_size: int, hidden_act: str):
        self.gate_up_proj = LinearColParallelMerged(hidden_size, [intermediate_size, intermediate_size],
                                                    has_bias=False)
        if hidden_act == "silu":
            self.act_fn = silu_and_mul
        elif hidden_act == "gelu":
            raise NotImplementedError("gelu_and_mul is not implemented by this library")
        else:
            raise ValueError(f"Unsupported activation function: {hidden_act}")
        self.down_proj = LinearRowParallel(intermediate_size, hidden_size, has_bias=False)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        if self.act_fn is silu_and_mul:
            x2 = _flat2d(x).contiguous()
            y = ops.gate_up_silu(x2, self.gate_up_proj.weight, self.gate_up_proj.bias)
            y = y.view(*x.shape[:-1], y.shape[-1])
        else:
            y = self.act_fn(self.gate_up_proj.forward(x))
        return self.down_proj.forward(y)


# ----------------------------------------------------------------- rotary --


class RotaryEmbedding(BaseOP):
    """layers/rotary.py:12-32: the [max_position, rotary_dim] float32 table the
    RoPE kernels read, the cosines of the rotary_dim/2 angles of each position
    followed by their sines. The angles are position * inv_freq with
    inv_freq = 1 / base^(2i / rotary_dim), optionally rescaled by
    `post_process`; the float32 steps are the reference's, so the table is
    bit-identical to its _cos_sin_cache."""

    def __init__(self, head_size: int, rotary_dim: int, max_position_embeddings: int, base: float,
                 post_process=None) -> None:
        if not (0 < rotary_dim <= head_size and rotary_dim % 2 == 0):
            raise ValueError(f"rotary_dim {rotary_dim} must be even and in (0, {head_size}]")
        self.head_size = head_size
        exponents = torch.arange(0, rotary_dim, 2, dtype=torch.float) / rotary_dim
        inv_freq = 1.0 / (base ** exponents)
        if post_process is not None:
            inv_freq = post_process(inv_freq)
        angles = torch.outer(torch.arange(max_position_embeddings, dtype=torch.float), inv_freq)
        self._cos_sin_cache = torch.cat((angles.cos(), angles.sin()), dim=-1)
        self._on_device: dict = {}

    def cache_on(self, device: torch.device) -> torch.Tensor:
        """The table on `device` (copied once per device)."""
        if self._cos_sin_cache.device == device:
            return self._cos_sin_cache
        c = self._on_device.get(device)
        if c is None:
            c = self._on_device[device] = self._cos_sin_cache.to(device).contiguous()
        return c


def _llama3_inv_freq(factor: float, low_freq_factor: float, high_freq_factor: float, original_max: int):
    """Llama 3 frequency rescaling: wavelengths above original_max / low_freq_factor are slowed
    by `factor`, those below original_max / high_freq_factor kept, and the band between
    interpolated linearly in original_max / wavelength (a hard switch if the factors are equal)."""

    def apply(inv_freq: torch.Tensor) -> torch.Tensor:
        wavelength = 2 * math.pi / inv_freq
        if low_freq_factor == high_freq_factor:
            return torch.where(wavelength < original_max / high_freq_factor, inv_freq, inv_freq / factor)
        t = ((original_max / wavelength - low_freq_factor) / (high_freq_factor - low_freq_factor)).clamp(0, 1)
        return ((1 - t) / factor + t) * inv_freq

    return apply


def _yarn_inv_freq(rotary_dim: int, base: float, factor: float, original_max: int, beta_fast: float,
                   beta_slow: float):
    """YaRN frequency blend: dimensions below the beta_fast correction dimension keep their
    frequency, those above the beta_slow one are divided by `factor`, with a linear ramp between."""

    def correction_dim(rotations: float) -> float:
        return rotary_dim * math.log(original_max / (rotations * 2 * math.pi)) / (2 * math.log(base))

    lo = max(math.floor(correction_dim(beta_fast)), 0)
    hi = min(math.ceil(correction_dim(beta_slow)), rotary_dim // 2 - 1)

    def apply(inv_freq: torch.Tensor) -> torch.Tensor:
        ramp = ((torch.arange(rotary_dim // 2, dtype=torch.float32) - lo) / max(hi - lo, 1)).clamp(0, 1)
        return (inv_freq / factor) * ramp + inv_freq * (1 - ramp)

    return apply


@functools.cache
def get_rope(head_dim: int, rotary_dim: int, max_position: int, base: float,
             rope_scaling: tuple | None = None) -> RotaryEmbedding:
    """layers/rotary.py:63-151: the table for rope_scaling None / default / llama3 / yarn."""
    cfg = dict(rope_scaling) if rope_scaling is not None else None
    kind = None if cfg is None else cfg["rope_type"]
    if kind in (None, "default"):
        post = None
    elif kind == "llama3":
        post = _llama3_inv_freq(cfg["factor"], cfg["low_freq_factor"], cfg["high_freq_factor"],
                                cfg["original_max_position_embeddings"])
    elif kind == "yarn":
        post = _yarn_inv_freq(rotary_dim, base, cfg["factor"], cfg["original_max_position_embeddings"],
                              cfg.get("beta_fast", 32.0), cfg.get("beta_slow", 1.0))
    else:
        raise ValueError(f"Unsupported {rope_scaling = }")
    return RotaryEmbedding(head_dim, rotary_dim, max_position, base, post)


class RotaryAttention(BaseOP):
    """layers/attention.py:46-117: the same constructor, shards and weight names.

    proj_store(x, positions, out_loc, k_cache, v_cache) is proj
    (attention.py:94-117) followed by the backend's store_kv
    (cache/kv/mha_pool.py:45-56) as one kernel: it returns the rotated query
    [..., nq, hd] and leaves the rotated key and the value in the given layer
    caches at out_loc. The attention itself belongs to the backend.
    """

    def __init__(self, hidden_size: int, head_dim: int, num_qo_heads: int, num_kv_heads: int, layer_id: int,
                 rotary_dim: int, max_position: int, rope_base: float, rope_scaling, *,
                 has_attn_bias: bool = False, qk_norm_eps: float | None = None):
        tp = get_tp_info()
        if qk_norm_eps is not None:
            raise NotImplementedError("per-head q/k RMSNorm before RoPE is not fused by this library")
        self.head_dim = head_dim
        self.num_qo_heads = div_even(num_qo_heads, tp.size)
        self.num_kv_heads = div_even(num_kv_heads, tp.size, allow_replicate=True)
        self._layer_id = layer_id
        self.qkv_proj = LinearColParallelPartitioned(hidden_size, head_dim,
                                                     [(num_qo_heads, False)] + [(num_kv_heads, True)] * 2,
                                                     has_bias=has_attn_bias)
        self.q_norm = None
        self.k_norm = None
        self.rotary = get_rope(head_dim, rotary_dim, max_position, rope_base, rope_scaling)
        self.o_proj = LinearRowParallel(head_dim * num_qo_heads, hidden_size, has_bias=False)

    def proj_store(self, x: torch.Tensor, positions: torch.Tensor, out_loc: torch.Tensor,
                   k_cache: torch.Tensor, v_cache: torch.Tensor) -> torch.Tensor:
        x2 = _flat2d(x).contiguous()
        q = ops.qkv_rope_store(x2, self.qkv_proj.weight, positions.reshape(-1), out_loc.reshape(-1),
                               self.rotary.cache_on(x2.device), self.num_qo_heads, self.num_kv_heads,
                               self.head_dim, k_cache, v_cache, bias=self.qkv_proj.bias)
        return q.view(*x.shape[:-1], self.num_qo_heads, self.head_dim)


class RMSNormFused(BaseOP):
    """norm.py:56-75 on libpgb kernels, aware of linked row-parallel producers."""

    def __init__(self, size: int, eps: float) -> None:
        self.eps = eps
        self.weight = torch.empty(size)

    def forward(self, x: torch.Tensor, residual: torch.Tensor | None = None):
        f = _CTX.fused
        if f is not None and f[0] is x and f[1] is self and f[2] is residual:
            _CTX.fused = None
            _CTX.residual = residual
            return x, residual
        _CTX.fused = None
        if residual is None:
            out = ops.rmsnorm(x, self.weight, self.eps)
            _CTX.residual = x
            return out, x
        ops.fused_add_rmsnorm(x, residual, self.weight, self.eps)
        _CTX.residual = residual
        return x, residual


def link_fused_norms(layers: list, final_norm: RMSNormFused | None = None) -> int:
    """Link o_proj -> post_attention_layernorm and down_proj -> the next
    layer's input_layernorm (the final norm after the last layer), following
    the decoder wiring of models/llama.py:77-86 and :103-108. Returns the
    number of links made."""
    n = 0
    for i, layer in enumerate(layers):
        attn = getattr(layer, "self_attn", None)
        if attn is not None and isinstance(getattr(attn, "o_proj", None), LinearRowParallel):
            attn.o_proj.link_norm(layer.post_attention_layernorm)
            n += 1
        mlp = getattr(layer, "mlp", None)
        if mlp is not None and isinstance(getattr(mlp, "down_proj", None), LinearRowParallel):
            nxt = layers[i + 1].input_layernorm if i + 1 < len(layers) else final_norm
            mlp.down_proj.link_norm(nxt)
            n += nxt is not None
    return n
