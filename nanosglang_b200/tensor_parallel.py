"""Tensor parallelism for the quantized linears, one process per GPU.

Same public names and constructor signatures as
``nano_sglang/distributed/tensor_parallel.py`` (xiehuanyi/nanoSGLang):
``init_distributed``, ``ColumnParallelLinear``, ``RowParallelLinear``,
``TPAttention``, ``TPMLP`` and ``tensor_parallel_model``. The reference's
versions only handle dense ``nn.Linear`` weights, build shards on the CPU in
fp32, crash on Qwen2's q/k/v bias and on quantized layers, and add the
row-parallel bias on every rank before the reduction. This module shards
dense, ``AWQLinear`` and ``FP8Linear`` layers in place on their own device and
dtype:

  column parallel (q, k, v, gate, up)  rows [r*N/tp, (r+1)*N/tp) of the
        weight (qweight/scales/zeros rows for AWQ, weight_fp8 rows for FP8)
        and of the bias; no communication.
  row parallel (o, down)  input columns [r*K/tp, (r+1)*K/tp) (qweight words,
        scale/zero groups for AWQ; weight_fp8 columns for FP8), then one
        ``all_reduce(SUM)`` of the partial [M, hidden] output over NCCL on the
        current stream (graph-capturable). Opt-in (``overlap_min_tokens``):
        the rows are split into chunks and each chunk's all-reduce runs on a
        side stream while the next chunk's GEMM runs. The bias is kept on rank 0
        only so it is added exactly once, inside rank 0's GEMM epilogue.
"""

from __future__ import annotations

import datetime
import os
from typing import Optional

import torch
import torch.distributed as dist
import torch.nn as nn

from .quantization import AWQLinear, FP8Linear

__all__ = [
    "init_distributed", "ColumnParallelLinear", "RowParallelLinear", "TPAttention", "TPMLP",
    "tensor_parallel_model", "shard_linear_rows", "shard_linear_cols", "enable_peer_allreduce",
    "disable_peer_allreduce",
]


def init_distributed(rank: Optional[int] = None, world_size: Optional[int] = None, backend: str = "nccl",
                     timeout_s: float = 600.0):
    """Initialize the process group from RANK / WORLD_SIZE (as tensor_parallel.py:31-53).

    Returns (rank, world_size). The CUDA device is LOCAL_RANK when set (one
    process per GPU under torchrun), else ``rank``.
    """
    if rank is None:
        rank = int(os.environ.get("RANK", 0))
    if world_size is None:
        world_size = int(os.environ.get("WORLD_SIZE", 1))
    if world_size <= 1:
        return rank, world_size
    if not dist.is_initialized():
        dist.init_process_group(backend=backend, rank=rank, world_size=world_size,
                                timeout=datetime.timedelta(seconds=timeout_s))
    if backend == "nccl":
        torch.cuda.set_device(int(os.environ.get("LOCAL_RANK", rank)))
    return rank, world_size


# ---------------------------------------------------------------------------
# Sharding of one linear (dense, AWQ or FP8)
# ---------------------------------------------------------------------------


def _span(total: int, world_size: int, rank: int, what: str):
    if total % world_size != 0:
        raise ValueError(f"{what}={total} is not divisible by world_size={world_size}")
    per = total // world_size
    return rank * per, (rank + 1) * per


def shard_linear_rows(module: nn.Module, world_size: int, rank: int) -> nn.Module:
    """Output-dim (column-parallel) shard of a dense / AWQ / FP8 linear."""
    if isinstance(module, AWQLinear):
        r0, r1 = _span(module.out_features, world_size, rank, "out_features")
        dev = module.qweight.device
        with torch.device(dev):
            out = AWQLinear(module.in_features, r1 - r0, module.group_size, bias=module.bias is not None)
        out.qweight.copy_(module.qweight[r0:r1])
        out.scales.copy_(module.scales[r0:r1])
        out.zeros.copy_(module.zeros[r0:r1])
        if module.bias is not None:
            out.bias = nn.Parameter(module.bias.data[r0:r1].clone())
        return out
    if isinstance(module, FP8Linear):
        r0, r1 = _span(module.out_features, world_size, rank, "out_features")
        with torch.device(module.weight_fp8.device):
            out = FP8Linear(module.in_features, r1 - r0, bias=module.bias is not None)
        out.weight_fp8 = module.weight_fp8[r0:r1].contiguous()
        out.weight_scale = module.weight_scale.clone()
        if module.bias is not None:
            out.bias = nn.Parameter(module.bias.data[r0:r1].clone())
        return out
    if isinstance(module, nn.Linear):
        r0, r1 = _span(module.out_features, world_size, rank, "out_features")
        w = module.weight.data
        out = nn.Linear(module.in_features, r1 - r0, bias=module.bias is not None, device=w.device, dtype=w.dtype)
        out.weight.data.copy_(w[r0:r1])
        if module.bias is not None:
            out.bias.data.copy_(module.bias.data[r0:r1])
        return out
    raise TypeError(f"cannot shard {type(module).__name__}")


def shard_linear_cols(module: nn.Module, world_size: int, rank: int, keep_bias: bool) -> nn.Module:
    """Input-dim (row-parallel) shard; the bias survives only where keep_bias."""
    has_bias = module.bias is not None and keep_bias
    if isinstance(module, AWQLinear):
        c0, c1 = _span(module.in_features, world_size, rank, "in_features")
        gs = module.group_size
        if (c1 - c0) % gs != 0 or (c1 - c0) % 8 != 0:
            raise ValueError(
                f"row-parallel AWQ needs in_features/world_size ({c1 - c0}) to be a multiple of "
                f"group_size ({gs}) so no quantisation group straddles two ranks")
        with torch.device(module.qweight.device):
            out = AWQLinear(c1 - c0, module.out_features, gs, bias=has_bias)
        out.qweight.copy_(module.qweight[:, c0 // 8:c1 // 8])
        out.scales.copy_(module.scales[:, c0 // gs:c1 // gs])
        out.zeros.copy_(module.zeros[:, c0 // gs:c1 // gs])
        if has_bias:
            out.bias = nn.Parameter(module.bias.data.clone())
        return out
    if isinstance(module, FP8Linear):
        c0, c1 = _span(module.in_features, world_size, rank, "in_features")
        with torch.device(module.weight_fp8.device):
            out = FP8Linear(c1 - c0, module.out_features, bias=has_bias)
        out.weight_fp8 = module.weight_fp8[:, c0:c1].contiguous()
        out.weight_scale = module.weight_scale.clone()
        if has_bias:
            out.bias = nn.Parameter(module.bias.data.clone())
        return out
    if isinstance(module, nn.Linear):
        c0, c1 = _span(module.in_features, world_size, rank, "in_features")
        w = module.weight.data
        out = nn.Linear(c1 - c0, module.out_features, bias=has_bias, device=w.device, dtype=w.dtype)
        out.weight.data.copy_(w[:, c0:c1])
        if has_bias:
            out.bias.data.copy_(module.bias.data)
        return out
    raise TypeError(f"cannot shard {type(module).__name__}")


# ---------------------------------------------------------------------------
# Parallel layers
# ---------------------------------------------------------------------------


class ColumnParallelLinear(nn.Module):
    """Linear split along the output dimension (tensor_parallel.py:56-105).

    Each rank holds rows [rank*N/tp, (rank+1)*N/tp) of the weight; the output
    stays sharded unless ``gather_output``.
    """

    def __init__(self, in_features: int, out_features: int, world_size: int, rank: int, bias: bool = False,
                 gather_output: bool = False, linear: Optional[nn.Module] = None):
        super().__init__()
        assert out_features % world_size == 0
        self.out_features_per_rank = out_features // world_size
        self.world_size = world_size
        self.rank = rank
        self.gather_output = gather_output
        self.linear = linear if linear is not None else nn.Linear(in_features, self.out_features_per_rank, bias=bias)

    @classmethod
    def from_linear(cls, module: nn.Module, world_size: int, rank: int,
                    gather_output: bool = False) -> "ColumnParallelLinear":
        shard = shard_linear_rows(module, world_size, rank)
        return cls(module.in_features, module.out_features, world_size, rank, gather_output=gather_output,
                   linear=shard)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        output = self.linear(x)
        if self.gather_output and self.world_size > 1:
            gathered = [torch.empty_like(output) for _ in range(self.world_size)]
            dist.all_gather(gathered, output.contiguous())
            output = torch.cat(gathered, dim=-1)
        return output

    def load_weight_shard(self, full_weight: torch.Tensor, full_bias: Optional[torch.Tensor] = None):
        """Copy this rank's rows of a full dense weight (tensor_parallel.py:93-105)."""
        r0 = self.rank * self.out_features_per_rank
        r1 = r0 + self.out_features_per_rank
        self.linear.weight.data.copy_(full_weight[r0:r1])
        if full_bias is not None and self.linear.bias is not None:
            self.linear.bias.data.copy_(full_bias[r0:r1])


_SIDE_STREAMS = {}
_PEER = None  # a peer.PeerAllReduce once enable_peer_allreduce() ran


def enable_peer_allreduce(max_bytes: int = 4 << 20, group=None):
    """Reduce row-parallel outputs of at most ``max_bytes`` with the one-shot
    NVLink peer all-reduce (nanosglang_b200.peer) instead of NCCL; larger ones
    keep ``dist.all_reduce``. Collective: every rank calls it once."""
    global _PEER
    from .peer import PeerAllReduce
    if _PEER is None:
        _PEER = PeerAllReduce(max_bytes=max_bytes, group=group)
    return _PEER


def disable_peer_allreduce():
    """Back to NCCL for every row-parallel output (collective)."""
    global _PEER
    if _PEER is not None:
        _PEER.close()
        _PEER = None


def _all_reduce_sum(t: torch.Tensor) -> None:
    if _PEER is not None and _PEER.reduce_(t):
        return
    dist.all_reduce(t, op=dist.ReduceOp.SUM)


def _side_stream(device) -> torch.cuda.Stream:
    """One side stream per device for the overlapped row-parallel reductions."""
    key = torch.device(device).index
    if key not in _SIDE_STREAMS:
        _SIDE_STREAMS[key] = torch.cuda.Stream(device)
    return _SIDE_STREAMS[key]


class RowParallelLinear(nn.Module):
    """Linear split along the input dimension + all-reduce (tensor_parallel.py:108-151).

    Each rank holds columns [rank*K/tp, (rank+1)*K/tp) of the weight and
    receives the matching slice of x; partial outputs are summed with one
    ``all_reduce``. A bias lives on rank 0's shard only.
    """

    def __init__(self, in_features: int, out_features: int, world_size: int, rank: int, bias: bool = False,
                 reduce_output: bool = True, linear: Optional[nn.Module] = None):
        super().__init__()
        assert in_features % world_size == 0
        self.in_features_per_rank = in_features // world_size
        self.world_size = world_size
        self.rank = rank
        self.reduce_output = reduce_output
        self.linear = linear if linear is not None else nn.Linear(
            self.in_features_per_rank, out_features, bias=bias and rank == 0)

    @classmethod
    def from_linear(cls, module: nn.Module, world_size: int, rank: int,
                    reduce_output: bool = True) -> "RowParallelLinear":
        shard = shard_linear_cols(module, world_size, rank, keep_bias=(rank == 0))
        return cls(module.in_features, module.out_features, world_size, rank, reduce_output=reduce_output,
                   linear=shard)

    # Opt-in: prefill-sized inputs split into token chunks, the all-reduce of
    # one chunk (on a side stream) running while the next chunk's GEMM does,
    # with the GEMMs leaving `overlap_sm_reserve` SMs free for the collective.
    # Off by default (overlap_min_tokens = None): on B200 with NCCL, the
    # serial GEMM + all_reduce was faster on the measured shapes.
    overlap_min_tokens = None
    overlap_chunks = 4
    overlap_sm_reserve = 24

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        if not (self.reduce_output and self.world_size > 1):
            return self.linear(x)
        lead = x.shape[:-1]
        x2 = x.reshape(-1, x.shape[-1])
        m = x2.shape[0]
        if self.overlap_min_tokens is None or m < self.overlap_min_tokens or not x2.is_cuda:
            output = self.linear(x2)
            _all_reduce_sum(output)
            return output.reshape(*lead, output.shape[-1])
        return self._forward_overlapped(x2).reshape(*lead, -1)

    def _forward_overlapped(self, x2: torch.Tensor) -> torch.Tensor:
        """GEMM chunk i+1 on the current stream while chunk i is all-reduced on
        a side stream; the caller's stream waits for the last reduction. Same
        result as one GEMM + one all_reduce (each output row is reduced once)."""
        compute = torch.cuda.current_stream(x2.device)
        side = _side_stream(x2.device)
        side.wait_stream(compute)
        m = x2.shape[0]
        step = (m + self.overlap_chunks - 1) // self.overlap_chunks
        step = (step + 127) // 128 * 128
        parts = []
        from . import _lib
        prev = _lib.set_sm_reserve(self.overlap_sm_reserve)
        try:
            for r0 in range(0, m, step):
                parts.append(self._chunk(x2[r0:r0 + step], compute, side))
        finally:
            _lib.set_sm_reserve(prev)
        compute.wait_stream(side)
        return torch.cat(parts) if len(parts) > 1 else parts[0]

    def _chunk(self, xc, compute, side):
        """GEMM of one token chunk on the compute stream; its all-reduce on the side stream."""
        y = self.linear(xc)
        done = torch.cuda.Event()
        done.record(compute)
        side.wait_event(done)
        with torch.cuda.stream(side):
            dist.all_reduce(y, op=dist.ReduceOp.SUM)
        y.record_stream(side)
        return y

    def load_weight_shard(self, full_weight: torch.Tensor, full_bias: Optional[torch.Tensor] = None):
        """Copy this rank's columns of a full dense weight (tensor_parallel.py:142-151);
        the bias goes to rank 0 only."""
        c0 = self.rank * self.in_features_per_rank
        c1 = c0 + self.in_features_per_rank
        self.linear.weight.data.copy_(full_weight[:, c0:c1])
        if full_bias is not None and self.linear.bias is not None:
            self.linear.bias.data.copy_(full_bias)


class TPAttention(nn.Module):
    """Container of the sharded attention projections (tensor_parallel.py:154-203).

    Kept for API compatibility with the reference, which also leaves its
    forward unimplemented: the attention computation belongs to the model,
    and ``tensor_parallel_model`` shards the projections of an existing
    attention module in place (and sets its per-rank head counts) instead of
    replacing it with this class. Its projections are usable directly
    (``q_proj`` .. ``o_proj`` are Column/RowParallelLinear).
    """

    def __init__(self, hidden_size: int, num_heads: int, num_kv_heads: int, head_dim: int, world_size: int,
                 rank: int, bias: bool = False):
        super().__init__()
        assert num_heads % world_size == 0
        assert num_kv_heads % world_size == 0
        self.num_heads_per_rank = num_heads // world_size
        self.num_kv_heads_per_rank = num_kv_heads // world_size
        self.head_dim = head_dim
        self.world_size = world_size
        self.rank = rank
        self.q_proj = ColumnParallelLinear(hidden_size, num_heads * head_dim, world_size, rank, bias=bias)
        self.k_proj = ColumnParallelLinear(hidden_size, num_kv_heads * head_dim, world_size, rank, bias=bias)
        self.v_proj = ColumnParallelLinear(hidden_size, num_kv_heads * head_dim, world_size, rank, bias=bias)
        self.o_proj = RowParallelLinear(num_heads * head_dim, hidden_size, world_size, rank, bias=False,
                                        reduce_output=True)

    def forward(self, hidden_states, **kwargs):
        raise NotImplementedError(
            "Full TP attention forward requires integration with the main model. "
            "See tensor_parallel_model() for how to replace layers.")


class TPMLP(nn.Module):
    """SwiGLU MLP with column-parallel gate/up and row-parallel down (tensor_parallel.py:206-233)."""

    def __init__(self, hidden_size: int, intermediate_size: int, world_size: int, rank: int):
        super().__init__()
        self.gate_proj = ColumnParallelLinear(hidden_size, intermediate_size, world_size, rank)
        self.up_proj = ColumnParallelLinear(hidden_size, intermediate_size, world_size, rank)
        self.down_proj = RowParallelLinear(intermediate_size, hidden_size, world_size, rank, reduce_output=True)

    @classmethod
    def from_mlp(cls, mlp: nn.Module, world_size: int, rank: int) -> "TPMLP":
        out = cls.__new__(cls)
        nn.Module.__init__(out)
        out.gate_proj = ColumnParallelLinear.from_linear(mlp.gate_proj, world_size, rank)
        out.up_proj = ColumnParallelLinear.from_linear(mlp.up_proj, world_size, rank)
        out.down_proj = RowParallelLinear.from_linear(mlp.down_proj, world_size, rank)
        return out

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        fused = getattr(self, "gate_up", None)  # a GateUpSiLU over this rank's gate/up shards, if installed
        if fused is not None:
            return self.down_proj(fused(x))
        return self.down_proj(torch.nn.functional.silu(self.gate_proj(x)) * self.up_proj(x))


def tensor_parallel_model(model, world_size: int, rank: int):
    """Shard every decoder layer's projections in place (tensor_parallel.py:236-301).

    Works for dense, AWQ and FP8 projections (quantize before or after), keeps
    each shard on the layer's device and dtype, shards q/k/v biases with their
    rows, and updates the attention head counts for this rank.
    """
    if world_size <= 1:
        return model
    config = model.config
    assert config.num_attention_heads % world_size == 0, "num_attention_heads must divide by world_size"
    assert config.num_key_value_heads % world_size == 0, "num_key_value_heads must divide by world_size"
    for layer in model.layers:
        layer.mlp = TPMLP.from_mlp(layer.mlp, world_size, rank)
        attn = layer.self_attn
        attn.q_proj = ColumnParallelLinear.from_linear(attn.q_proj, world_size, rank)
        attn.k_proj = ColumnParallelLinear.from_linear(attn.k_proj, world_size, rank)
        attn.v_proj = ColumnParallelLinear.from_linear(attn.v_proj, world_size, rank)
        attn.o_proj = RowParallelLinear.from_linear(attn.o_proj, world_size, rank)
        attn.num_heads = config.num_attention_heads // world_size
        attn.num_kv_heads = config.num_key_value_heads // world_size
    return model
