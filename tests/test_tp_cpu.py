"""Tensor-parallel host logic on CPU: shard math of dense / AWQ / FP8 buffers
against the oracle, and the row-parallel all-reduce path on world_size-2 gloo
ranks (the exchange NCCL performs on the GPU)."""

import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp
import torch.nn as nn

from oracle import nsq_oracle as O
from nanosglang_b200 import quantization as Q
from nanosglang_b200 import tensor_parallel as TP


def _rand_awq(n, k, gs, seed):
    rng = np.random.default_rng(seed)
    m = Q.AWQLinear(k, n, gs, bias=True)
    m.qweight.copy_(torch.from_numpy(rng.integers(-2 ** 31, 2 ** 31 - 1, (n, k // 8), dtype=np.int64)
                                     .astype(np.int32)))
    m.scales.copy_(torch.from_numpy((rng.random((n, m.num_groups)) * 0.009 + 0.001).astype(np.float16)))
    m.zeros.copy_(torch.from_numpy(rng.integers(0, 16, (n, m.num_groups)).astype(np.float16)))
    with torch.no_grad():
        m.bias.copy_(torch.randn(n))
    return m


def _deq(m):
    return O.awq_dequant(m.qweight.numpy(), m.scales.numpy(), m.zeros.numpy(), m.in_features, m.group_size)


@pytest.mark.parametrize("ws", [2, 4])
def test_awq_column_and_row_shards_dequantise_to_slices(ws):
    full = _rand_awq(64, 1024, 128, seed=ws)
    wf = _deq(full)
    for r in range(ws):
        col = TP.shard_linear_rows(full, ws, r)
        r0, r1 = O.column_shard_rows(64, ws, r)
        assert np.array_equal(_deq(col).view(np.uint16), wf[r0:r1].view(np.uint16))
        assert torch.equal(col.bias.data, full.bias.data[r0:r1])
        row = TP.shard_linear_cols(full, ws, r, keep_bias=(r == 0))
        c0, c1 = O.row_shard_cols(1024, ws, r)
        assert np.array_equal(_deq(row).view(np.uint16), wf[:, c0:c1].view(np.uint16))
        assert (row.bias is not None) == (r == 0)


def test_awq_row_shard_rejects_straddling_groups():
    full = _rand_awq(16, 896, 128, seed=0)
    with pytest.raises(ValueError, match="group_size"):
        TP.shard_linear_cols(full, 2, 0, keep_bias=True)  # 448 % 128 != 0


def test_fp8_shards_keep_scale():
    m = Q.FP8Linear(256, 64, bias=True)
    m.weight_fp8 = torch.randn(64, 256).to(torch.float8_e4m3fn)
    m.weight_scale = torch.tensor(0.0125)
    for r in range(4):
        col = TP.shard_linear_rows(m, 4, r)
        assert torch.equal(col.weight_fp8.view(torch.uint8), m.weight_fp8.view(torch.uint8)[16 * r:16 * (r + 1)])
        assert torch.equal(col.weight_scale, m.weight_scale) and col.weight_scale.shape == m.weight_scale.shape
        row = TP.shard_linear_cols(m, 4, r, keep_bias=(r == 0))
        assert torch.equal(row.weight_fp8.view(torch.uint8), m.weight_fp8.view(torch.uint8)[:, 64 * r:64 * (r + 1)])
        assert row.weight_fp8.is_contiguous()


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, ws, port, q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    try:
        TP.init_distributed(rank, ws, backend="gloo", timeout_s=60)
        torch.manual_seed(0)
        full_row = nn.Linear(64, 32, bias=True)
        full_col = nn.Linear(32, 48, bias=True)
        x = torch.randn(5, 64)
        mlp = nn.Module()
        mlp.gate_proj = nn.Linear(32, 64, bias=False)
        mlp.up_proj = nn.Linear(32, 64, bias=False)
        mlp.down_proj = nn.Linear(64, 32, bias=False)
        xm = torch.randn(3, 32)
        row = TP.RowParallelLinear.from_linear(full_row, ws, rank)
        c0, c1 = O.row_shard_cols(64, ws, rank)
        y_row = row(x[:, c0:c1])
        col = TP.ColumnParallelLinear.from_linear(full_col, ws, rank, gather_output=True)
        y_col = col(y_row)
        # MLP through TPMLP.from_mlp
        tpm = TP.TPMLP.from_mlp(mlp, ws, rank)
        ref_m = mlp.down_proj(torch.nn.functional.silu(mlp.gate_proj(xm)) * mlp.up_proj(xm))
        with torch.no_grad():
            q.put((rank, (y_row - full_row(x)).abs().max().item(),
                   (y_col - full_col(full_row(x))).abs().max().item(),
                   (tpm(xm) - ref_m).abs().max().item()))
        dist.barrier()
        dist.destroy_process_group()
    except Exception as e:  # surface worker failures to the test
        q.put((rank, repr(e), None, None))


def test_row_and_column_parallel_on_gloo_ranks():
    ws = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, ws, port, q)) for r in range(ws)]
    for p in procs:
        p.start()
    results = [q.get(timeout=120) for _ in range(ws)]
    for p in procs:
        p.join(timeout=60)
    for rank, e_row, e_col, e_mlp in results:
        assert not isinstance(e_row, str), e_row
        assert e_row < 1e-5, f"rank {rank}: row-parallel sum differs ({e_row})"
        assert e_col < 1e-5, f"rank {rank}: column-parallel gather differs ({e_col})"
        assert e_mlp < 1e-5, f"rank {rank}: TP MLP differs ({e_mlp})"


def test_tensor_parallel_model_updates_heads():
    class Cfg:
        num_attention_heads = 4
        num_key_value_heads = 2
        head_dim = 8
        hidden_size = 32
        intermediate_size = 64

    class Attn(nn.Module):
        def __init__(self):
            super().__init__()
            self.q_proj = nn.Linear(32, 32, bias=True)
            self.k_proj = nn.Linear(32, 16, bias=True)
            self.v_proj = nn.Linear(32, 16, bias=True)
            self.o_proj = nn.Linear(32, 32, bias=False)
            self.num_heads, self.num_kv_heads = 4, 2

    class Layer(nn.Module):
        def __init__(self):
            super().__init__()
            self.self_attn = Attn()
            self.mlp = nn.Module()
            self.mlp.gate_proj = nn.Linear(32, 64, bias=False)
            self.mlp.up_proj = nn.Linear(32, 64, bias=False)
            self.mlp.down_proj = nn.Linear(64, 32, bias=False)

    class M(nn.Module):
        def __init__(self):
            super().__init__()
            self.config = Cfg()
            self.layers = nn.ModuleList([Layer()])

    m = M()
    qb = m.layers[0].self_attn.q_proj.bias.data.clone()
    TP.tensor_parallel_model(m, 2, 1)
    a = m.layers[0].self_attn
    assert a.num_heads == 2 and a.num_kv_heads == 1
    assert a.q_proj.linear.weight.shape == (16, 32)
    assert torch.equal(a.q_proj.linear.bias.data, qb[16:])
    assert a.o_proj.linear.weight.shape == (32, 16) and a.o_proj.linear.bias is None
    assert isinstance(m.layers[0].mlp, TP.TPMLP)
