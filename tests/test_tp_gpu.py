"""Tensor-parallel quantized linears on NCCL across 2 GPUs, against the oracle.

Each rank builds the same full AWQ and FP8 layers (same seeds), shards them
with ColumnParallelLinear / RowParallelLinear / TPMLP.from_mlp, and runs its
shard on its own GPU; column outputs are all-gathered, row outputs summed by
the NCCL all-reduce. Rank 0 compares the result with the fp32 oracle of the
unsharded layer (tensor_parallel.py:56-151 semantics: rows [r*N/tp, ...),
columns [r*K/tp, ...), all_reduce(SUM), bias added once). Skipped on a box
with fewer than two GPUs.
"""

import os
import socket

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

from oracle import nsq_oracle as O

pytestmark = pytest.mark.gpu

GEMM_TOL = 1e-2
WS = 2


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _bf16_np(t):
    return O.from_bf16_bits(t.contiguous().view(torch.int16).cpu().numpy().view(np.uint16))


def _awq_full(n, k, gs, seed, bias):
    from nanosglang_b200.quantization import AWQLinear
    rng = np.random.default_rng(seed)
    g = k // gs
    qw = rng.integers(-2 ** 31, 2 ** 31 - 1, (n, k // 8), dtype=np.int64).astype(np.int32)
    s = (rng.random((n, g)) * 0.009 + 0.001).astype(np.float16)
    z = rng.integers(0, 16, (n, g)).astype(np.float16)
    m = AWQLinear(k, n, gs, bias=bias).cuda()
    m.qweight.copy_(torch.from_numpy(qw))
    m.scales.copy_(torch.from_numpy(s))
    m.zeros.copy_(torch.from_numpy(z))
    b = None
    if bias:
        b = (torch.randn(n, generator=torch.Generator().manual_seed(seed + 1)) * 0.1).to(torch.bfloat16)
        m.bias = torch.nn.Parameter(b.cuda())
    return m, (qw, s, z, b)


def _fp8_full(n, k, seed):
    from nanosglang_b200.quantization import FP8Linear
    rng = np.random.default_rng(seed)
    w = (rng.standard_normal((n, k)) * 0.02).astype(np.float32)
    codes, scale = O.fp8_quantize(w)
    m = FP8Linear(k, n).cuda()
    m.weight_fp8 = torch.from_numpy(codes).cuda().view(torch.float8_e4m3fn)
    m.weight_scale = torch.tensor(scale).cuda()
    return m, (codes, scale)


def _worker(rank, port, q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    os.environ["LOCAL_RANK"] = str(rank)
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    import torch.distributed as dist

    from nanosglang_b200 import tensor_parallel as TP
    res = {}
    try:
        TP.init_distributed(rank, WS, backend="nccl", timeout_s=120)
        k, n, gs = 1024, 2048, 128
        for m_tok in (16, 300):  # decode kernel and tcgen05 prefill kernel per shard
            x = torch.randn(m_tok, k, generator=torch.Generator().manual_seed(m_tok)).to(torch.bfloat16)
            xd = x.cuda()
            # AWQ column-parallel (with bias) and row-parallel
            col, (qw, s, z, b) = _awq_full(n, k, gs, seed=1, bias=True)
            cp = TP.ColumnParallelLinear.from_linear(col, WS, rank, gather_output=True)
            y = cp(xd)
            ref = O.awq_linear(x.float().numpy(), qw, s, z, k, gs, b.float().numpy())
            res[f"awq_col_m{m_tok}"] = O.rel_fro(_bf16_np(y), ref)
            row, (qw, s, z, _) = _awq_full(k, n, gs, seed=2, bias=False)
            rp = TP.RowParallelLinear.from_linear(row, WS, rank)
            c0, c1 = O.row_shard_cols(n, WS, rank)
            xr = torch.randn(m_tok, n, generator=torch.Generator().manual_seed(m_tok + 1)).to(torch.bfloat16)
            y = rp(xr[:, c0:c1].contiguous().cuda())
            ref = O.awq_linear(xr.float().numpy(), qw, s, z, n, gs)
            res[f"awq_row_m{m_tok}"] = O.rel_fro(_bf16_np(y), ref)
            # FP8 column / row
            col8, (codes, scale) = _fp8_full(n, k, seed=3)
            y = TP.ColumnParallelLinear.from_linear(col8, WS, rank, gather_output=True)(xd)
            res[f"fp8_col_m{m_tok}"] = O.rel_fro(_bf16_np(y), O.fp8_linear(x.float().numpy(), codes, scale))
            row8, (codes, scale) = _fp8_full(k, n, seed=4)
            y = TP.RowParallelLinear.from_linear(row8, WS, rank)(xr[:, c0:c1].contiguous().cuda())
            res[f"fp8_row_m{m_tok}"] = O.rel_fro(_bf16_np(y), O.fp8_linear(xr.float().numpy(), codes, scale))
            # MLP: gate/up column-parallel, down row-parallel + all-reduce
            mlp = torch.nn.Module()
            mlp.gate_proj, (gq, gsc, gz, _) = _awq_full(n, k, gs, seed=5, bias=False)
            mlp.up_proj, (uq, usc, uz, _) = _awq_full(n, k, gs, seed=6, bias=False)
            mlp.down_proj, (dq, dsc, dz, _) = _awq_full(k, n, gs, seed=7, bias=False)
            y = TP.TPMLP.from_mlp(mlp, WS, rank)(xd)
            g = O.awq_linear(x.float().numpy(), gq, gsc, gz, k, gs)
            u = O.awq_linear(x.float().numpy(), uq, usc, uz, k, gs)
            h = O.bf16_round((g / (1.0 + np.exp(-g))) * u)  # the kernel reads bf16 activations
            ref = O.awq_linear(h, dq, dsc, dz, n, gs)
            res[f"awq_mlp_m{m_tok}"] = O.rel_fro(_bf16_np(y), ref)
        # prefill-sized row-parallel input with the opt-in overlap: chunked GEMMs
        # with the all-reduces on a side stream (RowParallelLinear.overlap_min_tokens)
        row8, (codes, scale) = _fp8_full(k, n, seed=8)
        xr = torch.randn(4096, n, generator=torch.Generator().manual_seed(9)).to(torch.bfloat16)
        c0, c1 = O.row_shard_cols(n, WS, rank)
        rp = TP.RowParallelLinear.from_linear(row8, WS, rank)
        rp.overlap_min_tokens = 2048  # opt in for this layer
        y = rp(xr[:, c0:c1].contiguous().cuda())
        res["fp8_row_overlapped_m4096"] = O.rel_fro(_bf16_np(y), O.fp8_linear(xr.float().numpy(), codes, scale))
        torch.cuda.synchronize()
        dist.barrier()
        dist.destroy_process_group()
        q.put((rank, res))
    except Exception as e:  # surface worker failures to the test
        q.put((rank, repr(e)))


def test_tp_quantized_linears_on_nccl():
    if torch.cuda.device_count() < WS:
        pytest.skip(f"needs {WS} GPUs")
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, port, q)) for r in range(WS)]
    for p in procs:
        p.start()
    results = [q.get(timeout=600) for _ in range(WS)]
    for p in procs:
        p.join(timeout=120)
    for rank, res in results:
        assert not isinstance(res, str), f"rank {rank}: {res}"
        for name, err in res.items():
            assert err <= GEMM_TOL, f"rank {rank} {name}: rel err {err}"
