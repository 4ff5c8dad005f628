"""One-shot NVLink peer all-reduce (nanosglang_b200.peer, nsq_peer_allreduce)
on 2 GPUs against NCCL's all_reduce of the same data: the sum of the row-
parallel partials (tensor_parallel.py:134-140 semantics), bit-identical on
every rank, across alternating parities, inside a CUDA graph, and for every
activation dtype. Skipped on a box with fewer than two GPUs."""

import os
import socket

import pytest
import torch
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu

WS = 2


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, port, q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    import torch.distributed as dist

    from nanosglang_b200 import _lib
    from nanosglang_b200.peer import PeerAllReduce
    res = {}
    try:
        torch.cuda.set_device(rank)
        dist.init_process_group("nccl", rank=rank, world_size=WS, device_id=torch.device("cuda", rank))
        _lib.device_status_reset()
        peer = PeerAllReduce(max_bytes=1 << 20)
        g = torch.Generator(device="cuda").manual_seed(100 + rank)

        def check(name, shape, dtype, calls=3):
            worst = 0.0
            for c in range(calls):  # alternating parities
                t = torch.randn(*shape, generator=g, device="cuda").to(dtype)
                ref = t.clone()
                dist.all_reduce(ref)
                assert peer.reduce_(t)
                err = ((t.float() - ref.float()).norm() / ref.float().norm()).item()
                worst = max(worst, err)
                mine = t.contiguous().view(torch.uint8)
                other = torch.empty_like(mine)
                dist.broadcast(other.copy_(mine), src=0)
                res[f"{name}_identical_{c}"] = bool(torch.equal(mine, other))
            res[f"{name}_err"] = worst

        check("bf16_64x4096", (64, 4096), torch.bfloat16)
        check("bf16_16x896", (16, 896), torch.bfloat16)
        check("fp16_8x1024", (8, 1024), torch.float16)
        check("f32_3x1024", (3, 1024), torch.float32)
        # too large for the workspace: declines, caller falls back
        big = torch.zeros(1 << 20, device="cuda", dtype=torch.bfloat16)
        res["declines_large"] = not peer.reduce_(big)
        # inside a CUDA graph: three reductions per replay, replayed twice
        bufs = [torch.zeros(32, 4096, device="cuda", dtype=torch.bfloat16) for _ in range(3)]
        s = torch.cuda.Stream()
        s.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(s):
            for b in bufs:
                peer.reduce_(b)
        torch.cuda.synchronize()
        gph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(gph, stream=s):
            for b in bufs:
                peer.reduce_(b)
        for rep in range(2):
            vals = [torch.randn(32, 4096, generator=g, device="cuda").to(torch.bfloat16) for _ in bufs]
            refs = []
            for b, v in zip(bufs, vals):
                b.copy_(v)
                r = v.clone()
                dist.all_reduce(r)
                refs.append(r)
            gph.replay()
            torch.cuda.synchronize()
            res[f"graph_err_{rep}"] = max(((b.float() - r.float()).norm() / r.float().norm()).item()
                                          for b, r in zip(bufs, refs))
        del gph
        torch.cuda.synchronize()
        res["status"] = _lib.device_status()[0]
        peer.close()
        dist.barrier()
        dist.destroy_process_group()
        q.put((rank, res))
    except Exception as e:  # surface worker failures to the test
        q.put((rank, repr(e)))


def test_peer_allreduce_matches_nccl_on_two_gpus():
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
        assert res["status"] == 0
        assert res["declines_large"]
        for k, v in res.items():
            if k.endswith("_err") or k.startswith("graph_err"):
                assert v <= 1e-2, (rank, k, v)
            if "_identical_" in k:
                assert v, (rank, k)
