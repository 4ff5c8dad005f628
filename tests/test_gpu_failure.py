"""Failure path of the bounded device-side waits, on the GPU, without a fault.

The multi-wave decode kernel is asked (through a test hook of the C ABI) never
to request one weight box, so one of its waits can never complete: a flag that
nothing sets. With a short wait limit the kernel must record
NSQ_EDEVICE_TIMEOUT with its wait tag in the device status word, let every
copy it did request land, and return; the context must stay usable, so the
same call without the hook afterwards matches the oracle."""

import numpy as np
import pytest
import torch

from oracle import nsq_oracle as O

pytestmark = pytest.mark.gpu

GEMM_TOL = 1e-2
DECODE_WAIT_TAG = 1  # the multi-wave decode kernel's weight-box wait


@pytest.fixture(scope="module", autouse=True)
def _cuda():
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")


def _inputs():
    rng = np.random.default_rng(11)
    n, k, gs, m = 9728, 896, 128, 16  # config 0: the multi-wave decode kernel's shape
    qw = rng.integers(-2 ** 31, 2 ** 31 - 1, (n, k // 8), dtype=np.int64).astype(np.int32)
    s = (rng.random((n, k // gs)) * 0.009 + 0.001).astype(np.float16)
    z = rng.integers(0, 16, (n, k // gs)).astype(np.float16)
    x = torch.randn(m, k, generator=torch.Generator().manual_seed(12)).to(torch.bfloat16)
    return (qw, s, z), tuple(torch.from_numpy(a).cuda() for a in (qw, s, z)), x, k, gs


def test_bounded_wait_runs_out_and_context_survives():
    from nanosglang_b200 import _lib, ops
    (qw, s, z), (tq, ts, tz), x, k, gs = _inputs()
    xd = x.cuda()
    torch.cuda.synchronize()
    _lib.device_status_reset()
    _lib.set_wait_limit_ns(1_000_000)  # 1 ms
    prev = _lib.withhold_weight_load_for_test(True)
    try:
        ops.awq_linear(xd, tq, ts, tz, gs)
        torch.cuda.synchronize()  # the kernel returns: no hang, no fault
    finally:
        _lib.withhold_weight_load_for_test(prev)
    code, where, block = _lib.device_status()
    assert code == _lib.EDEVICE_TIMEOUT, (code, where, block)
    assert where == DECODE_WAIT_TAG
    assert 0 <= block < 4096
    # the status word and the limit reset; the context still runs kernels
    _lib.device_status_reset()
    y = ops.awq_linear(xd, tq, ts, tz, gs)
    torch.cuda.synchronize()
    assert _lib.device_status()[0] == 0
    ref = O.awq_linear(x.float().numpy(), qw, s, z, k, gs)
    yf = O.from_bf16_bits(y.view(torch.int16).cpu().numpy().view(np.uint16))
    assert O.rel_fro(yf, ref) <= GEMM_TOL
