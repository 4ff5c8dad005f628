"""Fused projections for decode batches (row-streaming kernel) against the
oracle: q/k/v (or any 1..3 layers reading the same x) in one launch, and
gate/up with SiLU(gate) * up applied in the epilogue (causal_lm.py:482).
Tolerance: relative Frobenius error <= 1e-2 against the fp32 oracle."""

import numpy as np
import pytest
import torch

from oracle import nsq_oracle as O

pytestmark = pytest.mark.gpu

GEMM_TOL = 1e-2


@pytest.fixture(scope="module", autouse=True)
def _cuda():
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    from nanosglang_b200 import _lib
    _lib.device_status_reset()
    yield
    code, where, block = _lib.device_status()
    assert code == 0, f"device status {code} (wait tag {where}, block {block})"


def _np(t):
    if t.dtype == torch.bfloat16:
        return O.from_bf16_bits(t.contiguous().view(torch.int16).cpu().numpy().view(np.uint16))
    return t.float().cpu().numpy()


def _awq_layer(k, n, seed, bias, dtype=torch.bfloat16, zm="int"):
    from nanosglang_b200.quantization import AWQLinear
    rng = np.random.default_rng(seed)
    g = k // 128
    qw = rng.integers(-2 ** 31, 2 ** 31 - 1, (n, k // 8), dtype=np.int64).astype(np.int32)
    s = (rng.random((n, g)) * 0.009 + 0.001).astype(np.float16)
    z = rng.integers(0, 16, (n, g)).astype(np.float16) if zm == "int" else \
        (rng.standard_normal((n, g)) * 6 + 7).astype(np.float16)
    m = AWQLinear(k, n, 128, bias=bias).cuda()
    m.qweight.copy_(torch.from_numpy(qw))
    m.scales.copy_(torch.from_numpy(s))
    m.zeros.copy_(torch.from_numpy(z))
    b = None
    if bias:
        b = torch.randn(n, generator=torch.Generator().manual_seed(seed)).to(dtype)
        m.bias = torch.nn.Parameter(b.cuda())
    return m, lambda x: O.awq_linear(x, qw, s, z, k, 128, None if b is None else _np(b))


def _fp8_layer(k, n, seed, bias, dtype=torch.bfloat16):
    from nanosglang_b200.quantization import FP8Linear
    rng = np.random.default_rng(seed)
    codes, scale = O.fp8_quantize((rng.standard_normal((n, k)) * 0.02).astype(np.float32))
    m = FP8Linear(k, n, bias=bias).cuda()
    m.weight_fp8 = torch.from_numpy(codes).cuda().view(torch.float8_e4m3fn)
    m.weight_scale = torch.tensor(scale).cuda()
    b = None
    if bias:
        b = torch.randn(n, generator=torch.Generator().manual_seed(seed)).to(dtype)
        m.bias = torch.nn.Parameter(b.cuda())
    return m, lambda x: O.fp8_linear(x, codes, scale, None if b is None else _np(b))


@pytest.mark.parametrize("fmt", ["awq", "fp8"])
@pytest.mark.parametrize("m", [1, 7, 16, 32])
@pytest.mark.parametrize("shape", [(896, (896, 128, 128)), (4096, (4096, 1024, 1024))])
def test_fused_qkv_matches_separate_layers(fmt, m, shape):
    from nanosglang_b200.quantization import FusedProjections
    k, ns = shape
    make = _awq_layer if fmt == "awq" else _fp8_layer
    layers = [make(k, n, seed=10 * i + m + k, bias=True) for i, n in enumerate(ns)]
    x = torch.randn(m, k, generator=torch.Generator().manual_seed(m)).to(torch.bfloat16)
    outs = FusedProjections(*[lyr for lyr, _ in layers])(x.cuda())
    assert len(outs) == 3
    for out, (lyr, ref) in zip(outs, layers):
        assert out.shape == (m, lyr.out_features)
        assert O.rel_fro(_np(out), ref(_np(x))) <= GEMM_TOL


@pytest.mark.parametrize("fmt", ["awq", "fp8"])
@pytest.mark.parametrize("m", [1, 16, 32, 48])
@pytest.mark.parametrize("kn", [(896, 4864), (4096, 14336), (512, 1000)])
def test_gate_up_silu_matches_mlp_expression(fmt, m, kn):
    """M = 48 takes the unfused path (two linears + SiLU * up) through the same module."""
    from nanosglang_b200.quantization import GateUpSiLU
    k, n = kn
    make = _awq_layer if fmt == "awq" else _fp8_layer
    (gate, gref), (up, uref) = make(k, n, seed=1 + m, bias=False), make(k, n, seed=2 + m, bias=False)
    x = torch.randn(m, k, generator=torch.Generator().manual_seed(m + 5)).to(torch.bfloat16)
    y = GateUpSiLU(gate, up)(x.cuda())
    xr = _np(x)
    g, u = gref(xr), uref(xr)
    ref = g / (1.0 + np.exp(-g)) * u
    assert y.shape == (m, n)
    assert O.rel_fro(_np(y), ref) <= GEMM_TOL


def test_fused_qkv_fp16_and_non_integer_zero_points():
    from nanosglang_b200.quantization import FusedProjections
    layers = [_awq_layer(1024, n, seed=n, bias=True, dtype=torch.float16, zm="frac") for n in (1024, 256, 256)]
    x = torch.randn(9, 1024, generator=torch.Generator().manual_seed(3)).to(torch.float16)
    for out, (lyr, ref) in zip(FusedProjections(*[lyr for lyr, _ in layers])(x.cuda()), layers):
        assert O.rel_fro(_np(out), ref(_np(x))) <= GEMM_TOL


def test_fused_entry_points_reject_large_batches():
    from nanosglang_b200 import _lib, ops
    gate, _ = _awq_layer(512, 256, seed=1, bias=False)
    up, _ = _awq_layer(512, 256, seed=2, bias=False)
    x = torch.randn(33, 512, device="cuda", dtype=torch.bfloat16)
    assert ops.gate_up_silu(x, gate, up) is None  # M > 32: the module falls back to the two linears
    lib = _lib.load()
    rc = lib.nsq_awq_gate_up_silu(x.data_ptr(), _lib.DTYPE_BF16, 33, 512, 256, gate.qweight.data_ptr(),
                                  gate.scales.data_ptr(), gate.zeros.data_ptr(), up.qweight.data_ptr(),
                                  up.scales.data_ptr(), up.zeros.data_ptr(), 128, x.data_ptr(), None)
    assert rc == _lib.ENOTSUP
