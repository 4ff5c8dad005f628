"""Parity of the CUDA path (through the C ABI) against the CPU oracle and the
reference-generated golden vectors. Tolerances: bit-exact for unpack,
dequantisation and quantisation; relative Frobenius error <= 1e-2 for the
GEMMs, against an fp32 ground truth."""

import os

import numpy as np
import pytest
import torch
import torch.nn as nn

from conftest import GOLDEN
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


def _f16(u):
    return np.asarray(u, dtype=np.uint16).view(np.float16)


def _g(name):
    return np.load(os.path.join(GOLDEN, name))


def _to_np(t):
    if t.dtype == torch.bfloat16:
        return O.from_bf16_bits(t.view(torch.int16).cpu().numpy().view(np.uint16))
    return t.float().cpu().numpy()


def rand_awq(n, k, gs, seed, zero_mode="int", device="cuda"):
    rng = np.random.default_rng(seed)
    g = (k + gs - 1) // gs
    qw = rng.integers(-2 ** 31, 2 ** 31 - 1, (n, k // 8), dtype=np.int64).astype(np.int32)
    s = (rng.random((n, g)) * 0.009 + 0.001).astype(np.float16)
    if zero_mode == "int":
        z = rng.integers(0, 16, (n, g)).astype(np.float16)
    elif zero_mode == "wide":
        z = rng.integers(-300, 300, (n, g)).astype(np.float16)
    else:
        z = (rng.standard_normal((n, g)) * 6 + 7).astype(np.float16)
    return (qw, s, z), tuple(torch.from_numpy(a).to(device) for a in (qw, s, z))


def rand_x(m, k, dtype, seed):
    g = torch.Generator().manual_seed(seed)
    return torch.randn(m, k, generator=g).to(dtype)


# ---------------------------------------------------------------------------
# AWQ dequant: bit-exact
# ---------------------------------------------------------------------------


def test_awq_dequant_golden_bit_exact():
    from nanosglang_b200 import ops
    d = _g("awq_dequant_forward.npz")
    for ci in range(int(d["ncases"][0])):
        n, k, gs = (int(v) for v in d[f"c{ci}_meta"])
        qw = torch.from_numpy(d[f"c{ci}_qweight"]).cuda()
        s = torch.from_numpy(_f16(d[f"c{ci}_scales"])).cuda()
        z = torch.from_numpy(_f16(d[f"c{ci}_zeros"])).cuda()
        w = ops.awq_dequant(qw, s, z, k, gs)
        assert np.array_equal(w.view(torch.int16).cpu().numpy().view(np.uint16), d[f"c{ci}_dequant"]), ci


@pytest.mark.parametrize("n,k,gs,zm", [(9728, 896, 128, "int"), (896, 4864, 128, "frac"), (130, 1024, 256, "wide")])
def test_awq_dequant_bit_exact_full_size(n, k, gs, zm):
    from nanosglang_b200 import ops
    (qw, s, z), (tq, ts, tz) = rand_awq(n, k, gs, seed=n + k, zero_mode=zm)
    w = ops.awq_dequant(tq, ts, tz, k, gs)
    ref = O.awq_dequant(qw, s, z, k, gs)
    assert np.array_equal(w.view(torch.int16).cpu().numpy().view(np.uint16), ref.view(np.uint16))


# ---------------------------------------------------------------------------
# FP8 dequant / quantisers: bit-exact
# ---------------------------------------------------------------------------


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
def test_fp8_dequant_bit_exact(dtype):
    from nanosglang_b200 import ops
    rng = np.random.default_rng(1)
    codes = rng.integers(0, 256, (333, 208), dtype=np.int64).astype(np.uint8)
    codes[codes == 0x7F] = 0x7E  # skip NaN codes
    codes[codes == 0xFF] = 0xFE
    scale = np.float32(0.000321)
    w = ops.fp8_dequant(torch.from_numpy(codes).cuda().view(torch.float8_e4m3fn),
                        torch.tensor(scale).cuda(), dtype)
    ref = O.fp8_dequant(codes, scale, "bf16" if dtype == torch.bfloat16 else "fp16")
    assert np.array_equal(_to_np(w), ref)


def test_awq_quantize_golden_bit_exact():
    from nanosglang_b200 import ops
    d = _g("awq_from_linear.npz")
    for ci in range(int(d["ncases"][0])):
        n, k, gs = (int(v) for v in d[f"c{ci}_meta"])
        qw, s, z = ops.awq_quantize(torch.from_numpy(d[f"c{ci}_w"]).cuda(), gs)
        assert np.array_equal(qw.cpu().numpy(), d[f"c{ci}_qweight"]), ci
        assert np.array_equal(s.cpu().numpy().view(np.uint16), d[f"c{ci}_scales"]), ci
        assert np.array_equal(z.cpu().numpy().view(np.uint16), d[f"c{ci}_zeros"]), ci


def test_awq_quantize_large_vs_oracle():
    from nanosglang_b200 import ops
    rng = np.random.default_rng(7)
    w = (rng.standard_normal((512, 4864)) * 0.02).astype(np.float32)
    qw, s, z = ops.awq_quantize(torch.from_numpy(w).cuda(), 128)
    rq, rs, rz = O.awq_quantize(w, 128)
    assert np.array_equal(qw.cpu().numpy(), rq)
    assert np.array_equal(s.cpu().numpy(), rs) and np.array_equal(z.cpu().numpy(), rz)


def test_fp8_quantize_golden_bit_exact():
    from nanosglang_b200.quantization import FP8Linear
    d = _g("fp8_from_linear_forward.npz")
    for ci in range(int(d["ncases"][0])):
        n, k = (int(v) for v in d[f"c{ci}_meta"])
        lin = nn.Linear(k, n, bias=False).cuda()
        with torch.no_grad():
            lin.weight.copy_(torch.from_numpy(d[f"c{ci}_w"]))
        m = FP8Linear.from_linear(lin)
        assert np.array_equal(m.weight_fp8.view(torch.uint8).cpu().numpy(), d[f"c{ci}_codes"]), ci
        assert m.weight_scale.float().cpu().reshape(-1).numpy()[0] == d[f"c{ci}_scale"][0], ci
        shape = list(d[f"c{ci}_scale_shape"])
        assert list(m.weight_scale.shape) == ([] if shape == [-1] else shape), ci


def test_fp8_quantize_special_values():
    from nanosglang_b200 import ops
    d = _g("scalar_casts.npz")
    v = d["e4m3_in"][np.isfinite(d["e4m3_in"])].astype(np.float32)
    v = v[np.abs(v) <= 448.0]
    w = np.concatenate([v, np.array([448.0], dtype=np.float32)])  # absmax 448 -> scale exactly 1
    w = np.resize(w, (w.size // 16) * 16).reshape(-1, 16)
    codes, scale, _ = ops.fp8_quantize(torch.from_numpy(w).cuda())
    rc, rs = O.fp8_quantize(w)
    assert float(scale) == float(rs)
    assert np.array_equal(codes.view(torch.uint8).cpu().numpy(), rc)


# ---------------------------------------------------------------------------
# AWQ linear (decode M <= 64 and prefill M > 64)
# ---------------------------------------------------------------------------


def _awq_case(m, n, k, gs, dtype, bias, zm, seed):
    from nanosglang_b200 import ops
    (qw, s, z), (tq, ts, tz) = rand_awq(n, k, gs, seed=seed, zero_mode=zm)
    x = rand_x(m, k, dtype, seed + 1)
    b = torch.randn(n, generator=torch.Generator().manual_seed(seed + 2)).to(dtype) if bias else None
    y = ops.awq_linear(x.cuda(), tq, ts, tz, gs, None if b is None else b.cuda())
    assert y.dtype == dtype and y.shape == (m, n)
    ref = O.awq_linear(_to_np(x), qw, s, z, k, gs, None if b is None else _to_np(b))
    return O.rel_fro(_to_np(y), ref)


@pytest.mark.parametrize("m", [1, 3, 8, 16, 17, 33, 64])
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
def test_awq_linear_decode_config0_shape(m, dtype):
    err = _awq_case(m, 9728, 896, 128, dtype, bias=False, zm="int", seed=m)
    assert err <= GEMM_TOL, err


@pytest.mark.parametrize("n,k,gs,zm,bias", [
    (128, 896, 128, "int", True), (896, 4864, 128, "frac", False), (200, 512, 256, "wide", True),
    (1000, 14336, 128, "int", False), (64, 96, 128, "int", True), (8, 65536, 128, "int", False)])
@pytest.mark.parametrize("m", [1, 16, 64])
def test_awq_linear_decode_shapes(n, k, gs, zm, bias, m):
    err = _awq_case(m, n, k, gs, torch.bfloat16, bias, zm, seed=n + k + m)
    assert err <= GEMM_TOL, err


@pytest.mark.parametrize("m", [1, 16, 24, 32])
def test_awq_linear_decode_large_layer(m):
    """Llama-3-8B gate shape: large enough for the streamed weight-ring kernel."""
    err = _awq_case(m, 14336, 4096, 128, torch.bfloat16, bias=(m == 1), zm="frac" if m == 24 else "int",
                    seed=500 + m)
    assert err <= GEMM_TOL, err


@pytest.mark.parametrize("m,n,k,gs,zm,dtype,bias", [
    (25, 10000, 2048, 128, "int", torch.bfloat16, True),    # 64 / 72 rows per CTA
    (32, 14336, 4096, 256, "frac", torch.bfloat16, False),  # groups of two k-blocks, fractional zero points
    (28, 12288, 2048, 128, "int", torch.float16, True),
    (16, 18944, 4096, 128, "int", torch.bfloat16, False),   # 128 rows per CTA; 56 M+ weight elements at M = 16
    (5, 18944, 8192, 128, "frac", torch.bfloat16, False),   # few tokens on a weight with no weight-ring plan
    (48, 14336, 4096, 128, "frac", torch.bfloat16, True),   # 64 token slots (precomputed x terms)
    (16, 7168, 4096, 128, "int", torch.bfloat16, True),     # fewer than 64 rows per SM: 112 CTAs of 64 rows
    (12, 18944, 3584, 128, "frac", torch.bfloat16, False),  # 28 groups per row: scales loaded one group at a time
    (64, 10000, 2048, 128, "int", torch.float16, False)])
def test_awq_linear_tensor_core_decode(m, n, k, gs, zm, dtype, bias):
    """Layers of 64-128 rows per SM at M <= 32, shapes the dispatch sends to the tcgen05 decode kernel (nibbles
    widened to u8 in tensor memory, x as two s8 terms per k-block, kind::i8 UMMAs, zero point and scale per k-block
    in the epilogue)."""
    err = _awq_case(m, n, k, gs, dtype, bias, zm, seed=900 + m + n)
    assert err <= GEMM_TOL, err


@pytest.mark.parametrize("gs", [32, 64])
@pytest.mark.parametrize("m", [1, 16, 32, 48, 100, 1000])
@pytest.mark.parametrize("n,k,zm", [(4864, 896, "int"), (1000, 1056, "frac"), (4096, 4096, "int")])
def test_awq_linear_small_groups(gs, m, n, k, zm):
    """Groups of 32 and 64 columns (the reference takes any group size,
    quantization.py:93-124): row-streaming decode kernel up to 32 tokens,
    one-CTA tcgen05 kernel above; K = 1056 leaves half a 64-column k-block."""
    err = _awq_case(m, n, k, gs, torch.bfloat16, bias=(m == 16), zm=zm, seed=gs + m + n)
    assert err <= GEMM_TOL, err


def test_quantize_model_group_64_forward():
    """quantize_model(..., group_size=64) gives working modules (bit-exact
    quantiser, forward against the fp32 oracle of the quantised weight)."""
    from nanosglang_b200 import quantization as Q
    torch.manual_seed(4)
    model = nn.Sequential(nn.Linear(512, 768, bias=True), nn.Linear(768, 512)).cuda()
    Q.quantize_model(model, "awq", 64)
    for mod in model:
        assert isinstance(mod, Q.AWQLinear) and mod.group_size == 64
    for m in (4, 40, 300):
        x = torch.randn(m, 512, device="cuda", dtype=torch.bfloat16)
        mod = model[0]
        ref = O.awq_linear(_to_np(x), mod.qweight.cpu().numpy(), mod.scales.cpu().numpy(), mod.zeros.cpu().numpy(),
                           512, 64, mod.bias.detach().float().cpu().numpy())
        assert O.rel_fro(_to_np(mod(x)), ref) <= GEMM_TOL


@pytest.mark.parametrize("m", [65, 128, 200, 1024])
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
def test_awq_linear_prefill(m, dtype):
    err = _awq_case(m, 4864, 896, 128, dtype, bias=(m == 200), zm="int", seed=100 + m)
    assert err <= GEMM_TOL, err


@pytest.mark.parametrize("n,k,gs,zm", [(896, 4864, 128, "frac"), (300, 640, 256, "wide"), (128, 96, 128, "int")])
def test_awq_linear_prefill_shapes(n, k, gs, zm):
    err = _awq_case(333, n, k, gs, torch.bfloat16, bias=True, zm=zm, seed=n + k)
    assert err <= GEMM_TOL, err


@pytest.mark.parametrize("m,n,k,gs,zm", [(77, 131, 1024, 128, "frac"), (200, 896, 896, 128, "int"),
                                         (1000, 896, 896, 256, "wide"), (8192, 128, 896, 128, "int"),
                                         (300, 300, 608, 128, "frac")])
def test_awq_linear_small_output_shapes(m, n, k, gs, zm):
    """Prefill problems with at most 2^20 outputs (the TMEM-operand kernel):
    groups spanning 2 or 4 k-blocks, a partial last group, non-integer and
    out-of-range zero points."""
    err = _awq_case(m, n, k, gs, torch.bfloat16, bias=True, zm=zm, seed=m * 3 + n)
    assert err <= GEMM_TOL, err
    err = _awq_case(m, n, k, gs, torch.float16, bias=False, zm=zm, seed=m * 3 + n + 1)
    assert err <= GEMM_TOL, err


@pytest.mark.parametrize("m,n,k,gs,zm", [(300, 4104, 896, 128, "frac"), (777, 2050, 1024, 256, "wide"),
                                         (1024, 4864, 4096, 128, "int")])
def test_awq_linear_paired_tmem_kernel_shapes(m, n, k, gs, zm):
    """Outputs beyond 2^20 on the paired-CTA TMEM-operand kernel (AWQ keeps the
    staged epilogue and a 4-stage ring): ragged token tiles, N % 8 != 0,
    groups of 2 and 4 k-blocks across two-k-block stages."""
    err = _awq_case(m, n, k, gs, torch.bfloat16, bias=(m % 2 == 0), zm=zm, seed=m * 5 + n)
    assert err <= GEMM_TOL, err
    err = _awq_case(m, n, k, gs, torch.float16, bias=(m % 2 == 1), zm=zm, seed=m * 5 + n + 1)
    assert err <= GEMM_TOL, err


def test_awq_linear_fp16_matches_reference_forward_golden():
    """The reference's own fp16 forward outputs (cases the kernels support)."""
    from nanosglang_b200 import ops
    d = _g("awq_dequant_forward.npz")
    for ci in range(int(d["ncases"][0])):
        n, k, gs = (int(v) for v in d[f"c{ci}_meta"])
        if (gs % 128 and gs not in (32, 64)) or k % 32:
            continue
        x = torch.from_numpy(_f16(d[f"c{ci}_x"])).cuda()
        b = torch.from_numpy(_f16(d[f"c{ci}_bias"])).cuda() if f"c{ci}_bias" in d else None
        y = ops.awq_linear(x, torch.from_numpy(d[f"c{ci}_qweight"]).cuda(),
                           torch.from_numpy(_f16(d[f"c{ci}_scales"])).cuda(),
                           torch.from_numpy(_f16(d[f"c{ci}_zeros"])).cuda(), gs, b)
        ref = _f16(d[f"c{ci}_y"]).astype(np.float32)
        assert O.rel_fro(y.float().cpu().numpy(), ref) <= GEMM_TOL, ci


def test_awq_linear_unsupported_group_size_raises():
    from nanosglang_b200 import _lib, ops
    (_, _, _), (tq, ts, tz) = rand_awq(64, 384, 96, seed=3)
    with pytest.raises(_lib.NsqError):
        ops.awq_linear(torch.randn(4, 384, device="cuda", dtype=torch.bfloat16), tq, ts, tz, 96)


# ---------------------------------------------------------------------------
# FP8 linear
# ---------------------------------------------------------------------------


def _fp8_case(m, n, k, dtype, bias, seed):
    from nanosglang_b200 import ops
    rng = np.random.default_rng(seed)
    w = (rng.standard_normal((n, k)) * 0.02).astype(np.float32)
    codes, scale = O.fp8_quantize(w)
    x = rand_x(m, k, dtype, seed + 1)
    b = torch.randn(n, generator=torch.Generator().manual_seed(seed + 2)).to(dtype) if bias else None
    y = ops.fp8_linear(x.cuda(), torch.from_numpy(codes).cuda().view(torch.float8_e4m3fn),
                       torch.tensor(scale).cuda(), None if b is None else b.cuda())
    assert y.dtype == dtype and y.shape == (m, n)
    ref = O.fp8_linear(_to_np(x), codes, scale, None if b is None else _to_np(b))
    return O.rel_fro(_to_np(y), ref)


QWEN05_SHAPES = [(896, 896), (896, 128), (896, 4864), (4864, 896)]  # (K, N)


@pytest.mark.parametrize("kn", QWEN05_SHAPES)
@pytest.mark.parametrize("m", [1, 8, 32, 64, 128, 1024])
def test_fp8_linear_config1(kn, m):
    k, n = kn
    err = _fp8_case(m, n, k, torch.bfloat16, bias=(n == 128), seed=m * 7 + n)
    assert err <= GEMM_TOL, err


@pytest.mark.parametrize("m", [1, 8, 32])
def test_fp8_linear_decode_large_layer(m):
    assert _fp8_case(m, 14336, 4096, torch.bfloat16, bias=(m == 8), seed=700 + m) <= GEMM_TOL
    assert _fp8_case(m, 4096, 14336, torch.float16, bias=False, seed=800 + m) <= GEMM_TOL


@pytest.mark.parametrize("m,n,k,dtype,bias", [
    (2, 9472, 2048, torch.bfloat16, False),   # 64 rows per CTA
    (13, 10000, 896, torch.bfloat16, True),   # 64 / 72 rows per CTA, K of seven k-blocks
    (16, 14336, 4096, torch.float16, True),
    (32, 18944, 2048, torch.bfloat16, False),  # 128 rows per CTA
    (64, 14336, 4096, torch.bfloat16, True),   # 64 token slots (precomputed x terms)
    (32, 6600, 4096, torch.float16, True),     # fewer than 64 rows per SM: 103 CTAs, some of 72 rows
    (40, 18944, 3584, torch.float16, False)])
def test_fp8_linear_tensor_core_decode(m, n, k, dtype, bias):
    """Layers of 64-128 rows per SM, shapes the dispatch sends to the tcgen05 decode kernel (kind::f8f6f4 UMMAs on
    the stored e4m3 codes, x as two e4m3 terms per token and k-block)."""
    assert _fp8_case(m, n, k, dtype, bias, seed=950 + m + n) <= GEMM_TOL


@pytest.mark.parametrize("fmt", ["fp8", "awq"])
def test_tensor_core_decode_nonfinite_x(fmt):
    """An infinite x makes its token's outputs NaN (the reference's matmul gives inf/NaN there); the other
    tokens are unaffected."""
    from nanosglang_b200 import ops
    m, n, k = 26, 9472, 2048  # the tensor-core decode kernel for both formats
    x = rand_x(m, k, torch.bfloat16, 77)
    x[3, 500] = float("inf")
    if fmt == "fp8":
        rng = np.random.default_rng(78)
        codes, scale = O.fp8_quantize((rng.standard_normal((n, k)) * 0.02).astype(np.float32))
        y = ops.fp8_linear(x.cuda(), torch.from_numpy(codes).cuda().view(torch.float8_e4m3fn),
                           torch.tensor(scale).cuda())
        with np.errstate(invalid="ignore"):  # the oracle's own inf * 0 in row 3
            ref = O.fp8_linear(_to_np(x), codes, scale)
    else:
        (qw, s, z), (tq, ts, tz) = rand_awq(n, k, 128, seed=79, zero_mode="int")
        y = ops.awq_linear(x.cuda(), tq, ts, tz, 128)
        with np.errstate(invalid="ignore"):
            ref = O.awq_linear(_to_np(x), qw, s, z, k, 128)
    yn = _to_np(y)
    assert np.isnan(yn[3]).all()
    keep = [i for i in range(m) if i != 3]
    assert O.rel_fro(yn[keep], ref[keep]) <= GEMM_TOL


@pytest.mark.parametrize("fmt", ["fp8", "awq"])
@pytest.mark.parametrize("m", [16, 32])
def test_tensor_core_decode_workspace_and_without(fmt, m):
    """The C ABI with and without the workspace nsq_linear_workspace_size asks for: with it the x terms are
    computed once by a kernel ahead of the linear, without it by every CTA; both match the oracle."""
    from nanosglang_b200 import _lib
    lib = _lib.load()
    n, k = 14336, 4096
    assert lib.nsq_linear_workspace_size(1 if fmt == "fp8" else 0, m, k, n, 128) == (k // 128) * 2 * m * 132
    assert lib.nsq_linear_workspace_size(1 if fmt == "fp8" else 0, m, 896, 896, 128) == 0  # not a tensor-core shape
    x = rand_x(m, k, torch.bfloat16, 61).cuda()
    y = torch.empty(m, n, dtype=torch.bfloat16, device="cuda")
    stream = torch.cuda.current_stream().cuda_stream
    if fmt == "fp8":
        rng = np.random.default_rng(62)
        codes, scale = O.fp8_quantize((rng.standard_normal((n, k)) * 0.02).astype(np.float32))
        cw, sw = torch.from_numpy(codes).cuda(), torch.tensor(scale).cuda()
        ref = O.fp8_linear(_to_np(x.cpu()), codes, scale)
        call = lambda ws, nb: lib.nsq_fp8_linear(x.data_ptr(), _lib.DTYPE_BF16, m, k, n, cw.data_ptr(), sw.data_ptr(),
                                                 None, _lib.DTYPE_NONE, y.data_ptr(), ws, nb, stream)
    else:
        (qw, s, z), (tq, ts, tz) = rand_awq(n, k, 128, seed=63, zero_mode="int")
        ref = O.awq_linear(_to_np(x.cpu()), qw, s, z, k, 128)
        call = lambda ws, nb: lib.nsq_awq_linear(x.data_ptr(), _lib.DTYPE_BF16, m, k, n, tq.data_ptr(), ts.data_ptr(),
                                                 tz.data_ptr(), 128, None, _lib.DTYPE_NONE, y.data_ptr(), ws, nb,
                                                 stream)
    nb = lib.nsq_linear_workspace_size(1 if fmt == "fp8" else 0, m, k, n, 128)
    ws = torch.empty(nb, dtype=torch.uint8, device="cuda")
    for wsp, wsb in [(ws.data_ptr(), nb), (None, 0), (ws.data_ptr(), nb - 16)]:  # too small a workspace is ignored
        y.fill_(float("nan"))
        assert call(wsp, wsb) == 0
        torch.cuda.synchronize()
        assert O.rel_fro(_to_np(y), ref) <= GEMM_TOL


def test_fp8_linear_tensor_core_decode_wide_range_x():
    """x spanning many binades within a k-block (per-token, per-k-block power-of-two scales of the terms)."""
    from nanosglang_b200 import ops
    rng = np.random.default_rng(31)
    n, k, m = 9472, 2048, 8
    w = (rng.standard_normal((n, k)) * 0.02).astype(np.float32)
    codes, scale = O.fp8_quantize(w)
    x = (rng.standard_normal((m, k)) * np.exp2(rng.integers(-12, 12, (m, k)))).astype(np.float32)
    xt = torch.from_numpy(x).to(torch.bfloat16)
    y = ops.fp8_linear(xt.cuda(), torch.from_numpy(codes).cuda().view(torch.float8_e4m3fn), torch.tensor(scale).cuda())
    ref = O.fp8_linear(_to_np(xt), codes, scale)
    assert O.rel_fro(_to_np(y), ref) <= GEMM_TOL


@pytest.mark.parametrize("m", [5, 64, 300])
def test_fp8_linear_fp16_and_odd_shapes(m):
    assert _fp8_case(m, 200, 112, torch.float16, bias=True, seed=m) <= GEMM_TOL
    assert _fp8_case(m, 520, 608, torch.bfloat16, bias=False, seed=m + 1) <= GEMM_TOL


@pytest.mark.parametrize("m,n,k", [(77, 130, 896), (200, 896, 512), (1000, 896, 896), (8192, 128, 896),
                                   (129, 4864, 896), (300, 520, 608)])
def test_fp8_linear_small_output_shapes(m, n, k):
    """Prefill problems with at most 2^20 outputs (the TMEM-operand kernel):
    ragged token tiles, odd N, a partial last k-block, bias, fp16."""
    assert _fp8_case(m, n, k, torch.bfloat16, bias=(m % 2 == 1), seed=m + n) <= GEMM_TOL
    assert _fp8_case(m, n, k, torch.float16, bias=(m % 2 == 0), seed=m + n + 1) <= GEMM_TOL


@pytest.mark.parametrize("m,n,k", [(300, 4104, 896), (777, 2050, 1024), (1024, 4864, 4096), (257, 8200, 512)])
def test_fp8_linear_paired_tmem_kernel_shapes(m, n, k):
    """Outputs beyond 2^20 on the paired-CTA TMEM-operand kernel: ragged last
    token tiles (the odd CTA's half starts at n_eff / 2), N % 8 != 0 (direct
    stores), long K (deeper ring, direct stores), staged TMA stores."""
    assert _fp8_case(m, n, k, torch.bfloat16, bias=(m % 2 == 1), seed=m + n) <= GEMM_TOL
    assert _fp8_case(m, n, k, torch.float16, bias=(m % 2 == 0), seed=m + n + 1) <= GEMM_TOL


def test_fp8_linear_vs_reference_forward_golden():
    from nanosglang_b200 import ops
    d = _g("fp8_from_linear_forward.npz")
    for ci in range(int(d["ncases"][0])):
        n, k = (int(v) for v in d[f"c{ci}_meta"])
        if int(d[f"c{ci}_raises"][0]) or k % 16:
            continue
        x = torch.from_numpy(d[f"c{ci}_x"].view(np.int16)).cuda().view(torch.bfloat16)
        b = torch.from_numpy(d[f"c{ci}_bias"].view(np.int16)).cuda().view(torch.bfloat16) \
            if f"c{ci}_bias" in d else None
        y = ops.fp8_linear(x, torch.from_numpy(d[f"c{ci}_codes"]).cuda().view(torch.float8_e4m3fn),
                           torch.from_numpy(d[f"c{ci}_scale"]).cuda(), b)
        assert O.rel_fro(_to_np(y), O.from_bf16_bits(d[f"c{ci}_y"])) <= GEMM_TOL, ci


@pytest.mark.parametrize("kn", QWEN05_SHAPES)
def test_fp8_linear_config1_m8192_oracle(kn):
    """The benchmarked M = 8192 launches of config 1 (q/o 896->896, k/v 896->128,
    gate/up 896->4864, down 4864->896) against the fp32 oracle."""
    k, n = kn
    err = _fp8_case(8192, n, k, torch.bfloat16, bias=False, seed=8192 + 3 * n + k)
    assert err <= GEMM_TOL, err


@pytest.mark.parametrize("kn", [(896, 4864), (4864, 896)])
def test_awq_linear_m8192_oracle(kn):
    """AWQ W4A16 at M = 8192 on the gate/up and down shapes against the fp32 oracle."""
    k, n = kn
    err = _awq_case(8192, n, k, 128, torch.bfloat16, bias=False, zm="int", seed=8192 + n)
    assert err <= GEMM_TOL, err


def test_fp8_linear_full_size_property_m8192():
    """Config-1 largest case, checked against an fp32 torch reference built from
    the bit-exact dequantised weight (size-independent property check)."""
    from nanosglang_b200 import ops
    torch.manual_seed(0)
    w = (torch.randn(4864, 896, device="cuda") * 0.02)
    codes, scale, _ = ops.fp8_quantize(w)
    x = torch.randn(8192, 896, device="cuda").to(torch.bfloat16)
    y = ops.fp8_linear(x, codes, scale)
    wd = ops.fp8_dequant(codes, torch.ones((), device="cuda"), torch.float16).float() * scale
    ref = x.float() @ wd.T
    err = ((y.float() - ref).norm() / ref.norm()).item()
    assert err <= GEMM_TOL, err


# ---------------------------------------------------------------------------
# Module level: drop-in classes, CUDA graphs
# ---------------------------------------------------------------------------


def test_modules_from_linear_forward():
    from nanosglang_b200.quantization import AWQLinear, FP8Linear
    torch.manual_seed(0)
    lin = nn.Linear(896, 1152, bias=True).cuda().to(torch.bfloat16)
    x = torch.randn(4, 7, 896, device="cuda", dtype=torch.bfloat16)
    a = AWQLinear.from_linear(lin, 128)
    assert a.qweight.is_cuda and a.qweight.shape == (1152, 112)
    wdq = a._dequantize()
    ref = x.float() @ wdq.float().T + lin.bias.float()
    ya = a(x)
    assert ya.shape == (4, 7, 1152) and ya.dtype == torch.bfloat16
    assert ((ya.float() - ref).norm() / ref.norm()).item() <= GEMM_TOL
    f = FP8Linear.from_linear(lin)
    yf = f(x)
    ref8 = x.float() @ f.dequantize(torch.float16).float().T + lin.bias.float()
    assert ((yf.float() - ref8).norm() / ref8.norm()).item() <= GEMM_TOL


def test_linears_capture_in_cuda_graph():
    from nanosglang_b200.quantization import AWQLinear, FP8Linear
    torch.manual_seed(1)
    lin = nn.Linear(896, 4864, bias=False).cuda().to(torch.bfloat16)
    a = AWQLinear.from_linear(lin, 128)
    f = FP8Linear.from_linear(lin)
    x = torch.randn(16, 896, device="cuda", dtype=torch.bfloat16)
    xb = torch.randn(256, 896, device="cuda", dtype=torch.bfloat16)
    eager = (a(x), f(x), a(xb), f(xb))
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        for _ in range(2):
            a(x), f(x), a(xb), f(xb)
    torch.cuda.current_stream().wait_stream(s)
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        outs = (a(x), f(x), a(xb), f(xb))
    g.replay()
    torch.cuda.synchronize()
    for e, o in zip(eager, outs):
        assert torch.equal(e, o)


@pytest.mark.parametrize("m,k,n", [(128, 4864, 896), (1024, 4864, 896), (300, 1024, 1000)])
def test_split_k_results_do_not_depend_on_timing(m, k, n):
    """Shapes whose K range is split over a thread-block cluster (the partial
    columns are exchanged through DSMEM and summed in rank order): repeated
    eager calls and CUDA-graph replays give bit-identical outputs."""
    from nanosglang_b200.quantization import AWQLinear, FP8Linear
    torch.manual_seed(m + n)
    lin = nn.Linear(k, n, bias=True).cuda().to(torch.bfloat16)
    mods = (AWQLinear.from_linear(lin, 128), FP8Linear.from_linear(lin))
    x = torch.randn(m, k, device="cuda", dtype=torch.bfloat16)
    first = [mod(x) for mod in mods]
    for _ in range(3):
        for mod, f in zip(mods, first):
            assert torch.equal(mod(x), f)
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        for mod in mods:
            mod(x)
    torch.cuda.current_stream().wait_stream(s)
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        outs = [mod(x) for mod in mods]
    for _ in range(2):
        g.replay()
        torch.cuda.synchronize()
        for o, f in zip(outs, first):
            assert torch.equal(o, f)


def test_quantize_model_on_cuda():
    from nanosglang_b200.quantization import AWQLinear, FP8Linear, quantize_model
    for method, cls in (("awq", AWQLinear), ("fp8", FP8Linear)):
        m = nn.Sequential()
        m.add_module("layers", nn.ModuleList([nn.Linear(256, 512), nn.Linear(512, 256)]))
        m.add_module("lm_head", nn.Linear(256, 100))
        m = m.cuda()
        quantize_model(m, method=method, group_size=128)
        assert isinstance(m.layers[0], cls) and isinstance(m.layers[1], cls)
        assert isinstance(m.lm_head, nn.Linear)
        x = torch.randn(3, 256, device="cuda", dtype=torch.float16)
        assert m.layers[1](m.layers[0](x)).shape == (3, 256)


@pytest.mark.parametrize("m", [4, 40, 200])
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
def test_fp8_linear_every_code(m, dtype):
    """Weights cycling through all 254 finite e4m3 codes (subnormals and signed
    zero included) through the in-register conversion of both kernels."""
    from nanosglang_b200 import ops
    n, k = 96, 512
    codes = (np.arange(n * k, dtype=np.int64) * 7 % 256).astype(np.uint8).reshape(n, k)
    codes[(codes & 0x7F) == 0x7F] = 0x01  # no NaN codes
    scale = np.float32(0.01)
    x = rand_x(m, k, dtype, seed=m)
    y = ops.fp8_linear(x.cuda(), torch.from_numpy(codes).cuda().view(torch.float8_e4m3fn),
                       torch.tensor(scale).cuda())
    ref = O.fp8_linear(_to_np(x), codes, scale)
    assert O.rel_fro(_to_np(y), ref) <= GEMM_TOL


# ---------------------------------------------------------------------------
# AutoAWQ checkpoint layout -> reference layout (the loader quantization.py:7 names)
# ---------------------------------------------------------------------------


@pytest.mark.parametrize("k,n,gs", [(896, 4864, 128), (4096, 1024, 128), (256, 72, 64), (128, 8, 32)])
def test_awq_from_autoawq_bit_exact(k, n, gs):
    from nanosglang_b200 import ops
    rng = np.random.default_rng(k + n)
    q = rng.integers(0, 16, (k, n))
    z = rng.integers(0, 16, (k // gs, n))
    s = (rng.random((k // gs, n)) * 0.009 + 0.001).astype(np.float16)
    aq, az = O.autoawq_pack(q, z)
    rq, rs, rz = O.autoawq_to_reference(aq, az, s)
    tq, ts, tz = ops.awq_from_autoawq(torch.from_numpy(aq).cuda(), torch.from_numpy(az).cuda(),
                                      torch.from_numpy(s).cuda(), gs)
    assert np.array_equal(tq.cpu().numpy(), rq)
    assert np.array_equal(ts.cpu().numpy().view(np.uint16), rs.view(np.uint16))
    assert np.array_equal(tz.cpu().numpy().view(np.uint16), rz.view(np.uint16))
    # the repacked layer dequantises to AutoAWQ's own weights, bit for bit
    w = ops.awq_dequant(tq, ts, tz, k, gs)
    assert np.array_equal(w.cpu().numpy().view(np.uint16), O.autoawq_dequant(aq, az, s, gs).view(np.uint16))


def test_load_autoawq_state_dict_into_quantized_model():
    from nanosglang_b200 import quantization as Q
    torch.manual_seed(0)
    model = nn.Sequential(nn.Linear(256, 512, bias=True), nn.Linear(512, 256, bias=False)).cuda()
    Q.quantize_model(model, "awq", 128)
    rng = np.random.default_rng(3)
    sd, refs = {}, {}
    for name, (k, n) in {"0": (256, 512), "1": (512, 256)}.items():
        q, z = rng.integers(0, 16, (k, n)), rng.integers(0, 16, (k // 128, n))
        s = (rng.random((k // 128, n)) * 0.009 + 0.001).astype(np.float16)
        aq, az = O.autoawq_pack(q, z)
        sd[f"model.{name}.qweight"], sd[f"model.{name}.qzeros"] = torch.from_numpy(aq), torch.from_numpy(az)
        sd[f"model.{name}.scales"] = torch.from_numpy(s)
        refs[name] = (aq, az, s, k)
    sd["model.0.bias"] = torch.randn(512)
    assert sorted(Q.load_autoawq_state_dict(model, sd, 128)) == ["0", "1"]
    x = torch.randn(5, 256, device="cuda", dtype=torch.float16)
    aq, az, s, k = refs["0"]
    ref = _to_np(x) @ O.autoawq_dequant(aq, az, s, 128).astype(np.float32).T + sd["model.0.bias"].numpy()
    assert O.rel_fro(_to_np(model[0](x)), ref) <= GEMM_TOL
