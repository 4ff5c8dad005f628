"""CPU oracle for the quantized-linear path -- TEST INFRASTRUCTURE ONLY.

This module restates, in numpy, the arithmetic of nanoSGLang's quantized
linears (``nano_sglang/decode/quantization.py`` in xiehuanyi/nanoSGLang) and of
its tensor-parallel sharding (``nano_sglang/distributed/tensor_parallel.py``).
It is the checker that the CUDA path in ``nanosglang_b200`` is compared
against. Only ``tests/``, ``__graft_entry__.smoke()`` and the ``cpu_baseline``
/ ``--impl reference`` legs of ``bench.py`` may import it; the product path
never does.

Parity of this oracle is pinned against vectors produced by the reference's
own Python code (imported in-process) -- see ``tests/golden/make_golden.py``
and ``tests/test_oracle_golden.py``. The reference ships no tests or golden
vectors of its own for this path.

numpy has no bfloat16 / float8 types, so those encodings are written out
explicitly here (round-to-nearest-even, as PyTorch's casts do).
"""

from __future__ import annotations

import numpy as np

# ---------------------------------------------------------------------------
# Scalar encodings
# ---------------------------------------------------------------------------

E4M3_MAX = 448.0


def _e4m3_decode_table() -> np.ndarray:
    """float32 value of every float8_e4m3fn code (bias 7, no inf, 0x7F/0xFF NaN)."""
    t = np.zeros(256, dtype=np.float32)
    for code in range(256):
        s = -1.0 if code & 0x80 else 1.0
        e = (code >> 3) & 0xF
        m = code & 0x7
        if e == 0xF and m == 0x7:
            t[code] = np.nan
        elif e == 0:
            t[code] = s * (m / 8.0) * 2.0 ** -6
        else:
            t[code] = s * (1.0 + m / 8.0) * 2.0 ** (e - 7)
    return t


E4M3_TABLE = _e4m3_decode_table()


def e4m3_decode(codes: np.ndarray) -> np.ndarray:
    return E4M3_TABLE[np.asarray(codes, dtype=np.uint8)]


def e4m3_encode(v: np.ndarray) -> np.ndarray:
    """float32 -> float8_e4m3fn codes, round-to-nearest-even, non-saturating.

    Matches ``Tensor.to(torch.float8_e4m3fn)`` as used by
    ``FP8Linear.from_linear`` (quantization.py:68): magnitudes that round
    above 448 (i.e. > 464) and non-finite inputs become NaN (0x7F | sign).
    """
    v = np.asarray(v, dtype=np.float32)
    sign = (np.signbit(v)).astype(np.uint8) << 7
    a = np.abs(v).astype(np.float64)
    out = np.zeros(v.shape, dtype=np.uint8)
    # candidate magnitudes: the 127 finite non-negative codes (0x00..0x7E)
    mags = E4M3_TABLE[:127].astype(np.float64)
    # index of the largest code <= a
    idx = np.searchsorted(mags, a, side="right") - 1
    idx = np.clip(idx, 0, 126)
    lo = mags[idx]
    hi_idx = np.minimum(idx + 1, 126)
    hi = mags[hi_idx]
    d_lo = a - lo
    d_hi = hi - a
    pick_hi = (d_hi < d_lo) | ((d_hi == d_lo) & (hi_idx % 2 == 0) & (hi_idx != idx))
    code = np.where(pick_hi, hi_idx, idx).astype(np.uint8)
    # above the largest finite value: ties at 464 go to 448 (even), beyond -> NaN
    over = a > 464.0
    nonfinite = ~np.isfinite(v)
    code = np.where(over | nonfinite, np.uint8(0x7F), code)
    out[...] = code | sign
    # torch encodes +NaN as 0x7F
    out[np.isnan(v)] = 0x7F
    return out


def bf16_round(v: np.ndarray) -> np.ndarray:
    """float32 -> bfloat16 (RNE), returned as float32 values."""
    v = np.ascontiguousarray(np.asarray(v, dtype=np.float32))
    u = v.view(np.uint32).astype(np.uint64)
    rounding = ((u >> 16) & 1) + 0x7FFF
    r = ((u + rounding) >> 16) << 16
    r = np.where(np.isnan(v), (u | 0x400000) >> 16 << 16, r)
    return r.astype(np.uint32).view(np.float32)


def to_bf16_bits(v: np.ndarray) -> np.ndarray:
    return (bf16_round(v).view(np.uint32) >> 16).astype(np.uint16)


def from_bf16_bits(b: np.ndarray) -> np.ndarray:
    return (np.asarray(b, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)


# ---------------------------------------------------------------------------
# AWQ W4A16  (quantization.py:83-194)
# ---------------------------------------------------------------------------


def awq_unpack(qweight: np.ndarray, in_features: int) -> np.ndarray:
    """int32 [N, K/8] -> uint8 [N, K]: nibble i of word j is column 8j+i.

    quantization.py:134-137 -- ``(qweight >> 4i) & 0xF`` into ``weight[:, i::8]``.
    The arithmetic shift of a negative word is harmless because of the mask.
    """
    q = np.asarray(qweight).astype(np.int64) & 0xFFFFFFFF
    n, k8 = q.shape
    if k8 * 8 != in_features:
        # the reference's strided assignment raises for in_features % 8 != 0
        raise ValueError("in_features must equal 8 * qweight.shape[1]")
    out = np.empty((n, in_features), dtype=np.uint8)
    for i in range(8):
        out[:, i::8] = ((q >> (4 * i)) & 0xF).astype(np.uint8)
    return out


def awq_dequant(qweight, scales, zeros, in_features: int, group_size: int) -> np.ndarray:
    """Bit-exact restatement of ``AWQLinear._dequantize`` (quantization.py:126-148).

    Returns float16 [N, K]. Per group: ``(w - z) * s`` evaluated in float16,
    one rounding per operation, exactly as the reference's fp16 tensor ops.
    """
    scales = np.asarray(scales, dtype=np.float16)
    zeros = np.asarray(zeros, dtype=np.float16)
    w = awq_unpack(qweight, in_features).astype(np.float16)
    num_groups = (in_features + group_size - 1) // group_size
    for g in range(num_groups):
        s0 = g * group_size
        e0 = min(s0 + group_size, in_features)
        w[:, s0:e0] = (w[:, s0:e0] - zeros[:, g:g + 1]) * scales[:, g:g + 1]
    return w


def awq_linear(x, qweight, scales, zeros, in_features, group_size, bias=None) -> np.ndarray:
    """float32 ground truth of ``AWQLinear.forward`` (quantization.py:150-152)."""
    w = awq_dequant(qweight, scales, zeros, in_features, group_size).astype(np.float32)
    x = np.asarray(x, dtype=np.float32)
    y = x.reshape(-1, in_features) @ w.T
    if bias is not None:
        y = y + np.asarray(bias, dtype=np.float32)
    return y.reshape(*x.shape[:-1], w.shape[0])


def awq_quantize(weight: np.ndarray, group_size: int = 128):
    """Restatement of ``AWQLinear.from_linear`` (quantization.py:154-194).

    Asymmetric min/max int4 per (row, group) in float32:
    ``scale = max((gmax-gmin)/15, 1e-8)``, ``zero = round(-gmin/scale)``,
    ``q = clamp(round((w-gmin)/scale), 0, 15)``; nibbles packed sequentially
    along K (column c -> word c//8, nibble c%8). Columns past 8*(K//8) are
    dropped, as the reference's ``byte_idx < qweight.shape[1]`` test does.
    Returns (qweight int32 [N, K//8], scales fp16 [N,G], zeros fp16 [N,G]).
    """
    w = np.asarray(weight, dtype=np.float32)
    n, k = w.shape
    num_groups = (k + group_size - 1) // group_size
    scales = np.ones((n, num_groups), dtype=np.float16)
    zeros = np.zeros((n, num_groups), dtype=np.float16)
    q_all = np.zeros((n, k), dtype=np.int64)
    for g in range(num_groups):
        s0 = g * group_size
        e0 = min(s0 + group_size, k)
        grp = w[:, s0:e0]
        gmin = grp.min(axis=1, keepdims=True)
        gmax = grp.max(axis=1, keepdims=True)
        scale = ((gmax - gmin) / np.float32(15.0)).astype(np.float32)
        scale = np.maximum(scale, np.float32(1e-8))
        zero = np.round(-gmin / scale)  # numpy rounds half to even, like torch.round
        scales[:, g] = scale[:, 0].astype(np.float16)
        zeros[:, g] = zero[:, 0].astype(np.float16)
        q = np.clip(np.round((grp - gmin) / scale), 0, 15).astype(np.int64)
        q_all[:, s0:e0] = q
    k8 = k // 8
    packed = np.zeros((n, k8), dtype=np.int64)
    for i in range(8):
        packed |= q_all[:, i:k8 * 8:8] << (4 * i)
    packed = packed.astype(np.uint32).view(np.int32) if packed.size else packed.astype(np.int32)
    return packed.astype(np.int32), scales, zeros


# ---------------------------------------------------------------------------
# AutoAWQ checkpoint layout -> the reference layout
# ---------------------------------------------------------------------------
#
# The reference's docstring (quantization.py:7) names AutoAWQ checkpoints, but
# it ships no loader. AutoAWQ's GEMM format (the published WQLinear_GEMM
# packing, restated here) stores, for in_features K, out_features N, groups G:
#   qweight int32 [K, N/8]: the eight int4 values of output columns 8c..8c+7
#           of input row k; nibble i (bits 4i..4i+3) holds column
#           8c + AUTOAWQ_ORDER[i]
#   qzeros  int32 [G, N/8]: the zero points of group g, packed the same way
#   scales  fp16  [G, N]
# and dequantises w[n, k] = (q[k, n] - z[g, n]) * s[g, n] with g = k // group.
# The reference layout holds the same numbers as qweight [N, K/8] (nibble i of
# word j = input column 8j+i), zeros fp16 [N, G] and scales fp16 [N, G].

AUTOAWQ_ORDER = (0, 2, 4, 6, 1, 3, 5, 7)


def autoawq_pack(q_kn: np.ndarray, z_gn: np.ndarray) -> tuple:
    """int values q [K, N] and z [G, N] (0..15) -> AutoAWQ qweight [K, N/8], qzeros [G, N/8]."""
    def pack(v):
        v = np.asarray(v).astype(np.int64)
        rows, n = v.shape
        out = np.zeros((rows, n // 8), dtype=np.int64)
        for i, col in enumerate(AUTOAWQ_ORDER):
            out |= (v[:, col::8] & 0xF) << (4 * i)
        return out.astype(np.uint32).view(np.int32)
    return pack(q_kn), pack(z_gn)


def autoawq_unpack(packed: np.ndarray) -> np.ndarray:
    """AutoAWQ-packed int32 [R, N/8] -> uint8 [R, N]."""
    p = np.asarray(packed).astype(np.int64) & 0xFFFFFFFF
    rows, n8 = p.shape
    out = np.empty((rows, n8 * 8), dtype=np.uint8)
    for i, col in enumerate(AUTOAWQ_ORDER):
        out[:, col::8] = ((p >> (4 * i)) & 0xF).astype(np.uint8)
    return out


def autoawq_to_reference(qweight, qzeros, scales):
    """AutoAWQ (qweight [K, N/8], qzeros [G, N/8], scales [G, N]) -> the
    reference's (qweight int32 [N, K/8], scales fp16 [N, G], zeros fp16 [N, G])."""
    q = autoawq_unpack(qweight).T  # [N, K]
    n, k = q.shape
    packed = np.zeros((n, k // 8), dtype=np.int64)
    for i in range(8):
        packed |= q[:, i::8].astype(np.int64) << (4 * i)
    z = autoawq_unpack(qzeros).T.astype(np.float16)  # [N, G]
    s = np.ascontiguousarray(np.asarray(scales, dtype=np.float16).T)
    return packed.astype(np.uint32).view(np.int32), s, np.ascontiguousarray(z)


def autoawq_dequant(qweight, qzeros, scales, group_size: int) -> np.ndarray:
    """fp16 [N, K] of an AutoAWQ layer with the reference's arithmetic
    (quantization.py:139-148: fp16 (q - z) * s)."""
    q = autoawq_unpack(qweight).T.astype(np.float16)
    z = autoawq_unpack(qzeros).T.astype(np.float16)
    s = np.asarray(scales, dtype=np.float16).T
    n, k = q.shape
    g = np.arange(k) // group_size
    return (q - z[:, g]) * s[:, g]


# ---------------------------------------------------------------------------
# FP8 E4M3 (quantization.py:24-75)
# ---------------------------------------------------------------------------


def fp8_dequant(weight_fp8_codes, weight_scale, out_dtype: str = "bf16") -> np.ndarray:
    """``weight_fp8.to(x.dtype) * weight_scale`` (quantization.py:51).

    The cast to bf16/fp16 is exact (every e4m3 value is representable); the
    product with the fp32 scalar is rounded once to ``out_dtype``.
    Returns float32 values of the rounded result.
    """
    w = e4m3_decode(weight_fp8_codes).astype(np.float32)
    p = (w * np.float32(weight_scale)).astype(np.float32)
    if out_dtype == "bf16":
        return bf16_round(p)
    if out_dtype == "fp16":
        return p.astype(np.float16).astype(np.float32)
    raise ValueError(out_dtype)


def fp8_linear(x, weight_fp8_codes, weight_scale, bias=None) -> np.ndarray:
    """float32 ground truth of ``FP8Linear.forward`` (quantization.py:49-52):
    ``x @ (fp8 * scale).T + bias`` with the weight kept exact in float32."""
    w = e4m3_decode(weight_fp8_codes).astype(np.float32) * np.float32(weight_scale)
    x = np.asarray(x, dtype=np.float32)
    k = w.shape[1]
    y = x.reshape(-1, k) @ w.T
    if bias is not None:
        y = y + np.asarray(bias, dtype=np.float32)
    return y.reshape(*x.shape[:-1], w.shape[0])


def fp8_quantize(weight: np.ndarray):
    """Restatement of ``FP8Linear.from_linear`` (quantization.py:54-75).

    ``scale = absmax / 448`` in float32 (1.0 if the weight is all zero);
    codes = RNE e4m3 of ``w / scale``. Returns (codes uint8 [N,K], scale f32).
    """
    w = np.asarray(weight, dtype=np.float32)
    absmax = np.float32(np.abs(w).max()) if w.size else np.float32(0.0)
    scale = np.float32(absmax / np.float32(448.0))
    if scale == 0:
        scale = np.float32(1.0)
    codes = e4m3_encode((w / scale).astype(np.float32))
    return codes, scale


# ---------------------------------------------------------------------------
# Tensor-parallel sharding (tensor_parallel.py:56-151)
# ---------------------------------------------------------------------------


def column_shard_rows(n: int, world_size: int, rank: int):
    """Output-dim shard ``[r*N/tp, (r+1)*N/tp)`` (tensor_parallel.py:93-98)."""
    assert n % world_size == 0
    per = n // world_size
    return rank * per, (rank + 1) * per


def row_shard_cols(k: int, world_size: int, rank: int):
    """Input-dim shard ``[r*K/tp, (r+1)*K/tp)`` (tensor_parallel.py:142-148)."""
    assert k % world_size == 0
    per = k // world_size
    return rank * per, (rank + 1) * per


def row_parallel_sum(partials):
    """``dist.all_reduce(SUM)`` of the row-parallel partial outputs
    (tensor_parallel.py:137-138), in float32."""
    acc = np.zeros_like(np.asarray(partials[0], dtype=np.float32))
    for p in partials:
        acc = acc + np.asarray(p, dtype=np.float32)
    return acc


# ---------------------------------------------------------------------------
# Error measure used by every floating-point parity test
# ---------------------------------------------------------------------------


def rel_fro(a, b) -> float:
    """Relative Frobenius error ||a-b|| / ||b|| in float64."""
    a = np.asarray(a, dtype=np.float64)
    b = np.asarray(b, dtype=np.float64)
    den = np.linalg.norm(b)
    if den == 0:
        return float(np.linalg.norm(a))
    return float(np.linalg.norm(a - b) / den)
