"""Pin the CPU oracle against vectors produced by the reference itself."""

import os

import numpy as np
import pytest

from oracle import nsq_oracle as O

from conftest import GOLDEN


def _load(name):
    return np.load(os.path.join(GOLDEN, name))


def _f16(u):
    return np.asarray(u, dtype=np.uint16).view(np.float16)


def test_e4m3_decode_table_matches_torch():
    d = _load("scalar_casts.npz")
    ref = d["e4m3_decoded"]
    ours = O.E4M3_TABLE
    nan = np.isnan(ref)
    assert np.array_equal(nan, np.isnan(ours))
    assert np.array_equal(ref[~nan], ours[~nan])


def test_e4m3_encode_matches_torch_cast():
    d = _load("scalar_casts.npz")
    assert np.array_equal(O.e4m3_encode(d["e4m3_in"]), d["e4m3_codes"])


def test_bf16_round_matches_torch_cast():
    d = _load("scalar_casts.npz")
    assert np.array_equal(O.to_bf16_bits(d["bf16_in"]), d["bf16_bits"])


def test_awq_dequant_bit_exact_vs_reference():
    d = _load("awq_dequant_forward.npz")
    for ci in range(int(d["ncases"][0])):
        n, k, gs = d[f"c{ci}_meta"]
        w = O.awq_dequant(d[f"c{ci}_qweight"], _f16(d[f"c{ci}_scales"]), _f16(d[f"c{ci}_zeros"]), int(k), int(gs))
        assert w.dtype == np.float16
        assert np.array_equal(w.view(np.uint16), d[f"c{ci}_dequant"]), f"case {ci}"


def test_awq_forward_fp16_vs_reference():
    """The reference forward (fp16 activations, fp16 GEMM) against the fp32 oracle."""
    d = _load("awq_dequant_forward.npz")
    for ci in range(int(d["ncases"][0])):
        n, k, gs = d[f"c{ci}_meta"]
        bias = _f16(d[f"c{ci}_bias"]) if f"c{ci}_bias" in d else None
        y = O.awq_linear(_f16(d[f"c{ci}_x"]), d[f"c{ci}_qweight"], _f16(d[f"c{ci}_scales"]),
                         _f16(d[f"c{ci}_zeros"]), int(k), int(gs), bias)
        ref = _f16(d[f"c{ci}_y"]).astype(np.float32)
        assert O.rel_fro(y, ref) < 2e-3, f"case {ci}"


def test_reference_awq_raises_on_bf16():
    d = _load("awq_dequant_forward.npz")
    assert int(d["bf16_raises"][0]) == 1


def test_awq_quantize_bit_exact_vs_reference():
    d = _load("awq_from_linear.npz")
    for ci in range(int(d["ncases"][0])):
        n, k, gs = d[f"c{ci}_meta"]
        qw, s, z = O.awq_quantize(d[f"c{ci}_w"], int(gs))
        assert np.array_equal(qw, d[f"c{ci}_qweight"]), f"case {ci}"
        assert np.array_equal(s.view(np.uint16), d[f"c{ci}_scales"]), f"case {ci}"
        assert np.array_equal(z.view(np.uint16), d[f"c{ci}_zeros"]), f"case {ci}"


def test_fp8_quantize_bit_exact_vs_reference():
    d = _load("fp8_from_linear_forward.npz")
    for ci in range(int(d["ncases"][0])):
        codes, scale = O.fp8_quantize(d[f"c{ci}_w"])
        assert np.array_equal(codes, d[f"c{ci}_codes"]), f"case {ci}"
        assert np.float32(scale) == d[f"c{ci}_scale"][0], f"case {ci}"


def test_fp8_forward_bf16_vs_reference():
    d = _load("fp8_from_linear_forward.npz")
    for ci in range(int(d["ncases"][0])):
        if int(d[f"c{ci}_raises"][0]):
            # only the all-zero weight (scale stored with shape [1]) raises
            assert list(d[f"c{ci}_scale_shape"]) == [1]
            continue
        x = O.from_bf16_bits(d[f"c{ci}_x"])
        bias = O.from_bf16_bits(d[f"c{ci}_bias"]) if f"c{ci}_bias" in d else None
        y = O.fp8_linear(x, d[f"c{ci}_codes"], d[f"c{ci}_scale"][0], bias)
        ref = O.from_bf16_bits(d[f"c{ci}_y"])
        assert O.rel_fro(y, ref) < 1e-2, f"case {ci}"
        # reference weight = bf16(fp8 * scale); the oracle's dequant reproduces it
        wq = O.fp8_dequant(d[f"c{ci}_codes"], d[f"c{ci}_scale"][0], "bf16")
        y2 = x @ wq.T + (0 if bias is None else bias)
        assert O.rel_fro(O.bf16_round(y2), ref) < 1e-2


def test_tp_shards_vs_reference():
    d = _load("tp_shards.npz")
    w, b = d["w"], d["b"]
    for ws in (2, 4):
        for r in range(ws):
            r0, r1 = O.column_shard_rows(w.shape[0], ws, r)
            assert np.array_equal(w[r0:r1], d[f"col_w{ws}_r{r}"])
            assert np.array_equal(b[r0:r1], d[f"col_b{ws}_r{r}"])
            c0, c1 = O.row_shard_cols(w.shape[1], ws, r)
            assert np.array_equal(w[:, c0:c1], d[f"row_w{ws}_r{r}"])


def test_row_parallel_sum_is_full_product():
    rng = np.random.default_rng(0)
    w = rng.standard_normal((16, 64)).astype(np.float32)
    x = rng.standard_normal((5, 64)).astype(np.float32)
    parts = []
    for r in range(4):
        c0, c1 = O.row_shard_cols(64, 4, r)
        parts.append(x[:, c0:c1] @ w[:, c0:c1].T)
    assert O.rel_fro(O.row_parallel_sum(parts), x @ w.T) < 1e-6
