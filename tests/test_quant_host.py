"""Host logic of the drop-in modules that needs no GPU: buffer layout contract,
state_dict compatibility, the quantize_model walk, loud failure on CPU."""

import os

import numpy as np
import pytest
import torch
import torch.nn as nn

from conftest import GOLDEN
from nanosglang_b200 import quantization as Q


def test_awq_buffers_match_reference_contract():
    m = Q.AWQLinear(896, 9728, group_size=128, bias=False)
    assert m.qweight.shape == (9728, 112) and m.qweight.dtype == torch.int32
    assert m.scales.shape == (9728, 7) and m.scales.dtype == torch.float16
    assert m.zeros.shape == (9728, 7) and m.zeros.dtype == torch.float16
    assert m.num_groups == 7 and m.group_size == 128 and m.bias is None
    m2 = Q.AWQLinear(200, 24, group_size=128, bias=True)
    assert m2.qweight.shape == (24, 25) and m2.scales.shape == (24, 2)
    assert m2.bias.shape == (24,) and m2.bias.dtype == torch.float32
    assert sorted(m2.state_dict()) == ["bias", "qweight", "scales", "zeros"]


def test_fp8_buffers_match_reference_contract():
    m = Q.FP8Linear(896, 128, bias=True)
    assert m.weight_fp8.shape == (128, 896) and m.weight_fp8.dtype == torch.float8_e4m3fn
    assert m.weight_scale.shape == (1,) and m.weight_scale.dtype == torch.float32
    assert sorted(m.state_dict()) == ["bias", "weight_fp8", "weight_scale"]


def test_cpu_forward_fails_loudly():
    m = Q.AWQLinear(128, 16)
    with pytest.raises(RuntimeError, match="no CPU fallback"):
        m(torch.randn(2, 128, dtype=torch.float16))
    f = Q.FP8Linear(128, 16)
    with pytest.raises(RuntimeError, match="no CPU fallback"):
        f(torch.randn(2, 128, dtype=torch.bfloat16))
    with pytest.raises(RuntimeError, match="no CPU fallback"):
        Q.AWQLinear.from_linear(nn.Linear(128, 16))


def _tiny_model():
    class Attn(nn.Module):
        def __init__(self):
            super().__init__()
            self.q_proj = nn.Linear(32, 32, bias=True)
            self.k_proj = nn.Linear(32, 16, bias=True)
            self.v_proj = nn.Linear(32, 16, bias=True)
            self.o_proj = nn.Linear(32, 32, bias=False)

    class MLP(nn.Module):
        def __init__(self):
            super().__init__()
            self.gate_proj = nn.Linear(32, 64, bias=False)
            self.up_proj = nn.Linear(32, 64, bias=False)
            self.down_proj = nn.Linear(64, 32, bias=False)

    class Layer(nn.Module):
        def __init__(self):
            super().__init__()
            self.self_attn = Attn()
            self.mlp = MLP()
            self.input_layernorm = nn.LayerNorm(32)

    class Model(nn.Module):
        def __init__(self):
            super().__init__()
            self.embed_tokens = nn.Embedding(10, 32)
            self.layers = nn.ModuleList([Layer(), Layer()])
            self.norm = nn.LayerNorm(32)
            self.lm_head = nn.Linear(32, 10, bias=False)
            self.extra_norm_proj = nn.Linear(32, 32)

    return Model()


class _Stub(nn.Module):
    def __init__(self, method):
        super().__init__()
        self.method = method


@pytest.mark.parametrize("method", ["fp8", "awq"])
def test_quantize_model_walk_matches_reference(method, monkeypatch, capsys):
    """Which layers get replaced (and which stay dense) is the reference's walk."""
    gold = np.load(os.path.join(GOLDEN, "quantize_model.npz"))
    monkeypatch.setitem(Q._QUANTIZERS, method, lambda child, gs: _Stub(method))
    m = _tiny_model()
    Q.quantize_model(m, method=method, group_size=32)
    replaced = [n for n, mod in m.named_modules() if isinstance(mod, _Stub)]
    dense = [n for n, mod in m.named_modules() if isinstance(mod, nn.Linear)]
    assert replaced == list(gold[f"{method}_quantized"])
    assert dense == list(gold[f"{method}_dense"])
    out = capsys.readouterr().out
    assert out.count(f"({method})") == len(replaced)


def test_quantize_model_unknown_method():
    m = _tiny_model()
    with pytest.raises(ValueError, match="Unknown quantization method"):
        Q.quantize_model(m, method="int3")
