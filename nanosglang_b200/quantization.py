"""Drop-in replacements for nanoSGLang's quantized linears.

Same module names, constructor arguments, buffer names, dtypes and shapes as
``nano_sglang/decode/quantization.py`` (xiehuanyi/nanoSGLang), so a model
quantised with either implementation has an identical ``state_dict`` and the
unchanged Llama/Qwen2 model, scheduler and CUDA-graph decode loop can call
these modules in place of the reference's. Switching is one import::

    from nanosglang_b200.quantization import quantize_model   # instead of
    # from nano_sglang.decode.quantization import quantize_model

What changes is where the arithmetic runs: forward passes call the libnsq
sm_100a kernels on the packed buffers directly (no dequantised copy of the
weight is ever materialised), and the offline quantisers run as CUDA kernels
on the layer's device. There is no CPU path: CPU tensors raise.

Deliberate differences from the reference, all fixes of reference defects:
  * AWQLinear.forward accepts bf16 activations (the reference raises because
    its dequantised weight is fp16); output dtype follows x.
  * from_linear builds the quantised buffers on the source layer's device (the
    reference builds them on the CPU and fails for CUDA layers at ``|=``).
  * FP8Linear.forward works with the all-zero-weight scale of shape [1] (the
    reference's product promotes to fp32 and F.linear then raises for bf16 x).
"""

from __future__ import annotations

from typing import Optional

import torch
import torch.nn as nn

from . import ops

__all__ = ["FP8Linear", "AWQLinear", "quantize_model", "load_autoawq_state_dict", "FusedProjections", "GateUpSiLU"]


class FP8Linear(nn.Module):
    """Linear layer with float8_e4m3fn weight storage and one fp32 scale.

    Reference: quantization.py:24-75. ``forward`` computes
    ``x @ (weight_fp8 * weight_scale)^T + bias`` with bf16/fp16 activations
    (W8A16: activations are never quantised, as in the reference).
    """

    def __init__(self, in_features: int, out_features: int, bias: bool = False):
        super().__init__()
        self.in_features = in_features
        self.out_features = out_features
        self.register_buffer("weight_fp8", torch.zeros(out_features, in_features, dtype=torch.float8_e4m3fn))
        self.register_buffer("weight_scale", torch.ones(1))
        if bias:
            self.bias = nn.Parameter(torch.zeros(out_features))
        else:
            self.bias = None

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        return ops.fp8_linear(x, self.weight_fp8, self.weight_scale, self.bias)

    def dequantize(self, dtype: torch.dtype = torch.bfloat16) -> torch.Tensor:
        """``weight_fp8.to(dtype) * weight_scale`` (quantization.py:51), bit-exact."""
        return ops.fp8_dequant(self.weight_fp8, self.weight_scale, dtype)

    @classmethod
    def from_linear(cls, linear: nn.Linear) -> "FP8Linear":
        """Quantise a Linear to FP8 (quantization.py:54-75): scale = absmax/448
        (1 if the weight is all zero), codes = RNE e4m3 of w/scale."""
        has_bias = linear.bias is not None
        dev = linear.weight.device
        with torch.device(dev):
            fp8_linear = cls(linear.in_features, linear.out_features, bias=has_bias)
        codes, scale, absmax_zero = ops.fp8_quantize(linear.weight.data)
        fp8_linear.weight_fp8 = codes
        # the reference stores a 0-dim scale, or torch.ones(1) (shape [1]) when
        # the weight is all zero; this offline step may read that flag
        fp8_linear.weight_scale = scale.reshape(1) if bool(absmax_zero) else scale
        if has_bias:
            fp8_linear.bias = nn.Parameter(linear.bias.data.clone())
        return fp8_linear


class AWQLinear(nn.Module):
    """INT4 group-wise quantized linear layer (AWQ style).

    Reference: quantization.py:83-194. Buffers: ``qweight`` int32 [N, K//8]
    (nibble i of word j = input column 8j+i), ``scales`` and ``zeros`` fp16
    [N, ceil(K/group_size)]. ``forward`` computes
    ``x @ ((q - zeros) * scales)^T + bias`` on the packed buffers.
    """

    def __init__(self, in_features: int, out_features: int, group_size: int = 128, bias: bool = False):
        super().__init__()
        self.in_features = in_features
        self.out_features = out_features
        self.group_size = group_size
        self.num_groups = (in_features + group_size - 1) // group_size
        self.register_buffer("qweight", torch.zeros(out_features, in_features // 8, dtype=torch.int32))
        self.register_buffer("scales", torch.ones(out_features, self.num_groups, dtype=torch.float16))
        self.register_buffer("zeros", torch.zeros(out_features, self.num_groups, dtype=torch.float16))
        if bias:
            self.bias = nn.Parameter(torch.zeros(out_features))
        else:
            self.bias = None

    def _dequantize(self) -> torch.Tensor:
        """Unpack INT4 weights and dequantize to float16, bit-exact with the
        reference (quantization.py:126-148)."""
        return ops.awq_dequant(self.qweight, self.scales, self.zeros, self.in_features, self.group_size)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        return ops.awq_linear(x, self.qweight, self.scales, self.zeros, self.group_size, self.bias)

    @classmethod
    def from_linear(cls, linear: nn.Linear, group_size: int = 128) -> "AWQLinear":
        """Quantize a Linear to AWQ INT4 (quantization.py:154-194): per (row,
        group) min/max, scale = max((max-min)/15, 1e-8), zero = round(-min/scale),
        q = clamp(round((w-min)/scale), 0, 15), nibbles packed along K."""
        has_bias = linear.bias is not None
        dev = linear.weight.device
        with torch.device(dev):
            awq = cls(linear.in_features, linear.out_features, group_size, has_bias)
        qweight, scales, zeros = ops.awq_quantize(linear.weight.data, group_size)
        awq.qweight.copy_(qweight)
        awq.scales.copy_(scales)
        awq.zeros.copy_(zeros)
        if has_bias:
            awq.bias = nn.Parameter(linear.bias.data.clone())
        return awq


class FusedProjections(nn.Module):
    """Projections that read the same x (q/k/v), run as one launch for decode
    batches (M <= 32) and as the separate layers otherwise.

    The layers stay where they are (``attn.q_proj`` etc.): this module keeps
    plain references, so the model's state_dict is unchanged. The reference
    calls q/k/v one by one (causal_lm.py:295-297); ``forward`` returns the
    same three tensors.
    """

    def __init__(self, *layers: nn.Module):
        super().__init__()
        self._layers = list(layers)  # not registered: no duplicate state

    def forward(self, x: torch.Tensor):
        outs = ops.linear_multi(x, self._layers)
        if outs is None:
            outs = [layer(x) for layer in self._layers]
        return tuple(outs)


class GateUpSiLU(nn.Module):
    """``F.silu(gate_proj(x)) * up_proj(x)`` (causal_lm.py:482) as one launch
    for decode batches (M <= 32; the activation is applied in fp32 and
    rounded once), the separate layers otherwise. Keeps plain references to
    the two layers (the state_dict is unchanged)."""

    def __init__(self, gate_proj: nn.Module, up_proj: nn.Module):
        super().__init__()
        self._gate = [gate_proj]
        self._up = [up_proj]

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        y = ops.gate_up_silu(x, self._gate[0], self._up[0])
        if y is None:
            y = torch.nn.functional.silu(self._gate[0](x)) * self._up[0](x)
        return y


def load_autoawq_state_dict(model: nn.Module, state_dict: dict, group_size: int = 128) -> list:
    """Load an AutoAWQ checkpoint (GEMM format) into a model whose projections
    are AWQLinear modules (after ``quantize_model(model, "awq", group_size)``).

    For every AWQLinear ``name``, the checkpoint's ``{prefix}{name}.qweight``
    [K, N/8], ``.qzeros`` [K/G, N/8] and ``.scales`` [K/G, N] are repacked on
    the module's device into the reference layout; ``.bias`` is copied when
    present. ``prefix`` is found automatically among "", "model." (Hugging
    Face checkpoints keep the decoder under ``model.``). Returns the names of
    the modules that were loaded.
    """
    loaded = []
    for name, mod in model.named_modules():
        if not isinstance(mod, AWQLinear):
            continue
        for prefix in ("", "model."):
            key = f"{prefix}{name}."
            if key + "qweight" in state_dict:
                break
        else:
            continue
        dev = mod.qweight.device
        qw, s, z = ops.awq_from_autoawq(state_dict[key + "qweight"].to(dev), state_dict[key + "qzeros"].to(dev),
                                        state_dict[key + "scales"].to(dev), group_size)
        if qw.shape != mod.qweight.shape or s.shape != mod.scales.shape:
            raise ValueError(f"{name}: checkpoint shape {tuple(qw.shape)} does not fit {tuple(mod.qweight.shape)}")
        mod.qweight.copy_(qw)
        mod.scales.copy_(s)
        mod.zeros.copy_(z)
        if mod.bias is not None and key + "bias" in state_dict:
            mod.bias.data.copy_(state_dict[key + "bias"].to(mod.bias.device, mod.bias.dtype))
        loaded.append(name)
    return loaded


def _quantize_fp8(child: nn.Linear, group_size: int) -> nn.Module:
    return FP8Linear.from_linear(child)


def _quantize_awq(child: nn.Linear, group_size: int) -> nn.Module:
    return AWQLinear.from_linear(child, group_size)


# method name -> converter; the walk below is the reference's
_QUANTIZERS = {"fp8": _quantize_fp8, "awq": _quantize_awq}


def quantize_model(
    model: nn.Module,
    method: str = "fp8",
    group_size: int = 128,
    skip_modules: Optional[list[str]] = None,
) -> nn.Module:
    """Quantize all nn.Linear layers in a model, in place.

    Same walk as the reference (quantization.py:202-243): every child
    ``nn.Linear`` whose owning module name and full name contain none of
    ``skip_modules`` (default ``["embed_tokens", "lm_head", "norm"]``) is
    replaced by its quantised form via ``setattr``.
    """
    if skip_modules is None:
        skip_modules = ["embed_tokens", "lm_head", "norm"]
    for name, module in model.named_modules():
        if any(skip in name for skip in skip_modules):
            continue

        for child_name, child in module.named_children():
            if isinstance(child, nn.Linear):
                full_name = f"{name}.{child_name}" if name else child_name
                if any(skip in full_name for skip in skip_modules):
                    continue
                if method not in _QUANTIZERS:
                    raise ValueError(f"Unknown quantization method: {method}")
                quantized = _QUANTIZERS[method](child, group_size)
                setattr(module, child_name, quantized)
                print(f"  Quantized {full_name} ({method})")

    return model
