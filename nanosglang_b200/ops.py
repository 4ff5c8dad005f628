"""Torch-level wrappers of libnsq: device memory, dtypes and streams come from
PyTorch, all arithmetic runs in the library's sm_100a kernels.

Every function launches on ``torch.cuda.current_stream()`` (the capture stream
while a CUDA graph is being recorded), allocates its outputs through the torch
caching allocator and never synchronises the host, so the linears can live
inside the reference's CUDA-graph decode loop. Tensors on any other device
raise: there is no CPU path.
"""

from __future__ import annotations

from typing import Optional

import torch

from . import _lib

_ACT_CODES = {torch.float16: _lib.DTYPE_F16, torch.bfloat16: _lib.DTYPE_BF16}
_BIAS_CODES = {torch.float16: _lib.DTYPE_F16, torch.bfloat16: _lib.DTYPE_BF16, torch.float32: _lib.DTYPE_F32}


def _stream(t: torch.Tensor) -> int:
    return torch.cuda.current_stream(t.device).cuda_stream


def _require_cuda(*ts, what: str) -> None:
    for t in ts:
        if t is not None and not t.is_cuda:
            raise RuntimeError(
                f"{what}: nanosglang_b200 runs on CUDA (sm_100a) only; got a tensor on {t.device}. "
                "There is no CPU fallback.")


def _aligned(t: torch.Tensor) -> torch.Tensor:
    """Contiguous, 16-byte aligned view (copies only when needed)."""
    if not t.is_contiguous():
        t = t.contiguous()
    if t.data_ptr() % 16 != 0:
        t = t.clone()
    return t


def _ptr(t: Optional[torch.Tensor]):
    return None if t is None else t.data_ptr()


def _bias_arg(bias: Optional[torch.Tensor]):
    if bias is None:
        return None, _lib.DTYPE_NONE
    if bias.dtype not in _BIAS_CODES:
        raise TypeError(f"bias dtype {bias.dtype} not supported")
    bias = bias.contiguous()
    return bias, _BIAS_CODES[bias.dtype]


# ---------------------------------------------------------------------------
# AWQ
# ---------------------------------------------------------------------------


def awq_dequant(qweight: torch.Tensor, scales: torch.Tensor, zeros: torch.Tensor, in_features: int,
                group_size: int) -> torch.Tensor:
    """Bit-exact ``AWQLinear._dequantize`` (quantization.py:126-148) -> fp16 [N, K]."""
    _require_cuda(qweight, scales, zeros, what="awq_dequant")
    n = qweight.shape[0]
    if in_features % 8 != 0 or qweight.shape[1] * 8 != in_features:
        raise RuntimeError("AWQ dequantisation needs in_features == 8 * qweight.shape[1] "
                           "(the reference raises in this case as well)")
    qweight = _aligned(qweight)
    scales = scales.contiguous()
    zeros = zeros.contiguous()
    if scales.dtype != torch.float16 or zeros.dtype != torch.float16:
        raise TypeError("scales and zeros must be float16 (reference layout)")
    out = torch.empty(n, in_features, dtype=torch.float16, device=qweight.device)
    rc = _lib.load().nsq_awq_dequant(_ptr(qweight), _ptr(scales), _ptr(zeros), _ptr(out), n, in_features,
                                     group_size, _stream(qweight))
    _lib.check(rc, "nsq_awq_dequant")
    return out


def awq_linear(x: torch.Tensor, qweight: torch.Tensor, scales: torch.Tensor, zeros: torch.Tensor,
               group_size: int, bias: Optional[torch.Tensor] = None) -> torch.Tensor:
    """``AWQLinear.forward`` (quantization.py:150-152) on the tensor cores.

    x: [..., K] fp16 or bf16 (the reference only accepts fp16); returns
    [..., N] in x's dtype.
    """
    _require_cuda(x, qweight, scales, zeros, bias, what="awq_linear")
    if x.dtype not in _ACT_CODES:
        raise TypeError(f"activation dtype {x.dtype} not supported (float16 / bfloat16)")
    k = qweight.shape[1] * 8
    n = qweight.shape[0]
    if x.shape[-1] != k:
        raise RuntimeError(f"x has {x.shape[-1]} features, the layer expects {k}")
    lead = x.shape[:-1]
    x2 = _aligned(x.reshape(-1, k))
    m = x2.shape[0]
    y = torch.empty(m, n, dtype=x.dtype, device=x.device)
    b, bcode = _bias_arg(bias)
    rc = _lib.load().nsq_awq_linear(_ptr(x2), _ACT_CODES[x.dtype], m, k, n, _ptr(_aligned(qweight)),
                                    _ptr(scales.contiguous()), _ptr(zeros.contiguous()), group_size, _ptr(b),
                                    bcode, _ptr(y), None, 0, _stream(x))
    _lib.check(rc, "nsq_awq_linear")
    return y.reshape(*lead, n)


def awq_quantize(weight: torch.Tensor, group_size: int = 128):
    """``AWQLinear.from_linear`` arithmetic (quantization.py:154-194) on the GPU.

    Returns (qweight int32 [N, K//8], scales fp16 [N, G], zeros fp16 [N, G]).
    """
    _require_cuda(weight, what="awq_quantize")
    if weight.dtype not in _BIAS_CODES:
        raise TypeError(f"weight dtype {weight.dtype} not supported")
    weight = weight.contiguous()
    n, k = weight.shape
    g = (k + group_size - 1) // group_size
    qweight = torch.empty(n, k // 8, dtype=torch.int32, device=weight.device)
    scales = torch.empty(n, g, dtype=torch.float16, device=weight.device)
    zeros = torch.empty(n, g, dtype=torch.float16, device=weight.device)
    rc = _lib.load().nsq_awq_quantize(_ptr(weight), _BIAS_CODES[weight.dtype], n, k, group_size, _ptr(qweight),
                                      _ptr(scales), _ptr(zeros), _stream(weight))
    _lib.check(rc, "nsq_awq_quantize")
    return qweight, scales, zeros


# ---------------------------------------------------------------------------
# FP8
# ---------------------------------------------------------------------------


def _u8(w: torch.Tensor) -> torch.Tensor:
    if w.dtype == torch.float8_e4m3fn:
        return w.view(torch.uint8)
    if w.dtype == torch.uint8:
        return w
    raise TypeError(f"fp8 weight must be float8_e4m3fn, got {w.dtype}")


def _scale_arg(weight_scale: torch.Tensor) -> torch.Tensor:
    if weight_scale.numel() != 1:
        raise RuntimeError("weight_scale must hold exactly one value (per-tensor scale)")
    if weight_scale.dtype != torch.float32:
        weight_scale = weight_scale.float()
    return weight_scale.contiguous()


def fp8_linear(x: torch.Tensor, weight_fp8: torch.Tensor, weight_scale: torch.Tensor,
               bias: Optional[torch.Tensor] = None) -> torch.Tensor:
    """``FP8Linear.forward`` (quantization.py:49-52): W8A16, the scale is read on
    the device (no host sync)."""
    _require_cuda(x, weight_fp8, weight_scale, bias, what="fp8_linear")
    if x.dtype not in _ACT_CODES:
        raise TypeError(f"activation dtype {x.dtype} not supported (float16 / bfloat16)")
    w = _aligned(_u8(weight_fp8))
    n, k = w.shape
    if x.shape[-1] != k:
        raise RuntimeError(f"x has {x.shape[-1]} features, the layer expects {k}")
    lead = x.shape[:-1]
    x2 = _aligned(x.reshape(-1, k))
    m = x2.shape[0]
    y = torch.empty(m, n, dtype=x.dtype, device=x.device)
    b, bcode = _bias_arg(bias)
    s = _scale_arg(weight_scale)
    rc = _lib.load().nsq_fp8_linear(_ptr(x2), _ACT_CODES[x.dtype], m, k, n, _ptr(w), _ptr(s), _ptr(b), bcode,
                                    _ptr(y), None, 0, _stream(x))
    _lib.check(rc, "nsq_fp8_linear")
    return y.reshape(*lead, n)


def fp8_dequant(weight_fp8: torch.Tensor, weight_scale: torch.Tensor, dtype: torch.dtype) -> torch.Tensor:
    """Bit-exact ``weight_fp8.to(dtype) * weight_scale`` (quantization.py:51)."""
    _require_cuda(weight_fp8, weight_scale, what="fp8_dequant")
    if dtype not in _ACT_CODES:
        raise TypeError(f"dtype {dtype} not supported")
    w = _aligned(_u8(weight_fp8))
    n, k = w.shape
    out = torch.empty(n, k, dtype=dtype, device=w.device)
    s = _scale_arg(weight_scale)
    rc = _lib.load().nsq_fp8_dequant(_ptr(w), _ptr(s), _ptr(out), _ACT_CODES[dtype], n, k, _stream(w))
    _lib.check(rc, "nsq_fp8_dequant")
    return out


def fp8_quantize(weight: torch.Tensor):
    """``FP8Linear.from_linear`` arithmetic (quantization.py:54-75) on the GPU.

    Returns (weight_fp8 float8_e4m3fn [N, K], scale fp32 0-dim, absmax_is_zero
    as a 0-dim bool tensor on the device)."""
    _require_cuda(weight, what="fp8_quantize")
    if weight.dtype not in _BIAS_CODES:
        raise TypeError(f"weight dtype {weight.dtype} not supported")
    weight = weight.contiguous()
    n, k = weight.shape
    lib = _lib.load()
    ws_bytes = lib.nsq_fp8_quantize_workspace_size(n, k)
    ws = torch.empty(ws_bytes, dtype=torch.uint8, device=weight.device)
    codes = torch.empty(n, k, dtype=torch.uint8, device=weight.device)
    scale = torch.empty((), dtype=torch.float32, device=weight.device)
    rc = lib.nsq_fp8_quantize(_ptr(weight), _BIAS_CODES[weight.dtype], n, k, _ptr(codes), _ptr(scale), _ptr(ws),
                              ws_bytes, _stream(weight))
    _lib.check(rc, "nsq_fp8_quantize")
    absmax_zero = ws[:4].view(torch.int32)[0] == 0
    return codes.view(torch.float8_e4m3fn), scale, absmax_zero
