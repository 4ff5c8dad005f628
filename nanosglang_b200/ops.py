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


try:  # the raw handle of the current stream without building a Stream object (hot path)
    _raw_stream = torch._C._cuda_getCurrentRawStream
except AttributeError:  # pragma: no cover - older torch
    _raw_stream = None


def _stream(t: torch.Tensor) -> int:
    if _raw_stream is not None:
        return _raw_stream(t.device.index)
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


def _decode_workspace(lib, quant: int, m: int, k: int, n: int, group_size: int, device):
    """(tensor, bytes) of a workspace for the decode batch sizes whose kernel
    runs faster with one (x converted once per call, ahead of the linear),
    else (None, 0). The tensor comes from the caching allocator on the
    current stream, so its reuse is stream-ordered after the launches that
    read it (also under CUDA-graph capture)."""
    if m > 64:
        return None, 0
    nbytes = lib.nsq_linear_workspace_size(quant, m, k, n, group_size)
    if not nbytes:
        return None, 0
    return torch.empty(nbytes, dtype=torch.uint8, device=device), nbytes


def awq_linear(x: torch.Tensor, qweight: torch.Tensor, scales: torch.Tensor, zeros: torch.Tensor,
               group_size: int, bias: Optional[torch.Tensor] = None) -> torch.Tensor:
    """``AWQLinear.forward`` (quantization.py:150-152) on the tensor cores.

    x: [..., K] fp16 or bf16 (the reference only accepts fp16); returns
    [..., N] in x's dtype.
    """
    if not (x.is_cuda and qweight.is_cuda and scales.is_cuda and zeros.is_cuda) or (
            bias is not None and not bias.is_cuda):
        _require_cuda(x, qweight, scales, zeros, bias, what="awq_linear")
    code = _ACT_CODES.get(x.dtype)
    if code is None:
        raise TypeError(f"activation dtype {x.dtype} not supported (float16 / bfloat16)")
    n, k8 = qweight.shape
    k = k8 * 8
    if x.shape[-1] != k:
        raise RuntimeError(f"x has {x.shape[-1]} features, the layer expects {k}")
    if not qweight.is_contiguous() or qweight.data_ptr() & 15:
        qweight = _aligned(qweight)
    if not scales.is_contiguous():
        scales = scales.contiguous()
    if not zeros.is_contiguous():
        zeros = zeros.contiguous()
    x2 = x if x.dim() == 2 else x.reshape(-1, k)
    if not x2.is_contiguous() or x2.data_ptr() & 15:
        x2 = _aligned(x2)
    m = x2.shape[0]
    y = torch.empty((m, n), dtype=x.dtype, device=x.device)
    if bias is None:
        bptr, bcode = None, _lib.DTYPE_NONE
    else:
        b, bcode = _bias_arg(bias)
        bptr = b.data_ptr()
    lib = _lib.load()
    ws, wsb = _decode_workspace(lib, 0, m, k, n, group_size, x.device)
    rc = lib.nsq_awq_linear(x2.data_ptr(), code, m, k, n, qweight.data_ptr(), scales.data_ptr(),
                            zeros.data_ptr(), group_size, bptr, bcode, y.data_ptr(),
                            None if ws is None else ws.data_ptr(), wsb, _stream(x))
    if rc:
        _lib.check(rc, "nsq_awq_linear")
    return y if x.dim() == 2 else y.reshape(*x.shape[:-1], n)


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


def awq_from_autoawq(qweight: torch.Tensor, qzeros: torch.Tensor, scales: torch.Tensor, group_size: int):
    """Repack one AutoAWQ (GEMM-format) layer into the reference layout, bit-exact.

    qweight int32 [K, N/8], qzeros int32 [K/group_size, N/8], scales fp16
    [K/group_size, N] -> (qweight int32 [N, K/8], scales fp16 [N, G], zeros
    fp16 [N, G]), the AWQLinear buffers of quantization.py:107-119.
    """
    _require_cuda(qweight, qzeros, scales, what="awq_from_autoawq")
    if qweight.dtype != torch.int32 or qzeros.dtype != torch.int32 or scales.dtype != torch.float16:
        raise TypeError("AutoAWQ layers hold int32 qweight/qzeros and float16 scales")
    k, n8 = qweight.shape
    n = n8 * 8
    g = k // group_size
    if qzeros.shape != (g, n8) or scales.shape != (g, n):
        raise ValueError(f"AutoAWQ shapes disagree: qweight {tuple(qweight.shape)}, qzeros {tuple(qzeros.shape)}, "
                         f"scales {tuple(scales.shape)}, group_size {group_size}")
    qweight, qzeros, scales = qweight.contiguous(), qzeros.contiguous(), scales.contiguous()
    out_q = torch.empty(n, k // 8, dtype=torch.int32, device=qweight.device)
    out_s = torch.empty(n, g, dtype=torch.float16, device=qweight.device)
    out_z = torch.empty(n, g, dtype=torch.float16, device=qweight.device)
    rc = _lib.load().nsq_awq_from_autoawq(_ptr(qweight), _ptr(qzeros), _ptr(scales), k, n, group_size, _ptr(out_q),
                                          _ptr(out_s), _ptr(out_z), _stream(qweight))
    _lib.check(rc, "nsq_awq_from_autoawq")
    return out_q, out_s, out_z


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


_FP8_TYPES = (torch.float8_e4m3fn, torch.uint8)


def fp8_linear(x: torch.Tensor, weight_fp8: torch.Tensor, weight_scale: torch.Tensor,
               bias: Optional[torch.Tensor] = None) -> torch.Tensor:
    """``FP8Linear.forward`` (quantization.py:49-52): W8A16, the scale is read on
    the device (no host sync). Every check is a cheap attribute test on this
    path (eager prefill pays it per linear); anything unusual takes the
    general route (copies, errors)."""
    if not (x.is_cuda and weight_fp8.is_cuda and weight_scale.is_cuda) or (bias is not None and not bias.is_cuda):
        _require_cuda(x, weight_fp8, weight_scale, bias, what="fp8_linear")
    code = _ACT_CODES.get(x.dtype)
    if code is None:
        raise TypeError(f"activation dtype {x.dtype} not supported (float16 / bfloat16)")
    if weight_fp8.dtype not in _FP8_TYPES:
        raise TypeError(f"fp8 weight must be float8_e4m3fn, got {weight_fp8.dtype}")
    w = weight_fp8
    if not w.is_contiguous() or w.data_ptr() & 15:
        w = _aligned(w)
    n, k = w.shape
    if x.shape[-1] != k:
        raise RuntimeError(f"x has {x.shape[-1]} features, the layer expects {k}")
    x2 = x if x.dim() == 2 else x.reshape(-1, k)
    if not x2.is_contiguous() or x2.data_ptr() & 15:
        x2 = _aligned(x2)
    m = x2.shape[0]
    y = torch.empty((m, n), dtype=x.dtype, device=x.device)
    if bias is None:
        bptr, bcode = None, _lib.DTYPE_NONE
    else:
        b, bcode = _bias_arg(bias)
        bptr = b.data_ptr()
    s = weight_scale
    if s.dtype != torch.float32 or s.numel() != 1 or not s.is_contiguous():
        s = _scale_arg(s)
    lib = _lib.load()
    ws, wsb = _decode_workspace(lib, 1, m, k, n, 0, x.device)
    rc = lib.nsq_fp8_linear(x2.data_ptr(), code, m, k, n, w.data_ptr(), s.data_ptr(), bptr, bcode,
                            y.data_ptr(), None if ws is None else ws.data_ptr(), wsb, _stream(x))
    if rc:
        _lib.check(rc, "nsq_fp8_linear")
    return y if x.dim() == 2 else y.reshape(*x.shape[:-1], n)


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


# ---------------------------------------------------------------------------
# Fused projections for decode batches (row-streaming kernel, M <= 32)
# ---------------------------------------------------------------------------

FUSED_MAX_M = 32


def _unwrap(mod):
    """The quantized module behind a tensor-parallel wrapper (its local shard)."""
    return getattr(mod, "linear", mod)


def _ptr_array(vals, ctype=None):
    import ctypes
    arr = (ctypes.c_void_p * len(vals))(*vals) if ctype is None else (ctype * len(vals))(*vals)
    return arr


def linear_multi(x: torch.Tensor, mods) -> Optional[list]:
    """One launch for 1..3 AWQLinear (or 1..3 FP8Linear) layers that read the
    same x, e.g. q/k/v. Returns their outputs as views of one [M, sum N]
    buffer, or None when the fused kernel does not apply (M > 32, mixed
    formats, bias dtypes that differ, group sizes that differ)."""
    import ctypes
    mods = [_unwrap(m) for m in mods]
    kinds = {type(m).__name__ for m in mods}
    if len(kinds) != 1 or x.dtype not in _ACT_CODES:
        return None
    k = x.shape[-1]
    lead = x.shape[:-1]
    x2 = _aligned(x.reshape(-1, k))
    m = x2.shape[0]
    if m == 0 or m > FUSED_MAX_M:
        return None
    biases = [mm.bias for mm in mods]
    has_bias = [b is not None for b in biases]
    if any(has_bias) and not all(has_bias):
        biases = [b if b is not None else torch.zeros(mm.out_features, device=x.device, dtype=x.dtype)
                  for b, mm in zip(biases, mods)]
    bias_dtypes = {b.dtype for b in biases if b is not None}
    if len(bias_dtypes) > 1:
        return None
    biases = [b.contiguous() for b in biases] if any(has_bias) else None
    bcode = _BIAS_CODES[biases[0].dtype] if biases else _lib.DTYPE_NONE
    ns = [mm.out_features for mm in mods]
    y = torch.empty(m, sum(ns), dtype=x.dtype, device=x.device)
    n_arr = (ctypes.c_int64 * len(ns))(*ns)
    b_arr = _ptr_array([b.data_ptr() for b in biases]) if biases else None
    lib = _lib.load()
    if kinds == {"AWQLinear"}:
        gs = {mm.group_size for mm in mods}
        if len(gs) != 1 or any(mm.in_features != k for mm in mods):
            return None
        qws = [_aligned(mm.qweight) for mm in mods]
        scs = [mm.scales.contiguous() for mm in mods]
        zrs = [mm.zeros.contiguous() for mm in mods]
        rc = lib.nsq_awq_linear_multi(_ptr(x2), _ACT_CODES[x.dtype], m, k, len(mods),
                                      _ptr_array([t.data_ptr() for t in qws]), _ptr_array([t.data_ptr() for t in scs]),
                                      _ptr_array([t.data_ptr() for t in zrs]), n_arr, gs.pop(), b_arr, bcode, _ptr(y),
                                      y.shape[1], _stream(x))
    elif kinds == {"FP8Linear"}:
        ws = [_aligned(_u8(mm.weight_fp8)) for mm in mods]
        if any(w.shape[1] != k for w in ws):
            return None
        scs = [_scale_arg(mm.weight_scale) for mm in mods]
        rc = lib.nsq_fp8_linear_multi(_ptr(x2), _ACT_CODES[x.dtype], m, k, len(mods),
                                      _ptr_array([t.data_ptr() for t in ws]), _ptr_array([t.data_ptr() for t in scs]),
                                      n_arr, b_arr, bcode, _ptr(y), y.shape[1], _stream(x))
    else:
        return None
    if rc == _lib.ENOTSUP:
        return None
    _lib.check(rc, "nsq_*_linear_multi")
    outs, c0 = [], 0
    for n in ns:
        outs.append(y[:, c0:c0 + n].reshape(*lead, n))
        c0 += n
    return outs


def gate_up_silu(x: torch.Tensor, gate, up) -> Optional[torch.Tensor]:
    """SiLU(gate(x)) * up(x) in one launch (MLP.forward's inner expression,
    causal_lm.py:482) for AWQ or FP8 gate/up layers without bias; None when
    the fused kernel does not apply (M > 32, bias, mismatched layers)."""
    gate, up = _unwrap(gate), _unwrap(up)
    if type(gate) is not type(up) or x.dtype not in _ACT_CODES or gate.bias is not None or up.bias is not None:
        return None
    k = x.shape[-1]
    lead = x.shape[:-1]
    x2 = _aligned(x.reshape(-1, k))
    m = x2.shape[0]
    n = gate.out_features
    if m == 0 or m > FUSED_MAX_M or up.out_features != n:
        return None
    y = torch.empty(m, n, dtype=x.dtype, device=x.device)
    lib = _lib.load()
    if type(gate).__name__ == "AWQLinear":
        if gate.group_size != up.group_size or gate.in_features != k or up.in_features != k:
            return None
        rc = lib.nsq_awq_gate_up_silu(_ptr(x2), _ACT_CODES[x.dtype], m, k, n, _ptr(_aligned(gate.qweight)),
                                      _ptr(gate.scales.contiguous()), _ptr(gate.zeros.contiguous()),
                                      _ptr(_aligned(up.qweight)), _ptr(up.scales.contiguous()),
                                      _ptr(up.zeros.contiguous()), gate.group_size, _ptr(y), _stream(x))
    elif type(gate).__name__ == "FP8Linear":
        wg, wu = _aligned(_u8(gate.weight_fp8)), _aligned(_u8(up.weight_fp8))
        if wg.shape[1] != k or wu.shape[1] != k:
            return None
        rc = lib.nsq_fp8_gate_up_silu(_ptr(x2), _ACT_CODES[x.dtype], m, k, n, _ptr(wg), _ptr(_scale_arg(gate.weight_scale)),
                                      _ptr(wu), _ptr(_scale_arg(up.weight_scale)), _ptr(y), _stream(x))
    else:
        return None
    if rc == _lib.ENOTSUP:
        return None
    _lib.check(rc, "nsq_*_gate_up_silu")
    return y.reshape(*lead, n)
