"""Host-side checks of libnsq that need no GPU: the C ABI loads, exports every
symbol include/nsq.h declares, and rejects bad arguments before launching."""

import ctypes
import os
import re

import pytest
import torch

from conftest import ROOT
from nanosglang_b200 import _lib, ops

HEADER = os.path.join(ROOT, "include", "nsq.h")


def _declared():
    src = open(HEADER).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    return sorted(set(re.findall(r"\b(nsq_[a-z0-9_]+)\s*\(", src)))


def test_library_loads_and_exports_header():
    lib = _lib.load()
    names = _declared()
    assert len(names) >= 12
    for n in names:
        assert hasattr(lib, n), f"libnsq.so does not export {n}"
    # the Python binding covers exactly the declared surface
    assert sorted(_lib.SIGNATURES) == names


def test_version_and_strerror():
    lib = _lib.load()
    assert lib.nsq_version() >= 100
    for code in range(0, 8):
        assert isinstance(_lib.strerror(code), str) and _lib.strerror(code)


FAKE = 0x100000  # never dereferenced: validation fails before any device access


@pytest.mark.parametrize("k,gs,expect", [(96 + 8, 128, _lib.ENOTSUP), (896, 96, _lib.ENOTSUP), (896, 0, _lib.ENOTSUP),
                                         (896, 48, _lib.ENOTSUP)])
def test_awq_linear_rejects_unsupported_shapes(k, gs, expect):
    lib = _lib.load()
    rc = lib.nsq_awq_linear(FAKE, _lib.DTYPE_BF16, 4, k, 64, FAKE, FAKE, FAKE, gs, None, _lib.DTYPE_NONE, FAKE,
                            None, 0, None)
    assert rc == expect


def test_linear_argument_validation():
    lib = _lib.load()
    # bad activation dtype
    assert lib.nsq_fp8_linear(FAKE, 7, 4, 64, 64, FAKE, FAKE, None, -1, FAKE, None, 0, None) == _lib.EINVAL
    # bias pointer without a bias dtype
    assert lib.nsq_fp8_linear(FAKE, 1, 4, 64, 64, FAKE, FAKE, FAKE, -1, FAKE, None, 0, None) == _lib.EINVAL
    # null x
    assert lib.nsq_fp8_linear(None, 1, 4, 64, 64, FAKE, FAKE, None, -1, FAKE, None, 0, None) == _lib.EINVAL
    # misaligned y
    assert lib.nsq_fp8_linear(FAKE, 1, 4, 64, 64, FAKE, FAKE, None, -1, FAKE + 2, None, 0, None) == _lib.EALIGN
    # K not a multiple of 16 (fp8 rows must be 16-byte multiples for TMA)
    assert lib.nsq_fp8_linear(FAKE, 1, 4, 72, 64, FAKE, FAKE, None, -1, FAKE, None, 0, None) == _lib.ENOTSUP
    # negative sizes
    assert lib.nsq_awq_linear(FAKE, 1, -1, 128, 64, FAKE, FAKE, FAKE, 128, None, -1, FAKE, None, 0,
                              None) == _lib.EINVAL
    # M == 0 is a no-op, needs no device
    assert lib.nsq_awq_linear(FAKE, 1, 0, 128, 64, FAKE, FAKE, FAKE, 128, None, -1, FAKE, None, 0,
                              None) == _lib.OK


def test_dequant_and_quantize_validation():
    lib = _lib.load()
    # in_features % 8 != 0 raises in the reference too
    assert lib.nsq_awq_dequant(FAKE, FAKE, FAKE, FAKE, 16, 100, 128, None) == _lib.EINVAL
    assert lib.nsq_awq_dequant(FAKE + 4, FAKE, FAKE, FAKE, 16, 128, 128, None) == _lib.EALIGN
    assert lib.nsq_fp8_dequant(FAKE, FAKE, FAKE, 2, 4, 16, None) == _lib.EINVAL  # fp32 output not offered
    assert lib.nsq_awq_quantize(FAKE, 1, 4, 4, 128, FAKE, FAKE, FAKE, None) == _lib.EINVAL  # K < 8
    ws = lib.nsq_fp8_quantize_workspace_size(16, 16)
    assert ws >= 4
    assert lib.nsq_fp8_quantize(FAKE, 1, 16, 16, FAKE, FAKE, FAKE, ws - 1, None) == _lib.EWORKSPACE


def test_ops_refuse_cpu_tensors():
    x = torch.randn(2, 128, dtype=torch.bfloat16)
    qw = torch.zeros(16, 16, dtype=torch.int32)
    s = torch.ones(16, 1, dtype=torch.float16)
    z = torch.zeros(16, 1, dtype=torch.float16)
    with pytest.raises(RuntimeError, match="no CPU fallback"):
        ops.awq_linear(x, qw, s, z, 128)
    with pytest.raises(RuntimeError, match="no CPU fallback"):
        ops.awq_dequant(qw, s, z, 128, 128)
    w8 = torch.zeros(16, 128, dtype=torch.float8_e4m3fn)
    with pytest.raises(RuntimeError, match="no CPU fallback"):
        ops.fp8_linear(x, w8, torch.ones(()))


def test_error_object_carries_code():
    e = _lib.NsqError(_lib.EALIGN, "nsq_fp8_linear")
    assert e.code == _lib.EALIGN and "aligned" in str(e)
    with pytest.raises(_lib.NsqError):
        _lib.check(_lib.EINVAL, "x")
