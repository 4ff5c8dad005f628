"""The allocation-free FP8 quantiser, called through the C ABI.

nsq_fp8_quantize_noalloc exists for callers that cannot allocate device
memory when they quantise a weight: code running inside a global-mode CUDA
stream capture (where cudaMalloc is not allowed), engines that reserve nearly
all HBM for their KV-cache pool up front, and C callers without a device
allocator. It must give exactly what the workspace-taking nsq_fp8_quantize
gives (the quantisation tests are bit-exact), call after call, even though
every call reuses the same scratch array inside the library.

This file is collected last on purpose: if it fails, a run that stops at the
first failure has already run every other test.
"""

import ctypes

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module", autouse=True)
def _cuda():
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")


def _noalloc(lib, w):
    n, k = w.shape
    codes = torch.empty(n, k, dtype=torch.uint8, device=w.device)
    scale = torch.empty((), dtype=torch.float32, device=w.device)
    rc = lib.nsq_fp8_quantize_noalloc(ctypes.c_void_p(w.data_ptr()), 2, n, k, ctypes.c_void_p(codes.data_ptr()),
                                      ctypes.c_void_p(scale.data_ptr()),
                                      ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
    return rc, codes, scale


def _with_workspace(lib, w):
    n, k = w.shape
    ws_bytes = lib.nsq_fp8_quantize_workspace_size(n, k)
    ws = torch.empty(ws_bytes, dtype=torch.uint8, device=w.device)
    codes = torch.empty(n, k, dtype=torch.uint8, device=w.device)
    scale = torch.empty((), dtype=torch.float32, device=w.device)
    rc = lib.nsq_fp8_quantize(ctypes.c_void_p(w.data_ptr()), 2, n, k, ctypes.c_void_p(codes.data_ptr()),
                              ctypes.c_void_p(scale.data_ptr()), ctypes.c_void_p(ws.data_ptr()), ws_bytes,
                              ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
    return rc, codes, scale


def test_noalloc_quantizer_matches_workspace_quantizer_call_after_call():
    from nanosglang_b200 import _lib
    lib = _lib.load()
    g = torch.Generator().manual_seed(11)
    # the second weight has a smaller absmax than the first, so a scratch word
    # left over from the first call would give a wrong scale; the third is all
    # zero (scale 1)
    weights = [torch.randn(320, 896, generator=g) * 0.05,
               torch.randn(96, 4864, generator=g) * 0.01,
               torch.zeros(16, 256)]
    for i, w in enumerate(weights):
        w = w.cuda()
        rc, codes, scale = _noalloc(lib, w)
        assert rc == 0, _lib.strerror(rc)
        rc_ref, codes_ref, scale_ref = _with_workspace(lib, w)
        assert rc_ref == 0
        torch.cuda.synchronize()
        assert torch.equal(codes, codes_ref), f"call {i}: codes differ"
        assert torch.equal(scale, scale_ref), f"call {i}: scale {scale.item()} vs {scale_ref.item()}"
    code, where, block = _lib.device_status()
    assert code == 0


def test_noalloc_quantizer_rejects_bad_arguments():
    from nanosglang_b200 import _lib
    lib = _lib.load()
    fake = ctypes.c_void_p(0x100000)
    assert lib.nsq_fp8_quantize_noalloc(fake, 9, 4, 16, fake, fake, None) == _lib.EINVAL
    assert lib.nsq_fp8_quantize_noalloc(fake, 2, -1, 16, fake, fake, None) == _lib.EINVAL
    assert lib.nsq_fp8_quantize_noalloc(fake, 2, 4, 16, fake, None, None) == _lib.EINVAL
