"""The allocation-free weight edit, through the C ABI.

Callers that cannot allocate device memory (a host whose pool owns all of
HBM, code that must not synchronise the device, a caller without a device
handle) use ditch_cuda_edit_weight_bf16_noalloc, whose scratch is a fixed
array in the library. Its result must match ditch_cuda_edit_weight_bf16 on
the same input, call after call: the shared scratch keeps the previous call's
contents, and the second, smaller call below would pick up stale partial sums
if the entry did not clear them.

This file is collected last so that a failure here comes after every other
test has run.
"""
import ctypes as C

import numpy as np
import pytest

import ditch_b200
import oracle
from ditch_b200 import cuda

pytestmark = pytest.mark.gpu


def _close(got, want, atol=2e-5, rtol=8e-3):
    err = np.abs(got.astype(np.float64) - want.astype(np.float64))
    assert np.all(err <= atol + rtol * np.abs(want)), f"max err {err.max():.3g}"


def test_no_alloc_edit_matches_edit_weight(device):
    torch = pytest.importorskip("torch")
    lib = ditch_b200.lib()
    fn = lib.ditch_cuda_edit_weight_bf16_noalloc
    rng = np.random.default_rng(4242)
    for rows, cols, alpha in ((512, 1536, 0.8), (96, 200, 1.3)):  # two calls in a row, the second smaller
        w0 = oracle.f32_to_bf16_bits((rng.standard_normal((rows, cols)) * 0.02).astype(np.float32))
        r = rng.standard_normal(rows).astype(np.float32)
        r /= np.linalg.norm(r)
        rt = torch.from_numpy(r).cuda()
        wa = torch.from_numpy(w0.view(np.int16).copy()).cuda()
        wb = torch.from_numpy(w0.view(np.int16).copy()).cuda()
        device.edit_weight_bf16(wa.data_ptr(), rows, cols, rt.data_ptr(), alpha)
        stream = torch.cuda.current_stream().cuda_stream
        assert fn(C.c_void_p(wb.data_ptr()), rows, cols, C.c_void_p(rt.data_ptr()), alpha, C.c_void_p(stream)) == 0
        torch.cuda.synchronize()
        got = oracle.bf16_bits_to_f32(wb.cpu().numpy().view(np.uint16))
        want = oracle.bf16_bits_to_f32(wa.cpu().numpy().view(np.uint16))
        _close(got, want)
        assert not np.array_equal(got, oracle.bf16_bits_to_f32(w0))  # the edit did something


def test_no_alloc_edit_rejects_oversize():
    lib = ditch_b200.lib()
    fn = lib.ditch_cuda_edit_weight_bf16_noalloc
    dummy = C.c_void_p(16)  # never dereferenced: the size check comes first
    assert fn(dummy, 1 << 20, 8, dummy, 1.0, None) == cuda.INVALID
    assert b"exceeds the fixed scratch" in lib.ditch_cuda_last_error()
