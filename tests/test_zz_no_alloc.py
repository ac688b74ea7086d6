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
    # two calls in a row, the second smaller; the third edits a matrix that
    # starts one element (2 bytes) past a 16-byte boundary, as a view at a
    # storage offset does, which the kernels read and write 2 bytes at a time
    for rows, cols, alpha, off in ((512, 1536, 0.8, 0), (96, 200, 1.3, 0), (64, 256, 0.9, 1)):
        w0 = oracle.f32_to_bf16_bits((rng.standard_normal((rows, cols)) * 0.02).astype(np.float32))
        r = rng.standard_normal(rows).astype(np.float32)
        r /= np.linalg.norm(r)
        rt = torch.from_numpy(r).cuda()
        flat = np.concatenate([np.zeros(off, np.uint16), w0.reshape(-1)])
        wa = torch.from_numpy(flat.view(np.int16).copy()).cuda()
        wb = torch.from_numpy(flat.view(np.int16).copy()).cuda()
        pa, pb = wa.data_ptr() + 2 * off, wb.data_ptr() + 2 * off
        assert (pb & 15) == (2 * off)  # torch's allocations start on 256-byte boundaries
        device.edit_weight_bf16(pa, rows, cols, rt.data_ptr(), alpha)
        stream = torch.cuda.current_stream().cuda_stream
        assert fn(C.c_void_p(pb), rows, cols, C.c_void_p(rt.data_ptr()), alpha, C.c_void_p(stream)) == 0
        torch.cuda.synchronize()
        got = oracle.bf16_bits_to_f32(wb.cpu().numpy().view(np.uint16)[off:].reshape(rows, cols))
        want = oracle.bf16_bits_to_f32(wa.cpu().numpy().view(np.uint16)[off:].reshape(rows, cols))
        _close(got, want)
        # and against the oracle's f32 edit (src/abliterate.zig:264-280) rounded once to bf16
        wf = oracle.bf16_bits_to_f32(w0)
        a, b = oracle.compute_delta_none(wf, r, alpha)
        _close(got, oracle.materialize(wf, a, b))
        assert not np.array_equal(got, wf)  # the edit did something


def test_no_alloc_edit_rejects_oversize():
    lib = ditch_b200.lib()
    fn = lib.ditch_cuda_edit_weight_bf16_noalloc
    dummy = C.c_void_p(16)  # never dereferenced: the size check comes first
    assert fn(dummy, 1 << 20, 8, dummy, 1.0, None) == cuda.INVALID
    assert b"exceeds the fixed scratch" in lib.ditch_cuda_last_error()


def test_no_alloc_edit_rejects_odd_pointers():
    """A bf16 matrix must start on a 2-byte boundary and r on a 4-byte one;
    anything else is refused before a kernel is launched (the pointers here
    are never dereferenced)."""
    lib = ditch_b200.lib()
    fn = lib.ditch_cuda_edit_weight_bf16_noalloc
    assert fn(C.c_void_p(17), 8, 8, C.c_void_p(16), 1.0, None) == cuda.INVALID
    assert b"aligned" in lib.ditch_cuda_last_error()
    assert fn(C.c_void_p(16), 8, 8, C.c_void_p(18), 1.0, None) == cuda.INVALID
