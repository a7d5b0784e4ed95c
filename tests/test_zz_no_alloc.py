"""The allocation-free C entry point ``radiance_argmax_rows_noalloc`` (csrc/argmax_noalloc.cu,
declared in csrc/radiance_noalloc.h), called through its exported C symbol in the torch-free
library libradiance_noalloc.so: it agrees with the torch-facing argmax op on two calls in a row,
allocates no device memory once set up, and rejects arguments beyond its fixed scratch.

Callers of this entry point cannot allocate when they need a token: a C or C++ host without torch
has no caching allocator, a process whose KV cache holds nearly all HBM may see a late cudaMalloc
fail, and a latency-bound decode loop cannot absorb cudaMalloc's device-wide synchronisation."""
import ctypes
import os

import pytest
import torch

pytestmark = pytest.mark.gpu

LIB = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))),
                   "vllm_sly_radiance_b200", "libradiance_noalloc.so")


def _lib():
    assert os.path.exists(LIB), "libradiance_noalloc.so is built by setup.py build_ext"
    lib = ctypes.CDLL(LIB)
    fn = lib.radiance_argmax_rows_noalloc
    fn.restype = ctypes.c_int
    fn.argtypes = [ctypes.c_void_p, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_longlong,
                   ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_char_p, ctypes.c_int]
    return fn


def _call(fn, x, ids, vals, dtype=None, ld=None):
    err = ctypes.create_string_buffer(256)
    if dtype is None:
        dtype = 0 if x.dtype == torch.bfloat16 else 1
    rc = fn(x.data_ptr(), dtype, x.shape[0], x.shape[1], x.stride(0) if ld is None else ld,
            ids.data_ptr(), vals.data_ptr() if vals is not None else None,
            torch.cuda.current_stream().cuda_stream, err, len(err))
    return rc, err.value.decode()


@pytest.mark.parametrize("dtype,rows,vocab", [(torch.bfloat16, 3, 248320),
                                              (torch.float32, 17, 4096 * 3 + 5),
                                              (torch.bfloat16, 64, 1000)])
def test_noalloc_argmax_matches_op(dtype, rows, vocab):
    from vllm_sly_radiance_b200.ops import kernels as K
    fn = _lib()
    torch.manual_seed(0)
    for call in range(2):
        x = torch.randn(rows, vocab, device="cuda").to(dtype)
        if call == 1:
            x[:, 7] = 50.0        # ties: the lowest index wins in both paths
            x[:, vocab - 3] = 50.0
        ids = torch.full((rows,), -1, dtype=torch.int64, device="cuda")
        vals = torch.zeros(rows, dtype=torch.float32, device="cuda")
        rc, msg = _call(fn, x, ids, vals)
        assert rc == 0, msg
        want = K.argmax(x)
        torch.cuda.synchronize()
        assert torch.equal(ids, want), (call, ids, want)
        ref_vals = x.float().gather(1, want[:, None])[:, 0]
        assert torch.allclose(vals, ref_vals, rtol=0, atol=0)


def test_noalloc_argmax_strided_rows():
    from vllm_sly_radiance_b200.ops import kernels as K
    fn = _lib()
    big = torch.randn(5, 9000, device="cuda", dtype=torch.bfloat16)
    x = big[:, :8192]                       # row stride 9000, vocab 8192
    ids = torch.empty(5, dtype=torch.int64, device="cuda")
    for _ in range(2):
        rc, msg = _call(fn, x, ids, None)
        assert rc == 0, msg
        assert torch.equal(ids, K.argmax(x.contiguous()))


def test_noalloc_argmax_allocates_no_device_memory():
    """Once the first call has set up the scratch, calls leave the device's free memory as it
    was (cudaMemGetInfo sees raw allocations; the tensors are made before the first reading)."""
    fn = _lib()
    x = torch.randn(8, 248320, device="cuda", dtype=torch.bfloat16)
    ids = torch.empty(8, dtype=torch.int64, device="cuda")
    vals = torch.empty(8, dtype=torch.float32, device="cuda")
    rc, msg = _call(fn, x, ids, vals)
    assert rc == 0, msg
    torch.cuda.synchronize()
    free0 = torch.cuda.mem_get_info()[0]
    for _ in range(20):
        rc, msg = _call(fn, x, ids, vals)
        assert rc == 0, msg
    torch.cuda.synchronize()
    assert torch.cuda.mem_get_info()[0] == free0
    assert torch.equal(ids, x.float().argmax(-1))


def test_noalloc_argmax_rejects_bad_arguments():
    fn = _lib()
    x = torch.zeros(1025, 8, device="cuda", dtype=torch.float32)
    ids = torch.empty(1025, dtype=torch.int64, device="cuda")
    rc, msg = _call(fn, x, ids, None)
    assert rc != 0 and "rows must be in [1, 1024]" in msg
    y = torch.zeros(2, 64, device="cuda", dtype=torch.float32)
    rc, msg = _call(fn, y, ids, None, ld=32)                  # row stride below the vocabulary
    assert rc == -1 and "ld >= vocab" in msg
    rc, msg = _call(fn, y, ids, None, dtype=2)
    assert rc == -1 and "dtype must be 0 (bf16) or 1 (fp32)" in msg
