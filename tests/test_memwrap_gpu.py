"""GPU checks of the CUDA memory wrappers through the C ABI, with the reference's return
conventions (src/cuda/api/cuda_mem_wrapper.cuh:10-16): b32 wrappers answer 1 on success,
cu_memcpy_htd / cu_memcpy_dth return Success (0)."""
import ctypes as C

import numpy as np
import pytest

import infb200 as I

pytestmark = pytest.mark.gpu


def test_memory_wrappers_round_trip(cuda):
    torch = cuda
    L = I.lib()
    p = I.vp()
    assert L.cu_malloc(C.byref(p), 4096) == 1 and p.value  # D10 fixed: the allocation reaches the caller
    assert L.cu_memset(p, 0x5A, 4096) == 1
    got = np.zeros(4096, np.uint8)
    assert L.cu_memcpy_dth(got.ctypes.data, p, 4096) == 0
    assert (got == 0x5A).all()
    src = np.arange(4096, dtype=np.uint8)
    assert L.cu_host_register_read_only(src.ctypes.data, src.nbytes) == 1
    stream = torch.cuda.Stream()
    assert L.cu_memcpy_htd_async(p, src.ctypes.data, 4096, I.vp(stream.cuda_stream)) == 1
    stream.synchronize()
    torch.cuda.cudart().cudaHostUnregister(src.ctypes.data)
    assert L.cu_memcpy_htd(p, src.ctypes.data, 1024) == 0
    assert L.cu_memcpy_dth(got.ctypes.data, p, 4096) == 0
    np.testing.assert_array_equal(got, src)
    assert L.cu_host_register_read_only(p, 16) == 0  # device memory is refused
    assert L.cu_free(p) == 1
    host = np.zeros(16, np.uint8)
    assert L.cu_free(host.ctypes.data) == 0
    assert L.cu_memset(host.ctypes.data, 0, 16) == 0
