"""The allocation-free Q4_K entry point, eosi_cuda_matmul_q4_k_noalloc.

It exists for hosts that may not allocate device memory once they run --
deployments that reserve every buffer at start-up, or hosts whose own pool
owns all device memory -- and keeps its packed activations in a 1 MiB array
built into the library instead of a caller scratch buffer.  Its results must
be bit-identical to the allocating entry point's (Q4_K is bit-exact in every
test of this suite), on consecutive calls that reuse the shared array.

This file is collected last (its name sorts after the others) and passes
both alone in a fresh process and after the rest of the suite.
"""
import ctypes as C

import numpy as np
import pytest
import torch

from conftest import same_bits

pytestmark = pytest.mark.gpu


def _call_noalloc(lib, a, w, c, m, n, k):
    st = torch.cuda.current_stream().cuda_stream
    return lib.eosi_cuda_matmul_q4_k_noalloc(C.c_void_p(a.data_ptr()), C.c_void_p(w.data_ptr()),
                                             C.c_void_p(c.data_ptr()), m, n, k, C.c_void_p(st))


def _call_reference_entry(lib, a, w, c, m, n, k, scratch):
    st = torch.cuda.current_stream().cuda_stream
    return lib.eosi_cuda_matmul_q4_k_dev(C.c_void_p(a.data_ptr()), C.c_void_p(w.data_ptr()),
                                         C.c_void_p(c.data_ptr()), m, n, k, C.c_void_p(scratch.data_ptr()),
                                         C.c_void_p(st))


# (1, 64, 131072): rows too long to stage in shared memory, the unstaged kernel
@pytest.mark.parametrize("m,n,k", [(1, 4096, 4096), (1, 4096, 11008), (3, 1000, 4096), (1, 2, 512),
                                   (1, 64, 131072)])
def test_noalloc_matches_allocating_entry_point(gpu, m, n, k):
    _compare_on_device(gpu, 0, m, n, k)


def test_noalloc_on_a_second_device(gpu):
    """The array's address is looked up per device: a call on device 1 must
    use device 1's copy."""
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    with torch.cuda.device(1):
        _compare_on_device(gpu, 1, 1, 4096, 4096)
    _compare_on_device(gpu, 0, 1, 4096, 4096)  # and device 0 still uses its own


def _compare_on_device(gpu, index, m, n, k):
    lib = gpu.load()
    dev = torch.device("cuda", index)
    w = torch.empty(n * (k // 256) * 144, dtype=torch.uint8, device=dev)
    gpu.q4_k_from_gauss_dev(w, n * k, 11, 0.02)
    scratch = torch.empty(gpu.q4_k_scratch_bytes(m, k), dtype=torch.uint8, device=dev)
    # two calls in a row with different activations: the second must not see
    # anything left in the shared array by the first
    for seed in (21, 22):
        a = torch.empty(m * k, dtype=torch.float32, device=dev)
        gpu.fill_gauss_dev(a, m * k, seed, 0, 1.0)
        c_ref = torch.full((m * n,), np.nan, dtype=torch.float32, device=dev)
        c_new = torch.full((m * n,), np.nan, dtype=torch.float32, device=dev)
        assert _call_reference_entry(lib, a, w, c_ref, m, n, k, scratch) == gpu.EOS_OK, gpu.last_error()
        assert _call_noalloc(lib, a, w, c_new, m, n, k) == gpu.EOS_OK, gpu.last_error()
        torch.cuda.synchronize()
        assert same_bits(c_new.cpu().numpy(), c_ref.cpu().numpy()), (m, n, k, seed)
        assert not np.isnan(c_new.cpu().numpy()).any()
        # no bounded wait of either entry point ran out (the no-alloc call
        # reports into its own word, read by the same query)
        bits = C.c_uint32(0xFFFFFFFF)
        assert lib.eosi_cuda_take_device_errors(C.byref(bits)) == gpu.EOS_OK, gpu.last_error()
        assert bits.value == 0


def test_noalloc_rejects_sizes_beyond_its_array(gpu):
    lib = gpu.load()
    dev = torch.device("cuda", 0)
    k = 4096
    m = 137  # 137 * 16 * 480 bytes > 1 MiB
    a = torch.zeros(m * k, dtype=torch.float32, device=dev)
    w = torch.zeros(8 * (k // 256) * 144, dtype=torch.uint8, device=dev)
    c = torch.full((m * 8,), 7.0, dtype=torch.float32, device=dev)
    assert _call_noalloc(lib, a, w, c, m, 8, k) == gpu.EOS_E_INVALID_ARG
    assert "1 MiB" in gpu.last_error()
    torch.cuda.synchronize()
    assert torch.all(c == 7.0)
    assert _call_noalloc(lib, a, w, c, 136, 8, k) == gpu.EOS_OK  # the largest m that fits


def test_noalloc_leaves_free_device_memory_unchanged(gpu):
    """After one warm-up call per shape class (the driver loads each kernel
    on its first launch under lazy module loading), calls of every class
    leave free device memory unchanged."""
    lib = gpu.load()
    dev = torch.device("cuda", 0)
    shapes = [(1, 2048, 4096), (2, 1024, 11008), (1, 2, 4096)]  # short rows, long rows, n < 4
    bufs = []
    for m, n, k in shapes:
        w = torch.empty(n * (k // 256) * 144, dtype=torch.uint8, device=dev)
        gpu.q4_k_from_gauss_dev(w, n * k, 5, 0.02)
        a = torch.ones(m * k, dtype=torch.float32, device=dev)
        c = torch.empty(m * n, dtype=torch.float32, device=dev)
        bufs.append((a, w, c, m, n, k))
        assert _call_noalloc(lib, a, w, c, m, n, k) == gpu.EOS_OK  # warm-up (the first also sets the device up)
    torch.cuda.synchronize()
    free_before, _ = torch.cuda.mem_get_info(dev)
    for _ in range(10):
        for a, w, c, m, n, k in bufs:
            assert _call_noalloc(lib, a, w, c, m, n, k) == gpu.EOS_OK
    torch.cuda.synchronize()
    free_after, _ = torch.cuda.mem_get_info(dev)
    assert free_after == free_before
