"""Tensor-core prefill GEMM (eosllm_b200/csrc/prefill_gemm.cu) against the
oracle's int8 matmul, which is the reference's own arithmetic
(eosi_avx2_matmul_q4_k_int8, matmul_q4_k_int8.c:164-269): the bar is bit for
bit.  Every sub-block dot is exact on the tensor cores (integers held in bf16,
f32 accumulation of integers below 2^16) and the epilogue rescales and sums
in the reference's f32 order, so the outputs must be identical, including
at extreme activation scales."""
from __future__ import annotations

import numpy as np
import pytest

from oracle.oracle import DT_Q4_K

pytestmark = pytest.mark.gpu


def _run(gpu, oracle, m, n, k, seed, a_scale=1.0, a=None):
    import torch
    dev = torch.device("cuda", 0)
    w = oracle.q4_k_quantize(oracle.gauss(n * k, 700 + seed, 0.02))
    if a is None:
        a = oracle.gauss(m * k, 800 + seed, a_scale)
    dw = torch.from_numpy(w).to(dev)
    da = torch.from_numpy(a).to(dev)
    wprep = torch.empty(gpu.prefill_weight_bytes(n, k), dtype=torch.uint8, device=dev)
    gpu.prefill_prepare_weights_dev(dw, n, k, wprep)
    scratch = torch.empty(gpu.prefill_scratch_bytes(m, k), dtype=torch.uint8, device=dev)
    dc = torch.full((m, n), float("nan"), dtype=torch.float32, device=dev)
    gpu.prefill_dev(da, wprep, dc, m, n, k, scratch)
    torch.cuda.synchronize()
    assert gpu.take_device_errors() == 0
    ref = oracle.matmul_q(a, w, DT_Q4_K, m, n, k, threads=0)[1]
    return dc.cpu().numpy(), ref, wprep, w


@pytest.mark.parametrize("m,n,k", [(128, 256, 256), (128, 512, 4096), (200, 300, 512), (384, 1000, 1024),
                                   (512, 11008, 4096), (64, 256, 11008), (1, 130, 512), (257, 4, 768),
                                   # odd n: a column pair straddles the last column, rows of odd length
                                   (200, 301, 512), (5, 7, 256)])
def test_prefill_bit_exact_with_int8_reference(gpu, oracle, m, n, k):
    got, ref, *_ = _run(gpu, oracle, m, n, k, seed=m + n)
    np.testing.assert_array_equal(got.view(np.uint32), ref.reshape(m, n).view(np.uint32))


@pytest.mark.parametrize("m", [128, 512, 2048])
def test_prefill_bit_exact_at_benchmark_shapes(gpu, oracle, m):
    """The timed prefill configurations, with the benchmark's own inputs:
    W 11008 x 4096 ~N(0, 0.02) from stream seed 2 (Q4_K on the device), A
    M x 4096 ~N(0, 1) from stream 1000 + M."""
    import torch
    n, k = 11008, 4096
    dev = torch.device("cuda", 0)
    dw = torch.empty(n * (k // 256) * 144, dtype=torch.uint8, device=dev)
    gpu.q4_k_from_gauss_dev(dw, n * k, 2, 0.02)
    da = torch.empty(m * k, dtype=torch.float32, device=dev)
    gpu.fill_gauss_dev(da, m * k, 1000 + m, 0, 1.0)
    wprep = torch.empty(gpu.prefill_weight_bytes(n, k), dtype=torch.uint8, device=dev)
    gpu.prefill_prepare_weights_dev(dw, n, k, wprep)
    scratch = torch.empty(gpu.prefill_scratch_bytes(m, k), dtype=torch.uint8, device=dev)
    dc = torch.full((m, n), float("nan"), dtype=torch.float32, device=dev)
    gpu.prefill_dev(da, wprep, dc, m, n, k, scratch)
    torch.cuda.synchronize()
    assert gpu.take_device_errors() == 0
    ref = oracle.matmul_q(da.cpu().numpy(), dw.cpu().numpy(), DT_Q4_K, m, n, k, threads=0)[1]
    np.testing.assert_array_equal(dc.cpu().numpy().view(np.uint32), ref.reshape(m, n).view(np.uint32))


def test_prefill_extreme_activation_scales(gpu, oracle):
    for s in (1e-30, 1e-3, 1e3, 1e30):
        got, ref, *_ = _run(gpu, oracle, 128, 256, 512, seed=3, a_scale=s)
        np.testing.assert_array_equal(got.view(np.uint32), ref.reshape(128, 256).view(np.uint32), err_msg=str(s))


def test_prefill_zero_and_ragged_rows(gpu, oracle):
    """All-zero groups (scale 0), a row of one repeated value, and a row
    count that leaves most of the last 128-row tile empty."""
    m, n, k = 131, 192, 512
    a = oracle.gauss(m * k, 41, 1.0).reshape(m, k)
    a[3] = 0.0
    a[7, :64] = 0.0
    a[9] = 0.25
    got, ref, *_ = _run(gpu, oracle, m, n, k, seed=41, a=np.ascontiguousarray(a.reshape(-1)))
    np.testing.assert_array_equal(got.view(np.uint32), ref.reshape(m, n).view(np.uint32))


def test_prefill_weight_layout(gpu, oracle):
    """The prepared weights hold the 4-bit values as bf16 and, per 32, rows of
    d*sc and -(dmin*m) whose combination d*sc*q - dmin*m is the reference's
    dequantization (matmul_q4_k.c:79-98)."""
    n, k = 64, 512
    _, _, wprep, w = _run(gpu, oracle, 128, n, k, seed=5)
    buf = wprep.cpu().numpy()
    q = (buf[:2 * n * k].view(np.uint16).astype(np.uint32) << 16).view(np.float32).reshape(n, k)  # bf16 values
    off = (2 * n * k + 1023) // 1024 * 1024
    npad = (n + 3) // 4 * 4
    sc = buf[off:off + (k // 32) * 2 * npad * 4].view(np.float32).reshape(k // 32, 2, npad)[:, :, :n]
    dsc = np.repeat(sc[:, 0, :].T, 32, axis=1)
    dmn = -np.repeat(sc[:, 1, :].T, 32, axis=1)
    assert q.min() >= 0 and q.max() <= 15 and np.all(q == np.round(q))
    deq = oracle.q4_k_dequantize(w, n * k).reshape(n, k)
    np.testing.assert_array_equal((dsc * q - dmn).astype(np.float32), deq)


def test_prefill_argument_errors(gpu):
    from eosllm_b200 import backend as B
    import torch
    t = torch.empty(1024, dtype=torch.float32, device="cuda")
    with pytest.raises(B.CudaBackendError) as ei:
        gpu.prefill_dev(t, t, t, 4, 4, 300, t)  # k % 256
    assert ei.value.status == B.EOS_E_INVALID_ARG
    with pytest.raises(B.CudaBackendError) as ei:
        gpu.prefill_dev(t, t, t, 4, 4, 256, 0)  # no scratch
    assert ei.value.status == B.EOS_E_INVALID_ARG
