"""Tensor-core prefill GEMM (eosllm_b200/csrc/prefill_gemm.cu) against the
oracle's int8 matmul, which is the reference's own arithmetic
(eosi_avx2_matmul_q4_k_int8).  Tolerance (per output):
    |gpu - ref| <= PREFILL_TOL * (|ref| + rms(ref))
The split-bf16 products carry ~2^-16 relative error each, so the observed
error is ~1e-5; PREFILL_TOL is the bound the decode path's Q8_0 tests use."""
from __future__ import annotations

import numpy as np
import pytest

from oracle.oracle import DT_Q4_K

pytestmark = pytest.mark.gpu

PREFILL_TOL = 1e-3


def _run(gpu, oracle, m, n, k, seed, a_scale=1.0):
    import torch
    dev = torch.device("cuda", 0)
    w = oracle.q4_k_quantize(oracle.gauss(n * k, 700 + seed, 0.02))
    a = oracle.gauss(m * k, 800 + seed, a_scale)
    dw = torch.from_numpy(w).to(dev)
    da = torch.from_numpy(a).to(dev)
    whi = torch.empty(n * k, dtype=torch.bfloat16, device=dev)
    wlo = torch.empty_like(whi)
    gpu.prefill_split_weights_dev(dw, n, k, whi, wlo)
    scratch = torch.empty(gpu.prefill_scratch_bytes(m, k), dtype=torch.uint8, device=dev)
    dc = torch.full((m, n), float("nan"), dtype=torch.float32, device=dev)
    gpu.prefill_dev(da, whi, wlo, dc, m, n, k, scratch)
    torch.cuda.synchronize()
    assert gpu.take_device_errors() == 0
    ref = oracle.matmul_q(a, w, DT_Q4_K, m, n, k, threads=0)[1]
    return dc.cpu().numpy(), ref, whi, wlo, w


def _check(got, ref):
    assert np.isfinite(got).all()
    rms = float(np.sqrt(np.mean(ref.astype(np.float64) ** 2)))
    err = np.abs(got.astype(np.float64) - ref) / (np.abs(ref) + rms)
    return float(err.max())


@pytest.mark.parametrize("m,n,k", [(128, 256, 256), (128, 512, 4096), (200, 300, 512), (384, 1000, 1024),
                                   (512, 11008, 4096), (64, 256, 11008)])
def test_prefill_matches_int8_reference(gpu, oracle, m, n, k):
    got, ref, *_ = _run(gpu, oracle, m, n, k, seed=m + n)
    e = _check(got, ref)
    print(f"prefill {m}x{n}x{k}: max err / (|ref| + rms) = {e:.2e}")
    assert e <= PREFILL_TOL


def test_prefill_extreme_activation_scales(gpu, oracle):
    for s in (1e-20, 1e-3, 1e3, 1e20):
        got, ref, *_ = _run(gpu, oracle, 128, 256, 512, seed=3, a_scale=s)
        assert _check(got, ref) <= PREFILL_TOL, s


def test_prefill_weight_split_is_exact_to_2e16(gpu, oracle):
    n, k = 64, 512
    _, _, whi, wlo, w = _run(gpu, oracle, 128, n, k, seed=5)
    deq = oracle.q4_k_dequantize(w, n * k)  # the reference's (d*sc)*q - dmin*m
    recon = whi.float().cpu().numpy() + wlo.float().cpu().numpy()
    assert np.all(np.abs(recon - deq) <= np.abs(deq) * 2.0 ** -16)


def test_prefill_argument_errors(gpu):
    from eosllm_b200 import backend as B
    import torch
    t = torch.empty(1024, dtype=torch.float32, device="cuda")
    with pytest.raises(B.CudaBackendError) as ei:
        gpu.prefill_dev(t, t, t, t, 4, 4, 300, t)  # k % 256
    assert ei.value.status == B.EOS_E_INVALID_ARG
