"""GPU parity: the sm_100a kernels, called through the C ABI, against the
oracle and the fixtures the reference itself produced.

Bars (stated per test):
  * Q4_K: BIT-EXACT with eosi_avx2_matmul_q4_k_int8 (and, for n < 4, with
    eosi_avx2_matmul_q4_k), the reference's production x86 dispatch;
  * activation packing, scale/min unpack, quantizers, generator: bit-exact;
  * Q8_0: |c - ref| <= 1e-3 |ref| + 1e-3 rms(ref) per output (different fp32
    summation order than the reference's sequential loop).
"""
import numpy as np
import pytest
import torch

from conftest import golden, same_bits
from oracle.oracle import DT_Q4_K, DT_Q8_0

pytestmark = pytest.mark.gpu

MODEL_SHAPES = [(4096, 4096), (11008, 4096), (4096, 11008), (32000, 4096)]


def dev(x: np.ndarray) -> torch.Tensor:
    return torch.from_numpy(np.ascontiguousarray(x)).cuda()


def host(t: torch.Tensor) -> np.ndarray:
    torch.cuda.synchronize()
    return t.cpu().numpy()


def q80_close(c, ref):
    c = np.asarray(c, np.float64)
    ref = np.asarray(ref, np.float64)
    floor = 1e-3 * np.sqrt(np.mean(ref ** 2)) if ref.size else 0.0
    return np.all(np.abs(c - ref) <= 1e-3 * np.abs(ref) + floor + 1e-30)


# ---------------------------------------------------------------------------
# activation packing (quantize_sub32, matmul_q4_k_int8.c:98-154)
# ---------------------------------------------------------------------------
def _pack_dev(B, a: np.ndarray, m: int, k: int):
    da = dev(a.astype(np.float32))
    aq = torch.empty(m * k, dtype=torch.int8, device="cuda")
    sc = torch.empty(m * k // 32, dtype=torch.float32, device="cuda")
    sm = torch.empty(m * k // 32, dtype=torch.int32, device="cuda")
    B.quantize_act_dev(da, m, k, aq, sc, sm)
    return host(aq), host(sc), host(sm)


def test_act_pack_golden_bitexact(gpu):
    g = golden("act_pack.npz")
    a = g["a"]
    aq, sc, sm = _pack_dev(gpu, a, 1, a.size)
    assert np.array_equal(aq, g["aq"])
    assert same_bits(sc, g["scales"])
    assert np.array_equal(sm, g["sums"])


def test_act_pack_random_bitexact(gpu, oracle):
    rng = np.random.default_rng(11)
    groups = 1 << 16
    scale = (10.0 ** rng.uniform(-42, 38, groups)).astype(np.float64)
    a = (rng.standard_normal((groups, 32)) * scale[:, None]).astype(np.float32)
    a[rng.integers(0, groups, 500), rng.integers(0, 32, 500)] = np.nan
    a[rng.integers(0, groups, 500), rng.integers(0, 32, 500)] = np.inf
    a[rng.integers(0, groups, 500), rng.integers(0, 32, 500)] = -np.inf
    a[rng.integers(0, groups, 300)] = 0.0
    a = a.ravel()
    aq, sc, sm = _pack_dev(gpu, a, 4, a.size // 4)
    oq, osc, osm = oracle.quantize_act(a)
    assert np.array_equal(aq, oq)
    assert same_bits(sc, osc)
    assert np.array_equal(sm, osm)


# ---------------------------------------------------------------------------
# scale/min unpack: exhaustive over every byte triple each sub-block reads
# ---------------------------------------------------------------------------
def test_scale_min_unpack_exhaustive(gpu, oracle):
    # sub-blocks j and j+4 read bytes (j, j+4, j+8) only; field i sets all
    # four triples to the 24-bit counter i, so 2^24 fields cover every case.
    i = np.arange(1 << 24, dtype=np.uint32)
    x, y, z = (i & 0xFF).astype(np.uint8), ((i >> 8) & 0xFF).astype(np.uint8), (i >> 16).astype(np.uint8)
    s12 = np.empty((1 << 24, 12), np.uint8)
    s12[:, 0:4] = x[:, None]
    s12[:, 4:8] = y[:, None]
    s12[:, 8:12] = z[:, None]
    d12 = dev(s12)
    dsc = torch.empty((1 << 24, 8), dtype=torch.uint8, device="cuda")
    dm = torch.empty((1 << 24, 8), dtype=torch.uint8, device="cuda")
    gpu.unpack_scale_min_dev(d12, 1 << 24, dsc, dm)
    osc, om = oracle.unpack_scale_min_batch(s12)
    assert np.array_equal(host(dsc), osc)
    assert np.array_equal(host(dm), om)


# ---------------------------------------------------------------------------
# Q4_K through the backend slot (host buffers)
# ---------------------------------------------------------------------------
def test_q4k_known_answer_and_int8_fixture(gpu):
    g = golden("q4k_known_answers.npz")
    blk = g["block"]
    # n = 1 -> the reference's f32-dequant path; 60*sum(sc) - 2*sum(m) = 5988
    c = gpu.matmul_q(np.ones(256, np.float32), blk, DT_Q4_K, 1, 1, 256)
    assert abs(c[0, 0] - 5988.0) <= 0.5
    c = gpu.matmul_q(g["a_xs"], blk, DT_Q4_K, 1, 1, 256)
    assert same_bits(c, g["xs_avx2_f32"])
    # N = 4 copies, xorshift32 seed 0x42424242 (test_runner.c:1075-1150)
    w4 = np.tile(blk, 4)
    c = gpu.matmul_q(g["a_xs"], w4, DT_Q4_K, 1, 4, 256)
    assert same_bits(c, g["xs_int8"])
    tol = max(5e-3 * abs(float(g["xs_scalar"][0, 0])), 1e-3)
    assert np.all(np.abs(c - g["xs_scalar"]) <= tol)
    # all-zero activation -> exactly 0.0f
    c = gpu.matmul_q(np.zeros(256, np.float32), w4, DT_Q4_K, 1, 4, 256)
    assert np.all(c == 0.0)


def int8_vs_f32_bound(oracle, a, w, m, n, k):
    """Worst-case gap between the int8-activation path and the f32 path:
    each packed activation is within scale/2 of the f32 value, so
    |c_int8 - c_f32| <= sum_k |w_jk| * scale_k / 2 (+ fp32 rounding)."""
    deq = oracle.q4_k_dequantize(w, n * k).reshape(n, k).astype(np.float64)
    bound = np.empty((m, n))
    for i in range(m):
        _, sc, _ = oracle.quantize_act(a[i * k:(i + 1) * k])
        half = np.repeat(sc.astype(np.float64), 32) / 2.0
        bound[i] = np.abs(deq) @ half + 1e-5 * (np.abs(deq) @ np.abs(a[i * k:(i + 1) * k].astype(np.float64)))
    return bound


def test_q4k_golden_cases_bitexact(gpu, oracle):
    g = golden("q4k_matmul.npz")
    idx = 0
    while f"c{idx}_shape" in g:
        m, n, k = (int(v) for v in g[f"c{idx}_shape"])
        a, w = g[f"c{idx}_a"], g[f"c{idx}_w"]
        c = gpu.matmul_q(a, w, DT_Q4_K, m, n, k)
        assert same_bits(c, g[f"c{idx}_matmul_q"]), (m, n, k)
        # and within the activation-rounding bound of the scalar f32 oracle
        assert np.all(np.abs(c - g[f"c{idx}_scalar"]) <= int8_vs_f32_bound(oracle, a, w, m, n, k)), (m, n, k)
        idx += 1
    assert idx == 10


@pytest.mark.parametrize("n,k", MODEL_SHAPES)
def test_q4k_model_shapes_bitexact(gpu, oracle, n, k):
    w = np.empty(n * (k // 256) * 144, np.uint8)
    dw = torch.empty(w.size, dtype=torch.uint8, device="cuda")
    gpu.q4_k_from_gauss_dev(dw, n * k, 0, 0.02)
    w[:] = host(dw)
    a = oracle.gauss(k, 1, 1.0)
    ref = oracle.matmul_q(a, w, DT_Q4_K, 1, n, k, threads=0)[1]
    c = gpu.matmul_q(a, w, DT_Q4_K, 1, n, k)
    assert same_bits(c, ref)
    # device-pointer entry point, same bits
    da, dc = dev(a), torch.empty(n, dtype=torch.float32, device="cuda")
    scratch = torch.empty(gpu.q4_k_scratch_bytes(1, k), dtype=torch.uint8, device="cuda")
    gpu.matmul_q4_k_dev(da, dw, dc, 1, n, k, scratch)
    assert same_bits(host(dc), ref[0])
    # fused packing (no scratch) and the two-kernel pack + gemv path agree too
    dc.zero_()
    gpu.matmul_q4_k_dev(da, dw, dc, 1, n, k, 0)
    assert same_bits(host(dc), ref[0])
    dc.zero_()
    gpu.q4_k_pack_act_dev(da, 1, k, scratch)
    gpu.q4_k_gemv_dev(scratch, dw, dc, n, k)
    assert same_bits(host(dc), ref[0])


# variant = config + 32 * rows_per_stage + 512 * ctas_per_sm + 4096 * chunk;
# configs 0-11 are the row-major kernel, 12-19 the column-major one (rows
# reuse activations), whose rows are staged whole (chunk 1) or in chunks of
# 8 (c - 1) super-blocks (chunk c >= 2; the last chunk of a row may be short)
@pytest.mark.parametrize("variant", [0, 1, 2, 3, 4, 5, 6, 7, 32, 64, 128, 256, 5 + 32 * 4, 2 * 512 + 2 + 32 * 2,
                                     12, 13, 14, 15, 16, 17, 18, 19, 2 * 512 + 15,
                                     16 + 4096 * 1, 16 + 4096 * 2, 16 + 4096 * 3, 19 + 4096 * 2, 18 + 4096 * 2,
                                     12 + 4096 * 5, 14 + 4096 * 3, 13 + 4096 * 2 + 512 * 1])
def test_q4k_kernel_variants_bitexact(gpu, oracle, variant):
    try:
        gpu.set_kernel_variant(DT_Q4_K, variant)
        for n, k in ((4096, 4096), (1000, 11008), (300, 256)):
            w = oracle.q4_k_quantize(oracle.gauss(n * k, 50 + variant, 0.02))
            a = oracle.gauss(k, 60 + variant, 1.0)
            ref = oracle.matmul_q(a, w, DT_Q4_K, 1, n, k, threads=0)[1]
            assert same_bits(gpu.matmul_q(a, w, DT_Q4_K, 1, n, k), ref), (variant, n, k)
    finally:
        gpu.set_kernel_variant(DT_Q4_K, -1)


def test_q4k_empty_k_gives_zeros(gpu, oracle):
    """k = 0: no super-blocks, so every output is the reference's c = 0
    (matmul_q4_k_int8.c:194) -- through the host slot and the device path."""
    import torch
    w = np.zeros(16, np.uint8)
    a = np.zeros(4, np.float32)
    ref = oracle.matmul_q(a, w, DT_Q4_K, 2, 40, 0)[1]
    assert np.array_equal(ref, np.zeros((2, 40), np.float32))
    got = gpu.matmul_q(a, w, DT_Q4_K, 2, 40, 0)
    assert same_bits(got, ref)
    dw = torch.zeros(16, dtype=torch.uint8, device="cuda")
    da = torch.zeros(4, dtype=torch.float32, device="cuda")
    dc = torch.full((40,), float("nan"), dtype=torch.float32, device="cuda")
    scratch = torch.zeros(64, dtype=torch.uint8, device="cuda")
    gpu.matmul_q4_k_dev(da, dw, dc, 1, 40, 0, scratch)
    torch.cuda.synchronize()
    assert same_bits(dc.cpu().numpy(), ref[0])


@pytest.mark.parametrize("m,n,k", [(2, 64, 4096), (3, 257, 1024), (5, 4, 512), (2, 3, 768), (4, 1, 256)])
def test_q4k_batched_rows_bitexact(gpu, oracle, m, n, k):
    w = oracle.q4_k_quantize(oracle.gauss(n * k, m + n, 0.02))
    a = oracle.gauss(m * k, m * 7 + k, 1.0)
    ref = oracle.matmul_q(a, w, DT_Q4_K, m, n, k)[1]
    assert same_bits(gpu.matmul_q(a, w, DT_Q4_K, m, n, k), ref)


def test_q4k_long_rows_fallback_bitexact(gpu, oracle):
    # rows too long for the staged ring take the unstaged kernel
    n, k = 6, 256 * 400
    w = oracle.q4_k_quantize(oracle.gauss(n * k, 70, 0.02))
    a = oracle.gauss(k, 71, 1.0)
    assert same_bits(gpu.matmul_q(a, w, DT_Q4_K, 1, n, k), oracle.matmul_q(a, w, DT_Q4_K, 1, n, k)[1])


def test_q4k_extreme_activations_bitexact(gpu, oracle):
    n, k = 64, 2048
    w = oracle.q4_k_quantize(oracle.gauss(n * k, 80, 0.02))
    rng = np.random.default_rng(3)
    a = (rng.standard_normal(k) * 10.0 ** rng.uniform(-40, 30, k)).astype(np.float32)
    a[:32] = 0.0
    a[32:64] *= 1e-30
    ref = oracle.matmul_q(a, w, DT_Q4_K, 1, n, k)[1]
    assert same_bits(gpu.matmul_q(a, w, DT_Q4_K, 1, n, k), ref)


# ---------------------------------------------------------------------------
# Q8_0
# ---------------------------------------------------------------------------
def test_q8_0_golden_cases(gpu):
    g = golden("q8_0_matmul.npz")
    idx = 0
    while f"c{idx}_shape" in g:
        m, n, k = (int(v) for v in g[f"c{idx}_shape"])
        c = gpu.matmul_q(g[f"c{idx}_a"], g[f"c{idx}_w"], DT_Q8_0, m, n, k)
        assert q80_close(c, g[f"c{idx}_matmul_q"]), (m, n, k)
        idx += 1
    assert idx == 8


@pytest.mark.parametrize("n,k", MODEL_SHAPES + [(100, 96), (37, 288), (9, 4128)])
def test_q8_0_shapes(gpu, oracle, n, k):
    w = oracle.gauss(n * k, n ^ k, 0.02)
    dsrc = dev(w)
    dq = torch.empty(n * (k // 32) * 34, dtype=torch.uint8, device="cuda")
    gpu.q8_0_quantize_dev(dsrc, dq, n * k)
    q8 = host(dq)
    assert np.array_equal(q8, oracle.q8_0_quantize(w))  # device quantizer == reference quantizer
    a = oracle.gauss(2 * k, k + 5, 1.0)
    ref = oracle.matmul_q(a, q8, DT_Q8_0, 2, n, k, threads=0)[1]
    assert q80_close(gpu.matmul_q(a, q8, DT_Q8_0, 2, n, k), ref)
    assert q80_close(gpu.matmul_q(a[:k], q8, DT_Q8_0, 1, n, k), ref[:1])


@pytest.mark.parametrize("variant", [0, 1, 2, 3, 4, 5])
def test_q8_0_kernel_variants(gpu, oracle, variant):
    try:
        gpu.set_kernel_variant(DT_Q8_0, variant)
        n, k = 777, 4096
        q8 = oracle.q8_0_quantize(oracle.gauss(n * k, 90, 0.02))
        a = oracle.gauss(k, 91, 1.0)
        ref = oracle.matmul_q(a, q8, DT_Q8_0, 1, n, k)[1]
        assert q80_close(gpu.matmul_q(a, q8, DT_Q8_0, 1, n, k), ref)
    finally:
        gpu.set_kernel_variant(DT_Q8_0, -1)


# ---------------------------------------------------------------------------
# formats and generator on the device: bit-exact with the host restatement
# ---------------------------------------------------------------------------
def test_device_generator_and_q4k_quantizer_bitexact(gpu, oracle):
    n = 1 << 20
    d = torch.empty(n, dtype=torch.float32, device="cuda")
    gpu.fill_gauss_dev(d, n, 123, 17, 0.5)
    x = oracle.gauss(n, 123, 0.5, offset=17)
    assert same_bits(host(d), x)
    dq = torch.empty(n // 256 * 144, dtype=torch.uint8, device="cuda")
    gpu.q4_k_quantize_dev(d, dq, n)
    assert np.array_equal(host(dq), oracle.q4_k_quantize(x))
    gpu.q4_k_from_gauss_dev(dq, n, 7, 0.02)
    assert np.array_equal(host(dq), oracle.q4_k_quantize(oracle.gauss(n, 7, 0.02)))


# ---------------------------------------------------------------------------
# backend behaviour: errors, cache, sharding
# ---------------------------------------------------------------------------
def test_error_codes_on_gpu(gpu):
    a = np.ones(512, np.float32)
    w = np.zeros(144 * 2 * 8, np.uint8)
    c = np.full(8, 7.0, np.float32)
    assert gpu.matmul_q_status(a, w, DT_Q4_K, c, 1, 8, 300) == gpu.EOS_E_INVALID_ARG
    assert gpu.matmul_q_status(a, w, 0, c, 1, 8, 512) == gpu.EOS_E_UNSUPPORTED
    assert gpu.matmul_q_status(None, w, DT_Q4_K, c, 1, 8, 512) == gpu.EOS_E_INVALID_ARG
    assert np.all(c == 7.0)
    # device-pointer layer rejects misaligned pointers instead of faulting
    dw = torch.zeros(144 * 64 + 16, dtype=torch.uint8, device="cuda")
    act = torch.zeros(gpu.q4_k_scratch_bytes(1, 256), dtype=torch.uint8, device="cuda")
    dc = torch.zeros(64, dtype=torch.float32, device="cuda")
    with pytest.raises(gpu.CudaBackendError):
        gpu.q4_k_gemv_dev(act, dw.data_ptr() + 2, dc, 64, 256)


def test_weight_cache_tracks_reused_buffers(gpu, oracle):
    n, k = 64, 1024
    w = oracle.q4_k_quantize(oracle.gauss(n * k, 1, 0.02))
    a = oracle.gauss(k, 2, 1.0)
    c1 = gpu.matmul_q(a, w, DT_Q4_K, 1, n, k)
    w[:] = oracle.q4_k_quantize(oracle.gauss(n * k, 3, 0.02))  # same address, new contents
    c2 = gpu.matmul_q(a, w, DT_Q4_K, 1, n, k)
    assert same_bits(c2, oracle.matmul_q(a, w, DT_Q4_K, 1, n, k)[1])
    assert not same_bits(c1, c2)


def test_host_calls_reuse_their_recorded_launches(gpu, oracle):
    """A host-pointer Q4_K call is a CUDA graph recorded once per weight and
    shape and then replayed: back-to-back calls with new activations, calls
    alternating between two weights of one shape (and m = 1 / m = 3), and a
    call after the weights were evicted (their graphs dropped) each give the
    oracle's bits."""
    n, k = 320, 2048
    w1 = oracle.q4_k_quantize(oracle.gauss(n * k, 31, 0.02))
    w2 = oracle.q4_k_quantize(oracle.gauss(n * k, 32, 0.02))
    for i in range(6):
        w = w1 if i % 2 == 0 else w2
        m = 1 if i < 4 else 3
        a = oracle.gauss(m * k, 40 + i, 1.0)
        c = gpu.matmul_q(a, w, DT_Q4_K, m, n, k)
        assert same_bits(c, oracle.matmul_q(a, w, DT_Q4_K, m, n, k)[1]), i
    assert gpu.load().eosi_cuda_cache_evict(w1.ctypes.data) == gpu.EOS_OK
    a = oracle.gauss(k, 50, 1.0)
    assert same_bits(gpu.matmul_q(a, w1, DT_Q4_K, 1, n, k), oracle.matmul_q(a, w1, DT_Q4_K, 1, n, k)[1])
    assert gpu.take_device_errors() == 0


def test_row_sharding_across_streams(gpu, oracle):
    # the multi-GPU path with every shard on device 0 (one stream each)
    n, k = 1001, 4096
    w = oracle.q4_k_quantize(oracle.gauss(n * k, 4, 0.02))
    q8 = oracle.q8_0_quantize(oracle.gauss(n * k, 4, 0.02))
    a = oracle.gauss(2 * k, 5, 1.0)
    ref4 = oracle.matmul_q(a, w, DT_Q4_K, 2, n, k)[1]
    ref8 = oracle.matmul_q(a, q8, DT_Q8_0, 2, n, k)[1]
    try:
        for ids in ([0, 0], [0, 0, 0], [0] * 8):
            gpu.set_devices(ids)
            assert same_bits(gpu.matmul_q(a, w, DT_Q4_K, 2, n, k), ref4), ids
            assert q80_close(gpu.matmul_q(a, q8, DT_Q8_0, 2, n, k), ref8), ids
            # fewer rows than shards
            assert same_bits(gpu.matmul_q(a[:k], w[:5 * 16 * 144], DT_Q4_K, 1, 5, k), ref4[:1, :5])
    finally:
        gpu.set_devices(None)


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="one GPU on this box")
def test_row_sharding_two_gpus(gpu, oracle):
    n, k = 11008, 4096
    w = oracle.q4_k_quantize(oracle.gauss(n * k, 6, 0.02))
    a = oracle.gauss(k, 7, 1.0)
    ref = oracle.matmul_q(a, w, DT_Q4_K, 1, n, k, threads=0)[1]
    before = torch.cuda.current_device()
    try:
        gpu.set_devices(list(range(torch.cuda.device_count())))
        assert same_bits(gpu.matmul_q(a, w, DT_Q4_K, 1, n, k), ref)
    finally:
        gpu.set_devices(None)
    # the caller's current device is left as it was (the *_dev entry points
    # run on it)
    assert torch.cuda.current_device() == before


def test_dev_entry_points_reject_foreign_pointers(gpu):
    """A *_dev call runs on the current device: host memory or another GPU's
    memory is rejected before any kernel is launched."""
    from eosllm_b200 import backend as B
    n, k = 256, 512
    w = torch.zeros(n * (k // 256) * 144, dtype=torch.uint8, device="cuda:0")
    act = torch.zeros(B.q4_k_scratch_bytes(1, k), dtype=torch.uint8, device="cuda:0")
    c = torch.zeros(n, dtype=torch.float32, device="cuda:0")
    host = np.zeros(n * (k // 256) * 144, np.uint8)
    with pytest.raises(B.CudaBackendError) as ei:
        gpu.q4_k_gemv_dev(act, host, c, n, k)
    assert ei.value.status == B.EOS_E_INVALID_ARG
    if torch.cuda.device_count() > 1:
        w1 = torch.zeros_like(w, device="cuda:1")
        with pytest.raises(B.CudaBackendError) as ei:
            gpu.q4_k_gemv_dev(act, w1, c, n, k)
        assert ei.value.status == B.EOS_E_INVALID_ARG
    gpu.q4_k_gemv_dev(act, w, c, n, k)  # same-device pointers still work
    torch.cuda.synchronize()


def test_no_device_errors_raised(gpu):
    assert gpu.take_device_errors() == 0
