"""The drop-in, proven inside the reference engine itself.

The unmodified engine, compiled from its sources (oracle/_ref/libeosllm_ref.so),
registers its own CPU backends (eos_init_defaults); the C99 glue this project
ships for it (eosllm_b200/host/cuda_backend.c, compiled against the engine's
headers with EOSLLM_HAVE_KERNEL_CUDA=1 into oracle/_ref/libengine_cuda_glue.so)
then registers the "cuda" backend exactly as src/kernels/register_all.c:3-15
would.  eos_session_open builds the per-op dispatch (src/core/session.c:43-81),
and the test reads the op table the session chose: matmul_q must resolve to
the glue, everything else to the CPU backends.  With that table the engine's
own eosi_text_step (src/modality/text/text.c:267-436) runs a synthetic GGUF
model, and the session's own greedy loop (eos_session_feed / eos_session_step)
generates tokens.

Each configuration runs in two fresh processes -- the engine alone (x86_avx2
matmul_q) and the engine with "cuda" registered -- since the engine's
registry freezes at the first session.  Q4_K logits must be BIT-IDENTICAL
(the GPU kernel is bit-exact with the AVX2 int8 kernel) and the session's
tokens equal; Q8_0 logits agree within 2e-3 rms (the scalar Q8_0 kernel's
summation order differs).  The library's own counters confirm every matmul_q
ran on the GPU."""
from __future__ import annotations

import ctypes as C
import os

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
GLUE = os.path.join(ROOT, "oracle", "_ref", "libengine_cuda_glue.so")
TEXT = b"The quick brown fox jumps over the lazy dog; eosllm on a B200."
N_GEN = 8

CASES = {
    "mha_q4k": dict(n_vocab=320),
    "gqa_q4k": dict(n_vocab=320, n_kv_head=2, seed=5),
    "mha_q80": dict(n_vocab=320, wdtype=32, out_dtype=32, seed=6),
    # one layer of the 7B shape, full vocabulary
    "layer7b_q4k": dict(n_embd=4096, n_layer=1, n_head=32, n_kv_head=32, n_ff=11008, n_vocab=32000, seed=3),
}


class _Params(C.Structure):  # eos_session_params_t (include/eosllm/eosllm.h:227-245)
    _fields_ = [("max_context", C.c_uint32), ("arena_bytes", C.c_size_t), ("temperature", C.c_float),
                ("top_k", C.c_uint32), ("top_p", C.c_float), ("rng_seed", C.c_uint64), ("scheduler", C.c_char_p),
                ("_reserved", C.c_uint8 * 16)]


class _Ops(C.Structure):  # eos_backend_ops_t (include/eosllm/backend.h:32-65)
    _fields_ = [(n, C.c_void_p) for n in ("matmul_f32", "matmul_q", "rmsnorm", "softmax", "rope", "silu", "gelu")]


class _Session(C.Structure):  # leading fields of struct eos_session (src/core/session.c:19-24)
    _fields_ = [("model", C.c_void_p), ("params", _Params), ("deadline_abs_ns", C.c_uint64), ("ops", _Ops)]


class _DlInfo(C.Structure):
    _fields_ = [("dli_fname", C.c_char_p), ("dli_fbase", C.c_void_p), ("dli_sname", C.c_char_p),
                ("dli_saddr", C.c_void_p)]


def _library_of(addr: int) -> str:
    libc = C.CDLL(None)
    libc.dladdr.argtypes = [C.c_void_p, C.POINTER(_DlInfo)]
    info = _DlInfo()
    return os.path.basename(info.dli_fname.decode()) if libc.dladdr(addr, C.byref(info)) and info.dli_fname else ""


def _engine_child(gguf: str, use_cuda: bool, tokens, n_vocab: int, max_ctx: int, q) -> None:
    """One fresh process: the engine (plus the "cuda" backend when asked)."""
    try:
        from oracle.oracle import REF_ENGINE
        L = C.CDLL(REF_ENGINE, mode=C.RTLD_GLOBAL)
        assert L.eos_init_defaults() == 0
        out = {}
        if use_cuda:
            glue = C.CDLL(GLUE, mode=C.RTLD_GLOBAL)
            out["register"] = glue.eosi_backend_cuda_register()
            L.eos_backend_available.argtypes = [C.c_char_p]
            out["available"] = L.eos_backend_available(b"cuda")
        L.eos_model_open.argtypes = [C.c_char_p, C.POINTER(C.c_void_p)]
        L.eos_session_open.argtypes = [C.c_void_p, C.POINTER(_Params), C.POINTER(C.c_void_p)]
        L.eosi_text_open.argtypes = [C.c_void_p, C.c_void_p, C.c_uint32, C.POINTER(C.c_void_p)]
        L.eosi_text_step.argtypes = [C.c_void_p, C.c_uint32, C.c_void_p]
        L.eosi_text_close.argtypes = [C.c_void_p]
        L.eos_session_feed.argtypes = [C.c_void_p, C.c_int, C.c_void_p, C.c_size_t]
        L.eos_session_step.argtypes = [C.c_void_p, C.POINTER(C.c_uint32)]
        L.eos_session_close.argtypes = [C.c_void_p]
        L.eos_model_close.argtypes = [C.c_void_p]
        model, sess, text = C.c_void_p(), C.c_void_p(), C.c_void_p()
        assert L.eos_model_open(gguf.encode(), C.byref(model)) == 0
        params = _Params()
        params.max_context = max_ctx
        assert L.eos_session_open(model, C.byref(params), C.byref(sess)) == 0
        view = _Session.from_address(sess.value)
        assert view.model == model.value  # the mirrored layout is the engine's
        ops = view.ops
        out["matmul_q_lib"] = _library_of(ops.matmul_q)
        out["matmul_q_is_avx2"] = ops.matmul_q == C.cast(L.eosi_avx2_matmul_q, C.c_void_p).value
        out["other_ops_libs"] = sorted({_library_of(getattr(ops, n)) for n, _ in _Ops._fields_
                                        if n != "matmul_q" and getattr(ops, n)})
        # the engine's own decoder step with the op table the session chose
        assert L.eosi_text_open(model, C.addressof(ops), max_ctx, C.byref(text)) == 0
        logits = []
        for t in tokens:
            row = np.empty(n_vocab, np.float32)
            assert L.eosi_text_step(text, int(t), row.ctypes.data) == 0
            logits.append(row)
        L.eosi_text_close(text)
        # the session's own greedy generation (tokenizer, prefill, scheduler)
        assert L.eos_session_feed(sess, 0, TEXT, len(TEXT)) == 0
        tok = C.c_uint32()
        gen = []
        for _ in range(N_GEN):
            assert L.eos_session_step(sess, C.byref(tok)) == 0
            gen.append(int(tok.value))
        L.eos_session_close(sess)
        L.eos_model_close(model)
        if use_cuda:
            from eosllm_b200 import backend as B
            calls, entries, nbytes = C.c_uint64(), C.c_uint64(), C.c_uint64()
            assert B.load().eosi_cuda_host_stats(C.byref(calls), C.byref(entries), C.byref(nbytes)) == 0
            out["gpu_calls"], out["gpu_weights"] = int(calls.value), int(entries.value)
        q.put((out, np.stack(logits), gen))
    except Exception as e:  # report, never hang the parent
        q.put(repr(e))


def _run(gguf, use_cuda, tokens, n_vocab, max_ctx):
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    p = ctx.Process(target=_engine_child, args=(gguf, use_cuda, tokens, n_vocab, max_ctx, q))
    p.start()
    res = q.get(timeout=900)
    p.join(timeout=120)
    assert not isinstance(res, str), res
    return res


@pytest.mark.parametrize("name", sorted(CASES))
def test_reference_engine_with_cuda_backend(gpu, oracle, tmp_path, name):
    from oracle.gguf_writer import byte_fallback_tokens, write_llama
    from oracle.llama import make_llama
    from oracle.oracle import REF_ENGINE
    if not (os.path.exists(REF_ENGINE) and os.path.exists(GLUE)):
        pytest.skip("oracle/_ref not built (make -C oracle ref where the reference tree exists)")
    kw = dict(CASES[name])
    max_ctx = 128  # the text is one token per byte (byte fallback) plus the picks
    model = make_llama(oracle, max_ctx=max_ctx, **kw)
    cfg = model["config"]
    path = str(tmp_path / f"{name}.gguf")
    write_llama(path, model, byte_fallback_tokens(cfg["n_vocab"]))
    del model
    tokens = np.random.default_rng(7).integers(0, cfg["n_vocab"], 12)
    cpu, lg_cpu, gen_cpu = _run(path, False, tokens, cfg["n_vocab"], max_ctx)
    gpu_, lg_gpu, gen_gpu = _run(path, True, tokens, cfg["n_vocab"], max_ctx)
    # dispatch: matmul_q from the glue, every other op from the CPU engine
    assert cpu["matmul_q_is_avx2"], cpu
    assert gpu_["register"] == 0 and gpu_["available"] == 1, gpu_
    assert not gpu_["matmul_q_is_avx2"] and gpu_["matmul_q_lib"] == "libengine_cuda_glue.so", gpu_
    assert gpu_["other_ops_libs"] == cpu["other_ops_libs"] == ["libeosllm_ref.so"], (gpu_, cpu)
    # every linear of every step and of the session ran on the GPU: 7 per
    # layer and the LM head, for the 12 stepped tokens and the session's
    # prompt tokens and picks
    per_step = 7 * cfg["n_layer"] + 1
    assert gpu_["gpu_calls"] >= per_step * (len(tokens) + N_GEN), gpu_
    assert gpu_["gpu_weights"] >= per_step, gpu_
    if cfg["wdtype"] == 33 and cfg["out_dtype"] == 33:
        np.testing.assert_array_equal(lg_gpu.view(np.uint32), lg_cpu.view(np.uint32))
        assert gen_gpu == gen_cpu
    else:
        rms = np.sqrt(np.mean(lg_cpu.astype(np.float64) ** 2, axis=1))
        err = np.max(np.abs(lg_gpu - lg_cpu), axis=1) / rms
        assert err.max() <= 2e-3, err
        assert len(gen_gpu) == N_GEN


# The engine's microbenchmark, tools/eosllm-bench/main.c: bench_matmul_q
# (:128-219) finds a backend by name in the engine's registry (find_backend,
# :83-93), probes it and times ops.matmul_q over k_shapes (:40-50), and main()
# lists the backends by name (:274-277), so timing the GPU needs one more
# line there: bench_matmul_q("cuda", "q4_k", EOS_DT_Q4_K, 256).  This runs that
# loop through the same registry for "cuda" and "x86_avx2", with records in
# emit()'s format (:64-78), and checks the two backends' outputs bit for bit.
BENCH_SHAPES = [(1, 1, 256), (1, 8, 512), (1, 64, 1024), (1, 128, 2048), (1, 512, 2048), (1, 256, 4096)]
EOSI_MAX_BACKENDS = 16  # src/core/internal.h:21


class _BackendVt(C.Structure):  # eos_backend_vt_t (include/eosllm/backend.h:67-82)
    _fields_ = [("name", C.c_char_p), ("priority", C.c_int32), ("probe", C.c_void_p), ("ops", _Ops)]


class _RegistryHead(C.Structure):  # leading fields of eosi_registry_t (src/core/internal.h:28-30)
    _fields_ = [("backends", C.POINTER(_BackendVt) * EOSI_MAX_BACKENDS), ("n_backends", C.c_size_t)]


def _n_iters(m, n, k):  # n_iters_for (main.c:53-61), capped lower to bound the test's time
    return int(min(max(5e8 / (2.0 * m * n * k), 1), 2000))


def _bench_child(shapes, weights, acts, q):
    try:
        import time
        from oracle.oracle import REF_ENGINE
        L = C.CDLL(REF_ENGINE, mode=C.RTLD_GLOBAL)
        assert L.eos_init_defaults() == 0
        glue = C.CDLL(GLUE, mode=C.RTLD_GLOBAL)
        assert glue.eosi_backend_cuda_register() == 0
        L.eosi_registry.restype = C.POINTER(_RegistryHead)
        reg = L.eosi_registry().contents
        vts = {}
        for i in range(reg.n_backends):
            vt = reg.backends[i]
            if vt:
                vts[vt.contents.name.decode()] = vt.contents
        probe_t = C.CFUNCTYPE(C.c_int)
        mm_t = C.CFUNCTYPE(C.c_int, C.c_void_p, C.c_void_p, C.c_int, C.c_void_p, C.c_uint32, C.c_uint32, C.c_uint32)
        out = {"names": sorted(vts), "records": [], "outputs": {}}
        for name in ("cuda", "x86_avx2"):
            vt = vts[name]
            if vt.probe:
                assert probe_t(vt.probe)() == 0, name
            mm = mm_t(vt.ops.matmul_q)
            outs = []
            for (m, n, k), w, a in zip(shapes, weights, acts):
                c = np.empty(m * n, np.float32)
                assert mm(a.ctypes.data, w.ctypes.data, 33, c.ctypes.data, m, n, k) == 0, (name, m, n, k)
                it = _n_iters(m, n, k)
                t0 = time.perf_counter_ns()
                for _ in range(it):
                    mm(a.ctypes.data, w.ctypes.data, 33, c.ctypes.data, m, n, k)
                t1 = time.perf_counter_ns()
                ops = 2.0 * m * n * k
                out["records"].append({"backend": name, "op": "matmul_q4_k", "m": m, "n": n, "k": k, "n_iters": it,
                                       "total_ns": t1 - t0, "ns_per_iter": round((t1 - t0) / it, 1),
                                       "giga_ops_per_s": round(ops * it / (t1 - t0), 2)})
                outs.append(c)
            out["outputs"][name] = outs
        q.put(out)
    except Exception as e:  # report, never hang the parent
        q.put(repr(e))


def test_engine_bench_matmul_q_through_the_registry(gpu, oracle, capsys):
    from oracle.oracle import REF_ENGINE
    if not (os.path.exists(REF_ENGINE) and os.path.exists(GLUE)):
        pytest.skip("oracle/_ref not built (make -C oracle ref where the reference tree exists)")
    import json

    import torch.multiprocessing as mp
    weights, acts = [], []
    for i, (m, n, k) in enumerate(BENCH_SHAPES):
        weights.append(oracle.q4_k_quantize(oracle.gauss(n * k, 60 + i, 0.1)))
        acts.append(oracle.gauss(m * k, 70 + i, 1.0))
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    p = ctx.Process(target=_bench_child, args=(BENCH_SHAPES, weights, acts, q))
    p.start()
    res = q.get(timeout=900)
    p.join(timeout=120)
    assert not isinstance(res, str), res
    assert "cuda" in res["names"] and "x86_avx2" in res["names"], res["names"]
    for (m, n, k), g, r in zip(BENCH_SHAPES, res["outputs"]["cuda"], res["outputs"]["x86_avx2"]):
        np.testing.assert_array_equal(g.view(np.uint32), r.view(np.uint32), err_msg=f"{m}x{n}x{k}")
    with capsys.disabled():
        for rec in res["records"]:
            print(json.dumps(rec))
