"""The C-ABI boundary on the CPU: the library loads, exports every entry
point include/eosllm_cuda.h declares, and validates arguments with the
reference's status codes before it ever touches a GPU."""
import ctypes as C
import os
import subprocess

import numpy as np
import pytest

from eosllm_b200 import backend as B

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def test_exports_every_declared_symbol(cuda_lib):
    declared = B.declared_symbols()
    assert len(declared) >= 20
    out = subprocess.run(["nm", "-D", "--defined-only", B.LIB_PATH], capture_output=True, text=True, check=True)
    exported = {line.split()[-1] for line in out.stdout.splitlines() if " T " in line}
    missing = [s for s in declared if s not in exported]
    assert not missing, missing
    # nothing else leaks out of the library
    extra = [s for s in exported if not s.startswith("eosi_cuda_")]
    assert not extra, extra
    for s in declared:
        assert hasattr(cuda_lib, s)


def test_header_is_plain_c(tmp_path):
    src = tmp_path / "t.c"
    src.write_text('#include "eosllm_cuda.h"\nint main(void){return eosi_cuda_probe() < 0;}\n')
    subprocess.run(["gcc", "-std=c99", "-Wall", "-Werror", "-pedantic", "-I", os.path.join(ROOT, "include"),
                    "-c", str(src), "-o", str(tmp_path / "t.o")], check=True)


def test_backend_glue_compiles_against_engine_headers(tmp_path):
    """eosllm_b200/host/cuda_backend.c is C99 against the engine's own
    include/eosllm/backend.h (present where the reference tree is)."""
    from oracle.oracle import reference_dir
    ref_inc = os.path.join(reference_dir(), "include")
    if not os.path.isdir(ref_inc):
        pytest.skip(f"engine headers not present on this machine ({ref_inc})")
    src = os.path.join(ROOT, "eosllm_b200", "host", "cuda_backend.c")
    for flag in ("-DEOSLLM_HAVE_KERNEL_CUDA=1", "-DEOSLLM_HAVE_KERNEL_CUDA=0"):
        subprocess.run(["gcc", "-std=c99", "-Wall", "-Wextra", "-Werror", "-pedantic", flag, "-I", ref_inc,
                        "-I", os.path.join(ROOT, "include"), "-c", src, "-o", str(tmp_path / "glue.o")], check=True)
    out = subprocess.run(["nm", str(tmp_path / "glue.o")], capture_output=True, text=True, check=True).stdout
    assert "eosi_backend_cuda_register" in out


def test_argument_validation_matches_reference(cuda_lib):
    a = np.ones(512, np.float32)
    w = np.zeros(144 * 2, np.uint8)
    c = np.full(2, 7.0, np.float32)
    # NULL pointers -> EOS_E_INVALID_ARG (matmul_q4_k_int8.c:172)
    assert B.matmul_q_status(None, w, B.DT_Q4_K, c, 1, 1, 512) == B.EOS_E_INVALID_ARG
    assert B.matmul_q_status(a, None, B.DT_Q4_K, c, 1, 1, 512) == B.EOS_E_INVALID_ARG
    assert B.matmul_q_status(a, w, B.DT_Q4_K, None, 1, 1, 512) == B.EOS_E_INVALID_ARG
    # k % 256 != 0 -> EOS_E_INVALID_ARG (:173-174); k % 32 for Q8_0 (matmul_q8.c:33)
    assert B.matmul_q_status(a, w, B.DT_Q4_K, c, 1, 1, 300) == B.EOS_E_INVALID_ARG
    assert B.matmul_q_status(a, w, B.DT_Q8_0, c, 1, 1, 40) == B.EOS_E_INVALID_ARG
    # any other dtype -> EOS_E_UNSUPPORTED (matmul_q4_k.c:168-169)
    for dt in (0, 1, 34, 35, 99):
        assert B.matmul_q_status(a, w, dt, c, 1, 1, 512) == B.EOS_E_UNSUPPORTED
    assert "dtype" in B.last_error()
    # outputs untouched on failure (eosllm.h:60-65)
    assert np.all(c == 7.0)
    # empty shapes succeed without work, like the reference's loops
    assert B.matmul_q_status(a, w, B.DT_Q4_K, c, 0, 1, 512) == B.EOS_OK
    assert B.matmul_q_status(a, w, B.DT_Q4_K, c, 1, 0, 512) == B.EOS_OK


def test_probe_without_gpu_is_an_error_not_a_crash(cuda_lib):
    import torch
    if torch.cuda.is_available():
        pytest.skip("a GPU is present")
    assert cuda_lib.eosi_cuda_probe() == B.EOS_E_UNSUPPORTED
    assert cuda_lib.eosi_cuda_device_count() == 0
    assert B.last_error()
    # a real call fails loudly with the probe's status; nothing falls back to the CPU
    a = np.ones(256, np.float32)
    w = np.zeros(144 * 4, np.uint8)
    c = np.zeros(4, np.float32)
    assert B.matmul_q_status(a, w, B.DT_Q4_K, c, 1, 4, 256) == B.EOS_E_UNSUPPORTED
    with pytest.raises(B.CudaBackendError):
        B.matmul_q(a, w, B.DT_Q4_K, 1, 4, 256)


def test_scratch_size_formula(cuda_lib):
    for m, k in ((1, 256), (3, 4096), (2, 11008)):
        assert B.q4_k_scratch_bytes(m, k) == m * (k // 256) * 480


def test_missing_library_fails_loudly(tmp_path, cuda_lib):
    saved = B._lib
    try:
        B._lib = None
        with pytest.raises(FileNotFoundError):
            B.load(str(tmp_path / "nope.so"))
    finally:
        B._lib = saved


def test_llama_desc_layout_matches_header(tmp_path):
    """eosllm_b200.text.LlamaDesc (ctypes) has the C layout of
    eosi_cuda_llama_t: same size and field offsets as gcc computes."""
    from eosllm_b200.text import LlamaDesc
    names = [f[0] for f in LlamaDesc._fields_]
    src = tmp_path / "layout.c"
    body = "".join(f'    printf("%s %zu\\n", "{n}", offsetof(eosi_cuda_llama_t, {n}));\n'
                   for n in names if n != "output_w") + \
        '    printf("output_w %zu\\n", offsetof(eosi_cuda_llama_t, output_w));\n'
    src.write_text('#include <stddef.h>\n#include <stdio.h>\n#include "eosllm_cuda.h"\nint main(void) {\n'
                   '    printf("sizeof %zu\\n", sizeof(eosi_cuda_llama_t));\n' + body + "    return 0;\n}\n")
    exe = tmp_path / "layout"
    subprocess.run(["gcc", "-std=c99", "-Wall", "-Werror", "-I", os.path.join(ROOT, "include"), str(src), "-o",
                    str(exe)], check=True)
    got = dict(line.split() for line in subprocess.run([str(exe)], capture_output=True, text=True,
                                                       check=True).stdout.splitlines())
    assert int(got["sizeof"]) == C.sizeof(LlamaDesc)
    for n in names:
        assert int(got[n]) == getattr(LlamaDesc, n).offset, n


def test_text_decoder_rejects_bad_descriptions(cuda_lib):
    """NULL or empty descriptions fail with EOS_E_INVALID_ARG before any
    device work (works without a GPU)."""
    from eosllm_b200.text import LlamaDesc
    h = C.c_void_p()
    assert cuda_lib.eosi_cuda_text_open(None, 0, 0, 1, C.byref(h)) == B.EOS_E_INVALID_ARG
    d = LlamaDesc()
    assert cuda_lib.eosi_cuda_text_open(C.byref(d), 0, 0, 1, C.byref(h)) == B.EOS_E_INVALID_ARG
    assert not h.value
    assert cuda_lib.eosi_cuda_text_step(None, 0, None) == B.EOS_E_INVALID_ARG
    assert cuda_lib.eosi_cuda_text_generate(None, None, 0, 0, None) == B.EOS_E_INVALID_ARG
    cuda_lib.eosi_cuda_text_close(None)
