"""Failure detection of the tensor-parallel decoder, on ONE GPU without a
fault: two ranks of a world-2 decoder are opened in this process and attached
to each other (eosi_cuda_text_attach_local), and only rank 0 is stepped.  Its
first exchange waits for a flag that nothing sets; the wait is bounded (here
50 ms, eosi_cuda_text_set_wait_limit), so the step must come back with
EOS_E_INTERNAL and a message naming the missing peer, within about the limit,
and both ranks must close cleanly.  Rank 1 never launches anything, so no two
kernels wait on each other on the GPU."""
from __future__ import annotations

import time

import pytest

pytestmark = pytest.mark.gpu


def test_missing_rank_turns_into_an_error_within_the_wait_limit(gpu, oracle):
    from oracle.llama import make_llama
    from eosllm_b200.text import TextDecoder
    model = make_llama(oracle, n_embd=256, n_layer=2, n_head=4, n_kv_head=4, n_ff=512, n_vocab=320, max_ctx=16)
    r0 = TextDecoder(model, device=0, rank=0, world=2)
    r1 = TextDecoder(model, device=0, rank=1, world=2)
    try:
        TextDecoder.attach_local([r0, r1])
        r0.set_wait_limit(50_000)
        t0 = time.perf_counter()
        status = r0.step_status(5)
        dt = time.perf_counter() - t0
        assert status == gpu.EOS_E_INTERNAL, status
        assert "peer did not arrive" in gpu.last_error(), gpu.last_error()
        # one limit for the first handshake; the later ones of the step give up
        # at once (the peer bit is already set)
        assert 0.05 <= dt < 1.0, dt
        # the error stays until a reset: the next step fails at once as well
        t0 = time.perf_counter()
        assert r0.step_status(6) == gpu.EOS_E_INTERNAL
        assert time.perf_counter() - t0 < 0.5
    finally:
        r0.close()
        r1.close()


def test_wait_limit_argument_checks(gpu, oracle):
    from oracle.llama import make_llama
    from eosllm_b200 import backend as B
    from eosllm_b200.text import TextDecoder
    model = make_llama(oracle, n_embd=256, n_layer=1, n_head=4, n_kv_head=4, n_ff=512, n_vocab=320, max_ctx=16)
    d = TextDecoder(model, device=0)
    try:
        with pytest.raises(B.CudaBackendError):
            d.set_wait_limit(0)
        d.set_wait_limit(2_000_000)
        d.step(3)  # one GPU: no exchange, the limit is never reached
    finally:
        d.close()
    r0 = TextDecoder(model, device=0, rank=0, world=2)
    try:
        with pytest.raises(B.CudaBackendError):
            TextDecoder.attach_local([r0])  # every rank is needed
    finally:
        r0.close()
