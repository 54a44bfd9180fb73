"""Tensor-parallel decoder on two GPUs (one child process per GPU, gloo for
the host-side handle exchange; the data path is the decoder's own pushes over
NVLink).  Every matrix is split by output rows, so each output element is
computed whole on one rank, exactly as on one GPU: the logits of stepped
tokens, of a greedy generation and of the steps after a batched prefill must
be BIT-IDENTICAL to the one-GPU decoder's on both ranks (and agree with the
decoder oracle within the reference's envelope).  Skipped on machines with
fewer than two GPUs."""
from __future__ import annotations

import os

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu

N_PREFILL = 33  # tokens fed by the batched prefill in the prefill check
N_GEN = 20
CASES = [dict(n_embd=512, n_head=4, n_kv_head=2, n_ff=768, n_vocab=1000, n_layer=2),
         dict(n_embd=512, n_head=8, n_kv_head=2, n_ff=512, n_vocab=77, n_layer=2, wdtype=32, out_dtype=32),
         dict(n_embd=4096, n_head=32, n_kv_head=32, n_ff=11008, n_vocab=512, n_layer=1, seed=9)]


def _run_decoder(dec, kw, tokens, prompt, barrier=lambda: None):
    """Stepped logits, a greedy generation, then prefill + stepped logits."""
    logits = []
    for t in tokens:
        barrier()
        logits.append(dec.step(int(t)))
    barrier()
    dec.reset()
    barrier()
    picks = dec.generate(prompt, N_GEN)  # Q4_K: the prompt through the batched prefill
    barrier()
    dec.reset()
    barrier()
    pf_logits = []
    if kw.get("wdtype", 33) == 33:
        dec.prefill(np.asarray(tokens[:N_PREFILL], np.uint32))
        for t in tokens[N_PREFILL:]:
            barrier()
            pf_logits.append(dec.step(int(t)))
    barrier()
    return np.stack(logits), picks.tolist(), (np.stack(pf_logits) if pf_logits else None)


def _tp_worker(rank: int, world: int, port: int, kw: dict, tokens, prompt, q, mode: int = 0) -> None:
    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        torch.cuda.set_device(rank)
        from oracle.llama import make_llama
        from oracle.oracle import Oracle
        from eosllm_b200.text import TextDecoder
        model = make_llama(Oracle(), max_ctx=96, **kw)
        dec = TextDecoder(model, device=rank, rank=rank, world=world)
        dec.set_step_mode(mode)
        dec.connect()
        out = _run_decoder(dec, kw, tokens, prompt, dist.barrier)
        dec.close()
        q.put((rank, out, None))
    except Exception as e:  # report, never hang the parent
        q.put((rank, None, repr(e)))
    finally:
        dist.destroy_process_group()


def _same(a, b) -> bool:
    return np.array_equal(np.asarray(a, np.float32).view(np.uint32), np.asarray(b, np.float32).view(np.uint32))


@pytest.mark.parametrize("mode", [2, 1], ids=["per_op", "persistent"])
@pytest.mark.parametrize("kw", CASES)
def test_two_gpu_decoder_is_bit_identical_to_one_gpu(gpu, oracle, kw, mode):
    """The ranks run the per-op step graph (the default) or the persistent
    step; the one-GPU reference runs the per-op graph."""
    if mode == 1 and kw.get("wdtype", 33) != 33:
        pytest.skip("the persistent step runs Q4_K models")
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    from oracle.llama import OracleDecoder, make_llama
    from eosllm_b200.text import TextDecoder
    from test_gpu_decoder import envelope_check
    world = 2
    rng = np.random.default_rng(21)
    tokens = rng.integers(0, kw["n_vocab"], 40)
    prompt = rng.integers(0, kw["n_vocab"], 30)
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = 29600 + os.getpid() % 300
    procs = [ctx.Process(target=_tp_worker, args=(r, world, port, kw, tokens, prompt, q, mode))
             for r in range(world)]
    for p in procs:
        p.start()
    res = {}
    for _ in procs:
        r, out, err = q.get(timeout=600)
        res[r] = (out, err)
    for p in procs:
        p.join(timeout=120)
    for r in range(world):
        assert res[r][0] is not None, res[r][1]
    model = make_llama(oracle, max_ctx=96, **kw)
    one = TextDecoder(model, device=0)
    one.set_step_mode(TextDecoder.STEP_PER_OP)
    ref = _run_decoder(one, kw, tokens, prompt)
    one.close()
    for r in range(world):
        logits, picks, pf = res[r][0]
        assert _same(logits, ref[0]), f"rank {r}: stepped logits differ from one GPU"
        assert picks == ref[1], f"rank {r}: generated tokens differ from one GPU"
        if ref[2] is not None:
            assert _same(pf, ref[2]), f"rank {r}: logits after the batched prefill differ from one GPU"
    # and those logits are within the reference's envelope of the oracle
    it = iter(ref[0])
    envelope_check(oracle, model, tokens, lambda t: next(it))
