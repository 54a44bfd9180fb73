"""Tensor-parallel sharding of the decoder, host side: two gloo ranks on the
CPU query their slice through the C ABI (eosi_cuda_text_partition, no GPU
needed) and check that the slices tile every dimension exactly once -- heads,
FFN units, vocabulary rows and the O / down output rows -- and that the
IPC-handle all-gather the decoder uses moves the bytes intact."""
from __future__ import annotations

import os

import pytest
import torch.distributed as dist
import torch.multiprocessing as mp

CONFIGS = [
    dict(n_embd=4096, n_layer=32, n_head=32, n_kv_head=32, n_ff=11008, n_vocab=32000, max_ctx=768, wdtype=33,
         out_dtype=33),
    dict(n_embd=4096, n_layer=2, n_head=32, n_kv_head=8, n_ff=14336, n_vocab=32003, max_ctx=64, wdtype=33,
         out_dtype=32),
    dict(n_embd=512, n_layer=1, n_head=4, n_kv_head=2, n_ff=768, n_vocab=1000, max_ctx=64, wdtype=32, out_dtype=33),
]


def _worker(rank: int, world: int, port: int, q) -> None:
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from eosllm_b200.text import partition
        parts = []
        for cfg in CONFIGS:
            mine = partition(cfg, rank, world)
            allp = [None] * world
            dist.all_gather_object(allp, mine)
            parts.append(allp)
        blob = bytes((rank * 37 + i) % 256 for i in range(64))  # stands in for an IPC handle
        handles = [None] * world
        dist.all_gather_object(handles, blob)
        q.put((rank, parts, handles))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2])
def test_two_rank_partitions_tile_the_model(cuda_lib, world):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = 29500 + os.getpid() % 1000
    procs = [ctx.Process(target=_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    results = dict((r, (parts, h)) for r, parts, h in (q.get(timeout=120) for _ in procs))
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    for ci, cfg in enumerate(CONFIGS):
        views = results[0][0][ci]
        assert views == results[1][0][ci]  # every rank sees the same table
        for key0, keyl, total in (("head0", "heads", cfg["n_head"]), ("kv_head0", "kv_heads", cfg["n_kv_head"]),
                                  ("ff0", "ff_len", cfg["n_ff"]), ("vocab0", "vocab_len", cfg["n_vocab"]),
                                  ("out_row0", "out_rows", cfg["n_embd"])):
            pos = 0
            for r in range(world):
                assert views[r][key0] == pos, (cfg, key0, r)
                assert views[r][keyl] > 0
                pos += views[r][keyl]
            assert pos == total, (cfg, key0)
        for r in range(world):  # FFN units in whole 32-element packing groups
            assert views[r]["ff0"] % 32 == 0 and views[r]["ff_len"] % 32 == 0
            assert views[r]["head_dim"] == cfg["n_embd"] // cfg["n_head"]
    for r in range(world):
        assert results[r][1] == [bytes((q * 37 + i) % 256 for i in range(64)) for q in range(world)]


def test_partition_rejects_bad_worlds(cuda_lib):
    from eosllm_b200 import backend as B
    from eosllm_b200.text import partition
    cfg = dict(CONFIGS[0])
    with pytest.raises(B.CudaBackendError):
        partition(cfg, 0, 3)  # 3 does not divide 32 heads
    with pytest.raises(B.CudaBackendError):
        partition(cfg, 2, 2)  # rank out of range
    with pytest.raises(B.CudaBackendError):
        partition(dict(cfg, n_head=128, n_kv_head=128), 0, 8)  # head_dim 32 unsupported
