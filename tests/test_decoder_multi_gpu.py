"""Full-model decode on two GPUs, one process per GPU over NCCL (needs 2 GPUs).

* KV-head shards with the replicated output projection and MLP (the attention
  rows all-gathered per layer, inside the graph) reproduce the single-GPU
  decode bit for bit: every head's retrieval and attention is computed the
  same way, and the gathered rows are copies.
* The tensor-parallel output projection and MLP (partial products summed by
  two all-reduces per layer) match it within bf16 tolerance: the partial sums
  are rounded to bf16 before they are added.  The peer-memory all-reduce
  (popkv_peer_sum) and NCCL's give the same bits at two ranks.  Checked with dense layers, where
  a last-bit difference in q cannot swap a near-tied token in the top-k.
"""
from __future__ import annotations

import os
import socket
from datetime import timedelta

import pytest
import torch

pytestmark = pytest.mark.gpu

WORLD = 2


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank: int, port: int, method: str) -> None:
    import torch.distributed as dist

    from popkv_b200.decoder import LlamaConfig, LlamaSparseDecoder, LlamaWeights
    from popkv_b200.popkv import RetrievalConfig
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=WORLD, timeout=timedelta(seconds=60), device_id=dev)
    decoders = []
    try:
        cfg = LlamaConfig(hidden_size=1024, num_attention_heads=8, num_key_value_heads=2, intermediate_size=2048,
                          vocab_size=2000, num_hidden_layers=4)
        weights = LlamaWeights.random(cfg, device=dev, seed=11, std=0.02)
        retrieval = RetrievalConfig(budget=64, group_size=64, dim_group_size=64) if method != "full" else None
        ids = torch.randint(0, cfg.vocab_size, (1, 150), generator=torch.Generator().manual_seed(5))
        single = LlamaSparseDecoder(weights, method=method, retrieval=retrieval, max_context=170)
        shard = LlamaSparseDecoder(weights, method=method, retrieval=retrieval, max_context=170, rank=rank,
                                   world=WORLD)
        tensor = LlamaSparseDecoder(weights, method=method, retrieval=retrieval, max_context=170, rank=rank,
                                    world=WORLD, mlp_parallel="tensor")
        tensor_nccl = LlamaSparseDecoder(weights, method=method, retrieval=retrieval, max_context=170,
                                         rank=rank, world=WORLD, mlp_parallel="tensor", all_reduce="nccl")
        decoders = [single, shard, tensor, tensor_nccl]
        for d in decoders:
            d.prefill(ids)
        for _ in range(8):
            tok = single.token.clone()
            shard.token.copy_(tok)
            tensor.token.copy_(tok)
            tensor_nccl.token.copy_(tok)
            want = single.decode().clone()
            got = shard.decode().clone()
            assert torch.equal(got, want), "replicated-MLP shard differs from the single-GPU decode"
            tp = tensor.decode().clone()
            assert not tensor.all_reduce_error()
            # Two ranks: both all-reduces round the exact sum of two bf16 values once.
            assert torch.equal(tp, tensor_nccl.decode()), "peer all-reduce differs from NCCL's"
            if method == "full":
                rel = float((tp - want).norm() / want.norm())
                assert rel < 1e-2, rel
        assert int(tensor.position.item()) == int(single.position.item()) == 158
    finally:
        for d in decoders:
            d.close()
        del decoders
        dist.destroy_process_group()


def _need_two_gpus():
    if not torch.cuda.is_available() or torch.cuda.device_count() < WORLD:
        pytest.skip("needs 2 GPUs")


@pytest.mark.parametrize("method", ["full", "popkv-s"])
def test_sharded_full_model_decode(method):
    _need_two_gpus()
    import torch.multiprocessing as mp
    mp.spawn(_worker, args=(_free_port(), method), nprocs=WORLD, join=True)
