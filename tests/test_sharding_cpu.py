"""KV-head sharding and the per-layer all-gather, on CPU ranks (gloo, world size 2).

Each rank computes its shard of a decode step with the CPU oracle standing in
for the GPU kernels (no GPU here), gathers the head outputs with
``popkv_b200.sharding.gather_heads``, and checks the result equals the
unsharded step.  A second case makes one rank fail before the collective and
checks the survivor's collective ends with an error instead of hanging.
"""
from __future__ import annotations

import os
import socket
import sys
from pathlib import Path

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

ROOT = Path(__file__).resolve().parents[1]


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _decode_step_oracle(x, heads_q, heads_kv, budget, tg, g):
    import oracle
    from popkv_b200.workloads import to_bf16_bits
    kbits = to_bf16_bits(x.keys[0][heads_kv])
    vbits = to_bf16_bits(x.values[0][heads_kv])
    qbits = to_bf16_bits(x.queries[:, heads_q])
    ck = to_bf16_bits(x.current_keys[0][heads_kv])
    cv = to_bf16_bits(x.current_values[0][heads_kv])
    q_local = qbits.shape[1]
    kv_local = kbits.shape[0]
    mapping = np.arange(q_local) // (q_local // kv_local)
    T = kbits.shape[1]
    planes = oracle.pack(kbits, "bf16", token_group_size=tg, dim_group_size=g)
    enc = oracle.query_encode(qbits, "bf16", dim_group_size=g)
    _, s16 = oracle.score(enc, planes, head_to_kv=mapping, tokens=T, dim_group_size=g, head_dim=128)
    idx = oracle.select_with_current(s16, budget, T)[0]
    return oracle.attention(qbits[0], "bf16", kbits, vbits, "bf16", ck, cv, idx, mapping)


def _worker(rank, world, port, mode, result_path):
    sys.path.insert(0, str(ROOT))
    import datetime
    import torch.distributed as dist
    from popkv_b200.sharding import gather_heads, head_shard
    from popkv_b200.workloads import decode_inputs
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=10))
    try:
        x = decode_inputs(context=512, seed=3, dtype="bf16")
        shard = head_shard(32, 8, world, rank)
        if mode == "fail" and rank == 1:
            raise SystemExit(3)  # this rank leaves before the collective
        local = _decode_step_oracle(x, shard.q_slice, shard.kv_slice, budget=128, tg=64, g=64)
        local_t = torch.from_numpy(local.astype(np.float32))[None]
        try:
            full = gather_heads(local_t)
        except Exception as exc:  # the failure mode: a peer never joined
            np.save(result_path, np.array([f"error: {type(exc).__name__}"]))
            return
        if rank == 0:
            np.save(result_path, full[0].numpy())
    finally:
        if dist.is_initialized():
            try:
                dist.destroy_process_group()
            except Exception:
                pass


def test_head_shard_arithmetic():
    from popkv_b200.sharding import head_shard
    for world in (1, 2, 4, 8):
        shards = [head_shard(32, 8, world, r) for r in range(world)]
        assert [s.q_start for s in shards] == [r * 32 // world for r in range(world)]
        assert all(s.kv_heads * 4 == s.q_heads for s in shards)
        assert shards[-1].kv_end == 8 and shards[-1].q_end == 32
        mapping = shards[0].local_head_to_kv()
        assert mapping.tolist() == [h // 4 for h in range(32 // world)]
    with pytest.raises(ValueError):
        head_shard(32, 8, 3, 0)


def test_sharded_step_equals_unsharded(tmp_path):
    from popkv_b200.workloads import decode_inputs
    world, port = 2, _free_port()
    result = tmp_path / "full.npy"
    ctx = mp.get_context("spawn")
    procs = [ctx.Process(target=_worker, args=(r, world, port, "ok", str(result))) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    got = np.load(result)
    x = decode_inputs(context=512, seed=3, dtype="bf16")
    want = _decode_step_oracle(x, slice(0, 32), slice(0, 8), budget=128, tg=64, g=64)
    np.testing.assert_allclose(got, want.astype(np.float32), rtol=0, atol=0)


def test_rank_failure_surfaces_as_error_not_hang(tmp_path):
    world, port = 2, _free_port()
    result = tmp_path / "survivor.npy"
    ctx = mp.get_context("spawn")
    procs = [ctx.Process(target=_worker, args=(r, world, port, "fail", str(result))) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
    assert procs[1].exitcode == 3
    assert procs[0].exitcode == 0
    assert str(np.load(result)[0]).startswith("error:")
