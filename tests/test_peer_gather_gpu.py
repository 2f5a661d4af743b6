"""Merge fused with the cross-GPU all-gather, and the one-shot all-reduce, over
peer memory (needs 2 GPUs).

Two processes, one per GPU, exchange CUDA IPC handles over a gloo group.  The
gathered output must equal every rank's popkv_attn_merge of its own rows, bit
for bit, over several launches (both receive-buffer parities), eagerly and
inside a replayed CUDA graph; and a KV-head-sharded decode step must equal the
unsharded step.  popkv_peer_sum must equal the fp32 rank-order sum rounded
once, eagerly, as two sums per replayed graph, and after a collective reset.
On one GPU, both kernels' bounded waits are made to run out (a peer area that
nobody writes) and must report it and return.
"""
from __future__ import annotations

import os
import socket

import pytest
import torch

pytestmark = pytest.mark.gpu

WORLD = 2


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _partials(rank: int, rows: int, splits: int) -> torch.Tensor:
    gen = torch.Generator().manual_seed(1000 + rank)
    p = torch.randn(rows, splits, 130, generator=gen)
    p[..., 1] = torch.rand(rows, splits, generator=gen) * 2 + 0.5  # positive softmax sums
    return p


def _merge_worker(rank: int, port: int, rows: int, splits: int) -> None:
    import torch.distributed as dist

    from popkv_b200 import _lib
    from popkv_b200.sharding import PeerGather
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("gloo", rank=rank, world_size=WORLD,
                            timeout=__import__("datetime").timedelta(seconds=60))
    try:
        lib = _lib.lib()
        want = []
        for r in range(WORLD):  # every rank's rows merged locally with popkv_attn_merge
            p = _partials(r, rows, splits).to(dev)
            out = torch.empty(rows, 128, dtype=torch.bfloat16, device=dev)
            _lib.check(lib.popkv_attn_merge(_lib.ptr(p), rows, splits, 128, _lib.ptr(out), _lib.BF16,
                                            _lib.stream_of(dev)))
            want.append(out)
        want = torch.cat(want)
        mine = _partials(rank, rows, splits).to(dev)
        gather = PeerGather(rows, torch.bfloat16, dev)
        for _ in range(3):
            gather.output.zero_()
            gather.launch(mine, splits, _lib.stream_of(dev))
            torch.cuda.synchronize(dev)
            assert not gather.error()
            assert torch.equal(gather.output, want), "eager merge+gather differs"
        side = torch.cuda.Stream(dev)
        side.wait_stream(torch.cuda.current_stream(dev))
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=side):
            gather.launch(mine, splits, _lib.stream_of(dev))
        for _ in range(3):
            gather.output.zero_()
            graph.replay()
            torch.cuda.synchronize(dev)
            assert not gather.error()
            assert torch.equal(gather.output, want), "graph merge+gather differs"
        del graph
        gather.close()
    finally:
        dist.destroy_process_group()


def _step_worker(rank: int, port: int) -> None:
    import torch.distributed as dist

    from popkv_b200 import popkv as P
    from popkv_b200.decode import SparseAttentionStep
    from popkv_b200.sharding import PeerGather, head_shard
    from popkv_b200.workloads import decode_inputs, head_to_kv
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("gloo", rank=rank, world_size=WORLD,
                            timeout=__import__("datetime").timedelta(seconds=60))
    try:
        x = decode_inputs(context=4000, seed=17, dtype="bf16")
        to = lambda a: torch.from_numpy(a).to(torch.bfloat16).to(dev)  # noqa: E731
        tg, g = P.POPKV_PRESETS["popkv-q"]
        keys, values = to(x.keys[0]), to(x.values[0])
        q, ck, cv = to(x.queries), to(x.current_keys[0]), to(x.current_values[0])
        full_cache = P.build_popkv_cache(keys, group_size=tg, dim_group_size=g, reserve_tokens=0)
        full = SparseAttentionStep(full_cache, keys, values, torch.from_numpy(head_to_kv(32, 8)).to(dev),
                                   budget=512)
        want = full(q, ck, cv).clone().view(32, 128)
        sh = head_shard(32, 8, WORLD, rank)
        lk, lv = keys[sh.kv_slice].contiguous(), values[sh.kv_slice].contiguous()
        cache = P.build_popkv_cache(lk, group_size=tg, dim_group_size=g, reserve_tokens=0)
        gather = PeerGather(sh.q_heads, torch.bfloat16, dev)
        step = SparseAttentionStep(cache, lk, lv, sh.local_head_to_kv(dev), budget=512, gather=gather)
        for _ in range(3):
            got = step(q[:, sh.q_slice], ck[sh.kv_slice], cv[sh.kv_slice])
            torch.cuda.synchronize(dev)
            assert not gather.error()
            assert torch.equal(got, want), "sharded step differs from the unsharded step"
        step.graph = None
        gather.close()
    finally:
        dist.destroy_process_group()


def _sum_worker(rank: int, port: int, count: int, dtype_name: str) -> None:
    import torch.distributed as dist

    from popkv_b200 import _lib
    from popkv_b200.sharding import PeerSum
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("gloo", rank=rank, world_size=WORLD,
                            timeout=__import__("datetime").timedelta(seconds=60))
    dtype = getattr(torch, dtype_name)
    try:
        def vec(r: int, step: int) -> torch.Tensor:
            gen = torch.Generator().manual_seed(100 * step + r)
            return (torch.randn(count, generator=gen) * (1 + r)).to(dtype)

        peer = PeerSum(count, dtype, dev)
        data = torch.empty(count, dtype=dtype, device=dev)
        stream = _lib.stream_of(dev)
        # Eager: three launches (both receive parities); the sum over ranks in
        # fp32, rank order, rounded once to the vector's type.
        for step in range(3):
            data.copy_(vec(rank, step))
            peer.launch(data, stream)
            torch.cuda.synchronize(dev)
            assert not peer.error()
            want = sum((vec(r, step).float() for r in range(WORLD)), torch.zeros(count)).to(dtype)
            assert torch.equal(data.cpu(), want), "eager peer sum differs"
        side = torch.cuda.Stream(dev)
        side.wait_stream(torch.cuda.current_stream(dev))
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=side):
            peer.launch(data, _lib.stream_of(dev))
            peer.launch(data, _lib.stream_of(dev))  # two sums per replay, as a decode layer issues
        for step in range(3, 6):
            data.copy_(vec(rank, step))
            graph.replay()
            torch.cuda.synchronize(dev)
            assert not peer.error()
            once = sum((vec(r, step).float() for r in range(WORLD)), torch.zeros(count)).to(dtype)
            want = (once.float() * WORLD).to(dtype)  # every rank holds `once`, summed again
            assert torch.equal(data.cpu(), want), "graph peer sum differs"
        del graph
        # A collective reset returns both ranks to epoch 0 with clean areas; the
        # next sums are exact again.
        peer.reset()
        assert peer.state.tolist()[:3] == [0, 0, 0]
        for step in range(6, 8):
            data.copy_(vec(rank, step))
            peer.launch(data, stream)
            torch.cuda.synchronize(dev)
            assert not peer.error()
            want = sum((vec(r, step).float() for r in range(WORLD)), torch.zeros(count)).to(dtype)
            assert torch.equal(data.cpu(), want), "peer sum after reset differs"
        peer.close()
    finally:
        dist.destroy_process_group()


def _need_two_gpus():
    if not torch.cuda.is_available() or torch.cuda.device_count() < WORLD:
        pytest.skip("needs 2 GPUs")


@pytest.mark.parametrize("rows,splits", [(16, 16), (32, 3), (1, 1)])
def test_merge_gather_equals_local_merges(rows, splits):
    _need_two_gpus()
    import torch.multiprocessing as mp
    mp.spawn(_merge_worker, args=(_free_port(), rows, splits), nprocs=WORLD, join=True)


def test_sharded_step_with_peer_gather_equals_unsharded_step():
    _need_two_gpus()
    import torch.multiprocessing as mp
    mp.spawn(_step_worker, args=(_free_port(),), nprocs=WORLD, join=True)


@pytest.mark.parametrize("count,dtype_name", [(4096, "bfloat16"), (16384, "bfloat16"), (2, "float16"),
                                              (1000, "float32")])
def test_peer_sum_equals_rank_order_sum(count, dtype_name):
    _need_two_gpus()
    import torch.multiprocessing as mp
    mp.spawn(_sum_worker, args=(_free_port(), count, dtype_name), nprocs=WORLD, join=True)


# ---------------------------------------------------------------------------
# Bounded waits that run out, on one GPU.  Rank 0 of a world of 2 whose "peer"
# area is a second local buffer that nobody writes: every poll of the peer's
# words fails, the waits give up after the poll limit in state[3], the kernel
# sets state[2] and returns, and the stream stays usable.  No GPU fault or hang
# is involved: the waits are bounded and the status is read on the host.
# ---------------------------------------------------------------------------

def _lonely_areas(dev, words_per_rank: int, poll_limit: int):
    own = torch.zeros(2 * WORLD * words_per_rank, dtype=torch.int64, device=dev)
    silent_peer = torch.zeros_like(own)
    ptrs = torch.tensor([own.data_ptr(), silent_peer.data_ptr()], dtype=torch.int64, device=dev)
    state = torch.tensor([0, 0, 0, poll_limit], dtype=torch.int32, device=dev)
    return own, silent_peer, ptrs, state


def test_peer_sum_wait_runs_out_and_reports(cuda_device):
    import ctypes

    from popkv_b200 import _lib
    lib, dev = _lib.lib(), cuda_device
    count = 4096
    data = torch.randn(count, device=dev).to(torch.bfloat16)
    own, silent_peer, ptrs, state = _lonely_areas(dev, count // 2, poll_limit=2000)
    _lib.check(lib.popkv_peer_sum(_lib.ptr(data), _lib.BF16, count, 0, WORLD, _lib.ptr(ptrs),
                                  ctypes.c_void_p(own.data_ptr()), _lib.ptr(state), _lib.stream_of(dev)))
    torch.cuda.synchronize(dev)
    assert state.tolist()[:3] == [1, 0, 1]  # the launch ended, its epoch advanced, the flag is set
    # This rank's words went out to the silent peer's area with epoch 1.
    assert int((silent_peer.view(2, WORLD, -1)[1, 0] >> 32).eq(1).sum()) == count // 2
    # The stream and the context still work: a one-rank sum is the identity.
    again = data.clone()
    solo_state = torch.zeros(4, dtype=torch.int32, device=dev)
    solo_ptrs = torch.tensor([own.data_ptr()], dtype=torch.int64, device=dev)
    _lib.check(lib.popkv_peer_sum(_lib.ptr(again), _lib.BF16, count, 0, 1, _lib.ptr(solo_ptrs),
                                  ctypes.c_void_p(own.data_ptr()), _lib.ptr(solo_state), _lib.stream_of(dev)))
    torch.cuda.synchronize(dev)
    assert torch.equal(again, data) and solo_state.tolist()[:3] == [1, 0, 0]


def test_merge_gather_wait_runs_out_and_reports(cuda_device):
    import ctypes

    from popkv_b200 import _lib
    lib, dev = _lib.lib(), cuda_device
    rows, splits = 8, 4
    partials = _partials(0, rows, splits).to(dev)
    own, silent_peer, ptrs, state = _lonely_areas(dev, rows * 128, poll_limit=2000)
    out = torch.empty(WORLD * rows, 128, dtype=torch.bfloat16, device=dev)
    for launch in (1, 2):  # both receive parities
        _lib.check(lib.popkv_attn_merge_gather(_lib.ptr(partials), rows, splits, 128, _lib.BF16, 0, WORLD,
                                               _lib.ptr(ptrs), ctypes.c_void_p(own.data_ptr()), _lib.ptr(state),
                                               _lib.ptr(out), _lib.stream_of(dev)))
        torch.cuda.synchronize(dev)
        assert state.tolist()[:3] == [launch, 0, 1]
    # The rank's own rows are still merged correctly.
    want = torch.empty(rows, 128, dtype=torch.bfloat16, device=dev)
    _lib.check(lib.popkv_attn_merge(_lib.ptr(partials), rows, splits, 128, _lib.ptr(want), _lib.BF16,
                                    _lib.stream_of(dev)))
    torch.cuda.synchronize(dev)
    assert torch.equal(out[:rows], want)
