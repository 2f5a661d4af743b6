"""The oracle and the CUDA path against recorded outputs of the reference's CUDA kernels.

``tests/golden/reference_cuda.npz`` holds what the reference's compiled
extension (built with its own flags, --use_fast_math included) returned on the
seeded config-0, config-1 and popkv-normal inputs
(``tests/golden/make_reference_cuda.py``).  These tests need neither the
reference nor its build:

* sign and magnitude planes, key and query: identical (comparisons only);
* fp16 key representatives: at most one unit in the last place apart, in at
  most 1% of the entries (the reference's fast-math divide against the
  correctly rounded one); query representatives at most 4 units;
* scores: the oracle's scorer on the reference's own encodings reproduces the
  reference's fp16 scores bit for bit;
* selections: a token selected by one side only sits at the row's selection
  boundary -- its score within two fp16 units of the k-th score.
"""
from __future__ import annotations

from pathlib import Path

import numpy as np
import pytest

import oracle
from popkv_b200.workloads import decode_inputs, head_to_kv

FIXTURE = Path(__file__).resolve().parent / "golden" / "reference_cuda.npz"
CASES = ("config0", "config1", "popkv_normal")
# The oracle runs on the CPU cases only: config 1's inputs are hundreds of MB of
# arrays, which the CUDA-path test (on a GPU host) covers.
CPU_CASES = ("config0", "popkv_normal")

pytestmark = pytest.mark.skipif(not FIXTURE.exists(), reason="reference CUDA fixture not recorded")


@pytest.fixture(scope="module")
def fx():
    return np.load(FIXTURE)


def _ulps16(a, b):
    def order(x):
        x = np.asarray(x).view(np.uint16).astype(np.int32)
        return np.where(x & 0x8000, 0x8000 - (x & 0x7FFF), 0x8000 + x)
    return np.abs(order(a) - order(b))


def _ulps32(a, b):
    def order(x):
        x = np.asarray(x, np.float32).view(np.int32).astype(np.int64)
        return np.where(x < 0, -(x & 0x7FFFFFFF), x)
    return np.abs(order(a) - order(b))


def _digest(array) -> str:
    import hashlib
    return hashlib.sha256(np.ascontiguousarray(array).tobytes()).hexdigest()


_ORACLE_CACHE = {}


def _oracle_case(name, fx):
    """The oracle's planes, query encodings, scores and selection on the case's inputs."""
    if name in _ORACLE_CACHE:
        return _ORACLE_CACHE[name]
    tg, g, context, budget, k = (int(v) for v in fx[f"{name}/meta"])
    dtype = "f32" if name == "config0" else "bf16"
    x = decode_inputs(context=context, seed=0, dtype=dtype)
    # bf16 inputs are stored as the fp32 values of bf16 numbers: the same elements.
    planes = oracle.pack(x.keys[0].astype(np.float32), "f32", token_group_size=tg, dim_group_size=g)
    enc = oracle.query_encode(x.queries.astype(np.float32), "f32", dim_group_size=g)
    mapping = head_to_kv(32, 8)
    _, scores = oracle.score(enc, planes, head_to_kv=mapping, tokens=context, dim_group_size=g, head_dim=128)
    selected = np.sort(oracle.topk(scores, k), axis=-1)
    _ORACLE_CACHE[name] = (planes, enc, scores, selected, k)
    return _ORACLE_CACHE[name]


def _boundary_check(name, selected_ref, selected_ours, scores_ours, kth_ref):
    """Tokens in one selection only: score within 2 fp16 units of the reference's k-th score."""
    sym, far = 0, []
    for h in range(selected_ref.shape[0]):
        diff = set(selected_ref[h].astype(np.int64).tolist()) ^ set(selected_ours[h].astype(np.int64).tolist())
        sym += len(diff)
        for t in diff:
            u = int(_ulps16(scores_ours[h, t], kth_ref[h]))
            if u > 2:
                far.append((h, t, u))
    assert not far, f"{name}: selection differences away from the boundary: {far[:5]}"
    return sym


@pytest.mark.parametrize("name", CPU_CASES)
def test_oracle_planes_and_query_encoding_match_reference_cuda(fx, name):
    planes, enc, _, _, _ = _oracle_case(name, fx)
    digests = [str(d) for d in fx[f"{name}/digests"]]
    assert _digest(planes[0]) == digests[0], "sign planes differ"
    assert _digest(planes[1]) == digests[1], "magnitude planes differ"
    for i, plane in enumerate(("q_sign", "q_mag")):
        assert np.array_equal(enc[i], fx[f"{name}/{plane}"]), plane
    for i, plane in ((2, "q_low"), (3, "q_delta")):
        assert int(_ulps32(enc[i], fx[f"{name}/{plane}"]).max()) <= 4, plane
    if f"{name}/k_low" in fx:
        for i, plane in ((2, "k_low"), (3, "k_delta")):
            u = _ulps16(planes[i], fx[f"{name}/{plane}"])
            assert int(u.max()) <= 1, plane
            assert int((u > 0).sum()) <= 0.01 * u.size, plane


def test_oracle_scorer_reproduces_reference_scores_bit_for_bit(fx):
    name = "config0"
    tg, g, context, budget, k = (int(v) for v in fx[f"{name}/meta"])
    enc = tuple(fx[f"{name}/{p}"] for p in ("q_sign", "q_mag", "q_low", "q_delta"))
    planes = tuple(fx[f"{name}/{p}"] for p in ("k_sign", "k_mag", "k_low", "k_delta"))
    _, scores = oracle.score(enc, planes, head_to_kv=head_to_kv(32, 8), tokens=context, dim_group_size=g,
                             head_dim=128)
    assert np.array_equal(scores, fx[f"{name}/scores"])


@pytest.mark.parametrize("name", CPU_CASES)
def test_oracle_selection_matches_reference_cuda_at_the_boundary(fx, name):
    _, _, scores, selected, k = _oracle_case(name, fx)
    sym = _boundary_check(name, fx[f"{name}/selected"], selected[0], scores[0], fx[f"{name}/kth_score"])
    assert sym <= max(4, 1e-4 * 32 * k)


@pytest.mark.gpu
@pytest.mark.parametrize("name", CASES)
def test_cuda_path_matches_reference_cuda_fixture(fx, name, cuda_device):
    import torch
    from popkv_b200 import popkv as P
    from popkv_b200 import popkv_cuda as C
    tg, g, context, budget, k = (int(v) for v in fx[f"{name}/meta"])
    dtype = torch.float32 if name == "config0" else torch.bfloat16
    x = decode_inputs(context=context, seed=0, dtype="f32" if name == "config0" else "bf16")
    keys = torch.from_numpy(x.keys[0]).to(dtype).to(cuda_device).contiguous()
    queries = torch.from_numpy(x.queries).to(dtype).to(cuda_device).contiguous()
    mapping = torch.from_numpy(head_to_kv(32, 8)).to(cuda_device)
    planes = C.pack_keys(keys, token_capacity=context, token_group_size=tg, dim_group_size=g)
    enc = C.query_encode(queries, dim_group_size=g)
    scores = C.score_encoded(enc, planes, head_to_kv=mapping, tokens=context, dim_group_size=g)
    selected = np.sort(P.topk(scores, k)[0].cpu().numpy(), axis=-1)
    torch.cuda.synchronize()
    digests = [str(d) for d in fx[f"{name}/digests"]]
    assert _digest(planes[0].cpu().numpy()) == digests[0]
    assert _digest(planes[1].cpu().numpy()) == digests[1]
    for i, plane in enumerate(("q_sign", "q_mag")):
        assert np.array_equal(enc[i].cpu().numpy(), fx[f"{name}/{plane}"]), plane
    scores_np = scores[0].cpu().numpy().view(np.uint16)
    sym = _boundary_check(name, fx[f"{name}/selected"], selected, scores_np, fx[f"{name}/kth_score"])
    assert sym <= max(4, 1e-4 * 32 * k)
