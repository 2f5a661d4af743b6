"""Record the reference's compiled CUDA kernels' outputs as fixtures: ``reference_cuda.npz``.

Test infrastructure.  Runs on a CUDA host where ``oracle/build_ref.py`` has
built the reference's own extension (csrc/popkv_ext.cu + popkv_ext.cpp with its
flags, --use_fast_math included) into ``oracle/_ref/``.  It feeds the seeded
inputs of ``popkv_b200.workloads.decode_inputs`` through the reference's
decode path -- pack / pack_dim (popkv_cuda.py:53-69), query_encode_out
(:157-167), score_encoded (:170-187) and torch.topk(scores, k, sorted=False)
(popkv.py:1090-1099) -- and stores what they return:

* ``config0`` (token group 64, dim group 64, 4096 tokens, budget 512, fp32
  inputs): every output -- key planes and representatives, query encodings,
  fp16 scores, and the selected token set of every query row (sorted);
* ``config1`` (token group 128, dim group 16, 32768 tokens, budget 4096, bf16)
  and ``popkv_normal`` (32 / 32, 8192 tokens, budget 1024, bf16): the query
  encodings, the selected token sets (sorted) and each row's k-th largest
  score, plus SHA-256 digests of the planes and scores (the arrays themselves
  are megabytes).

The tests read the fixture without the reference: the oracle against it on
the CPU (tests/test_reference_fixtures.py) and the CUDA path against it on a
GPU.  Usage (on the GPU host): ``python tests/golden/make_reference_cuda.py
[--out PATH]``.
"""
from __future__ import annotations

import argparse
import hashlib
import sys
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parents[2]
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))

CASES = {
    # name: (token group, dim group, context, budget, input dtype, full arrays)
    "config0": (64, 64, 4096, 512, "f32", True),
    "config1": (128, 16, 32768, 4096, "bf16", False),
    "popkv_normal": (32, 32, 8192, 1024, "bf16", False),
}


def digest(array) -> str:
    return hashlib.sha256(np.ascontiguousarray(array).tobytes()).hexdigest()


def run_case(ref, name, dev):
    import torch
    from popkv_b200.workloads import decode_inputs, head_to_kv
    tg, g, context, budget, dtype, full = CASES[name]
    torch_dtype = torch.float32 if dtype == "f32" else torch.bfloat16
    x = decode_inputs(context=context, seed=0, dtype=dtype)
    keys = torch.from_numpy(x.keys[0]).to(torch_dtype).to(dev).contiguous()
    queries = torch.from_numpy(x.queries).to(torch_dtype).to(dev).contiguous()
    mapping = torch.from_numpy(head_to_kv(32, 8)).to(dev)
    k = min(budget - 1, context)
    planes = ref.pack(keys, context, tg) if g == 32 else ref.pack_dim(keys, context, g, tg)
    enc = (torch.empty((1, 32, 4), dtype=torch.int32, device=dev),
           torch.empty((1, 32, 4), dtype=torch.int32, device=dev),
           torch.empty((1, 32, 128 // g), dtype=torch.float32, device=dev),
           torch.empty((1, 32, 128 // g), dtype=torch.float32, device=dev))
    ref.query_encode_out(queries, *enc, g)
    scores = ref.score_encoded(*enc, *planes, mapping, context, g)
    top = torch.topk(scores, k, dim=-1, sorted=False)
    torch.cuda.synchronize()
    npy = lambda t: t.cpu().numpy()  # noqa: E731
    sel = np.sort(npy(top.indices[0]), axis=-1).astype(np.uint16 if context <= 65536 else np.int64)
    kth = npy(top.values[0]).min(axis=-1).view(np.uint16)
    scores_bits = npy(scores).view(np.uint16)
    out = {
        f"{name}/meta": np.array([tg, g, context, budget, k], np.int64),
        f"{name}/q_sign": npy(enc[0]), f"{name}/q_mag": npy(enc[1]),
        f"{name}/q_low": npy(enc[2]), f"{name}/q_delta": npy(enc[3]),
        f"{name}/selected": sel, f"{name}/kth_score": kth,
        f"{name}/digests": np.array([digest(npy(p)) for p in planes] + [digest(scores_bits)]),
    }
    if full:
        out[f"{name}/k_sign"] = npy(planes[0])
        out[f"{name}/k_mag"] = npy(planes[1])
        out[f"{name}/k_low"] = npy(planes[2]).view(np.uint16)
        out[f"{name}/k_delta"] = npy(planes[3]).view(np.uint16)
        out[f"{name}/scores"] = scores_bits
    return out


def main(argv=None) -> int:
    p = argparse.ArgumentParser(description=__doc__.split("\n")[0])
    p.add_argument("--out", default=str(Path(__file__).resolve().parent / "reference_cuda.npz"))
    args = p.parse_args(argv)
    import torch
    from oracle.build_ref import load_reference_extension
    ref = load_reference_extension()
    if ref is None:
        print("reference extension not built (oracle/build_ref.py)", file=sys.stderr)
        return 1
    dev = torch.device("cuda", 0)
    arrays = {}
    for name in CASES:
        arrays.update(run_case(ref, name, dev))
    np.savez_compressed(args.out, **arrays)
    print(f"wrote {args.out}: {len(arrays)} arrays")
    return 0


if __name__ == "__main__":
    sys.exit(main())
