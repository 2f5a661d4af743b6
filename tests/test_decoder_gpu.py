"""Device-resident step lengths and the graph-replayed full-model decode.

* Each ``*_dyn`` kernel equals its static-length counterpart bit for bit (the
  static kernels are themselves pinned to the CPU oracle elsewhere).
* The model-loop glue kernels follow the reference model's eager ops.
* ``LlamaSparseDecoder`` (one CUDA graph per token, device-side position)
  produces bit-identical logits and tokens to the same loop run eagerly with
  the static-length kernels and Python-integer lengths (the reference decoder's
  launch pattern, popkv.py:988-1115), across token-group boundaries.
* With every layer dense it matches transformers' LlamaForCausalLM on the same
  weights within bf16 tolerance.
"""
from __future__ import annotations

import math

import pytest
import torch
import torch.nn.functional as F

from popkv_b200 import _lib, popkv_cuda
from popkv_b200.decoder import (LlamaConfig, LlamaSparseDecoder, LlamaWeights, apply_rope, rms_norm,
                                rope_tables)
from popkv_b200.popkv import RetrievalConfig

pytestmark = pytest.mark.gpu

TINY = LlamaConfig(hidden_size=1024, num_attention_heads=8, num_key_value_heads=2, head_dim=128,
                   intermediate_size=2048, vocab_size=2000, num_hidden_layers=4)


def _stream(dev):
    return _lib.stream_of(dev)


def _planes(dev, kvh, cap, g, keys, tg):
    packed = popkv_cuda.pack_keys(keys, token_capacity=cap, token_group_size=tg, dim_group_size=g)
    return packed


@pytest.mark.parametrize("g,tg", [(16, 128), (64, 64), (32, 32)])
def test_score_and_topk_dyn_match_static(cuda_device, g, tg):
    dev = cuda_device
    gen = torch.Generator().manual_seed(g)
    kvh, qh, T, max_tokens = 2, 8, 1000, 1200
    keys = torch.randn(kvh, T, 128, generator=gen).to(torch.bfloat16).to(dev)
    cap = math.ceil(max_tokens / tg) * tg
    packed = _planes(dev, kvh, cap, g, keys, tg)
    q = torch.randn(1, qh, 128, generator=gen).to(torch.bfloat16).to(dev)
    h2k = torch.arange(qh, device=dev) // (qh // kvh)
    lib, check, ptr = _lib.lib(), _lib.check, _lib.ptr
    for t, k_max in ((T, 255), (137, 255), (1, 7), (0, 7)):
        pos = torch.tensor([t], device=dev, dtype=torch.int64)
        stride = 1208
        scores = torch.full((qh, stride), -7.0, device=dev, dtype=torch.float16)
        check(lib.popkv_score_dyn(ptr(q), _lib.BF16, 1, qh, *(ptr(x) for x in packed), kvh, cap, ptr(h2k),
                                  ptr(pos), max_tokens, g, ptr(scores), stride, _stream(dev)))
        out = torch.full((qh, k_max + 1), -5, device=dev, dtype=torch.int64)
        check(lib.popkv_topk_dyn(ptr(scores), qh, ptr(pos), max_tokens, stride, k_max, ptr(out), k_max + 1,
                                 _stream(dev)))
        torch.cuda.synchronize()
        assert torch.all(scores[:, t:] == -7.0), "scores past the device count were written"
        k = min(k_max, t)
        if t > 0:
            ref = popkv_cuda.score(q, packed, head_to_kv=h2k, tokens=t, dim_group_size=g)[0]
            assert torch.equal(scores[:, :t], ref)
            ref_idx = torch.empty((qh, k + 1), device=dev, dtype=torch.int64)
            check(lib.popkv_topk(ptr(ref), _lib.F16, qh, t, t, k, t, ptr(ref_idx), k + 1, _stream(dev)))
            torch.cuda.synchronize()
            assert torch.equal(out[:, :k + 1], ref_idx)
        else:
            assert torch.all(out[:, 0] == 0)
        assert torch.all(out[:, k + 1:] == -5)


def _attn_static(q, pk, pv, ck, cv, idx, t, h2k, splits_tokens=256):
    lib, check, ptr = _lib.lib(), _lib.check, _lib.ptr
    dev = q.device
    rows, sel = idx.shape
    kvh = pk.shape[0]
    partials = torch.empty((rows, math.ceil(sel / splits_tokens), 130), device=dev, dtype=torch.float32)
    out = torch.empty((rows, 128), device=dev, dtype=q.dtype)
    check(lib.popkv_attn_partial(ptr(q), _lib.dtype_code(q), 1, rows, 128, ptr(pk), ptr(pv), _lib.dtype_code(pk),
                                 kvh, t, 0, pk.stride(0), pk.stride(1), 0, pv.stride(0), pv.stride(1), ptr(ck),
                                 ptr(cv), ptr(idx), sel, None, ptr(h2k), splits_tokens, ptr(partials),
                                 _stream(dev)))
    check(lib.popkv_attn_merge(ptr(partials), rows, partials.shape[1], 128, ptr(out), _lib.dtype_code(out),
                               _stream(dev)))
    return out


@pytest.mark.parametrize("t", [1, 300, 700, 2049])
def test_attention_dyn_matches_static(cuda_device, t):
    dev = cuda_device
    gen = torch.Generator().manual_seed(t)
    kvh, qh, cap = 2, 8, 2100
    pk = torch.randn(kvh, cap, 128, generator=gen).to(torch.bfloat16).to(dev)
    pv = torch.randn(kvh, cap, 128, generator=gen).to(torch.bfloat16).to(dev)
    ck = torch.randn(kvh, 128, generator=gen).to(torch.bfloat16).to(dev)
    cv = torch.randn(kvh, 128, generator=gen).to(torch.bfloat16).to(dev)
    q = torch.randn(qh, 128, generator=gen).to(torch.bfloat16).to(dev)
    h2k = torch.arange(qh, device=dev) // (qh // kvh)
    lib, check, ptr = _lib.lib(), _lib.check, _lib.ptr
    pos = torch.tensor([t], device=dev, dtype=torch.int64)
    max_tokens = cap - 1
    # Dense: every prefix row plus the current token.
    dense_splits = math.ceil((max_tokens + 1) / 256)
    partials = torch.empty((qh, dense_splits, 130), device=dev, dtype=torch.float32)
    out = torch.empty((qh, 128), device=dev, dtype=torch.bfloat16)
    check(lib.popkv_attn_dyn(ptr(q), _lib.BF16, 1, qh, ptr(pk), ptr(pv), _lib.BF16, kvh, max_tokens, 0,
                             pk.stride(0), pk.stride(1), 0, pv.stride(0), pv.stride(1), ptr(ck), ptr(cv), ptr(pos),
                             None, 0, 0, ptr(h2k), 256, ptr(partials), ptr(out), _lib.BF16, _stream(dev)))
    idx = torch.arange(t + 1, device=dev).expand(qh, t + 1).contiguous()
    ref = _attn_static(q, pk, pv, ck, cv, idx, t, h2k)
    torch.cuda.synchronize()
    assert torch.equal(out, ref)
    # Materialised check of the dense attention itself.
    kk = torch.cat([pk[:, :t], ck[:, None]], 1).float()[h2k]
    vv = torch.cat([pv[:, :t], cv[:, None]], 1).float()[h2k]
    p = torch.softmax((kk @ q.float()[:, :, None])[..., 0] / math.sqrt(128), -1)
    dense = (p[:, :, None] * vv).sum(1)
    assert torch.allclose(out.float(), dense, atol=2e-2, rtol=2e-2)
    # Sparse: selected rows from a top-k-like index list (k_max larger than t for small t).
    k_max = 511
    k = min(k_max, t)
    sel = torch.stack([torch.randperm(t, generator=gen)[:k].sort().values for _ in range(qh)]).to(dev)
    idx = torch.cat([sel, torch.full((qh, 1), t, device=dev)], 1)
    padded = torch.full((qh, k_max + 1), 10**9, device=dev, dtype=torch.int64)
    padded[:, :k + 1] = idx
    sp = torch.empty((qh, math.ceil((k_max + 1) / 256), 130), device=dev, dtype=torch.float32)
    out2 = torch.empty_like(out)
    check(lib.popkv_attn_dyn(ptr(q), _lib.BF16, 1, qh, ptr(pk), ptr(pv), _lib.BF16, kvh, max_tokens, 0,
                             pk.stride(0), pk.stride(1), 0, pv.stride(0), pv.stride(1), ptr(ck), ptr(cv), ptr(pos),
                             ptr(padded), k_max + 1, k_max, ptr(h2k), 256, ptr(sp), ptr(out2), _lib.BF16,
                             _stream(dev)))
    ref2 = _attn_static(q, pk, pv, ck, cv, idx.contiguous(), t, h2k)
    torch.cuda.synchronize()
    assert torch.equal(out2, ref2)


@pytest.mark.parametrize("g,tg", [(16, 128), (64, 64)])
def test_append_kv_dyn_matches_static(cuda_device, g, tg):
    dev = cuda_device
    gen = torch.Generator().manual_seed(tg)
    kvh, cap = 3, 4 * tg
    keys = torch.randn(kvh, cap, 128, generator=gen).to(torch.bfloat16).to(dev)
    vals = torch.randn(kvh, cap, 128, generator=gen).to(torch.bfloat16).to(dev)
    lib, check, ptr = _lib.lib(), _lib.check, _lib.ptr
    for pos in (0, tg - 1, tg, 2 * tg + 5, cap - 1):
        base = _planes(dev, kvh, cap, g, keys[:, :max(pos, 1)].contiguous(), tg)
        newk = torch.randn(kvh, 128, generator=gen).to(torch.bfloat16).to(dev)
        newv = torch.randn(kvh, 128, generator=gen).to(torch.bfloat16).to(dev)
        # Static append.
        k1, v1 = keys.clone(), vals.clone()
        p1 = tuple(x.clone() for x in base)
        sealed = pos - pos % tg
        check(lib.popkv_append_kv(ptr(newk), ptr(newv), _lib.BF16, kvh, 128, ptr(k1), ptr(v1), k1.stride(0),
                                  k1.stride(1), v1.stride(0), v1.stride(1), pos, *(ptr(x) for x in p1), cap,
                                  sealed, tg, g, _stream(dev)))
        # Device-position append, new rows passed in.
        k2, v2 = keys.clone(), vals.clone()
        p2 = tuple(x.clone() for x in base)
        d = torch.tensor([pos], device=dev, dtype=torch.int64)
        check(lib.popkv_append_kv_dyn(ptr(newk), ptr(newv), _lib.BF16, kvh, 128, ptr(k2), ptr(v2), k2.stride(0),
                                      k2.stride(1), v2.stride(0), v2.stride(1), ptr(d), cap, *(ptr(x) for x in p2),
                                      cap, tg, g, _stream(dev)))
        # Device-position append, row already in the cache.
        k3, v3 = keys.clone(), vals.clone()
        k3[:, pos], v3[:, pos] = newk, newv
        p3 = tuple(x.clone() for x in base)
        check(lib.popkv_append_kv_dyn(None, None, _lib.BF16, kvh, 128, ptr(k3), ptr(v3), k3.stride(0),
                                      k3.stride(1), v3.stride(0), v3.stride(1), ptr(d), cap, *(ptr(x) for x in p3),
                                      cap, tg, g, _stream(dev)))
        torch.cuda.synchronize()
        assert torch.equal(k1, k2) and torch.equal(v1, v2) and torch.equal(k1, k3) and torch.equal(v1, v3)
        for a, b, c in zip(p1, p2, p3):
            assert torch.equal(a, b) and torch.equal(a, c)


def test_glue_kernels_follow_eager_ops(cuda_device):
    dev = cuda_device
    gen = torch.Generator().manual_seed(5)
    lib, check, ptr = _lib.lib(), _lib.check, _lib.ptr
    B, H = 3, 4096
    hidden = torch.randn(B, H, generator=gen).to(torch.bfloat16).to(dev)
    delta = torch.randn(B, H, generator=gen).to(torch.bfloat16).to(dev)
    w = (1 + 0.1 * torch.randn(H, generator=gen)).to(torch.bfloat16).to(dev)
    ref_h = hidden + delta
    ref = rms_norm(ref_h, w, 1e-5)
    out = torch.empty_like(hidden)
    h = hidden.clone()
    check(lib.popkv_rms_norm(ptr(delta), ptr(h), ptr(w), B, H, 1e-5, ptr(out), _stream(dev)))
    torch.cuda.synchronize()
    assert torch.equal(h, ref_h)
    diff = (out.float() - ref.float()).abs()
    assert diff.max() <= 2 ** -6 * ref.float().abs().max()  # one bf16 ulp at most (sum order)
    assert (diff == 0).float().mean() > 0.98
    # RoPE + append: bit-exact against the eager rounding.
    cfg = LlamaConfig()
    cos, sin = rope_tables(cfg, 64, dev)
    QH, KVH, cap = 32, 8, 64
    qkv = torch.randn(B, (QH + 2 * KVH) * 128, generator=gen).to(torch.bfloat16).to(dev)
    kc = torch.zeros(B, KVH, cap, 128, device=dev, dtype=torch.bfloat16)
    vc = torch.zeros_like(kc)
    q = torch.empty(B, QH, 128, device=dev, dtype=torch.bfloat16)
    kcur = torch.empty(B, KVH, 128, device=dev, dtype=torch.bfloat16)
    vcur = torch.empty_like(kcur)
    pos = 37
    d = torch.tensor([pos], device=dev, dtype=torch.int64)
    check(lib.popkv_rope_append(ptr(qkv), B, QH, KVH, 128, ptr(cos), ptr(sin), ptr(d), cap - 1, ptr(q), ptr(kcur),
                                ptr(vcur), ptr(kc), ptr(vc), kc.stride(0), kc.stride(1), kc.stride(2), vc.stride(0),
                                vc.stride(1), vc.stride(2), _stream(dev)))
    torch.cuda.synchronize()
    x = qkv.view(B, QH + 2 * KVH, 128)
    rq = apply_rope(x[:, :QH], cos[pos:pos + 1], sin[pos:pos + 1])
    rk = apply_rope(x[:, QH:QH + KVH], cos[pos:pos + 1], sin[pos:pos + 1])
    assert torch.equal(q, rq) and torch.equal(kcur, rk) and torch.equal(vcur, x[:, QH + KVH:])
    assert torch.equal(kc[:, :, pos], rk) and torch.equal(vc[:, :, pos], x[:, QH + KVH:])
    assert torch.count_nonzero(kc[:, :, :pos]) == 0 and torch.count_nonzero(kc[:, :, pos + 1:]) == 0
    # SiLU * up.
    I = 14336
    gu = torch.randn(B, 2 * I, generator=gen).to(torch.bfloat16).to(dev) * 3
    act = torch.empty(B, I, device=dev, dtype=torch.bfloat16)
    check(lib.popkv_silu_mul(ptr(gu), B, I, ptr(act), _stream(dev)))
    torch.cuda.synchronize()
    ref = F.silu(gu[:, :I]) * gu[:, I:]
    diff = (act.float() - ref.float()).abs()
    assert (diff == 0).float().mean() > 0.999
    assert torch.allclose(act.float(), ref.float(), rtol=2 ** -7, atol=0)


class _StaticLengthDecoder(LlamaSparseDecoder):
    """The same loop run eagerly with the static-length kernels and a Python-integer
    cache length per call, as the reference decoder launches its stages
    (popkv.py:1076-1115, append afterwards as popkv.py:884-972)."""

    def _attention(self, layer, s, after_score=None):
        lib, check, ptr = _lib.lib(), _lib.check, _lib.ptr
        t = int(self.position.item())
        B, rows = self.batch, self.batch * self.qh
        kc, vc = self.k_cache[layer], self.v_cache[layer]
        dev = self.device
        if layer in self.packed:
            sign, mag, low, delta = self.packed[layer]
            k = min(self.k_max, t)
            idx = torch.empty((rows, k + 1), device=dev, dtype=torch.int64)
            if t > 0:
                scores = torch.empty((rows, t), device=dev, dtype=torch.float16)
                check(lib.popkv_score(ptr(self.q), _lib.BF16, 1, rows, 128, ptr(sign), ptr(mag), ptr(low),
                                      ptr(delta), B * self.kvh, self.meta_capacity, ptr(self.head_to_kv), t,
                                      self.g, ptr(scores), _lib.F16, s))
                check(lib.popkv_topk(ptr(scores), _lib.F16, rows, t, t, k, t, ptr(idx), k + 1, s))
            else:
                idx.fill_(0)
        else:
            idx = torch.arange(t + 1, device=dev).expand(rows, t + 1).contiguous()
        sel = idx.shape[1]
        partials = torch.empty((rows, math.ceil(sel / self.split_tokens), 130), device=dev, dtype=torch.float32)
        check(lib.popkv_attn_partial(ptr(self.q), _lib.BF16, 1, rows, 128, ptr(kc), ptr(vc), _lib.BF16,
                                     B * self.kvh, t, 0, kc.stride(1), kc.stride(2), 0, vc.stride(1), vc.stride(2),
                                     ptr(self.k_cur), ptr(self.v_cur), ptr(idx), sel, None, ptr(self.head_to_kv),
                                     self.split_tokens, ptr(partials), s))
        check(lib.popkv_attn_merge(ptr(partials), rows, partials.shape[1], 128, ptr(self.attn), _lib.BF16, s))
        if layer in self.packed:
            sign, mag, low, delta = self.packed[layer]
            check(lib.popkv_append_kv(ptr(self.k_cur), ptr(self.v_cur), _lib.BF16, B * self.kvh, 128, ptr(kc),
                                      ptr(vc), kc.stride(1), kc.stride(2), vc.stride(1), vc.stride(2), t,
                                      ptr(sign), ptr(mag), ptr(low), ptr(delta), self.meta_capacity,
                                      t - t % self.tg, self.tg, self.g, s))


def _prefix(cfg, batch, T, seed=3):
    gen = torch.Generator().manual_seed(seed)
    return torch.randint(0, cfg.vocab_size, (batch, T), generator=gen)


@pytest.mark.parametrize("method,batch,T,steps", [("popkv-s", 1, 250, 24), ("popkv-q", 2, 200, 12),
                                                  ("full", 1, 100, 6), ("popkv-s", 5, 120, 4)])
def test_graph_decoder_matches_static_length_loop(cuda_device, method, batch, T, steps):
    weights = LlamaWeights.random(TINY, device=cuda_device, seed=1, std=0.05)
    tg = {"popkv-s": 64, "popkv-q": 128, "full": 32}[method]
    g = {"popkv-s": 64, "popkv-q": 16, "full": 32}[method]
    retrieval = RetrievalConfig(budget=64, group_size=tg, dim_group_size=g)
    ids = _prefix(TINY, batch, T)
    graph = LlamaSparseDecoder(weights, method=method, retrieval=retrieval, batch=batch, max_context=T + steps + 1)
    static = _StaticLengthDecoder(weights, method=method, retrieval=retrieval, batch=batch,
                                  max_context=T + steps + 1, use_graph=False)
    first_a = graph.prefill(ids)
    first_b = static.prefill(ids)
    assert torch.equal(first_a, first_b)
    for l in graph.packed:
        for a, b in zip(graph.packed[l], static.packed[l]):
            assert torch.equal(a, b)
    for step in range(steps):
        la = graph.decode().clone()
        lb = static.decode().clone()
        assert torch.equal(la, lb), f"step {step}: logits differ"
        assert torch.equal(graph.token, static.token)
    assert int(graph.position.item()) == T + steps
    for l in range(TINY.num_hidden_layers):
        assert torch.equal(graph.k_cache[l], static.k_cache[l])
        assert torch.equal(graph.v_cache[l], static.v_cache[l])
    for l in graph.packed:
        for a, b in zip(graph.packed[l], static.packed[l]):
            assert torch.equal(a, b)
    graph.close()


def test_generate_replays_without_host_round_trips(cuda_device):
    weights = LlamaWeights.random(TINY, device=cuda_device, seed=2, std=0.05)
    ids = _prefix(TINY, 1, 150, seed=9)
    a = LlamaSparseDecoder(weights, method="popkv-s", retrieval=RetrievalConfig(budget=64, group_size=64,
                                                                                dim_group_size=64),
                           max_context=200)
    b = LlamaSparseDecoder(weights, method="popkv-s", retrieval=RetrievalConfig(budget=64, group_size=64,
                                                                                dim_group_size=64),
                           max_context=200, use_graph=False)
    a.prefill(ids)
    b.prefill(ids)
    out = a.generate(20)
    ref = torch.stack([b.decode().argmax(-1).cpu() for _ in range(20)], 1)
    assert torch.equal(out, ref)
    with pytest.raises(RuntimeError, match="capacity"):
        a.generate(100)


def test_dense_decode_matches_transformers_llama(cuda_device):
    """method="full" against transformers' LlamaForCausalLM on the same weights.

    Both run in bf16 with different rounding paths, so the yardstick is an fp32
    run of the transformers model: our logits must be no further from it than
    twice the bf16 transformers run is.
    """
    import copy
    transformers = pytest.importorskip("transformers")
    cfg = transformers.LlamaConfig(hidden_size=1024, intermediate_size=2048, num_attention_heads=8,
                                   num_key_value_heads=2, head_dim=128, num_hidden_layers=3, vocab_size=2000,
                                   rope_theta=500000.0, rms_norm_eps=1e-5, max_position_embeddings=4096,
                                   tie_word_embeddings=False)
    torch.manual_seed(0)
    model = transformers.LlamaForCausalLM(cfg).eval()
    for p in model.parameters():
        if p.ndim == 2:
            torch.nn.init.normal_(p, 0.0, 0.02)
    model = model.to(device=cuda_device, dtype=torch.bfloat16)
    model32 = copy.deepcopy(model).float()
    inv_freq = 1.0 / (500000.0 ** (torch.arange(0, 128, 2, device=cuda_device).float() / 128))
    # Keep the rotary inverse frequencies in fp32, as a bf16 checkpoint load does.
    model.model.rotary_emb.inv_freq = inv_freq
    model32.model.rotary_emb.inv_freq = inv_freq
    weights = LlamaWeights.from_module(model)
    T, steps = 120, 4
    ids = _prefix(weights.config, 1, T, seed=4)
    dec = LlamaSparseDecoder(weights, method="full", max_context=T + steps + 1)
    dec.prefill(ids)
    seq = ids[0].tolist()
    for _ in range(steps):
        seq.append(int(dec.token.item()))
        logits = dec.decode()[0].clone()
        with torch.no_grad():
            x = torch.tensor([seq], device=cuda_device)
            ref32 = model32(input_ids=x).logits[0, -1].float()
            hf16 = model(input_ids=x).logits[0, -1].float()
        err = (logits - ref32).norm() / ref32.norm()
        hf_err = (hf16 - ref32).norm() / ref32.norm()
        assert err <= max(2 * hf_err, 5e-3), (err, hf_err)
        assert (logits.argmax() == ref32.argmax()) or (ref32.max() - ref32[logits.argmax()] < 0.05)
    dec.close()


def test_fused_products_match_cublas_path(cuda_device):
    """The weight-streaming products (batch <= 4) against the cuBLAS + separate-kernel step.

    Dense layers only: with sparse layers a last-bit difference in q can swap a
    near-tied token in or out of the top-k, which says nothing about the
    products (the PopKV layers are pinned bit-exact above).
    """
    weights = LlamaWeights.random(TINY, device=cuda_device, seed=7, std=0.02)
    ids = _prefix(TINY, 2, 180, seed=11)
    fused = LlamaSparseDecoder(weights, method="full", batch=2, max_context=200)
    plain = LlamaSparseDecoder(weights, method="full", batch=2, max_context=200)
    plain.fused = False
    plain.capture()
    assert fused.fused
    fused.prefill(ids)
    plain.prefill(ids)
    for _ in range(8):
        tok = fused.token.clone()
        plain.token.copy_(tok)
        a = fused.decode().clone()
        b = plain.decode().clone()
        # Different fp32 summation orders round some bf16 activations the other
        # way; through four layers that leaves ~0.5% relative logit differences.
        rel = (a - b).norm() / b.norm()
        assert rel < 1e-2, rel
        # Greedy choices agree unless the top two logits are within rounding.
        top2 = b.topk(2, -1).values
        agree = fused.token == plain.token
        assert bool((agree | (top2[:, 0] - top2[:, 1] < 0.05)).all())
    assert int(fused.position.item()) == int(plain.position.item()) == 188


def test_lm_head_argmax_ties_and_state(cuda_device):
    """Greedy choice: largest bf16 logit, lowest index among equals; state left zeroed."""
    dev = cuda_device
    lib, check, ptr = _lib.lib(), _lib.check, _lib.ptr
    V, H = 5000, 256
    w = torch.zeros(V, H, device=dev, dtype=torch.bfloat16)
    w[[17, 4000, 4999], 0] = 1.0  # three equal maxima
    w[[3, 9], 0] = -2.0
    hidden = torch.zeros(2, H, device=dev, dtype=torch.bfloat16)
    hidden[:, 0] = 1.0
    hidden[1, 0] = -1.0  # row 1: maxima at the -2 rows... ties at 3 and 9
    norm_w = torch.ones(H, device=dev, dtype=torch.bfloat16)
    logits = torch.empty(2, V, device=dev, dtype=torch.bfloat16)
    state = torch.zeros(3, device=dev, dtype=torch.int64)
    tok = torch.full((2,), -1, device=dev, dtype=torch.int64)
    pos = torch.tensor([41], device=dev, dtype=torch.int64)
    for _ in range(2):
        check(lib.popkv_norm_lm_head_argmax(ptr(w), V, H, 2, ptr(hidden), None, ptr(norm_w), 1e-5, None,
                                            ptr(logits), ptr(state), ptr(tok), ptr(pos), _stream(dev)))
    torch.cuda.synchronize()
    assert tok.tolist() == [17, 3]
    assert torch.equal(tok, logits.float().argmax(-1))
    assert int(pos.item()) == 43 and int(state.abs().sum().item()) == 0


def _ulps_bf16(a: torch.Tensor, b: torch.Tensor) -> torch.Tensor:
    """Distance in bf16 units in the last place (same-sign values)."""
    ai = a.view(torch.int16).to(torch.int32)
    bi = b.view(torch.int16).to(torch.int32)
    return (ai - bi).abs()


@pytest.mark.parametrize("batch", [1, 2, 4])
def test_weight_streaming_products_match_fp32_matmul(cuda_device, batch):
    """Each product equals fp32 matmul rounded to bf16, up to one bf16 ulp (summation order)."""
    dev = cuda_device
    gen = torch.Generator().manual_seed(batch)
    lib, check, ptr = _lib.lib(), _lib.check, _lib.ptr
    H, I, QH, KVH = 1024, 1536, 8, 2
    x = torch.randn(batch, H, generator=gen).to(torch.bfloat16).to(dev)
    w = (0.05 * torch.randn(3000, H, generator=gen)).to(torch.bfloat16).to(dev)
    out = torch.empty(batch, 3000, device=dev, dtype=torch.bfloat16)
    check(lib.popkv_linear(ptr(w), 3000, H, ptr(x), batch, ptr(out), 3000, _stream(dev)))
    ref = (x.float() @ w.float().t()).to(torch.bfloat16)
    torch.cuda.synchronize()
    d = _ulps_bf16(out, ref)
    assert int(d.max()) <= 1 and float((d == 0).float().mean()) > 0.97
    # Norm prologue (residual add) + SwiGLU epilogue.
    hidden = torch.randn(batch, H, generator=gen).to(torch.bfloat16).to(dev)
    delta = torch.randn(batch, H, generator=gen).to(torch.bfloat16).to(dev)
    nw = (1 + 0.1 * torch.randn(H, generator=gen)).to(torch.bfloat16).to(dev)
    gu = (0.05 * torch.randn(2 * I, H, generator=gen)).to(torch.bfloat16).to(dev)
    act = torch.empty(batch, I, device=dev, dtype=torch.bfloat16)
    hout = torch.empty_like(hidden)
    check(lib.popkv_norm_gate_up_swiglu(ptr(gu), I, H, batch, ptr(hidden), ptr(delta), ptr(nw), 1e-5, ptr(hout),
                                        ptr(act), _stream(dev)))
    h = hidden + delta
    xn = rms_norm(h, nw, 1e-5)
    y = (xn.float() @ gu.float().t()).to(torch.bfloat16)
    ref_act = F.silu(y[:, :I]) * y[:, I:]
    torch.cuda.synchronize()
    assert torch.equal(hout, h)
    close = (act.float() - ref_act.float()).abs() <= 2 ** -6 * ref_act.float().abs() + 1e-6
    assert float(close.float().mean()) > 0.98
    # Norm prologue (embedding rows) + RoPE epilogue + KV append.
    cfg = LlamaConfig(hidden_size=H, num_attention_heads=QH, num_key_value_heads=KVH, intermediate_size=I,
                      vocab_size=100, num_hidden_layers=1)
    cap = 50
    cos, sin = rope_tables(cfg, cap, dev)
    wqkv = (0.05 * torch.randn((QH + 2 * KVH) * 128, H, generator=gen)).to(torch.bfloat16).to(dev)
    embed = torch.randn(100, H, generator=gen).to(torch.bfloat16).to(dev)
    token = torch.randint(0, 100, (batch,), generator=gen).to(dev)
    q = torch.empty(batch, QH, 128, device=dev, dtype=torch.bfloat16)
    kcur = torch.empty(batch, KVH, 128, device=dev, dtype=torch.bfloat16)
    vcur = torch.empty_like(kcur)
    kc = torch.zeros(batch, KVH, cap, 128, device=dev, dtype=torch.bfloat16)
    vc = torch.zeros_like(kc)
    pos = torch.tensor([33], device=dev, dtype=torch.int64)
    hout2 = torch.empty_like(hidden)
    check(lib.popkv_norm_qkv_rope(ptr(wqkv), QH, KVH, H, batch, None, None, ptr(embed), ptr(token), ptr(nw), 1e-5,
                                  ptr(hout2), ptr(cos), ptr(sin), ptr(pos), cap - 1, ptr(q), ptr(kcur), ptr(vcur),
                                  ptr(kc), ptr(vc), kc.stride(0), kc.stride(1), kc.stride(2), vc.stride(0),
                                  vc.stride(1), vc.stride(2), _stream(dev)))
    h2 = embed[token]
    y = (rms_norm(h2, nw, 1e-5).float() @ wqkv.float().t()).to(torch.bfloat16).view(batch, QH + 2 * KVH, 128)
    rq = apply_rope(y[:, :QH], cos[33:34], sin[33:34])
    rk = apply_rope(y[:, QH:QH + KVH], cos[33:34], sin[33:34])
    torch.cuda.synchronize()
    assert torch.equal(hout2, h2)
    for got, want in ((q, rq), (kcur, rk), (vcur, y[:, QH + KVH:]), (kc[:, :, 33], rk), (vc[:, :, 33], y[:, QH + KVH:])):
        close = (got.float() - want.float()).abs() <= 2 ** -6 * want.float().abs() + 1e-3
        assert float(close.float().mean()) > 0.98
    assert torch.count_nonzero(kc[:, :, :33]) == 0 and torch.count_nonzero(kc[:, :, 34:]) == 0


def test_topk_dyn_beyond_128k_tokens(cuda_device):
    """Rows longer than 131072 keys (config 4's 128K context plus decoded tokens)."""
    dev = cuda_device
    lib, check, ptr = _lib.lib(), _lib.check, _lib.ptr
    gen = torch.Generator().manual_seed(3)
    rows, max_tokens, k_max = 6, 131072 + 700, 4095
    stride = (max_tokens + 7) // 8 * 8
    scores = (torch.randn(rows, stride, generator=gen) * 4).to(torch.float16).to(dev)
    scores[:, 5000:5100] = 7.5  # a block of ties
    for t in (max_tokens, 131072 + 3, 90000):
        pos = torch.tensor([t], device=dev, dtype=torch.int64)
        out = torch.empty(rows, k_max + 1, device=dev, dtype=torch.int64)
        check(lib.popkv_topk_dyn(ptr(scores), rows, ptr(pos), max_tokens, stride, k_max, ptr(out), k_max + 1,
                                 _stream(dev)))
        ref = torch.empty_like(out)
        check(lib.popkv_topk(ptr(scores), _lib.F16, rows, t, stride, k_max, t, ptr(ref), k_max + 1, _stream(dev)))
        torch.cuda.synchronize()
        assert torch.equal(out, ref)
        # Selection semantics: every chosen score >= every unchosen one.
        sel = out[:, :k_max]
        chosen = torch.gather(scores[:, :t].float(), 1, sel)
        mask = torch.ones(rows, t, dtype=torch.bool, device=dev)
        mask.scatter_(1, sel, False)
        rest = scores[:, :t].float().masked_fill(~mask, float("-inf"))
        assert torch.all(chosen.min(1).values >= rest.max(1).values)
        assert torch.all(out[:, k_max] == t)


@pytest.mark.parametrize("method", ["popkv-s", "full"])
def test_layer_tail_matches_separate_products(cuda_device, method):
    """The persistent layer tail (batch 1) reproduces the separate products bit for bit."""
    import ctypes
    weights = LlamaWeights.random(TINY, device=cuda_device, seed=5, std=0.05)
    retrieval = RetrievalConfig(budget=64, group_size=64, dim_group_size=64)
    ids = _prefix(TINY, 1, 150, seed=2)
    a = LlamaSparseDecoder(weights, method=method, retrieval=retrieval, max_context=180)
    b = LlamaSparseDecoder(weights, method=method, retrieval=retrieval, max_context=180)
    a.tail = True
    a.capture()
    assert not b.tail
    a.prefill(ids)
    b.prefill(ids)
    for _ in range(12):
        la, lb = a.decode().clone(), b.decode().clone()
        assert torch.equal(la, lb)
        assert torch.equal(a.token, b.token)
    assert int(a.position.item()) == int(b.position.item()) == 162
    for l in range(TINY.num_hidden_layers):
        assert torch.equal(a.k_cache[l], b.k_cache[l]) and torch.equal(a.v_cache[l], b.v_cache[l])
    for name in ("popkv_layer_tail_timeouts", "popkv_gemv_timeouts"):
        count = ctypes.c_uint32(99)
        _lib.check(getattr(_lib.lib(), name)(ctypes.byref(count)))
        assert count.value == 0, name


def test_synthetic_prefill_fills_caches_and_planes(cuda_device):
    """prefill_synthetic writes K/V rows [0, T) of every layer, packs the sparse layers'
    planes exactly as popkv_pack does from those rows, and leaves a valid next token."""
    weights = LlamaWeights.random(TINY, device=cuda_device, seed=4, std=0.02)
    retrieval = RetrievalConfig(budget=64, group_size=64, dim_group_size=64)
    dec = LlamaSparseDecoder(weights, method="popkv-s", retrieval=retrieval, batch=2, max_context=300)
    T = 250
    first = dec.prefill_synthetic(T, seed=3)
    assert int(dec.position.item()) == T
    assert torch.all((first >= 0) & (first < TINY.vocab_size))
    for l in range(TINY.num_hidden_layers):
        kc, vc = dec.k_cache[l], dec.v_cache[l]
        assert torch.count_nonzero(kc[:, :, T:]) == 0 and torch.count_nonzero(vc[:, :, T:]) == 0
        assert bool((kc[:, :, :T].abs().sum(-1) > 0).all()) and bool((vc[:, :, :T].abs().sum(-1) > 0).all())
    for l, planes in dec.packed.items():
        keys = dec.k_cache[l].reshape(-1, dec.max_context, 128)[:, :T].contiguous()
        want = popkv_cuda.pack_keys(keys, token_capacity=dec.meta_capacity, token_group_size=64, dim_group_size=64)
        for a, b in zip(planes, want):
            assert torch.equal(a[:, :T], b[:, :T])
    for _ in range(3):  # decodes from there
        logits = dec.decode()
        assert torch.isfinite(logits).all()
    dec.close()
