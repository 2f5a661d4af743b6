"""Full-model greedy decode of a Llama-shaped model around the PopKV retrieval path.

The reference decodes one token per ``LlamaSparseDecoder.decode`` call
(popkv.py:988-1115): per layer, RMSNorm, q/k/v projections, rotary embedding,
full attention on the dense layers (``full_layers``, layers 0-1) or the PopKV
branch (query encode, popcount score, top-k + current slot, split attention and
merge) on the rest, output projection and the MLP; then the final norm and the
LM head.  After each call the caller appends the token's keys and values
(``append_kv``, popkv.py:965-972) and re-encodes the open token group
(``append_retrieval_caches``, popkv.py:884-943).  Every stage is an eager launch
with the cache length as a Python integer.

``LlamaSparseDecoder`` here runs the same computation as ONE CUDA graph per
token, replayed for every decode step:

* the cache length lives in device memory (``position``); the retrieval and
  attention kernels read it at run time (the ``*_dyn`` entry points), and the
  step advances it, so the graph captured once serves every step;
* the step appends the token's keys/values (``popkv_rope_append``) and
  re-encodes the open group of every sparse layer (``popkv_append_kv_dyn``)
  inside the graph, after that layer's score (the reference's order: decode,
  then append);
* greedy selection (argmax) feeds the next step's token id on the device, so a
  run of ``generate`` steps needs no host round trip;
* for batch <= 4 the projections are the library's weight-streaming
  products (fused q|k|v and gate|up weights) with the element-wise work in
  their prologues and epilogues: residual add + RMSNorm (and the embedding
  lookup of layer 0), RoPE + KV append, SwiGLU, and the LM head's greedy
  argmax + position advance -- four launches per layer besides attention;
  larger batches use cuBLAS GEMMs and separate RMSNorm / RoPE / SwiGLU kernels;
* the dense layers use the split-attention kernel over every cached token.

The prefill (``prefill``) is plain PyTorch (causal SDPA); it is not on the
decode path.  Weights are random (``LlamaWeights.random``) or taken from a
``LlamaForCausalLM``-shaped module tree (``LlamaWeights.from_module``).
"""
from __future__ import annotations

import ctypes
import math
from dataclasses import dataclass

import torch
import torch.nn.functional as F

from . import _lib
from .popkv import POPKV_PRESETS, RetrievalConfig


@dataclass(frozen=True)
class LlamaConfig:
    """Shape of a Llama decoder (defaults: Llama-3.1-8B)."""

    hidden_size: int = 4096
    num_attention_heads: int = 32
    num_key_value_heads: int = 8
    head_dim: int = 128
    intermediate_size: int = 14336
    vocab_size: int = 128256
    num_hidden_layers: int = 32
    rope_theta: float = 500000.0
    rms_norm_eps: float = 1e-5

    def validate(self) -> None:
        if self.head_dim != 128:
            raise ValueError("the decode kernels need head_dim 128")
        if self.num_attention_heads % self.num_key_value_heads:
            raise ValueError("query heads must be a multiple of KV heads")
        if self.num_attention_heads // self.num_key_value_heads > 4:
            raise ValueError("at most 4 query heads per KV head")
        if self.hidden_size % 8 or self.intermediate_size % 8:
            raise ValueError("hidden and intermediate sizes must be multiples of 8")


LLAMA31_8B = LlamaConfig()


@dataclass
class LayerWeights:
    input_norm: torch.Tensor   # [H]
    qkv: torch.Tensor          # [(QH + 2 KVH) * D, H]: q_proj | k_proj | v_proj rows
    o: torch.Tensor            # [H, QH * D]
    post_norm: torch.Tensor    # [H]
    gate_up: torch.Tensor      # [2 I, H]: gate_proj | up_proj rows
    down: torch.Tensor         # [H, I]


@dataclass
class LlamaWeights:
    config: LlamaConfig
    embed: torch.Tensor        # [V, H]
    layers: list[LayerWeights]
    norm: torch.Tensor         # [H]
    lm_head: torch.Tensor      # [V, H]

    @classmethod
    def random(cls, config: LlamaConfig = LLAMA31_8B, *, device="cuda", seed: int = 0,
               std: float = 0.02, dtype=torch.bfloat16) -> "LlamaWeights":
        """Random-init weights: N(0, std) matrices (the Llama initializer), unit norms."""
        config.validate()
        device = torch.device(device)
        gen = torch.Generator(device=device)
        gen.manual_seed(seed)
        H, I = config.hidden_size, config.intermediate_size
        D, QH, KVH = config.head_dim, config.num_attention_heads, config.num_key_value_heads

        def mat(rows, cols):
            w = torch.empty((rows, cols), device=device, dtype=dtype)
            return w.normal_(0.0, std, generator=gen)

        def ones(n):
            return torch.ones(n, device=device, dtype=dtype)

        layers = [LayerWeights(ones(H), mat((QH + 2 * KVH) * D, H), mat(H, QH * D), ones(H),
                               mat(2 * I, H), mat(H, I)) for _ in range(config.num_hidden_layers)]
        return cls(config, mat(config.vocab_size, H), layers, ones(H), mat(config.vocab_size, H))

    @classmethod
    def from_module(cls, model, *, device=None, dtype=torch.bfloat16) -> "LlamaWeights":
        """Weights of a LlamaForCausalLM-shaped module tree (model.model.layers[i].self_attn.q_proj ...)."""
        cfg = model.config
        rope = getattr(cfg, "rope_parameters", None) or getattr(cfg, "rope_scaling", None) or {}
        if rope.get("rope_type", rope.get("type", "default")) != "default":
            raise ValueError("only the default rotary embedding (no frequency scaling) is supported")
        theta = getattr(cfg, "rope_theta", None) or rope.get("rope_theta", 10000.0)
        config = LlamaConfig(
            hidden_size=int(cfg.hidden_size), num_attention_heads=int(cfg.num_attention_heads),
            num_key_value_heads=int(getattr(cfg, "num_key_value_heads", cfg.num_attention_heads)),
            head_dim=int(getattr(cfg, "head_dim", None) or cfg.hidden_size // cfg.num_attention_heads),
            intermediate_size=int(cfg.intermediate_size), vocab_size=int(cfg.vocab_size),
            num_hidden_layers=int(cfg.num_hidden_layers), rope_theta=float(theta),
            rms_norm_eps=float(cfg.rms_norm_eps))
        config.validate()
        backbone = model.model

        def t(w):
            w = w.detach()
            return w.to(device=device or w.device, dtype=dtype).contiguous()

        layers = []
        for layer in backbone.layers:
            a, m = layer.self_attn, layer.mlp
            layers.append(LayerWeights(
                t(layer.input_layernorm.weight),
                t(torch.cat([a.q_proj.weight, a.k_proj.weight, a.v_proj.weight], 0)),
                t(a.o_proj.weight), t(layer.post_attention_layernorm.weight),
                t(torch.cat([m.gate_proj.weight, m.up_proj.weight], 0)), t(m.down_proj.weight)))
        return cls(config, t(backbone.embed_tokens.weight), layers, t(backbone.norm.weight),
                   t(model.lm_head.weight))

    def bytes_per_token(self) -> int:
        """Weight bytes one batch-1 decode step streams from HBM (all matrices except the embedding)."""
        total = self.lm_head.numel() * self.lm_head.element_size() + self.norm.numel() * 2
        for layer in self.layers:
            for w in (layer.input_norm, layer.qkv, layer.o, layer.post_norm, layer.gate_up, layer.down):
                total += w.numel() * w.element_size()
        return int(total)


def rope_tables(config: LlamaConfig, positions: int, device, dtype=torch.bfloat16):
    """cos/sin [positions, head_dim / 2] as the reference model's rotary embedding makes them.

    transformers' LlamaRotaryEmbedding (default rope type): inv_freq =
    1 / theta^(2i / D) in fp32, freqs = position * inv_freq in fp32, cos/sin in
    fp32 cast to the activation dtype (both halves of the head share them).
    """
    D = config.head_dim
    inv_freq = 1.0 / (config.rope_theta ** (torch.arange(0, D, 2, dtype=torch.int64, device=device).float() / D))
    pos = torch.arange(positions, device=device, dtype=torch.float32)
    freqs = pos[:, None] * inv_freq[None, :]
    return freqs.cos().to(dtype).contiguous(), freqs.sin().to(dtype).contiguous()


def rms_norm(x: torch.Tensor, weight: torch.Tensor, eps: float) -> torch.Tensor:
    """LlamaRMSNorm in eager PyTorch (fp32 statistics, bf16 output)."""
    h = x.float()
    h = h * torch.rsqrt(h.pow(2).mean(-1, keepdim=True) + eps)
    return weight * h.to(x.dtype)


def apply_rope(x: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor) -> torch.Tensor:
    """x [..., T, D] with cos/sin [T, D/2]: x*cos + rotate_half(x)*sin (popkv.py:740-749)."""
    cos2, sin2 = torch.cat([cos, cos], -1), torch.cat([sin, sin], -1)
    half = x.shape[-1] // 2
    rotated = torch.cat([-x[..., half:], x[..., :half]], -1)
    return x * cos2 + rotated * sin2


def ctypes_stream(stream: torch.cuda.Stream):
    return ctypes.c_void_p(stream.cuda_stream)


DECODE_METHODS = ("full",) + tuple(POPKV_PRESETS)


class LlamaSparseDecoder:
    """Graph-replayed greedy decode of a Llama-shaped model with PopKV sparse layers.

    Args:
        weights: the model (all heads; a sharded decoder keeps the full weights
            for the prefill and slices its heads' q/k/v rows for the decode).
        method: "full" (every layer dense) or a PopKV preset ("popkv-q",
            "popkv-s", "popkv-normal"; popkv.py:20-24), with the dense layers of
            ``retrieval.full_layers``.
        retrieval: budget, token/dim group sizes and dense layers; default the
            preset's sizes with budget 4096 and layers 0-1 dense.
        batch: sequences decoded together (all of one length).
        max_context: KV-cache rows per sequence (prefix + decoded tokens).
        rank, world, group: KV-head shard of a ``world``-GPU run (one process per
            GPU): this rank owns KV heads [rank*KVH/world, (rank+1)*KVH/world) and
            their query heads; the attention outputs are all-gathered (NCCL) per
            layer into the replicated output projection and MLP.
        mlp_parallel: "replicated" (the plan above: every rank streams the whole
            output projection and MLP) or "tensor" (batch <= 4, several ranks):
            o_proj and down_proj keep this rank's input columns (its heads, its
            1/world of the intermediate dims), gate/up its intermediate rows;
            the two partial outputs are summed with an all-reduce each layer
            instead of all-gathering the attention rows.  Each rank then
            streams 1/world of those weights.  The LM head stays replicated.
        all_reduce: how tensor mode sums the partial outputs: "peer" (one
            popkv_peer_sum launch over NVLink peer memory, fp32 sum in rank order)
            or "nccl" (torch.distributed.all_reduce).
    """

    def __init__(self, weights: LlamaWeights, *, method: str = "popkv-s",
                 retrieval: RetrievalConfig | None = None, batch: int = 1, max_context: int,
                 split_tokens: int = 256, rank: int = 0, world: int = 1, group=None,
                 use_graph: bool = True, mlp_parallel: str = "replicated",
                 all_reduce: str = "peer") -> None:
        if method not in DECODE_METHODS:
            raise ValueError(f"method must be one of {DECODE_METHODS}")
        cfg = weights.config
        cfg.validate()
        if retrieval is None:
            tg, g = POPKV_PRESETS.get(method, (32, 32))
            retrieval = RetrievalConfig(budget=4096, group_size=tg, dim_group_size=g)
        retrieval.validate()
        if retrieval.group_size > 128:
            raise ValueError("the in-graph append re-encodes token groups of at most 128")
        if cfg.num_key_value_heads % world:
            raise ValueError("KV heads must divide evenly over the ranks")
        if mlp_parallel not in ("replicated", "tensor"):
            raise ValueError("mlp_parallel must be 'replicated' or 'tensor'")
        self.tensor_mlp = mlp_parallel == "tensor" and world > 1
        if all_reduce not in ("peer", "nccl"):
            raise ValueError("all_reduce must be 'peer' or 'nccl'")
        if self.tensor_mlp and (batch > 4 or cfg.intermediate_size % (8 * world)):
            raise ValueError("mlp_parallel='tensor' needs batch <= 4 and intermediate dims divisible by 8 * world")
        self.w, self.cfg, self.method, self.retrieval = weights, cfg, method, retrieval
        self.device = weights.embed.device
        self.batch, self.max_context = int(batch), int(max_context)
        self.rank, self.world, self.group = int(rank), int(world), group
        self.split_tokens = int(split_tokens)
        B, H, I, D = self.batch, cfg.hidden_size, cfg.intermediate_size, cfg.head_dim
        QH, KVH = cfg.num_attention_heads, cfg.num_key_value_heads
        self.kvh, self.qh = KVH // world, QH // world
        self.group_heads = QH // KVH
        L = cfg.num_hidden_layers
        if method == "full":
            self.sparse_layers = ()
        else:
            self.sparse_layers = tuple(l for l in range(L) if l not in retrieval.full_layers)
        self.tg, self.g = retrieval.group_size, retrieval.dim_group_size
        self.budget = retrieval.budget
        dev = self.device
        cap = self.max_context
        if cap < 2:
            raise ValueError("max_context must hold at least one prefix and one decoded token")
        self.meta_capacity = math.ceil(cap / self.tg) * self.tg
        # Step state on the device.
        self.position = torch.zeros(1, device=dev, dtype=torch.int64)
        self.token = torch.zeros(B, device=dev, dtype=torch.int64)
        self.next_token = torch.zeros(B, device=dev, dtype=torch.int64)
        # Activations.
        bf = torch.bfloat16
        self.hidden = torch.zeros((B, H), device=dev, dtype=bf)
        self.hidden_b = torch.zeros((B, H), device=dev, dtype=bf)  # ping-pong partner (fused path)
        self.x = torch.zeros((B, H), device=dev, dtype=bf)
        # Fused weight-streaming products (batch <= 4); cuBLAS + separate kernels otherwise.
        self.fused = B <= 4
        # Batch 1, opt-in: each layer's o_proj .. next q/k/v as one persistent
        # launch (bit-identical results; see layer_tail).
        self.tail = False
        self.tail_barrier = torch.zeros(2, device=dev, dtype=torch.int32)
        self.argmax_state = torch.zeros(B + 1, device=dev, dtype=torch.int64)
        self.qkv = torch.zeros((B, (self.qh + 2 * self.kvh) * D), device=dev, dtype=bf)
        self.q = torch.zeros((B, self.qh, D), device=dev, dtype=bf)
        self.k_cur = torch.zeros((B, self.kvh, D), device=dev, dtype=bf)
        self.v_cur = torch.zeros((B, self.kvh, D), device=dev, dtype=bf)
        self.attn = torch.zeros((B, self.qh, D), device=dev, dtype=bf)
        self.attn_full = self.attn if world == 1 else torch.zeros((B, QH, D), device=dev, dtype=bf)
        self._gathered = None if world == 1 else torch.zeros((world, B, self.qh, D), device=dev, dtype=bf)
        self.o = torch.zeros((B, H), device=dev, dtype=bf)
        self.gate_up = torch.zeros((B, 2 * I), device=dev, dtype=bf)
        self.inter_local = I // world if self.tensor_mlp else I
        self.act = torch.zeros((B, self.inter_local), device=dev, dtype=bf)
        self.down = torch.zeros((B, H), device=dev, dtype=bf)
        # Tensor mode: the partial products' all-reduce over peer memory.
        self._peer_sum = None
        if self.tensor_mlp and all_reduce == "peer":
            from .sharding import PeerSum
            self._peer_sum = PeerSum(B * H, bf, dev, group)
        self.logits = torch.zeros((B, cfg.vocab_size), device=dev, dtype=bf)
        self.logits_f32 = torch.zeros((B, cfg.vocab_size), device=dev, dtype=torch.float32)
        # This rank's q | k | v rows of every layer's fused projection.
        self.qkv_weights = [self._local_qkv(lw.qkv) for lw in weights.layers]
        # This rank's output-projection columns and MLP slice (tensor mode), else the whole matrices.
        self.o_weights, self.gate_up_weights, self.down_weights = [], [], []
        for lw in weights.layers:
            if self.tensor_mlp:
                r, il = rank, self.inter_local
                self.o_weights.append(lw.o[:, r * self.qh * D:(r + 1) * self.qh * D].contiguous())
                self.gate_up_weights.append(torch.cat([lw.gate_up[r * il:(r + 1) * il],
                                                       lw.gate_up[I + r * il:I + (r + 1) * il]]).contiguous())
                self.down_weights.append(lw.down[:, r * il:(r + 1) * il].contiguous())
            else:
                self.o_weights.append(lw.o)
                self.gate_up_weights.append(lw.gate_up)
                self.down_weights.append(lw.down)
        # KV caches [B, KVH_local, cap, D] and the sparse layers' packed planes
        # [B * KVH_local, meta_capacity, ...] (batch entries flattened into heads).
        self.k_cache = [torch.zeros((B, self.kvh, cap, D), device=dev, dtype=bf) for _ in range(L)]
        self.v_cache = [torch.zeros((B, self.kvh, cap, D), device=dev, dtype=bf) for _ in range(L)]
        reps = D // self.g
        rows = B * self.kvh
        self.packed = {}
        for l in self.sparse_layers:
            self.packed[l] = (
                torch.zeros((rows, self.meta_capacity, D // 32), device=dev, dtype=torch.int32),
                torch.zeros((rows, self.meta_capacity, D // 32), device=dev, dtype=torch.int32),
                torch.zeros((rows, self.meta_capacity, reps), device=dev, dtype=torch.float16),
                torch.zeros((rows, self.meta_capacity, reps), device=dev, dtype=torch.float16))
        # Retrieval scratch shared by the layers (they run one after another).
        self.max_tokens = cap - 1  # prefix tokens when the last row is decoded
        self.k_max = min(self.budget - 1, self.max_tokens)
        self.score_stride = (self.max_tokens + 7) // 8 * 8
        self.scores = torch.zeros((B * self.qh, self.score_stride), device=dev, dtype=torch.float16)
        self.indices = torch.zeros((B * self.qh, self.k_max + 1), device=dev, dtype=torch.int64)
        dense_splits = math.ceil((self.max_tokens + 1) / self.split_tokens)
        sparse_splits = math.ceil((self.k_max + 1) / self.split_tokens)
        splits = dense_splits if len(self.sparse_layers) < L else sparse_splits
        self.partials = torch.zeros((B * self.qh, splits, D + 2), device=dev, dtype=torch.float32)
        self.head_to_kv = (torch.arange(B * self.qh, device=dev, dtype=torch.int64) // self.group_heads)
        self.cos, self.sin = rope_tables(cfg, cap, dev)
        self._side = torch.cuda.Stream(dev) if dev.type == "cuda" else None
        self.graph = None
        self.use_graph = use_graph
        self.prefix_length = 0
        if use_graph:
            self.capture()

    # -- setup -------------------------------------------------------------------
    def _local_qkv(self, qkv: torch.Tensor) -> torch.Tensor:
        if self.world == 1:
            return qkv
        D, QH, KVH = self.cfg.head_dim, self.cfg.num_attention_heads, self.cfg.num_key_value_heads
        r = self.rank
        q = qkv[r * self.qh * D:(r + 1) * self.qh * D]
        k = qkv[QH * D + r * self.kvh * D:QH * D + (r + 1) * self.kvh * D]
        v = qkv[(QH + KVH) * D + r * self.kvh * D:(QH + KVH) * D + (r + 1) * self.kvh * D]
        return torch.cat([q, k, v], 0).contiguous()

    # -- the decode step ---------------------------------------------------------
    def _append(self, layer: int, s) -> None:
        """Re-encode the open token group of a sparse layer (the token's key is in
        the cache already: the q/k/v product wrote it)."""
        lib, check, ptr = _lib.lib(), _lib.check, _lib.ptr
        kc, vc = self.k_cache[layer], self.v_cache[layer]
        sign, mag, low, delta = self.packed[layer]
        check(lib.popkv_append_kv_dyn(
            None, None, _lib.BF16, self.batch * self.kvh, 128, ptr(kc), ptr(vc), kc.stride(1), kc.stride(2),
            vc.stride(1), vc.stride(2), ptr(self.position), self.max_context, ptr(sign), ptr(mag), ptr(low),
            ptr(delta), self.meta_capacity, self.tg, self.g, s))

    def _attention(self, layer: int, s, after_score=None) -> None:
        """Score, top-k and attention of one layer; ``after_score(layer)`` forks the
        append re-encode (it must follow the score, nothing else waits for it).
        Without ``after_score`` the append runs inline after the score."""
        lib, check, ptr = _lib.lib(), _lib.check, _lib.ptr
        B = self.batch
        kc, vc = self.k_cache[layer], self.v_cache[layer]
        # Batch entries are flattened into heads: one sequence = KVH_local heads.
        ks, vs = kc.stride(1), vc.stride(1)
        out = self.attn if (self.world == 1 or self.tensor_mlp) else None
        if layer in self.packed:
            sign, mag, low, delta = self.packed[layer]
            check(lib.popkv_score_dyn(
                ptr(self.q), _lib.BF16, 1, B * self.qh, ptr(sign), ptr(mag), ptr(low), ptr(delta),
                B * self.kvh, self.meta_capacity, ptr(self.head_to_kv), ptr(self.position),
                self.max_tokens, self.g, ptr(self.scores), self.score_stride, s))
            # The open group is re-encoded once the score has read the old planes
            # (the reference's order: decode, then append_retrieval_caches).
            if after_score is not None:
                after_score(layer)
            else:
                self._append(layer, s)
            check(lib.popkv_topk_dyn(
                ptr(self.scores), B * self.qh, ptr(self.position), self.max_tokens, self.score_stride,
                self.k_max, ptr(self.indices), self.k_max + 1, s))
            indices, index_stride = ptr(self.indices), self.k_max + 1
        else:
            indices, index_stride = None, 0
        check(lib.popkv_attn_dyn(
            ptr(self.q), _lib.BF16, 1, B * self.qh, ptr(kc), ptr(vc), _lib.BF16, B * self.kvh,
            self.max_tokens, 0, ks, kc.stride(2), 0, vs, vc.stride(2), ptr(self.k_cur),
            ptr(self.v_cur), ptr(self.position), indices, index_stride, self.k_max,
            ptr(self.head_to_kv), self.split_tokens, ptr(self.partials), ptr(out), _lib.BF16, s))
        if self.world > 1 and not self.tensor_mlp:
            selected = self.k_max + 1 if layer in self.packed else self.max_tokens + 1
            self._gather(s, math.ceil(selected / self.split_tokens))

    def _sum_partials(self, t: torch.Tensor, stream) -> None:
        """Tensor mode: sum the ranks' partial products (NCCL all-reduce, inside the graph)."""
        if self._peer_sum is not None:
            self._peer_sum.launch(t, ctypes_stream(stream))
        elif self.tensor_mlp:
            import torch.distributed as dist
            with torch.cuda.stream(stream):
                dist.all_reduce(t, group=self.group)

    def weight_bytes_per_step(self) -> int:
        """Weight bytes this rank streams per decode step (batch <= 4; norms included)."""
        total = self.w.lm_head.numel() * 2 + self.w.norm.numel() * 2
        for l, lw in enumerate(self.w.layers):
            total += (self.qkv_weights[l].numel() + self.o_weights[l].numel() + self.gate_up_weights[l].numel()
                      + self.down_weights[l].numel() + lw.input_norm.numel() + lw.post_norm.numel()) * 2
        return int(total)

    def _gather(self, s, splits: int) -> None:
        """Merge, then all-gather the shards' attention rows [B, QH/N, D] into [B, QH, D]."""
        import torch.distributed as dist
        B, D = self.batch, self.cfg.head_dim
        rows = self.partials.shape[0]
        check, lib, ptr = _lib.check, _lib.lib(), _lib.ptr
        check(lib.popkv_attn_merge(ptr(self.partials), rows, splits, D, ptr(self.attn), _lib.BF16, s))
        dist.all_gather_into_tensor(self._gathered.view(-1), self.attn.view(-1), group=self.group)
        self.attn_full.view(B, self.world, self.qh * D).copy_(
            self._gathered.view(self.world, B, self.qh * D).transpose(0, 1))

    def _launch(self, stream: torch.cuda.Stream) -> None:
        """Enqueue one decode step on ``stream``."""
        if self.fused:
            self._launch_fused(stream)
        else:
            self._launch_cublas(stream)

    def _launch_fused(self, stream: torch.cuda.Stream) -> None:
        """The step as 4 weight-streaming products per layer plus the attention chain.

        The residual stream ping-pongs between ``hidden`` (before a layer) and
        ``hidden_b`` (after its attention): each norm prologue adds the pending
        delta (the previous product's output), stores the sum and normalises it.
        """
        lib, check, ptr = _lib.lib(), _lib.check, _lib.ptr
        s = ctypes_stream(stream)
        cfg, B = self.cfg, self.batch
        H, I, eps = cfg.hidden_size, cfg.intermediate_size, cfg.rms_norm_eps
        QH, D = cfg.num_attention_heads, cfg.head_dim
        side = self._side
        forked = []

        def fork(fn):
            ev = torch.cuda.Event()
            ev.record(stream)
            side.wait_event(ev)
            fn(ctypes_stream(side))
            forked.append(True)

        L = len(self.w.layers)
        for l, lw in enumerate(self.w.layers):
            kc, vc = self.k_cache[l], self.v_cache[l]
            first = l == 0
            if first or not self.tail:
                check(lib.popkv_norm_qkv_rope(
                    ptr(self.qkv_weights[l]), self.qh, self.kvh, H, B, None if first else ptr(self.hidden),
                    None if first else ptr(self.down), ptr(self.w.embed) if first else None, ptr(self.token),
                    ptr(lw.input_norm), eps, ptr(self.hidden_b), ptr(self.cos), ptr(self.sin), ptr(self.position),
                    self.max_context - 1, ptr(self.q), ptr(self.k_cur), ptr(self.v_cur), ptr(kc), ptr(vc),
                    kc.stride(0), kc.stride(1), kc.stride(2), vc.stride(0), vc.stride(1), vc.stride(2), s))
            with torch.cuda.stream(stream):
                self._attention(l, s, after_score=lambda layer: fork(lambda ss: self._append(layer, ss)))
            if self.tail and not self.tensor_mlp:
                # o_proj, gate/up + SwiGLU, down and the next layer's q/k/v (or the LM
                # head) in one persistent launch.  The side branch (the appends)
                # rejoins before the LM head advances the position.
                last = l == L - 1
                if last and forked:
                    stream.wait_stream(side)
                nk, nv = (kc, vc) if last else (self.k_cache[l + 1], self.v_cache[l + 1])
                check(lib.popkv_layer_tail(
                    H, I, QH * D, ptr(lw.o), ptr(self.attn_full), ptr(self.o), ptr(lw.gate_up), ptr(lw.post_norm),
                    ptr(self.hidden_b), ptr(self.hidden), ptr(self.act), eps, ptr(lw.down), ptr(self.down),
                    None if last else ptr(self.qkv_weights[l + 1]), self.qh, self.kvh,
                    None if last else ptr(self.w.layers[l + 1].input_norm), ptr(self.hidden_b), ptr(self.cos),
                    ptr(self.sin), ptr(self.position), self.max_context - 1, ptr(self.q), ptr(self.k_cur),
                    ptr(self.v_cur), ptr(nk), ptr(nv), nk.stride(0), nk.stride(1), nk.stride(2), nv.stride(0),
                    nv.stride(1), nv.stride(2), ptr(self.w.lm_head) if last else None, cfg.vocab_size,
                    ptr(self.w.norm), ptr(self.logits), ptr(self.argmax_state), ptr(self.token),
                    ptr(self.tail_barrier), s))
                continue
            o_in, o_k, il = ((self.attn, self.qh * D, self.inter_local) if self.tensor_mlp
                             else (self.attn_full, QH * D, I))
            check(lib.popkv_linear(ptr(self.o_weights[l]), H, o_k, ptr(o_in), B, ptr(self.o), H, s))
            self._sum_partials(self.o, stream)
            check(lib.popkv_norm_gate_up_swiglu(ptr(self.gate_up_weights[l]), il, H, B, ptr(self.hidden_b),
                                                ptr(self.o), ptr(lw.post_norm), eps, ptr(self.hidden),
                                                ptr(self.act), s))
            check(lib.popkv_linear(ptr(self.down_weights[l]), H, il, ptr(self.act), B, ptr(self.down), H, s))
            self._sum_partials(self.down, stream)
        if self.tail and not self.tensor_mlp:
            return
        # The side branch (the appends) rejoins before the position advances.
        if forked:
            stream.wait_stream(side)
        check(lib.popkv_norm_lm_head_argmax(
            ptr(self.w.lm_head), cfg.vocab_size, H, B, ptr(self.hidden), ptr(self.down), ptr(self.w.norm), eps,
            None, ptr(self.logits), ptr(self.argmax_state), ptr(self.token), ptr(self.position), s))

    def _launch_cublas(self, stream: torch.cuda.Stream) -> None:
        lib, check, ptr = _lib.lib(), _lib.check, _lib.ptr
        s = ctypes_stream(stream)
        cfg, B = self.cfg, self.batch
        H, I, eps = cfg.hidden_size, cfg.intermediate_size, cfg.rms_norm_eps
        with torch.cuda.stream(stream):
            torch.index_select(self.w.embed, 0, self.token, out=self.hidden)
            delta = None
            for l, lw in enumerate(self.w.layers):
                check(lib.popkv_rms_norm(ptr(delta), ptr(self.hidden), ptr(lw.input_norm), B, H, eps,
                                         ptr(self.x), s))
                torch.mm(self.x, self.qkv_weights[l].t(), out=self.qkv)
                kc, vc = self.k_cache[l], self.v_cache[l]
                check(lib.popkv_rope_append(
                    ptr(self.qkv), B, self.qh, self.kvh, 128, ptr(self.cos), ptr(self.sin),
                    ptr(self.position), self.max_context - 1, ptr(self.q), ptr(self.k_cur),
                    ptr(self.v_cur), ptr(kc), ptr(vc), kc.stride(0), kc.stride(1), kc.stride(2),
                    vc.stride(0), vc.stride(1), vc.stride(2), s))
                self._attention(l, s)
                torch.mm(self.attn_full.view(B, -1), lw.o.t(), out=self.o)
                check(lib.popkv_rms_norm(ptr(self.o), ptr(self.hidden), ptr(lw.post_norm), B, H, eps,
                                         ptr(self.x), s))
                torch.mm(self.x, lw.gate_up.t(), out=self.gate_up)
                check(lib.popkv_silu_mul(ptr(self.gate_up), B, I, ptr(self.act), s))
                torch.mm(self.act, lw.down.t(), out=self.down)
                delta = self.down
            check(lib.popkv_rms_norm(ptr(delta), ptr(self.hidden), ptr(self.w.norm), B, H, eps,
                                     ptr(self.x), s))
            torch.mm(self.x, self.w.lm_head.t(), out=self.logits)
            torch.argmax(self.logits, dim=-1, out=self.next_token)
            self.token.copy_(self.next_token)
            self.position.add_(1)

    def capture(self) -> None:
        """Capture the decode step as a CUDA graph (at position 0, before the prefill).

        Warm-up and capture run the step on empty caches; the prefill then
        overwrites every cache row and plane they touched.
        """
        with torch.cuda.device(self.device):
            side = torch.cuda.Stream(self.device)
            self.position.zero_()
            if self.world > 1:
                # Every rank reaches the eager warm-up together, so no peer
                # all-reduce of it waits on a rank that is still building.
                import torch.distributed as dist
                torch.cuda.synchronize(self.device)
                dist.barrier(group=self.group)
            side.wait_stream(torch.cuda.current_stream(self.device))
            self._launch(side)  # sets kernel attributes, cuBLAS workspaces
            side.synchronize()
            self.position.zero_()
            torch.cuda.synchronize(self.device)
            graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(graph, stream=side):
                self._launch(side)
            torch.cuda.current_stream(self.device).wait_stream(side)
            self.graph = graph
            self.position.zero_()
            self.token.zero_()

    # -- prefill -----------------------------------------------------------------
    @torch.inference_mode()
    def prefill(self, prefix_ids: torch.Tensor, *, chunk: int = 8192) -> torch.Tensor:
        """Run the prefix [B, T] through the model (eager PyTorch, causal SDPA).

        Fills KV-cache rows [0, T) of every layer and the packed planes of the
        sparse layers (popkv_pack, the reference's build_popkv_cache), sets the
        position to T and the next input token to the greedy choice after the
        prefix.  Returns that token [B].
        """
        cfg, dev = self.cfg, self.device
        if bool(((prefix_ids < 0) | (prefix_ids >= cfg.vocab_size)).any()):
            raise ValueError(f"token ids must be in [0, {cfg.vocab_size})")
        ids = prefix_ids.to(dev).view(self.batch, -1)
        T = int(ids.shape[1])
        if not 0 < T <= self.max_tokens:
            raise ValueError(f"prefix length must be in [1, {self.max_tokens}]")
        D, QH, KVH = cfg.head_dim, cfg.num_attention_heads, cfg.num_key_value_heads
        kv0 = self.rank * self.kvh
        cos, sin = self.cos[:T], self.sin[:T]
        last = []
        for b in range(self.batch):
            h = self.w.embed[ids[b]]  # [T, H]
            for l, lw in enumerate(self.w.layers):
                q_all = torch.empty((QH, T, D), device=dev, dtype=h.dtype)
                k_all = torch.empty((KVH, T, D), device=dev, dtype=h.dtype)
                v_all = torch.empty((KVH, T, D), device=dev, dtype=h.dtype)
                for c0 in range(0, T, chunk):
                    c1 = min(T, c0 + chunk)
                    x = rms_norm(h[c0:c1], lw.input_norm, cfg.rms_norm_eps)
                    qkv = F.linear(x, lw.qkv)
                    q = qkv[:, :QH * D].view(c1 - c0, QH, D).transpose(0, 1)
                    k = qkv[:, QH * D:(QH + KVH) * D].view(c1 - c0, KVH, D).transpose(0, 1)
                    v = qkv[:, (QH + KVH) * D:].view(c1 - c0, KVH, D).transpose(0, 1)
                    q_all[:, c0:c1] = apply_rope(q, cos[c0:c1], sin[c0:c1])
                    k_all[:, c0:c1] = apply_rope(k, cos[c0:c1], sin[c0:c1])
                    v_all[:, c0:c1] = v
                self.k_cache[l][b, :, :T] = k_all[kv0:kv0 + self.kvh]
                self.v_cache[l][b, :, :T] = v_all[kv0:kv0 + self.kvh]
                group = QH // KVH
                attn = F.scaled_dot_product_attention(
                    q_all[None], k_all.repeat_interleave(group, 0)[None],
                    v_all.repeat_interleave(group, 0)[None], is_causal=True)[0]
                del q_all, k_all, v_all
                attn = attn.transpose(0, 1).reshape(T, QH * D)
                for c0 in range(0, T, chunk):
                    c1 = min(T, c0 + chunk)
                    hc = h[c0:c1] + F.linear(attn[c0:c1], lw.o)
                    x = rms_norm(hc, lw.post_norm, cfg.rms_norm_eps)
                    gu = F.linear(x, lw.gate_up)
                    g, u = gu[:, :cfg.intermediate_size], gu[:, cfg.intermediate_size:]
                    h[c0:c1] = hc + F.linear(F.silu(g) * u, lw.down)
                del attn
            last.append(h[-1])
        h_last = torch.stack(last)
        logits = F.linear(rms_norm(h_last, self.w.norm, cfg.rms_norm_eps), self.w.lm_head).float()
        first = logits.argmax(-1)
        self._pack_prefix(T)
        self.prefix_length = T
        self.position.fill_(T)
        self.token.copy_(first)
        torch.cuda.synchronize(dev)
        return first

    @torch.inference_mode()
    def prefill_synthetic(self, T: int, *, seed: int = 0, chunk: int = 16384) -> torch.Tensor:
        """Fill KV-cache rows [0, T) with the synthetic key/value distributions instead
        of running the model over a prefix (for contexts where a model prefill would
        take minutes, e.g. batch 16 x 131072 tokens).

        Keys: N(0, 1) per element times a per-(sequence, KV head, channel) factor
        exp(N(0, 0.5)) (outlier channels), then RoPE at the token's position;
        values N(0, 1) -- the benchmark configuration's stand-in distributions
        (popkv_b200.workloads), drawn on the device.  Packs the sparse layers'
        planes, sets the position to T and the next input token to a seeded id.
        """
        if not 0 < T <= self.max_tokens:
            raise ValueError(f"prefix length must be in [1, {self.max_tokens}]")
        dev, D = self.device, self.cfg.head_dim
        gen = torch.Generator(device=dev)
        gen.manual_seed(seed)
        for l in range(self.cfg.num_hidden_layers):
            kc, vc = self.k_cache[l], self.v_cache[l]
            for b in range(self.batch):
                factors = torch.empty((self.kvh, 1, D), device=dev).normal_(0.0, 0.5, generator=gen).exp_()
                for c0 in range(0, T, chunk):
                    c1 = min(T, c0 + chunk)
                    k = torch.empty((self.kvh, c1 - c0, D), device=dev).normal_(generator=gen).mul_(factors)
                    kc[b, :, c0:c1] = apply_rope(k.to(torch.bfloat16), self.cos[c0:c1], self.sin[c0:c1])
                    vc[b, :, c0:c1] = torch.empty((self.kvh, c1 - c0, D), device=dev).normal_(generator=gen)
        self._pack_prefix(T)
        self.prefix_length = T
        self.position.fill_(T)
        first = torch.randint(0, self.cfg.vocab_size, (self.batch,), device=dev, generator=gen)
        self.token.copy_(first)
        torch.cuda.synchronize(dev)
        return first

    def _pack_prefix(self, T: int) -> None:
        lib, check, ptr = _lib.lib(), _lib.check, _lib.ptr
        s = _lib.stream_of(self.device)
        for l, (sign, mag, low, delta) in self.packed.items():
            kc = self.k_cache[l]
            check(lib.popkv_pack(ptr(kc), _lib.BF16, self.batch * self.kvh, T, 128, kc.stride(1),
                                 kc.stride(2), ptr(sign), ptr(mag), ptr(low), ptr(delta),
                                 self.meta_capacity, 0, self.tg, self.g, s))

    # -- decoding ----------------------------------------------------------------
    def step(self) -> None:
        """One decode step (graph replay): consumes ``token``, leaves the next in ``token``."""
        if self.graph is None:
            with torch.cuda.device(self.device):
                self._launch(torch.cuda.current_stream(self.device))
        else:
            self.graph.replay()

    def decode(self, token_id=None) -> torch.Tensor:
        """Decode one token (default: the greedy choice of the previous step).

        Returns the fp32 logits [B, vocab] (a view of a static buffer: copy it
        before the next step).  The token's keys/values and packed planes are
        appended in the same step.
        """
        if int(self.position.item()) >= self.max_context:
            raise RuntimeError("static KV cache capacity exhausted")
        if token_id is not None:
            ids = torch.as_tensor(token_id, dtype=torch.int64).view(-1).expand(self.batch)
            if bool(((ids < 0) | (ids >= self.cfg.vocab_size)).any()):
                raise ValueError(f"token ids must be in [0, {self.cfg.vocab_size})")
            self.token.copy_(ids)
        self.step()
        self.logits_f32.copy_(self.logits)
        self._check_collectives()
        return self.logits_f32

    def generate(self, steps: int) -> torch.Tensor:
        """Greedy-decode ``steps`` tokens; returns them [B, steps] (host)."""
        start = int(self.position.item())
        if start + steps > self.max_context:
            raise RuntimeError("static KV cache capacity exhausted")
        out = torch.empty((self.batch, steps), device=self.device, dtype=torch.int64)
        for i in range(steps):
            self.step()
            out[:, i].copy_(self.token)
        tokens = out.cpu()
        self._check_collectives()
        return tokens

    def all_reduce_error(self) -> bool:
        """True when a peer all-reduce gave up waiting for a peer (tensor mode)."""
        return self._peer_sum is not None and self._peer_sum.error()

    def _check_collectives(self) -> None:
        if self.all_reduce_error():
            raise RuntimeError(
                "a peer all-reduce gave up waiting for another rank: this step's outputs are invalid; "
                "call reset_collectives() on every rank before decoding again")

    def reset_collectives(self) -> None:
        """Clear the peer all-reduce's areas and launch state on every rank (collective).

        After ``all_reduce_error()`` the ranks' launch epochs may disagree, so
        every later all-reduce would give up too; all ranks call this with no
        step in flight, then decode again.
        """
        if self._peer_sum is not None:
            self._peer_sum.reset()

    def close(self) -> None:
        """Release the CUDA graph and the peer areas (before the process group is
        destroyed; collective in tensor mode)."""
        self.graph = None
        if self._peer_sum is not None:
            self._peer_sum.close()
            self._peer_sum = None
