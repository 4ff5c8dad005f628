"""Model-level harness: the Llama/Qwen2 decoder that consumes the quantized
linears, restated so the drop-in can be exercised on a GPU box that does not
carry the reference.

This is measurement and parity infrastructure, not part of the product path.
It restates the batched forward of nanoSGLang's ``nano_sglang/model/
causal_lm.py`` (xiehuanyi/nanoSGLang): ``RMSNorm`` with the fused residual
(:131-154), half-split RoPE (:157-206), ``Attention.forward`` with a
preallocated KV cache (:209-257), ``MLP`` (:474-482), ``DecoderLayer``
(:485-505) and ``CausalLM.forward`` (:540-583). Module and parameter names are
the reference's, so a state_dict moves between the two models unchanged, and
the projections are plain ``nn.Linear`` children that ``quantize_model``
(the reference's or ``nanosglang_b200.quantization``'s) swaps in place, as
``main.py:104-108`` does. ``tests/golden/make_model_golden.py`` pins this
restatement against the reference model itself.

The decode path used for throughput (``forward_decode``) is this harness's
own: per-request positions in one batch over a static KV cache, written for
CUDA-graph capture. Attention there is torch's SDPA; it is outside the path
this repository rebuilds.
"""

from __future__ import annotations

import math
from dataclasses import dataclass
from typing import Optional

import torch
import torch.nn as nn
import torch.nn.functional as F


@dataclass
class ModelConfig:
    """The reference's ModelConfig fields that the forward reads (causal_lm.py:77-98)."""
    model_type: str = "qwen2"
    vocab_size: int = 151936
    hidden_size: int = 896
    intermediate_size: int = 4864
    num_hidden_layers: int = 24
    num_attention_heads: int = 14
    num_key_value_heads: int = 2
    max_position_embeddings: int = 4096
    rms_norm_eps: float = 1e-6
    rope_theta: float = 1000000.0
    attention_bias: bool = True

    @property
    def head_dim(self) -> int:
        return self.hidden_size // self.num_attention_heads


# BASELINE configs 2-4 and a tiny shape for CPU checks
QWEN2_5_0_5B = ModelConfig()
LLAMA3_8B = ModelConfig(model_type="llama", vocab_size=128256, hidden_size=4096, intermediate_size=14336,
                        num_hidden_layers=32, num_attention_heads=32, num_key_value_heads=8,
                        max_position_embeddings=8192, rms_norm_eps=1e-5, rope_theta=500000.0,
                        attention_bias=False)
QWEN2_5_72B = ModelConfig(model_type="qwen2", vocab_size=152064, hidden_size=8192, intermediate_size=29568,
                          num_hidden_layers=80, num_attention_heads=64, num_key_value_heads=8,
                          max_position_embeddings=32768, rms_norm_eps=1e-6, rope_theta=1000000.0,
                          attention_bias=True)
TINY = ModelConfig(model_type="qwen2", vocab_size=512, hidden_size=256, intermediate_size=512,
                   num_hidden_layers=2, num_attention_heads=4, num_key_value_heads=2,
                   max_position_embeddings=256)

PROJECTIONS = ("self_attn.q_proj", "self_attn.k_proj", "self_attn.v_proj", "self_attn.o_proj",
               "mlp.gate_proj", "mlp.up_proj", "mlp.down_proj")


class RMSNorm(nn.Module):
    """causal_lm.py:131-154 (the torch branch)."""

    def __init__(self, hidden_size: int, eps: float = 1e-5):
        super().__init__()
        self.weight = nn.Parameter(torch.ones(hidden_size))
        self.eps = eps

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        input_dtype = x.dtype
        variance = x.float().pow(2).mean(-1, keepdim=True)
        x = x * torch.rsqrt(variance + self.eps)
        return (self.weight * x).to(input_dtype)

    def forward_fused_residual(self, x: torch.Tensor, residual: torch.Tensor):
        residual = residual + x
        return self.forward(residual), residual

    def fast(self, x: torch.Tensor) -> torch.Tensor:
        """The same normalisation as one fused torch kernel (fp32 inside), for
        the harness's own decode/prefill paths (fewer launches per step)."""
        return F.rms_norm(x, (x.shape[-1],), self.weight.to(x.dtype), self.eps)


def precompute_rope_freqs(head_dim: int, max_seq_len: int, theta: float, device=None):
    """causal_lm.py:157-164: cos/sin tables (max_seq_len, head_dim/2), float32."""
    freqs = 1.0 / (theta ** (torch.arange(0, head_dim, 2, device=device).float() / head_dim))
    t = torch.arange(max_seq_len, device=device).float()
    freqs = torch.outer(t, freqs)
    return freqs.cos(), freqs.sin()


def apply_rope_full(x: torch.Tensor, cos_full: torch.Tensor, sin_full: torch.Tensor, positions: torch.Tensor):
    """apply_rope with the cos/sin tables already duplicated to head_dim and in
    x's dtype ((max_seq_len, head_dim)); x is (tokens, heads, dim)."""
    half = x.shape[-1] // 2
    c = cos_full[positions].unsqueeze(1)
    s = sin_full[positions].unsqueeze(1)
    rotated = torch.cat([-x[..., half:], x[..., :half]], dim=-1)
    return torch.addcmul(x * c, rotated, s)


def apply_rope(x: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor, position_ids: torch.Tensor) -> torch.Tensor:
    """Half-split RoPE (causal_lm.py:167-206): dim i pairs with dim i + head_dim/2.
    x is (batch, heads, seq, dim) with position_ids (batch, seq), or
    (tokens, heads, dim) with position_ids (tokens,)."""
    dtype = x.dtype
    half = x.shape[-1] // 2
    c = cos[position_ids]
    s = sin[position_ids]
    c = torch.cat([c, c], dim=-1).to(dtype).unsqueeze(1)
    s = torch.cat([s, s], dim=-1).to(dtype).unsqueeze(1)
    rotated = torch.cat([-x[..., half:], x[..., :half]], dim=-1)
    return (x * c + rotated * s).to(dtype)


class Attention(nn.Module):
    def __init__(self, config: ModelConfig):
        super().__init__()
        self.num_heads = config.num_attention_heads
        self.num_kv_heads = config.num_key_value_heads
        self.head_dim = config.head_dim
        bias = config.attention_bias
        self.q_proj = nn.Linear(config.hidden_size, self.num_heads * self.head_dim, bias=bias)
        self.k_proj = nn.Linear(config.hidden_size, self.num_kv_heads * self.head_dim, bias=bias)
        self.v_proj = nn.Linear(config.hidden_size, self.num_kv_heads * self.head_dim, bias=bias)
        self.o_proj = nn.Linear(self.num_heads * self.head_dim, config.hidden_size, bias=False)

    def forward(self, hidden_states, cos, sin, position_ids, kv_cache=None, cache_position=None,
                attention_mask=None):
        """causal_lm.py:223-257: batched (batch, seq, hidden) with an optional
        preallocated cache written at ``cache_position``."""
        bsz, seq_len, _ = hidden_states.shape
        # head counts follow the shard (tensor_parallel_model updates them)
        nh, nkv = self.num_heads, self.num_kv_heads
        q = self.q_proj(hidden_states).view(bsz, seq_len, nh, self.head_dim).transpose(1, 2)
        k = self.k_proj(hidden_states).view(bsz, seq_len, nkv, self.head_dim).transpose(1, 2)
        v = self.v_proj(hidden_states).view(bsz, seq_len, nkv, self.head_dim).transpose(1, 2)
        q = apply_rope(q, cos, sin, position_ids)
        k = apply_rope(k, cos, sin, position_ids)
        if kv_cache is not None:
            k_cache, v_cache = kv_cache
            k_cache[:bsz, :, cache_position:cache_position + seq_len, :] = k
            v_cache[:bsz, :, cache_position:cache_position + seq_len, :] = v
            k = k_cache[:bsz, :, :cache_position + seq_len, :]
            v = v_cache[:bsz, :, :cache_position + seq_len, :]
        if nh // nkv > 1:
            k = k.repeat_interleave(nh // nkv, dim=1)
            v = v.repeat_interleave(nh // nkv, dim=1)
        attn = torch.matmul(q, k.transpose(-2, -1)) / math.sqrt(self.head_dim)
        if attention_mask is not None:
            attn = attn + attention_mask
        attn = F.softmax(attn, dim=-1, dtype=torch.float32).to(q.dtype)
        out = torch.matmul(attn, v).transpose(1, 2).contiguous().view(bsz, seq_len, -1)
        return self.o_proj(out)

    def forward_decode(self, hidden_states, cos, sin, positions, k_cache, v_cache, mask):
        """One token per request (rows of a static cache): hidden (bs, hidden),
        positions (bs,), caches (slots, kv_heads, max_len, dim) whose first bs
        slots are this batch, mask (bs, 1, 1, max_len) additive."""
        bs = hidden_states.shape[0]
        nh, nkv = self.num_heads, self.num_kv_heads
        q, k, v = self._qkv(hidden_states)
        q = q.reshape(bs, nh, self.head_dim)
        k = k.reshape(bs, nkv, self.head_dim)
        v = v.reshape(bs, nkv, self.head_dim)
        q = apply_rope_full(q, cos, sin, positions)
        k = apply_rope_full(k, cos, sin, positions)
        rows = torch.arange(bs, device=hidden_states.device)
        k_cache[rows, :, positions, :] = k
        v_cache[rows, :, positions, :] = v
        # grouped-query decode as multi-query attention: the nh / nkv query
        # heads that share a KV head take the place of query positions, so
        # every KV head is read once and the masked kernel needs no GQA support
        qg = q.view(bs, nkv, nh // nkv, self.head_dim)
        out = F.scaled_dot_product_attention(qg, k_cache[:bs], v_cache[:bs], attn_mask=mask,
                                             scale=1.0 / math.sqrt(self.head_dim))
        return self.o_proj(out.reshape(bs, nh * self.head_dim))

    def _qkv(self, h):
        fused = getattr(self, "qkv", None)  # set by fuse_projections
        if fused is not None:
            return fused(h)
        return self.q_proj(h), self.k_proj(h), self.v_proj(h)

    def forward_prefill(self, hidden_states, cos, sin, positions, k_cache, v_cache, slot):
        """One request's prompt (seq, hidden) into cache slot ``slot`` (causal)."""
        seq = hidden_states.shape[0]
        nh, nkv = self.num_heads, self.num_kv_heads
        q = self.q_proj(hidden_states).view(seq, nh, self.head_dim)
        k = self.k_proj(hidden_states).view(seq, nkv, self.head_dim)
        v = self.v_proj(hidden_states).view(seq, nkv, self.head_dim)
        q = apply_rope(q, cos, sin, positions)
        k = apply_rope(k, cos, sin, positions)
        k_cache[slot, :, :seq, :] = k.transpose(0, 1)
        v_cache[slot, :, :seq, :] = v.transpose(0, 1)
        out = F.scaled_dot_product_attention(q.transpose(0, 1).unsqueeze(0), k.transpose(0, 1).unsqueeze(0),
                                             v.transpose(0, 1).unsqueeze(0), is_causal=True,
                                             scale=1.0 / math.sqrt(self.head_dim), enable_gqa=nh != nkv)
        return self.o_proj(out[0].transpose(0, 1).reshape(seq, nh * self.head_dim))


class MLP(nn.Module):
    """causal_lm.py:474-482."""

    def __init__(self, config: ModelConfig):
        super().__init__()
        self.gate_proj = nn.Linear(config.hidden_size, config.intermediate_size, bias=False)
        self.up_proj = nn.Linear(config.hidden_size, config.intermediate_size, bias=False)
        self.down_proj = nn.Linear(config.intermediate_size, config.hidden_size, bias=False)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        fused = getattr(self, "gate_up", None)  # set by fuse_projections
        if fused is not None:
            return self.down_proj(fused(x))
        return self.down_proj(F.silu(self.gate_proj(x)) * self.up_proj(x))


class DecoderLayer(nn.Module):
    """causal_lm.py:485-505."""

    def __init__(self, config: ModelConfig):
        super().__init__()
        self.self_attn = Attention(config)
        self.mlp = MLP(config)
        self.input_layernorm = RMSNorm(config.hidden_size, config.rms_norm_eps)
        self.post_attention_layernorm = RMSNorm(config.hidden_size, config.rms_norm_eps)

    def _finish(self, hidden_states, residual):
        hidden_states, residual = self.post_attention_layernorm.forward_fused_residual(hidden_states, residual)
        return residual + self.mlp(hidden_states)

    def forward(self, hidden_states, cos, sin, position_ids, kv_cache=None, cache_position=None,
                attention_mask=None):
        residual = hidden_states
        h = self.self_attn(self.input_layernorm(hidden_states), cos, sin, position_ids, kv_cache, cache_position,
                           attention_mask)
        return self._finish(h, residual)

    def forward_decode(self, hidden_states, cos_full, sin_full, positions, k_cache, v_cache, mask):
        h = self.self_attn.forward_decode(self.input_layernorm.fast(hidden_states), cos_full, sin_full, positions,
                                          k_cache, v_cache, mask)
        residual = hidden_states + h
        return residual + self.mlp(self.post_attention_layernorm.fast(residual))

    def forward_prefill(self, hidden_states, cos, sin, positions, k_cache, v_cache, slot):
        h = self.self_attn.forward_prefill(self.input_layernorm(hidden_states), cos, sin, positions, k_cache,
                                           v_cache, slot)
        return self._finish(h, hidden_states)


class CausalLM(nn.Module):
    """causal_lm.py:540-583 (batched forward) plus the harness's decode/prefill paths."""

    def __init__(self, config: ModelConfig):
        super().__init__()
        self.config = config
        self.embed_tokens = nn.Embedding(config.vocab_size, config.hidden_size)
        self.layers = nn.ModuleList([DecoderLayer(config) for _ in range(config.num_hidden_layers)])
        self.norm = RMSNorm(config.hidden_size, config.rms_norm_eps)
        self.lm_head = nn.Linear(config.hidden_size, config.vocab_size, bias=False)
        cos, sin = precompute_rope_freqs(config.head_dim, config.max_position_embeddings, config.rope_theta)
        self.register_buffer("rope_cos", cos, persistent=False)
        self.register_buffer("rope_sin", sin, persistent=False)

    def forward(self, input_ids, position_ids, kv_caches=None, cache_position=None, attention_mask=None):
        h = self.embed_tokens(input_ids)
        for i, layer in enumerate(self.layers):
            h = layer(h, self.rope_cos, self.rope_sin, position_ids,
                      kv_caches[i] if kv_caches is not None else None, cache_position, attention_mask)
        return self.lm_head(self.norm(h))

    def rope_tables(self, dtype):
        """cos/sin duplicated to head_dim in ``dtype`` (cached), for the decode path."""
        key = ("rope_full", dtype)
        if getattr(self, "_rope_key", None) != key:
            self._rope_full = (torch.cat([self.rope_cos, self.rope_cos], -1).to(dtype),
                               torch.cat([self.rope_sin, self.rope_sin], -1).to(dtype))
            self._rope_key = key
        return self._rope_full

    def forward_decode(self, tokens, positions, caches, mask):
        """tokens/positions (bs,), caches [(k, v)] per layer -> logits (bs, vocab)."""
        h = self.embed_tokens(tokens)
        cos_full, sin_full = self.rope_tables(h.dtype)
        for layer, (kc, vc) in zip(self.layers, caches):
            h = layer.forward_decode(h, cos_full, sin_full, positions, kc, vc, mask)
        return self.lm_head(self.norm.fast(h))

    def forward_prefill(self, tokens, caches, slot):
        """One prompt (seq,) into cache slot ``slot`` -> logits of its last token (vocab,)."""
        positions = torch.arange(tokens.shape[0], device=tokens.device)
        h = self.embed_tokens(tokens)
        for layer, (kc, vc) in zip(self.layers, caches):
            h = layer.forward_prefill(h, self.rope_cos, self.rope_sin, positions, kc, vc, slot)
        return self.lm_head(self.norm(h[-1:]))[0]


def fuse_projections(model: CausalLM) -> CausalLM:
    """Run q/k/v as one launch and gate/up with SiLU * up as one launch for
    decode batches (nanosglang_b200.quantization.FusedProjections /
    GateUpSiLU); larger batches keep the separate layers. Call after any
    tensor-parallel sharding. The reference-shaped ``forward`` is unchanged."""
    from nanosglang_b200.quantization import FusedProjections, GateUpSiLU
    for layer in model.layers:
        a, m = layer.self_attn, layer.mlp
        a.qkv = FusedProjections(a.q_proj, a.k_proj, a.v_proj)
        if hasattr(m, "gate_proj"):
            m.gate_up = GateUpSiLU(m.gate_proj, m.up_proj)
    return model


def causal_mask(seq: int, dtype, device) -> torch.Tensor:
    """Additive causal mask (1, 1, seq, seq) for a prefill through ``forward``."""
    m = torch.full((seq, seq), float("-inf"), device=device).triu(1)
    return m.to(dtype)[None, None]


# ---------------------------------------------------------------------------
# Seeded random weights
# ---------------------------------------------------------------------------


def build_model(config: ModelConfig, device="cpu", dtype=torch.float16) -> CausalLM:
    """A model with uninitialised weights on ``device`` (fill with init_dense or init_awq)."""
    with torch.device("meta"):
        model = CausalLM(config)
    model = model.to_empty(device=device)
    cos, sin = precompute_rope_freqs(config.head_dim, config.max_position_embeddings, config.rope_theta,
                                     device=device)
    model.rope_cos, model.rope_sin = cos, sin
    for p in model.parameters():
        p.data = p.data.to(dtype)
    return model


def _uniform(gen, shape, bound, device):
    return (torch.rand(shape, generator=gen, device=device) * 2 - 1) * bound


@torch.no_grad()
def init_common(model: CausalLM, gen: torch.Generator):
    """Embedding N(0,1), norms 1, q/k/v biases U(-1/sqrt(K), 1/sqrt(K)),
    lm_head U(-1/sqrt(hidden), 1/sqrt(hidden)) -- nn.Embedding / nn.Linear's
    default distributions -- drawn in a fixed order from ``gen``."""
    cfg = model.config
    dev = gen.device
    model.embed_tokens.weight.copy_(torch.randn(model.embed_tokens.weight.shape, generator=gen, device=dev))
    for layer in model.layers:
        layer.input_layernorm.weight.fill_(1.0)
        layer.post_attention_layernorm.weight.fill_(1.0)
        for name in ("q_proj", "k_proj", "v_proj"):
            lin = getattr(layer.self_attn, name)
            if lin.bias is not None:
                lin.bias.copy_(_uniform(gen, lin.bias.shape, 1.0 / math.sqrt(cfg.hidden_size), dev))
    model.norm.weight.fill_(1.0)
    model.lm_head.weight.copy_(_uniform(gen, model.lm_head.weight.shape, 1.0 / math.sqrt(cfg.hidden_size), dev))


@torch.no_grad()
def init_dense(model: CausalLM, seed: int):
    """Every projection weight U(-1/sqrt(K), 1/sqrt(K)) (nn.Linear's default), seeded."""
    gen = torch.Generator(device=model.embed_tokens.weight.device).manual_seed(seed)
    init_common(model, gen)
    for layer in model.layers:
        for path in PROJECTIONS:
            lin = layer.get_submodule(path)
            lin.weight.copy_(_uniform(gen, lin.weight.shape, 1.0 / math.sqrt(lin.in_features), gen.device))


def build_model_fp8(config: ModelConfig, device="cpu", dtype=torch.bfloat16, seed: int = 5) -> CausalLM:
    """A model whose projections are nanosglang_b200 FP8Linear modules from the
    start, for sizes whose dense projections never fit (Qwen2.5-72B: 140 GB in
    bf16): the model is built on the meta device, every projection is replaced
    by an FP8Linear there, and only then is memory allocated. Weights are
    seeded random e4m3 codes (every finite code but the two largest, either
    sign; no NaN codes) with a per-tensor scale that puts the largest at 0.06,
    the range of N(0, 0.02) weights; the other weights as ``init_common``."""
    from nanosglang_b200 import quantization as Q
    with torch.device("meta"):
        model = CausalLM(config)
        for layer in model.layers:
            for path in PROJECTIONS:
                parent_path, name = path.rsplit(".", 1)
                parent = layer.get_submodule(parent_path)
                lin = getattr(parent, name)
                setattr(parent, name, Q.FP8Linear(lin.in_features, lin.out_features, bias=lin.bias is not None))
    model = model.to_empty(device=device)
    cos, sin = precompute_rope_freqs(config.head_dim, config.max_position_embeddings, config.rope_theta,
                                     device=device)
    model.rope_cos, model.rope_sin = cos, sin
    for p in model.parameters():
        p.data = p.data.to(dtype)
    gen = torch.Generator(device=device).manual_seed(seed)
    with torch.no_grad():
        init_common(model, gen)
        for layer in model.layers:
            for path in PROJECTIONS:
                m = layer.get_submodule(path)
                codes = torch.randint(0, 126, m.weight_fp8.shape, generator=gen, device=device, dtype=torch.uint8)
                sign = torch.randint(0, 2, m.weight_fp8.shape, generator=gen, device=device, dtype=torch.uint8)
                m.weight_fp8.view(torch.uint8).copy_(codes | (sign << 7))
                m.weight_scale.fill_(0.06 / 448.0)
                del codes, sign
    return model


def awq_buffers(gen: torch.Generator, n: int, k: int, group_size: int = 128):
    """BASELINE config-0 distributions in the reference layout: int4 values
    uniform on 0..15 packed 8 per int32 along K (qweight [N, K/8]), zero
    points uniform on 0..15 (fp16 [N, G]), scales uniform on [0.001, 0.01]
    (fp16 [N, G]). Any nibble order of uniform nibbles is the same
    distribution of words."""
    g = (k + group_size - 1) // group_size
    dev = gen.device
    qw = torch.randint(-2 ** 31, 2 ** 31 - 1, (n, k // 8), generator=gen, device=dev, dtype=torch.int64)
    qw = qw.to(torch.int32)
    s = (torch.rand(n, g, generator=gen, device=dev) * 0.009 + 0.001).half()
    z = torch.randint(0, 16, (n, g), generator=gen, device=dev).half()
    return qw, s, z


@torch.no_grad()
def init_awq(model: nn.Module, seed: int, group_size: int = 128):
    """Fill a model whose projections are already AWQ modules (any
    implementation with the reference's buffers) with seeded config-0
    distributions; common weights as ``init_common``."""
    dev = model.embed_tokens.weight.device
    gen = torch.Generator(device=dev).manual_seed(seed)
    init_common(model, gen)
    for layer in model.layers:
        for path in PROJECTIONS:
            m = layer.get_submodule(path)
            qw, s, z = awq_buffers(gen, m.out_features, m.in_features, group_size)
            m.qweight.copy_(qw)
            m.scales.copy_(s)
            m.zeros.copy_(z)


def quantize_projections_awq(model: CausalLM, group_size: int = 128):
    """Swap every projection for nanosglang_b200's AWQLinear through its
    quantize_model (the reference's walk and skip list: embed_tokens, lm_head
    and norm stay dense), without running the quantiser on the placeholder
    dense weights: the buffers are then filled by ``init_awq``."""
    from nanosglang_b200 import quantization as Q

    orig = Q._QUANTIZERS["awq"]

    def empty_awq(child, gs):
        with torch.device(child.weight.device):
            out = Q.AWQLinear(child.in_features, child.out_features, gs, bias=child.bias is not None)
        if child.bias is not None:
            out.bias = nn.Parameter(child.bias.data.clone())
        return out

    Q._QUANTIZERS["awq"] = empty_awq
    try:
        import contextlib
        import io
        with contextlib.redirect_stdout(io.StringIO()):
            Q.quantize_model(model, "awq", group_size)
    finally:
        Q._QUANTIZERS["awq"] = orig
    return model


# ---------------------------------------------------------------------------
# Teacher-forced greedy decoding (the model-level parity check)
# ---------------------------------------------------------------------------


@torch.no_grad()
def teacher_forced_greedy(model: nn.Module, prompt: torch.Tensor, forced: Optional[torch.Tensor] = None,
                          steps: int = 32, topk: int = 8):
    """Prefill ``prompt`` (seq,), then one decode step per token of ``forced``,
    feeding the forced token each time (so every step sees the same prefix on
    both sides of a comparison); with ``forced=None`` it feeds its own argmax
    (plain greedy decoding of ``steps`` tokens). Returns, per step (the
    prefill's last position, then after each fed token but the last): the
    argmax token, the top-2 logit gap, and the top-k (indices, values) in
    float32. Works on the reference's CausalLM and on this harness's (same
    forward signature)."""
    cfg = model.config
    dev = model.embed_tokens.weight.device
    dtype = model.embed_tokens.weight.dtype
    seq = prompt.shape[0]
    steps = forced.shape[0] if forced is not None else steps
    max_len = seq + steps
    caches = [(torch.zeros(1, cfg.num_key_value_heads, max_len, cfg.head_dim, device=dev, dtype=dtype),
               torch.zeros(1, cfg.num_key_value_heads, max_len, cfg.head_dim, device=dev, dtype=dtype))
              for _ in range(cfg.num_hidden_layers)]
    ids = prompt.to(dev)[None]
    pos = torch.arange(seq, device=dev)[None]
    logits = model(ids, pos, caches, 0, causal_mask(seq, dtype, dev))[0, -1]
    argmax, gaps, top_i, top_v = [], [], [], []
    for t in range(steps):
        lf = logits.float()
        v, i = lf.topk(topk)
        argmax.append(int(i[0]))
        gaps.append(float(v[0] - v[1]))
        top_i.append(i.cpu())
        top_v.append(v.cpu())
        if t + 1 == steps:
            break
        tok = (forced[t].to(dev) if forced is not None else i[0]).view(1, 1)
        p = torch.tensor([[seq + t]], device=dev)
        logits = model(tok, p, caches, seq + t, None)[0, -1]
    return (torch.tensor(argmax), torch.tensor(gaps), torch.stack(top_i), torch.stack(top_v))
