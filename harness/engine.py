"""Throughput harness: continuous greedy decoding of a fixed workload on the
harness model, with every decode step a CUDA-graph replay.

Measurement infrastructure (not the product path). It plays the part of
nanoSGLang's engine (``nano_sglang/engine/engine.py:163-216``: decode CUDA
graphs captured per padded batch size; ``benchmarks/bench_throughput.py``:
output tokens / wall-clock seconds) for a workload whose requests all arrive
at once, as BASELINE config 2 describes:

  * prefill: all prompts in one packed forward (one launch per linear over
    every prompt token; attention per request), first token = argmax;
  * decode: one token per active request per step, as a replay of the graph
    captured for the smallest batch bucket that holds the active requests.
    The graph embeds, runs every layer (the quantized linears, RoPE, the
    cache write, SDPA over the static cache), takes the argmax, appends it to
    a token history on the device and advances the positions, so the host
    only chooses the bucket: no host synchronisation between steps.
    Requests are placed in cache slots by descending output length, so the
    active requests are always the leading slots (the order a compacting
    scheduler would keep them in) and no cache rows are ever moved.

``run_workload`` returns tokens/s over the wall clock of the whole job, with
the prompts copied from pinned host memory at the start and the token history
copied back at the end inside the timed region.
"""

from __future__ import annotations

import math
import time
from typing import List, Sequence

import torch

from .model import CausalLM, apply_rope

BUCKETS = (1, 2, 4, 8, 16, 32, 64, 128)


class DecodeEngine:
    def __init__(self, model: CausalLM, max_slots: int, max_len: int, max_steps: int):
        cfg = model.config
        self.model = model
        dev = model.embed_tokens.weight.device
        dt = model.embed_tokens.weight.dtype
        self.device, self.dtype = dev, dt
        attn0 = model.layers[0].self_attn
        kvh, hd = attn0.num_kv_heads, attn0.head_dim  # per-rank heads under tensor parallelism
        self.max_slots, self.max_len, self.max_steps = max_slots, max_len, max_steps
        self.caches = [(torch.zeros(max_slots, kvh, max_len, hd, device=dev, dtype=dt),
                        torch.zeros(max_slots, kvh, max_len, hd, device=dev, dtype=dt))
                       for _ in range(cfg.num_hidden_layers)]
        self.tokens = torch.zeros(max_slots, dtype=torch.long, device=dev)
        self.positions = torch.zeros(max_slots, dtype=torch.long, device=dev)
        self.history = torch.zeros(max_steps + 1, max_slots, dtype=torch.long, device=dev)
        self.step = torch.zeros(1, dtype=torch.long, device=dev)
        self.cols = torch.arange(max_len, device=dev)
        self.graphs = {}
        self.buckets = [b for b in BUCKETS if b <= max_slots]
        if not self.buckets or self.buckets[-1] < max_slots:
            self.buckets.append(max_slots)

    # -- one decode step over the first bs slots (captured per bucket) --------
    def _step(self, bs: int):
        pos = self.positions[:bs]
        mask = torch.zeros(bs, 1, 1, self.max_len, device=self.device, dtype=self.dtype)
        mask.masked_fill_(self.cols[None, None, None, :] > pos[:, None, None, None], float("-inf"))
        logits = self.model.forward_decode(self.tokens[:bs], pos, self.caches, mask)
        nxt = logits.argmax(dim=-1)
        self.tokens[:bs].copy_(nxt)
        self.history[:, :bs].index_copy_(0, self.step, nxt[None])
        self.positions[:bs].add_(1)
        self.step.add_(1)

    @torch.no_grad()
    def capture(self, buckets: Sequence[int] = ()):
        s = torch.cuda.Stream(self.device)
        s.wait_stream(torch.cuda.current_stream(self.device))
        for bs in (buckets or self.buckets):
            if bs in self.graphs:
                continue
            saved = (self.tokens.clone(), self.positions.clone(), self.history.clone(), self.step.clone())
            with torch.cuda.stream(s):
                for _ in range(2):
                    self._step(bs)
            torch.cuda.synchronize(self.device)
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g, stream=s):
                self._step(bs)
            self.graphs[bs] = g
            for dst, src in zip((self.tokens, self.positions, self.history, self.step), saved):
                dst.copy_(src)
        torch.cuda.current_stream(self.device).wait_stream(s)
        torch.cuda.synchronize(self.device)

    def bucket(self, n: int) -> int:
        for b in self.buckets:
            if b >= n:
                return b
        raise ValueError(f"{n} active requests exceed {self.max_slots} slots")

    # -- prefill --------------------------------------------------------------
    @torch.no_grad()
    def prefill(self, prompts: List[torch.Tensor]):
        """Packed prefill of prompts (device tensors) into slots 0..n-1."""
        model = self.model
        lens = [int(p.shape[0]) for p in prompts]
        tokens = torch.cat(prompts)
        positions = torch.cat([torch.arange(n, device=self.device) for n in lens])
        h = model.embed_tokens(tokens)
        starts = [0]
        for n in lens:
            starts.append(starts[-1] + n)
        for layer, (kc, vc) in zip(model.layers, self.caches):
            attn = layer.self_attn
            x = layer.input_layernorm(h)
            nh, nkv, hd = attn.num_heads, attn.num_kv_heads, attn.head_dim
            q = attn.q_proj(x).view(-1, nh, hd)
            k = attn.k_proj(x).view(-1, nkv, hd)
            v = attn.v_proj(x).view(-1, nkv, hd)
            q = apply_rope(q, model.rope_cos, model.rope_sin, positions)
            k = apply_rope(k, model.rope_cos, model.rope_sin, positions)
            outs = []
            for slot, (a, b) in enumerate(zip(starts[:-1], starts[1:])):
                kc[slot, :, :b - a] = k[a:b].transpose(0, 1)
                vc[slot, :, :b - a] = v[a:b].transpose(0, 1)
                o = torch.nn.functional.scaled_dot_product_attention(
                    q[a:b].transpose(0, 1)[None], k[a:b].transpose(0, 1)[None], v[a:b].transpose(0, 1)[None],
                    is_causal=True, scale=1.0 / math.sqrt(hd), enable_gqa=nh != nkv)
                outs.append(o[0].transpose(0, 1).reshape(b - a, nh * hd))
            a_out = attn.o_proj(torch.cat(outs))
            h = layer._finish(a_out, h)
        last = torch.tensor([b - 1 for b in starts[1:]], device=self.device)
        logits = model.lm_head(model.norm(h[last]))
        n = len(prompts)
        first = logits.argmax(dim=-1)
        self.tokens[:n].copy_(first)
        self.positions[:n].copy_(torch.tensor(lens, device=self.device))
        self.history[0, :n].copy_(first)
        self.step.fill_(1)

    def decode_steps(self, active_counts: Sequence[int]):
        for n in active_counts:
            self.graphs[self.bucket(n)].replay()


def make_workload(num_requests: int, prompt_min: int, prompt_max: int, out_min: int, out_max: int, vocab: int,
                  seed: int = 0):
    """BASELINE config 2's workload shape (bench_throughput.py:34-42 with ids
    uniform in the vocab): seeded prompt lengths, token ids and output lengths."""
    g = torch.Generator().manual_seed(seed)
    lens = torch.randint(prompt_min, prompt_max + 1, (num_requests,), generator=g).tolist()
    prompts = [torch.randint(0, vocab, (n,), generator=g) for n in lens]
    outs = torch.randint(out_min, out_max + 1, (num_requests,), generator=g).tolist()
    return prompts, outs


@torch.no_grad()
def run_workload(engine: DecodeEngine, prompts: List[torch.Tensor], out_lens: List[int]):
    """Generate out_lens[i] greedy tokens for every prompt (the first from the
    prefill). Returns (tokens/s over the wall clock, details). Inside the timed
    region: pinned-host -> device copy of the prompts, the prefill, every
    decode step, the device -> host copy of all generated tokens."""
    order = sorted(range(len(prompts)), key=lambda i: -out_lens[i])
    ps = [prompts[i] for i in order]
    outs = [out_lens[i] for i in order]
    host = [p.pin_memory() for p in ps]
    steps = max(outs) - 1
    counts = [sum(1 for o in outs if o > j) for j in range(1, steps + 1)]
    # every cache position and history row the steps touch stays in bounds
    if max(len(p) for p in ps) + max(outs) > engine.max_len or steps > engine.max_steps:
        raise ValueError("workload exceeds the engine's max_len / max_steps")
    if len(ps) > engine.max_slots:
        raise ValueError("more requests than cache slots")
    torch.cuda.synchronize(engine.device)
    t0 = time.perf_counter()
    dev = [h.to(engine.device, non_blocking=True) for h in host]
    engine.prefill(dev)
    engine.decode_steps(counts)
    hist = engine.history[:steps + 1, :len(ps)].to("cpu")
    torch.cuda.synchronize(engine.device)
    elapsed = time.perf_counter() - t0
    total = sum(outs)
    gen = [hist[:o, i] for i, o in enumerate(outs)]
    inv = [0] * len(order)
    for pos, i in enumerate(order):
        inv[i] = pos
    return total / elapsed, {"elapsed_s": elapsed, "output_tokens": total, "prompt_tokens": sum(len(p) for p in ps),
                             "decode_steps": steps, "requests": len(ps),
                             "tokens": [gen[inv[i]] for i in range(len(order))]}


@torch.no_grad()
def time_decode_step(engine: DecodeEngine, bs: int, iters: int = 20):
    """Device time (ms) of one decode-step graph replay at batch bs (CUDA events)."""
    g = engine.graphs[engine.bucket(bs)]
    if iters + 3 > engine.max_steps or iters + 3 >= engine.max_len:
        raise ValueError("too many timing steps for the engine's history / cache")
    saved = (engine.tokens.clone(), engine.positions.clone(), engine.history.clone(), engine.step.clone())
    # each replay advances positions and the history row: start both at 0
    engine.positions.zero_()
    engine.step.zero_()
    for _ in range(3):
        g.replay()
    torch.cuda.synchronize(engine.device)
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s.record()
    for _ in range(iters):
        g.replay()
    e.record()
    torch.cuda.synchronize(engine.device)
    for dst, src in zip((engine.tokens, engine.positions, engine.history, engine.step), saved):
        dst.copy_(src)
    return s.elapsed_time(e) / iters
