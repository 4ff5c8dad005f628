"""Generate the model-level golden vectors from the reference model itself.

Run in a container where the reference checkout is present::

    python tests/golden/make_model_golden.py [--ref PATH_TO_nanoSGLang] [--steps 32]

Two fixtures, both produced by importing the reference's own
``nano_sglang/model/causal_lm.py`` and ``nano_sglang/decode/quantization.py``
in-process (CPU; ``_FLASHINFER_NORM_AVAILABLE`` switched off so RMSNorm takes
its torch branch):

``model_tiny.npz``
    A 2-layer Qwen2-shaped model (q/k/v bias, GQA), float32, dense weights
    from ``harness.model.init_dense``: the reference's logits for a prefill
    and three cached decode steps. Pins ``harness.model`` (the restated
    consumer model that runs on the GPU box) against the reference model.

``greedy_qwen2_5_0_5b_awq.npz``
    BASELINE config 2's architecture (Qwen2.5-0.5B, 24 layers) with every
    projection an AWQ int4 layer (group 128, config-0 distributions from
    ``harness.model.init_awq``), the reference's ``AWQLinear`` in float16
    (its forward works in fp16 only): for two seeded prompts, the reference's
    greedy tokens over ``--steps`` steps, the top-2 logit gap at each step and
    the top-8 logits. The GPU test feeds the same tokens to the harness model
    with nanosglang_b200's AWQLinear and requires the same argmax wherever
    the reference's top-2 gap is at least 1e-3.

The weights themselves are not stored: both sides regenerate them from the
seeds with torch's CPU generator.
"""

from __future__ import annotations

import argparse
import importlib
import os
import sys
import time

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, ROOT)

from harness import model as H  # noqa: E402

TINY_SEED = 1
GREEDY_SEED = 2
PROMPT_SEED = 3
PROMPT_LENS = (24, 40)


def _ref_modules(ref_root):
    sys.path.insert(0, ref_root)
    cl = importlib.import_module("nano_sglang.model.causal_lm")
    cl._FLASHINFER_NORM_AVAILABLE = False
    q = importlib.import_module("nano_sglang.decode.quantization")
    return cl, q


def _ref_config(cl, cfg: H.ModelConfig):
    return cl.ModelConfig(model_type=cfg.model_type, vocab_size=cfg.vocab_size, hidden_size=cfg.hidden_size,
                          intermediate_size=cfg.intermediate_size, num_hidden_layers=cfg.num_hidden_layers,
                          num_attention_heads=cfg.num_attention_heads, num_key_value_heads=cfg.num_key_value_heads,
                          max_position_embeddings=cfg.max_position_embeddings, rms_norm_eps=cfg.rms_norm_eps,
                          rope_theta=cfg.rope_theta, attention_bias=cfg.attention_bias)


def prompts(vocab):
    g = torch.Generator().manual_seed(PROMPT_SEED)
    return [torch.randint(0, vocab, (n,), generator=g) for n in PROMPT_LENS]


def tiny_inputs(vocab):
    g = torch.Generator().manual_seed(TINY_SEED + 100)
    return torch.randint(0, vocab, (2, 12), generator=g), torch.randint(0, vocab, (2, 3), generator=g)


@torch.no_grad()
def tiny_logits(model, cfg, prompt, forced):
    """Prefill (batch 2, 12 tokens, causal mask) then 3 cached decode steps
    through ``forward(input_ids, position_ids, kv_caches, cache_position,
    attention_mask)`` -- the reference's batched path."""
    bsz, seq = prompt.shape
    steps = forced.shape[1]
    caches = [(torch.zeros(bsz, cfg.num_key_value_heads, seq + steps, cfg.head_dim),
               torch.zeros(bsz, cfg.num_key_value_heads, seq + steps, cfg.head_dim))
              for _ in range(cfg.num_hidden_layers)]
    pos = torch.arange(seq)[None].expand(bsz, seq)
    out = [model(prompt, pos, caches, 0, H.causal_mask(seq, torch.float32, "cpu"))]
    for t in range(steps):
        p = torch.full((bsz, 1), seq + t)
        out.append(model(forced[:, t:t + 1], p, caches, seq + t, None))
    return torch.cat(out, dim=1)


def make_tiny(cl):
    cfg = H.TINY
    mine = H.build_model(cfg, dtype=torch.float32)
    H.init_dense(mine, TINY_SEED)
    ref = cl.CausalLM(_ref_config(cl, cfg))
    ref.load_state_dict(mine.state_dict())
    prompt, forced = tiny_inputs(cfg.vocab_size)
    logits = tiny_logits(ref, cfg, prompt, forced)
    return {"logits": logits.numpy().astype(np.float32), "prompt": prompt.numpy(), "forced": forced.numpy(),
            "seed": np.array([TINY_SEED])}


def make_greedy(cl, q, steps):
    cfg = H.QWEN2_5_0_5B
    mine = H.build_model(cfg, dtype=torch.float16)
    H.quantize_projections_awq(mine)  # nanosglang_b200 AWQLinear modules (CPU buffers only; no forward here)
    H.init_awq(mine, GREEDY_SEED)
    ref = cl.CausalLM(_ref_config(cl, cfg))
    for layer in ref.layers:
        for path in H.PROJECTIONS:
            parent_path, name = path.rsplit(".", 1)
            parent = layer.get_submodule(parent_path)
            lin = getattr(parent, name)
            setattr(parent, name, q.AWQLinear(lin.in_features, lin.out_features, 128, bias=lin.bias is not None))
    ref.load_state_dict(mine.state_dict())
    ref = ref.half()
    ref.rope_cos, ref.rope_sin = cl.precompute_rope_freqs(cfg.head_dim, cfg.max_position_embeddings,
                                                          cfg.rope_theta)
    out = {"steps": np.array([steps]), "seed": np.array([GREEDY_SEED]), "prompt_seed": np.array([PROMPT_SEED])}
    for pi, prompt in enumerate(prompts(cfg.vocab_size)):
        t0 = time.time()
        tokens, gaps, top_i, top_v = H.teacher_forced_greedy(ref, prompt, None, steps=steps)
        print(f"prompt {pi}: {len(prompt)} tokens, {steps} greedy steps in {time.time() - t0:.1f} s; "
              f"min top-2 gap {float(gaps.min()):.4g}")
        out[f"p{pi}_prompt"] = prompt.numpy()
        out[f"p{pi}_tokens"] = tokens.numpy()
        out[f"p{pi}_gaps"] = gaps.numpy().astype(np.float32)
        out[f"p{pi}_top_i"] = top_i.numpy()
        out[f"p{pi}_top_v"] = top_v.numpy().astype(np.float32)
    return out


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--ref", default=os.environ.get("NSQ_REFERENCE", "/root/reference"))
    ap.add_argument("--steps", type=int, default=32)
    ap.add_argument("--only", choices=["tiny", "greedy"], default=None)
    args = ap.parse_args()
    torch.set_num_threads(len(os.sched_getaffinity(0)))
    cl, q = _ref_modules(args.ref)
    if args.only in (None, "tiny"):
        np.savez_compressed(os.path.join(HERE, "model_tiny.npz"), **make_tiny(cl))
    if args.only in (None, "greedy"):
        np.savez_compressed(os.path.join(HERE, "greedy_qwen2_5_0_5b_awq.npz"), **make_greedy(cl, q, args.steps))


if __name__ == "__main__":
    main()
