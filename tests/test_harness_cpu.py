"""The model-level harness (harness/model.py, a restatement of the reference's
Llama/Qwen2 model that consumes the quantized linears) against logits the
reference model itself produced (tests/golden/model_tiny.npz, written by
tests/golden/make_model_golden.py): CPU, float32, dense weights."""

import os

import numpy as np
import torch

from conftest import GOLDEN
from harness import model as H


def test_harness_model_matches_reference_logits():
    d = np.load(os.path.join(GOLDEN, "model_tiny.npz"))
    cfg = H.TINY
    m = H.build_model(cfg, dtype=torch.float32)
    H.init_dense(m, int(d["seed"][0]))
    prompt, forced = torch.from_numpy(d["prompt"]), torch.from_numpy(d["forced"])
    bsz, seq = prompt.shape
    steps = forced.shape[1]
    caches = [(torch.zeros(bsz, cfg.num_key_value_heads, seq + steps, cfg.head_dim),
               torch.zeros(bsz, cfg.num_key_value_heads, seq + steps, cfg.head_dim))
              for _ in range(cfg.num_hidden_layers)]
    with torch.no_grad():
        pos = torch.arange(seq)[None].expand(bsz, seq)
        out = [m(prompt, pos, caches, 0, H.causal_mask(seq, torch.float32, "cpu"))]
        for t in range(steps):
            out.append(m(forced[:, t:t + 1], torch.full((bsz, 1), seq + t), caches, seq + t, None))
    logits = torch.cat(out, dim=1).numpy()
    np.testing.assert_allclose(logits, d["logits"], rtol=1e-4, atol=1e-5)


def test_harness_decode_and_prefill_paths_match_batched_forward():
    """The harness's own decode path (per-request positions over a static
    cache, SDPA) computes the same logits as the reference-shaped forward."""
    cfg = H.TINY
    m = H.build_model(cfg, dtype=torch.float32)
    H.init_dense(m, 5)
    g = torch.Generator().manual_seed(6)
    lens = [7, 11]
    prompts = [torch.randint(0, cfg.vocab_size, (n,), generator=g) for n in lens]
    max_len = 16
    caches = [(torch.zeros(2, cfg.num_key_value_heads, max_len, cfg.head_dim),
               torch.zeros(2, cfg.num_key_value_heads, max_len, cfg.head_dim)) for _ in range(cfg.num_hidden_layers)]
    with torch.no_grad():
        last = [m.forward_prefill(p, caches, slot) for slot, p in enumerate(prompts)]
        for p, lg in zip(prompts, last):
            full = m(p[None], torch.arange(len(p))[None], None, None, H.causal_mask(len(p), torch.float32, "cpu"))
            np.testing.assert_allclose(lg.numpy(), full[0, -1].numpy(), rtol=1e-4, atol=1e-5)
        nxt = torch.stack([lg.argmax() for lg in last])
        pos = torch.tensor(lens)
        mask = torch.where(torch.arange(max_len)[None] <= pos[:, None], 0.0, float("-inf"))[:, None, None, :]
        dec = m.forward_decode(nxt, pos, caches, mask)
        for i, p in enumerate(prompts):
            seq = torch.cat([p, nxt[i:i + 1]])
            full = m(seq[None], torch.arange(len(seq))[None], None, None,
                     H.causal_mask(len(seq), torch.float32, "cpu"))
            np.testing.assert_allclose(dec[i].numpy(), full[0, -1].numpy(), rtol=1e-4, atol=1e-5)


def test_build_model_fp8_never_allocates_dense_projections():
    """Config-4-sized models: every projection is an FP8Linear from the start
    (meta-device build), codes are finite e4m3 of either sign, the scale puts
    the largest at 0.06, and tensor-parallel sharding takes the modules as is."""
    from nanosglang_b200 import quantization as Q
    from nanosglang_b200 import tensor_parallel as TP
    cfg = H.TINY
    m = H.build_model_fp8(cfg, device="cpu", seed=3)
    for layer in m.layers:
        for path in H.PROJECTIONS:
            mod = layer.get_submodule(path)
            assert isinstance(mod, Q.FP8Linear) and not hasattr(mod, "weight")
            codes = mod.weight_fp8.view(torch.uint8)
            assert int((codes & 0x7F).max()) <= 125  # no NaN code (0x7F / 0xFF)
            assert int(codes.max()) >= 128  # both signs
            assert float(mod.weight_scale) == np.float32(0.06 / 448.0)
    assert m.layers[0].self_attn.q_proj.bias.dtype == torch.bfloat16
    again = H.build_model_fp8(cfg, device="cpu", seed=3)  # seeded
    assert torch.equal(again.layers[1].mlp.down_proj.weight_fp8.view(torch.uint8),
                       m.layers[1].mlp.down_proj.weight_fp8.view(torch.uint8))
    TP.tensor_parallel_model(m, 2, 1)
    q = m.layers[0].self_attn.q_proj
    assert q.linear.weight_fp8.shape[0] == cfg.num_attention_heads * cfg.head_dim // 2
