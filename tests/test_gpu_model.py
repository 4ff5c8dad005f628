"""Model-level parity on the GPU: the quantized linears dropped into the
Llama/Qwen2 decoder (harness/model.py, pinned to the reference model by
tests/test_harness_cpu.py) through quantize_model, as the reference's
main.py:104-108 installs them.

Greedy tokens: BASELINE config 2's architecture (Qwen2.5-0.5B, 24 layers, AWQ
int4 on every projection, float16) is fed the reference's own greedy tokens
(tests/golden/greedy_qwen2_5_0_5b_awq.npz, produced by the reference model
with the reference AWQLinear on the CPU); at every step the argmax must equal
the reference's token, except where the reference's top-2 logit gap is below
GAP_TOL. GAP_TOL is the north-star 1e-3, raised to one float16 ulp of the top
logit where that is larger: the reference's logits are float16, so a gap it
reports as one ulp may be anything from zero to two ulps.
"""

import os

import numpy as np
import pytest
import torch

from conftest import GOLDEN

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module", autouse=True)
def _cuda():
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    from nanosglang_b200 import _lib
    _lib.device_status_reset()
    yield
    code, where, block = _lib.device_status()
    assert code == 0, f"device status {code} (wait tag {where}, block {block})"


def _fp16_ulp(v):
    return float(np.spacing(np.float16(abs(v))))


@pytest.fixture(scope="module")
def qwen_awq():
    from harness import model as H
    d = np.load(os.path.join(GOLDEN, "greedy_qwen2_5_0_5b_awq.npz"))
    m = H.build_model(H.QWEN2_5_0_5B, dtype=torch.float16)
    H.quantize_projections_awq(m)
    H.init_awq(m, int(d["seed"][0]))  # the same CPU generator stream as the reference side
    return m.cuda(), d


def test_greedy_tokens_match_reference_qwen2_5_0_5b_awq(qwen_awq):
    from harness import model as H
    from nanosglang_b200.quantization import AWQLinear
    m, d = qwen_awq
    n_awq = sum(isinstance(x, AWQLinear) for x in m.modules())
    assert n_awq == 7 * H.QWEN2_5_0_5B.num_hidden_layers
    steps = int(d["steps"][0])
    report = []
    for p in (0, 1):
        prompt = torch.from_numpy(d[f"p{p}_prompt"])
        ref_tok = d[f"p{p}_tokens"]
        ref_gap = d[f"p{p}_gaps"]
        ref_top = d[f"p{p}_top_v"]
        tok, gap, top_i, top_v = H.teacher_forced_greedy(m, prompt, torch.from_numpy(ref_tok), topk=8)
        assert tok.shape[0] == steps
        for t in range(steps):
            tol = max(1e-3, _fp16_ulp(ref_top[t, 0]))
            if int(tok[t]) != int(ref_tok[t]):
                assert ref_gap[t] <= tol, (
                    f"prompt {p} step {t}: token {int(tok[t])} != reference {int(ref_tok[t])} "
                    f"with reference top-2 gap {ref_gap[t]:.4g} > {tol:.4g}")
                # a permitted divergence picks the reference's runner-up
                assert int(tok[t]) in d[f"p{p}_top_i"][t, :2]
                report.append((p, t))
        # the top logits themselves agree closely (float16 model on both sides)
        err = np.abs(top_v[:, 0].numpy() - ref_top[:, 0]).max()
        assert err < 0.05, err
    assert len(report) <= 2, report


def test_engine_decodes_workload_consistently(qwen_awq):
    """The throughput harness (packed prefill, CUDA-graph decode steps per
    batch bucket) produces the tokens the model's own greedy decoding gives,
    except at float16 near-ties."""
    from harness import engine as E
    from harness import model as H
    m, _ = qwen_awq
    prompts, outs = E.make_workload(6, 20, 60, 4, 12, H.QWEN2_5_0_5B.vocab_size, seed=7)
    eng = E.DecodeEngine(m, max_slots=8, max_len=80, max_steps=16)
    eng.capture()
    tps, info = E.run_workload(eng, prompts, outs)
    assert tps > 0 and info["output_tokens"] == sum(outs)
    # the engine's attention (SDPA over the masked static cache) rounds
    # differently from the model's batched path; every token it picks must
    # still be a top logit there, within a few float16 ulps of the maximum
    worst = 0.0
    for p, o, got in zip(prompts, outs, info["tokens"]):
        assert got.shape[0] == o
        tok, gap, top_i, top_v = H.teacher_forced_greedy(m, p, got, topk=8)
        for t in range(o):
            hit = (top_i[t] == got[t]).nonzero()
            assert hit.numel() == 1, f"step {t}: engine token {int(got[t])} not among the top 8"
            short = float(top_v[t, 0] - top_v[t, int(hit[0])])
            worst = max(worst, short / _fp16_ulp(float(top_v[t, 0])))
    assert worst <= 8, worst
