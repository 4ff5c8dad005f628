"""Generate the golden vectors that pin the CPU oracle to the reference.

Run in a container where the reference checkout is present::

    python tests/golden/make_golden.py [--ref PATH_TO_nanoSGLang]

It imports the reference's own ``nano_sglang/decode/quantization.py`` and
``nano_sglang/distributed/tensor_parallel.py`` in-process (both import only
torch), drives them on seeded inputs and stores inputs + outputs in
``tests/golden/*.npz``. The reference cannot travel to the GPU box, so the
tests read only these committed fixtures.
"""

from __future__ import annotations

import argparse
import importlib.util
import os
import sys

import numpy as np
import torch
import torch.nn as nn

HERE = os.path.dirname(os.path.abspath(__file__))


def _load(path: str, name: str):
    spec = importlib.util.spec_from_file_location(name, path)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def _u16(t: torch.Tensor) -> np.ndarray:
    return t.contiguous().view(torch.int16).numpy().view(np.uint16).copy()


def _awq_inputs(g: torch.Generator, n: int, k: int, gs: int, zero_mode: str):
    ng = (k + gs - 1) // gs
    qweight = torch.randint(-(2 ** 31), 2 ** 31 - 1, (n, k // 8), generator=g, dtype=torch.int64).to(torch.int32)
    scales = (torch.rand(n, ng, generator=g) * 0.009 + 0.001).half()
    if zero_mode == "int":
        zeros = torch.randint(0, 16, (n, ng), generator=g).half()
    elif zero_mode == "wide":
        zeros = torch.randint(-300, 300, (n, ng), generator=g).half()
    else:  # arbitrary fp16 values
        zeros = (torch.randn(n, ng, generator=g) * 6 + 7).half()
    return qweight, scales, zeros


def make_awq(Q, g):
    cases = [
        (16, 128, 128, "int"), (24, 256, 128, "int"), (40, 384, 128, "wide"),
        (8, 200, 128, "frac"), (32, 512, 64, "int"), (16, 96, 32, "frac"),
        (48, 1024, 128, "int"), (64, 640, 256, "int"),
    ]
    out = {}
    for ci, (n, k, gs, zm) in enumerate(cases):
        qw, s, z = _awq_inputs(g, n, k, gs, zm)
        mod = Q.AWQLinear(k, n, group_size=gs, bias=(ci % 2 == 1))
        mod.qweight.copy_(qw)
        mod.scales.copy_(s)
        mod.zeros.copy_(z)
        w = mod._dequantize()
        out[f"c{ci}_meta"] = np.array([n, k, gs], dtype=np.int64)
        out[f"c{ci}_qweight"] = qw.numpy()
        out[f"c{ci}_scales"] = _u16(s)
        out[f"c{ci}_zeros"] = _u16(z)
        out[f"c{ci}_dequant"] = _u16(w)
        # reference forward as-is: only works with fp16 activations
        m = 1 + (ci * 5) % 17
        x = torch.randn(m, k, generator=g).half()
        if mod.bias is not None:
            with torch.no_grad():
                mod.bias.copy_(torch.randn(n, generator=g))
            mod.bias.data = mod.bias.data.half()
            out[f"c{ci}_bias"] = _u16(mod.bias.data)
        y = mod(x)
        out[f"c{ci}_x"] = _u16(x)
        out[f"c{ci}_y"] = _u16(y)
    out["ncases"] = np.array([len(cases)])
    # bf16 activations: the reference raises (dequant is fp16); record that.
    mod = Q.AWQLinear(128, 16)
    try:
        mod(torch.randn(2, 128).bfloat16())
        out["bf16_raises"] = np.array([0])
    except RuntimeError:
        out["bf16_raises"] = np.array([1])
    return out


def make_awq_quant(Q, g):
    cases = [(16, 128, 128), (24, 256, 128), (8, 200, 128), (32, 512, 64), (12, 136, 128)]
    out = {}
    for ci, (n, k, gs) in enumerate(cases):
        w = torch.randn(n, k, generator=g) * 0.02
        if ci == 1:
            w[:4] = w[:4].abs() + 0.01        # all-positive groups -> negative zero points
            w[4:6, :128] = 0.0                 # constant group -> scale clamp
        lin = nn.Linear(k, n, bias=(ci % 2 == 0))
        with torch.no_grad():
            lin.weight.copy_(w)
        mod = Q.AWQLinear.from_linear(lin, group_size=gs)
        out[f"c{ci}_meta"] = np.array([n, k, gs], dtype=np.int64)
        out[f"c{ci}_w"] = w.numpy()
        out[f"c{ci}_qweight"] = mod.qweight.numpy()
        out[f"c{ci}_scales"] = _u16(mod.scales)
        out[f"c{ci}_zeros"] = _u16(mod.zeros)
    out["ncases"] = np.array([len(cases)])
    return out


def make_fp8(Q, g):
    cases = [(16, 128), (24, 256), (128, 896), (8, 72), (32, 4864 // 8)]
    out = {}
    for ci, (n, k) in enumerate(cases):
        w = torch.randn(n, k, generator=g) * 0.02
        if ci == 3:
            w.zero_()  # all-zero weight -> scale = ones(1) (shape [1])
        lin = nn.Linear(k, n, bias=(ci % 2 == 1))
        with torch.no_grad():
            lin.weight.copy_(w)
            if lin.bias is not None:
                lin.bias.copy_(torch.randn(n, generator=g))
        mod = Q.FP8Linear.from_linear(lin)
        out[f"c{ci}_meta"] = np.array([n, k], dtype=np.int64)
        out[f"c{ci}_w"] = w.numpy()
        out[f"c{ci}_codes"] = mod.weight_fp8.view(torch.uint8).numpy()
        out[f"c{ci}_scale"] = mod.weight_scale.float().reshape(-1).numpy()
        out[f"c{ci}_scale_shape"] = np.array(list(mod.weight_scale.shape) or [-1])
        m = 1 + (ci * 7) % 13
        x = torch.randn(m, k, generator=g).bfloat16()
        mod.bias = None if mod.bias is None else nn.Parameter(mod.bias.data.bfloat16())
        out[f"c{ci}_x"] = _u16(x)
        try:
            y = mod(x)
            out[f"c{ci}_y"] = _u16(y)
            out[f"c{ci}_raises"] = np.array([0])
        except RuntimeError:
            # all-zero weight: scale becomes a 1-element fp32 tensor, the
            # product promotes to fp32 and F.linear(bf16, fp32) raises
            out[f"c{ci}_raises"] = np.array([1])
        if mod.bias is not None:
            out[f"c{ci}_bias"] = _u16(mod.bias.data)
    out["ncases"] = np.array([len(cases)])
    return out


def make_scalars(g):
    special = torch.tensor([0.0, -0.0, 2 ** -10, 2 ** -9, 1.5 * 2 ** -9, 2.5 * 2 ** -9, 2 ** -6, 0.1, 1.0, 1.0625,
                            1.1875, 17.0, 240.0, 440.0, 448.0, 456.0, 464.0, 465.0, 479.9, 480.0, 1e6,
                            -448.0, -464.0, -500.0, float("inf"), -float("inf"), float("nan")])
    rnd = torch.randn(20000, generator=g) * 100
    v = torch.cat([special, rnd, -special[:20]])
    e4 = v.to(torch.float8_e4m3fn).view(torch.uint8)
    bv = torch.randn(20000, generator=g) * 10
    bf = bv.bfloat16()
    return {"e4m3_in": v.numpy(), "e4m3_codes": e4.numpy(),
            "e4m3_decoded": torch.arange(256, dtype=torch.int32).to(torch.uint8).view(torch.float8_e4m3fn).float().numpy(),
            "bf16_in": bv.numpy(), "bf16_bits": _u16(bf)}


def make_quantize_model(Q):
    class Attn(nn.Module):
        def __init__(self):
            super().__init__()
            self.q_proj = nn.Linear(32, 32, bias=True)
            self.k_proj = nn.Linear(32, 16, bias=True)
            self.v_proj = nn.Linear(32, 16, bias=True)
            self.o_proj = nn.Linear(32, 32, bias=False)

    class MLP(nn.Module):
        def __init__(self):
            super().__init__()
            self.gate_proj = nn.Linear(32, 64, bias=False)
            self.up_proj = nn.Linear(32, 64, bias=False)
            self.down_proj = nn.Linear(64, 32, bias=False)

    class Layer(nn.Module):
        def __init__(self):
            super().__init__()
            self.self_attn = Attn()
            self.mlp = MLP()
            self.input_layernorm = nn.LayerNorm(32)

    class Model(nn.Module):
        def __init__(self):
            super().__init__()
            self.embed_tokens = nn.Embedding(10, 32)
            self.layers = nn.ModuleList([Layer(), Layer()])
            self.norm = nn.LayerNorm(32)
            self.lm_head = nn.Linear(32, 10, bias=False)
            self.extra_norm_proj = nn.Linear(32, 32)

    out = {}
    for method in ("fp8", "awq"):
        torch.manual_seed(0)
        m = Model()
        Q.quantize_model(m, method=method, group_size=32)
        names = [n for n, mod in m.named_modules() if type(mod).__name__ in ("FP8Linear", "AWQLinear")]
        out[f"{method}_quantized"] = np.array(names)
        out[f"{method}_dense"] = np.array([n for n, mod in m.named_modules() if isinstance(mod, nn.Linear)])
    return out


def make_tp(T, g):
    out = {}
    n, k = 32, 48
    w = torch.randn(n, k, generator=g)
    b = torch.randn(n, generator=g)
    for ws in (2, 4):
        for r in range(ws):
            col = T.ColumnParallelLinear(k, n, ws, r, bias=True)
            col.load_weight_shard(w, b)
            out[f"col_w{ws}_r{r}"] = col.linear.weight.data.numpy().copy()
            out[f"col_b{ws}_r{r}"] = col.linear.bias.data.numpy().copy()
            row = T.RowParallelLinear(k, n, ws, r, bias=False)
            row.load_weight_shard(w)
            out[f"row_w{ws}_r{r}"] = row.linear.weight.data.numpy().copy()
    out["w"] = w.numpy()
    out["b"] = b.numpy()
    return out


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--ref", default=os.environ.get("NSQ_REFERENCE", "/root/reference"))
    args = ap.parse_args()
    Q = _load(os.path.join(args.ref, "nano_sglang/decode/quantization.py"), "ref_quantization")
    T = _load(os.path.join(args.ref, "nano_sglang/distributed/tensor_parallel.py"), "ref_tensor_parallel")
    g = torch.Generator().manual_seed(20261201)
    import contextlib
    import io
    with contextlib.redirect_stdout(io.StringIO()):
        qm = make_quantize_model(Q)
    np.savez_compressed(os.path.join(HERE, "awq_dequant_forward.npz"), **make_awq(Q, g))
    np.savez_compressed(os.path.join(HERE, "awq_from_linear.npz"), **make_awq_quant(Q, g))
    np.savez_compressed(os.path.join(HERE, "fp8_from_linear_forward.npz"), **make_fp8(Q, g))
    np.savez_compressed(os.path.join(HERE, "scalar_casts.npz"), **make_scalars(g))
    np.savez_compressed(os.path.join(HERE, "quantize_model.npz"), **qm)
    np.savez_compressed(os.path.join(HERE, "tp_shards.npz"), **make_tp(T, g))
    print("wrote", sorted(f for f in os.listdir(HERE) if f.endswith(".npz")))


if __name__ == "__main__":
    sys.exit(main())
