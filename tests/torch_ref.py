"""Float64 restatement of a spec'd network in torch (autograd for the
gradients), used as the reference at sizes the C oracle cannot finish in
seconds (the config-4 step at 16384 rows with its 8192-way head).

Test infrastructure only. It follows the same definitions as the C oracle
(oracle/ns_oracle.c, itself pinned to the reference's CPU emit): GELU in the
erf form of src/codegen/codegen.cpp:1244-1255, LayerNorm without affine and
eps 1e-5 (codegen.cpp:1280-1291) with the reference's backward formula
(codegen.cpp:1346-1371, see _ref_layernorm), per-sequence attention with scale
1/sqrt(head_dim) (codegen.cpp:1724-1777), mean softmax cross-entropy over
rows (codegen.cpp:1598-1613), gradient SUM for values consumed twice.
tests/test_torch_ref_cpu.py pins it to the C oracle on a small model.
"""
from __future__ import annotations

import math
from typing import Dict, Tuple

import numpy as np

from neuralscript_b200.spec import ACT_CODES, parse


def _act(t, code):
    import torch
    if code == 0:
        return t
    if code == 1:
        return torch.relu(t)
    if code == 2:
        return torch.where(t > 0, t, 0.01 * t)
    if code == 3:
        return torch.sigmoid(t)
    if code == 4:
        return torch.tanh(t)
    if code == 5:
        return t * torch.sigmoid(t)
    if code == 6:
        return 0.5 * t * (1.0 + torch.erf(t / math.sqrt(2.0)))
    raise ValueError(code)


def _ref_layernorm(u):
    """LayerNorm whose backward is the reference's formula
    (codegen.cpp:1346-1371): dx = (d - mean(d) - xc * mean(xc * d)) * rstd with
    xc = x - mean(x). The exact derivative has xc * rstd^2 in the last term;
    the reference (and the engine, for parity) omits the rstd^2."""
    import torch

    class _LN(torch.autograd.Function):
        @staticmethod
        def forward(ctx, x):
            mu = x.mean(dim=1, keepdim=True)
            xc = x - mu
            inv = 1.0 / torch.sqrt((xc * xc).mean(dim=1, keepdim=True) + 1e-5)
            ctx.save_for_backward(xc, inv)
            return xc * inv

        @staticmethod
        def backward(ctx, d):
            xc, inv = ctx.saved_tensors
            gamma = (xc * d).mean(dim=1, keepdim=True)
            return (d - d.mean(dim=1, keepdim=True) - xc * gamma) * inv

    return _LN.apply(u)


def forward_backward(spec_text: str, weights: np.ndarray, x: np.ndarray, targets: np.ndarray, device="cpu",
                     dtype=None) -> Tuple[float, Dict[str, np.ndarray], np.ndarray]:
    """Mean cross-entropy loss, gradients by weight name and the output of
    one forward/backward pass, computed in float64 (by default)."""
    import torch
    dtype = dtype or torch.float64
    s = parse(spec_text)
    params = {}
    for name, off, cnt, shp in s.layout():
        params[name] = torch.tensor(np.asarray(weights[off:off + cnt], np.float64).reshape(shp), dtype=dtype,
                                    device=device, requires_grad=True)
    xv = np.asarray(x, np.float32).reshape(-1)
    rows = xv.size // s.in_cols
    if s.tokens:
        vals = {"x": torch.tensor(xv[:rows], dtype=dtype, device=device)}
    else:
        vals = {"x": torch.tensor(xv.reshape(rows, s.in_cols), dtype=dtype, device=device)}
    for op in s.ops:
        a = [vals[t] for t in op.args]
        if op.fn in ("add", "sub", "mul", "div"):
            vals[op.out] = {"add": a[0] + a[1], "sub": a[0] - a[1], "mul": a[0] * a[1],
                            "div": a[0] / a[1]}[op.fn]
            continue
        if op.fn in ACT_CODES:
            vals[op.out] = _act(a[0], ACT_CODES[op.fn])
            continue
        l = s.layer(op.fn)
        u = a[0]
        if l.kind == "dense":
            vals[op.out] = _act(u @ params[f"{l.name}_w"], l.act)
        elif l.kind == "embedding":
            idx = u.to(torch.int64)  # truncation toward zero, as (int) in the reference
            V = l.i("vocab")
            idx = torch.where((idx >= 0) & (idx < V), idx, torch.zeros_like(idx))
            vals[op.out] = params[f"{l.name}_w"][idx]
        elif l.kind == "attention":
            D, H = l.i("dim"), l.i("heads")
            S = l.i("seq", 0) or u.shape[0]
            B, dh = u.shape[0] // S, D // H
            q = (u @ params[f"{l.name}_q_w"]).reshape(B, S, H, dh).transpose(1, 2)
            k = (u @ params[f"{l.name}_k_w"]).reshape(B, S, H, dh).transpose(1, 2)
            v = (u @ params[f"{l.name}_v_w"]).reshape(B, S, H, dh).transpose(1, 2)
            p = torch.softmax(q @ k.transpose(-1, -2) / math.sqrt(dh), dim=-1)
            ctx = (p @ v).transpose(1, 2).reshape(B * S, D)
            vals[op.out] = ctx @ params[f"{l.name}_o_w"]
        elif l.kind == "layernorm":
            vals[op.out] = _ref_layernorm(u)
        else:
            raise ValueError(f"torch reference: unsupported layer {l.kind}")
    out = vals[s.output]
    t = torch.tensor(np.asarray(targets, np.int64), device=device)
    loss = torch.nn.functional.cross_entropy(out, t, reduction="mean")
    loss.backward()
    grads = {n: p.grad.detach().cpu().numpy() for n, p in params.items() if p.grad is not None}
    return float(loss.item()), grads, out.detach().cpu().numpy()
