"""Pins the float64 torch restatement (tests/torch_ref.py) to the C oracle on
a small config-4-structured model: forward output, loss and every weight
gradient. The torch reference then stands in for the oracle at sizes the
oracle cannot finish in seconds (the full config-4 step on the GPU)."""
import numpy as np
import pytest

torch = pytest.importorskip("torch")

import torch_ref  # noqa: E402
from model_oracle import OracleModel, make_weights  # noqa: E402
from neuralscript_b200 import synth  # noqa: E402

SMALL4 = """network S4
input tokens
layer emb embedding vocab=40 dim=16
layer attn attention dim=16 heads=2 seq=8
layer ln1 layernorm
layer ff1 dense in=16 out=32 act=gelu
layer ff2 dense in=32 out=16
layer ln2 layernorm
layer head dense in=16 out=24
h = emb(x)
a = attn(h)
r1 = add(a, h)
n1 = ln1(r1)
f1 = ff1(n1)
f = ff2(f1)
r2 = add(f, n1)
y = ln2(r2)
logits = head(y)
output logits
loss cross_entropy
optimizer adamw
"""


def rel(a, b):
    a, b = np.asarray(a, np.float64), np.asarray(b, np.float64)
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30))


def test_torch_reference_matches_oracle():
    w = make_weights(SMALL4, 951, default_sd=0.2)
    tok = synth.tokens(4 * 8, 952, 40)
    tgt = synth.tokens(4 * 8, 953, 24).astype(np.int64)
    o = OracleModel(SMALL4, w)
    out, vals, cache = o.forward(tok, keep=True)
    y = synth.one_hot(tgt, 24)
    loss, seed = o._loss_and_seed(out, y)
    grads = o.backward(vals, cache, seed)
    tl, tg, tout = torch_ref.forward_backward(SMALL4, w, tok, tgt)
    assert rel(tout, out) < 1e-5
    assert abs(tl - float(loss)) < 1e-5 * abs(tl)
    for name, g in grads.items():
        assert rel(tg[name], g) < 1e-4, name
