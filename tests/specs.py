"""Specs of the small reference-trainable models in oracle/models/*.ns
(same layers, same weight order), used by the golden and GPU tests."""

TMLP = """network TMLP
input 6
layer fc1 dense in=6 out=16 act=gelu
layer fc2 dense in=16 out=8 act=relu
layer fc3 dense in=8 out=4
h1 = fc1(x)
h2 = fc2(h1)
y = fc3(h2)
output y
loss cross_entropy
optimizer reference
"""

TTFM = """network TTFM
input tokens
layer emb embedding vocab=32 dim=6
layer attn attention dim=6 heads=2 seq=0
layer ln layernorm
layer mlp1 dense in=6 out=12 act=gelu
layer mlp2 dense in=12 out=6
layer fc dense in=6 out=16
h = emb(x)
a = attn(h)
n = ln(a)
m1 = mlp1(n)
m2 = mlp2(m1)
y = fc(m2)
output y
loss cross_entropy
optimizer reference
"""

TMOE = """network TMOE
input tokens
layer emb embedding vocab=16 dim=8
layer moe moe dim=8 experts=4 ffn=16 initial=3
layer fc dense in=8 out=4
h = emb(x)
m = moe(h)
y = fc(m)
output y
loss cross_entropy
optimizer reference
"""

SMALL = {"tmlp": TMLP, "ttfm": TTFM, "tmoe": TMOE}
