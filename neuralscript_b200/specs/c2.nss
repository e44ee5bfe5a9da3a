network C2
input tokens
layer emb embedding vocab=8192 dim=512
layer attn attention dim=512 heads=8 seq=256
layer ln1 layernorm
layer ff1 dense in=512 out=2048 act=gelu
layer ff2 dense in=2048 out=512
layer ln2 layernorm
h = emb(x)
a = attn(h)
r1 = add(a, h)
n1 = ln1(r1)
f1 = ff1(n1)
f = ff2(f1)
r2 = add(f, n1)
y = ln2(r2)
output y
