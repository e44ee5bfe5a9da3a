network C4
input tokens
layer emb embedding vocab=8192 dim=512
layer attn attention dim=512 heads=8 seq=256
layer ln1 layernorm
layer ff1 dense in=512 out=2048 act=gelu
layer ff2 dense in=2048 out=512
layer ln2 layernorm
layer head dense in=512 out=8192
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
optimizer adamw beta1=0.9 beta2=0.95 eps=1e-8 decay=0.1
schedule cosine warmup=100 total=10000 min=0.05
