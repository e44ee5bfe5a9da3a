network C3
input 1024
layer moe moe dim=1024 experts=8 ffn=1024
y = moe(x)
output y
loss mse
optimizer adamw
grad input
