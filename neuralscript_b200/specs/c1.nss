network C1
input 784
layer fc1 dense in=784 out=1024 act=relu
layer fc2 dense in=1024 out=1024 act=relu
layer fc3 dense in=1024 out=10
h1 = fc1(x)
h2 = fc2(h1)
y = fc3(h2)
output y
