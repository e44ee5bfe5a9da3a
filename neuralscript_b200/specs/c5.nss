network C5
input 4096
layer fc1 dense in=4096 out=4096 act=relu
layer fc2 dense in=4096 out=4096 act=relu
layer fc3 dense in=4096 out=4096 act=relu
layer fc4 dense in=4096 out=4096 act=relu
layer fc5 dense in=4096 out=4096 act=relu
layer fc6 dense in=4096 out=4096 act=relu
layer fc7 dense in=4096 out=4096 act=relu
layer fc8 dense in=4096 out=4096 act=identity
h1 = fc1(x)
h2 = fc2(h1)
h3 = fc3(h2)
h4 = fc4(h3)
h5 = fc5(h4)
h6 = fc6(h5)
h7 = fc7(h6)
h8 = fc8(h7)
output h8
loss mse
optimizer muon momentum=0.95 steps=5 decay=0.01
