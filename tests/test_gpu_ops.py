"""Elementwise, dropout and data-movement kernels on the GPU through the
C-ABI (include/ns_b200_ops.h), against the oracle (bit-exact: these are
copies and single IEEE operations), and a network using every one of them
trained against the model-level oracle."""
import ctypes as C

import numpy as np
import pytest

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

import neuralscript_b200 as nsb  # noqa: E402
import oracle_lib as R  # noqa: E402
from model_oracle import DROP_KEY, OracleModel, make_weights  # noqa: E402
from neuralscript_b200 import synth  # noqa: E402


def _lib():
    L = nsb.lib()
    vp, sz, i, f, u = C.c_void_p, C.c_size_t, C.c_int, C.c_float, C.c_uint
    sig = {
        "nsb_op_softmax": [vp, i, i, vp, vp, vp],
        "nsb_op_binop": [vp, vp, sz, i, vp, vp, vp],
        "nsb_op_binop_bwd": [vp, vp, vp, sz, i, vp, vp, vp],
        "nsb_op_dropout_fwd": [vp, sz, f, u, u, u, u, vp, vp, vp],
        "nsb_op_dropout_bwd": [vp, sz, f, u, u, u, u, vp, vp],
        "nsb_op_transpose": [vp, i, i, vp, vp],
        "nsb_op_concat": [vp, vp, i, i, i, i, i, vp, vp],
        "nsb_op_slice": [vp, i, i, i, i, i, vp, vp],
        "nsb_op_index": [vp, i, i, i, vp, i, vp, vp],
        "nsb_op_scatter": [vp, i, i, i, vp, i, vp, vp, vp],
    }
    for n, a in sig.items():
        getattr(L, n).restype = C.c_int
        getattr(L, n).argtypes = a
    return L


def P(t):
    return None if t is None else C.c_void_p(t.data_ptr())


def dev(a, dtype=torch.float32):
    return torch.from_numpy(np.ascontiguousarray(a)).to("cuda", dtype)


def host(t):
    torch.cuda.synchronize()
    return t.cpu().numpy()


def test_binops_forward_and_gradients():
    L = _lib()
    a = synth.uniform(1001, 11, -2, 2)
    b = synth.uniform(1001, 12, 0.5, 2)
    d = synth.uniform(1001, 13, -1, 1)
    A, B, Dd = dev(a), dev(b), dev(d)
    for code in range(4):
        out = torch.empty_like(A)
        assert L.nsb_op_binop(P(A), P(B), a.size, code, P(out), None, None) == 0
        exp = np.empty_like(a)
        R.lib.orc_binop(a, a.size, b, b.size, exp, code)
        assert np.array_equal(host(out), exp), code
        da, db = torch.empty_like(A), torch.empty_like(A)
        assert L.nsb_op_binop_bwd(P(Dd), P(A), P(B), a.size, code, P(da), P(db), None) == 0
        ga = [d, d, d * b, d / b][code]
        gb = [d, -d, d * a, -d * a / (b * b)][code]
        assert np.array_equal(host(da), ga.astype(np.float32)), code
        assert np.array_equal(host(db), gb.astype(np.float32)), code


def test_softmax_rows_match_oracle():
    L = _lib()
    x = synth.normal(300 * 77, 21, 0, 3).reshape(300, 77)
    X = dev(x)
    out = torch.empty_like(X)
    assert L.nsb_op_softmax(P(X), 300, 77, P(out), None, None) == 0
    got, exp = host(out), R.softmax(x)
    assert np.max(np.abs(got - exp)) < 1e-6 and np.allclose(got.sum(axis=1), 1.0, atol=1e-5)


@pytest.mark.parametrize("n", [4096 * 512, 1001])
def test_dropout_mask_statistics_and_identity(n):
    """The mask equals the oracle's Philox mask element for element; about
    1 - rate of the elements are kept; kept ones are scaled by 1/(1 - rate);
    the backward regenerates exactly the forward's mask."""
    L = _lib()
    rate, step, site = 0.1, 5, 3
    x = synth.normal(n, 31, 0, 1)
    X = dev(x)
    y, y16 = torch.empty_like(X), torch.empty(n, dtype=torch.bfloat16, device="cuda")
    assert L.nsb_op_dropout_fwd(P(X), n, rate, DROP_KEY[0], DROP_KEY[1], step, site, P(y), P(y16), None) == 0
    mask = R.dropout_mask(n, rate, DROP_KEY[0], DROP_KEY[1], step, site)
    got = host(y)
    assert np.array_equal(got, (x * mask).astype(np.float32))
    assert torch.equal(y16, y.to(torch.bfloat16))
    kept = mask > 0
    if n > 100000:
        assert abs(float(kept.mean()) - (1 - rate)) < 1e-3
    assert np.allclose(mask[kept], 1.0 / (1.0 - rate))
    dy = dev(synth.normal(n, 32, 0, 1))
    dx = torch.empty_like(dy)
    assert L.nsb_op_dropout_bwd(P(dy), n, rate, DROP_KEY[0], DROP_KEY[1], step, site, P(dx), None) == 0
    assert np.array_equal(host(dx), (host(dy) * mask).astype(np.float32))
    # another step or site draws another mask
    y2 = torch.empty_like(X)
    assert L.nsb_op_dropout_fwd(P(X), n, rate, DROP_KEY[0], DROP_KEY[1], step + 1, site, P(y2), None, None) == 0
    assert not np.array_equal(host(y2) != 0, got != 0)


def test_data_movement_kernels_match_reference_helpers():
    """The device kernels against the golden outputs of the reference's own
    CPU helpers (tests/golden, the same inputs), plus an out-of-range index."""
    import os
    G = np.load(os.path.join(os.path.dirname(__file__), "golden", "golden.npz"))
    L = _lib()
    X, Y, Z = dev(G["dm_x"]), dev(G["dm_y"]), dev(G["dm_z"])
    R_, C_ = 9, 11

    def run(fn, shape, *args):
        out = torch.full(shape, float("nan"), device="cuda")
        assert getattr(L, fn)(*args[:-1], P(out), None) == 0
        return host(out)

    def ix(v):
        return dev(np.array(v, np.int64), torch.int64)

    assert np.array_equal(run("nsb_op_transpose", (C_, R_), P(X), R_, C_, None), G["dm_transpose"])
    assert np.array_equal(run("nsb_op_concat", (R_, C_ + 5), P(X), P(Y), 1, R_, R_, C_, 5, None), G["dm_concat2"])
    assert np.array_equal(run("nsb_op_concat", (R_ + 4, C_), P(X), P(Z), 0, R_, 4, C_, C_, None), G["dm_concat0"])
    assert np.array_equal(run("nsb_op_slice", (R_, 6), P(X), 1, R_, C_, 3, 9, None), G["dm_slice2"])
    assert np.array_equal(run("nsb_op_slice", (3, C_), P(X), 0, R_, C_, 2, 5, None), G["dm_slicerows"])
    i1, i2, i3, i4 = ix([7, 2, 7, 0]), ix([5, 1, 5]), ix([3, 9, 3, 1, 10]), ix([2, 6, 2, 8])
    assert np.array_equal(run("nsb_op_index", (R_, 4), P(X), 1, R_, C_, P(i1), 4, None), G["dm_index2"])
    assert np.array_equal(run("nsb_op_index", (3, C_), P(X), 0, R_, C_, P(i2), 3, None), G["dm_indexrows"])
    assert np.array_equal(run("nsb_op_scatter", (R_, C_), P(X), 1, R_, C_, P(i3), 5, P(Y), None), G["dm_scatter2"])
    assert np.array_equal(run("nsb_op_scatter", (R_, C_), P(X), 0, R_, C_, P(i4), 4, P(Z), None),
                          G["dm_scatterrows"])
    # an index outside the source reads 0 (the reference reads out of bounds)
    i5 = ix([1, 11])  # held: the kernel reads it after the output is allocated
    oob = run("nsb_op_index", (R_, 2), P(X), 1, R_, C_, P(i5), 2, None)
    assert np.array_equal(oob[:, 0], G["dm_x"][:, 1]) and np.all(oob[:, 1] == 0)
    # a large transpose (several 32 x 32 tiles, ragged edges)
    big = synth.normal(1000 * 777, 41, 0, 1).reshape(1000, 777)
    bigd = dev(big)
    assert np.array_equal(run("nsb_op_transpose", (777, 1000), P(bigd), 1000, 777, None), big.T)


OPS_NET = """network OPS
input 6
layer fc1 dense in=6 out=8 act=gelu
layer dr dropout rate=0.25
layer fc2 dense in=8 out=8
layer fc3 dense in=13 out=4
h = fc1(x)
d = dr(h)
g = fc2(d)
e = sigmoid(g)
m = mul(g, d)
q = div(m, e)
s = slice(q, 1, 6)
c = concat(m, s)
i = index(c, 3, 3, 0)
t = scatter(c, i, 7, 2, 7)
u = sub(t, t)
v = add(t, u)
y = fc3(v)
output y
loss cross_entropy
grad input
optimizer adamw
"""


@pytest.mark.parametrize("mode", ["fp32", "tf32", "bf16"])
def test_network_with_every_new_op_trains_like_oracle(mode):
    """Training through dropout (Philox mask regenerated in the backward),
    mul / div / sub / add, slice, concat, index (repeated column) and scatter
    (repeated column: the last update wins), with the input gradient formed;
    fp32 against the oracle at 1e-5, the tensor-core modes at their
    loss tolerances."""
    w = make_weights(OPS_NET, 1401, default_sd=0.5)
    x = synth.uniform(96 * 6, 1402, -1, 1)
    y = synth.one_hot(synth.tokens(96, 1403, 4), 4)
    m = nsb.Model(OPS_NET, w, precision=mode)
    ref = OracleModel(OPS_NET, w)
    tol = {"fp32": 1e-5, "tf32": 3e-3, "bf16": 1.5e-2}[mode]
    got = [m.train_step(x, y, 0.01) for _ in range(5)]
    exp = [ref.train_step(x, y, 0.01) for _ in range(5)]
    assert np.max(np.abs(np.array(got) - exp) / np.abs(exp)) < tol, (got, exp)
    gx = m.get_input_gradient()
    e = float(np.linalg.norm(gx - ref.input_grad) / np.linalg.norm(ref.input_grad))
    assert e < 10 * tol, e
    # inference: dropout is the identity
    assert np.allclose(m.infer(x), ref.forward(x), rtol=10 * tol, atol=10 * tol)
