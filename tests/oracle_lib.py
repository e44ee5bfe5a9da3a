"""ctypes bindings for the CPU oracle (oracle/libns_oracle.so).

Test infrastructure: only tests/, __graft_entry__.smoke() and bench.py's
CPU-baseline leg use this, as the checker or the timed CPU baseline.
"""
import ctypes as C
import os
import subprocess

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
LIB_PATH = os.path.join(ROOT, "oracle", "libns_oracle.so")

_f32p = np.ctypeslib.ndpointer(np.float32, flags="C_CONTIGUOUS")
_i32p = np.ctypeslib.ndpointer(np.int32, flags="C_CONTIGUOUS")
_u8p = np.ctypeslib.ndpointer(np.uint8, flags="C_CONTIGUOUS")
_i64p = np.ctypeslib.ndpointer(np.int64, flags="C_CONTIGUOUS")
_i64 = C.c_int64


def _load():
    if not os.path.exists(LIB_PATH):
        subprocess.run(["make", "-s", "-f", "oracle/Makefile"], cwd=ROOT, check=True)
    lib = C.CDLL(LIB_PATH)
    sig = {
        "orc_act": (C.c_float, [C.c_float, C.c_int]),
        "orc_act_deriv": (C.c_float, [C.c_float, C.c_int]),
        "orc_act_vec": (None, [_f32p, _f32p, C.c_size_t, C.c_int]),
        "orc_act_grad": (None, [_f32p, _f32p, _f32p, C.c_size_t, C.c_int]),
        "orc_matmul": (None, [_f32p, _f32p, _f32p, _i64, _i64, _i64]),
        "orc_matmul_grad_a": (None, [_f32p, _f32p, _f32p, _i64, _i64, _i64]),
        "orc_matmul_grad_w": (None, [_f32p, _f32p, _f32p, _i64, _i64, _i64]),
        "orc_binop": (None, [_f32p, C.c_size_t, _f32p, C.c_size_t, _f32p, C.c_int]),
        "orc_layernorm": (None, [_f32p, _f32p, _i64, _i64]),
        "orc_layernorm_grad": (None, [_f32p, _f32p, _f32p, _i64, _i64]),
        "orc_softmax": (None, [_f32p, _f32p, _i64, _i64]),
        "orc_embedding": (None, [_f32p, _f32p, _f32p, _i64, _i64, _i64]),
        "orc_embedding_grad_w": (None, [_f32p, _f32p, _f32p, _i64, _i64, _i64]),
        "orc_attention_fwd": (None, [_f32p] * 6 + [_i64] * 4),
        "orc_attention_bwd": (None, [_f32p] * 6 + [C.c_void_p] * 5 + [_i64] * 4),
        "orc_moe_route": (None, [_f32p, _f32p, C.c_void_p, _i32p, C.c_void_p, C.c_void_p, _i64, _i64, _i64]),
        "orc_moe_fwd": (None, [_f32p] * 4 + [C.c_void_p, _f32p] + [_i64] * 4),
        "orc_loss_grad": (None, [_f32p, _f32p, _f32p, _i64, _i64, C.c_float]),
        "orc_cross_entropy": (C.c_float, [_f32p, _f32p, _i64, _i64]),
        "orc_cross_entropy_rows": (None, [_f32p, _f32p, _f32p, _i64, _i64]),
        "orc_orthonom": (None, [_f32p, C.c_size_t, C.c_size_t]),
        "orc_lr_schedule": (C.c_float, [_i64, C.c_int, _i64, _i64, C.c_float]),
        "orc_adamw_step": (None, [_f32p, _f32p, _f32p, _f32p, C.c_size_t, _i64] + [C.c_float] * 7),
        "orc_muon_mgs_step": (None, [_f32p, _f32p, _f32p, _i64, _i64, C.c_float, C.c_float, C.c_float]),
        "orc_newton_schulz5": (None, [_f32p, _i64, _i64, C.c_int]),
        "orc_mse": (C.c_float, [_f32p, _f32p, C.c_size_t]),
        "orc_mse_grad": (None, [_f32p, _f32p, _f32p, C.c_size_t, C.c_float]),
        "orc_transpose2d": (None, [_f32p, _f32p, _i64, _i64]),
        "orc_concat2": (None, [_f32p, _f32p, _f32p, _i64, _i64, _i64]),
        "orc_concat0": (None, [_f32p, _f32p, _f32p, _i64, _i64, _i64]),
        "orc_slice2": (None, [_f32p, _f32p, _i64, _i64, _i64, _i64]),
        "orc_slicerows": (None, [_f32p, _f32p, _i64, _i64, _i64]),
        "orc_index2": (None, [_f32p, _i64p, _f32p, _i64, _i64, _i64]),
        "orc_indexrows": (None, [_f32p, _i64, _i64p, _f32p, _i64, _i64]),
        "orc_scatter2": (None, [_f32p, _i64p, _f32p, _f32p, _i64, _i64, _i64]),
        "orc_scatterrows": (None, [_f32p, _i64p, _f32p, _f32p, _i64, _i64, _i64]),
        "orc_dropout_mask": (None, [_f32p, C.c_size_t, C.c_float, C.c_uint32, C.c_uint32, C.c_uint32, C.c_uint32]),
        "orc_fill_uniform": (None, [_f32p, C.c_size_t, C.c_uint64, C.c_double, C.c_double]),
        "orc_fill_normal": (None, [_f32p, C.c_size_t, C.c_uint64, C.c_double, C.c_double]),
        "orc_fill_tokens": (None, [_f32p, C.c_size_t, C.c_uint64, _i64]),
    }
    for name in ("orc_moe_grad_x", "orc_moe_grad_wg", "orc_moe_grad_we1", "orc_moe_grad_we2"):
        sig[name] = (None, [_f32p] * 5 + [C.c_void_p, _f32p] + [_i64] * 4)
    for name, (res, args) in sig.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    return lib


lib = _load()


def f32(a):
    return np.ascontiguousarray(a, dtype=np.float32)


def _ptr(a):
    return None if a is None else a.ctypes.data_as(C.c_void_p)


def matmul(A, B):
    A, B = f32(A), f32(B)
    M, K = A.shape
    N = B.shape[1]
    out = np.empty((M, N), np.float32)
    lib.orc_matmul(A, B, out, M, K, N)
    return out


def matmul_grad_a(dC, B):
    dC, B = f32(dC), f32(B)
    M, N = dC.shape
    K = B.shape[0]
    out = np.empty((M, K), np.float32)
    lib.orc_matmul_grad_a(dC, B, out, M, K, N)
    return out


def matmul_grad_w(A, dC):
    A, dC = f32(A), f32(dC)
    M, K = A.shape
    N = dC.shape[1]
    out = np.empty((K, N), np.float32)
    lib.orc_matmul_grad_w(A, dC, out, M, K, N)
    return out


def act(x, code):
    x = f32(x)
    out = np.empty_like(x)
    lib.orc_act_vec(x.reshape(-1), out.reshape(-1), x.size, code)
    return out


def act_grad(din, pre, code):
    din, pre = f32(din), f32(pre)
    out = np.empty_like(din)
    lib.orc_act_grad(din.reshape(-1), pre.reshape(-1), out.reshape(-1), din.size, code)
    return out


def act_deriv(x, code):
    return act_grad(np.ones_like(f32(x)), x, code)


def layernorm(x):
    x = f32(x)
    out = np.empty_like(x)
    lib.orc_layernorm(x, out, x.shape[0], x.shape[1])
    return out


def layernorm_grad(dout, x):
    dout, x = f32(dout), f32(x)
    out = np.empty_like(x)
    lib.orc_layernorm_grad(dout, x, out, x.shape[0], x.shape[1])
    return out


def softmax(x):
    x = f32(x)
    out = np.empty_like(x)
    lib.orc_softmax(x, out, x.shape[0], x.shape[1])
    return out


def embedding(W, idx):
    W, idx = f32(W), f32(idx)
    V, D = W.shape
    out = np.empty((idx.size, D), np.float32)
    lib.orc_embedding(W, idx, out, idx.size, V, D)
    return out


def embedding_grad_w(dout, idx, V):
    dout, idx = f32(dout), f32(idx)
    D = dout.shape[1]
    out = np.empty((V, D), np.float32)
    lib.orc_embedding_grad_w(dout, idx, out, idx.size, D, V)
    return out


def attention_fwd(x, Wq, Wk, Wv, Wo, H, S):
    x = f32(x)
    BS, D = x.shape
    out = np.empty_like(x)
    lib.orc_attention_fwd(x, f32(Wq), f32(Wk), f32(Wv), f32(Wo), out, BS, D, H, S)
    return out


def attention_bwd(dout, x, Wq, Wk, Wv, Wo, H, S):
    x, dout = f32(x), f32(dout)
    BS, D = x.shape
    dX = np.empty_like(x)
    dW = [np.empty((D, D), np.float32) for _ in range(4)]
    lib.orc_attention_bwd(dout, x, f32(Wq), f32(Wk), f32(Wv), f32(Wo), _ptr(dX), *[_ptr(d) for d in dW],
                          BS, D, H, S)
    return dX, dW[0], dW[1], dW[2], dW[3]


def moe_route(x, Wg, active=None):
    x, Wg = f32(x), f32(Wg)
    M, D = x.shape
    E = Wg.shape[1]
    best = np.empty(M, np.int32)
    pb = np.empty(M, np.float32)
    p = np.empty((M, E), np.float32)
    act_arr = None if active is None else np.ascontiguousarray(active, np.uint8)
    lib.orc_moe_route(x, Wg, _ptr(act_arr), best, _ptr(pb), _ptr(p), M, D, E)
    return best, pb, p


def moe_fwd(x, Wg, We1, We2, H, active=None):
    x = f32(x)
    M, D = x.shape
    E = Wg.shape[1]
    out = np.empty_like(x)
    act_arr = None if active is None else np.ascontiguousarray(active, np.uint8)
    lib.orc_moe_fwd(x, f32(Wg), f32(We1), f32(We2), _ptr(act_arr), out, M, D, H, E)
    return out


def moe_grads(dout, x, Wg, We1, We2, H, active=None):
    x, dout = f32(x), f32(dout)
    M, D = x.shape
    E = Wg.shape[1]
    act_arr = None if active is None else np.ascontiguousarray(active, np.uint8)
    args = (dout, x, f32(Wg), f32(We1), f32(We2), _ptr(act_arr))
    dx = np.zeros_like(x)
    dWg = np.empty((D, E), np.float32)
    dWe1 = np.empty((E, D * H), np.float32)
    dWe2 = np.empty((E, H * D), np.float32)
    lib.orc_moe_grad_x(*args, dx, M, D, H, E)
    lib.orc_moe_grad_wg(*args, dWg, M, D, H, E)
    lib.orc_moe_grad_we1(*args, dWe1, M, D, H, E)
    lib.orc_moe_grad_we2(*args, dWe2, M, D, H, E)
    return dx, dWg, dWe1, dWe2


def loss_grad(preds, labels, denom=None):
    preds, labels = f32(preds), f32(labels)
    R, Cc = preds.shape
    out = np.empty_like(preds)
    lib.orc_loss_grad(preds, labels, out, R, Cc, float(R if denom is None else denom))
    return out


def cross_entropy(preds, labels):
    preds, labels = f32(preds), f32(labels)
    return lib.orc_cross_entropy(preds, labels, preds.shape[0], preds.shape[1])


def cross_entropy_rows(preds, labels):
    preds, labels = f32(preds), f32(labels)
    out = np.empty(preds.shape[0], np.float32)
    lib.orc_cross_entropy_rows(preds, labels, out, preds.shape[0], preds.shape[1])
    return out


def orthonom(G):
    G = f32(G).copy()
    lib.orc_orthonom(G, G.shape[0], G.shape[1])
    return G


def newton_schulz5(X, steps=5):
    X = f32(X).copy()
    lib.orc_newton_schulz5(X, X.shape[0], X.shape[1], steps)
    return X


def lr_schedule(step, kind, warmup=100, total=10000, min_factor=0.05):
    return lib.orc_lr_schedule(step, kind, warmup, total, min_factor)


def fill_uniform(n, seed, lo, hi):
    out = np.empty(n, np.float32)
    lib.orc_fill_uniform(out, n, seed, lo, hi)
    return out


def fill_normal(n, seed, mu, sd):
    out = np.empty(n, np.float32)
    lib.orc_fill_normal(out, n, seed, mu, sd)
    return out


def fill_tokens(n, seed, vocab):
    out = np.empty(n, np.float32)
    lib.orc_fill_tokens(out, n, seed, vocab)
    return out


# ---- data movement and dropout (restated reference CPU helpers) -------------
def _i64a(v):
    return np.ascontiguousarray(v, dtype=np.int64)


def transpose2d(x):
    x = f32(x)
    out = np.empty((x.shape[1], x.shape[0]), np.float32)
    lib.orc_transpose2d(x, out, x.shape[0], x.shape[1])
    return out


def concat_cols(a, b):
    a, b = f32(a), f32(b)
    out = np.empty((a.shape[0], a.shape[1] + b.shape[1]), np.float32)
    lib.orc_concat2(a, b, out, a.shape[0], a.shape[1], b.shape[1])
    return out


def concat_rows(a, b):
    a, b = f32(a), f32(b)
    out = np.empty((a.shape[0] + b.shape[0], a.shape[1]), np.float32)
    lib.orc_concat0(a, b, out, a.shape[0], b.shape[0], a.shape[1])
    return out


def slice_cols(x, cs, ce):
    x = f32(x)
    out = np.empty((x.shape[0], ce - cs), np.float32)
    lib.orc_slice2(x, out, x.shape[0], x.shape[1], cs, ce)
    return out


def slice_rows(x, rs, re):
    x = f32(x)
    out = np.empty((re - rs, x.shape[1]), np.float32)
    lib.orc_slicerows(x, out, x.shape[1], rs, re)
    return out


def index_cols(x, idx):
    x, idx = f32(x), _i64a(idx)
    out = np.empty((x.shape[0], idx.size), np.float32)
    lib.orc_index2(x, idx, out, x.shape[0], x.shape[1], idx.size)
    return out


def index_rows(x, idx):
    x, idx = f32(x), _i64a(idx)
    out = np.empty((idx.size, x.shape[1]), np.float32)
    lib.orc_indexrows(x, x.shape[0], idx, out, idx.size, x.shape[1])
    return out


def scatter_cols(x, idx, upd):
    x, idx, upd = f32(x), _i64a(idx), f32(upd)
    out = np.empty_like(x)
    lib.orc_scatter2(x, idx, upd, out, x.shape[0], x.shape[1], idx.size)
    return out


def scatter_rows(x, idx, upd):
    x, idx, upd = f32(x), _i64a(idx), f32(upd)
    out = np.empty_like(x)
    lib.orc_scatterrows(x, idx, upd, out, x.shape[0], x.shape[1], idx.size)
    return out


def dropout_mask(n, rate, k0, k1, step, site):
    out = np.empty(n, np.float32)
    lib.orc_dropout_mask(out, n, rate, k0, k1, step, site)
    return out
