"""ctypes bindings of the kernel-level C-ABI (include/ns_b200_ops.h) taking
torch CUDA tensors; device memory comes from torch (plumbing only)."""
from __future__ import annotations

import ctypes as C

from . import lib as _core_lib

F32, BF16 = 0, 1
AUTO, SIMT, TENSOR = 0, 1, 2

_sigs = {
    "nsb_op_gemm": (C.c_int, [C.c_int, C.c_int, C.c_int, C.c_void_p, C.c_int, C.c_longlong, C.c_int, C.c_void_p,
                              C.c_int, C.c_longlong, C.c_int, C.c_float, C.c_void_p, C.c_longlong, C.c_int,
                              C.c_void_p, C.c_longlong, C.c_void_p, C.c_longlong, C.c_int, C.c_void_p, C.c_size_t,
                              C.c_void_p, C.c_void_p]),
    "nsb_op_gemm_workspace_floats": (C.c_size_t, [C.c_int, C.c_int, C.c_int, C.c_void_p, C.c_int, C.c_longlong,
                                                  C.c_int, C.c_void_p, C.c_int, C.c_longlong, C.c_int, C.c_int]),
    "nsb_op_gemm_uses_tensor_cores": (C.c_int, [C.c_int, C.c_int, C.c_int, C.c_void_p, C.c_int, C.c_longlong,
                                                C.c_int, C.c_void_p, C.c_int, C.c_longlong, C.c_int, C.c_int]),
    "nsb_op_embedding_fwd": (C.c_int, [C.c_void_p, C.c_void_p, C.c_int, C.c_int, C.c_int, C.c_void_p, C.c_void_p,
                                       C.c_void_p]),
    "nsb_op_embedding_bwd_scratch_bytes": (C.c_size_t, [C.c_int, C.c_int]),
    "nsb_op_embedding_bwd": (C.c_int, [C.c_void_p, C.c_void_p, C.c_int, C.c_int, C.c_int, C.c_void_p, C.c_void_p,
                                       C.c_void_p]),
    "nsb_op_layernorm_fwd": (C.c_int, [C.c_void_p, C.c_int, C.c_int, C.c_void_p, C.c_void_p, C.c_void_p]),
    "nsb_op_layernorm_bwd": (C.c_int, [C.c_void_p, C.c_void_p, C.c_void_p, C.c_int, C.c_int, C.c_void_p, C.c_void_p,
                                       C.c_void_p]),
    "nsb_op_attention_fwd": (C.c_int, [C.c_int, C.c_int, C.c_int, C.c_int, C.c_int, C.c_void_p, C.c_longlong,
                                       C.c_void_p, C.c_longlong, C.c_void_p, C.c_void_p]),
    "nsb_op_attention_bwd": (C.c_int, [C.c_int, C.c_int, C.c_int, C.c_int, C.c_int, C.c_void_p, C.c_longlong,
                                       C.c_void_p, C.c_longlong, C.c_void_p, C.c_void_p, C.c_longlong, C.c_void_p,
                                       C.c_longlong, C.c_void_p, C.c_void_p]),
    "nsb_op_cross_entropy": (C.c_int, [C.c_void_p, C.c_void_p, C.c_void_p, C.c_int, C.c_int, C.c_float, C.c_void_p,
                                       C.c_void_p, C.c_void_p, C.c_void_p]),
    "nsb_op_reduce_sum": (C.c_int, [C.c_void_p, C.c_int, C.c_float, C.c_void_p, C.c_void_p]),
    "nsb_op_adamw": (C.c_int, [C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p, C.c_longlong, C.c_longlong,
                               C.c_float, C.c_float, C.c_float, C.c_float, C.c_float, C.c_float, C.c_float,
                               C.c_void_p]),
    "nsb_op_mgs": (C.c_int, [C.c_void_p, C.c_int, C.c_int, C.c_void_p]),
    "nsb_op_moe_route": (C.c_int, [C.c_void_p, C.c_void_p, C.c_void_p, C.c_int, C.c_int, C.c_int, C.c_void_p,
                                   C.c_void_p, C.c_void_p, C.c_void_p]),
    "nsb_op_act_fwd": (C.c_int, [C.c_void_p, C.c_size_t, C.c_int, C.c_void_p, C.c_void_p, C.c_void_p]),
    "nsb_op_act_bwd": (C.c_int, [C.c_void_p, C.c_void_p, C.c_int, C.c_size_t, C.c_void_p, C.c_void_p]),
}
_bound = None


def L():
    global _bound
    if _bound is None:
        lib = _core_lib()
        for n, (res, args) in _sigs.items():
            f = getattr(lib, n)
            f.restype = res
            f.argtypes = args
        _bound = lib
    return _bound


def p(t):
    return None if t is None else C.c_void_p(t.data_ptr())


def _stream():
    import torch
    return C.c_void_p(torch.cuda.current_stream().cuda_stream)


def _check(rc, what):
    if rc != 0:
        raise RuntimeError(f"{what} returned {rc}")


def _dt(t):
    import torch
    return BF16 if t.dtype == torch.bfloat16 else F32


def gemm(A, B, M, N, K, lda, a_mn, ldb, b_mn, alpha=1.0, add=None, act=0, c32=None, c16=None, engine=AUTO,
         err=None):
    """C = act(alpha * A.B^T + add); see include/ns_b200_ops.h for layouts."""
    import torch
    ws_n = L().nsb_op_gemm_workspace_floats(M, N, K, p(A), _dt(A), lda, a_mn, p(B), _dt(B), ldb, b_mn, engine)
    ws = torch.empty(max(ws_n, 1), dtype=torch.float32, device=A.device) if ws_n else None
    ld32 = c32.stride(0) if c32 is not None else 0
    ld16 = c16.stride(0) if c16 is not None else 0
    ldadd = add.stride(0) if add is not None else 0
    rc = L().nsb_op_gemm(M, N, K, p(A), _dt(A), lda, a_mn, p(B), _dt(B), ldb, b_mn, alpha, p(add), ldadd, act,
                         p(c32), ld32, p(c16), ld16, engine, p(ws), ws_n, p(err), _stream())
    _check(rc, "nsb_op_gemm")


def uses_tensor_cores(A, B, M, N, K, lda, a_mn, ldb, b_mn, engine=AUTO) -> bool:
    return bool(L().nsb_op_gemm_uses_tensor_cores(M, N, K, p(A), _dt(A), lda, a_mn, p(B), _dt(B), ldb, b_mn, engine))


def embedding_fwd(W, ids, out32=None, out16=None):
    V, D = W.shape
    _check(L().nsb_op_embedding_fwd(p(W), p(ids), ids.numel(), V, D, p(out32), p(out16), _stream()), "embedding_fwd")


def embedding_bwd(dout, ids, V, dW):
    import torch
    M, D = dout.shape
    n = L().nsb_op_embedding_bwd_scratch_bytes(M, V)
    scratch = torch.empty(n, dtype=torch.uint8, device=dout.device)
    _check(L().nsb_op_embedding_bwd(p(dout), p(ids), M, V, D, p(dW), p(scratch), _stream()), "embedding_bwd")


def layernorm_fwd(x, out32=None, out16=None):
    M, D = x.shape
    _check(L().nsb_op_layernorm_fwd(p(x), M, D, p(out32), p(out16), _stream()), "layernorm_fwd")


def layernorm_bwd(dy, x, add=None, dx32=None, dx16=None):
    M, D = x.shape
    _check(L().nsb_op_layernorm_bwd(p(dy), p(x), p(add), M, D, p(dx32), p(dx16), _stream()), "layernorm_bwd")


def attention_fwd(B, S, H, D, qkv, ctx, lse):
    _check(L().nsb_op_attention_fwd(B, S, H, D, _dt(qkv), p(qkv), qkv.stride(0), p(ctx), ctx.stride(0), p(lse),
                                    _stream()), "attention_fwd")


def attention_bwd(B, S, H, D, qkv, ctx, lse, dctx, dqkv, dvec):
    _check(L().nsb_op_attention_bwd(B, S, H, D, _dt(qkv), p(qkv), qkv.stride(0), p(ctx), ctx.stride(0), p(lse),
                                    p(dctx), dctx.stride(0), p(dqkv), dqkv.stride(0), p(dvec), _stream()),
           "attention_bwd")


def cross_entropy(logits, labels=None, targets=None, denom=None, row_loss=None, d32=None, d16=None):
    M, Cc = logits.shape
    _check(L().nsb_op_cross_entropy(p(logits), p(labels), p(targets), M, Cc, float(M if denom is None else denom),
                                    p(row_loss), p(d32), p(d16), _stream()), "cross_entropy")


def reduce_sum(x, scale, out):
    _check(L().nsb_op_reduce_sum(p(x), x.numel(), scale, p(out), _stream()), "reduce_sum")


def adamw(w, g, m, v, t, lr, beta1=0.9, beta2=0.999, omb1=0.1, omb2=0.001, eps=1e-8, decay=0.01):
    _check(L().nsb_op_adamw(p(w), p(g), p(m), p(v), w.numel(), t, lr, beta1, beta2, omb1, omb2, eps, decay,
                            _stream()), "adamw")


def mgs(G):
    r, c = G.shape
    _check(L().nsb_op_mgs(p(G), r, c, _stream()), "mgs")


def act_fwd(x, act, out32):
    _check(L().nsb_op_act_fwd(p(x), x.numel(), act, p(out32), None, _stream()), "act_fwd")


def act_bwd(dy, z, act, out32):
    _check(L().nsb_op_act_bwd(p(dy), p(z), act, dy.numel(), p(out32), _stream()), "act_bwd")


def moe_route(x, Wg, active, best, pb, probs=None):
    M, D = x.shape
    E = Wg.shape[1]
    _check(L().nsb_op_moe_route(p(x), p(Wg), p(active), M, D, E, p(best), p(pb), p(probs), _stream()), "moe_route")
