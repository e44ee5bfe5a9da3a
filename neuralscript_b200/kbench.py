"""Kernel micro-benchmarks: time one hot-path kernel family through the
kernel-level C-ABI (include/ns_b200_ops.h) on synthetic operands, with CUDA
events on the launching stream after warm-up.

    python -m neuralscript_b200.kbench gemm --M 16384 --N 2048 --K 512 --act gelu
    python -m neuralscript_b200.kbench gemm --M 16384 --N 8192 --K 512 --out f32
    python -m neuralscript_b200.kbench gemm_ln --M 16384 --K 2048
    python -m neuralscript_b200.kbench attention --B 64 --S 256 --H 8 --D 512
    python -m neuralscript_b200.kbench layernorm --M 16384 --D 512
    python -m neuralscript_b200.kbench ce --M 16384 --C 8192
    python -m neuralscript_b200.kbench embedding --M 16384 --V 8192 --D 512 --backward
    python -m neuralscript_b200.kbench adamw --n 11534336

Prints one JSON line per run: average launch time, achieved TFLOP/s or GB/s
and the fraction of the measured peak (MEASURED_PEAKS.json).
"""
from __future__ import annotations

import argparse
import json
import os

ACTS = {"none": 0, "relu": 1, "gelu": 6}
ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            return json.load(f), "measured"
    except Exception:
        return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0}, "fallback"


def _time(fn, iters, warmup=3):
    import torch
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(iters):
        fn()
    e1.record()
    torch.cuda.synchronize()
    return e0.elapsed_time(e1) / iters / 1e3


def gemm_case(M, N, K, act="none", dtype="bf16", iters=20, out="bf16", residual=False, a_mn=0, b_mn=1):
    """C[M,N] = A B^T with A stored [M,K] (K-major) or [K,M] (a_mn=1) and B
    stored [N,K] or [K,N] (b_mn=1). Defaults are the engine's forward layout
    (W [K,N] row-major); input gradients use a_mn=0, b_mn=0 and weight
    gradients a_mn=1, b_mn=1. Output bf16 or fp32, optionally plus an fp32
    residual [M,N]."""
    import torch
    from . import ops as O
    dt = torch.bfloat16 if dtype == "bf16" else torch.float32
    A = torch.randn(*((K, M) if a_mn else (M, K)), device="cuda").to(dt)
    B = torch.randn(*((K, N) if b_mn else (N, K)), device="cuda").to(dt)
    kw = {"act": ACTS[act]}
    if out == "bf16":
        kw["c16"] = torch.empty(M, N, device="cuda", dtype=torch.bfloat16)
    else:
        kw["c32"] = torch.empty(M, N, device="cuda")
    if residual:
        kw["add"] = torch.randn(M, N, device="cuda")
    lda, ldb = A.stride(0), B.stride(0)
    t = _time(lambda: O.gemm(A, B, M, N, K, lda, a_mn, ldb, b_mn, **kw), iters)
    pk, kind = _peaks()
    tf = 2.0 * M * N * K / t / 1e12
    return {"kernel": "gemm", "M": M, "N": N, "K": K, "act": act, "dtype": dtype, "out": out,
            "residual": residual, "us": t * 1e6, "tflops": tf, "frac_of_bf16_peak": tf / pk["bf16_tflops"],
            "a_mn": a_mn, "b_mn": b_mn, "peak_kind": kind,
            "tensor_cores": O.uses_tensor_cores(A, B, M, N, K, lda, a_mn, ldb, b_mn)}


def attention_case(B, S, H, D, iters=20, backward=False):
    import torch
    from . import ops as O
    qkv = torch.randn(B * S, 3 * D, device="cuda").bfloat16()
    ctx = torch.empty(B * S, D, device="cuda", dtype=torch.bfloat16)
    lse = torch.empty(B * H * S, device="cuda")
    t = _time(lambda: O.attention_fwd(B, S, H, D, qkv, ctx, lse), iters)
    fl = 4.0 * B * H * S * S * (D // H)
    res = {"kernel": "attention_fwd", "B": B, "S": S, "H": H, "D": D, "us": t * 1e6, "tflops": fl / t / 1e12}
    if backward:
        g = torch.randn(B * S, D, device="cuda").bfloat16()
        dq = torch.empty(B * S, 3 * D, device="cuda", dtype=torch.bfloat16)
        dv = torch.empty(B * H * S, device="cuda")
        tb = _time(lambda: O.attention_bwd(B, S, H, D, qkv, ctx, lse, g, dq, dv), iters)
        res.update({"bwd_us": tb * 1e6, "bwd_tflops": 2.5 * fl / tb / 1e12})
    return res


def layernorm_case(M, D, iters=50):
    import torch
    from . import ops as O
    x = torch.randn(M, D, device="cuda")
    y = torch.empty_like(x)
    y16 = torch.empty(M, D, device="cuda", dtype=torch.bfloat16)
    t = _time(lambda: O.layernorm_fwd(x, y, y16), iters)
    pk, kind = _peaks()
    gbs = (M * D * (4 + 4 + 2)) / t / 1e9
    return {"kernel": "layernorm_fwd", "M": M, "D": D, "us": t * 1e6, "gbs": gbs,
            "frac_of_hbm": gbs / pk["hbm_gbs"], "peak_kind": kind}


def cross_entropy_case(M, C, iters=20):
    """Single-pass CE over fp32 logits [M, C] with int32 targets, bf16 seed gradient."""
    import torch
    from . import ops as O
    logits = torch.randn(M, C, device="cuda")
    tgt = torch.randint(0, C, (M,), device="cuda", dtype=torch.int32)
    row = torch.empty(M, device="cuda")
    d16 = torch.empty(M, C, device="cuda", dtype=torch.bfloat16)
    t = _time(lambda: O.cross_entropy(logits, targets=tgt, row_loss=row, d16=d16), iters)
    pk, kind = _peaks()
    gbs = M * C * (4 + 2) / t / 1e9
    return {"kernel": "cross_entropy", "M": M, "C": C, "us": t * 1e6, "gbs": gbs, "frac_of_hbm": gbs / pk["hbm_gbs"],
            "peak_kind": kind}


def cross_entropy_finish_case(M, C, iters=20):
    """The loss pass of the fused head: fp16 logits [M, C] read, the bf16 seed
    gradient written over them in place, one loss per row. The pass rewrites
    its input, so later iterations read the previous seed as fp16 (finite
    values; the work per element does not depend on them). Bytes: 2 read +
    2 written per element."""
    import ctypes as C_
    import torch
    from . import ops as O
    L = O.L()
    L.nsb_op_cross_entropy_finish.restype = C_.c_int
    vp = C_.c_void_p
    L.nsb_op_cross_entropy_finish.argtypes = [vp, C_.c_int, C_.c_int, vp, vp, C_.c_float, vp, vp]
    g = (torch.randn(M, C, device="cuda") * 3).half()
    tgt = torch.randint(0, C, (M,), device="cuda", dtype=torch.int32)
    tl = torch.randn(M, device="cuda")
    row = torch.empty(M, device="cuda")
    P = lambda t: C_.c_void_p(t.data_ptr())

    def run():
        rc = L.nsb_op_cross_entropy_finish(P(g), M, C, P(tgt), P(tl), float(M), P(row),
                                           C_.c_void_p(torch.cuda.current_stream().cuda_stream))
        assert rc == 0, rc

    t = _time(run, iters)
    pk, kind = _peaks()
    gbs = M * C * 4 / t / 1e9
    return {"kernel": "cross_entropy_finish", "M": M, "C": C, "us": t * 1e6, "gbs": gbs,
            "frac_of_hbm": gbs / pk["hbm_gbs"], "peak_kind": kind}


def embedding_case(M, V, D, iters=20, backward=False):
    """Gather (fp32 + bf16 out) and the deterministic sort-then-segment gradient."""
    import torch
    from . import ops as O
    W = torch.randn(V, D, device="cuda")
    ids = torch.randint(0, V, (M,), device="cuda").float()
    o32 = torch.empty(M, D, device="cuda")
    o16 = torch.empty(M, D, device="cuda", dtype=torch.bfloat16)
    t = _time(lambda: O.embedding_fwd(W, ids, o32, o16), iters)
    pk, kind = _peaks()
    res = {"kernel": "embedding_fwd", "M": M, "V": V, "D": D, "us": t * 1e6,
           "gbs": M * D * (4 + 4 + 2) / t / 1e9, "peak_kind": kind}
    res["frac_of_hbm"] = res["gbs"] / pk["hbm_gbs"]
    if backward:
        dW = torch.empty(V, D, device="cuda")
        tb = _time(lambda: O.embedding_bwd(o32, ids, V, dW), iters)
        res.update({"bwd_us": tb * 1e6, "bwd_gbs": (M * D + V * D) * 4 / tb / 1e9})
    return res


def adamw_case(n, iters=20):
    """One AdamW tensor of n parameters (w, g, m, v read; w, m, v written)."""
    import torch
    from . import ops as O
    w, g, m, v = (torch.randn(n, device="cuda") for _ in range(4))
    v.abs_()
    t = _time(lambda: O.adamw(w, g, m, v, 1, 1e-4), iters)
    pk, kind = _peaks()
    gbs = n * 4 * 7 / t / 1e9
    return {"kernel": "adamw", "n": n, "us": t * 1e6, "gbs": gbs, "frac_of_hbm": gbs / pk["hbm_gbs"], "peak_kind": kind}


def gemm_layernorm_case(M, K, iters=20):
    """C[M,512] = LayerNorm(A B + residual) in one GEMM (the out-projection /
    ff2 + residual + LayerNorm of the c2/c4 block): bf16 A [M,K] K-major,
    B [K,512] MN-major, fp32 residual; fp32 and bf16 outputs and 1/sigma.
    Bytes: A + residual read, both outputs written (the tensor-or-HBM floor
    is the larger of FLOPs / peak and bytes / bandwidth)."""
    import ctypes as C
    import torch
    from . import ops as O
    L = O.L()
    L.nsb_op_gemm_layernorm.restype = C.c_int
    vp, ll = C.c_void_p, C.c_longlong
    L.nsb_op_gemm_layernorm.argtypes = [C.c_int, C.c_int, vp, C.c_int, ll, vp, ll, C.c_float, vp, ll, vp, ll, vp,
                                        ll, vp, vp, vp]
    A = torch.randn(M, K, device="cuda").bfloat16()
    B = (torch.randn(K, 512, device="cuda") * 0.05).bfloat16()
    add = torch.randn(M, 512, device="cuda")
    c32 = torch.empty(M, 512, device="cuda")
    c16 = torch.empty(M, 512, device="cuda", dtype=torch.bfloat16)
    rstd = torch.empty(M, device="cuda")
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    P = lambda t: C.c_void_p(t.data_ptr())

    def run():
        rc = L.nsb_op_gemm_layernorm(M, K, P(A), 1, K, P(B), 512, 1.0, P(add), 512, P(c32), 512, P(c16), 512,
                                     P(rstd), P(err), C.c_void_p(torch.cuda.current_stream().cuda_stream))
        assert rc == 0, rc

    t = _time(run, iters)
    pk, kind = _peaks()
    fl = 2.0 * M * 512 * K
    by = M * K * 2 + M * 512 * 4 + M * 512 * (4 + 2) + M * 4
    floor = max(fl / (pk["bf16_tflops"] * 1e12), by / (pk["hbm_gbs"] * 1e9))
    return {"kernel": "gemm_layernorm", "M": M, "N": 512, "K": K, "us": t * 1e6, "tflops": fl / t / 1e12,
            "gbs": by / t / 1e9, "floor_us": floor * 1e6, "frac_of_floor": floor / t, "peak_kind": kind}


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("kernel", choices=["gemm", "gemm_ln", "attention", "layernorm", "ce", "ce_finish", "embedding", "adamw"])
    ap.add_argument("--C", type=int, default=8192)
    ap.add_argument("--V", type=int, default=8192)
    ap.add_argument("--n", type=int, default=11_534_336)
    ap.add_argument("--M", type=int, default=16384)
    ap.add_argument("--N", type=int, default=2048)
    ap.add_argument("--K", type=int, default=512)
    ap.add_argument("--act", default="none", choices=sorted(ACTS))
    ap.add_argument("--dtype", default="bf16", choices=["bf16", "tf32"])
    ap.add_argument("--B", type=int, default=64)
    ap.add_argument("--S", type=int, default=256)
    ap.add_argument("--H", type=int, default=8)
    ap.add_argument("--D", type=int, default=512)
    ap.add_argument("--iters", type=int, default=20)
    ap.add_argument("--backward", action="store_true")
    ap.add_argument("--out", default="bf16", choices=["bf16", "f32"])
    ap.add_argument("--residual", action="store_true")
    ap.add_argument("--a-mn", type=int, default=0)
    ap.add_argument("--b-mn", type=int, default=1)
    a = ap.parse_args()
    if a.kernel == "gemm":
        r = gemm_case(a.M, a.N, a.K, a.act, a.dtype, a.iters, a.out, a.residual, a.a_mn, a.b_mn)
    elif a.kernel == "gemm_ln":
        r = gemm_layernorm_case(a.M, a.K, a.iters)
    elif a.kernel == "attention":
        r = attention_case(a.B, a.S, a.H, a.D, a.iters, a.backward)
    elif a.kernel == "layernorm":
        r = layernorm_case(a.M, a.D, a.iters)
    elif a.kernel == "ce":
        r = cross_entropy_case(a.M, a.C, a.iters)
    elif a.kernel == "ce_finish":
        r = cross_entropy_finish_case(a.M, a.C, a.iters)
    elif a.kernel == "embedding":
        r = embedding_case(a.M, a.V, a.D, a.iters, a.backward)
    else:
        r = adamw_case(a.n, a.iters)
    print(json.dumps(r))


if __name__ == "__main__":
    main()
