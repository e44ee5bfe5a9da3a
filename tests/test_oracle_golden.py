"""Pins the CPU oracle (oracle/) to golden vectors produced by the reference's
own emitted code (tests/golden/golden.npz, made by tests/golden/gen_golden.py).

Kernel-level cases compare against the reference's static helpers; ABI-level
cases compare a model-level composition of the oracle against the
reference's compiled runtime driver (forward, 30-40 train steps with the
reference optimizer, MoE expert lifecycle, NSM2 checkpoint bytes).
"""
import os
import struct

import numpy as np
import pytest

import oracle_lib as O
from model_oracle import OracleModel, make_weights
from neuralscript_b200 import synth
from neuralscript_b200.spec import C1, C2, C3, parse
from specs import TMLP, TMOE, TTFM

G = np.load(os.path.join(os.path.dirname(__file__), "golden", "golden.npz"))


def close(a, b, rtol=1e-6, atol=1e-6):
    np.testing.assert_allclose(np.asarray(a, np.float64), np.asarray(b, np.float64), rtol=rtol, atol=atol)


def test_generator_matches_numpy():
    for seed in (0, 7, 12345):
        assert np.array_equal(O.fill_uniform(1000, seed, -1, 1), synth.uniform(1000, seed, -1, 1))
        assert np.array_equal(O.fill_normal(1000, seed, 0.3, 0.02), synth.normal(1000, seed, 0.3, 0.02))
        assert np.array_equal(O.fill_tokens(1000, seed, 8192), synth.tokens(1000, seed, 8192))
    x = synth.normal(200000, 3)
    assert abs(float(x.mean())) < 0.01 and abs(float(x.std()) - 1.0) < 0.01


def test_matmul_and_grads():
    A, B, dC = synth.uniform(37 * 29, 101, -1, 1).reshape(37, 29), synth.uniform(29 * 23, 102, -1, 1).reshape(29, 23), \
        synth.uniform(37 * 23, 103, -1, 1).reshape(37, 23)
    assert np.array_equal(O.matmul(A, B), G["matmul_C"])
    assert np.array_equal(O.matmul_grad_a(dC, B), G["matmul_dA"])
    # GCC's code for the reference's k-j-i loop nest does not round like a
    # plain sequential chain; the values agree to a few ulp
    close(O.matmul_grad_w(A, dC), G["matmul_dB"], rtol=1e-6, atol=1e-6)


def test_activations():
    x = synth.uniform(2000, 110, -6, 6)
    for c in range(7):
        assert np.array_equal(O.act(x, c), G["act_y"][c]), c
        assert np.array_equal(O.act_deriv(x, c), G["act_dy"][c]), c


def test_layernorm_softmax():
    x = synth.normal(13 * 48, 120, 0.3, 2.0).reshape(13, 48)
    d = synth.normal(13 * 48, 121, 0, 1).reshape(13, 48)
    assert np.array_equal(O.layernorm(x), G["ln_y"])
    assert np.array_equal(O.layernorm_grad(d, x), G["ln_dx"])
    assert np.array_equal(O.softmax(synth.normal(60, 190, 0, 3).reshape(6, 10)), G["softmax_y"])


def test_embedding_with_out_of_range_ids():
    idx = np.array([0, 3, 10, -1, 11, 3.7, 2.2, 5, 5, 0, -0.5, 7], np.float32)
    W = synth.normal(88, 130, 0, 1).reshape(11, 8)
    d = synth.normal(idx.size * 8, 131, 0, 1).reshape(-1, 8)
    assert np.array_equal(O.embedding(W, idx), G["emb_out"])
    assert np.array_equal(O.embedding_grad_w(d, idx, 11), G["emb_dW"])


@pytest.mark.parametrize("tag,B,S,D,H,seed", [("attn_a", 3, 8, 16, 4, 140), ("attn_b", 2, 64, 64, 2, 240)])
def test_attention(tag, B, S, D, H, seed):
    BS = B * S
    x = synth.normal(BS * D, seed, 0, 1).reshape(BS, D)
    Ws = [synth.normal(D * D, seed + i, 0, 0.25).reshape(D, D) for i in range(1, 5)]
    dout = synth.normal(BS * D, seed + 5, 0, 1).reshape(BS, D)
    assert np.array_equal(O.attention_fwd(x, *Ws, H, S), G[f"{tag}_out"])
    dX, dq, dk, dv, do = O.attention_bwd(dout, x, *Ws, H, S)
    for got, name in ((dX, "dX"), (dq, "dWq"), (dk, "dWk"), (dv, "dWv"), (do, "dWo")):
        assert np.array_equal(got, G[f"{tag}_{name}"]), name


def test_moe_forward_and_grads():
    M, D, E, H = 37, 8, 4, 16
    act = np.array([1, 1, 0, 1], np.uint8)
    x = synth.normal(M * D, 150, 0, 1).reshape(M, D)
    Wg = synth.normal(D * E, 151, 0, 0.5).reshape(D, E)
    We1 = synth.normal(E * D * H, 152, 0, 0.35).reshape(E, D * H)
    We2 = synth.normal(E * H * D, 153, 0, 0.35).reshape(E, H * D)
    dout = synth.normal(M * D, 154, 0, 1).reshape(M, D)
    assert np.array_equal(O.moe_fwd(x, Wg, We1, We2, H, act), G["moe_out"])
    dx, dwg, dwe1, dwe2 = O.moe_grads(dout, x, Wg, We1, We2, H, act)
    close(dx, G["moe_dx"], rtol=1e-5, atol=1e-6)
    close(dwg, G["moe_dWg"], rtol=1e-5, atol=1e-6)
    close(dwe1, G["moe_dWe1"], rtol=1e-5, atol=1e-6)
    close(dwe2, G["moe_dWe2"], rtol=1e-5, atol=1e-6)
    best, _, _ = O.moe_route(x, Wg, act)
    assert not np.any(best == 2)  # the dead expert never wins


def test_routing_at_config3_router_scale():
    M, D, E, H = 1024, 1024, 8, 8
    x = synth.normal(M * D, 160, 0, 1).reshape(M, D)
    Wg = synth.normal(D * E, 161, 0, 0.02).reshape(D, E)
    We1 = synth.normal(E * D * H, 162, 0, 1 / 32).reshape(E, D * H)
    We2 = synth.normal(E * H * D, 163, 0, 1 / 32).reshape(E, H * D)
    out = O.moe_fwd(x, Wg, We1, We2, H)
    assert np.array_equal(out.astype(np.float64).sum(axis=1), G["route_rowsum"])


def test_cross_entropy():
    p = synth.normal(63, 170, 0, 2).reshape(9, 7)
    y = np.zeros((9, 7), np.float32)
    y[np.arange(9), (np.arange(9) * 3) % 7] = 1
    assert np.array_equal(O.loss_grad(p, y), G["ce_d"])
    assert np.float32(O.cross_entropy(p, y)) == G["ce_loss"][0]


def test_mgs():
    assert np.array_equal(O.orthonom(synth.normal(108, 180, 0, 1).reshape(12, 9)), G["mgs_a"])
    assert np.array_equal(O.orthonom(synth.normal(55, 181, 0, 1).reshape(5, 11)), G["mgs_b"])


def test_lr_schedule_formula():
    # optim_params.hpp:54-62 restated: warmup ramp, cosine to min_factor
    assert O.lr_schedule(0, 0) == 1.0
    assert O.lr_schedule(0, 1) == 0.0
    assert O.lr_schedule(50, 1) == np.float32(0.5)
    assert abs(O.lr_schedule(100, 1) - 1.0) < 1e-6
    assert abs(O.lr_schedule(10000, 1) - 0.05) < 1e-6
    assert abs(O.lr_schedule(20000, 1) - 0.05) < 1e-6
    mid = O.lr_schedule(5050, 1)
    assert abs(mid - (0.05 + 0.5 * 0.95 * (1 + np.cos(np.pi * 0.5)))) < 1e-5


def test_c1_forward():
    w = make_weights(C1, 211, sds=[1 / 28.0, 1 / 32.0, 1 / 32.0])
    x = synth.uniform(64 * 784, 201, -1, 1)
    out = OracleModel(C1, w).forward(x)
    assert np.array_equal(out, G["c1_out"])


def test_c2_forward_per_sequence():
    w = make_weights(C2, 311, default_sd=0.02)
    tok = synth.tokens(512, 301, 8192)
    out = OracleModel(C2, w).forward(tok)  # seq=256: same as one reference call per sequence
    close(out.astype(np.float64).sum(axis=1), G["c2_rowsum"], rtol=1e-5, atol=1e-4)
    close(np.concatenate([out[:128], out[256:384]]), G["c2_rows"], rtol=1e-5, atol=1e-5)


def test_c3_forward():
    w = make_weights(C3, 411, sds=[0.02, 1 / 32.0, 1 / 32.0])
    x = synth.normal(64 * 1024, 401, 0, 1)
    out = OracleModel(C3, w).forward(x)
    # float work: within a few ulps (rows 32..63 differ from the reference
    # emit by one ulp in places; routing is pinned bit-exactly elsewhere)
    close(out.astype(np.float64).sum(axis=1), G["c3_rowsum"], rtol=1e-6, atol=1e-5)
    close(out, G["c3_rows"], rtol=1e-6, atol=2e-7)


def test_binops_match_reference_helper():
    a, b = G["binop_a"], G["binop_b"]
    assert np.array_equal(a, synth.uniform(7 * 13, 190, -2, 2).reshape(7, 13))
    for code in range(4):
        out = np.empty_like(a)
        O.lib.orc_binop(a.reshape(-1), a.size, b.reshape(-1), b.size, out.reshape(-1), code)
        assert np.array_equal(out, G[f"binop_{code}"]), code


def test_data_movement_matches_reference_helpers():
    """The reference's CPU data-movement helpers on a [9, 11] tensor; the
    scatters repeat an index, which pins their last-write order."""
    X, Y, Z = G["dm_x"], G["dm_y"], G["dm_z"]
    assert np.array_equal(X, synth.uniform(9 * 11, 195, -1, 1).reshape(9, 11))
    assert np.array_equal(O.transpose2d(X), G["dm_transpose"])
    assert np.array_equal(O.concat_cols(X, Y), G["dm_concat2"])
    assert np.array_equal(O.concat_rows(X, Z), G["dm_concat0"])
    assert np.array_equal(O.slice_cols(X, 3, 9), G["dm_slice2"])
    assert np.array_equal(O.slice_rows(X, 2, 5), G["dm_slicerows"])
    assert np.array_equal(O.index_cols(X, [7, 2, 7, 0]), G["dm_index2"])
    assert np.array_equal(O.index_rows(X, [5, 1, 5]), G["dm_indexrows"])
    assert np.array_equal(O.scatter_cols(X, [3, 9, 3, 1, 10], Y), G["dm_scatter2"])
    assert np.array_equal(O.scatter_rows(X, [2, 6, 2, 8], Z), G["dm_scatterrows"])


def _philox_py(c, k):
    """Philox4x32-10 written independently in Python (Salmon et al., SC 2011)."""
    c = list(c)
    k0, k1 = k
    for _ in range(10):
        p0, p1 = 0xD2511F53 * c[0], 0xCD9E8D57 * c[2]
        c = [(p1 >> 32) ^ c[1] ^ k0, p1 & 0xFFFFFFFF, (p0 >> 32) ^ c[3] ^ k1, p0 & 0xFFFFFFFF]
        k0, k1 = (k0 + 0x9E3779B9) & 0xFFFFFFFF, (k1 + 0xBB67AE85) & 0xFFFFFFFF
    return c


def test_philox_known_answers_and_dropout_mask():
    """The published Philox4x32-10 known-answer vectors (Random123), then the
    C oracle's dropout mask against masks derived from this Python Philox."""
    assert _philox_py([0, 0, 0, 0], [0, 0]) == [0x6627E8D5, 0xE169C58D, 0xBC57AC4C, 0x9B00DBD8]
    assert _philox_py([0xFFFFFFFF] * 4, [0xFFFFFFFF] * 2) == [0x408F276D, 0x41C83B0E, 0xA20BC7C6, 0x6D5451FD]
    assert _philox_py([0x243F6A88, 0x85A308D3, 0x13198A2E, 0x03707344], [0xA4093822, 0x299F31D0]) == \
        [0xD16CFE09, 0x94FDCCEB, 0x5001E420, 0x24126EA1]
    rate, k0, k1, step, site = 0.3, 0x243F6A88, 0x85A308D3, 7, 2
    n = 1003
    got = O.dropout_mask(n, rate, k0, k1, step, site)
    exp = np.empty(n, np.float32)
    for q in range((n + 3) // 4):
        w = _philox_py([q & 0xFFFFFFFF, q >> 32, step, site], [k0, k1])
        for j in range(4):
            if 4 * q + j < n:
                u = np.float32(w[j] >> 8) * np.float32(1.0 / 16777216.0)
                exp[4 * q + j] = np.float32(1.0) / np.float32(1.0 - np.float32(rate)) if u >= np.float32(rate) else 0.0
    assert np.array_equal(got, exp)
    big = O.dropout_mask(1 << 20, rate, k0, k1, 1, 0)
    keep = float(np.mean(big > 0))
    assert abs(keep - 0.7) < 3e-3  # ~6 sigma for 2^20 Bernoulli(0.7) draws
    assert np.allclose(big[big > 0], 1.0 / 0.7)


SMALL = {
    "tmlp": (TMLP, [0.41, 0.25, 0.35], 501, lambda: synth.uniform(96, 502, -1, 1), 503, 4, 40, 0.05),
    "ttfm": (TTFM, [0.5, 0.4, 0.4, 0.4, 0.4, 0.4, 0.3, 0.4], 601, lambda: synth.tokens(64, 602, 32), 603, 16,
             30, 0.01),
    "tmoe": (TMOE, [0.5, 0.5, 0.35, 0.25, 0.35], 701, lambda: synth.tokens(24, 702, 16), 703, 4, 30, 0.01),
}


@pytest.mark.parametrize("tag", sorted(SMALL))
def test_train_matches_reference_runtime(tag):
    spec, sds, wseed, xf, lseed, classes, steps, lr = SMALL[tag]
    w = make_weights(spec, wseed, sds=sds)
    assert np.array_equal(w, G[f"{tag}_w0"])
    x = xf()
    assert np.array_equal(x, G[f"{tag}_x"])
    s = parse(spec)
    rows = x.size // s.in_cols
    y = synth.one_hot(synth.tokens(rows, lseed, classes), classes)
    assert np.array_equal(y, G[f"{tag}_y"])
    m = OracleModel(spec, w)
    losses = np.array([m.train_step(x, y, lr) for _ in range(steps)], np.float32)
    # ulp-level differences (gradient loop rounding) grow slowly through the
    # Gram-Schmidt updates over the run
    close(losses, G[f"{tag}_losses"], rtol=1e-4, atol=1e-5)
    close(m.w, G[f"{tag}_w"], rtol=1e-3, atol=5e-4)
    close(m.objective(x, y), G[f"{tag}_obj"][0], rtol=1e-4, atol=1e-5)
    close(m.forward(x), G[f"{tag}_out"], rtol=1e-3, atol=5e-4)


def test_checkpoint_format_nsm2():
    # NSM2: u32 magic, size_t count, floats, then (MoE) u32 n_layers, size_t cap, mask
    b = G["tmlp_ckpt_bytes"].astype(np.uint8).tobytes()
    magic, n = struct.unpack("<IQ", b[:12])
    assert magic == 0x4E534D32 and n == G["tmlp_w"].size and len(b) == 12 + 4 * n
    assert np.array_equal(np.frombuffer(b[12:], np.float32), G["tmlp_w"])
    b = G["tmoe_lifecycle_ckpt_bytes"].astype(np.uint8).tobytes()
    magic, n = struct.unpack("<IQ", b[:12])
    nl, cap = struct.unpack("<IQ", b[12 + 4 * n:12 + 4 * n + 12])
    assert (magic, nl, cap) == (0x4E534D32, 1, 4)
    assert list(b[12 + 4 * n + 12:]) == [1, 0, 0, 0]  # kill(1), merge(0,2) from {0,1,2}


def test_moe_lifecycle_counts():
    # count 3 -> kill(1) 2 -> kill(1) again 2 -> merge(0,2) 1 -> merge(0,0) 1
    assert list(G["tmoe_lifecycle_counts"]) == [3, 2, 2, 1, 1]
