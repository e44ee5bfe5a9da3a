"""Model-level parity on the GPU through the C-ABI: the drop-in ns_runtime.h
libraries against the reference's own outputs (tests/golden), and the
engine against the model-level oracle for what the reference cannot run
(per-sequence attention with residuals, AdamW/cosine configuration modes).

Tolerances (relative Frobenius norm) on forward activations: pure-fp32
SIMT mode 1e-5; the tensor-core modes 2e-3 (the contract's bound) in each
configuration's contract mode: bf16 for the config-2 block, TF32 for the
config-1 MLP. bf16 on config 1 is held to 6e-3 and documented as outside
the contract: three chained GEMMs over bf16-rounded operands put its output
about 4.6e-3 from fp32 by rounding alone. Losses after training as stated
per test (1e-3 relative over 100 steps in the tensor-core modes).
"""
import os
import struct

import numpy as np
import pytest

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

import neuralscript_b200 as nsb  # noqa: E402
from model_oracle import OracleModel, make_weights  # noqa: E402
from neuralscript_b200 import synth  # noqa: E402
from neuralscript_b200.spec import C1, C2, parse  # noqa: E402
from specs import SMALL, TMLP, TTFM  # noqa: E402

G = np.load(os.path.join(os.path.dirname(__file__), "golden", "golden.npz"))
TOL = {"fp32": 1e-5, "tf32": 2e-3, "bf16": 2e-3}
C1_TOL = {"fp32": 1e-5, "tf32": 2e-3, "bf16": 6e-3}


def relerr(a, b):
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30))


@pytest.fixture
def precision_env():
    old = os.environ.get("NS_B200_PRECISION")
    yield
    if old is None:
        os.environ.pop("NS_B200_PRECISION", None)
    else:
        os.environ["NS_B200_PRECISION"] = old


@pytest.mark.parametrize("mode", ["fp32", "tf32", "bf16"])
def test_c1_dropin_abi_matches_reference(mode, precision_env):
    """libns_c1.so through the reference's own entry-point names."""
    os.environ["NS_B200_PRECISION"] = mode
    L = nsb.RuntimeLib("c1")
    w = make_weights(C1, 211, sds=[1 / 28.0, 1 / 32.0, 1 / 32.0])
    x = synth.uniform(64 * 784, 201, -1, 1)
    m = L.ns_runtime_init(w.ctypes.data, w.size)
    assert m
    out = np.empty(64 * 10, np.float32)
    assert L.ns_eval_infer(m, x.ctypes.data, out.ctypes.data, x.size) == 0
    assert L.ns_model_output_numel(m, x.size) == 640
    e = relerr(out.reshape(64, 10), G["c1_out"])
    L.ns_free(m)
    assert e < C1_TOL[mode], e


@pytest.mark.parametrize("mode", ["fp32", "tf32"])
def test_c1_full_batch_matches_oracle(mode, precision_env):
    """The config-1 batch (4096 rows) in its contract modes through the
    drop-in ABI, against the oracle on every 16th row (rows are independent)."""
    os.environ["NS_B200_PRECISION"] = mode
    L = nsb.RuntimeLib("c1")
    w = make_weights(C1, 212, sds=[1 / 28.0, 1 / 32.0, 1 / 32.0])
    x = synth.uniform(4096 * 784, 202, -1, 1)
    m = L.ns_runtime_init(w.ctypes.data, w.size)
    out = np.empty(4096 * 10, np.float32)
    assert L.ns_eval_infer(m, x.ctypes.data, out.ctypes.data, x.size) == 0
    L.ns_free(m)
    sample = x.reshape(4096, 784)[::16]
    exp = OracleModel(C1, w).forward(sample)
    assert relerr(out.reshape(4096, 10)[::16], exp) < TOL[mode]


@pytest.mark.parametrize("mode", ["fp32", "tf32", "bf16"])
def test_c2_forward_matches_reference(mode):
    """Config-2 block on two 256-token sequences vs the reference CPU emit
    called once per sequence: 256 rows (the first 128 of each sequence)."""
    w = make_weights(C2, 311, default_sd=0.02)
    tok = synth.tokens(512, 301, 8192)
    m = nsb.Model(C2, w, precision=mode)
    out = m.infer(tok)
    rows = np.concatenate([out[:128], out[256:384]])
    assert relerr(rows, G["c2_rows"]) < TOL[mode]
    for r in range(0, 256, 8):  # and row by row on a sample
        assert relerr(rows[r], G["c2_rows"][r]) < 2 * TOL[mode], r
    rs = out.astype(np.float64).sum(axis=1)
    # LayerNorm outputs have ~zero row sums; compare them absolutely
    assert np.max(np.abs(rs - G["c2_rowsum"])) < (1e-3 if mode == "fp32" else 0.05)


@pytest.mark.parametrize("mode", ["tf32", "bf16"])
def test_c2_forward_full_batch_matches_oracle(mode):
    """64 x 256 tokens (the config-2 batch) against the oracle on 4
    sequences spread over the batch (the oracle is too slow for all 64);
    rows are independent across sequences, so a sample pins the batch."""
    w = make_weights(C2, 311, default_sd=0.02)
    tok = synth.tokens(64 * 256, 302, 8192)
    m = nsb.Model(C2, w, precision=mode)
    out = m.infer(tok)
    seqs = [0, 21, 42, 63]
    sel = np.concatenate([np.arange(q * 256, (q + 1) * 256) for q in seqs])
    ref = OracleModel(C2, w).forward(tok[sel])
    assert relerr(out[sel], ref) < TOL[mode]
    assert np.all(np.isfinite(out))


def test_c2_pipelined_host_inference_equals_one_pass():
    """ns_eval_infer into page-locked host memory splits the batch into row
    chunks and copies each chunk's output back while the next one computes;
    rows are independent, so it matches the single-pass result (pageable
    output) up to the fp32 summation order of a GEMM whose K is split at the
    smaller row count."""
    w = make_weights(C2, 311, default_sd=0.02)
    tok = synth.tokens(64 * 256, 303, 8192)
    m = nsb.Model(C2, w, precision="bf16")
    one = m.infer(tok).copy()
    pinned = torch.empty(64 * 256 * 512, dtype=torch.float32).pin_memory().numpy()
    got = m.infer(tok, pinned).copy()
    assert np.allclose(got, one, rtol=1e-5, atol=1e-5), float(np.max(np.abs(got - one)))
    got2 = m.infer(tok, pinned)  # second call reuses the staging buffer and events
    assert np.array_equal(got2, got)


@pytest.mark.parametrize("tag", ["tmlp", "ttfm"])
def test_train_fp32_matches_reference_runtime(tag):
    spec = SMALL[tag]
    if tag == "tmlp":
        w = make_weights(spec, 501, sds=[0.41, 0.25, 0.35])
        x, steps, lr, classes = synth.uniform(96, 502, -1, 1), 40, 0.05, 4
    else:
        w = make_weights(spec, 601, sds=[0.5, 0.4, 0.4, 0.4, 0.4, 0.4, 0.3, 0.4])
        x, steps, lr, classes = synth.tokens(64, 602, 32), 30, 0.01, 16
    rows = x.size // parse(spec).in_cols
    y = synth.one_hot(synth.tokens(rows, {"tmlp": 503, "ttfm": 603}[tag], classes), classes)
    m = nsb.Model(spec, w, precision="fp32")
    losses = np.array([m.train_step(x, y, lr) for _ in range(steps)], np.float32)
    np.testing.assert_allclose(losses, G[f"{tag}_losses"], rtol=1e-4, atol=1e-5)
    np.testing.assert_allclose(m.get_weights(), G[f"{tag}_w"], rtol=1e-3, atol=5e-4)
    np.testing.assert_allclose(m.objective(x, y), G[f"{tag}_obj"][0], rtol=1e-4, atol=1e-5)
    np.testing.assert_allclose(m.infer(x), G[f"{tag}_out"], rtol=1e-3, atol=5e-4)


RESID = """network RESID
input tokens
layer emb embedding vocab=64 dim=32
layer attn attention dim=32 heads=4 seq=16
layer ln1 layernorm
layer ff1 dense in=32 out=64 act=gelu
layer ff2 dense in=64 out=32
layer ln2 layernorm
layer head dense in=32 out=48
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
schedule cosine warmup=3 total=40 min=0.05
"""


@pytest.mark.parametrize("mode", ["fp32", "tf32", "bf16"])
def test_residual_block_training_matches_oracle(mode):
    """The config-4 structure at small size: residual sum rule, per-sequence
    attention, AdamW (0.9, 0.95, wd 0.1) with cosine-warmup schedule."""
    w = make_weights(RESID, 801, default_sd=0.1)
    tok = synth.tokens(4 * 16, 802, 64)
    y = synth.one_hot(synth.tokens(64, 803, 48), 48)
    ref = OracleModel(RESID, w)
    m = nsb.Model(RESID, w, precision=mode)
    got, exp = [], []
    for _ in range(12):
        got.append(m.train_step(tok, y, 0.01))
        exp.append(ref.train_step(tok, y, 0.01))
    tol = {"fp32": 1e-5, "tf32": 2e-3, "bf16": 1e-2}[mode]
    assert relerr(got, exp) < tol, (got, exp)
    assert relerr(m.get_weights(), ref.w) < tol * 10


def test_index_labels_equal_one_hot_and_objective_is_pure():
    w = make_weights(RESID, 811, default_sd=0.1)
    tok = synth.tokens(64, 812, 64)
    t = synth.tokens(64, 813, 48).astype(np.int32)
    y = synth.one_hot(t, 48)
    a = nsb.Model(RESID, w, precision="fp32")
    b = nsb.Model(RESID, w, precision="fp32")
    w0 = a.get_weights()
    o1 = a.objective(tok, y)
    assert np.array_equal(a.get_weights(), w0)
    assert o1 == a.objective(tok, y)
    for _ in range(3):
        la = a.train_step(tok, y, 0.01)
        lb = b.train_step_idx(tok, t, 0.01)
        assert la == lb
    assert np.array_equal(a.get_weights(), b.get_weights())


def test_training_is_bitwise_deterministic():
    w = make_weights(RESID, 821, default_sd=0.1)
    tok = synth.tokens(64, 822, 64)
    y = synth.one_hot(synth.tokens(64, 823, 48), 48)
    runs = []
    for _ in range(2):
        m = nsb.Model(RESID, w, precision="bf16")
        ls = [m.train_step(tok, y, 0.01) for _ in range(3)]
        runs.append((ls, m.get_weights()))
    assert runs[0][0] == runs[1][0]
    assert np.array_equal(runs[0][1], runs[1][1])


def test_checkpoint_bytes_and_reference_files(tmp_path):
    w = G["tmlp_w"]
    m = nsb.Model(TMLP, make_weights(TMLP, 501, sds=[0.41, 0.25, 0.35]))
    # a checkpoint written by the reference loads here
    p = str(tmp_path / "ref.ckpt")
    open(p, "wb").write(G["tmlp_ckpt_bytes"].astype(np.uint8).tobytes())
    m.load(p)
    assert np.array_equal(m.get_weights(), w)
    # and ours is byte-identical to the reference's file for the same weights
    q = str(tmp_path / "ours.ckpt")
    m.save(q)
    assert open(q, "rb").read() == open(p, "rb").read()
    # NSM1 (weights only) loads too
    n1 = str(tmp_path / "nsm1.ckpt")
    open(n1, "wb").write(struct.pack("<IQ", 0x4E534D31, w.size) + w.tobytes())
    m.load(n1)
    assert np.array_equal(m.get_weights(), w)
    # wrong size / missing file fail with -1
    bad = str(tmp_path / "bad.ckpt")
    open(bad, "wb").write(struct.pack("<IQ", 0x4E534D32, w.size + 1))
    with pytest.raises(RuntimeError):
        m.load(bad)
    with pytest.raises(RuntimeError):
        m.load(str(tmp_path / "missing.ckpt"))


def test_error_returns():
    L = nsb.RuntimeLib("c1")
    w = np.zeros(10, np.float32)
    assert not L.ns_runtime_init(w.ctypes.data, w.size)
    assert L.ns_eval_infer(None, None, None, 0) == -1
    assert L.ns_model_get_weights(None, None, 0) == -1
    full = make_weights(C1, 1, default_sd=0.01)
    m = L.ns_runtime_init(full.ctypes.data, full.size)
    assert L.ns_model_get_weights(m, full.ctypes.data, full.size - 1) == -1
    assert L.ns_expert_count(m) == 0 and L.ns_expert_kill(m, 0) == 0
    L.ns_free(m)


def test_launches_are_counted():
    w = make_weights(C2, 311, default_sd=0.02)
    m = nsb.Model(C2, w, precision="bf16")
    m.infer(synth.tokens(512, 301, 8192))
    # embedding, qkv GEMM, attention, out-projection GEMM (+ residual +
    # LayerNorm), ff1 GEMM (+ GELU), ff2 GEMM (+ residual + LayerNorm)
    assert m.last_launch_count() == 6


# The config-4 structure at tensor-core shapes: head dim 64 and 128-token
# sequences, so the tcgen05 attention forward and backward, the tcgen05 GEMMs
# and the fused residual epilogues all run in bf16 / TF32 mode.
TC4 = """network TC4
input tokens
layer emb embedding vocab=128 dim=128
layer attn attention dim=128 heads=2 seq=128
layer ln1 layernorm
layer ff1 dense in=128 out=256 act=gelu
layer ff2 dense in=256 out=128
layer ln2 layernorm
layer head dense in=128 out=128
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
schedule cosine warmup=10 total=100 min=0.1
"""
TC4_STEPS = 100


@pytest.fixture(scope="module")
def tc4_oracle_losses():
    w = make_weights(TC4, 901, default_sd=0.05)
    tok = synth.tokens(2 * 128, 902, 128)
    y = synth.one_hot(synth.tokens(2 * 128, 903, 128), 128)
    ref = OracleModel(TC4, w)
    losses = np.array([ref.train_step(tok, y, 3e-3) for _ in range(TC4_STEPS)], np.float64)
    return w, tok, y, losses


@pytest.mark.parametrize("mode", ["fp32", "tf32", "bf16"])
def test_config4_structure_100_steps_losses_track_oracle(mode, tc4_oracle_losses):
    """Losses of 100 AdamW/cosine steps against the fp32 oracle: within 1e-3
    relative at every step in TF32 / bf16 mode, 1e-4 in fp32 SIMT mode."""
    w, tok, y, exp = tc4_oracle_losses
    m = nsb.Model(TC4, w, precision=mode)
    got = np.array([m.train_step(tok, y, 3e-3) for _ in range(TC4_STEPS)], np.float64)
    rel = np.abs(got - exp) / np.abs(exp)
    assert exp[-1] < 0.8 * exp[0]  # the run actually trains
    assert rel.max() < (1e-4 if mode == "fp32" else 1e-3), (rel.max(), int(rel.argmax()), got[-1], exp[-1])


@pytest.mark.parametrize("mode", ["fp32", "tf32", "bf16"])
def test_config5_structure_muon_matches_oracle(mode):
    """The config-5 structure at small size: a ReLU MLP under MSE trained by
    Muon (momentum 0.95, five Newton-Schulz iterations per weight matrix on
    the tensor cores) against the oracle's restatement."""
    from neuralscript_b200.spec import c5
    spec = c5(3, 128)
    w = make_weights(spec, 1201, default_sd=1.0 / np.sqrt(128))
    x = synth.normal(64 * 128, 1202, 0.0, 1.0)
    y = synth.normal(64 * 128, 1203, 0.0, 1.0)
    ref = OracleModel(spec, w)
    m = nsb.Model(spec, w, precision=mode)
    got = np.array([m.train_step(x, y, 0.02) for _ in range(8)], np.float64)
    exp = np.array([ref.train_step(x, y, 0.02) for _ in range(8)], np.float64)
    assert exp[-1] < exp[0]  # it trains
    tol = {"fp32": 1e-4, "tf32": 3e-3, "bf16": 2e-2}[mode]
    assert np.abs(got - exp).max() / np.abs(exp).max() < tol, (got, exp)
    if mode == "fp32":
        assert relerr(m.get_weights(), ref.w) < 1e-3
    # In TF32 / bf16 mode the Newton-Schulz GEMMs round their operands; with
    # Muon's large normalised steps (each one moves a weight by a sizeable
    # fraction of itself) the weights drift apart by several percent within
    # a few steps (7.5 % after 8 in TF32) while the losses stay together.


# The config-2 block at small size with the loss taken on the block output
# itself (no head layer): the smoke network. Its forward output is a config
# block output, so the contract's 2e-3 applies in bf16.
SMOKE = RESID.replace("layer head dense in=32 out=48\n", "").replace("logits = head(y)\noutput logits",
                                                                       "output y")


def test_smoke_block_bf16_forward_and_step():
    w = make_weights(SMOKE, 901, default_sd=0.1)
    tok = synth.tokens(64, 902, 64)
    y = synth.one_hot(synth.tokens(64, 903, 32), 32)
    m = nsb.Model(SMOKE, w, precision="bf16")
    ref = OracleModel(SMOKE, w)
    assert relerr(m.infer(tok), ref.forward(tok)) < TOL["bf16"]
    l_gpu, l_ref = m.train_step(tok, y, 0.01), ref.train_step(tok, y, 0.01)
    assert abs(l_gpu - l_ref) < 1e-3 * abs(l_ref), (l_gpu, l_ref)


def test_config4_full_size_step_matches_reference():
    """One config-4 train step at its full per-GPU size (64 x 256 tokens,
    512 -> 8192 head, bf16) against the float64 restatement
    (tests/torch_ref.py, pinned to the oracle on CPU): the loss within 1e-3
    and every weight gradient within 2e-2 (relative Frobenius). The cosine
    schedule's first step has a zero learning rate, so the weights stay put
    and a second step must reproduce the loss."""
    import torch_ref
    from neuralscript_b200.spec import C4
    w = make_weights(C4, 1301, default_sd=0.02)
    tok = synth.tokens(64 * 256, 1302, 8192)
    tgt = synth.tokens(64 * 256, 1303, 8192).astype(np.int32)
    m = nsb.Model(C4, w, precision="bf16")
    l1 = m.train_step_idx(tok, tgt, 3e-4)
    g = m.get_gradients()
    l_ref, g_ref, _ = torch_ref.forward_backward(C4, w, tok, tgt, device="cuda")
    assert abs(l1 - l_ref) < 1e-3 * abs(l_ref), (l1, l_ref)
    for name, off, cnt, shp in parse(C4).layout():
        e = relerr(g[off:off + cnt], g_ref[name].reshape(-1))
        assert e < 2e-2, (name, e)
    assert np.array_equal(m.get_weights(), w)  # lr factor 0 at step 0
    l2 = m.train_step_idx(tok, tgt, 3e-4)
    assert abs(l2 - l1) < 1e-6 * abs(l1)


# TC4 with a 512-way head: wide enough for the head GEMM + cross-entropy
# fusion (bf16, int32 targets), which the 128-class TC4 does not take.
TC4W = TC4.replace("layer head dense in=128 out=128", "layer head dense in=128 out=512")


def test_fused_head_cross_entropy_tracks_oracle_for_60_steps(monkeypatch):
    """bf16 training with int32 targets runs the fused head GEMM + loss
    (fp16 logits and the fp32 target logit from the GEMM epilogue, then one
    pass for the loss and the seed). Losses within 1e-3 of the fp32 oracle at
    every step, and within 1e-3 of the same model trained through the unfused
    dense-label path (the host label scan switched off)."""
    w = make_weights(TC4W, 1501, default_sd=0.05)
    tok = synth.tokens(2 * 128, 1502, 128)
    tgt = synth.tokens(2 * 128, 1503, 512).astype(np.int32)
    y = synth.one_hot(tgt, 512)
    ref = OracleModel(TC4W, w)
    fused = nsb.Model(TC4W, w, precision="bf16")
    plain = nsb.Model(TC4W, w, precision="bf16")
    got, base, exp = [], [], []
    for _ in range(60):
        got.append(fused.train_step_idx(tok, tgt, 3e-3))
        monkeypatch.setenv("NS_B200_LABEL_SCAN", "0")
        base.append(plain.train_step(tok, y, 3e-3))  # dense labels: the unfused loss kernel
        monkeypatch.delenv("NS_B200_LABEL_SCAN")
        exp.append(ref.train_step(tok, y, 3e-3))
    got, base, exp = (np.array(v, np.float64) for v in (got, base, exp))
    assert exp[-1] < 0.8 * exp[0]
    e_fused, e_plain = np.max(np.abs(got - exp) / exp), np.max(np.abs(base - exp) / exp)
    print(f"max relative loss deviation from the oracle: fused {e_fused:.2e}, unfused {e_plain:.2e}")
    assert e_fused < 1e-3 and e_plain < 1e-3, (e_fused, e_plain)


def test_one_hot_labels_take_the_target_path_exactly(monkeypatch):
    """ns_runtime_train_step reads one-hot label rows on the host and sends
    class indices: the losses and weights equal the integer-target step bit
    for bit (an all-zero row acts as a target outside the classes). A label
    row that is not one-hot keeps the dense path: that run equals the run
    with the host scan switched off."""
    w = make_weights(TC4W, 1511, default_sd=0.05)
    tok = synth.tokens(2 * 128, 1512, 128)
    tgt = synth.tokens(2 * 128, 1513, 512).astype(np.int32)
    y = synth.one_hot(tgt, 512)
    y[7] = 0.0
    tgt_z = tgt.copy()
    tgt_z[7] = -1  # the all-zero row
    a = nsb.Model(TC4W, w, precision="bf16")
    b = nsb.Model(TC4W, w, precision="bf16")
    la = [a.train_step(tok, y, 3e-3) for _ in range(3)]
    lb = [b.train_step_idx(tok, tgt_z, 3e-3) for _ in range(3)]
    assert la == lb
    assert np.array_equal(a.get_weights(), b.get_weights())
    soft = y.copy()
    soft[3] = 0.0
    soft[3, 5] = soft[3, 9] = 0.5  # not one-hot: the whole batch stays dense
    c = nsb.Model(TC4W, w, precision="bf16")
    d = nsb.Model(TC4W, w, precision="bf16")
    lc = [c.train_step(tok, soft, 3e-3) for _ in range(2)]
    monkeypatch.setenv("NS_B200_LABEL_SCAN", "0")
    ld = [d.train_step(tok, soft, 3e-3) for _ in range(2)]
    monkeypatch.delenv("NS_B200_LABEL_SCAN")
    assert lc == ld
    assert np.array_equal(c.get_weights(), d.get_weights())
