"""In-call multi-GPU through the unchanged ABI (two GPUs; skipped with
fewer): with NS_B200_GPUS=2 set when the model is created, one
ns_runtime_train_step / ns_eval_infer call splits the caller's rows (whole
sequences) over both GPUs of this process, which all-reduce their gradients
over NCCL. The results must equal one GPU running the whole batch."""
import os

import numpy as np
import pytest

torch = pytest.importorskip("torch")
pytestmark = [pytest.mark.gpu,
              pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2,
                                 reason="needs 2 GPUs")]

import neuralscript_b200 as nsb  # noqa: E402
from model_oracle import make_weights  # noqa: E402
from neuralscript_b200 import synth  # noqa: E402
from test_gpu_dist import MUON, TC4D, _muon_data  # noqa: E402
from test_gpu_ops import OPS_NET  # noqa: E402


def two_gpu_model(spec, w, mode):
    """A model created with NS_B200_GPUS=2 (read by ns_runtime_init)."""
    old = os.environ.get("NS_B200_GPUS")
    os.environ["NS_B200_GPUS"] = "2"
    os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
    try:
        return nsb.Model(spec, w, precision=mode)
    finally:
        if old is None:
            os.environ.pop("NS_B200_GPUS", None)
        else:
            os.environ["NS_B200_GPUS"] = old


def rel(a, b):
    a, b = np.asarray(a, np.float64), np.asarray(b, np.float64)
    return float(np.linalg.norm(a - b) / np.linalg.norm(b))


@pytest.mark.parametrize("mode", ["bf16", "fp32"])
def test_in_call_two_gpu_train_equals_one_gpu(mode):
    w = make_weights(TC4D, 2001, default_sd=0.05)
    tok = synth.tokens(4 * 128, 2002, 128)
    tgt = synth.tokens(4 * 128, 2003, 128).astype(np.int32)
    y = synth.one_hot(tgt, 128)
    one = nsb.Model(TC4D, w, precision=mode)
    two = two_gpu_model(TC4D, w, mode)
    # the reference ABI form (one-hot labels) and the index form, alternating
    got = [two.train_step(tok, y, 3e-3) if i % 2 == 0 else two.train_step_idx(tok, tgt, 3e-3) for i in range(6)]
    exp = [one.train_step(tok, y, 3e-3) if i % 2 == 0 else one.train_step_idx(tok, tgt, 3e-3) for i in range(6)]
    tol = 1e-5 if mode == "fp32" else 2e-3
    np.testing.assert_allclose(got, exp, rtol=tol)
    assert rel(two.get_weights(), one.get_weights()) < (1e-4 if mode == "fp32" else 2e-3)
    # forward-only objective and inference split the rows too
    assert abs(two.objective(tok, y) - one.objective(tok, y)) < tol * abs(one.objective(tok, y))
    # after training, the weights agree to the tolerance above, so outputs do
    assert rel(two.infer(tok), one.infer(tok)) < (1e-4 if mode == "fp32" else 5e-3)
    assert two.last_launch_count() > one.last_launch_count()  # both GPUs launched work
    two.close()


def test_in_call_two_gpu_inference_uneven_rows():
    """Inference accepts any row count: 5 sequences split 3 + 2."""
    w = make_weights(TC4D, 2011, default_sd=0.05)
    tok = synth.tokens(5 * 128, 2012, 128)
    one = nsb.Model(TC4D, w, precision="bf16")
    two = two_gpu_model(TC4D, w, "bf16")
    np.testing.assert_allclose(two.infer(tok), one.infer(tok), rtol=1e-4, atol=1e-5)
    # a train step whose rows cannot split evenly fails cleanly
    with pytest.raises(RuntimeError):
        two.train_step_idx(tok, synth.tokens(5 * 128, 2013, 128).astype(np.int32), 1e-3)
    two.close()


def test_in_call_two_gpu_dropout_masks_equal_one_gpu():
    """Dropout masks are indexed by the element's row in the whole batch, so
    the split batch draws the same masks as the unsplit one."""
    w = make_weights(OPS_NET, 2021, default_sd=0.5)
    x = synth.uniform(96 * 6, 2022, -1, 1)
    y = synth.one_hot(synth.tokens(96, 2023, 4), 4)
    one = nsb.Model(OPS_NET, w, precision="fp32")
    two = two_gpu_model(OPS_NET, w, "fp32")
    got = [two.train_step(x, y, 0.01) for _ in range(4)]
    exp = [one.train_step(x, y, 0.01) for _ in range(4)]
    np.testing.assert_allclose(got, exp, rtol=1e-5)
    np.testing.assert_allclose(two.get_input_gradient(), one.get_input_gradient(), rtol=1e-4, atol=1e-6)
    two.close()


def test_in_call_two_gpu_sharded_muon():
    w, x, y = _muon_data()
    one = nsb.Model(MUON, w, precision="fp32")
    two = two_gpu_model(MUON, w, "fp32")
    got = [two.train_step(x, y, 0.02) for _ in range(4)]
    exp = [one.train_step(x, y, 0.02) for _ in range(4)]
    np.testing.assert_allclose(got, exp, rtol=1e-4)
    assert rel(two.get_weights(), one.get_weights()) < 1e-3
    two.close()
