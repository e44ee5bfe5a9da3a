"""Per-weight gradient parity on the GPU (pure fp32 mode) against the
model-level oracle: every trainable tensor of every layer kind, including
values consumed twice (residual sum rule) and MoE with a dead expert."""
import numpy as np
import pytest

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

import neuralscript_b200 as nsb  # noqa: E402
from model_oracle import OracleModel, make_weights  # noqa: E402
from neuralscript_b200 import synth  # noqa: E402
from specs import TMLP, TMOE, TTFM  # noqa: E402
from test_gpu_model import RESID  # noqa: E402


def oracle_grads(spec, w, x, y):
    r = OracleModel(spec, w)
    out, vals, cache = r.forward(x, keep=True)
    _, seed = r._loss_and_seed(out, y)
    return r.backward(vals, cache, seed), r


CASES = {
    "resid": (RESID, lambda: (make_weights(RESID, 801, default_sd=0.1), synth.tokens(64, 802, 64),
                              synth.one_hot(synth.tokens(64, 803, 48), 48))),
    "tmlp": (TMLP, lambda: (make_weights(TMLP, 501, sds=[0.41, 0.25, 0.35]), synth.uniform(96, 502, -1, 1),
                            synth.one_hot(synth.tokens(16, 503, 4), 4))),
    "ttfm": (TTFM, lambda: (make_weights(TTFM, 601, sds=[0.5, 0.4, 0.4, 0.4, 0.4, 0.4, 0.3, 0.4]),
                            synth.tokens(64, 602, 32), synth.one_hot(synth.tokens(64, 603, 16), 16))),
    "tmoe": (TMOE, lambda: (make_weights(TMOE, 701, sds=[0.5, 0.5, 0.35, 0.25, 0.35]), synth.tokens(24, 702, 16),
                            synth.one_hot(synth.tokens(24, 703, 4), 4))),
}


@pytest.mark.parametrize("case", sorted(CASES))
def test_every_gradient_matches_oracle_fp32(case):
    spec, make = CASES[case]
    w, x, y = make()
    g_ref, r = oracle_grads(spec, w, x, y)
    m = nsb.Model(spec, w, precision="fp32")
    m.train_step(x, y, 0.0)
    g = m.get_gradients()
    bad = []
    for name, off, cnt, shp in r.s.layout():
        ref = g_ref[name].reshape(-1).astype(np.float64)
        got = g[off:off + cnt].astype(np.float64)
        e = np.linalg.norm(got - ref) / max(np.linalg.norm(ref), 1e-30)
        if e > 1e-5:
            bad.append((name, e))
    assert not bad, bad
