"""Data-parallel host logic on CPU with two gloo ranks (no GPU):

* the decomposition the engine uses — each rank seeds its loss gradient with
  the GLOBAL row count and gradients are SUM-all-reduced — reproduces the
  full-batch gradient of the oracle;
* the NCCL unique-id hand-off pattern (rank 0 creates 128 bytes, the others
  receive them via a broadcast) round-trips;
* a rank that fails before the collective makes the survivor's collective
  end with an error within the process-group timeout (failure detection on
  the host; no GPU involved).
"""
import datetime
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from model_oracle import OracleModel, make_weights
from neuralscript_b200 import synth

SPEC = """network DP
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
optimizer adamw beta2=0.95 decay=0.1
"""


def free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def grads_for(m, tok, y, denom):
    out, vals, cache = m.forward(tok, keep=True)
    _, seed = m._loss_and_seed(out, y, denom)
    return m.backward(vals, cache, seed)


def _dp_worker(rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=30))
    try:
        w = make_weights(SPEC, 701, default_sd=0.1)
        tok = synth.tokens(4 * 16, 702, 64)
        y = synth.one_hot(synth.tokens(64, 703, 48), 48)
        rows = 64 // world
        sl = slice(rank * rows, (rank + 1) * rows)  # whole 16-token sequences per rank
        g = grads_for(OracleModel(SPEC, w), tok[sl], y[sl], denom=64)
        names = sorted(g)
        flat = torch.from_numpy(np.concatenate([g[n].reshape(-1) for n in names]).astype(np.float64))
        dist.all_reduce(flat)
        uid = [os.urandom(128) if rank == 0 else None]
        dist.broadcast_object_list(uid, src=0)
        if rank == 0:
            full = grads_for(OracleModel(SPEC, w), tok, y, denom=64)
            ref = np.concatenate([full[n].reshape(-1) for n in names]).astype(np.float64)
            err = float(np.linalg.norm(flat.numpy() - ref) / np.linalg.norm(ref))
            q.put(("ok", err, len(uid[0])))
        else:
            q.put(("uid", len(uid[0])))
    finally:
        dist.destroy_process_group()


def test_global_row_seed_and_sum_allreduce_equal_full_batch_gradient():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = free_port()
    ps = [ctx.Process(target=_dp_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in ps:
        p.start()
    for p in ps:
        p.join(timeout=240)
        assert p.exitcode == 0
    res = [q.get(timeout=5) for _ in range(2)]
    ok = [r for r in res if r[0] == "ok"][0]
    assert ok[1] < 1e-5, ok
    assert all(r[-1] == 128 for r in res)


def _fail_worker(rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=5))
    if rank == 1:
        os._exit(3)  # dies between steps, before joining the collective
    t = torch.ones(4)
    try:
        dist.all_reduce(t)
        q.put("no-error")
    except Exception as e:  # timeout / connection closed: detected on the host
        q.put(type(e).__name__)


def test_peer_failure_is_detected_by_the_survivor():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = free_port()
    ps = [ctx.Process(target=_fail_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in ps:
        p.start()
    for p in ps:
        p.join(timeout=120)
    assert q.get(timeout=5) != "no-error"


MUON_SPEC = """network MU
input 32
layer fc1 dense in=32 out=32 act=relu
layer fc2 dense in=32 out=32 act=relu
layer fc3 dense in=32 out=32
h1 = fc1(x)
h2 = fc2(h1)
y = fc3(h2)
output y
loss mse
optimizer muon momentum=0.95 steps=5 decay=0.01
"""


def _muon_worker(rank, world, port, q):
    """The sharded Muon step the engine runs under data parallelism: each
    rank's gradient (global-row seed) is SUM-reduced to the matrix's owner
    (matrix k owned by rank k % world), the owner alone applies momentum,
    Newton-Schulz-5 and the update, then broadcasts the new matrix."""
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=30))
    try:
        w = make_weights(MUON_SPEC, 711, default_sd=0.18)
        x = synth.normal(64 * 32, 712, 0.0, 1.0)
        t = synth.normal(64 * 32, 713, 0.0, 1.0)
        rows = 64 // world
        sl = slice(rank * rows * 32, (rank + 1) * rows * 32)
        m = OracleModel(MUON_SPEC, w)
        layout = m.s.layout()
        for step in range(3):
            out, vals, cache = m.forward(x[sl], keep=True)
            _, seed = m._loss_and_seed(out, t[sl].reshape(out.shape), 64 * 32)
            g = m.backward(vals, cache, seed)
            upd = {}
            for k, (name, off, cnt, _) in enumerate(layout):
                owner = k % world
                gk = torch.from_numpy(np.ascontiguousarray(g[name], np.float32).reshape(-1))
                dist.reduce(gk, dst=owner)
                if rank == owner:
                    upd[name] = gk.numpy()
            m.apply(upd, 0.02)  # the owner updates only its matrices
            for k, (name, off, cnt, _) in enumerate(layout):
                wk = torch.from_numpy(m.w[off:off + cnt].copy())
                dist.broadcast(wk, src=k % world)
                m.w[off:off + cnt] = wk.numpy()
        if rank == 0:
            ref = OracleModel(MUON_SPEC, w)
            for step in range(3):
                ref.train_step(x, t, 0.02)
            err = float(np.linalg.norm(m.w - ref.w) / np.linalg.norm(ref.w))
            q.put(("ok", err))
        else:
            q.put(("done", 0.0))
    finally:
        dist.destroy_process_group()


def test_sharded_muon_decomposition_equals_full_batch_step():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = free_port()
    ps = [ctx.Process(target=_muon_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in ps:
        p.start()
    for p in ps:
        p.join(timeout=240)
        assert p.exitcode == 0
    res = [q.get(timeout=5) for _ in range(2)]
    ok = [r for r in res if r[0] == "ok"][0]
    assert ok[1] < 1e-4, ok
