"""Model-level CPU oracle: composes the C oracle's kernels (oracle/) along a
model spec, restating the reference's emitted forward function
(src/codegen/codegen.cpp:1962-2288) and AOT train core (:2659-3157).

Test infrastructure only. Differences from the reference, each deliberate:
* attention uses the layer's ``seq`` (0 = the whole call, which is the
  reference's behaviour, codegen.cpp:2225);
* a value consumed twice (a residual) receives the SUM of its consumers'
  gradients; the reference keeps only one of them (mlir_compiler.cpp:452);
* ``optimizer adamw`` / ``muon`` / ``schedule cosine`` are the configuration
  modes; ``optimizer reference`` + ``schedule constant`` is the reference.
"""
from __future__ import annotations

import math
from typing import Dict, Optional

import numpy as np

import oracle_lib as O
from neuralscript_b200.spec import ACT_CODES, Spec, parse

# Dropout key of every model (the engine's default Philox key); the step
# counter advances once per training step and the site is the dropout op's
# index among the network's dropout ops.
DROP_KEY = (0x243F6A88, 0x85A308D3)

# include/ns/optim/optim_params.hpp:20-32
REF_OPT = dict(momentum=0.95, muon_decay=0.01, beta1=0.9, beta2=0.999, eps=1e-8, decay=0.01,
               omb1=0.1, omb2=0.001)


def _f(x):
    return np.float32(x)


class OracleModel:
    def __init__(self, spec_text: str, weights: np.ndarray):
        self.s: Spec = parse(spec_text)
        self.w = np.array(weights, dtype=np.float32, copy=True)
        assert self.w.size == self.s.weight_count
        self.lr_step = 0
        self.drop_step = 0
        self.input_grad = None  # dLoss/dx of the last train step (`grad input` specs)
        self.state: Dict[str, dict] = {}
        self.active = None
        for l in self.s.layers:
            if l.kind == "moe":
                e = l.i("experts")
                k0 = l.i("initial", e)
                if k0 <= 0 or k0 > e:
                    k0 = e
                self.active = np.zeros(e, np.uint8)
                self.active[:k0] = 1

    # -- weights ---------------------------------------------------------------
    def W(self, name: str) -> np.ndarray:
        for n, off, cnt, shp in self.s.layout():
            if n == name:
                return self.w[off:off + cnt].reshape(shp)
        raise KeyError(name)

    # -- forward ---------------------------------------------------------------
    def forward(self, x: np.ndarray, keep: bool = False, train: bool = False):
        s = self.s
        x = np.asarray(x, np.float32).reshape(-1)
        rows = x.size // s.in_cols
        vals = {"x": x.reshape(rows, s.in_cols) if not s.tokens else x[:rows]}
        cache = {}
        site = 0
        for op in s.ops:
            a = [vals[t] for t in op.args]
            if op.fn == "concat":
                vals[op.out] = O.concat_cols(a[0], a[1])
                continue
            if op.fn == "slice":
                vals[op.out] = O.slice_cols(a[0], op.ints[0], op.ints[1])
                continue
            if op.fn == "index":
                vals[op.out] = O.index_cols(a[0], op.ints)
                continue
            if op.fn == "scatter":
                vals[op.out] = O.scatter_cols(a[0], op.ints, a[1])
                continue
            if op.fn in ("add", "sub", "mul", "div"):
                code = {"add": 0, "sub": 1, "mul": 2, "div": 3}[op.fn]
                out = np.empty_like(a[0])
                O.lib.orc_binop(a[0].reshape(-1), a[0].size, np.ascontiguousarray(a[1]).reshape(-1),
                                a[1].size, out.reshape(-1), code)
                vals[op.out] = out
                continue
            if op.fn in ACT_CODES:
                vals[op.out] = O.act(a[0], ACT_CODES[op.fn])
                continue
            if op.fn == "softmax":
                vals[op.out] = O.softmax(a[0])
                continue
            l = s.layer(op.fn)
            u = a[0]
            if l.kind == "dense":
                z = O.matmul(u, self.W(f"{l.name}_w"))
                cache[op.out] = z
                vals[op.out] = O.act(z, l.act) if l.act else z
            elif l.kind == "embedding":
                vals[op.out] = O.embedding(self.W(f"{l.name}_w"), u)
            elif l.kind == "attention":
                seq = l.i("seq", 0) or u.shape[0]
                vals[op.out] = O.attention_fwd(u, *[self.W(f"{l.name}_{t}_w") for t in "qkvo"],
                                               l.i("heads"), seq)
            elif l.kind == "layernorm":
                vals[op.out] = O.layernorm(u)
            elif l.kind == "moe":
                vals[op.out] = self._moe_fwd(l, u)
            elif l.kind == "dropout":
                rate = float(l.p.get("rate", "0"))
                if train and rate > 0:
                    mask = O.dropout_mask(u.size, rate, DROP_KEY[0], DROP_KEY[1], self.drop_step, site)
                    cache[op.out] = mask.reshape(u.shape)
                    vals[op.out] = (u * cache[op.out]).astype(np.float32)
                else:
                    vals[op.out] = u.copy()
                site += 1
            else:
                raise ValueError(l.kind)
        out = vals[s.output]
        return (out, vals, cache) if keep else out

    def _moe_fwd(self, l, u):
        d, e = l.i("dim"), l.i("experts")
        wg = self.W(f"{l.name}_g_w")
        if l.p.get("expert", "ffn") == "linear":
            best, pb, _ = O.moe_route(u, wg, self.active)
            we = self.W(f"{l.name}_e1_w").reshape(e, d, d)
            out = np.zeros_like(u)
            for ex in range(e):
                idx = np.nonzero(best == ex)[0]
                if idx.size:
                    out[idx] = O.matmul(u[idx], we[ex]) * pb[idx, None]
            return out
        return O.moe_fwd(u, wg, self.W(f"{l.name}_e1_w"), self.W(f"{l.name}_e2_w"), l.i("ffn", 4 * d),
                         self.active)

    # -- backward --------------------------------------------------------------
    def backward(self, vals, cache, dout: np.ndarray) -> Dict[str, np.ndarray]:
        s = self.s
        grads: Dict[str, np.ndarray] = {}
        g: Dict[str, np.ndarray] = {s.output: dout}

        def add(name, d):
            if name == "x" and s.tokens:
                return
            g[name] = d if name not in g else (g[name] + d).astype(np.float32)

        for op in reversed(s.ops):
            if op.out not in g:
                continue
            dv = g[op.out]
            a = [vals[t] for t in op.args]
            if op.fn == "add":
                add(op.args[0], dv)
                add(op.args[1], dv)
                continue
            if op.fn == "sub":
                add(op.args[0], dv)
                add(op.args[1], (-dv).astype(np.float32))
                continue
            if op.fn == "mul":
                add(op.args[0], (dv * a[1]).astype(np.float32))
                add(op.args[1], (dv * a[0]).astype(np.float32))
                continue
            if op.fn == "div":
                add(op.args[0], (dv / a[1]).astype(np.float32))
                add(op.args[1], (-dv * a[0] / (a[1] * a[1])).astype(np.float32))
                continue
            if op.fn == "concat":
                ca = a[0].shape[1]
                add(op.args[0], np.ascontiguousarray(dv[:, :ca]))
                add(op.args[1], np.ascontiguousarray(dv[:, ca:]))
                continue
            if op.fn == "slice":
                d = np.zeros_like(a[0])
                d[:, op.ints[0]:op.ints[1]] = dv
                add(op.args[0], d)
                continue
            if op.fn == "index":
                d = np.zeros_like(a[0])
                for k, c in enumerate(op.ints):  # duplicates add in increasing k
                    d[:, c] = (d[:, c] + dv[:, k]).astype(np.float32)
                add(op.args[0], d)
                continue
            if op.fn == "scatter":
                last = {c: k for k, c in enumerate(op.ints)}  # the update each column keeps
                d_in = dv.copy()
                d_upd = np.zeros_like(a[1])
                for c, k in last.items():
                    d_in[:, c] = 0.0
                    d_upd[:, k] = dv[:, c]
                add(op.args[0], d_in)
                add(op.args[1], d_upd)
                continue
            if op.fn in ACT_CODES:
                add(op.args[0], O.act_grad(dv, a[0], ACT_CODES[op.fn]))
                continue
            if op.fn == "softmax":
                # the reference lowers softmax's gradient to ns_act_grad with
                # code 0, i.e. a pass-through (codegen.cpp:3073-3085)
                add(op.args[0], dv)
                continue
            l = s.layer(op.fn)
            u = a[0]
            if l.kind == "dense":
                dz = O.act_grad(dv, cache[op.out], l.act) if l.act else dv
                grads[f"{l.name}_w"] = O.matmul_grad_w(u, dz)
                add(op.args[0], O.matmul_grad_a(dz, self.W(f"{l.name}_w")))
            elif l.kind == "embedding":
                grads[f"{l.name}_w"] = O.embedding_grad_w(dv, u, l.i("vocab"))
            elif l.kind == "attention":
                seq = l.i("seq", 0) or u.shape[0]
                dX, dq, dk, dvw, do = O.attention_bwd(dv, u, *[self.W(f"{l.name}_{t}_w") for t in "qkvo"],
                                                      l.i("heads"), seq)
                grads.update({f"{l.name}_q_w": dq, f"{l.name}_k_w": dk, f"{l.name}_v_w": dvw,
                              f"{l.name}_o_w": do})
                add(op.args[0], dX)
            elif l.kind == "layernorm":
                add(op.args[0], O.layernorm_grad(dv, u))
            elif l.kind == "moe":
                d = l.i("dim")
                if l.p.get("expert", "ffn") == "linear":
                    dx, dwg, dwe = linear_moe_grads(dv, u, self.W(f"{l.name}_g_w"), self.W(f"{l.name}_e1_w"),
                                                    self.active)
                    grads.update({f"{l.name}_g_w": dwg, f"{l.name}_e1_w": dwe})
                    add(op.args[0], dx)
                    continue
                dx, dwg, dwe1, dwe2 = O.moe_grads(dv, u, self.W(f"{l.name}_g_w"), self.W(f"{l.name}_e1_w"),
                                                  self.W(f"{l.name}_e2_w"), l.i("ffn", 4 * d), self.active)
                grads.update({f"{l.name}_g_w": dwg, f"{l.name}_e1_w": dwe1, f"{l.name}_e2_w": dwe2})
                add(op.args[0], dx)
            elif l.kind == "dropout":
                mask = cache.get(op.out)
                add(op.args[0], dv if mask is None else (dv * mask).astype(np.float32))
        if s.input_grad:
            grads["__input__"] = g.get("x")
        return grads

    # -- loss ------------------------------------------------------------------
    def _loss_and_seed(self, out, labels, denom=None):
        rows = out.shape[0]
        if self.s.loss == "mse":
            y = np.asarray(labels, np.float32).reshape(out.shape)
            return O.lib.orc_mse(out.reshape(-1), y.reshape(-1), out.size), None if denom is False else \
                self._mse_seed(out, y, denom)
        y = np.asarray(labels, np.float32).reshape(out.shape)
        loss = O.cross_entropy(out, y)
        return loss, O.loss_grad(out, y, rows if denom is None else denom)

    def _mse_seed(self, out, y, denom):
        d = np.empty_like(out)
        O.lib.orc_mse_grad(out.reshape(-1), y.reshape(-1), d.reshape(-1), out.size,
                           float(out.size if denom is None else denom))
        return d

    def objective(self, x, labels) -> float:
        out = self.forward(x)
        return float(self._loss_and_seed(out, labels)[0])

    def schedule(self, step: int) -> float:
        if self.s.schedule == "cosine":
            return O.lr_schedule(step, 1, int(self.s.sched.get("warmup", 100)), int(self.s.sched.get("total", 10000)),
                                 float(self.s.sched.get("min", 0.05)))
        return 1.0

    def train_step(self, x, labels, lr: float) -> float:
        st = self.lr_step
        self.lr_step += 1
        lr_eff = _f(_f(lr) * _f(self.schedule(st)))
        out, vals, cache = self.forward(x, keep=True, train=True)
        loss, seed = self._loss_and_seed(out, labels)
        grads = self.backward(vals, cache, seed)
        self.input_grad = grads.pop("__input__", None)
        self.apply(grads, lr_eff)
        self.drop_step += 1
        return float(loss)

    def apply(self, grads, lr_eff):
        s = self.s
        for name, off, cnt, (r, c) in s.layout():
            if name not in grads:
                continue
            g = np.ascontiguousarray(grads[name], np.float32).reshape(-1)
            w = self.w[off:off + cnt]
            st = self.state.setdefault(name, {"m": np.zeros(cnt, np.float32), "v": np.zeros(cnt, np.float32),
                                              "t": 0})
            mode = s.optimizer
            matrix = r > 1 and c > 1
            if mode == "reference" and matrix and min(r, c) >= 8:
                wc = w.copy()
                O.lib.orc_muon_mgs_step(wc, g, st["m"], r, c, lr_eff, REF_OPT["momentum"], REF_OPT["muon_decay"])
                self.w[off:off + cnt] = wc
            elif mode == "muon" and matrix and min(r, c) >= 8:
                mu = float(s.opt.get("momentum", 0.95))
                st["m"] = (_f(mu) * st["m"] + g).astype(np.float32)
                o = O.newton_schulz5(st["m"].reshape(r, c), int(s.opt.get("steps", 5))).reshape(-1)
                le = _f(lr_eff * math.sqrt(min(r, c)))
                dec = _f(s.opt.get("decay", 0.01)) * _f(lr_eff)
                self.w[off:off + cnt] = (w - (le * o + dec * w)).astype(np.float32)
            else:
                st["t"] += 1
                if mode in ("adamw", "muon"):
                    b1 = float(s.opt.get("beta1", 0.9))
                    b2 = float(s.opt.get("beta2", 0.999))
                    eps = float(s.opt.get("eps", 1e-8))
                    dec = float(s.opt.get("decay", 0.01))
                    omb1, omb2 = 1.0 - b1, 1.0 - b2
                else:
                    b1, b2, eps, dec = REF_OPT["beta1"], REF_OPT["beta2"], REF_OPT["eps"], REF_OPT["decay"]
                    omb1, omb2 = REF_OPT["omb1"], REF_OPT["omb2"]
                wc = w.copy()
                O.lib.orc_adamw_step(wc, g, st["m"], st["v"], cnt, st["t"], lr_eff, b1, b2, omb1, omb2, eps, dec)
                self.w[off:off + cnt] = wc


def make_weights(spec_text: str, seed: int, sds: Optional[list] = None, default_sd: Optional[float] = None):
    """Blob of N(0, sd_l) per weight from stream seed + l (as the golden
    harness builds it)."""
    from neuralscript_b200 import synth
    s = parse(spec_text)
    parts = []
    for l_idx, (name, off, cnt, (r, c)) in enumerate(s.layout()):
        sd = sds[l_idx] if sds is not None else (default_sd if default_sd is not None else 1.0 / math.sqrt(r))
        parts.append(synth.normal(cnt, seed + l_idx, 0.0, sd))
    return np.concatenate(parts) if parts else np.zeros(0, np.float32)


def linear_moe_grads(dy, x, Wg, We, active=None):
    """Gradients of y_i = pb_i (x_i We[b_i]) with the reference router (no
    reference counterpart: its experts are FFNs). Same gate rule as
    codegen.cpp:1420-1428: dg_ie = p_ie ((e == b_i) dpb_i - dpb_i pb_i)."""
    x = np.asarray(x, np.float64)
    dy = np.asarray(dy, np.float64)
    M, D = x.shape
    E = Wg.shape[1]
    best, pb, p = O.moe_route(np.asarray(x, np.float32), Wg, active)
    we = np.asarray(We, np.float64).reshape(E, D, D)
    dx = np.zeros_like(x)
    dwe = np.zeros_like(we)
    dpb = np.zeros(M)
    for e in range(E):
        idx = np.nonzero(best == e)[0]
        if idx.size == 0:
            continue
        ys = x[idx] @ we[e]
        dpb[idx] = (ys * dy[idx]).sum(axis=1)
        sd = dy[idx] * pb[idx, None]
        dwe[e] = x[idx].T @ sd
        dx[idx] += sd @ we[e].T
    dg = p.astype(np.float64) * ((np.arange(E)[None, :] == best[:, None]) * dpb[:, None] - (dpb * pb)[:, None])
    dwg = x.T @ dg
    dx += dg @ np.asarray(Wg, np.float64).T
    return dx.astype(np.float32), dwg.astype(np.float32), dwe.reshape(E, D * D).astype(np.float32)
