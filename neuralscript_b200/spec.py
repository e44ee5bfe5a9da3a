"""Model specifications: the compile-time description a NeuralScript network
lowers to, in the text form the native engine parses (csrc/spec.cpp).

The reference bakes every dimension of a network into its emitted
translation unit (src/codegen/codegen.cpp:552-558); here the same facts are
carried by a small text spec that the model's translation unit embeds and
hands to the engine. Weight order and names follow the reference's
TENSOR_ALLOC order (src/mlir/mlir_compiler.cpp:100-222): ``<layer>_w`` for
Dense and Embedding, ``<layer>_{q,k,v,o}_w`` for Attention and
``<layer>_{g,e1,e2}_w`` for MoE, in layer-declaration order.

Grammar (one statement per line, ``#`` comments)::

    network <Name>
    input <cols> | input tokens
    layer <name> dense in=<K> out=<N> [act=<identity|relu|leaky_relu|sigmoid|tanh|silu|gelu>]
    layer <name> embedding vocab=<V> dim=<D>
    layer <name> attention dim=<D> heads=<H> [seq=<S>]      # seq 0 = whole call
    layer <name> layernorm
    layer <name> moe dim=<D> experts=<E> ffn=<F> [initial=<K0>] [expert=ffn|linear]
    layer <name> dropout rate=<p>
    <v> = <layer>(<u>)
    <v> = add(<a>, <b>) | sub(..) | mul(..) | div(..)
    <v> = <act>(<u>) | softmax(<u>)
    <v> = concat(<a>, <b>) | slice(<u>, <cs>, <ce>) | index(<u>, <c0>, <c1>, ..)
        | scatter(<u>, <upd>, <c0>, <c1>, ..)               # column data movement
    output <v>
    loss cross_entropy | mse
    optimizer reference | adamw [beta1= beta2= eps= decay=] | muon [momentum= steps= decay= ...]
    schedule constant | cosine [warmup= total= min=]
    precision bf16 | tf32 | fp32
    grad input                                              # train steps also form dLoss/dx
"""
from __future__ import annotations

from dataclasses import dataclass, field
from typing import Dict, List, Optional, Tuple

ACT_CODES = {"identity": 0, "relu": 1, "leaky_relu": 2, "sigmoid": 3, "tanh": 4, "silu": 5, "swish": 5,
             "gelu": 6}


@dataclass
class Layer:
    name: str
    kind: str
    p: Dict[str, str] = field(default_factory=dict)

    def i(self, key: str, default: Optional[int] = None) -> int:
        if key in self.p:
            return int(self.p[key])
        if default is None:
            raise KeyError(f"layer {self.name}: missing {key}=")
        return default

    @property
    def act(self) -> int:
        return ACT_CODES[self.p.get("act", "identity").lower()]

    def weights(self) -> List[Tuple[str, Tuple[int, int]]]:
        k = self.kind
        if k == "dense":
            return [(f"{self.name}_w", (self.i("in"), self.i("out")))]
        if k == "embedding":
            return [(f"{self.name}_w", (self.i("vocab"), self.i("dim")))]
        if k == "attention":
            d = self.i("dim")
            return [(f"{self.name}_{s}_w", (d, d)) for s in ("q", "k", "v", "o")]
        if k == "moe":
            d, e = self.i("dim"), self.i("experts")
            f = self.i("ffn", 4 * d)
            if self.p.get("expert", "ffn") == "linear":
                return [(f"{self.name}_g_w", (d, e)), (f"{self.name}_e1_w", (e, d * d))]
            return [(f"{self.name}_g_w", (d, e)), (f"{self.name}_e1_w", (e, d * f)),
                    (f"{self.name}_e2_w", (e, f * d))]
        return []


# data-movement functions: value operands first, then integers
DATA_FNS = {"concat": 2, "slice": 1, "index": 1, "scatter": 2}


@dataclass
class Op:
    out: str
    fn: str
    args: List[str]
    ints: List[int] = field(default_factory=list)


@dataclass
class Spec:
    name: str = "model"
    in_cols: int = 1
    tokens: bool = False
    layers: List[Layer] = field(default_factory=list)
    ops: List[Op] = field(default_factory=list)
    output: str = ""
    loss: str = "cross_entropy"
    optimizer: str = "reference"
    opt: Dict[str, float] = field(default_factory=dict)
    schedule: str = "constant"
    sched: Dict[str, float] = field(default_factory=dict)
    precision: str = "bf16"
    input_grad: bool = False
    text: str = ""

    def layer(self, name: str) -> Layer:
        for l in self.layers:
            if l.name == name:
                return l
        raise KeyError(name)

    def layout(self) -> List[Tuple[str, int, int, Tuple[int, int]]]:
        """[(name, offset, count, (rows, cols))] in blob order."""
        out, off = [], 0
        for l in self.layers:
            for n, shp in l.weights():
                cnt = shp[0] * shp[1]
                out.append((n, off, cnt, shp))
                off += cnt
        return out

    @property
    def weight_count(self) -> int:
        return sum(c for _, _, c, _ in self.layout())


def _kv(tokens: List[str]) -> Dict[str, str]:
    d = {}
    for t in tokens:
        if "=" not in t:
            raise ValueError(f"expected key=value, got {t!r}")
        k, v = t.split("=", 1)
        d[k.strip()] = v.strip()
    return d


def parse(text: str) -> Spec:
    s = Spec(text=text)
    for raw in text.splitlines():
        line = raw.split("#", 1)[0].strip()
        if not line:
            continue
        if "=" in line.split()[0] or (len(line.split()) > 1 and line.split()[1] == "="):
            lhs, rhs = line.split("=", 1)
            rhs = rhs.strip()
            fn, rest = rhs.split("(", 1)
            fn = fn.strip()
            args = [a.strip() for a in rest.rstrip(")").split(",") if a.strip()]
            ints: List[int] = []
            if fn in DATA_FNS:
                ints = [int(a) for a in args[DATA_FNS[fn]:]]
                args = args[:DATA_FNS[fn]]
            s.ops.append(Op(lhs.strip(), fn, args, ints))
            continue
        tok = line.split()
        kw = tok[0]
        if kw == "network":
            s.name = tok[1]
        elif kw == "input":
            if tok[1] == "tokens":
                s.tokens, s.in_cols = True, 1
            else:
                s.in_cols = int(tok[1])
        elif kw == "layer":
            s.layers.append(Layer(tok[1], tok[2].lower(), _kv(tok[3:])))
        elif kw == "output":
            s.output = tok[1]
        elif kw == "loss":
            s.loss = tok[1]
        elif kw == "optimizer":
            s.optimizer = tok[1]
            s.opt = {k: float(v) for k, v in _kv(tok[2:]).items()}
        elif kw == "schedule":
            s.schedule = tok[1]
            s.sched = {k: float(v) for k, v in _kv(tok[2:]).items()}
        elif kw == "precision":
            s.precision = tok[1]
        elif kw == "grad":
            if tok[1:] != ["input"]:
                raise ValueError(f"expected 'grad input': {line}")
            s.input_grad = True
        else:
            raise ValueError(f"unknown statement: {line}")
    if not s.output and s.ops:
        s.output = s.ops[-1].out
    return s


def out_cols(s: Spec) -> int:
    """Width of the output value (propagated through the graph)."""
    width = {"x": s.in_cols}
    for op in s.ops:
        if op.fn in ACT_CODES or op.fn in ("softmax", "add", "sub", "mul", "div", "scatter"):
            width[op.out] = width[op.args[0]]
            continue
        if op.fn == "concat":
            width[op.out] = width[op.args[0]] + width[op.args[1]]
            continue
        if op.fn == "slice":
            width[op.out] = op.ints[1] - op.ints[0]
            continue
        if op.fn == "index":
            width[op.out] = len(op.ints)
            continue
        l = s.layer(op.fn)
        if l.kind == "dense":
            width[op.out] = l.i("out")
        elif l.kind == "embedding":
            width[op.out] = l.i("dim")
        elif l.kind in ("attention", "moe"):
            width[op.out] = l.i("dim")
        else:
            width[op.out] = width[op.args[0]]
    return width[s.output]


# ---- the benchmark configurations ------------------------------------------------

C1 = """network C1
input 784
layer fc1 dense in=784 out=1024 act=relu
layer fc2 dense in=1024 out=1024 act=relu
layer fc3 dense in=1024 out=10
h1 = fc1(x)
h2 = fc2(h1)
y = fc3(h2)
output y
"""

C2 = """network C2
input tokens
layer emb embedding vocab=8192 dim=512
layer attn attention dim=512 heads=8 seq=256
layer ln1 layernorm
layer ff1 dense in=512 out=2048 act=gelu
layer ff2 dense in=2048 out=512
layer ln2 layernorm
h = emb(x)
a = attn(h)
r1 = add(a, h)
n1 = ln1(r1)
f1 = ff1(n1)
f = ff2(f1)
r2 = add(f, n1)
y = ln2(r2)
output y
"""

C3 = """network C3
input 1024
layer moe moe dim=1024 experts=8 ffn=1024
y = moe(x)
output y
loss mse
optimizer adamw
grad input
"""

C4 = """network C4
input tokens
layer emb embedding vocab=8192 dim=512
layer attn attention dim=512 heads=8 seq=256
layer ln1 layernorm
layer ff1 dense in=512 out=2048 act=gelu
layer ff2 dense in=2048 out=512
layer ln2 layernorm
layer head dense in=512 out=8192
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
schedule cosine warmup=100 total=10000 min=0.05
"""


def c5(layers: int = 8, dim: int = 4096) -> str:
    lines = ["network C5", f"input {dim}"]
    for i in range(layers):
        act = "relu" if i + 1 < layers else "identity"
        lines.append(f"layer fc{i + 1} dense in={dim} out={dim} act={act}")
    prev = "x"
    for i in range(layers):
        lines.append(f"h{i + 1} = fc{i + 1}({prev})")
        prev = f"h{i + 1}"
    lines += [f"output {prev}", "loss mse", "optimizer muon momentum=0.95 steps=5 decay=0.01"]
    return "\n".join(lines) + "\n"


C5 = c5()

CONFIGS = {"c1": C1, "c2": C2, "c3": C3, "c4": C4, "c5": C5}

# Config 3 as BASELINE.json words it: each expert a single [D, D] matrix scaled
# by its routing weight (no counterpart in the reference's code, whose
# experts are D -> ffn -> D FFNs; C3 above is that reference-expressible form).
C3_LINEAR = """network C3L
input 1024
layer moe moe dim=1024 experts=8 expert=linear
y = moe(x)
output y
"""
