"""IR-direct model builders for the benchmark configurations.

``onnx`` is not available on the machines this backend is built and measured on, so the models
are built straight into the reference compiler's IR (``ml_graph_compiler.ir.Graph``) with the
node patterns ``torch.onnx`` emits at opset 17 for the same modules (the pattern catalogue is the
reference's ``samples.py:82-245``): Conv followed by BatchNormalization, Relu / Clip(0, 6),
residual Add, GlobalAveragePool + Flatten + Gemm(transB=1), LayerNormalization, the erf and tanh
GELU subgraphs, Shape->Gather->Concat->Reshape head splits, Split of the fused QKV projection,
Where-based causal masks and a tied LM head via Transpose.

Weights are random-init as the benchmark configurations specify, drawn with numpy from a seeded
generator (``weight_seed``); inputs come from ``feeds``. The graphs are returned un-optimised
(O0): ``ml_graph_compiler.passes.optimize`` turns them into the fused O3 graphs that the CUDA
target consumes.
"""

from __future__ import annotations

import math
from collections.abc import Callable
from typing import Any

import numpy as np

from mgc_cuda import _reference  # noqa: F401  (makes ml_graph_compiler importable)
from ml_graph_compiler.ir import Graph, TensorType, Value
from ml_graph_compiler.shape_inference import infer_shapes

WEIGHT_SEED_OFFSET = 10_000


class _Net:
    """Thin helper over ``Graph.add_node`` / ``Graph.constant`` with a seeded weight generator."""

    def __init__(self, name: str, seed: int) -> None:
        self.g = Graph(name)
        self.rng = np.random.default_rng(WEIGHT_SEED_OFFSET + seed)

    def const(self, array: Any, name: str = "const") -> Value:
        return self.g.constant(np.asarray(array), name)

    def scalar(self, v: float, name: str = "s") -> Value:
        return self.const(np.asarray(v, np.float32), name)

    def normal(self, shape: tuple[int, ...], std: float, name: str = "w") -> Value:
        data = (self.rng.standard_normal(shape, dtype=np.float32) * np.float32(std)).astype(
            np.float32
        )
        return self.const(data, name)

    def op(self, op: str, inputs: list[Value | None], n_outputs: int = 1, **attrs: Any) -> Any:
        node = self.g.add_node(op, inputs, n_outputs=n_outputs, attrs=attrs)
        return node.outputs[0] if n_outputs == 1 else list(node.outputs)

    def done(self, *outputs: tuple[Value, str]) -> Graph:
        for value, name in outputs:
            self.g.add_output(value, name)
        infer_shapes(self.g)
        return self.g

    # -- CNN pieces -------------------------------------------------------------------------
    def conv(
        self,
        x: Value,
        cin: int,
        cout: int,
        k: int,
        stride: int = 1,
        pad: int | None = None,
        group: int = 1,
        bias: bool = False,
        std: float | None = None,
    ) -> Value:
        fan_out = cout // group * k * k if group > 1 else cout * k * k
        std = math.sqrt(2.0 / fan_out) if std is None else std
        w = self.normal((cout, cin // group, k, k), std, "conv_w")
        p = k // 2 if pad is None else pad
        inputs: list[Value | None] = [x, w]
        if bias:
            inputs.append(self.normal((cout,), 0.1, "conv_b"))
        return self.op(
            "Conv",
            inputs,
            kernel_shape=[k, k],
            strides=[stride, stride],
            pads=[p, p, p, p],
            dilations=[1, 1],
            group=group,
        )

    def bn(self, x: Value, c: int, randomize: bool = False) -> Value:
        if randomize:
            scale = (1.0 + 0.1 * self.rng.standard_normal(c)).astype(np.float32)
            beta = (0.1 * self.rng.standard_normal(c)).astype(np.float32)
            mean = (0.1 * self.rng.standard_normal(c)).astype(np.float32)
            var = (0.5 + self.rng.random(c)).astype(np.float32)
        else:  # torchvision init: gamma 1, beta 0, running mean 0, running var 1
            scale, beta = np.ones(c, np.float32), np.zeros(c, np.float32)
            mean, var = np.zeros(c, np.float32), np.ones(c, np.float32)
        params = [self.const(a, n) for a, n in ((scale, "bn_s"), (beta, "bn_b"), (mean, "bn_m"))]
        params.append(self.const(var, "bn_v"))
        return self.op("BatchNormalization", [x, *params], epsilon=1e-5)

    def relu(self, x: Value) -> Value:
        return self.op("Relu", [x])

    def relu6(self, x: Value) -> Value:
        return self.op("Clip", [x, self.scalar(0.0, "clip_lo"), self.scalar(6.0, "clip_hi")])

    def head(self, x: Value, cin: int, classes: int, std: float = 0.01) -> Value:
        x = self.op("GlobalAveragePool", [x])
        x = self.op("Flatten", [x], axis=1)
        w = self.normal((classes, cin), std, "fc_w")
        b = self.const(np.zeros(classes, np.float32), "fc_b")
        return self.op("Gemm", [x, w, b], transB=1)

    # -- transformer pieces -------------------------------------------------------------------
    def layer_norm(self, x: Value, d: int, decomposed: bool = False) -> Value:
        gamma = self.const(np.ones(d, np.float32), "ln_g")
        beta = self.const(np.zeros(d, np.float32), "ln_b")
        if not decomposed:
            return self.op("LayerNormalization", [x, gamma, beta], axis=-1, epsilon=1e-5)
        mean = self.op("ReduceMean", [x], axes=[-1], keepdims=1)
        diff = self.op("Sub", [x, mean])
        var = self.op("ReduceMean", [self.op("Pow", [diff, self.scalar(2.0)])], axes=[-1], keepdims=1)
        std = self.op("Sqrt", [self.op("Add", [var, self.scalar(1e-5)])])
        y = self.op("Div", [diff, std])
        return self.op("Add", [self.op("Mul", [y, gamma]), beta])

    def gelu_erf(self, x: Value) -> Value:
        e = self.op("Erf", [self.op("Div", [x, self.scalar(math.sqrt(2.0))])])
        return self.op("Mul", [self.op("Mul", [x, self.op("Add", [e, self.scalar(1.0)])]), self.scalar(0.5)])

    def gelu_tanh(self, x: Value) -> Value:
        cube = self.op("Pow", [x, self.scalar(3.0)])
        inner = self.op("Add", [x, self.op("Mul", [self.scalar(0.044715), cube])])
        t = self.op("Tanh", [self.op("Mul", [self.scalar(math.sqrt(2.0 / math.pi)), inner])])
        return self.op("Mul", [self.op("Mul", [self.scalar(0.5), x]), self.op("Add", [self.scalar(1.0), t])])

    def dense(self, x: Value, din: int, dout: int, std: float = 0.02) -> Value:
        """MatMul + bias Add, as torch.onnx exports ``nn.Linear`` on a rank-3 input."""
        w = self.normal((din, dout), std, "dense_w")
        b = self.const(np.zeros(dout, np.float32), "dense_b")
        return self.op("Add", [self.op("MatMul", [x, w]), b])

    def conv1d(self, x: Value, batch_seq: tuple[int, int], din: int, dout: int) -> Value:
        """GPT-2 ``Conv1D``: view to 2-D, addmm (Gemm), view back."""
        b, s = batch_seq
        flat = self.op("Reshape", [x, self.const(np.asarray([-1, din], np.int64), "shape")])
        w = self.normal((din, dout), 0.02, "c_w")
        bias = self.const(np.zeros(dout, np.float32), "c_b")
        y = self.op("Gemm", [flat, w, bias])
        return self.op("Reshape", [y, self.const(np.asarray([b, s, dout], np.int64), "shape")])

    def dynamic_reshape(self, x: Value, tail: list[int]) -> Value:
        """Reshape whose target is computed from Shape at run time (folds statically)."""
        shape = self.op("Shape", [x])
        dims = [
            self.op(
                "Unsqueeze",
                [
                    self.op("Gather", [shape, self.const(np.asarray(i, np.int64), "i")], axis=0),
                    self.const(np.asarray([0], np.int64), "ax"),
                ],
            )
            for i in (0, 1)
        ]
        target = self.op("Concat", [*dims, self.const(np.asarray(tail, np.int64), "tail")], axis=0)
        return self.op("Reshape", [x, target])


# ---------------------------------------------------------------------------------------------
# CNNs
# ---------------------------------------------------------------------------------------------
def resnet50(batch: int = 1, seed: int = 0, classes: int = 1000) -> Graph:
    """torchvision ResNet-50 v1.5 (stride on the 3x3 conv of each bottleneck)."""
    n = _Net("resnet50", seed)
    x = n.g.add_input("image", TensorType("float32", (batch, 3, 224, 224)))
    y = n.relu(n.bn(n.conv(x, 3, 64, 7, stride=2, pad=3), 64))
    y = n.op("MaxPool", [y], kernel_shape=[3, 3], strides=[2, 2], pads=[1, 1, 1, 1])
    cin = 64
    for width, blocks, stride in ((64, 3, 1), (128, 4, 2), (256, 6, 2), (512, 3, 2)):
        for i in range(blocks):
            s = stride if i == 0 else 1
            h = n.relu(n.bn(n.conv(y, cin, width, 1, pad=0), width))
            h = n.relu(n.bn(n.conv(h, width, width, 3, stride=s), width))
            h = n.bn(n.conv(h, width, width * 4, 1, pad=0), width * 4)
            if i == 0:
                sc = n.bn(n.conv(y, cin, width * 4, 1, stride=s, pad=0), width * 4)
            else:
                sc = y
            y = n.relu(n.op("Add", [h, sc]))
            cin = width * 4
    return n.done((n.head(y, 2048, classes), "logits"))


def mobilenet_v2(batch: int = 1, seed: int = 1, classes: int = 1000) -> Graph:
    """torchvision MobileNetV2 (width 1.0, ReLU6 exported as Clip with constant bounds)."""
    n = _Net("mobilenet_v2", seed)

    def std(cout: int, k: int, group: int = 1) -> float:  # kaiming_normal_(mode="fan_out")
        return math.sqrt(2.0 / (cout // group * k * k))

    x = n.g.add_input("image", TensorType("float32", (batch, 3, 224, 224)))
    y = n.relu6(n.bn(n.conv(x, 3, 32, 3, stride=2, std=std(32, 3)), 32))
    cin = 32
    for t, c, reps, s in (
        (1, 16, 1, 1),
        (6, 24, 2, 2),
        (6, 32, 3, 2),
        (6, 64, 4, 2),
        (6, 96, 3, 1),
        (6, 160, 3, 2),
        (6, 320, 1, 1),
    ):
        for i in range(reps):
            stride = s if i == 0 else 1
            hidden = cin * t
            h = y
            if t != 1:
                h = n.relu6(n.bn(n.conv(h, cin, hidden, 1, pad=0, std=std(hidden, 1)), hidden))
            h = n.relu6(
                n.bn(n.conv(h, hidden, hidden, 3, stride=stride, group=hidden, std=std(hidden, 3, hidden)), hidden)
            )
            h = n.bn(n.conv(h, hidden, c, 1, pad=0, std=std(c, 1)), c)
            y = n.op("Add", [y, h]) if stride == 1 and cin == c else h
            cin = c
    y = n.relu6(n.bn(n.conv(y, cin, 1280, 1, pad=0, std=std(1280, 1)), 1280))
    return n.done((n.head(y, 1280, classes), "logits"))


def tiny_cnn(batch: int = 1, size: int = 32, channels: int = 16, classes: int = 10, seed: int = 0) -> Graph:
    """ResNet and MobileNetV2 style blocks at toy size (the reference's ``samples.tiny_cnn``
    topology, ``samples.py:101-133``), with randomised BatchNorm statistics."""
    n = _Net("tiny_cnn", seed)

    def cbn(x: Value, cin: int, cout: int, k: int, stride: int = 1, group: int = 1) -> Value:
        return n.bn(n.conv(x, cin, cout, k, stride=stride, group=group, std=0.3), cout, randomize=True)

    x = n.g.add_input("image", TensorType("float32", (batch, 3, size, size)))
    y = n.relu(cbn(x, 3, channels, 3, stride=2))
    y = n.op("MaxPool", [y], kernel_shape=[3, 3], strides=[2, 2], pads=[1, 1, 1, 1])
    h = n.relu(cbn(y, channels, channels, 3))
    h = cbn(h, channels, channels, 3)
    y = n.relu(n.op("Add", [h, y]))
    e = n.relu6(cbn(y, channels, channels * 2, 1))
    e = n.relu6(cbn(e, channels * 2, channels * 2, 3, group=channels * 2))
    e = cbn(e, channels * 2, channels, 1)
    y = n.op("Add", [y, e])
    h = n.relu(cbn(y, channels, channels * 2, 3, stride=2))
    h = cbn(h, channels * 2, channels * 2, 3)
    sc = cbn(y, channels, channels * 2, 1, stride=2)
    y = n.relu(n.op("Add", [h, sc]))
    return n.done((n.head(y, channels * 2, classes, std=0.3), "logits"))


# ---------------------------------------------------------------------------------------------
# transformers
# ---------------------------------------------------------------------------------------------
def _attention(
    n: _Net, h: Value, batch: int, seq: int, d: int, heads: int, causal: bool, mask: Value | None,
    gpt2: bool,
) -> Value:
    dh = d // heads
    if gpt2:
        qkv = n.conv1d(h, (batch, seq), d, 3 * d)
        q, k, v = n.op("Split", [qkv, n.const(np.asarray([d, d, d], np.int64), "split")], 3, axis=2)
    else:
        q, k, v = (n.dense(h, d, d) for _ in range(3))

    def heads_first(t: Value) -> Value:
        return n.op("Transpose", [n.dynamic_reshape(t, [heads, dh])], perm=[0, 2, 1, 3])

    q, k, v = heads_first(q), heads_first(k), heads_first(v)
    kt = n.op("Transpose", [k], perm=[0, 1, 3, 2])
    scores = n.op("Div", [n.op("MatMul", [q, kt]), n.scalar(math.sqrt(dh))])
    if causal:
        upper = np.triu(np.ones((seq, seq), dtype=bool), 1)[None, None]
        neg = n.const(np.asarray(np.finfo(np.float32).min, np.float32), "mask_value")
        scores = n.op("Where", [n.const(upper, "causal"), neg, scores])
    if mask is not None:
        scores = n.op("Add", [scores, mask])
    ctx = n.op("MatMul", [n.op("Softmax", [scores], axis=-1), v])
    ctx = n.op("Transpose", [ctx], perm=[0, 2, 1, 3])
    ctx = n.dynamic_reshape(ctx, [d])
    return n.conv1d(ctx, (batch, seq), d, d) if gpt2 else n.dense(ctx, d, d)


def bert(
    batch: int = 1,
    seq: int = 128,
    layers: int = 12,
    d: int = 768,
    heads: int = 12,
    ffn: int = 3072,
    vocab: int = 30522,
    max_pos: int = 512,
    seed: int = 2,
    pooler: bool = True,
    decomposed_ln: bool = False,
) -> Graph:
    """BERT encoder (post-LayerNorm, erf GELU) with the HF extended attention mask."""
    n = _Net("bert", seed)
    ids = n.g.add_input("input_ids", TensorType("int64", (batch, seq)))
    am = n.g.add_input("attention_mask", TensorType("int64", (batch, seq)))
    word = n.normal((vocab, d), 0.02, "word_emb")
    pos = n.normal((max_pos, d), 0.02, "pos_emb")
    tok = n.normal((2, d), 0.02, "tok_emb")
    x = n.op("Gather", [word, ids], axis=0)
    pos_ids = n.const(np.arange(seq, dtype=np.int64)[None, :], "pos_ids")
    x = n.op("Add", [x, n.op("Gather", [tok, n.const(np.zeros((1, seq), np.int64), "tt")], axis=0)])
    x = n.op("Add", [x, n.op("Gather", [pos, pos_ids], axis=0)])
    x = n.layer_norm(x, d, decomposed_ln)
    ext = n.op("Unsqueeze", [am, n.const(np.asarray([1, 2], np.int64), "ax")])
    ext = n.op("Cast", [ext], to=1)
    ext = n.op("Sub", [n.scalar(1.0), ext])
    ext = n.op("Mul", [ext, n.const(np.asarray(np.finfo(np.float32).min, np.float32), "fmin")])
    for _ in range(layers):
        a = _attention(n, x, batch, seq, d, heads, False, ext, gpt2=False)
        x = n.layer_norm(n.op("Add", [a, x]), d, decomposed_ln)
        f = n.dense(n.gelu_erf(n.dense(x, d, ffn)), ffn, d)
        x = n.layer_norm(n.op("Add", [f, x]), d, decomposed_ln)
    outputs = [(x, "last_hidden_state")]
    if pooler:
        first = n.op("Gather", [x, n.const(np.asarray(0, np.int64), "first")], axis=1)
        w = n.normal((d, d), 0.02, "pool_w")
        pooled = n.op("Tanh", [n.op("Gemm", [first, w, n.const(np.zeros(d, np.float32), "pool_b")], transB=1)])
        outputs.append((pooled, "pooler_output"))
    return n.done(*outputs)


def gpt2(
    batch: int = 1,
    seq: int = 128,
    layers: int = 12,
    d: int = 768,
    heads: int = 12,
    vocab: int = 50257,
    max_pos: int = 1024,
    seed: int = 3,
    decomposed_ln: bool = False,
) -> Graph:
    """GPT-2 decoder (pre-LayerNorm, tanh GELU, causal mask, LM head tied to ``wte``)."""
    n = _Net("gpt2", seed)
    ids = n.g.add_input("input_ids", TensorType("int64", (batch, seq)))
    wte = n.normal((vocab, d), 0.02, "wte")
    wpe = n.normal((max_pos, d), 0.01, "wpe")
    x = n.op("Gather", [wte, ids], axis=0)
    x = n.op("Add", [x, n.op("Gather", [wpe, n.const(np.arange(seq, dtype=np.int64)[None, :], "pos")], axis=0)])
    for _ in range(layers):
        a = _attention(n, n.layer_norm(x, d, decomposed_ln), batch, seq, d, heads, True, None, gpt2=True)
        x = n.op("Add", [x, a])
        h = n.conv1d(n.layer_norm(x, d, decomposed_ln), (batch, seq), d, 4 * d)
        x = n.op("Add", [x, n.conv1d(n.gelu_tanh(h), (batch, seq), 4 * d, d)])
    x = n.layer_norm(x, d, decomposed_ln)
    logits = n.op("MatMul", [x, n.op("Transpose", [wte], perm=[1, 0])])
    return n.done((logits, "logits"))


def tiny_transformer(
    batch: int = 1, seq: int = 8, d: int = 32, heads: int = 4, layers: int = 2, vocab: int = 128,
    kind: str = "gpt", seed: int = 0,
) -> Graph:
    """Toy GPT-2 (``kind="gpt"``) or BERT (``kind="bert"``) at the reference's tiny sizes
    (``samples.py:183-245``), using the decomposed LayerNorm that LN fusion must find."""
    if kind == "gpt":
        g = gpt2(batch, seq, layers, d, heads, vocab, max_pos=seq, seed=seed, decomposed_ln=True)
    else:
        g = bert(batch, seq, layers, d, heads, 4 * d, vocab, max_pos=seq, seed=seed,
                 decomposed_ln=True)
    return g


def mlp(batch: int = 4, sizes: tuple[int, ...] = (16, 32, 32, 10), seed: int = 0) -> Graph:
    """MatMul + Add + Relu layers, then Softmax (the reference's ``samples.mlp``)."""
    n = _Net("mlp", seed)
    x = n.g.add_input("x", TensorType("float32", (batch, sizes[0])))
    for i in range(len(sizes) - 1):
        x = n.op("MatMul", [x, n.normal((sizes[i], sizes[i + 1]), 0.3, "w")])
        x = n.op("Add", [x, n.normal((sizes[i + 1],), 0.1, "b")])
        if i < len(sizes) - 2:
            x = n.relu(x)
    return n.done((n.op("Softmax", [x], axis=-1), "y"))


# ---------------------------------------------------------------------------------------------
# inputs
# ---------------------------------------------------------------------------------------------
def feeds(graph: Graph, seed: int) -> dict[str, np.ndarray]:
    """Seeded inputs: N(0,1) float images, token ids uniform in [0, vocab), all-ones masks."""
    rng = np.random.default_rng(seed)
    out: dict[str, np.ndarray] = {}
    for v in graph.inputs:
        t = v.tensor_type
        if t.dtype == "float32":
            out[v.name] = rng.standard_normal(t.shape).astype(np.float32)
        elif v.name == "attention_mask":
            out[v.name] = np.ones(t.shape, np.int64)
        else:
            vocab = _vocab_of(graph, v)
            out[v.name] = rng.integers(0, vocab, t.shape).astype(np.int64)
    return out


def _vocab_of(graph: Graph, ids: Value) -> int:
    for user in ids.users:
        if user.op == "Gather" and user.inputs[0] is not None and user.inputs[0].type is not None:
            return int(user.inputs[0].tensor_type.shape[0])
    return 100


MODELS: dict[str, Callable[..., Graph]] = {
    "resnet50": resnet50,
    "mobilenet_v2": mobilenet_v2,
    "bert": bert,
    "gpt2": gpt2,
    "tiny_cnn": tiny_cnn,
    "tiny_transformer": tiny_transformer,
    "mlp": mlp,
}
