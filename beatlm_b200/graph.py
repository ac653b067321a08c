"""The kernel IR of the encoder path and its lowering to fused kernels.

A restatement of the reference's ``Graph`` / ``Graph::lower`` / ``fuse``
(crates/beatlm-core/src/kernel.rs:1285-1403, rules at kernel.rs:67-149) for
the operations the ViT encoder uses, plus the fused forms this backend adds.
A ``Graph`` lists typed operations over tensor ids in program order;
``lower`` turns it into a ``Program``: the kernels to launch, each a main
operation with an optional prologue and an epilogue chain, and every
remaining tensor's lifetime derived from those kernels (rule 1).

The reference's rules, kept as they are:

* rule 2, backward fusion: an element-wise operation (Add, Relu, Gelu,
  GeluErf, Scale, ChannelScale) becomes a step of the previous kernel's
  epilogue when that kernel's main operation is heavy (not a Map), the
  operation reads the tensor the kernel writes, that tensor has no other
  consumer and is not a graph output, and the kernel's bindings stay within
  the profile's limit (``binding_limit``; 8 on the reference's WebGPU
  baseline, none for this backend's pointer arguments);
* ``Fusion.OFF`` lowers to one kernel per operation;
* malformed graphs are errors (rule 5): unknown or repeated tensors, a write
  to an input or a weight, a tensor written twice or read before it is
  written, an activation or output nothing writes.

The forms this backend adds (``forms``), each folding only tensors nothing
else reads (single consumer, an activation, never a graph output):

* ``"attention"``: AttentionScores, its Scale, Softmax and AttentionValues
  become one ``Attention`` main operation (the online-softmax kernel the
  reference anticipates at kernel.rs:232-234): the scores and probabilities
  never exist;
* ``"ln_prologue"``: a LayerNorm read only by the MatMul right after it, as
  that MatMul's A operand, becomes the MatMul's prologue (it reads the
  LayerNorm's input and normalises each row as it loads it), when the
  LayerNorm's input is written by a MatMul kernel (whose epilogue then writes
  the row statistics the prologue uses);
* ``"ln_epilogue"``: a LayerNorm read only as a MatMul's A operand joins the
  epilogue of the MatMul kernel that wrote its input, as a second output,
  when that kernel has no such step yet and its rows are at most 512 wide;
* ``"embedding"``: a PrependToken whose tokens are a PatchEmbed's output
  folds into the PatchEmbed kernel (its rows are placed after the class
  token), so the position Add joins that kernel by rule 2;
* ``"tokens_to_map"``: a TokensToMap of a kernel's output folds into that
  kernel (the class row is left out as rows are stored).

``B200_FORMS`` is what the encoder uses; ``lower(Fusion.ON, forms=())`` is the
reference's own lowering, checked against its test
(kernel.rs:3796-3844).
"""
from __future__ import annotations

import dataclasses
import enum

INPUT, WEIGHT, ACTIVATION, OUTPUT = "input", "weight", "activation", "output"

# ------------------------------------------------------------------ operations


@dataclasses.dataclass(frozen=True)
class LayerNorm:
    input: int
    gamma: int
    beta: int
    rows: int
    channels: int
    eps: float


@dataclasses.dataclass(frozen=True)
class MatMul:
    a: int
    b: int
    bias: int | None
    m: int
    k: int
    n: int


@dataclasses.dataclass(frozen=True)
class PatchEmbed:
    input: int
    weights: int
    bias: int | None
    grid_h: int
    grid_w: int
    patch: int
    cin: int
    cout: int


@dataclasses.dataclass(frozen=True)
class PrependToken:
    token: int
    tokens: int
    rows: int
    channels: int


@dataclasses.dataclass(frozen=True)
class TokensToMap:
    input: int
    rows: int  # rows of the input, the class row included
    channels: int


@dataclasses.dataclass(frozen=True)
class AttentionScores:
    qkv: int
    tokens: int
    heads: int
    head_dim: int


@dataclasses.dataclass(frozen=True)
class Softmax:
    input: int
    rows: int
    cols: int


@dataclasses.dataclass(frozen=True)
class AttentionValues:
    probs: int
    qkv: int
    tokens: int
    heads: int
    head_dim: int


@dataclasses.dataclass(frozen=True)
class Add:
    a: int
    b: int
    elements: int


@dataclasses.dataclass(frozen=True)
class Relu:
    input: int
    elements: int


@dataclasses.dataclass(frozen=True)
class Gelu:
    input: int
    elements: int


@dataclasses.dataclass(frozen=True)
class GeluErf:
    input: int
    elements: int


@dataclasses.dataclass(frozen=True)
class Scale:
    input: int
    factor: float
    elements: int


@dataclasses.dataclass(frozen=True)
class ChannelScale:
    input: int
    scale: int
    rows: int
    channels: int


# main operations that exist only after lowering


@dataclasses.dataclass(frozen=True)
class Attention:
    """AttentionScores -> Scale -> Softmax -> AttentionValues as one kernel."""
    qkv: int
    tokens: int
    heads: int
    head_dim: int
    scale: float


@dataclasses.dataclass(frozen=True)
class Map:
    """A standalone element-wise kernel (the reference's MainOp::Map)."""
    input: int
    elements: int


ELEMENTWISE = (Add, Relu, Gelu, GeluErf, Scale, ChannelScale)


def reads(op) -> list[int]:
    """The tensors an operation (or main operation) reads, in binding order,
    with repeats (kernel.rs:899 for operations, 1450 for main operations)."""
    if isinstance(op, LayerNorm):
        return [op.input, op.gamma, op.beta]
    if isinstance(op, MatMul):
        return [op.a, op.b] + ([op.bias] if op.bias is not None else [])
    if isinstance(op, PatchEmbed):
        return [op.input, op.weights] + ([op.bias] if op.bias is not None else [])
    if isinstance(op, PrependToken):
        return [op.token, op.tokens]
    if isinstance(op, TokensToMap):
        return [op.input]
    if isinstance(op, (AttentionScores, Attention)):
        return [op.qkv]
    if isinstance(op, Softmax):
        return [op.input]
    if isinstance(op, AttentionValues):
        return [op.probs, op.qkv]
    if isinstance(op, Add):
        return [op.a, op.b]
    if isinstance(op, ChannelScale):
        return [op.input, op.scale]
    if isinstance(op, (Relu, Gelu, GeluErf, Scale, Map)):
        return [op.input]
    raise TypeError("unknown operation %r" % (op,))


MAIN_NAMES = {LayerNorm: "layernorm", MatMul: "matmul", PatchEmbed: "patch_embed",
              PrependToken: "prepend_token", TokensToMap: "tokens_to_map",
              AttentionScores: "attention_scores", Softmax: "softmax",
              AttentionValues: "attention_values", Attention: "attention", Map: "map"}

# ------------------------------------------------------------------ kernels


@dataclasses.dataclass(frozen=True)
class Step:
    """One epilogue step (kernel.rs:1595-1655) or prologue step.

    kind: "add" (tensor), "relu", "gelu", "gelu_erf", "scale" (value: the
    factor), "channel_scale" (tensor, channels); this backend's
    "prepend_token" (tensor: the class token), "tokens_to_map", and
    "layernorm" (tensor: gamma, beta, value: eps; as an epilogue step also
    `out`, its second output)."""
    kind: str
    tensor: int | None = None
    value: float | None = None
    channels: int | None = None
    beta: int | None = None
    out: int | None = None

    def operands(self) -> list[int]:
        if self.kind == "layernorm":
            return [t for t in (self.tensor, self.beta) if t is not None]
        return [self.tensor] if self.tensor is not None else []


@dataclasses.dataclass
class Kernel:
    """A kernel of the program (the reference's KernelSpec): its main
    operation, prologue and epilogue steps, the tensor it writes (and, for a
    LayerNorm epilogue step, a second one) and the operations it covers."""
    main: object
    prologue: list
    epilogue: list
    output: int
    ops: tuple  # (start, end) operation indices, end exclusive
    label: str = ""

    def name(self) -> str:
        """kernel.rs:2119: prologue steps, the main operation, the epilogue
        steps, as in ``layernorm-matmul+gelu_erf``."""
        s = "".join(p.kind + "-" for p in self.prologue) + MAIN_NAMES[type(self.main)]
        return s + "".join("+" + e.kind for e in self.epilogue)

    def writes(self) -> list[int]:
        return [self.output] + [e.out for e in self.epilogue if e.out is not None]

    def bindings(self) -> list[int]:
        """kernel.rs:2096-2112: the main operation's reads, then the tensors
        the prologue and epilogue steps read, each once, then the output(s)."""
        out: list[int] = []
        for t in reads(self.main) + [t for p in self.prologue for t in p.operands()] + \
                [t for e in self.epilogue for t in e.operands()]:
            if t not in out:
                out.append(t)
        return out + self.writes()


class Fusion(enum.Enum):
    ON = "on"
    OFF = "off"


B200_FORMS = ("attention", "embedding", "tokens_to_map")
FORMS = ("attention", "ln_prologue", "ln_epilogue", "embedding", "tokens_to_map")


class GraphError(ValueError):
    """A malformed graph (the reference's KernelError, kernel.rs:2454)."""


class Graph:
    """Operations in program order over declared tensors."""

    def __init__(self):
        self.tensors: dict[int, tuple[str, int]] = {}  # id -> (role, elements)
        self.ops: list[tuple[object, int, str]] = []  # (op, output, name)
        self._written: set[int] = set()

    def tensor(self, tid: int, role: str, elements: int) -> int:
        if tid in self.tensors:
            raise GraphError("tensor %d declared twice" % tid)
        if role not in (INPUT, WEIGHT, ACTIVATION, OUTPUT):
            raise GraphError("tensor %d: role %r" % (tid, role))
        if elements < 1:
            raise GraphError("tensor %d: no elements" % tid)
        self.tensors[tid] = (role, int(elements))
        return tid

    def role(self, tid: int) -> str | None:
        return self.tensors.get(tid, (None, 0))[0]

    def op(self, op, output: int, name: str = "") -> int:
        for t in reads(op):
            if t not in self.tensors:
                raise GraphError("operation reads unknown tensor %d" % t)
            if self.role(t) in (ACTIVATION, OUTPUT) and t not in self._written:
                raise GraphError("tensor %d is read before it is written" % t)
        if output not in self.tensors:
            raise GraphError("operation writes unknown tensor %d" % output)
        if self.role(output) in (INPUT, WEIGHT):
            raise GraphError("operation writes %s tensor %d" % (self.role(output), output))
        if output in self._written:
            raise GraphError("tensor %d is written twice" % output)
        self._written.add(output)
        self.ops.append((op, output, name))
        return output

    def _consumers(self) -> dict[int, int]:
        n: dict[int, int] = {}
        for op, _, _ in self.ops:
            for t in reads(op):
                n[t] = n.get(t, 0) + 1
        return n

    def _alone(self, tid: int, consumers) -> bool:
        """A tensor fusion may make disappear: an activation read once."""
        return self.role(tid) == ACTIVATION and consumers.get(tid, 0) == 1

    def lower(self, fusion: Fusion = Fusion.ON, forms=B200_FORMS, binding_limit=None,
              ln_rows_limit: int = 512) -> "Program":
        """Graph::lower (kernel.rs:1285-1339) with this backend's forms."""
        if not self.ops:
            raise GraphError("the graph has no operations")
        for tid, (role, _) in self.tensors.items():
            if role in (ACTIVATION, OUTPUT) and tid not in self._written:
                raise GraphError("tensor %d is never written" % tid)
        forms = set(forms) if fusion == Fusion.ON else set()
        unknown = forms - set(FORMS)
        if unknown:
            raise ValueError("unknown fusion forms %s" % sorted(unknown))
        consumers = self._consumers()
        kernels: list[Kernel] = []
        writer: dict[int, int] = {}  # tensor -> index of the kernel that writes it
        skip = set()
        for index, (op, output, name) in enumerate(self.ops):
            if index in skip:
                continue
            if fusion == Fusion.ON and kernels:
                if self._fuse(kernels, op, output, index, consumers, binding_limit):
                    writer[output] = len(kernels) - 1
                    continue
                if self._fold_forms(kernels, writer, op, output, name, index, consumers, forms,
                                    skip, ln_rows_limit):
                    continue
            main, epilogue = self._standalone(op)
            kernels.append(Kernel(main, [], epilogue, output, (index, index + 1), name))
            writer[output] = len(kernels) - 1
        return Program(kernels, self)

    # rule 2 (kernel.rs:1347-1375)
    def _fuse(self, kernels, op, output, index, consumers, limit) -> bool:
        last = kernels[-1]
        if isinstance(last.main, Map) or not isinstance(op, ELEMENTWISE):
            return False
        chain = last.output
        if not self._alone(chain, consumers):
            return False
        step = _as_epilogue(op, chain)
        if step is None:
            return False
        fused = dataclasses.replace(last, epilogue=last.epilogue + [step], output=output,
                                    ops=(last.ops[0], index + 1))
        if limit is not None and len(fused.bindings()) > limit:
            return False
        kernels[-1] = fused
        return True

    def _fold_forms(self, kernels, writer, op, output, name, index, consumers, forms, skip,
                    ln_rows_limit) -> bool:
        last = kernels[-1]
        # AttentionScores (+ Scale) -> Softmax -> AttentionValues
        if ("attention" in forms and isinstance(op, Softmax)
                and isinstance(last.main, AttentionScores)
                and all(e.kind == "scale" for e in last.epilogue) and len(last.epilogue) <= 1
                and op.input == last.output and self._alone(last.output, consumers)
                and index + 1 < len(self.ops)):
            nxt, nout, nname = self.ops[index + 1]
            if (isinstance(nxt, AttentionValues) and nxt.probs == output
                    and nxt.qkv == last.main.qkv and self._alone(output, consumers)):
                s = last.main
                scale = last.epilogue[0].value if last.epilogue else 1.0
                kernels[-1] = Kernel(Attention(s.qkv, s.tokens, s.heads, s.head_dim, scale), [],
                                     [], nout, (last.ops[0], index + 2), last.label or nname)
                writer[nout] = len(kernels) - 1
                skip.add(index + 1)
                return True
        # LayerNorm as the prologue of the MatMul right after it
        if ("ln_prologue" in forms and isinstance(op, MatMul)
                and isinstance(last.main, LayerNorm) and not last.epilogue
                and not last.prologue and op.a == last.output
                and self._alone(last.output, consumers)):
            ln = last.main
            src = writer.get(ln.input)
            if src is not None and isinstance(kernels[src].main, MatMul):
                kernels[-1] = Kernel(dataclasses.replace(op, a=ln.input),
                                     [Step("layernorm", ln.gamma, ln.eps, beta=ln.beta)], [],
                                     output, (last.ops[0], index + 1), name)
                writer[output] = len(kernels) - 1
                return True
        # LayerNorm as a second output of the MatMul kernel that wrote its input
        if "ln_epilogue" in forms and isinstance(op, LayerNorm) and op.channels <= ln_rows_limit:
            src = writer.get(op.input)
            feeds_matmul = any(isinstance(o, MatMul) and o.a == output for o, _, _ in self.ops)
            if (src is not None and isinstance(kernels[src].main, MatMul)
                    and kernels[src].output == op.input and feeds_matmul
                    and self._alone(output, consumers)
                    and not any(e.kind == "layernorm" for e in kernels[src].epilogue)):
                k = kernels[src]
                kernels[src] = dataclasses.replace(
                    k, epilogue=k.epilogue + [Step("layernorm", op.gamma, op.eps, beta=op.beta,
                                                   out=output)])
                writer[output] = src
                return True
        # PrependToken of a PatchEmbed's rows
        if ("embedding" in forms and isinstance(op, PrependToken)
                and isinstance(last.main, PatchEmbed) and not last.epilogue
                and op.tokens == last.output and self._alone(last.output, consumers)):
            kernels[-1] = dataclasses.replace(
                last, epilogue=[Step("prepend_token", op.token)], output=output,
                ops=(last.ops[0], index + 1))
            writer[output] = len(kernels) - 1
            return True
        # TokensToMap of the last kernel's rows
        if ("tokens_to_map" in forms and isinstance(op, TokensToMap)
                and op.input == last.output and self._alone(last.output, consumers)):
            kernels[-1] = dataclasses.replace(
                last, epilogue=last.epilogue + [Step("tokens_to_map")], output=output,
                ops=(last.ops[0], index + 1))
            writer[output] = len(kernels) - 1
            return True
        return False

    @staticmethod
    def _standalone(op):
        """OpKind::standalone (kernel.rs:1050-1089)."""
        if isinstance(op, Add):
            return Map(op.a, op.elements), [Step("add", op.b)]
        if isinstance(op, Relu):
            return Map(op.input, op.elements), [Step("relu")]
        if isinstance(op, Gelu):
            return Map(op.input, op.elements), [Step("gelu")]
        if isinstance(op, GeluErf):
            return Map(op.input, op.elements), [Step("gelu_erf")]
        if isinstance(op, Scale):
            return Map(op.input, op.elements), [Step("scale", value=op.factor)]
        if isinstance(op, ChannelScale):
            return (Map(op.input, op.rows * op.channels),
                    [Step("channel_scale", op.scale, channels=op.channels)])
        return op, []


def _as_epilogue(op, chain) -> Step | None:
    """OpKind::as_epilogue (kernel.rs:1093-1112)."""
    if isinstance(op, Add):
        if op.a == chain and op.b != chain:
            return Step("add", op.b)
        if op.b == chain and op.a != chain:
            return Step("add", op.a)
        return None
    if isinstance(op, Relu) and op.input == chain:
        return Step("relu")
    if isinstance(op, Gelu) and op.input == chain:
        return Step("gelu")
    if isinstance(op, GeluErf) and op.input == chain:
        return Step("gelu_erf")
    if isinstance(op, Scale) and op.input == chain:
        return Step("scale", value=op.factor)
    if isinstance(op, ChannelScale) and op.input == chain and op.scale != chain:
        return Step("channel_scale", op.scale, channels=op.channels)
    return None


@dataclasses.dataclass(frozen=True)
class Lifetime:
    id: int
    elements: int
    first_use: int
    last_use: int


class Program:
    """Kernels in order and the lifetime of every tensor a kernel binds
    (rule 1, kernel.rs:2280-2330): an input, weight or output lives for the
    whole program; an activation from the kernel that writes it to the last
    kernel that reads it. A tensor no kernel binds (a fused intermediate)
    has none."""

    def __init__(self, kernels: list[Kernel], graph: Graph):
        self.kernels = kernels
        self.graph = graph
        last = len(kernels) - 1
        first: dict[int, int] = {}
        final: dict[int, int] = {}
        for i, k in enumerate(kernels):
            for t in k.bindings():
                first.setdefault(t, i)
                final[t] = i
        self.lifetimes = {}
        for t, (role, elements) in graph.tensors.items():
            if t not in first:
                continue
            if role == ACTIVATION:
                self.lifetimes[t] = Lifetime(t, elements, first[t], final[t])
            else:
                self.lifetimes[t] = Lifetime(t, elements, 0, last)

    def lifetime(self, tid: int):
        lt = self.lifetimes.get(tid)
        return None if lt is None else (lt.first_use, lt.last_use)

    def names(self) -> list[str]:
        return [k.name() for k in self.kernels]
