"""Neural-network modules with the reference's names and parameter layout.

Reference: nn.py:28-670.  Every module keeps its constructor signature,
parameter names and deterministic LCG initialisation.  Extensions for real
training on B200:

* inputs may carry a batch dimension ([B, T, F]); attention is multi-head
  (``heads=1`` reproduces the reference's single-head layer);
* RMSNorm / LayerNorm propagate gradients to their input (the reference
  stops them, nn.py:163 and :181; ``compat="reference"`` restores that);
* ``Module.to(device, dtype)`` moves parameters; on CUDA every layer runs this
  package's kernels (tcgen05 GEMMs, flash attention, fused RMSNorm, GELU,
  embedding, softmax cross-entropy, conv2d);
* a TransformerLM moved to CUDA in bf16 executes as one fused engine over
  flat parameter / gradient buffers (models/transformer.py).
"""

from __future__ import annotations

import math
from collections import OrderedDict
from dataclasses import dataclass
from typing import Any, Iterable, Iterator

import torch

from underhfs_b200 import functional as F
from underhfs_b200.tensor import (
    CUDA_TORCH_DTYPE,
    Device,
    DType,
    Layout,
    Tensor,
    kaiming_uniform,
    ones,
    tensor,
    torch_dtype_for,
    uniform,
    zeros,
)


@dataclass(frozen=True)
class BackendStatus:
    name: str
    backend: str
    available: bool
    reason: str = ""

    def to_dict(self) -> dict[str, str | bool]:
        return {"name": self.name, "backend": self.backend, "available": self.available, "reason": self.reason}


class Parameter(Tensor):
    """A Tensor that a Module registers as trainable (always requires grad)."""

    def __init__(self, data: Any, **kwargs: Any) -> None:
        if isinstance(data, Tensor):
            t = data._data.detach().clone()
            super().__init__(_data=t, dtype=data.dtype, device=data.device, layout=data.layout)
        else:
            kwargs.pop("requires_grad", None)
            super().__init__(data, **kwargs)
        self._data.requires_grad_(True)

    def _rebind(self, t: torch.Tensor, *, requires_grad: bool = True, dtype: DType | None = None) -> None:
        self._data = t
        if requires_grad and t.is_floating_point():
            t.requires_grad_(True)
        self.device = Device.parse(t.device)
        if dtype is not None:
            self.dtype = dtype


def _wrap(t: torch.Tensor, like: Tensor, op: str, parents: tuple, backend: str | None = None) -> Tensor:
    if backend is None:
        backend = "native_cuda" if t.is_cuda else "python"
    return Tensor._wrap(t, like=like, backend=backend, op=op, parents=parents)


class Module:
    def __init__(self) -> None:
        object.__setattr__(self, "_parameters", OrderedDict())
        object.__setattr__(self, "_modules", OrderedDict())
        object.__setattr__(self, "training", True)

    def __setattr__(self, name: str, value: Any) -> None:
        if isinstance(value, Parameter):
            self._parameters[name] = value
        elif isinstance(value, Module):
            self._modules[name] = value
        object.__setattr__(self, name, value)

    def parameters(self) -> Iterator[Parameter]:
        for _, p in self.named_parameters():
            yield p

    def named_parameters(self, prefix: str = "") -> Iterator[tuple[str, Parameter]]:
        for name, p in self._parameters.items():
            yield f"{prefix}{name}", p
        for name, m in self._modules.items():
            yield from m.named_parameters(f"{prefix}{name}.")

    def iter_modules(self) -> Iterator["Module"]:
        yield self
        for m in self._modules.values():
            yield from m.iter_modules()

    def train(self, mode: bool = True) -> "Module":
        object.__setattr__(self, "training", mode)
        for m in self._modules.values():
            m.train(mode)
        return self

    def eval(self) -> "Module":
        return self.train(False)

    def zero_grad(self) -> None:
        for p in self.parameters():
            p.zero_grad()

    def state_dict(self, *, as_tensors: bool = False) -> dict[str, Any]:
        """Nested Python lists like the reference (exact: the parameter's own
        values, widened to Python floats), or detached fp32 CPU torch tensors
        with ``as_tensors=True`` (what large checkpoints use).  The live
        parameter is read, not an fp32 master copy: under ZeRO a rank's master
        is current only for its own shard."""
        out: dict[str, Any] = {}
        for name, p in self.named_parameters():
            value = p._data.detach()
            out[name] = value.float().cpu().clone() if as_tensors else value.double().cpu().tolist()
        return out

    def load_state_dict(self, state: dict[str, Any]) -> None:
        for name, p in self.named_parameters():
            if name not in state:
                raise KeyError(f"missing parameter {name}")
            value = state[name]
            if isinstance(value, Tensor):
                value = value._data
            src = value if isinstance(value, torch.Tensor) else torch.tensor(value, dtype=torch.float64)
            src = src.detach().reshape(p.shape).to(p._data.device, p._data.dtype)
            with torch.no_grad():
                p._data.copy_(src)
            master = getattr(p, "_master", None)
            if master is not None:
                master.copy_(src.float())

    def to(self, device: Device | str | None = None, dtype: DType | str | None = None) -> "Module":
        target = None if device is None else Device.parse(device)
        for p in self.parameters():
            moved = p.to(device=target, dtype=dtype)
            p._rebind(moved._data, dtype=moved.dtype)
        return self

    def cuda(self, index: int = 0, dtype: DType | str | None = None) -> "Module":
        return self.to(Device("cuda", index), dtype)

    def cpu(self) -> "Module":
        return self.to("cpu")

    def __call__(self, *args: Any, **kwargs: Any) -> Any:
        return self.forward(*args, **kwargs)

    def forward(self, *args: Any, **kwargs: Any) -> Any:
        raise NotImplementedError


# ------------------------------------------------------------------- layers
def _linear_t(x: torch.Tensor, w: torch.Tensor, b: torch.Tensor | None) -> torch.Tensor:
    if x.is_cuda:
        from underhfs_b200.ops import functions as OF

        return OF.linear(x, w, b)
    y = x @ w.t()
    return y + b if b is not None else y


class Linear(Module):
    def __init__(self, in_features: int, out_features: int, bias: bool = True) -> None:
        super().__init__()
        self.in_features = in_features
        self.out_features = out_features
        self.weight = Parameter(kaiming_uniform(out_features, in_features))
        self.bias = Parameter(zeros((out_features,))) if bias else None

    def forward(self, x: Tensor) -> Tensor:
        b = self.bias._data if self.bias is not None else None
        parents = (x, self.weight) + ((self.bias,) if self.bias is not None else ())
        return _wrap(_linear_t(x._data, self.weight._data, b), x, "linear", parents)


class ReLU(Module):
    def forward(self, x: Tensor) -> Tensor:
        return x.relu()


class GELU(Module):
    def forward(self, x: Tensor) -> Tensor:
        return F.gelu(x)


class Sequential(Module):
    def __init__(self, *modules: Module) -> None:
        super().__init__()
        object.__setattr__(self, "modules", list(modules))
        for i, m in enumerate(modules):
            setattr(self, str(i), m)

    def forward(self, x: Tensor) -> Tensor:
        for m in self.modules:
            x = m(x)
        return x


class ModuleList(Module):
    def __init__(self, modules: Iterable[Module] = ()) -> None:
        super().__init__()
        object.__setattr__(self, "modules", [])
        for m in modules:
            self.append(m)

    def __iter__(self) -> Iterator[Module]:
        return iter(self.modules)

    def __len__(self) -> int:
        return len(self.modules)

    def __getitem__(self, i: int) -> Module:
        return self.modules[i]

    def append(self, module: Module) -> None:
        self.modules.append(module)
        setattr(self, str(len(self.modules) - 1), module)


class LayerNorm(Module):
    def __init__(self, features: int, eps: float = 1e-5, compat: str | None = None) -> None:
        super().__init__()
        self.weight = Parameter(ones((features,)))
        self.bias = Parameter(zeros((features,)))
        self.eps = eps
        self.compat = compat

    def forward(self, x: Tensor) -> Tensor:
        t = x._data
        if self.compat == "reference":
            t = t.detach()
        y = torch.nn.functional.layer_norm(t, (t.shape[-1],), None, None, self.eps)
        y = y * self.weight._data.to(y.dtype) + self.bias._data.to(y.dtype)
        return _wrap(y, x, "layer_norm", (x, self.weight, self.bias))


class RMSNorm(Module):
    def __init__(self, features: int, eps: float = 1e-8, compat: str | None = None) -> None:
        super().__init__()
        self.weight = Parameter(ones((features,)))
        self.eps = eps
        self.compat = compat

    def forward(self, x: Tensor) -> Tensor:
        t = x._data
        if self.compat == "reference":
            t = t.detach()
        if t.is_cuda:
            from underhfs_b200.ops import functions as OF

            y = OF.rmsnorm(t, self.weight._data, self.eps)
        else:
            y = t * torch.rsqrt(t.pow(2).mean(-1, keepdim=True) + self.eps) * self.weight._data
        return _wrap(y, x, "rms_norm", (x, self.weight))


class Embedding(Module):
    def __init__(self, num_embeddings: int, embedding_dim: int) -> None:
        super().__init__()
        self.weight = Parameter(kaiming_uniform(num_embeddings, embedding_dim))

    def forward(self, indices: Tensor) -> Tensor:
        ids = indices._data.detach().to(torch.int64)
        n = self.weight.shape[0]
        if ids.numel() and (int(ids.min()) < 0 or int(ids.max()) >= n):
            bad = int(ids[(ids < 0) | (ids >= n)][0])
            raise ValueError(f"embedding index {bad} outside [0, {n})")
        w = self.weight._data
        ids = ids.to(w.device)
        if w.is_cuda:
            from underhfs_b200.ops import functions as OF

            out = OF.embedding(ids, w)
        else:
            out = w[ids]
        return _wrap(out, self.weight, "embedding", (self.weight,))


class MLP(Module):
    def __init__(self, in_features: int, hidden_features: int, out_features: int) -> None:
        super().__init__()
        self.net = Sequential(Linear(in_features, hidden_features), GELU(), Linear(hidden_features, out_features))

    def forward(self, x: Tensor) -> Tensor:
        return self.net(x)


class SelfAttention(Module):
    """Multi-head self-attention (heads=1 is the reference's layer, nn.py:229-249)."""

    causal = False

    def __init__(self, features: int, bias: bool = True, heads: int = 1) -> None:
        super().__init__()
        if features % heads:
            raise ValueError("features must be divisible by heads")
        self.features = features
        self.heads = heads
        self.q_proj = Linear(features, features, bias=bias)
        self.k_proj = Linear(features, features, bias=bias)
        self.v_proj = Linear(features, features, bias=bias)
        self.out_proj = Linear(features, features, bias=bias)

    def forward(self, x: Tensor) -> Tensor:
        if x.ndim not in (2, 3):
            raise ValueError(f"{type(self).__name__} expects [tokens, features] or [batch, tokens, features]")
        t = x._data
        batched = t.dim() == 3
        if not batched:
            t = t.unsqueeze(0)
        B, T, Fd = t.shape
        H = self.heads
        D = Fd // H
        scale = 1.0 / math.sqrt(D)
        native = self._try_native(t, B, T, H, D, scale)
        if native is not None:
            o, backend = native
        else:
            q = _linear_t(t, self.q_proj.weight._data, _b(self.q_proj))
            k = _linear_t(t, self.k_proj.weight._data, _b(self.k_proj))
            v = _linear_t(t, self.v_proj.weight._data, _b(self.v_proj))
            qh, kh, vh = (z.view(B, T, H, D).transpose(1, 2) for z in (q, k, v))
            s = (qh @ kh.transpose(-1, -2)) * scale
            if self.causal:
                mask = torch.triu(torch.ones(T, T, dtype=torch.bool, device=t.device), 1)
                s = s.masked_fill(mask, -1.0e9)
            o = (torch.softmax(s, -1) @ vh).transpose(1, 2).reshape(B, T, Fd)
            backend = "native_cuda" if t.is_cuda else "python"
        y = _linear_t(o, self.out_proj.weight._data, _b(self.out_proj))
        if not batched:
            y = y.squeeze(0)
        out = _wrap(y, x, "attention", (x,), backend=backend)
        return out

    def _try_native(self, t: torch.Tensor, B: int, T: int, H: int, D: int, scale: float):
        if not t.is_cuda:
            return None
        from underhfs_b200.ops import functions as OF

        if t.dtype == torch.bfloat16 and D in (64, 128):
            w = torch.cat([self.q_proj.weight._data, self.k_proj.weight._data, self.v_proj.weight._data], 0)
            b = None
            if self.q_proj.bias is not None:
                b = torch.cat([self.q_proj.bias._data, self.k_proj.bias._data, self.v_proj.bias._data], 0)
            qkv = OF.linear(t.reshape(B * T, -1), w, b)
            o = OF.flash_attention(qkv, B, T, H, D, self.causal)
            return o.view(B, T, H * D), "native_cuda_attention"
        if t.dtype == torch.float32 and H == 1 and B == 1:
            q = OF.linear(t[0], self.q_proj.weight._data, _b(self.q_proj))
            k = OF.linear(t[0], self.k_proj.weight._data, _b(self.k_proj))
            v = OF.linear(t[0], self.v_proj.weight._data, _b(self.v_proj))
            o = OF.attention_f32(q, k, v, scale, self.causal)
            return o.unsqueeze(0), "native_cuda_attention"
        return None


def _b(lin: Linear) -> torch.Tensor | None:
    return lin.bias._data if lin.bias is not None else None


class CausalSelfAttention(SelfAttention):
    causal = True


class TransformerBlock(Module):
    def __init__(self, features: int, hidden_features: int, *, causal: bool = False, heads: int = 1) -> None:
        super().__init__()
        self.attn_norm = RMSNorm(features)
        self.attn = CausalSelfAttention(features, heads=heads) if causal else SelfAttention(features, heads=heads)
        self.mlp_norm = RMSNorm(features)
        self.mlp = MLP(features, hidden_features, features)

    def forward(self, x: Tensor) -> Tensor:
        x = x + self.attn(self.attn_norm(x))
        return x + self.mlp(self.mlp_norm(x))


class _EngineLoss(torch.autograd.Function):
    """Connects the fused engine to torch autograd through a scalar anchor."""

    @staticmethod
    def forward(ctx, anchor, engine, ids, targets, fuse):
        loss, _ = engine.forward(ids, targets, fuse_loss_grad=fuse)
        ctx.engine = engine
        ctx.fused = fuse
        return loss

    @staticmethod
    def backward(ctx, g):
        if ctx.fused:
            ctx.engine.backward()
        else:
            ctx.engine.backward(loss_grad=g.reshape(()).float().contiguous())
        return torch.zeros((), device=g.device), None, None, None, None


class _EngineLogits(torch.autograd.Function):
    @staticmethod
    def forward(ctx, anchor, engine, ids):
        _, logits = engine.forward(ids, None, fuse_loss_grad=False, keep_logits=True)
        ctx.engine = engine
        return logits

    @staticmethod
    def backward(ctx, g):
        ctx.engine.backward(dlogits=g)
        return torch.zeros((), device=g.device), None, None


class TransformerLM(Module):
    """Decoder-only LM (reference nn.py:287-334) with batch, heads and tying.

    ``forward(ids)`` returns logits ([T, V] for 1-D ids like the reference,
    [B, T, V] for 2-D); ``forward(ids, targets)`` returns the mean
    cross-entropy directly, which on the CUDA engine fuses the loss gradient
    into the forward pass.
    """

    def __init__(
        self,
        vocab_size: int,
        max_seq_len: int,
        features: int,
        hidden_features: int,
        layers: int,
        *,
        heads: int = 1,
        tied: bool = False,
        init: str = "reference",
        seed: int = 0,
        eps: float = 1e-8,
    ) -> None:
        super().__init__()
        self.vocab_size = vocab_size
        self.max_seq_len = max_seq_len
        self.features = features
        self.hidden_features = hidden_features
        self.heads = heads
        self.tied = tied
        self.token_embedding = Embedding(vocab_size, features)
        self.position_embedding = Embedding(max_seq_len, features)
        self.blocks = ModuleList(
            TransformerBlock(features, hidden_features, causal=True, heads=heads) for _ in range(layers)
        )
        self.norm = RMSNorm(features, eps=eps)
        for b in self.blocks:
            b.attn_norm.eps = eps
            b.mlp_norm.eps = eps
        if not tied:
            self.head = Linear(features, vocab_size, bias=False)
        object.__setattr__(self, "_engine", None)
        object.__setattr__(self, "_flat", None)
        object.__setattr__(self, "_zero3", None)
        if init != "reference":
            self._reinit(init, seed)

    # ---------------------------------------------------------- setup
    @property
    def spec(self):
        from underhfs_b200.models.transformer import LMSpec

        return LMSpec(self.vocab_size, self.max_seq_len, self.features, self.hidden_features, len(self.blocks),
                      self.heads, self.tied, self.norm.eps, True)

    def _reinit(self, init: str, seed: int) -> None:
        from underhfs_b200.models.transformer import initial_value

        gen = torch.Generator().manual_seed(seed)
        spec = self.spec
        for name, p in self.named_parameters():
            v = initial_value(spec, name, p.shape, init, gen)
            with torch.no_grad():
                p._data.copy_(v.to(p._data.dtype))

    def to(self, device: Device | str | None = None, dtype: DType | str | None = None,
           *, grad_alloc=None) -> "TransformerLM":
        if self._zero3 is not None:
            raise RuntimeError("this TransformerLM is sharded by ZeRO-3; its parameters live in the shards "
                               "(use state_dict() to gather them)")
        target = self.token_embedding.weight.device if device is None else Device.parse(device)
        want = DType(dtype) if dtype is not None else self.token_embedding.weight.dtype
        if target.kind == "cuda" and want is DType.BF16 and self.features // self.heads in (64, 128):
            self._materialize_engine(target, grad_alloc=grad_alloc)
            return self
        object.__setattr__(self, "_engine", None)
        object.__setattr__(self, "_flat", None)
        return super().to(device, dtype)

    def _materialize_engine(self, device: Device, grad_alloc=None) -> None:
        """Move every parameter into flat bf16/fp32 buffers on `device`."""
        from underhfs_b200.models.transformer import LMEngine, build_layout
        from underhfs_b200.parallel.flat import FlatBuffers

        _require_cuda(device)
        spec = self.spec
        flat = FlatBuffers(build_layout(spec), device.torch(), grad_alloc=grad_alloc)
        named = dict(self.named_parameters())
        for slot in flat.layout.slots:
            flat.load_from(slot.name, named[slot.name]._data.detach().float())
        for name, p in named.items():
            p._rebind(flat.param(name), requires_grad=False, dtype=DType.BF16)
            object.__setattr__(p, "_main_grad", flat.grad(name))
            object.__setattr__(p, "_master", flat.master_view(name))
            object.__setattr__(p, "_flat", flat)
        anchor = torch.zeros((), device=device.torch(), requires_grad=True)
        flat.rehome = self.rehome_buffers
        flat.owner = self
        object.__setattr__(self, "_flat", flat)
        object.__setattr__(self, "_anchor", anchor)
        object.__setattr__(self, "_engine", LMEngine(spec, flat))

    def rehome_buffers(self, *, params: torch.Tensor | None = None, grads: torch.Tensor | None = None) -> None:
        """Move the flat parameter and/or gradient storage into caller-provided
        1-D tensors (e.g. symmetric memory for the fused collectives) and
        rebind every parameter view and the engine to them."""
        from underhfs_b200.models.transformer import LMEngine

        flat = self._flat
        if flat is None:
            raise RuntimeError("rehome_buffers needs the CUDA engine (call .to('cuda', dtype='bf16') first)")
        if params is not None:
            params[: flat.numel].copy_(flat.params)
            flat.params = params[: flat.numel]
        if grads is not None:
            grads.zero_()
            grads[: flat.numel].copy_(flat.grads)
            flat.grads = grads[: flat.numel]
        for name, p in self.named_parameters():
            p._rebind(flat.param(name), requires_grad=False, dtype=DType.BF16)
            object.__setattr__(p, "_main_grad", flat.grad(name))
        old = self._engine
        engine = LMEngine(self.spec, flat)
        if old is not None:  # keep the hooks installed on the previous engine
            engine.grad_ready = old.grad_ready
            engine.context_attention = old.context_attention
            engine.positions = old.positions
        object.__setattr__(self, "_engine", engine)

    def attach_zero3(self, zero3) -> None:
        """Hand this model to a ZeRO-3 sharded runtime (parallel.zero3.Zero3LM,
        built by ``ZeroAwareAdamW(..., stage=3)``): forward / backward run on its
        engine, which gathers each unit's weights before use, and the full
        flat buffers are released, so the rank keeps only its shard.  The
        parameters become shape-only placeholders (meta tensors);
        ``state_dict()`` / ``load_state_dict()`` gather / scatter through the
        shards (collectives: call them on every rank)."""
        object.__setattr__(self, "_zero3", zero3)
        object.__setattr__(self, "_engine", zero3.engine)
        object.__setattr__(self, "_flat", None)
        for _, p in self.named_parameters():
            p._data = torch.empty(p.shape, dtype=torch.bfloat16, device="meta")
            for attr in ("_main_grad", "_master", "_flat"):
                if hasattr(p, attr):
                    object.__setattr__(p, attr, None)

    @property
    def zero3(self):
        return self._zero3

    def _engine_device(self) -> torch.device:
        return self._zero3.device if self._zero3 is not None else self._flat.device

    def state_dict(self, *, as_tensors: bool = False) -> dict[str, Any]:
        if self._zero3 is None:
            return super().state_dict(as_tensors=as_tensors)
        full = self._zero3.full_state()  # all-gather of every shard (fp32, CPU)
        return {name: (full[name].clone() if as_tensors else full[name].double().tolist())
                for name, _ in self.named_parameters()}

    def load_state_dict(self, state: dict[str, Any]) -> None:
        if self._zero3 is None:
            return super().load_state_dict(state)
        full = {}
        for name, p in self.named_parameters():
            if name not in state:
                raise KeyError(f"missing parameter {name}")
            value = state[name]._data if isinstance(state[name], Tensor) else state[name]
            full[name] = (value if isinstance(value, torch.Tensor) else torch.tensor(value)).reshape(p.shape)
        self._zero3.load_full_state(full)

    @property
    def engine(self):
        return self._engine

    @property
    def flat(self):
        return self._flat

    def zero_grad(self) -> None:
        if self._zero3 is not None:
            return  # ZeRO-3 clears each unit's gradient slot as its backward begins
        if self._flat is not None:
            self._flat.zero_grad()
        else:
            super().zero_grad()

    # -------------------------------------------------------- forward
    def forward(self, token_ids: Tensor | torch.Tensor, targets: Tensor | torch.Tensor | None = None) -> Tensor:
        ids = token_ids._data if isinstance(token_ids, Tensor) else token_ids
        if ids.dim() not in (1, 2):
            raise ValueError("TransformerLM expects token ids shaped [T] or [B, T]")
        T = ids.shape[-1]
        if T > self.max_seq_len:
            raise ValueError(f"sequence length {T} exceeds max_seq_len {self.max_seq_len}")
        if self._engine is not None:
            return self._engine_forward(ids, targets)
        batched = ids.dim() == 2
        ids2 = ids if batched else ids.unsqueeze(0)
        x = self.token_embedding(Tensor._wrap(ids2))
        pos = torch.arange(T, device=ids2.device)
        x = x + self.position_embedding(Tensor._wrap(pos))
        for block in self.blocks:
            x = block(x)
        h = self.norm(x)
        head_w = self.token_embedding.weight if self.tied else self.head.weight
        logits = _wrap(_linear_t(h._data, head_w._data, None), h, "linear", (h, head_w))
        if not batched:
            logits = _wrap(logits._data.squeeze(0), logits, "view", (logits,))
        if targets is None:
            return logits
        tg = targets._data if isinstance(targets, Tensor) else targets
        return F.cross_entropy(logits.reshape(-1, self.vocab_size), Tensor._wrap(tg.reshape(-1)))

    def _engine_forward(self, ids: torch.Tensor, targets) -> Tensor:
        dev = self._engine_device()
        batched = ids.dim() == 2
        ids2 = (ids if batched else ids.unsqueeze(0)).to(dev, torch.int64)
        like = self.token_embedding.weight
        if targets is not None:
            tg = targets._data if isinstance(targets, Tensor) else targets
            tg = tg.reshape(ids2.shape).to(dev, torch.int64)
            if torch.is_grad_enabled():
                loss = _EngineLoss.apply(self._anchor, self._engine, ids2, tg, True)
            else:
                loss, _ = self._engine.forward(ids2, tg, fuse_loss_grad=False)
            return Tensor._wrap(loss, dtype=DType.FP32, backend="native_cuda", op="cross_entropy", parents=(like,))
        if torch.is_grad_enabled():
            logits = _EngineLogits.apply(self._anchor, self._engine, ids2)
        else:
            _, logits = self._engine.forward(ids2, None, fuse_loss_grad=False, keep_logits=True)
            self._engine._saved = None
        logits = logits.view(ids2.shape[0], ids2.shape[1], self.vocab_size)
        if not batched:
            logits = logits[0]
        return Tensor._wrap(logits, like=like, backend="native_cuda", op="transformer_lm", parents=(like,))

    def generate(self, token_ids: Tensor, max_new_tokens: int) -> Tensor:
        """Greedy decoding; the context is the last max_seq_len tokens."""
        ids = token_ids._data if isinstance(token_ids, Tensor) else token_ids
        if ids.dim() != 1:
            raise ValueError("TransformerLM.generate expects 1D token ids")
        generated = [int(v) for v in ids.tolist()]
        with torch.no_grad():
            for _ in range(max_new_tokens):
                context = generated[-self.max_seq_len:]
                dev = (self._engine_device() if self._engine is not None
                       else self.token_embedding.weight._data.device)
                logits = self(torch.tensor(context, dtype=torch.int64, device=dev))
                generated.append(int(torch.argmax(logits._data[-1].float()).item()))
        return tensor(generated)


def _require_cuda(device: Device) -> None:
    from underhfs_b200.native import status

    st = status()
    if not st.cuda_enabled:
        raise RuntimeError(f"cannot move module to CUDA because the native core is unavailable: {st.reason}")


class Conv2d(Module):
    def __init__(
        self,
        in_channels: int,
        out_channels: int,
        kernel_size: int | tuple[int, int],
        stride: int | tuple[int, int] = 1,
        padding: int | tuple[int, int] = 0,
        bias: bool = True,
    ) -> None:
        super().__init__()
        self.in_channels = in_channels
        self.out_channels = out_channels
        self.kernel_size = _pair(kernel_size)
        self.stride = _pair(stride)
        self.padding = _pair(padding)
        fan_in = in_channels * self.kernel_size[0] * self.kernel_size[1]
        self.weight = Parameter(
            uniform((out_channels, in_channels, *self.kernel_size), (1.0 / max(1, fan_in)) ** 0.5)
        )
        self.bias = Parameter(zeros((out_channels,))) if bias else None

    def backend_status(self, x: Tensor | None = None) -> BackendStatus:
        if x is not None and x.device.kind == "cuda":
            ok = (
                x.dtype is DType.FP32
                and self.weight.dtype is DType.FP32
                and x.layout is Layout.DENSE
                and self.weight.device == x.device
            )
            if not ok:
                return BackendStatus("conv2d", "cudnn", False,
                                     "CUDA Conv2d requires fp32 dense input, weight, and bias on the same CUDA device")
            from underhfs_b200.native import status

            if status().cudnn_enabled:
                return BackendStatus("conv2d", "cudnn", True, "native sm_100a fp32 convolution kernels")
            return BackendStatus("conv2d", "cudnn", False,
                                 "CUDA fp32 Conv2d requires native core built with UNDERHFS_WITH_CUDNN=ON")
        return BackendStatus("conv2d", "python", True, "portable fallback convolution")

    def forward(self, x: Tensor) -> Tensor:
        st = self.backend_status(x)
        if x.device.kind == "cuda" and not st.available:
            raise RuntimeError(st.reason)
        if x.ndim != 4:
            raise ValueError("Conv2d expects input shape [batch, channels, height, width]")
        if x.shape[1] != self.in_channels:
            raise ValueError(f"expected {self.in_channels} channels, got {x.shape[1]}")
        kh, kw = self.kernel_size
        oh = (x.shape[2] + 2 * self.padding[0] - kh) // self.stride[0] + 1
        ow = (x.shape[3] + 2 * self.padding[1] - kw) // self.stride[1] + 1
        if oh <= 0 or ow <= 0:
            raise ValueError("kernel/stride/padding produce empty output")
        b = self.bias._data if self.bias is not None else None
        parents = (x, self.weight) + ((self.bias,) if self.bias is not None else ())
        if x.device.kind == "cuda":
            from underhfs_b200.ops import functions as OF

            y = OF.conv2d(x._data, self.weight._data, b, self.stride, self.padding)
            return _wrap(y, x, "conv2d", parents, backend="native_cudnn")
        y = torch.nn.functional.conv2d(x._data, self.weight._data, b, self.stride, self.padding)
        return _wrap(y, x, "conv2d", parents)


class PolicyValueHead(Module):
    def __init__(self, features: int, actions: int) -> None:
        super().__init__()
        self.policy = Linear(features, actions)
        self.value = Linear(features, 1)

    def forward(self, x: Tensor) -> tuple[Tensor, Tensor]:
        return self.policy(x), self.value(x)


class MSELoss(Module):
    def __init__(self, reduction: str = "mean") -> None:
        super().__init__()
        self.reduction = reduction

    def forward(self, input: Tensor, target: Tensor) -> Tensor:
        return F.mse_loss(input, target, self.reduction)


class CrossEntropyLoss(Module):
    def __init__(self, reduction: str = "mean") -> None:
        super().__init__()
        self.reduction = reduction

    def forward(self, logits: Tensor, target: Tensor) -> Tensor:
        return F.cross_entropy(logits, target, self.reduction)


def _pair(value: int | tuple[int, int]) -> tuple[int, int]:
    return value if isinstance(value, tuple) else (value, value)


__all__ = [
    "BackendStatus", "Parameter", "Module", "Linear", "ReLU", "GELU", "Sequential", "ModuleList", "LayerNorm",
    "RMSNorm", "Embedding", "MLP", "SelfAttention", "CausalSelfAttention", "TransformerBlock", "TransformerLM",
    "Conv2d", "PolicyValueHead", "MSELoss", "CrossEntropyLoss", "CUDA_TORCH_DTYPE", "torch_dtype_for",
]
