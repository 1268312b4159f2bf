"""Pipeline split of an arbitrary ``nn.Module`` by tracing (the reference's tracer frontend,
BERT/pipelining/_IR.py: ``pipe_split``, ``SplitPoint``, ``pipeline``, ``Pipe``,
``Pipe.build_stage``; exported there but unused by its CLI, whose stages are built by hand).

The module is traced with torch.fx.  Split points come from ``x = pipe_split(x)`` calls
inside its ``forward`` (on the tensor that crosses the boundary) or from ``split_spec`` (submodule name -> ``SplitPoint.BEGINNING`` /
``SplitPoint.END``); the graph is cut there into ``submod_0 .. submod_{n-1}``, one per
pipeline stage, each taking the previous stage's output (one tensor between stages).
``Pipe.build_stage(i, ...)`` returns a stage runtime for ``PipelineExecutor``: forward keeps
the submodule's autograd graph per in-flight micro-batch, backward runs autograd with the
received gradient and accumulates the parameter gradients, like the reference's generic
``PipelineStage`` (BERT/pipelining/stage.py).  This path serves arbitrary models; the BERT /
ViT encoders use the hand-built stages with the sm_100a kernels.
"""
from __future__ import annotations

import contextlib
import enum
from typing import Callable, Dict, List, Optional, Sequence

import torch
import torch.fx as fx
import torch.nn as nn
from torch.fx.passes.split_module import split_module

from .p2p import TensorSpec


class SplitPoint(enum.Enum):
    BEGINNING = 1
    END = 2


def pipe_split(x=None):
    """Marks a stage boundary inside ``forward``: ``x = pipe_split(x)`` on the tensor that
    crosses it.  The identity when the module runs eagerly; recorded while ``pipeline``
    traces."""
    return x


_PIPE_SPLIT = pipe_split


def _tracing_pipe_split(x=None):
    if isinstance(x, fx.Proxy):
        return x.tracer.create_proxy("call_function", _PIPE_SPLIT, (x,), {})
    raise RuntimeError("pipe_split(x) must be given the tensor that crosses the stage boundary")


@contextlib.contextmanager
def _markers_traced(module: nn.Module):
    """Point every ``pipe_split`` name visible to the module's forward methods (and this
    file's wrappers) at the tracing version while tracing."""
    real = _PIPE_SPLIT  # this file's own global is patched too: compare with a fixed reference
    spaces, seen = [globals()], set()
    for m in module.modules():
        g = getattr(type(m).forward, "__globals__", None)
        if g is not None and id(g) not in seen:
            seen.add(id(g))
            spaces.append(g)
    patched = []
    for g in spaces:
        for name, v in list(g.items()):
            if v is real:
                g[name] = _tracing_pipe_split
                patched.append((g, name))
    try:
        yield
    finally:
        for g, name in patched:
            g[name] = real


def annotate_split_points(module: nn.Module, spec: Dict[str, SplitPoint]) -> None:
    """Record split points on named submodules: the stage boundary falls before
    (BEGINNING) or after (END) the submodule's call."""
    for name in spec:
        module.get_submodule(name)  # must exist
    prev = getattr(module, "_revpp_split_spec", {})
    module._revpp_split_spec = {**prev, **spec}


class _LeafTracer(fx.Tracer):
    """Keeps the submodules that carry a split point as single calls (leaves)."""

    def __init__(self, leaves):
        super().__init__()
        self.leaves = set(leaves)

    def is_leaf_module(self, m: nn.Module, qualname: str) -> bool:
        return qualname in self.leaves or super().is_leaf_module(m, qualname)


class Pipe(nn.Module):
    """The split module: ``split_gm`` runs the stages in order; ``stages[i]`` is stage i."""

    def __init__(self, split_gm: fx.GraphModule, num_stages: int):
        super().__init__()
        self.split_gm = split_gm
        self.num_stages = num_stages

    def forward(self, *args, **kwargs):
        return self.split_gm(*args, **kwargs)

    def get_stage_module(self, i: int) -> nn.Module:
        if not 0 <= i < self.num_stages:
            raise IndexError(f"stage {i} of {self.num_stages}")
        return getattr(self.split_gm, f"submod_{i}")

    @property
    def stages(self) -> List[nn.Module]:
        return [self.get_stage_module(i) for i in range(self.num_stages)]

    def build_stage(self, stage_index: int, device: torch.device, microbatch_size: int, num_microbatches: int,
                    in_spec: Optional[TensorSpec] = None, out_spec: Optional[TensorSpec] = None,
                    loss_fn: Optional[Callable] = None) -> "TracedStage":
        mod = self.get_stage_module(stage_index).to(device)
        return TracedStage(mod, stage_index, self.num_stages, device, num_microbatches, in_spec, out_spec,
                           loss_fn or nn.functional.cross_entropy)


def pipeline(module: nn.Module, mb_args: Sequence = (), mb_kwargs: Optional[dict] = None,
             split_spec: Optional[Dict[str, SplitPoint]] = None,
             split_policy: Optional[Callable[[fx.GraphModule], fx.GraphModule]] = None) -> Pipe:
    """Trace ``module`` and cut it into pipeline stages at its split points.  ``mb_args`` are
    accepted for the reference's signature (torch.fx tracing is symbolic and needs none);
    ``split_policy`` may rewrite the traced graph (e.g. insert ``pipe_split`` calls)."""
    if split_spec is not None and split_policy is not None:
        raise ValueError("give split_spec or split_policy, not both")
    if split_spec:
        annotate_split_points(module, split_spec)
    spec = dict(getattr(module, "_revpp_split_spec", {}))
    with _markers_traced(module):
        graph = _LeafTracer(spec).trace(module)
    gm = fx.GraphModule(module, graph)
    if split_policy is not None:
        gm = split_policy(gm)
    # partition index of every node = number of boundaries before it (pipe_split markers,
    # and the calls of submodules with a split point)
    part, cur = {}, 0
    markers = []
    for node in gm.graph.nodes:
        if node.op == "call_function" and node.target in (_PIPE_SPLIT, _tracing_pipe_split):
            cur += 1
            markers.append(node)
            continue
        point = spec.get(node.target) if node.op == "call_module" else None
        if point == SplitPoint.BEGINNING:
            cur += 1
        part[node.name] = cur
        if point == SplitPoint.END:
            cur += 1
    for m in markers:
        m.replace_all_uses_with(m.args[0])
        gm.graph.erase_node(m)
    gm.recompile()
    n = cur + 1
    split = split_module(gm, module, lambda node: part[node.name])
    got = sum(1 for name, _ in split.named_children() if name.startswith("submod_"))
    if got != n:
        raise RuntimeError(f"expected {n} stages from {cur} split points, got {got} (empty stage?)")
    return Pipe(split, n)


class TracedStage:
    """Stage runtime of a traced submodule for ``PipelineExecutor`` (one tensor per message).
    Forward keeps the autograd graph of every in-flight micro-batch; the last stage computes
    ``loss_fn(output, labels) / num_microbatches`` and its gradient right away."""

    kind = "traced"

    def __init__(self, module: nn.Module, stage_index: int, num_stages: int, device, num_microbatches: int,
                 in_spec: Optional[TensorSpec], out_spec: Optional[TensorSpec], loss_fn: Callable):
        self.module = module
        self.stage_index = stage_index
        self.num_stages = num_stages
        self.is_first = stage_index == 0
        self.is_last = stage_index == num_stages - 1
        self.device = device
        self.n_mb = num_microbatches
        self.in_spec, self.out_spec = in_spec, out_spec
        self.loss_fn = loss_fn
        self.labels = None
        self.losses: list = []
        self.logits: list = []
        self._cache: dict = {}

    def fwd_specs(self):
        return [self.out_spec]

    def bwd_specs(self, receiver_stage: int):
        return [self.in_spec]

    def clear(self) -> None:
        self._cache.clear()
        self.losses, self.logits = [], []

    def forward(self, mb: int, inputs, train: bool = True):
        x = inputs[0] if isinstance(inputs, (tuple, list)) else inputs
        if not self.is_first:
            x = x.detach().clone().requires_grad_(train)
        with torch.set_grad_enabled(train):
            y = self.module(x)
        if self.is_last:
            if self.labels is not None:
                loss = self.loss_fn(y, self.labels[mb])
                self.losses.append(loss.detach())
                if train:
                    self._cache[mb] = (x, loss / self.n_mb, None)
            self.logits.append(y.detach())
            return None
        if train:
            self._cache[mb] = (x, y, None)
        return (y.detach().contiguous(),)

    def backward(self, mb: int, msg):
        x, y, _ = self._cache.pop(mb)
        if self.is_last:
            y.backward()
        else:
            y.backward(msg[0])
        if self.is_first:
            return None
        return (x.grad.contiguous(),)


__all__ = ["SplitPoint", "pipe_split", "annotate_split_points", "pipeline", "Pipe", "TracedStage"]
