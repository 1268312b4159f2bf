"""Pipeline stage runtimes: what a stage computes for one micro-batch forward / backward,
what it keeps in between, and what it sends.

* ``ReversibleStage`` - the reference's main path (BERT/pipelining/
  reversible_stage_with_pareprop.py:141-945).  Forward runs the blocks without keeping
  anything; the first stage keeps only the token ids (or images) of each in-flight
  micro-batch.  Backward receives (dY2, dY1, Y2, Y1) from the next stage - the gradients
  *and* that stage's reconstructed input ("racts") - reconstructs its own inputs while
  it back-propagates, and sends (dX2, dX1, X2, X1) upstream.  Activation memory is O(1)
  in pipeline depth and in blocks per stage.  ``pareprop`` selects the two-stream
  backward.
* ``StandardStage`` - keeps every block's intermediates per in-flight micro-batch
  (BERT/pipelining/stage.py), O(P * N).
* ``CheckpointStage`` - keeps only the stage input per in-flight micro-batch and re-runs
  the stage forward in backward (BERT/pipelining/stage_with_cp.py:730-817), O(P); the
  last stage keeps its intermediates as in the reference.
* ``InverseStage`` - "inverse" mode (BERT/pipelining/reversible_stage.py:944-1093):
  backward inverts the whole stage first, then re-runs its forward keeping every
  block's intermediates, then back-propagates; stage 0 recomputes from its cached
  inputs and receives no reconstructed activations.

The last stage computes the loss and its gradient right after its forward, scaled by
1 / num_microbatches (the reference divides the accumulated gradients by the number of
micro-batches before clipping, BERT/src/engine.py:56-67; folding the factor into the
loss gradient gives the same update).
"""
from __future__ import annotations

from types import SimpleNamespace
from typing import Dict, List, Optional, Tuple

import torch

from revpp.models.blockmath import (KernelMath, rev_block_forward, rev_block_grads, std_block_backward,
                                    std_block_forward)
from revpp.models.encoder import EncoderStage
from revpp.models.reversible import inverse_sequence, rev_backward, rev_forward

from .p2p import TensorSpec


class StageBase:
    kind = "base"

    def __init__(self, module: EncoderStage, math_, embed_head, microbatch_size: int, num_microbatches: int,
                 device: torch.device, pareprop: bool = False, eval_actv_err: bool = False):
        self.module = module
        self.math = math_
        self.eh = embed_head
        self.cfg = module.cfg
        self.mbs = microbatch_size
        self.n_mb = num_microbatches
        self.device = device
        self.is_first = module.is_first
        self.is_last = module.is_last
        self.stage_index = module.stage_index
        self.num_stages = module.num_stages
        self.blocks = module.blocks
        self.pareprop = pareprop
        self.streams = None
        if pareprop and device.type == "cuda":
            self.streams = (torch.cuda.Stream(device=device), torch.cuda.Stream(device=device))
        self.input_cache: Dict[int, tuple] = {}
        self.labels: Optional[List[torch.Tensor]] = None
        self.losses: List[torch.Tensor] = []
        self.logits: List[torch.Tensor] = []
        self.eval_actv_err = eval_actv_err
        self.actv_records: List[dict] = []
        self.grad_scale = 1.0 / num_microbatches

    # message layouts
    @property
    def act_shape(self):
        return (self.mbs, self.cfg.seq_len, self.cfg.hidden_size)

    def fwd_specs(self) -> List[TensorSpec]:
        raise NotImplementedError

    def bwd_specs(self, receiver_stage: int) -> List[TensorSpec]:
        raise NotImplementedError

    def clear(self) -> None:
        self.input_cache.clear()
        self.losses = []
        self.logits = []

    # embedding / head helpers
    def _embed(self, mb: int, inputs):
        self.input_cache[mb] = inputs
        return self.eh.embed_fwd(inputs)

    def _head(self, mb: int, y2, y1, train: bool):
        labels = self.labels[mb] if self.labels is not None else None
        if train:
            loss, logits, dy2, dy1 = self.eh.head_fwd_bwd(y2, y1, labels, self.grad_scale)
            self.losses.append(loss)
            self.logits.append(logits)
            return dy2, dy1
        loss, logits = self.eh.head_eval(y2, y1, labels)
        if loss is not None:
            self.losses.append(loss)
        self.logits.append(logits)
        return None

    def forward(self, mb: int, inputs, train: bool = True):
        raise NotImplementedError

    def backward(self, mb: int, msg):
        raise NotImplementedError


class ReversibleStage(StageBase):
    kind = "reversible"

    def __init__(self, *a, **kw):
        super().__init__(*a, **kw)
        self.last_cache: Dict[int, tuple] = {}
        self.fwd_input_copy: Dict[int, tuple] = {}

    def fwd_specs(self):
        return [TensorSpec(self.act_shape, torch.float32)] * 2

    def bwd_specs(self, receiver_stage: int):
        return [TensorSpec(self.act_shape, torch.float32)] * 4

    def forward(self, mb, inputs, train=True):
        if self.is_first:
            x = self._embed(mb, inputs)
            x2, x1 = x, x  # coupling duplicates the embedding (bert_stages.py:18-21)
        else:
            x2, x1 = inputs
            if self.eval_actv_err and train:
                self.fwd_input_copy[mb] = (x2.clone(), x1.clone())
        y2, y1 = rev_forward(self.math, self.blocks, x2, x1)
        if self.is_last:
            dy = self._head(mb, y2, y1, train)
            if train:
                self.last_cache[mb] = (y2, y1, dy[0], dy[1])
            return None
        return (y2, y1)

    def backward(self, mb, msg, on_input=None):
        """``on_input(x2, x1)``: called as soon as the stage input is reconstructed (before the
        first block's gradients), so the executor can send the racts while they run."""
        if self.is_last:
            y2, y1, dy2, dy1 = self.last_cache.pop(mb)
        else:
            dy2, dy1, y2, y1 = msg
        hook = None
        if on_input is not None:
            def hook(i, x2_, x1_):
                if i == 0:
                    on_input(x2_, x1_)
        (dx2, dx1), (x2, x1) = rev_backward(self.math, self.blocks, y2, y1, dy2, dy1, pareprop=self.pareprop,
                                            streams=self.streams, on_recover=hook)
        if self.eval_actv_err and mb in self.fwd_input_copy:
            self._record_actv_err(mb, (x2, x1), self.fwd_input_copy.pop(mb))
        if self.is_first:
            inputs = self.input_cache.pop(mb)
            self.eh.embed_bwd(inputs, dx2, dx1)
            return None
        return (dx2, dx1, x2, x1)

    def _record_actv_err(self, mb, rec, ref):
        """Per-sample MSE and cosine of the reconstructed stage input against the input seen in
        forward, in fp64 (reversible_stage_with_pareprop.py:535-560)."""
        for which, (r, t) in enumerate(zip(rec, ref)):
            rr = r.double().reshape(r.shape[0], -1)
            tt = t.double().reshape(t.shape[0], -1)
            mse = ((rr - tt) ** 2).mean(dim=1)
            cos = torch.nn.functional.cosine_similarity(rr, tt, dim=1, eps=1e-15)
            for i in range(rr.shape[0]):
                self.actv_records.append(dict(stage=self.stage_index, mb=mb, sample=i, tensor=f"X{2 - which}",
                                              mse=float(mse[i]), cos=float(cos[i])))


class StandardStage(StageBase):
    kind = "standard"

    def __init__(self, *a, **kw):
        super().__init__(*a, **kw)
        self.ctx_cache: Dict[int, list] = {}

    def fwd_specs(self):
        return [TensorSpec(self.act_shape, torch.float32)]

    def bwd_specs(self, receiver_stage: int):
        return [TensorSpec(self.act_shape, torch.float32)]

    def _run(self, x, save: bool):
        ctxs = []
        with torch.no_grad():
            for blk in self.blocks:
                x, c = std_block_forward(self.math, blk, x, save)
                ctxs.append(c)
        return x, ctxs

    def forward(self, mb, inputs, train=True):
        # the received buffer belongs to a receive ring; keep a copy when it must outlive this call
        x = self._embed(mb, inputs) if self.is_first else (inputs[0].clone() if train else inputs[0])
        y, ctxs = self._run(x, save=train)
        if train:
            self.ctx_cache[mb] = ctxs
        if self.is_last:
            dy = self._head(mb, y, None, train)
            if train:
                self.ctx_cache[mb] = (ctxs, dy[0])
            return None
        return (y,)

    def _backprop(self, ctxs, dy):
        with torch.no_grad():
            for blk, c in zip(reversed(self.blocks), reversed(ctxs)):
                dy = std_block_backward(self.math, blk, c, dy)
        return dy

    def backward(self, mb, msg):
        if self.is_last:
            ctxs, dy = self.ctx_cache.pop(mb)
        else:
            ctxs = self.ctx_cache.pop(mb)
            dy = msg[0]
        dx = self._backprop(ctxs, dy)
        if self.is_first:
            self.eh.embed_bwd(self.input_cache.pop(mb), dx)
            return None
        return (dx,)


class CheckpointStage(StandardStage):
    kind = "checkpoint"

    def forward(self, mb, inputs, train=True):
        if self.is_last:
            return super().forward(mb, inputs, train)
        x = self._embed(mb, inputs) if self.is_first else inputs[0]
        if train and not self.is_first:
            self.input_cache[mb] = (x.clone(),)  # the receive ring reuses its buffers
        y, _ = self._run(x, save=False)
        return (y,)

    def backward(self, mb, msg):
        if self.is_last:
            return super().backward(mb, msg)
        if self.is_first:
            inputs = self.input_cache.pop(mb)
            x = self.eh.embed_fwd(inputs)
        else:
            (x,) = self.input_cache.pop(mb)
        _, ctxs = self._run(x, save=True)
        dx = self._backprop(ctxs, msg[0])
        if self.is_first:
            self.eh.embed_bwd(inputs, dx)
            return None
        return (dx,)


class InverseStage(StageBase):
    kind = "inverse"

    def __init__(self, *a, **kw):
        super().__init__(*a, **kw)
        self.last_cache: Dict[int, tuple] = {}
        self.fwd_input_copy: Dict[int, tuple] = {}

    def fwd_specs(self):
        return [TensorSpec(self.act_shape, torch.float32)] * 2

    def bwd_specs(self, receiver_stage: int):
        n = 2 if receiver_stage == 0 else 4
        return [TensorSpec(self.act_shape, torch.float32)] * n

    def forward(self, mb, inputs, train=True):
        if self.is_first:
            x = self._embed(mb, inputs)
            x2, x1 = x, x
        else:
            x2, x1 = inputs
            if self.eval_actv_err and train:
                self.fwd_input_copy[mb] = (x2.clone(), x1.clone())
        y2, y1 = rev_forward(self.math, self.blocks, x2, x1)
        if self.is_last:
            dy = self._head(mb, y2, y1, train)
            if train:
                self.last_cache[mb] = (y2, y1, dy[0], dy[1])
            return None
        return (y2, y1)

    def backward(self, mb, msg):
        inputs = None
        if self.is_last:
            y2, y1, dy2, dy1 = self.last_cache.pop(mb)
            if self.is_first:  # single stage: recompute from the cached inputs
                inputs = self.input_cache.pop(mb)
                x = self.eh.embed_fwd(inputs)
                x2, x1 = x, x
            else:
                x2, x1 = inverse_sequence(self.math, self.blocks, y2, y1)
        elif self.is_first:
            dy2, dy1 = msg[0], msg[1]
            inputs = self.input_cache.pop(mb)
            x = self.eh.embed_fwd(inputs)
            x2, x1 = x, x
        else:
            dy2, dy1, y2, y1 = msg
            x2, x1 = inverse_sequence(self.math, self.blocks, y2, y1)
        if self.eval_actv_err and mb in self.fwd_input_copy:
            ReversibleStage._record_actv_err(self, mb, (x2, x1), self.fwd_input_copy.pop(mb))
        # re-run the stage forward keeping every block's intermediates, then back-propagate
        rcs = []
        with torch.no_grad():
            a2, a1 = x2, x1
            for blk in self.blocks:
                y1_, cf = self.math.f_fwd(blk, a2, a1, 1.0, save=True)
                y2_, cg = self.math.g_fwd(blk, y1_, a2, 1.0, save=True)
                rcs.append(SimpleNamespace(x2=a2, x1=a1, ctx_f=cf, ctx_g=cg))
                a2, a1 = y2_, y1_
            dy = (dy2, dy1)
            for blk, rc in zip(reversed(self.blocks), reversed(rcs)):
                dx2_, dx1_, _ = rev_block_grads(self.math, blk, rc, *dy)
                dy = (dx2_, dx1_)
        dx2, dx1 = dy
        if self.is_first:
            self.eh.embed_bwd(inputs, dx2, dx1)
            return None
        if self.stage_index == 1:
            return (dx2, dx1)
        return (dx2, dx1, x2, x1)


STAGE_TYPES = {"reversible": ReversibleStage, "standard": StandardStage, "checkpoint": CheckpointStage,
               "inverse": InverseStage}
