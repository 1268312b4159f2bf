"""Pipeline-stage modules of the BERT / ViT encoders and their embedding / head math.

One class, ``EncoderStage``, covers every stage the reference builds by hand
(BERT/models/bert_stages.py, normal_bert_stages.py, bert_stages_with_inverse.py,
Vit/models/vit_stages.py, normal_vit_stages.py): a stage owns

  * the embedding (first stage): BERT word+position+type+LN, or ViT patch+CLS+pos+LN;
  * ``num_blocks`` encoder blocks;
  * the head (last stage): decoupling, pooling, LayerNorm and Linear(., classes).

Submodule names follow the reference so ``state_dict`` keys match:

  kind        first stage          middle / last stage     single-stage (PP=1)
  reversible  rev.layers.{i}.F/G   mod.layers.{i}.F/G      body.layers.{i}.F/G
  standard    rev.{i}.F/G (BERT)   mod.{i}.F/G             body.{i}.F/G
              body.{i}.F/G (ViT)
  inverse     rev.{i}.F/G          mod.{i}.F/G             body.{i}.F/G

Pooling: reversible BERT averages over the sequence (bert_stages.py:440); standard BERT,
the inverse variant and every ViT use the CLS token.  Reversible decoupling is x2 + x1;
the inverse variant concatenates [x1, x2] and its head is LayerNorm(2H) -> Linear(2H, C).
"""
from __future__ import annotations

from types import SimpleNamespace
from typing import List, Optional

import torch
import torch.nn as nn
import torch.nn.functional as Fn

from revpp.config import GlobalConfig

from .modules import BertEmbeddings, EncoderBlock, ViTEmbeddings, init_weights
from .params import FlatParams


class _Layers(nn.Module):
    """Holds blocks under ``layers`` (reversible sequences in the reference)."""

    def __init__(self, blocks: List[EncoderBlock]):
        super().__init__()
        self.layers = nn.ModuleList(blocks)


class EncoderStage(nn.Module):
    def __init__(self, cfg: GlobalConfig, stage_index: int, num_stages: int, num_blocks: int, kind: str):
        super().__init__()
        assert kind in ("reversible", "standard", "inverse")
        self.cfg = cfg
        self.kind = kind
        self.stage_index = stage_index
        self.num_stages = num_stages
        self.is_first = stage_index == 0
        self.is_last = stage_index == num_stages - 1
        H = cfg.hidden_size
        if self.is_first:
            if cfg.model == "bert":
                self.embeddings = BertEmbeddings(cfg.vocab_size, H, cfg.max_position_embeddings, cfg.type_vocab_size)
            else:
                self.embeddings = ViTEmbeddings(cfg.img_size, cfg.patch_size, cfg.num_channels, H)
        blocks = [EncoderBlock(H, cfg.num_attention_heads, cfg.mlp_ratio) for _ in range(num_blocks)]
        single = self.is_first and self.is_last
        if kind == "reversible":
            name = "body" if single else ("rev" if self.is_first else "mod")
            setattr(self, name, _Layers(blocks))
            self._body_prefix = f"{name}.layers"
        else:
            # reference container names: full stages "body"; first stages "rev", except the
            # standard ViT first stage ("body", Vit/models/normal_vit_stages.py:105); others "mod"
            if single:
                name = "body"
            elif self.is_first:
                name = "body" if (kind == "standard" and cfg.model == "vit") else "rev"
            else:
                name = "mod"
            setattr(self, name, nn.ModuleList(blocks))
            self._body_prefix = name
        self.blocks: List[EncoderBlock] = blocks
        if self.is_last:
            width = 2 * H if kind == "inverse" else H
            self.norm = nn.LayerNorm(width)
            self.head = nn.Linear(width, cfg.num_classes)
        init_weights(self, conv_kaiming=(cfg.model == "vit"))

    @property
    def pool(self) -> str:
        if self.cfg.model == "bert" and self.kind == "reversible":
            return "mean"
        return "cls"

    def block_prefix(self, i: int) -> str:
        return f"{self._body_prefix}.{i}"


# ====================================================================== embedding / head math (PyTorch)
def _autocast(device_type, dtype):
    return torch.autocast(device_type=device_type, dtype=dtype, enabled=dtype != torch.float32)


class TorchEmbedHead:
    """Embedding and classifier-head math in PyTorch (CPU runs and oracle)."""

    def __init__(self, stage: EncoderStage, flat: FlatParams, dtype: torch.dtype):
        self.stage = stage
        self.flat = flat
        self.dtype = dtype

    # -------------------------------------------------------------- embeddings
    def _embed(self, inputs):
        st = self.stage
        emb = st.embeddings
        if st.cfg.model == "bert":
            ids, tt = inputs
            S = ids.shape[1]
            pos = torch.arange(S, device=ids.device)
            with _autocast(ids.device.type, self.dtype):
                e = (Fn.embedding(ids, emb.word_embeddings.weight, padding_idx=0)
                     + Fn.embedding(pos, emb.position_embeddings.weight)[None]
                     + Fn.embedding(tt, emb.token_type_embeddings.weight))
                return Fn.layer_norm(e.float(), (e.shape[-1],), emb.norm.weight, emb.norm.bias, emb.norm.eps).float()
        (img,) = inputs
        B = img.shape[0]
        with _autocast(img.device.type, self.dtype):
            x = Fn.conv2d(img, emb.proj.weight, emb.proj.bias, stride=emb.patch_size)
            x = x.flatten(2).transpose(1, 2)
            x = torch.cat((emb.cls_token.expand(B, -1, -1).to(torch.float32), x.to(torch.float32)), dim=1)
            x = x + emb.pos_embed
            return Fn.layer_norm(x, (x.shape[-1],), emb.norm.weight, emb.norm.bias, emb.norm.eps).float()

    def embed_fwd(self, inputs) -> torch.Tensor:
        with torch.no_grad():
            return self._embed(inputs).contiguous()

    def embed_bwd(self, inputs, dx: torch.Tensor, dx1: Optional[torch.Tensor] = None) -> None:
        if dx1 is not None:
            dx = dx + dx1  # the coupling duplicated the embedding into both streams
        params = list(self.stage.embeddings.parameters())
        with torch.enable_grad():
            x = self._embed(inputs)
            grads = torch.autograd.grad(x, params, grad_outputs=dx, allow_unused=True)
        for p, g in zip(params, grads):
            if g is not None:
                self.flat.grad_of(p).add_(g.float())

    # -------------------------------------------------------------- head
    def _head(self, x2, x1):
        st = self.stage
        if x1 is None:  # standard (non-reversible) stage: single stream
            z = x2
        elif st.kind == "inverse":
            z = torch.cat([x1, x2], dim=-1)
        else:
            z = x2 + x1
        pooled = z.mean(dim=1) if st.pool == "mean" else z[:, 0]
        with _autocast(z.device.type, self.dtype):
            h = Fn.layer_norm(pooled, (pooled.shape[-1],), st.norm.weight, st.norm.bias, st.norm.eps)
            return Fn.linear(h, st.head.weight, st.head.bias)

    def head_fwd_bwd(self, y2, y1, labels, grad_scale: float):
        """Loss (mean CE of this micro-batch), logits, and (dY2, dY1) of ``grad_scale * loss``."""
        st = self.stage
        params = list(st.norm.parameters()) + list(st.head.parameters())
        y2r = y2.detach().requires_grad_(True)
        y1r = y1.detach().requires_grad_(True) if y1 is not None else None
        leaves = [y2r] + ([y1r] if y1r is not None else [])
        with torch.enable_grad():
            logits = self._head(y2r, y1r)
            loss = Fn.cross_entropy(logits.float(), labels)
            grads = torch.autograd.grad(loss * grad_scale, leaves + params)
        for p, g in zip(params, grads[len(leaves):]):
            self.flat.grad_of(p).add_(g.float())
        dy2 = grads[0].float().contiguous()
        dy1 = grads[1].float().contiguous() if y1r is not None else None
        return loss.detach(), logits.detach().float(), dy2, dy1

    def head_eval(self, y2, y1, labels):
        with torch.no_grad():
            logits = self._head(y2, y1).float()
            loss = Fn.cross_entropy(logits, labels) if labels is not None else None
        return loss, logits


def make_embed_head(stage: EncoderStage, flat: FlatParams, dtype: torch.dtype, device: torch.device):
    if device.type == "cuda" and dtype == torch.bfloat16:
        from .embed_head_kernels import KernelEmbedHead

        return KernelEmbedHead(stage, flat, dtype)
    return TorchEmbedHead(stage, flat, dtype)


def build_stage_module(cfg: GlobalConfig, stage_index: int, num_stages: int, kind: str) -> EncoderStage:
    if cfg.num_hidden_layers % num_stages != 0:
        raise ValueError(f"num_hidden_layers {cfg.num_hidden_layers} must be divisible by the "
                         f"number of pipeline stages {num_stages}")
    return EncoderStage(cfg, stage_index, num_stages, cfg.num_hidden_layers // num_stages, kind)


def stage_kind(cfg: GlobalConfig) -> str:
    if cfg.reversible:
        return "inverse" if cfg.inverse else "reversible"
    return "standard"


__all__ = ["EncoderStage", "TorchEmbedHead", "make_embed_head", "build_stage_module", "stage_kind", "SimpleNamespace"]
