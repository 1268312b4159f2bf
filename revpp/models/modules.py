"""Parameter containers of the BERT / ViT encoders.

Module and parameter names follow the reference so that ``state_dict`` keys line up
(BERT/models/bert_blocks.py:9-145, Vit/models/vit_blocks.py:9-62):

    F.norm.{weight,bias}                 LayerNorm(H, eps=1e-6)
    F.attn.in_proj_{weight,bias}         packed QKV projection [3H, H]
    F.attn.out_proj.{weight,bias}        Linear(H, H)
    G.norm.{weight,bias}                 LayerNorm(H, eps=1e-5)
    G.mlp.0.{weight,bias}                Linear(H, 4H)
    G.mlp.2.{weight,bias}                Linear(4H, H)

These modules hold parameters only; the math lives in ``revpp.models.blockmath``
(one implementation on the sm_100a kernels, one in plain PyTorch for CPU runs and
as the numerical oracle).
"""
from __future__ import annotations

import math

import torch
import torch.nn as nn


class MultiheadAttentionParams(nn.Module):
    """Same parameters and initialisation as ``nn.MultiheadAttention`` (batch_first,
    bias=True): xavier-uniform packed in_proj, zero biases."""

    def __init__(self, dim: int, num_heads: int):
        super().__init__()
        self.embed_dim = dim
        self.num_heads = num_heads
        self.in_proj_weight = nn.Parameter(torch.empty(3 * dim, dim))
        self.in_proj_bias = nn.Parameter(torch.zeros(3 * dim))
        self.out_proj = nn.Linear(dim, dim)
        nn.init.xavier_uniform_(self.in_proj_weight)
        nn.init.zeros_(self.out_proj.bias)


class AttentionSubBlock(nn.Module):
    """F: LayerNorm(eps 1e-6) -> multi-head self-attention (no mask, no dropout)."""

    eps = 1e-6

    def __init__(self, dim: int, num_heads: int):
        super().__init__()
        self.norm = nn.LayerNorm(dim, eps=self.eps)
        self.attn = MultiheadAttentionParams(dim, num_heads)


class MLPSubblock(nn.Module):
    """G: LayerNorm(eps 1e-5) -> Linear(H, 4H) -> GELU(erf) -> Linear(4H, H)."""

    eps = 1e-5

    def __init__(self, dim: int, mlp_ratio: int = 4):
        super().__init__()
        self.norm = nn.LayerNorm(dim, eps=self.eps)
        self.mlp = nn.Sequential(nn.Linear(dim, dim * mlp_ratio), nn.GELU(), nn.Linear(dim * mlp_ratio, dim))


class EncoderBlock(nn.Module):
    """One encoder layer.  Reversible use: Y1 = X1 + F(X2), Y2 = X2 + G(Y1).
    Standard use: x = x + F(x); x = x + G(x)."""

    def __init__(self, dim: int, num_heads: int, mlp_ratio: int = 4):
        super().__init__()
        self.F = AttentionSubBlock(dim, num_heads)
        self.G = MLPSubblock(dim, mlp_ratio)


class BertEmbeddings(nn.Module):
    """word + position + token-type embeddings, then LayerNorm(eps 1e-5)
    (BERT/models/bert_blocks.py:9-31); the word table's padding row is 0."""

    eps = 1e-5

    def __init__(self, vocab_size: int, dim: int, max_positions: int, type_vocab_size: int):
        super().__init__()
        self.word_embeddings = nn.Embedding(vocab_size, dim, padding_idx=0)
        self.position_embeddings = nn.Embedding(max_positions, dim)
        self.token_type_embeddings = nn.Embedding(type_vocab_size, dim)
        self.norm = nn.LayerNorm(dim, eps=self.eps)


class ViTEmbeddings(nn.Module):
    """Conv2d(k = s = patch) patch projection, prepended CLS token, learned position
    embedding, LayerNorm(eps 1e-5) (Vit/models/vit_blocks.py:9-62)."""

    eps = 1e-5

    def __init__(self, img_size: int, patch_size: int, in_chans: int, dim: int):
        super().__init__()
        self.img_size = img_size
        self.patch_size = patch_size
        self.grid_size = img_size // patch_size
        self.num_patches = self.grid_size * self.grid_size
        self.proj = nn.Conv2d(in_chans, dim, kernel_size=patch_size, stride=patch_size)
        self.cls_token = nn.Parameter(torch.zeros(1, 1, dim))
        self.pos_embed = nn.Parameter(torch.zeros(1, self.num_patches + 1, dim))
        self.norm = nn.LayerNorm(dim, eps=self.eps)
        nn.init.trunc_normal_(self.pos_embed, std=0.02)
        nn.init.trunc_normal_(self.cls_token, std=0.02)


def init_weights(module: nn.Module, conv_kaiming: bool = False) -> None:
    """Reference initialisation (BERT/models/bert_stages.py:31-44, Vit/models/vit_stages.py:30-48):
    Linear / Embedding N(0, 0.02) with zero bias and zeroed padding row, LayerNorm 1/0,
    Conv2d kaiming-normal (fan_out) for ViT.  The packed attention in_proj is a bare
    Parameter and keeps its xavier init."""
    for m in module.modules():
        if isinstance(m, nn.Linear):
            nn.init.normal_(m.weight, mean=0.0, std=0.02)
            if m.bias is not None:
                nn.init.zeros_(m.bias)
        elif isinstance(m, nn.Embedding):
            nn.init.normal_(m.weight, mean=0.0, std=0.02)
            if m.padding_idx is not None:
                with torch.no_grad():
                    m.weight[m.padding_idx].zero_()
        elif isinstance(m, nn.LayerNorm):
            nn.init.ones_(m.weight)
            nn.init.zeros_(m.bias)
        elif isinstance(m, nn.Conv2d) and conv_kaiming:
            nn.init.kaiming_normal_(m.weight, mode="fan_out", nonlinearity="relu")
            if m.bias is not None:
                nn.init.zeros_(m.bias)


def param_count(module: nn.Module) -> int:
    return sum(p.numel() for p in module.parameters())


def gelu_erf(x: torch.Tensor) -> torch.Tensor:
    return 0.5 * x * (1.0 + torch.erf(x * (1.0 / math.sqrt(2.0))))
