"""Embedding and classifier-head math on the sm_100a kernels (bf16 runs on CUDA).

Same interface and numerics as ``TorchEmbedHead``: BERT embeddings (gather + sum +
LayerNorm, fp32 out) and their backward (recompute + LayerNorm backward + scatter into
the tables), the ViT patch embedding as im2col + tcgen05 GEMM + CLS/position/LayerNorm
assembly, and the head (decouple, pool, LayerNorm, bf16 Linear, cross-entropy) with its
backward in one pass per micro-batch.
"""
from __future__ import annotations

import torch

from revpp import ops

from .encoder import EncoderStage
from .params import FlatParams


class KernelEmbedHead:
    def __init__(self, stage: EncoderStage, flat: FlatParams, dtype: torch.dtype):
        self.stage = stage
        self.flat = flat
        self.dtype = dtype
        self.C = ops.ext()
        self._cache = {}

    # -------------------------------------------------------------- embeddings
    def embed_fwd(self, inputs) -> torch.Tensor:
        st = self.stage
        emb = st.embeddings
        H = st.cfg.hidden_size
        if st.cfg.model == "bert":
            ids, tt = inputs
            B, S = ids.shape
            out = torch.empty(B, S, H, dtype=torch.float32, device=ids.device)
            self.C.bert_embed_fwd(ids.contiguous(), tt.contiguous(), emb.word_embeddings.weight,
                                  emb.position_embeddings.weight, emb.token_type_embeddings.weight, emb.norm.weight,
                                  emb.norm.bias, emb.norm.eps, out)
            return out
        (img,) = inputs
        conv, B, S = self._patch_conv(img)
        out = torch.empty(B, S, H, dtype=torch.float32, device=img.device)
        self.C.vit_assemble_fwd(conv, emb.cls_token.view(-1), emb.pos_embed.view(-1), emb.norm.weight, emb.norm.bias,
                                emb.norm.eps, B, S, out)
        return out

    def _patch_conv(self, img):
        st = self.stage
        emb = st.embeddings
        H = st.cfg.hidden_size
        img = img.contiguous().float()
        B = img.shape[0]
        p = emb.patch_size
        np_ = emb.num_patches
        K = img.shape[1] * p * p
        patches = torch.empty(B * np_, K, dtype=torch.bfloat16, device=img.device)
        self.C.im2col_patches(img, p, patches)
        conv = torch.empty(B * np_, H, dtype=torch.bfloat16, device=img.device)
        w = self.flat.shadow_of(emb.proj.weight).view(H, K)
        ops.linear(patches, w, conv, bias=self.flat.shadow_of(emb.proj.bias))
        self._cache["patches"] = patches
        return conv, B, np_ + 1

    def embed_bwd(self, inputs, dx: torch.Tensor, dx1: torch.Tensor | None = None) -> None:
        st = self.stage
        emb = st.embeddings
        g = self.flat.grad_of
        H = st.cfg.hidden_size
        if st.cfg.model == "bert":
            ids, tt = inputs
            self.C.bert_embed_bwd(ids.contiguous(), tt.contiguous(), emb.word_embeddings.weight,
                                  emb.position_embeddings.weight, emb.token_type_embeddings.weight, emb.norm.weight,
                                  emb.norm.eps, dx.contiguous(), dx1, g(emb.word_embeddings.weight),
                                  g(emb.position_embeddings.weight), g(emb.token_type_embeddings.weight),
                                  g(emb.norm.weight), g(emb.norm.bias))
            return
        (img,) = inputs
        conv, B, S = self._patch_conv(img)
        patches = self._cache.pop("patches")
        dconv = torch.empty_like(conv)
        self.C.vit_assemble_bwd(conv, emb.cls_token.view(-1), emb.pos_embed.view(-1), emb.norm.weight, emb.norm.eps,
                                B, S, dx.contiguous(), dx1, dconv, g(emb.cls_token).view(-1),
                                g(emb.pos_embed).view(-1), g(emb.norm.weight), g(emb.norm.bias))
        K = patches.shape[1]
        ops.cast_colsum(dconv, colsum=g(emb.proj.bias))
        ops.linear_wgrad(dconv, patches, g(emb.proj.weight).view(H, K))

    # -------------------------------------------------------------- head
    def _mode(self, y1):
        st = self.stage
        if y1 is None:
            return 1
        if st.kind == "inverse":
            return 2
        return 0 if st.pool == "mean" else 1

    def _run_head(self, y2, y1, labels, grad_scale: float, want_grad: bool):
        st = self.stage
        B, S, H = y2.shape
        mode = self._mode(y1)
        W = 2 * H if mode == 2 else H
        Cn = st.cfg.num_classes
        dev = y2.device
        f = self.flat
        pooled = torch.empty(B, W, dtype=torch.float32, device=dev)
        logits = torch.empty(B, Cn, dtype=torch.float32, device=dev)
        loss = torch.empty(B, dtype=torch.float32, device=dev)
        kw = {}
        dy2 = dy1 = None
        if want_grad:
            dy2 = torch.empty_like(y2)
            dy1 = torch.empty_like(y2) if mode == 2 else None
            kw = dict(dlogits=torch.empty(B, Cn, dtype=torch.float32, device=dev),
                      hb=torch.empty(B, W, dtype=torch.bfloat16, device=dev),
                      dpooled=torch.empty(B, W, dtype=torch.float32, device=dev), dW=f.grad_of(st.head.weight),
                      db=f.grad_of(st.head.bias), dgamma=f.grad_of(st.norm.weight), dbeta=f.grad_of(st.norm.bias),
                      dy2=dy2, dy1=dy1)
        self.C.head_fwd_bwd(y2.contiguous(), None if y1 is None else y1.contiguous(), mode, st.norm.weight,
                            st.norm.bias, st.norm.eps, f.shadow_of(st.head.weight), f.shadow_of(st.head.bias),
                            labels, grad_scale, pooled, logits, loss, want_grad, **kw)
        if want_grad and dy1 is None and y1 is not None:
            dy1 = dy2  # sum decoupling: both streams get the same gradient
        return loss.mean(), logits, dy2, dy1

    def head_fwd_bwd(self, y2, y1, labels, grad_scale: float):
        return self._run_head(y2, y1, labels, grad_scale, True)

    def head_eval(self, y2, y1, labels):
        loss, logits, _, _ = self._run_head(y2, y1, labels, 0.0, False)
        return (loss if labels is not None else None), logits
