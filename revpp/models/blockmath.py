"""Math of the encoder sub-blocks F (attention) and G (MLP), forward and VJP.

Two implementations share one interface:

* ``KernelMath`` - the sm_100a path (bf16 compute, fp32 residual stream).  Every op is
  a kernel of ``revpp._C``: LayerNorm -> tcgen05 GEMM (bias, GELU, residual add/sub
  fused in the epilogue) -> flash attention; the VJPs use the input-gradient GEMM with
  the GELU derivative fused, weight-gradient GEMMs that accumulate fp32 gradients in
  place, and a LayerNorm backward that also adds the residual gradient and emits the
  bf16 operand of the next GEMM.
* ``TorchMath`` - the same math in plain PyTorch under autocast.  It runs the CPU
  tests, the fp32 / fp16 modes, and is the numerical oracle of the kernels.

Interface (activations are contiguous [B, S, H] tensors; the residual stream is fp32):

    out, ctx = f_fwd(blk, x, resid, sign, save)     out = resid + sign * F(x)
    out, ctx = g_fwd(blk, x, resid, sign, save)     out = resid + sign * G(x)
    dx       = f_vjp(blk, ctx, dy, resid_grad)      dx  = resid_grad + (dF/dx)^T dy
    dx       = g_vjp(blk, ctx, dy, resid_grad)      dx  = resid_grad + (dG/dx)^T dy

Parameter gradients are accumulated into the stage's flat fp32 gradient buffer.  The
numerics follow the reference under autocast (BERT/models/bert_blocks.py:34-63): LN in
fp32, GEMMs in bf16, F/G outputs rounded to bf16 before the fp32 residual add.
"""
from __future__ import annotations

import math
import os
from types import SimpleNamespace
from typing import List, Optional

import torch
import torch.nn.functional as Fn

from .modules import AttentionSubBlock, EncoderBlock, MLPSubblock
from .params import FlatParams


def _autocast(device_type: str, dtype: torch.dtype):
    return torch.autocast(device_type=device_type, dtype=dtype, enabled=dtype != torch.float32)


# ====================================================================== PyTorch
class TorchMath:
    """PyTorch implementation of F, G and their VJPs (autocast semantics)."""

    name = "torch"

    def __init__(self, flat: FlatParams, dtype: torch.dtype, heads: int):
        self.flat = flat
        self.dtype = dtype
        self.heads = heads

    # -------------------------------------------------------------- raw F / G
    def attn(self, F: AttentionSubBlock, x: torch.Tensor) -> torch.Tensor:
        B, S, H = x.shape
        h = self.heads
        d = H // h
        with _autocast(x.device.type, self.dtype):
            y = Fn.layer_norm(x, (H,), F.norm.weight, F.norm.bias, F.norm.eps)
            qkv = Fn.linear(y, F.attn.in_proj_weight, F.attn.in_proj_bias)
            q, k, v = qkv.view(B, S, 3, h, d).permute(2, 0, 3, 1, 4)
            s = torch.matmul(q * (1.0 / math.sqrt(d)), k.transpose(-1, -2))
            p = torch.softmax(s.float(), dim=-1).to(v.dtype)
            o = torch.matmul(p, v).transpose(1, 2).reshape(B, S, H)
            return Fn.linear(o, F.attn.out_proj.weight, F.attn.out_proj.bias)

    def mlp(self, G: MLPSubblock, x: torch.Tensor) -> torch.Tensor:
        H = x.shape[-1]
        with _autocast(x.device.type, self.dtype):
            y = Fn.layer_norm(x, (H,), G.norm.weight, G.norm.bias, G.norm.eps)
            u = Fn.linear(y, G.mlp[0].weight, G.mlp[0].bias)
            return Fn.linear(Fn.gelu(u), G.mlp[2].weight, G.mlp[2].bias)

    # -------------------------------------------------------------- interface
    def f_fwd(self, blk: EncoderBlock, x, resid, sign: float, save: bool):
        with torch.no_grad():
            f = self.attn(blk.F, x)
            out = resid + sign * f.float() if sign != 1.0 else resid + f.float()
        return out, (SimpleNamespace(x=x) if save else None)

    def g_fwd(self, blk: EncoderBlock, x, resid, sign: float, save: bool):
        with torch.no_grad():
            g = self.mlp(blk.G, x)
            out = resid + sign * g.float() if sign != 1.0 else resid + g.float()
        return out, (SimpleNamespace(x=x) if save else None)

    def _vjp(self, fn, module, ctx, dy, resid_grad):
        params = [p for p in module.parameters()]
        x = ctx.x.detach().requires_grad_(True)
        with torch.enable_grad():
            out = fn(module, x)
            grads = torch.autograd.grad(out, [x] + params, grad_outputs=dy.to(out.dtype))
        for p, g in zip(params, grads[1:]):
            self.flat.grad_of(p).add_(g.to(torch.float32))
        dx = grads[0].to(torch.float32)
        return dx + resid_grad if resid_grad is not None else dx

    def f_vjp(self, blk: EncoderBlock, ctx, dy, resid_grad):
        return self._vjp(self.attn, blk.F, ctx, dy, resid_grad)

    def g_vjp(self, blk: EncoderBlock, ctx, dy, resid_grad):
        return self._vjp(self.mlp, blk.G, ctx, dy, resid_grad)


# ====================================================================== kernels
class _WeightViews:
    """bf16 shadows (GEMM operands) and fp32 grad views of one encoder block."""

    def __init__(self, flat: FlatParams, blk: EncoderBlock):
        F, G = blk.F, blk.G
        s, g = flat.shadow_of, flat.grad_of
        self.ln1_w, self.ln1_b = F.norm.weight, F.norm.bias
        self.ln2_w, self.ln2_b = G.norm.weight, G.norm.bias
        self.wqkv, self.bqkv = s(F.attn.in_proj_weight), s(F.attn.in_proj_bias)
        self.wo, self.bo = s(F.attn.out_proj.weight), s(F.attn.out_proj.bias)
        self.w1, self.b1 = s(G.mlp[0].weight), s(G.mlp[0].bias)
        self.w2, self.b2 = s(G.mlp[2].weight), s(G.mlp[2].bias)
        self.d_ln1_w, self.d_ln1_b = g(F.norm.weight), g(F.norm.bias)
        self.d_ln2_w, self.d_ln2_b = g(G.norm.weight), g(G.norm.bias)
        self.d_wqkv, self.d_bqkv = g(F.attn.in_proj_weight), g(F.attn.in_proj_bias)
        self.d_wo, self.d_bo = g(F.attn.out_proj.weight), g(F.attn.out_proj.bias)
        self.d_w1, self.d_b1 = g(G.mlp[0].weight), g(G.mlp[0].bias)
        self.d_w2, self.d_b2 = g(G.mlp[2].weight), g(G.mlp[2].bias)


class KernelMath:
    """sm_100a kernel implementation of F, G and their VJPs (bf16 compute)."""

    name = "kernels"

    def __init__(self, flat: FlatParams, dtype: torch.dtype, heads: int):
        from revpp import ops

        if dtype != torch.bfloat16:
            raise ValueError("the sm_100a kernels compute in bf16; use TorchMath for fp32 / fp16")
        self.ops = ops
        ops.ext()  # fail loudly if the extension is missing
        self.flat = flat
        self.dtype = dtype
        self.heads = heads
        self._views: dict = {}
        self._scratch: dict = {}
        self._side: dict = {}
        # weight-gradient GEMMs on a side stream, concurrent with the input-gradient chain
        # (each pair reads the same operands; the persistent GEMM that starts second fills
        # the SMs that the first one's last wave leaves idle)
        self.wgrad_overlap = os.environ.get("REVPP_WGRAD_OVERLAP", "1") != "0"

    def views(self, blk: EncoderBlock) -> _WeightViews:
        v = self._views.get(id(blk))
        if v is None:
            v = self._views[id(blk)] = _WeightViews(self.flat, blk)
        return v

    def side_stream(self) -> Optional[torch.cuda.Stream]:
        """The weight-gradient stream paired with the current stream (None: no overlap)."""
        if not self.wgrad_overlap:
            return None
        cur = torch.cuda.current_stream()
        st = self._side.get(cur.cuda_stream)
        if st is None:
            st = self._side[cur.cuda_stream] = torch.cuda.Stream(device=self.flat.device)
        return st

    def _wgrad(self, side, dy, x, dw) -> None:
        """dw += dy^T x, on ``side`` after everything queued so far on the current stream."""
        if side is None:
            self.ops.linear_wgrad(dy, x, dw)
            return
        side.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(side):
            self.ops.linear_wgrad(dy, x, dw)

    def scratch(self, name: str, shape, dtype) -> torch.Tensor:
        """Reusable per-stream buffer (same stream -> same buffer)."""
        key = (name, torch.cuda.current_stream().cuda_stream)
        t = self._scratch.get(key)
        numel = 1
        for s in shape:
            numel *= s
        if t is None or t.numel() < numel or t.dtype != dtype:
            t = torch.empty(numel, dtype=dtype, device=self.flat.device)
            self._scratch[key] = t
        return t[:numel].view(*shape)

    # -------------------------------------------------------------- forward
    def f_fwd(self, blk: EncoderBlock, x, resid, sign: float, save: bool, out: Optional[torch.Tensor] = None):
        ops = self.ops
        w = self.views(blk)
        B, S, H = x.shape
        M = B * S
        x2d = x.view(M, H)
        dev = x.device
        if save:
            a = torch.empty(M, H, dtype=torch.bfloat16, device=dev)
            qkv = torch.empty(M, 3 * H, dtype=torch.bfloat16, device=dev)
            o = torch.empty(M, H, dtype=torch.bfloat16, device=dev)
            lse = torch.empty(B, self.heads, S, dtype=torch.float32, device=dev)
            mean = torch.empty(M, dtype=torch.float32, device=dev)
            rstd = torch.empty(M, dtype=torch.float32, device=dev)
        else:
            a = self.scratch("a", (M, H), torch.bfloat16)
            qkv = self.scratch("qkv", (M, 3 * H), torch.bfloat16)
            o = self.scratch("o", (M, H), torch.bfloat16)
            lse = self.scratch("lse", (B, self.heads, S), torch.float32)
            mean = rstd = None
        if out is None:
            out = torch.empty_like(x)
        ops.layernorm_fwd(x2d, w.ln1_w, w.ln1_b, blk.F.norm.eps, y_bf16=a, mean=mean, rstd=rstd)
        ops.linear(a, w.wqkv, qkv, bias=w.bqkv)
        ops.attention_fwd(qkv, o, lse, B, S, self.heads)
        ops.linear(o, w.wo, out.view(M, H), bias=w.bo, epi=ops.EPI_RESID, resid=resid.view(M, H), sign=sign)
        ctx = SimpleNamespace(x=x, a=a, qkv=qkv, o=o, lse=lse, mean=mean, rstd=rstd, B=B, S=S) if save else None
        return out, ctx

    def g_fwd(self, blk: EncoderBlock, x, resid, sign: float, save: bool, out: Optional[torch.Tensor] = None):
        ops = self.ops
        w = self.views(blk)
        B, S, H = x.shape
        M = B * S
        I = w.w1.shape[0]
        x2d = x.view(M, H)
        dev = x.device
        if save:
            b = torch.empty(M, H, dtype=torch.bfloat16, device=dev)
            u = torch.empty(M, I, dtype=torch.bfloat16, device=dev)
            h = torch.empty(M, I, dtype=torch.bfloat16, device=dev)
            mean = torch.empty(M, dtype=torch.float32, device=dev)
            rstd = torch.empty(M, dtype=torch.float32, device=dev)
        else:
            b = self.scratch("b", (M, H), torch.bfloat16)
            h = self.scratch("h", (M, I), torch.bfloat16)
            u = mean = rstd = None
        if out is None:
            out = torch.empty_like(x)
        ops.layernorm_fwd(x2d, w.ln2_w, w.ln2_b, blk.G.norm.eps, y_bf16=b, mean=mean, rstd=rstd)
        ops.linear(b, w.w1, h, bias=w.b1, epi=ops.EPI_GELU, aux_out=u)
        ops.linear(h, w.w2, out.view(M, H), bias=w.b2, epi=ops.EPI_RESID, resid=resid.view(M, H), sign=sign)
        ctx = SimpleNamespace(x=x, b=b, u=u, h=h, mean=mean, rstd=rstd, B=B, S=S) if save else None
        return out, ctx

    # -------------------------------------------------------------- VJPs
    def g_vjp(self, blk: EncoderBlock, ctx, dy, resid_grad, out: Optional[torch.Tensor] = None,
              dy_bf16: Optional[torch.Tensor] = None, out_colsum: Optional[torch.Tensor] = None):
        """dx = resid_grad + dG/dx^T dy  for G(x) = W2 gelu(W1 LN2(x) + b1) + b2.

        ``dy_bf16``: bf16 copy of dy whose column sums are already in this block's b2
        gradient (fused into the previous LayerNorm backward).  ``out_colsum``: where the
        LayerNorm backward also accumulates the column sums of dx (the out-proj bias
        gradient when dx feeds F's VJP)."""
        ops = self.ops
        w = self.views(blk)
        B, S, H = dy.shape
        M = B * S
        I = w.w1.shape[0]
        dy2d = dy.view(M, H)
        du = self.scratch("g_du", (M, I), torch.bfloat16)
        dln = self.scratch("g_dln", (M, H), torch.bfloat16)
        if dy_bf16 is None:
            dy_bf16 = self.scratch("g_dyb", (M, H), torch.bfloat16)
            ops.cast_colsum(dy2d, out=dy_bf16, colsum=w.d_b2)           # bf16(dy), db2 += sum(dy)
        side = self.side_stream()
        self._wgrad(side, dy_bf16, ctx.h, w.d_w2)                      # dW2 += dy^T h
        # du = (dy W2) * gelu'(u), db1 += sum(du) in the same epilogue
        ops.linear_dgrad(dy_bf16, w.w2, du, epi=ops.EPI_DGELU, aux=ctx.u, colsum=w.d_b1)
        self._wgrad(side, du, ctx.b, w.d_w1)                           # dW1 += du^T LN2(x)
        ops.linear_dgrad(du, w.w1, dln)                                 # d LN2 out = du W1
        if out is None:
            out = torch.empty_like(dy)
        dxb = self.scratch("g_dxb", (M, H), torch.bfloat16)
        ops.layernorm_bwd(dln, ctx.x.view(M, H), w.ln2_w, ctx.mean, ctx.rstd, dgamma=w.d_ln2_w, dbeta=w.d_ln2_b,
                          resid=None if resid_grad is None else resid_grad.view(M, H), dx_f32=out.view(M, H),
                          dx_bf16=dxb, colsum=out_colsum)
        if side is not None:  # scratch and saved activations are reused after this VJP
            torch.cuda.current_stream().wait_stream(side)
        ctx.dx_bf16 = dxb
        ctx.dx_colsum_done = out_colsum is not None
        return out

    def f_vjp(self, blk: EncoderBlock, ctx, dy, resid_grad, out: Optional[torch.Tensor] = None,
              dy_bf16: Optional[torch.Tensor] = None, colsum_done: bool = False,
              out_bf16: Optional[torch.Tensor] = None, out_colsum: Optional[torch.Tensor] = None):
        """dx = resid_grad + dF/dx^T dy  for F(x) = Wo attn(Wqkv LN1(x) + bqkv) + bo.

        ``out_bf16`` / ``out_colsum``: the LayerNorm backward also writes bf16(dx) and adds
        the column sums of dx there (the next G VJP's operand and bias gradient)."""
        ops = self.ops
        w = self.views(blk)
        B, S, H = dy.shape
        M = B * S
        dy2d = dy.view(M, H)
        if dy_bf16 is None:
            dy_bf16 = self.scratch("f_dyb", (M, H), torch.bfloat16)
            ops.cast_colsum(dy2d, out=dy_bf16, colsum=w.d_bo)
        elif not colsum_done:
            ops.cast_colsum(dy2d, colsum=w.d_bo)
        do = self.scratch("f_do", (M, H), torch.bfloat16)
        dqkv = self.scratch("f_dqkv", (M, 3 * H), torch.bfloat16)
        dq_acc = self.scratch("f_dqacc", (M, H), torch.float32)
        dbuf = self.scratch("f_D", (B, self.heads, S), torch.float32)
        dln = self.scratch("f_dln", (M, H), torch.bfloat16)
        side = self.side_stream()
        self._wgrad(side, dy_bf16, ctx.o, w.d_wo)                      # dWo += dy^T o
        ops.linear_dgrad(dy_bf16, w.wo, do)                             # do = dy Wo
        # dqkv, and dbqkv += sum(dqkv) fused into the attention backward's write-out
        ops.attention_bwd(ctx.qkv, ctx.o, do, ctx.lse, dqkv, dq_acc, dbuf, B, S, self.heads, colsum=w.d_bqkv)
        self._wgrad(side, dqkv, ctx.a, w.d_wqkv)                       # dWqkv += dqkv^T LN1(x)
        ops.linear_dgrad(dqkv, w.wqkv, dln)                             # d LN1 out = dqkv Wqkv
        if out is None:
            out = torch.empty_like(dy)
        ops.layernorm_bwd(dln, ctx.x.view(M, H), w.ln1_w, ctx.mean, ctx.rstd, dgamma=w.d_ln1_w, dbeta=w.d_ln1_b,
                          resid=None if resid_grad is None else resid_grad.view(M, H), dx_f32=out.view(M, H),
                          dx_bf16=out_bf16, colsum=out_colsum)
        if side is not None:
            torch.cuda.current_stream().wait_stream(side)
        return out


def make_math(flat: FlatParams, dtype: torch.dtype, heads: int, device: torch.device):
    """Kernel math for bf16 on CUDA, PyTorch math otherwise (CPU runs, fp32 / fp16 modes)."""
    if device.type == "cuda" and dtype == torch.bfloat16:
        return KernelMath(flat, dtype, heads)
    return TorchMath(flat, dtype, heads)


# ====================================================================== block-level algorithms
def rev_block_forward(math_, blk: EncoderBlock, x2, x1):
    """(X2, X1) -> (Y2, Y1):  Y1 = X1 + F(X2), Y2 = X2 + G(Y1)."""
    y1, _ = math_.f_fwd(blk, x2, x1, 1.0, save=False)
    y2, _ = math_.g_fwd(blk, y1, x2, 1.0, save=False)
    return y2, y1


def rev_block_recover(math_, blk: EncoderBlock, y2, y1):
    """Reconstruct the inputs and keep what the VJPs need:
    X2 = Y2 - G(Y1), X1 = Y1 - F(X2)   (BERT/models/reversible.py:64-87)."""
    x2, ctx_g = math_.g_fwd(blk, y1, y2, -1.0, save=True)
    x1, ctx_f = math_.f_fwd(blk, x2, y1, -1.0, save=True)
    return SimpleNamespace(x2=x2, x1=x1, ctx_g=ctx_g, ctx_f=ctx_f)


def rev_block_grads(math_, blk: EncoderBlock, rc, dy2, dy1, dy2_bf16=None, prev_blk: Optional[EncoderBlock] = None):
    """dY1' = dY1 + dG/dY1^T dY2;  dX2 = dY2 + dF/dX2^T dY1';  dX1 = dY1'
    (BERT/models/reversible.py:90-110).  Returns (dX2, dX1, bf16(dX2) or None).

    Kernel path fusions: the LayerNorm backward of G also sums dY1' into the out-proj bias
    gradient and writes its bf16 copy for F's VJP; with ``prev_blk`` the LayerNorm backward
    of F writes bf16(dX2) and sums it into the previous block's FFN2 bias gradient, which
    is exactly what that block's G VJP needs first."""
    if isinstance(math_, KernelMath):
        w = math_.views(blk)
        dy1p = math_.g_vjp(blk, rc.ctx_g, dy2, dy1, dy_bf16=dy2_bf16, out_colsum=w.d_bo)
        nxt_bf16 = nxt_colsum = None
        if prev_blk is not None:
            B, S, H = dy2.shape
            nxt_bf16 = torch.empty(B * S, H, dtype=torch.bfloat16, device=dy2.device)
            nxt_colsum = math_.views(prev_blk).d_b2
        dx2 = math_.f_vjp(blk, rc.ctx_f, dy1p, dy2, dy_bf16=rc.ctx_g.dx_bf16, colsum_done=True,
                          out_bf16=nxt_bf16, out_colsum=nxt_colsum)
        return dx2, dy1p, nxt_bf16
    dy1p = math_.g_vjp(blk, rc.ctx_g, dy2, dy1)
    dx2 = math_.f_vjp(blk, rc.ctx_f, dy1p, dy2)
    return dx2, dy1p, None


def std_block_forward(math_, blk: EncoderBlock, x, save: bool):
    """Pre-LN residual block: x1 = x + F(x); x2 = x1 + G(x1)."""
    x1, cf = math_.f_fwd(blk, x, x, 1.0, save=save)
    x2, cg = math_.g_fwd(blk, x1, x1, 1.0, save=save)
    return x2, (cf, cg)


def std_block_backward(math_, blk: EncoderBlock, ctxs, dx2):
    cf, cg = ctxs
    if isinstance(math_, KernelMath):
        dx1 = math_.g_vjp(blk, cg, dx2, dx2, out_colsum=math_.views(blk).d_bo)
        return math_.f_vjp(blk, cf, dx1, dx1, dy_bf16=cg.dx_bf16, colsum_done=True)
    dx1 = math_.g_vjp(blk, cg, dx2, dx2)
    return math_.f_vjp(blk, cf, dx1, dx1)


def block_params(blk: EncoderBlock) -> List[torch.nn.Parameter]:
    return list(blk.parameters())
