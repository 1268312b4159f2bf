"""Thin Python entry points of the sm_100a kernels (module ``revpp._C``).

Every function here takes CUDA tensors and launches the extension's kernels on the
current stream; there is no PyTorch fallback on the GPU.  CPU execution goes through
``revpp.models.blockmath.TorchMath`` instead.
"""
from __future__ import annotations

import os
from typing import Optional

import torch

from ._ext import available, check_status, ext

EPI_BF16, EPI_GELU, EPI_RESID, EPI_ATOMIC, EPI_DGELU, EPI_F32 = range(6)

_SM_RESERVE = 0


def set_sm_reserve(n: int) -> None:
    """Leave ``n`` SMs free of persistent GEMM CTAs (for concurrent NCCL kernels)."""
    global _SM_RESERVE
    _SM_RESERVE = max(0, int(n))
    if available():
        ext().set_sm_reserve(_SM_RESERVE)


def linear(x: torch.Tensor, w: torch.Tensor, out: torch.Tensor, bias: Optional[torch.Tensor] = None,
           epi: int = EPI_BF16, aux_out: Optional[torch.Tensor] = None, resid: Optional[torch.Tensor] = None,
           sign: float = 1.0) -> torch.Tensor:
    """out[M, N] = epi(x[M, K] @ w[N, K]^T + bias)   (forward GEMM, both operands K-major)."""
    M, K = x.shape
    N = w.shape[0]
    ext().gemm_tc(x, False, w, False, M, N, K, epi, out, bias=bias, aux_out=aux_out, resid=resid, sign=sign)
    return out


def linear_dgrad(dy: torch.Tensor, w: torch.Tensor, out: torch.Tensor, epi: int = EPI_BF16,
                 aux: Optional[torch.Tensor] = None, colsum: Optional[torch.Tensor] = None) -> torch.Tensor:
    """out[M, K] = epi(dy[M, N] @ w[N, K])   (input gradient; w read MN-major).  With the
    GELU-backward epilogue, ``colsum`` (fp32 [K]) accumulates the column sums of ``out``."""
    M, N = dy.shape
    K = w.shape[1]
    ext().gemm_tc(dy, False, w, True, M, K, N, epi, out, aux=aux, colsum=colsum)
    return out


def linear_wgrad(dy: torch.Tensor, x: torch.Tensor, dw: torch.Tensor, splits: Optional[int] = None) -> torch.Tensor:
    """dw[N, K] += dy[M, N]^T @ x[M, K]   (weight gradient, fp32 accumulation with atomics)."""
    M, N = dy.shape
    K = x.shape[1]
    C = ext()
    if splits is None:
        splits = C.gemm_suggest_splits(N, K, M)
    C.gemm_tc(dy, True, x, True, N, K, M, EPI_ATOMIC, dw, splits=splits)
    return dw


def layernorm_fwd(x, gamma, beta, eps, y_bf16=None, y_f32=None, y2_f32=None, mean=None, rstd=None):
    ext().layernorm_fwd(x, gamma, beta, eps, y_bf16=y_bf16, y_f32=y_f32, y2_f32=y2_f32, mean=mean, rstd=rstd)


def layernorm_bwd(dy, x, gamma, mean, rstd, dgamma=None, dbeta=None, resid=None, dx_f32=None, dx_bf16=None,
                  colsum=None):
    ext().layernorm_bwd(dy, x, gamma, mean, rstd, dgamma=dgamma, dbeta=dbeta, resid=resid, dx_f32=dx_f32,
                        dx_bf16=dx_bf16, colsum=colsum)


def cast_colsum(inp, out=None, colsum=None):
    ext().cast_colsum(inp, out=out, colsum=colsum)


_ATTN_TC = os.environ.get("REVPP_ATTN_TC", "1") != "0"
_ATTN_FWD = os.environ.get("REVPP_ATTN_FWD", "grid")


def attention_fwd(qkv, out, lse, B, S, heads):
    """Flash attention forward: the tcgen05 kernel with one CTA per query tile, two CTAs per
    SM (REVPP_ATTN_FWD=persistent selects the persistent kernel, measured slower at head
    dim 64; REVPP_ATTN_TC=0 the warp-level mma.sync kernel; both kept as comparison points)."""
    if not _ATTN_TC:
        ext().attn_fwd(qkv, out, lse, B, S, heads)
    elif _ATTN_FWD == "persistent":
        ext().attn_fwd_persistent(qkv, out, lse, B, S, heads)
    else:
        ext().attn_fwd_tc(qkv, out, lse, B, S, heads)


def attention_bwd(qkv, out, dout, lse, dqkv, dq_acc, dbuf, B, S, heads, colsum=None):
    """Flash attention backward (tcgen05; REVPP_ATTN_TC=0 selects the mma.sync kernel).
    ``colsum`` (fp32 [3H]) accumulates the column sums of dqkv (the in-projection bias
    gradient); the tcgen05 path fuses it into its write-out."""
    if _ATTN_TC:
        ext().attn_bwd_tc(qkv, out, dout, lse, dqkv, dq_acc, dbuf, B, S, heads, colsum=colsum)
    else:
        ext().attn_bwd(qkv, out, dout, lse, dqkv, dq_acc, dbuf, B, S, heads)
        if colsum is not None:
            cast_colsum(dqkv, colsum=colsum)


__all__ = [
    "available", "check_status", "ext", "set_sm_reserve", "linear", "linear_dgrad", "linear_wgrad",
    "layernorm_fwd", "layernorm_bwd", "cast_colsum", "attention_fwd", "attention_bwd",
    "EPI_BF16", "EPI_GELU", "EPI_RESID", "EPI_ATOMIC", "EPI_DGELU", "EPI_F32",
]
