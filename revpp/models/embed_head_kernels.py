"""Embedding and classifier-head math on the sm_100a kernels (bf16 runs on CUDA)."""
from __future__ import annotations

from .encoder import TorchEmbedHead


class KernelEmbedHead(TorchEmbedHead):
    """Placeholder until the embedding / head kernels land: same math as TorchEmbedHead."""
