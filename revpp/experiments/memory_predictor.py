"""Analytic peak-memory model of one pipeline stage (the reference's memory predictor,
BERT/experiment/profiling/memory_predictor.py:15-167, re-derived for these kernels).

Per parameter: fp32 master + fp32 gradient + two fp32 Adam moments + bf16 shadow = 18 B
(the reference: fp32 params + grads + 2 Adam states = 16 B).

Activations with M = micro-batch * seq tokens and H the hidden size (bytes):
  reversible  one block's reconstruction context (LN outputs, packed QKV, attention output,
              GELU pre-activation and output, both reconstructed inputs) ~ 36 M H, plus the
              kernels' reusable scratch of the forward and of the VJPs and the block's fp32
              gradients ~ 90 M H (fitted to a measured peak: 126.6 M H of activations at
              M = 8192, H = 1024); PaReprop keeps two contexts.  Independent of the pipeline
              depth and of the blocks per stage.
  standard    ~ 36 M H per block per in-flight micro-batch, blocks x (P - stage) in flight.
  checkpoint  the fp32 stage input per in-flight micro-batch (P - stage) plus one stage of
              recomputed contexts.
Flash attention keeps no [heads, S, S] probabilities (the reference's math path does).
Receive buffers: a ring of 2 per channel; reversible messages are 2 (forward) and 4
(backward) fp32 [m, S, H] tensors, standard ones 1 and 1.
"""
from __future__ import annotations

from revpp.config import GlobalConfig


def stage_param_count(cfg: GlobalConfig, stage_index: int, num_stages: int, kind: str) -> int:
    H, I = cfg.hidden_size, cfg.intermediate_size
    per_block = (3 * H * H + 3 * H) + (H * H + H) + (H * I + I) + (I * H + H) + 4 * H
    n = per_block * (cfg.num_hidden_layers // num_stages)
    if stage_index == 0:
        if cfg.model == "bert":
            n += (cfg.vocab_size + cfg.max_position_embeddings + cfg.type_vocab_size) * H + 2 * H
        else:
            p = cfg.patch_size
            n += cfg.num_channels * p * p * H + H + H + cfg.seq_len * H + 2 * H
    if stage_index == num_stages - 1:
        w = 2 * H if kind == "inverse" else H
        n += 2 * w + w * cfg.num_classes + cfg.num_classes
    return n


def predict_breakdown(cfg: GlobalConfig, stage_index: int, num_stages: int, kind: str,
                      pareprop: bool = False) -> dict:
    H = cfg.hidden_size
    M = cfg.microbatch_size * cfg.seq_len
    blocks = cfg.num_hidden_layers // num_stages
    in_flight = min(num_stages - stage_index, cfg.num_microbatches)
    params = stage_param_count(cfg, stage_index, num_stages, kind)
    msg = M * H * 4
    if kind in ("reversible", "inverse"):
        recv = 2 * (2 * msg) * (stage_index > 0) + 2 * (4 * msg) * (stage_index < num_stages - 1)
        ctx = 36 * M * H
        act = ctx * (2 if pareprop else 1) + 90 * M * H
        if kind == "inverse":
            act = 36 * M * H * blocks + 38 * M * H
        if stage_index == num_stages - 1:
            act += 4 * msg  # cached outputs and their gradients for the head
    elif kind == "standard":
        recv = 2 * msg * ((stage_index > 0) + (stage_index < num_stages - 1))
        act = 36 * M * H * blocks * in_flight + 38 * M * H
    else:  # checkpoint
        recv = 2 * msg * ((stage_index > 0) + (stage_index < num_stages - 1))
        act = msg * in_flight + 36 * M * H * blocks + 38 * M * H
    first_inputs = 0
    if stage_index == 0:
        per_sample = cfg.seq_len * 16 if cfg.model == "bert" else cfg.num_channels * cfg.img_size ** 2 * 4
        first_inputs = per_sample * cfg.microbatch_size * in_flight
    return {"params_and_optimizer": 18 * params, "receive_buffers": recv, "activations": act,
            "first_stage_inputs": first_inputs, "param_count": params}


def predict_peak_bytes(cfg: GlobalConfig, stage_index: int, num_stages: int, kind: str, pareprop: bool = False) -> int:
    b = predict_breakdown(cfg, stage_index, num_stages, kind, pareprop)
    return int(b["params_and_optimizer"] + b["receive_buffers"] + b["activations"] + b["first_stage_inputs"])


def max_microbatch_for_budget(cfg: GlobalConfig, num_stages: int, kind: str, budget_bytes: int,
                              pareprop: bool = False, limit: int = 4096) -> int:
    """PaBER: the largest micro-batch whose predicted peak fits the budget on every stage."""
    best = 0
    mb = 1
    while mb <= limit:
        c = cfg.with_(microbatch_size=mb, batch_size=mb * cfg.num_microbatches)
        if all(predict_peak_bytes(c, s, num_stages, kind, pareprop) <= budget_bytes for s in range(num_stages)):
            best = mb
            mb *= 2
        else:
            break
    return best
