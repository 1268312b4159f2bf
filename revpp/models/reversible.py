"""Reversible block sequences: no-grad forward, and the backward that reconstructs
inputs instead of storing them.

``rev_backward`` walks the blocks from last to first; for block i it reconstructs the
block input (X2 = Y2 - G(Y1), X1 = Y1 - F(X2)) and then runs the two VJPs
(BERT/models/reversible.py:64-110, 223-258).  The stage therefore holds one block's
intermediates at a time, whatever the number of blocks or pipeline stages.

``pareprop=True`` runs the reference's two-stream schedule
(BERT/models/reversible.py:132-221): the gradient step of block i runs on one stream
while the reconstruction of block i-1 runs on the other; event f{i} marks "block i
reconstructed", b{i} marks "block i gradients done".  Unlike the reference, every tensor
handed from one stream to the other is registered with ``record_stream`` so the caching
allocator cannot recycle it while the other stream still reads it.
"""
from __future__ import annotations

from typing import List, Optional, Sequence, Tuple

import torch

from .blockmath import rev_block_forward, rev_block_grads, rev_block_recover
from .modules import EncoderBlock


def rev_forward(math_, blocks: Sequence[EncoderBlock], x2: torch.Tensor, x1: torch.Tensor):
    with torch.no_grad():
        for blk in blocks:
            x2, x1 = rev_block_forward(math_, blk, x2, x1)
    return x2, x1


def _record(ts, stream) -> None:
    if stream is None:
        return
    for t in ts:
        if t is not None and isinstance(t, torch.Tensor) and t.is_cuda:
            t.record_stream(stream)


def _record_ctx(rc, stream) -> None:
    if stream is None:
        return
    _record([rc.x2, rc.x1], stream)
    for c in (rc.ctx_g, rc.ctx_f):
        _record([v for v in vars(c).values() if isinstance(v, torch.Tensor)], stream)


def rev_backward(math_, blocks: Sequence[EncoderBlock], y2, y1, dy2, dy1, pareprop: bool = False,
                 streams: Optional[Tuple[torch.cuda.Stream, torch.cuda.Stream]] = None,
                 on_recover=None):
    """Returns ((dX2, dX1), (X2, X1)) for the first block's input.

    ``on_recover(i, x2, x1)`` is called after block i's input is reconstructed (used by
    the activation-error experiment)."""
    n = len(blocks)
    if n == 0:
        return (dy2, dy1), (y2, y1)
    with torch.no_grad():
        if not pareprop or streams is None or not y2.is_cuda:
            rc = rev_block_recover(math_, blocks[-1], y2, y1)
            dy = (dy2, dy1)
            dyb = None
            for i in range(n - 1, -1, -1):
                if on_recover is not None:
                    on_recover(i, rc.x2, rc.x1)
                prev = blocks[i - 1] if i > 0 else None
                dx2, dx1, dyb = rev_block_grads(math_, blocks[i], rc, dy[0], dy[1], dy2_bf16=dyb, prev_blk=prev)
                dy = (dx2, dx1)
                if i > 0:
                    rc = rev_block_recover(math_, blocks[i - 1], rc.x2, rc.x1)
            return dy, (rc.x2, rc.x1)
        return _pareprop_backward(math_, blocks, y2, y1, dy2, dy1, streams, on_recover)


def _pareprop_backward(math_, blocks, y2, y1, dy2, dy1, streams, on_recover):
    s1, s2 = streams
    main = torch.cuda.current_stream()
    n = len(blocks)
    f_ev = [torch.cuda.Event() for _ in range(n)]
    b_ev = [torch.cuda.Event() for _ in range(n)]
    s1.wait_stream(main)
    s2.wait_stream(main)
    _record([y2, y1, dy2, dy1], s1)
    _record([y2, y1, dy2, dy1], s2)
    # reconstruct the last block on s1
    with torch.cuda.stream(s1):
        rc = rev_block_recover(math_, blocks[n - 1], y2, y1)
        f_ev[0].record(s1)
    dy = (dy2, dy1)
    dyb = None
    # step i handles block n-1-i: gradient on one stream, reconstruction of the next on the other
    for i in range(n - 1):
        this_blk = blocks[n - 1 - i]
        next_blk = blocks[n - 2 - i]
        s_grad, s_rec = (s1, s2) if i % 2 == 0 else (s2, s1)
        _record_ctx(rc, s_grad)
        _record_ctx(rc, s_rec)
        _record(list(dy) + [dyb], s_grad)
        with torch.cuda.stream(s_grad):
            if i > 0:
                s_grad.wait_event(b_ev[i - 1])
            s_grad.wait_event(f_ev[i])
            if on_recover is not None:
                on_recover(n - 1 - i, rc.x2, rc.x1)
            dx2, dx1, dyb = rev_block_grads(math_, this_blk, rc, dy[0], dy[1], dy2_bf16=dyb, prev_blk=next_blk)
            dy = (dx2, dx1)
            b_ev[i].record(s_grad)
        with torch.cuda.stream(s_rec):
            s_rec.wait_event(f_ev[i])
            rc = rev_block_recover(math_, next_blk, rc.x2, rc.x1)
            f_ev[i + 1].record(s_rec)
    s_grad = s1 if (n - 1) % 2 == 0 else s2
    _record_ctx(rc, s_grad)
    _record(list(dy) + [dyb], s_grad)
    with torch.cuda.stream(s_grad):
        if n > 1:
            s_grad.wait_event(b_ev[n - 2])
        s_grad.wait_event(f_ev[n - 1])
        if on_recover is not None:
            on_recover(0, rc.x2, rc.x1)
        dx2, dx1, _ = rev_block_grads(math_, blocks[0], rc, dy[0], dy[1], dy2_bf16=dyb)
        dy = (dx2, dx1)
        b_ev[n - 1].record(s_grad)
    main.wait_stream(s1)
    main.wait_stream(s2)
    _record([dy[0], dy[1], rc.x2, rc.x1], main)
    return dy, (rc.x2, rc.x1)


def inverse_sequence(math_, blocks: Sequence[EncoderBlock], y2, y1):
    """Inputs of the first block from the outputs of the last, without any VJP
    (BertMidStageWithInverse.inverse, bert_stages_with_inverse.py:150-154)."""
    with torch.no_grad():
        for blk in reversed(blocks):
            rc = rev_block_recover(math_, blk, y2, y1)
            y2, y1 = rc.x2, rc.x1
    return y2, y1


__all__ = ["rev_forward", "rev_backward", "inverse_sequence"]
