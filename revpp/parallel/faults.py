"""Host-side fault injection for pipeline tests (no GPU fault is ever injected).

    REVPP_FAULT_DROP_SEND="<channel name>:<n>"   skip the n-th send (0-based) on that channel
    REVPP_FAULT_RAISE_AT="<rank>:<micro-batch>"  raise on that rank before that forward
    REVPP_FAULT_EXIT_AT="<rank>:<micro-batch>"   exit the process there (os._exit)

Survivors learn of the failure through the process group: a receive whose sender never
sends, or whose peer died, ends with an error when the group's timeout (or the broken
connection) fires, instead of waiting forever.
"""
from __future__ import annotations

import os


class InjectedFault(RuntimeError):
    pass


def _parse(var: str):
    v = os.environ.get(var)
    if not v:
        return None
    a, b = v.rsplit(":", 1)
    return a, int(b)


def should_drop(channel: str, index: int) -> bool:
    spec = _parse("REVPP_FAULT_DROP_SEND")
    return spec is not None and spec[0] == channel and spec[1] == index


def before_forward(rank: int, mb: int) -> None:
    spec = _parse("REVPP_FAULT_RAISE_AT")
    if spec is not None and int(spec[0]) == rank and spec[1] == mb:
        raise InjectedFault(f"injected failure on rank {rank} before micro-batch {mb}")
    spec = _parse("REVPP_FAULT_EXIT_AT")
    if spec is not None and int(spec[0]) == rank and spec[1] == mb:
        os._exit(17)
