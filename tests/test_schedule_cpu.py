"""Schedules as action lists, the schedule simulator and its trace dump, and the receive-ring
reuse check (all host-side)."""
import json

import pytest
import torch

from revpp.parallel.p2p import RecvRing, RingSlotError, TensorSpec
from revpp.parallel.schedule import SCHEDULES, dump_chrometrace, forward_only, one_f_one_b, simulate


@pytest.mark.parametrize("P,n", [(1, 4), (2, 4), (4, 8), (8, 32), (4, 2)])
def test_one_f_one_b_order(P, n):
    for s in range(P):
        acts = one_f_one_b(s, P, n)
        assert sorted(a for a in acts if a[0] == "F") == [("F", i) for i in range(n)]
        assert sorted(a for a in acts if a[0] == "B") == [("B", i) for i in range(n)]
        # each micro-batch's forward comes before its backward
        for i in range(n):
            assert acts.index(("F", i)) < acts.index(("B", i))
        # warm-up of min(n, P - s) forwards, then strictly alternating 1B1F while forwards remain
        warm = min(n, P - s)
        assert acts[:warm] == [("F", i) for i in range(warm)]
        steady = acts[warm:warm + 2 * (n - warm)]
        assert [k for k, _ in steady] == ["B", "F"] * (n - warm)
        # in-flight micro-batches (forward done, backward not yet) never exceed P - s
        live = peak = 0
        for k, _ in acts:
            live += 1 if k == "F" else -1
            peak = max(peak, live)
        assert peak == warm


def test_forward_only_and_gpipe():
    assert forward_only(1, 4, 3) == [("F", 0), ("F", 1), ("F", 2)]
    g = SCHEDULES["gpipe"](2, 4, 3)
    assert g == [("F", 0), ("F", 1), ("F", 2), ("B", 0), ("B", 1), ("B", 2)]


@pytest.mark.parametrize("schedule", ["1f1b", "gpipe"])
@pytest.mark.parametrize("P,n", [(2, 8), (4, 8), (8, 32)])
def test_simulated_makespan_matches_pipeline_bubble(schedule, P, n):
    t_f, t_b = 1.0, 2.0
    makespan, busy = simulate(P, n, schedule, t_f, t_b)
    assert makespan == pytest.approx((n + P - 1) * (t_f + t_b))
    assert all(b == pytest.approx(n * (t_f + t_b)) for b in busy)


def test_chrometrace_dump(tmp_path):
    path = tmp_path / "sched.json"
    makespan = dump_chrometrace(4, 8, path)
    tr = json.loads(path.read_text())["traceEvents"]
    slices = [e for e in tr if e["ph"] == "X"]
    assert len(slices) == 2 * 4 * 8
    assert max(e["ts"] + e["dur"] for e in slices) == pytest.approx(makespan * 1e3)
    # no two slices of one stage overlap
    for s in range(4):
        sl = sorted((e["ts"], e["ts"] + e["dur"]) for e in slices if e["tid"] == s)
        assert all(a[1] <= b[0] + 1e-9 for a, b in zip(sl, sl[1:]))


def test_recv_ring_detects_reuse_before_consume():
    ring = RecvRing("fwd", [TensorSpec((2, 3), torch.float32)], torch.device("cpu"), depth=2)
    s0, b0 = ring.acquire()
    s1, b1 = ring.acquire()
    assert s0 != s1 and b0[0].shape == (2, 3)
    with pytest.raises(RingSlotError):
        ring.acquire()  # slot 0 again while its message is still unconsumed
    ring.release(s0)
    s2, b2 = ring.acquire()
    assert s2 == s0 and b2[0].data_ptr() == b0[0].data_ptr()
    assert ring.gen[s0] == 2


@pytest.mark.parametrize("P,v,n", [(2, 2, 8), (4, 2, 8), (4, 3, 32), (8, 3, 32), (4, 2, 4)])
def test_interleaved_order(P, v, n):
    """Every rank runs the forward and the backward of every (chunk, micro-batch) exactly
    once, each forward before its backward, with the reference's warm-up length."""
    from revpp.parallel.schedule import interleaved_1f1b

    for r in range(P):
        acts = interleaved_1f1b(r, P, v, n)
        want = sorted((c, m) for c in range(v) for m in range(n))
        assert sorted((c, m) for k, c, m in acts if k == "F") == want
        assert sorted((c, m) for k, c, m in acts if k == "B") == want
        for c in range(v):
            for m in range(n):
                assert acts.index(("F", c, m)) < acts.index(("B", c, m))
        warm = n * v if n == P else min((P - r - 1) * 2 + (v - 1) * P, n * v)
        assert all(k == "F" for k, _, _ in acts[:warm]) and acts[warm][0] == "F" or warm == n * v


def test_interleaved_reduces_bubble():
    """The simulated makespan of interleaved 1F1B beats plain 1F1B at the same work, and the
    gain grows with the pipeline depth."""
    from revpp.parallel.schedule import simulate_virtual

    gains = []
    for P in (2, 4, 8):
        base, _ = simulate_virtual(P, 1, 32, "1f1b", 1.0, 3.0)
        il, busy = simulate_virtual(P, 3, 32, "interleaved", 1.0 / 3, 1.0)
        assert il < base
        assert abs(sum(busy) / P - 32 * 4.0) < 1e-6  # same work per rank
        gains.append(base / il)
    assert gains == sorted(gains)


@pytest.mark.parametrize("P,v", [(2, 1), (4, 1), (8, 1), (2, 2), (4, 3), (8, 3)])
def test_channel_depth_is_deadlock_free_and_minimal(P, v):
    """The host-level run of the channel protocol finishes two steps with the chosen ring
    depth (and with a deeper ring)."""
    from revpp.parallel.schedule import host_deadlock_free, min_channel_depth

    sched = "interleaved" if v > 1 else "1f1b"
    d = min_channel_depth(P, v, 32, sched)
    assert host_deadlock_free(P, v, 32, sched, d)
    assert host_deadlock_free(P, v, 32, sched, d + 1)


def test_pipeline_breakdown_splits_idle_into_bubble_and_exposed():
    from revpp.parallel.schedule import pipeline_breakdown

    P, n, tf, tb = 4, 8, 1.0, 2.0
    bubble = (P - 1) * (tf + tb)  # 1F1B idle time of every rank with equal stages
    step = n * (tf + tb) + bubble
    summ = [{"step_ms": step + 0.5, "compute_ms": n * (tf + tb), "idle_ms": bubble + 0.5, "fwd_action_ms": tf,
             "bwd_action_ms": tb} for _ in range(P)]
    out = pipeline_breakdown(summ, P, 1, n, "1f1b")
    for d in out:
        assert abs(d["bubble_ms"] - bubble) < 1e-9
        assert abs(d["exposed_p2p_ms"] - 0.5) < 1e-9
    # interleaving with 2 chunks per rank (per-chunk times halve) shrinks the simulated bubble
    summ2 = [dict(s, fwd_action_ms=tf / 2, bwd_action_ms=tb / 2) for s in summ]
    out2 = pipeline_breakdown(summ2, P, 2, n, "interleaved")
    assert all(d2["bubble_ms"] < d["bubble_ms"] for d, d2 in zip(out, out2))
