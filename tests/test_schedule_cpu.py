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
