"""Host logic of bench.py (CPU only): which launches of the dominant kernel
count as having had the GPU to themselves on the overlapped path, and the
per-phase summary the roofline is computed from."""

import bench


class FakeEvent:
    """Stands in for a CUDA event recorded at time ``t`` (ms)."""

    def __init__(self, t):
        self.t = t

    def elapsed_time(self, other):
        return other.t - self.t


def _rec(name, t0, t1):
    return (name, FakeEvent(t0), FakeEvent(t1))


def test_solo_launches_are_those_after_the_last_state_pass():
    t0 = FakeEvent(0.0)
    step = [_rec("fwd_intra", 0, 1), _rec("fwd_state", 1, 3),
            _rec("bwd_state", 3, 4), _rec("bwd_intra", 4, 6),    # beside the next state pass
            _rec("bwd_state", 4, 5.5), _rec("bwd_intra", 6, 7)]  # after the chain ended
    second = [(n, FakeEvent(s.t + 10), FakeEvent(e.t + 10)) for n, s, e in step]
    solo, every, per_step = bench.solo_launches(step + second, t0)
    assert per_step == 2
    assert every == [2, 1, 2, 1]
    assert solo == [1, 1]


def test_phase_summary_is_per_step_mean():
    rec = [_rec("bwd_intra", 0, 2), _rec("bwd_intra", 2, 3), _rec("fwd_state", 0, 4)]
    ph = bench.phase_summary(rec, steps=2)
    assert ph["bwd_intra"] == {"ms": 1.5, "launches": 2}
    assert ph["fwd_state"] == {"ms": 2.0, "launches": 1}
