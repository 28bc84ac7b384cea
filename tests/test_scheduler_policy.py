"""Scheduler bridge port and the scheduler-aware prefetch policy, on CPU with
fake scheduler objects and a fake staging target (no GPU)."""

from adapterslotsplusplus_b200.scheduler_bridge import (AdapterIdMap, GwarHistory, PrefetchPolicy, SchedulerBridge,
                                                        segments_to_warp_pipe)


class FakeEngine:
    def __init__(self):
        self.bridge = None

    def write_bridge(self, whittle, t_rem, gwar, lam, burst, promo, hot, tile, n, nseg, step, load):
        self.bridge = {"whittle_scores": whittle.tolist(), "t_remaining_ms": t_rem.tolist(),
                       "gwar_pred_next3": gwar.tolist(), "lambda_hat": lam.tolist(), "burst_active": burst.tolist(),
                       "promo_eligible": promo.tolist(), "is_hot": hot.tolist(), "tile_size_code": tile.tolist(),
                       "num_active_adapters": n, "num_segments": nseg, "step_id": step, "global_load": load}

    def read_bridge_debug(self):
        return dict(self.bridge)


class FakeTarget:
    """Staging slots: prefetch returns a slot while one is free."""

    def __init__(self, slots):
        self.free = list(range(slots))
        self.held = {}
        self.log = []

    def prefetch(self, i):
        self.log.append(("prefetch", i))
        if i in self.held:
            return self.held[i]
        if not self.free:
            return -1
        self.held[i] = self.free.pop(0)
        return self.held[i]

    def is_prefetch_ready(self, i):
        return i in self.held

    def release_prefetch(self, i):
        self.log.append(("release", i))
        if i in self.held:
            self.free.append(self.held.pop(i))


class Whittle:
    def compute_indices(self, fill, lam):
        return {a: fill[a] * lam[a] for a in fill}


class Rates:
    def __init__(self, r):
        self.r = r

    def get_rate(self, a):
        return self.r.get(a, 0.0)


class Merged:
    def is_merged(self, a):
        return a == "c"


def test_id_map_and_segments():
    m = AdapterIdMap()
    assert [m.get_or_assign(s) for s in ("x", "y", "x", "z")] == [0, 1, 0, 2]
    assert m.ordered_ids() == ["x", "y", "z"] and len(m) == 3 and m.to_int("z") == 2

    class Seg:
        def __init__(self, a, n):
            self.adapter_id, self.segment_size = a, n

    ids, offs = segments_to_warp_pipe([Seg("y", 3), Seg("q", 5), Seg("x", 2)], m)
    assert ids == [1, 3, 0] and offs == [0, 3, 8, 10]


def test_gwar_history_ewma():
    g = GwarHistory(alpha=0.5)
    assert g.update("a", 1.0) == 1.0
    assert abs(g.update("a", 0.0) - 0.5) < 1e-9
    assert g.get("missing") == 0.0


def test_scheduler_bridge_writes_tick():
    eng = FakeEngine()
    m = AdapterIdMap()
    for a in ("a", "b", "c"):
        m.get_or_assign(a)
    br = SchedulerBridge(eng, m)
    br.write(7, whittle_dispatcher=Whittle(), fill_fracs={"a": 0.5, "b": 1.0, "c": 0.0},
             lambda_est={"a": 2.0, "b": 4.0, "c": 1.0}, estimator=Rates({"b": 30.0}), gwar_readings={"a": 0.9},
             mwc=Merged(), global_load=0.3, queued=["c"])
    b = eng.bridge
    assert b["num_active_adapters"] == 3 and b["num_segments"] == 7 and b["step_id"] == 0
    assert b["whittle_scores"] == [1.0, 4.0, 0.0]
    assert b["lambda_hat"] == [0.0, 30.0, 0.0]
    assert abs(b["gwar_pred_next3"][0] - 0.9) < 1e-6 and b["tile_size_code"][0] == 2
    assert b["promo_eligible"] == [0, 0, 1] and b["is_hot"] == [0, 0, 1]
    br.write(1)
    assert eng.bridge["step_id"] == 1


def _bridge(n, hot=(), lam=None, whittle=None):
    return {"num_active_adapters": n, "is_hot": [1 if i in hot else 0 for i in range(n)],
            "whittle_scores": whittle or [0.0] * n, "lambda_hat": lam or [0.0] * n,
            "gwar_pred_next3": [0.0] * n}


def test_policy_prefetches_queued_then_likely_arrivals():
    t = FakeTarget(slots=3)
    pol = PrefetchPolicy(t, budget=2, horizon_s=0.01)
    out = pol.tick(_bridge(6, hot={4}, lam=[0, 50.0, 0, 0, 0, 20.0]))
    # the queued adapter first, then the highest arrival rate
    assert out["prefetched"] == [4, 1] and out["held"] == [1, 4]
    # next tick: adapter 4 was scheduled (not hot any more), 5 is queued
    out = pol.tick(_bridge(6, hot={5}, lam=[0, 50.0, 0, 0, 0, 20.0]), protected=[4])
    assert 5 in out["prefetched"] and out["released"] == []  # 4 is protected by the step in flight
    out = pol.tick(_bridge(6, hot=set(), lam=[0, 50.0, 0, 0, 0, 0]))
    assert set(out["released"]) == {4, 5} and out["held"] == [1]


def test_policy_respects_budget_threshold_and_full_target():
    t = FakeTarget(slots=1)
    pol = PrefetchPolicy(t, budget=4, min_priority=0.1, horizon_s=0.01)
    out = pol.tick(_bridge(4, lam=[1.0, 30.0, 20.0, 5.0]))  # priorities 0.01, 0.3, 0.2, 0.05
    assert out["prefetched"] == [1] and pol.refused == 1  # one slot: 2 refused, then stop
    assert ("prefetch", 0) not in t.log and ("prefetch", 3) not in t.log  # below the threshold
