"""CPU: the vectorized resident-set planner (tidegs_b200/resident_policy.py)
against the reference planner's transitions recorded in
tests/golden/planner.json (7 policy/capacity/seed-fraction cases x 30 steps,
recency scores and resident sets fed back between steps): every field of
every transition equal (per-field digests of the canonical JSON), with the
recency scores passed as the reference's dict and as RecencyScores."""
import json
import sys
from pathlib import Path

import pytest

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE / "golden"))
import make_planner_golden as G  # noqa: E402

from tidegs_b200 import resident_policy as rp  # noqa: E402

FIX = json.loads((HERE / "golden" / "planner.json").read_text())


def _replay(case, dense: bool):
    sched = G.camera_schedule(case["seed"], case["steps"] + 1)
    recency = rp.RecencyScores() if dense else {}
    resident = None
    for k in range(case["steps"]):
        cur, nxt = G.union(sched[k]), G.union(sched[k + 1])
        given = resident if (resident is None or k % 7 != 3) else resident[: len(resident) // 2]
        kw = dict(current_active_blocks=cur, next_active_blocks=nxt,
                  current_resident_blocks=given, next_camera_ids=sorted(sched[k + 1]),
                  next_camera_blocks=sched[k + 1], previous_recency_scores=recency,
                  recency_decay=0.9)
        if case["policy"] == "passthrough":
            tr = rp.compute_passthrough_resident_transition(**kw)
        else:
            tr = rp.compute_topc_resident_transition(
                **kw, lambda_weight=0.7, resident_capacity_blocks=case["capacity"],
                balanced_camera_seeds=(case["policy"] == "topc_balanced"),
                balanced_seed_fraction=case["fraction"])
        got = G.field_digests(tr)
        want = case["records"][k]
        bad = [f for f in want if got.get(f) != want[f]]
        assert not bad, f"{case['policy']} cap {case['capacity']} step {k}: {bad}"
        assert isinstance(tr.updated_recency_scores, rp.RecencyScores if dense else dict)
        recency = tr.updated_recency_scores
        resident = list(tr.next_resident_blocks)


@pytest.mark.parametrize("dense", [False, True])
@pytest.mark.parametrize("k", range(len(FIX["cases"])))
def test_planner_matches_reference(k, dense):
    _replay(FIX["cases"][k], dense)


def test_recency_scores_mapping():
    s = rp.RecencyScores.from_dict({5: 0.5, 2: 1.0})
    assert dict(s) == {2: 1.0, 5: 0.5} and len(s) == 2 and 3 not in s
    tr = rp.compute_passthrough_resident_transition([1, 2], [2, 3], previous_recency_scores=s,
                                                    recency_decay=0.5)
    assert dict(tr.updated_recency_scores) == {1: 1.0, 2: 1.0, 5: 0.25}
    empty = rp.compute_topc_resident_transition([], [], resident_capacity_blocks=4)
    assert empty.next_resident_blocks == [] and empty.topc_cutoff_score == 0.0


def test_recency_update_fast_path_equals_converting_path():
    """The returned dict passed back (no per-entry conversions) and a copy of
    it (converted like the reference converts foreign dicts) give the same
    scores; foreign key / value types are converted to int / float."""
    import numpy as np

    prev = {np.int64(5): np.float64(0.5), 7: 1e-6, "9": 0.3, 11: np.float32(0.25)}
    upd, look = rp._updated_recency(prev, np.array([3, 5]), 0.9)
    assert upd == {5: 1.0, 9: 0.27, 11: np.float32(0.25) * 0.9, 3: 1.0}
    assert all(type(k) is int for k in upd) and all(type(v) is float for v in upd.values())
    np.testing.assert_array_equal(look(np.array([3, 100, 9])), [1.0, 0.0, 0.27])
    fast, _ = rp._updated_recency(upd, np.array([100]), 0.5)     # the dict returned last
    slow, _ = rp._updated_recency(dict(upd), np.array([100]), 0.5)  # a foreign copy
    assert fast == slow and list(fast.items()) == list(slow.items())



def test_recency_dict_edited_in_place_is_converted_again():
    """A caller that writes numpy scalars into the returned dict gets the
    reference's conversions on the next transition (resident_policy.py:
    115-119), exactly as for a foreign dict with the same entries."""
    import numpy as np

    upd, _ = rp._updated_recency({1: 0.5, 2: 0.25}, np.array([3]), 0.9)
    upd[np.int64(8)] = np.float32(0.7)
    upd[1] = np.float32(0.3)
    edited, _ = rp._updated_recency(upd, np.array([4]), 0.5)
    foreign, _ = rp._updated_recency(dict(upd), np.array([4]), 0.5)
    assert list(edited.items()) == list(foreign.items())
    assert all(type(k) is int for k in edited) and all(type(v) is float for v in edited.values())
    # an untouched returned dict takes the fast path and gives the same result
    clean, _ = rp._updated_recency({1: 0.5, 2: 0.25}, np.array([3]), 0.9)
    assert clean.pristine
    a, _ = rp._updated_recency(clean, np.array([4]), 0.5)
    b, _ = rp._updated_recency(dict(clean), np.array([4]), 0.5)
    assert list(a.items()) == list(b.items())
