"""Generates tests/golden/planner.json by running the reference resident-set
planner (strategies/tide_engine/resident_policy.py, loaded by file path) on
seeded multi-step camera schedules, feeding each step's updated recency
scores and next resident set into the next step.

    python tests/golden/make_planner_golden.py --reference <TideGS checkout>
"""
from __future__ import annotations

import argparse
import hashlib
import importlib.util
import json
import sys
import time
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent

CASES = [  # (policy, capacity, balanced seed fraction)
    ("passthrough", -1, 1.0),
    ("topc_strict", -1, 1.0),
    ("topc_strict", 600, 1.0),
    ("topc_balanced", 600, 1.0),
    ("topc_balanced", 900, 0.5),
    ("topc_balanced", 400, 0.0),
    ("topc_balanced", 1500, 0.3),
]


def camera_schedule(seed: int, steps: int, n_blocks: int = 3000, cams: int = 8):
    """Per step {camera id: visible blocks}: contiguous runs drifting along
    the scene, so consecutive steps overlap."""
    rng = np.random.default_rng(seed)
    out = []
    pos = rng.integers(0, n_blocks)
    for _ in range(steps):
        pos = (pos + int(rng.integers(20, 120))) % n_blocks
        step = {}
        for c in rng.choice(64, cams, replace=False).tolist():
            start = (pos + int(rng.integers(-150, 150))) % n_blocks
            length = int(rng.integers(30, 140))
            ids = [(start + k) % n_blocks for k in range(length)]
            if rng.random() < 0.3:
                ids += rng.integers(0, n_blocks, 5).tolist()
            step[int(c)] = ids
        out.append(step)
    return out


def union(step) -> list:
    return sorted(set(b for ids in step.values() for b in ids))


def field_digests(tr) -> dict:
    """{field: sha256 prefix of its canonical JSON} of a transition's to_dict()
    (recency scores as sorted [block, score] pairs)."""
    d = tr.to_dict()
    d["updated_recency_scores"] = sorted([int(b), float(v)]
                                         for b, v in tr.updated_recency_scores.items())
    return {k: hashlib.sha256(json.dumps(v, separators=(",", ":")).encode()).hexdigest()[:16]
            for k, v in sorted(d.items())}


def run_case(rp, policy, capacity, fraction, seed, steps=30):
    sched = camera_schedule(seed, steps + 1)
    recency = {}
    resident = None
    records = []
    t_total = 0.0
    for k in range(steps):
        cur, nxt = union(sched[k]), union(sched[k + 1])
        given_resident = resident if (resident is None or k % 7 != 3) else resident[: len(resident) // 2]
        kw = dict(current_active_blocks=cur, next_active_blocks=nxt,
                  current_resident_blocks=given_resident,
                  next_camera_ids=sorted(sched[k + 1]), next_camera_blocks=sched[k + 1],
                  previous_recency_scores=recency, recency_decay=0.9)
        t0 = time.perf_counter()
        if policy == "passthrough":
            tr = rp.compute_passthrough_resident_transition(**kw)
        else:
            tr = rp.compute_topc_resident_transition(
                **kw, lambda_weight=0.7, resident_capacity_blocks=capacity,
                balanced_camera_seeds=(policy == "topc_balanced"),
                balanced_seed_fraction=fraction)
        t_total += time.perf_counter() - t0
        records.append(field_digests(tr))
        recency = tr.updated_recency_scores
        resident = list(tr.next_resident_blocks)
    return {"policy": policy, "capacity": capacity, "fraction": fraction, "seed": seed,
            "steps": steps, "records": records, "reference_seconds": t_total}


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", required=True)
    args = ap.parse_args()
    spec = importlib.util.spec_from_file_location(
        "ref_resident_policy",
        Path(args.reference) / "strategies" / "tide_engine" / "resident_policy.py")
    rp = importlib.util.module_from_spec(spec)
    sys.modules[spec.name] = rp
    spec.loader.exec_module(rp)
    cases = [run_case(rp, p, c, f, seed=100 + i) for i, (p, c, f) in enumerate(CASES)]
    (HERE / "planner.json").write_text(json.dumps({"cases": cases}, separators=(",", ":")))
    print("wrote", HERE / "planner.json",
          {c["policy"] + str(c["capacity"]): round(c["reference_seconds"] * 1e3, 1) for c in cases})


if __name__ == "__main__":
    main()
