"""Resident-set planner (strategies/tide_engine/resident_policy.py), vectorized.

`compute_topc_resident_transition` and `compute_passthrough_resident_transition`
return the reference's `ResidentTransition` for the same arguments, field for
field (block lists, policy strings, float scores and the updated recency
scores): set algebra on sorted int64 arrays, the TopC ranking as one
lexicographic argsort of (-score, -recency, -resident, id), and the recency
decay as one float64 array operation (the same double-precision products and
comparisons as the reference's per-entry loop).

Recency scores may be passed as the reference's dict (a dict comes back) or as
a `RecencyScores` mapping, which keeps them in a dense float64 array over the
block ids so that a step costs no per-entry Python work; feed
`transition.updated_recency_scores` back as `previous_recency_scores`.
"""
from __future__ import annotations

from collections.abc import Mapping
from dataclasses import dataclass
from typing import Dict, Iterator, List, Optional, Set, Tuple

import numpy as np

__all__ = ["ResidentTransition", "RecencyScores", "compute_passthrough_resident_transition",
           "compute_topc_resident_transition"]

_DROP_BELOW = 1e-6  # decayed scores at or below this leave the map


@dataclass
class ResidentTransition:
    """Explicit resident-set transition (resident_policy.py:5-81)."""

    current_active_blocks: List[int]
    next_active_blocks: List[int]
    current_resident_blocks: List[int]
    candidate_blocks: List[int]
    next_resident_blocks: List[int]
    keep_resident_blocks: List[int]
    stream_in_blocks: List[int]
    evict_blocks: List[int]
    active_overlap_blocks: List[int]
    active_delta_plus_blocks: List[int]
    active_delta_minus_blocks: List[int]
    next_camera_ids: List[int]
    resident_selection_policy: str = "passthrough_active_set"
    resident_capacity_blocks: int = -1
    requested_resident_capacity_blocks: int = -1
    resident_capacity_bytes: int = -1
    current_resident_source: str = "current_active_fallback"
    resident_lambda_weight: float = 1.0
    resident_recency_decay: float = 1.0
    balanced_seed_fraction: float = 1.0
    topc_cutoff_score: float = 0.0
    next_active_coverage: int = 0
    next_camera_coverage: int = 0
    next_camera_total: int = 0
    enforce_next_active_coverage: bool = False
    updated_recency_scores: Optional[Mapping] = None
    optional_selected_blocks: Optional[List[int]] = None
    camera_seed_blocks: Optional[List[int]] = None

    def __post_init__(self):
        if self.updated_recency_scores is None:
            self.updated_recency_scores = {}
        if self.optional_selected_blocks is None:
            self.optional_selected_blocks = []
        if self.camera_seed_blocks is None:
            self.camera_seed_blocks = []

    def to_dict(self) -> Dict[str, object]:
        return {
            "current_blocks": self.current_active_blocks,
            "next_blocks": self.next_active_blocks,
            "omega_blocks": self.active_overlap_blocks,
            "delta_plus_blocks": self.active_delta_plus_blocks,
            "delta_minus_blocks": self.active_delta_minus_blocks,
            "current_resident_blocks": self.current_resident_blocks,
            "candidate_blocks": self.candidate_blocks,
            "next_resident_blocks": self.next_resident_blocks,
            "keep_resident_blocks": self.keep_resident_blocks,
            "stream_in_blocks": self.stream_in_blocks,
            "evict_blocks": self.evict_blocks,
            "next_camera_ids": self.next_camera_ids,
            "resident_selection_policy": self.resident_selection_policy,
            "resident_capacity_blocks": self.resident_capacity_blocks,
            "requested_resident_capacity_blocks": self.requested_resident_capacity_blocks,
            "resident_capacity_bytes": self.resident_capacity_bytes,
            "current_resident_source": self.current_resident_source,
            "resident_lambda_weight": self.resident_lambda_weight,
            "resident_recency_decay": self.resident_recency_decay,
            "balanced_seed_fraction": self.balanced_seed_fraction,
            "topc_cutoff_score": self.topc_cutoff_score,
            "next_active_coverage": self.next_active_coverage,
            "next_camera_coverage": self.next_camera_coverage,
            "next_camera_total": self.next_camera_total,
            "enforce_next_active_coverage": self.enforce_next_active_coverage,
            "updated_recency_scores": self.updated_recency_scores,
            "optional_selected_blocks": self.optional_selected_blocks,
            "camera_seed_blocks": self.camera_seed_blocks,
        }


class RecencyScores(Mapping):
    """block id -> recency score, stored densely (0 = absent)."""

    def __init__(self, values: Optional[np.ndarray] = None):
        self.values = np.zeros(0, np.float64) if values is None else np.asarray(values, np.float64)

    @classmethod
    def from_dict(cls, scores: Optional[Mapping]) -> "RecencyScores":
        if isinstance(scores, RecencyScores):
            return cls(scores.values.copy())
        if not scores:
            return cls()
        keys = np.fromiter((int(k) for k in scores.keys()), np.int64, len(scores))
        vals = np.fromiter((float(v) for v in scores.values()), np.float64, len(scores))
        if keys.size and keys.min() < 0:
            raise ValueError("RecencyScores: negative block id")
        out = np.zeros(int(keys.max()) + 1 if keys.size else 0, np.float64)
        out[keys] = vals
        return cls(out)

    def lookup(self, ids: np.ndarray) -> np.ndarray:
        out = np.zeros(ids.size, np.float64)
        ok = ids < self.values.size
        out[ok] = self.values[ids[ok]]
        return out

    def __getitem__(self, block_id):
        b = int(block_id)
        if 0 <= b < self.values.size and self.values[b] != 0.0:
            return float(self.values[b])
        raise KeyError(block_id)

    def __iter__(self) -> Iterator[int]:
        return iter(np.nonzero(self.values)[0].tolist())

    def __len__(self) -> int:
        return int(np.count_nonzero(self.values))


def _ids(block_ids) -> np.ndarray:
    """Sorted unique int64 array (resident_policy.py:84-87)."""
    if block_ids is None or len(block_ids) == 0:
        return np.zeros(0, np.int64)
    if isinstance(block_ids, (set, frozenset)):
        arr = np.fromiter(block_ids, np.int64, len(block_ids))
    else:
        arr = np.asarray(block_ids).astype(np.int64, copy=False).reshape(-1)
    return np.unique(arr)


def _member(a: np.ndarray, sorted_b: np.ndarray) -> np.ndarray:
    """a[i] in sorted_b, for a sorted unique `sorted_b`."""
    if sorted_b.size == 0 or a.size == 0:
        return np.zeros(a.size, bool)
    pos = np.minimum(np.searchsorted(sorted_b, a), sorted_b.size - 1)
    return sorted_b[pos] == a


def _list(a: np.ndarray) -> List[int]:
    return a.tolist()


def _updated_recency(previous, accessed: np.ndarray, decay: float):
    """Decay every score by `decay`, drop those at or below 1e-6, set the
    accessed blocks to 1.0 (resident_policy.py:112-123). Returns the mapping
    in the caller's representation and a lookup function."""
    if isinstance(previous, RecencyScores):
        vals = previous.values * float(decay)
        vals[~(vals > _DROP_BELOW)] = 0.0
        if accessed.size and int(accessed[-1]) >= vals.size:
            vals = np.concatenate([vals, np.zeros(int(accessed[-1]) + 1 - vals.size)])
        vals[accessed] = 1.0
        out = RecencyScores(vals)
        return out, out.lookup
    prev = previous or {}
    decay = float(decay)
    updated = _RecencyDict()
    if type(prev) is _RecencyDict and prev.pristine:
        # a dict this function returned and nobody has written to since (int
        # keys, float values already): no per-entry conversions
        dict.update(updated, {b: d for b, s in prev.items() if (d := s * decay) > _DROP_BELOW})
    else:
        dict.update(updated, {int(b): d for b, s in prev.items()
                              if (d := float(s) * decay) > _DROP_BELOW})
    dict.update(updated, dict.fromkeys(accessed.tolist(), 1.0))
    get = updated.get

    def lookup(ids: np.ndarray) -> np.ndarray:
        return np.fromiter((get(b, 0.0) for b in ids.tolist()), np.float64, ids.size)

    return updated, lookup


class _RecencyDict(dict):
    """The recency map a transition returns (a plain dict to its callers):
    int block ids to float scores. Writing to it through any dict method
    clears `pristine`, and the next transition then converts every entry as
    the reference does (resident_policy.py:115-119) instead of trusting the
    types."""

    __slots__ = ("pristine",)

    def __init__(self, *args, **kwargs):
        super().__init__(*args, **kwargs)
        self.pristine = True

    def _touched(self):
        self.pristine = False

    def __setitem__(self, key, value):
        self._touched()
        super().__setitem__(key, value)

    def __delitem__(self, key):
        self._touched()
        super().__delitem__(key)

    def __ior__(self, other):
        self._touched()
        return super().__ior__(other)

    def update(self, *args, **kwargs):
        self._touched()
        super().update(*args, **kwargs)

    def setdefault(self, key, default=None):
        self._touched()
        return super().setdefault(key, default)

    def pop(self, *args):
        self._touched()
        return super().pop(*args)

    def popitem(self):
        self._touched()
        return super().popitem()

    def clear(self):
        self._touched()
        super().clear()


def _normalized_cameras(camera_blocks, allowed: Optional[np.ndarray]) -> List[Tuple[int, np.ndarray]]:
    """(camera, sorted blocks within `allowed`) for cameras in ascending id
    with at least one block (resident_policy.py:126-139)."""
    if not camera_blocks:
        return []
    out = []
    for cam in sorted(camera_blocks):
        blocks = _ids(camera_blocks.get(cam, []))
        if allowed is not None:
            blocks = blocks[_member(blocks, allowed)]
        if blocks.size:
            out.append((int(cam), blocks))
    return out


def _camera_coverage(cams: List[Tuple[int, np.ndarray]], selected: np.ndarray) -> Tuple[int, int]:
    """(cameras with a selected block, cameras) over the cameras normalized to
    the next active set (resident_policy.py:142-155)."""
    covered = sum(1 for _, blocks in cams if _member(blocks, selected).any())
    return covered, len(cams)


def _balanced_seed_capacity(cams: List[Tuple[int, np.ndarray]], capacity: int,
                            fraction: float) -> int:
    """resident_policy.py:219-238 (cams normalized to the candidates)."""
    if capacity <= 0:
        return 0
    fraction = max(0.0, min(1.0, float(fraction)))
    if fraction >= 1.0:
        return int(capacity)
    if fraction <= 0.0:
        return 0
    n_cams = len(cams)
    quota = int(capacity * fraction)
    if quota <= 0:
        quota = 1
    if n_cams > 0:
        quota = max(quota, min(int(capacity), n_cams))
    return min(int(capacity), quota)


def _balanced_seeds(cams: List[Tuple[int, np.ndarray]], score_of, resident: np.ndarray,
                    capacity: int) -> List[int]:
    """Round robin over the cameras (ascending id, normalized to the
    candidates), each taking its best not-yet-selected block by (-score,
    -cameras seeing it, -resident, id) (resident_policy.py:158-216)."""
    if capacity <= 0 or not cams:
        return []
    every = np.concatenate([b for _, b in cams])
    uniq, freq = np.unique(every, return_counts=True)
    ordered = []
    for _, blocks in cams:
        f = freq[np.searchsorted(uniq, blocks)]
        s = score_of(blocks)
        r = _member(blocks, resident).astype(np.int64)
        ordered.append(blocks[np.lexsort((blocks, -r, -f, -s))].tolist())
    positions = [0] * len(ordered)
    selected: List[int] = []
    taken: Set[int] = set()
    while len(selected) < capacity:
        progress = False
        for i, blocks in enumerate(ordered):
            p = positions[i]
            while p < len(blocks) and blocks[p] in taken:
                p += 1
            if p >= len(blocks):
                positions[i] = p
                continue
            b = blocks[p]
            positions[i] = p + 1
            selected.append(b)
            taken.add(b)
            progress = True
            if len(selected) >= capacity:
                break
        if not progress:
            break
    return selected


def _resolve_current_resident(current_active: np.ndarray, current_resident_blocks,
                              scored: bool) -> Tuple[np.ndarray, str]:
    """resident_policy.py:90-109."""
    if current_resident_blocks:
        requested = _ids(current_resident_blocks)
        if np.array_equal(requested, current_active):
            return requested, "expected_resident_match"
        if scored:
            return requested, "loaded_resident_state"
    return current_active, "current_active_fallback"


def _active_deltas(current_active: np.ndarray, next_active: np.ndarray):
    return (np.intersect1d(current_active, next_active, assume_unique=True),
            np.setdiff1d(next_active, current_active, assume_unique=True),
            np.setdiff1d(current_active, next_active, assume_unique=True))


def compute_passthrough_resident_transition(
        current_active_blocks: List[int], next_active_blocks: List[int],
        current_resident_blocks: Optional[List[int]] = None,
        next_camera_ids: Optional[List[int]] = None,
        next_camera_blocks: Optional[Dict[int, List[int]]] = None,
        previous_recency_scores=None, recency_decay: float = 0.95) -> ResidentTransition:
    """The next resident set is the next active set (resident_policy.py:241-310)."""
    cur_act = _ids(current_active_blocks)
    nxt_act = _ids(next_active_blocks)
    cur_res, source = _resolve_current_resident(cur_act, current_resident_blocks, scored=False)
    nxt_res = nxt_act
    omega, plus, minus = _active_deltas(cur_act, nxt_act)
    updated, _ = _updated_recency(previous_recency_scores, cur_act, recency_decay)
    covered, total = _camera_coverage(_normalized_cameras(next_camera_blocks, nxt_act), nxt_res)
    return ResidentTransition(
        current_active_blocks=_list(cur_act), next_active_blocks=_list(nxt_act),
        current_resident_blocks=_list(cur_res),
        candidate_blocks=_list(np.union1d(cur_res, nxt_act)),
        next_resident_blocks=_list(nxt_res),
        keep_resident_blocks=_list(np.intersect1d(cur_res, nxt_res, assume_unique=True)),
        stream_in_blocks=_list(np.setdiff1d(nxt_res, cur_res, assume_unique=True)),
        evict_blocks=_list(np.setdiff1d(cur_res, nxt_res, assume_unique=True)),
        active_overlap_blocks=_list(omega), active_delta_plus_blocks=_list(plus),
        active_delta_minus_blocks=_list(minus), next_camera_ids=list(next_camera_ids or []),
        current_resident_source=source, resident_lambda_weight=1.0,
        resident_recency_decay=recency_decay, topc_cutoff_score=1.0 if nxt_res.size else 0.0,
        next_active_coverage=int(nxt_act.size), next_camera_coverage=covered,
        next_camera_total=total, updated_recency_scores=updated)


def compute_topc_resident_transition(
        current_active_blocks: List[int], next_active_blocks: List[int],
        current_resident_blocks: Optional[List[int]] = None,
        next_camera_ids: Optional[List[int]] = None,
        next_camera_blocks: Optional[Dict[int, List[int]]] = None,
        previous_recency_scores=None, lambda_weight: float = 0.7, recency_decay: float = 0.95,
        resident_capacity_blocks: int = -1, balanced_camera_seeds: bool = False,
        balanced_seed_fraction: float = 1.0) -> ResidentTransition:
    """Keep the C best candidates (current resident + next active) by
    lambda * [in next active] + (1 - lambda) * recency, optionally seeding
    each next camera round robin first (resident_policy.py:313-442)."""
    cur_act = _ids(current_active_blocks)
    nxt_act = _ids(next_active_blocks)
    cur_res, source = _resolve_current_resident(cur_act, current_resident_blocks, scored=True)
    updated, recency_of = _updated_recency(previous_recency_scores, cur_act, recency_decay)
    cand = np.union1d(cur_res, nxt_act)
    requested = int(resident_capacity_blocks)
    capacity = cand.size if requested < 0 else max(0, requested)
    capacity = min(capacity, int(cand.size))

    lam = float(lambda_weight)
    useful = _member(cand, nxt_act)
    rec = recency_of(cand)
    scores = lam * useful.astype(np.float64) + (1.0 - lam) * rec
    resident = _member(cand, cur_res).astype(np.int64)
    cams = _normalized_cameras(next_camera_blocks, nxt_act)

    def score_of(blocks: np.ndarray) -> np.ndarray:
        return scores[np.searchsorted(cand, blocks)]

    seeds: List[int] = []
    if balanced_camera_seeds and capacity > 0:
        seed_cap = _balanced_seed_capacity(cams, capacity, balanced_seed_fraction)
        seeds = _balanced_seeds(cams, score_of, cur_res, seed_cap)
    remaining = max(0, capacity - len(seeds))
    selected = np.asarray(seeds, np.int64)
    if remaining > 0:
        ranked = cand[np.lexsort((cand, -resident, -rec, -scores))]
        if seeds:
            ranked = ranked[~_member(ranked, np.unique(selected))]
        selected = np.concatenate([selected, ranked[:remaining]])
    selected = selected[:capacity]
    nxt_res = np.unique(selected)
    omega, plus, minus = _active_deltas(cur_act, nxt_act)
    cutoff = float(score_of(nxt_res).min()) if nxt_res.size else 0.0
    covered, total = _camera_coverage(cams, nxt_res)
    return ResidentTransition(
        current_active_blocks=_list(cur_act), next_active_blocks=_list(nxt_act),
        current_resident_blocks=_list(cur_res), candidate_blocks=_list(cand),
        next_resident_blocks=_list(nxt_res),
        keep_resident_blocks=_list(np.intersect1d(cur_res, nxt_res, assume_unique=True)),
        stream_in_blocks=_list(np.setdiff1d(nxt_res, cur_res, assume_unique=True)),
        evict_blocks=_list(np.setdiff1d(cur_res, nxt_res, assume_unique=True)),
        active_overlap_blocks=_list(omega), active_delta_plus_blocks=_list(plus),
        active_delta_minus_blocks=_list(minus), next_camera_ids=list(next_camera_ids or []),
        resident_selection_policy="topc_balanced" if balanced_camera_seeds else "topc_strict",
        resident_capacity_blocks=int(capacity), requested_resident_capacity_blocks=requested,
        current_resident_source=source, resident_lambda_weight=lam,
        resident_recency_decay=float(recency_decay),
        balanced_seed_fraction=float(balanced_seed_fraction) if balanced_camera_seeds else 0.0,
        topc_cutoff_score=cutoff,
        next_active_coverage=int(np.intersect1d(nxt_act, nxt_res, assume_unique=True).size),
        next_camera_coverage=covered, next_camera_total=total, enforce_next_active_coverage=False,
        updated_recency_scores=updated,
        optional_selected_blocks=_list(np.setdiff1d(nxt_res, nxt_act, assume_unique=True)),
        camera_seed_blocks=list(seeds))
