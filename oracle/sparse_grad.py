"""CPU restatement of the touched-only gradient accumulation -- TEST
INFRASTRUCTURE ONLY (see oracle/__init__.py).

Follows strategies/tide_engine/engine.py:
  :1801-1807  touched rows = ascending union of the cameras' local filters
  :1815       visibility = local_to_global[touched]
  :1816-1823  compact gradients zero-filled, [touched, W] per component
  :2434-2471  per camera: idx = searchsorted(touched, filter); every component
              gets scatter_add_ of the camera's gradient rows at idx (the SH
              gradient [n, 48] splits into dc = [:, :3], rest = [:, 3:48])

Pinned: tests/test_oracle_golden.py runs these very torch operations
(torch.searchsorted, Tensor.scatter_add_, CPU) on seeded inputs and requires
bit-equal results.
"""
from __future__ import annotations

from typing import Dict, Optional, Sequence

import numpy as np

WIDTHS = {"xyz": 3, "opacity": 1, "scaling": 3, "rotation": 4, "features_dc": 3,
          "features_rest": 45}


def touched_rows(filters: Sequence[np.ndarray], num_rows: int) -> np.ndarray:
    """engine.py:1803-1807 (mask, scatter_ True, nonzero)."""
    mask = np.zeros(num_rows, bool)
    for f in filters:
        if f is not None and len(f):
            mask[np.asarray(f, np.int64)] = True
    return np.nonzero(mask)[0].astype(np.int64)


def zero_components(n: int) -> Dict[str, np.ndarray]:
    return {name: np.zeros((n, w), np.float32) for name, w in WIDTHS.items()}


def accumulate(acc: Dict[str, np.ndarray], touched: np.ndarray, filt: np.ndarray,
               xyz: np.ndarray, opacity: np.ndarray, scaling: np.ndarray, rotation: np.ndarray,
               shs: Optional[np.ndarray]) -> None:
    """engine.py:2434-2471 for one camera: fp32 additions in row order."""
    idx = np.searchsorted(touched, np.asarray(filt, np.int64))
    srcs = {"xyz": xyz, "opacity": opacity, "scaling": scaling, "rotation": rotation}
    if shs is not None:
        srcs["features_dc"] = shs[:, :3]
        srcs["features_rest"] = shs[:, 3:48]
    for name, src in srcs.items():
        np.add.at(acc[name], idx, np.asarray(src, np.float32))
