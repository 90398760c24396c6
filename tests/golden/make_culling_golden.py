"""Generates tests/golden/culling.npz by running the reference's
FrustumCuller (storage/gaussian_block.py, loaded by file path) on a seeded
scene: block spheres, each camera's planes, full culls, a subset cull, a
cull after update_block_bounds and a front-to-back order.

    python tests/golden/make_culling_golden.py --reference <TideGS checkout>
"""
from __future__ import annotations

import argparse
import importlib.util
import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent


def scene(seed: int = 7, n_blocks: int = 4000):
    rng = np.random.default_rng(seed)
    centers = rng.uniform(-100.0, 100.0, (n_blocks, 3))
    half = rng.uniform(1.0, 6.0, (n_blocks, 3))
    bounds = np.concatenate([centers - half, centers + half], axis=1).astype(np.float32)
    return rng, bounds


def look_at(eye, target, up=(0.0, 0.0, 1.0)) -> np.ndarray:
    """OpenGL view matrix (camera looks down -Z)."""
    eye, target, up = (np.asarray(v, dtype=np.float64) for v in (eye, target, up))
    f = target - eye
    f /= np.linalg.norm(f)
    s = np.cross(f, up)
    s /= np.linalg.norm(s)
    u = np.cross(s, f)
    m = np.eye(4)
    m[0, :3], m[1, :3], m[2, :3] = s, u, -f
    m[:3, 3] = -m[:3, :3] @ eye
    return m


def perspective(fovy_deg: float, aspect: float, near: float, far: float) -> np.ndarray:
    t = 1.0 / np.tan(np.radians(fovy_deg) / 2.0)
    m = np.zeros((4, 4))
    m[0, 0], m[1, 1] = t / aspect, t
    m[2, 2], m[2, 3] = (far + near) / (near - far), 2.0 * far * near / (near - far)
    m[3, 2] = -1.0
    return m


def cameras(rng, n: int):
    views, projs, eyes = [], [], []
    for _ in range(n):
        ang = rng.uniform(0, 2 * np.pi)
        eye = np.array([110 * np.cos(ang), 110 * np.sin(ang), rng.uniform(10, 60)])
        target = rng.uniform(-60, 60, 3)
        views.append(look_at(eye, target))
        projs.append(perspective(rng.uniform(25, 45), 16 / 9, 0.5, 260.0))
        eyes.append(eye)
    return np.stack(views), np.stack(projs), np.stack(eyes)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", required=True)
    args = ap.parse_args()
    spec = importlib.util.spec_from_file_location(
        "ref_gaussian_block", Path(args.reference) / "storage" / "gaussian_block.py")
    gb = importlib.util.module_from_spec(spec)
    sys.modules[spec.name] = gb
    spec.loader.exec_module(gb)

    rng, bounds = scene()
    views, projs, eyes = cameras(rng, 8)
    culler = gb.FrustumCuller(bounds, verbose=False)
    out = {"bounds": bounds, "views": views, "projs": projs, "eyes": eyes,
           "centers": culler.block_centers.astype(np.float32),
           "radii": culler.block_radii.astype(np.float32)}
    out["planes"] = np.stack([gb.extract_frustum_planes(v, p) for v, p in zip(views, projs)])
    vis = [np.asarray(culler.cull(e, v, p), np.int64) for e, v, p in zip(eyes, views, projs)]
    subset = rng.choice(bounds.shape[0], 1500, replace=True)
    sub = [np.asarray(culler.cull_subset(e, v, p, subset), np.int64)
           for e, v, p in zip(eyes, views, projs)]
    upd_ids = rng.choice(bounds.shape[0], 300, replace=False)
    c = rng.uniform(-100.0, 100.0, (300, 3))
    h = rng.uniform(0.5, 9.0, (300, 3))
    new_bounds = np.concatenate([c - h, c + h], axis=1).astype(np.float32)
    culler.update_block_bounds(upd_ids, new_bounds)
    vis2 = [np.asarray(culler.cull(e, v, p), np.int64) for e, v, p in zip(eyes, views, projs)]
    order = np.asarray(culler.get_visibility_order(vis2[0].tolist(), eyes[0]), np.int64)

    def pack(lists, key):
        out[key + "_ids"] = np.concatenate(lists) if lists else np.zeros(0, np.int64)
        out[key + "_off"] = np.concatenate([[0], np.cumsum([len(x) for x in lists])]).astype(np.int64)

    pack(vis, "visible")
    pack(sub, "subset_visible")
    pack(vis2, "updated_visible")
    out.update({"subset": subset.astype(np.int64), "update_ids": upd_ids.astype(np.int64),
                "new_bounds": new_bounds, "order0": order,
                "centers_updated": culler.block_centers.astype(np.float32),
                "radii_updated": culler.block_radii.astype(np.float32)})
    np.savez_compressed(HERE / "culling.npz", **out)
    print("wrote", HERE / "culling.npz", [len(x) for x in vis])


if __name__ == "__main__":
    main()
