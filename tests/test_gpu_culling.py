"""GPU: BlockCuller (tgs_block_spheres + tgs_frustum_cull) against the
reference FrustumCuller's outputs (tests/golden/culling.npz) and, at the
configs[3] scene size (61,036 blocks x 16 cameras), against the CPU oracle;
all comparisons exact (index lists and float32 spheres)."""
import numpy as np
import pytest
import torch
from pathlib import Path

from oracle import culling as oc

pytestmark = [pytest.mark.gpu, pytest.mark.filterwarnings("ignore:Suspicious plane orientations")]

G = np.load(Path(__file__).resolve().parent / "golden" / "culling.npz")


def _lists(key):
    ids, off = G[key + "_ids"], G[key + "_off"]
    return [ids[off[i]:off[i + 1]].tolist() for i in range(off.size - 1)]


def test_culler_matches_reference_outputs():
    from tidegs_b200 import BlockCuller

    cu = BlockCuller(G["bounds"], verbose=False)
    np.testing.assert_array_equal(cu.block_centers.cpu().numpy(), G["centers"])
    np.testing.assert_array_equal(cu.block_radii.cpu().numpy(), G["radii"])
    cams = list(zip(G["views"], G["projs"]))
    vis = _lists("visible")
    for c, (e, (v, p)) in enumerate(zip(G["eyes"], cams)):
        assert cu.cull(e, v, p) == vis[c]
        assert cu.cull_subset(e, v, p, G["subset"]) == _lists("subset_visible")[c]
    assert cu.cull_cameras(cams) == vis
    assert cu.cull_cameras(None, planes=G["planes"]) == vis
    assert cu.cull_cameras([]) == []
    ids, counts = cu.cull_cameras(cams, as_tensors=True)
    assert counts.tolist() == [len(x) for x in vis]
    assert ids[3, :counts[3]].tolist() == vis[3]
    # bounds update from a device tensor (the write-back bounds stay on the GPU)
    assert cu.update_block_bounds(G["update_ids"], torch.from_numpy(G["new_bounds"]).cuda()) == 300
    np.testing.assert_array_equal(cu.block_centers.cpu().numpy(), G["centers_updated"])
    np.testing.assert_array_equal(cu.block_radii.cpu().numpy(), G["radii_updated"])
    assert cu.cull_cameras(cams) == _lists("updated_visible")
    order = cu.get_visibility_order(_lists("updated_visible")[0], G["eyes"][0])
    assert order == G["order0"].tolist()
    assert cu.cull_subset(G["eyes"][0], *cams[0], set()) == []
    with pytest.raises(ValueError):
        cu.cull_subset(G["eyes"][0], *cams[0], [0, len(G["bounds"])])
    with pytest.raises(NotImplementedError):
        cu.cull(G["eyes"][0], *cams[0], use_6plane=False)


def test_culler_full_scene_against_oracle():
    """61,036 blocks of a MatrixCity-sized scene, 16 cameras in one launch."""
    import importlib.util

    from tidegs_b200 import BlockCuller

    spec = importlib.util.spec_from_file_location(
        "culling_golden", Path(__file__).resolve().parent / "golden" / "make_culling_golden.py")
    mk = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mk)
    rng, bounds = mk.scene(seed=11, n_blocks=61036)
    views, projs, eyes = mk.cameras(rng, 16)
    cu = BlockCuller(torch.from_numpy(bounds).cuda(), verbose=False)
    centers, radii = oc.spheres(bounds)
    np.testing.assert_array_equal(cu.block_centers.cpu().numpy(), centers)
    np.testing.assert_array_equal(cu.block_radii.cpu().numpy(), radii)
    got = cu.cull_cameras(list(zip(views, projs)))
    total = 0
    for c in range(16):
        want = oc.visible(centers, radii, oc.planes(views[c], projs[c]))
        assert got[c] == want.tolist(), c
        total += len(want)
    assert 0.1 < total / (16 * 61036) < 0.6
