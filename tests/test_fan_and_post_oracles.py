"""Direction, rotation and post-processing cases of the reference's environment tests.

- the local fan (navi_b200/fan.py) against the cardinal-direction, unit-norm, pole and
  index-mapping cases of projects/environment/tests/unit/test_ray_direction_oracle.py:30-137;
- the oracle's yaw rotation (oracle/oracle.py rotate_fan, the formula the fan kernel is
  checked against bit for bit on the GPU) against the cases of test_yaw_rotation_oracle.py:25-113;
- the torch restatement of the backend post-processing (oracle/postprocess_ref.py, which the
  fused observation epilogue is checked against on the GPU) against the finite-distance cases of
  test_postprocessing_oracle.py:45-135.  That test's own helper differs from the backend it
  describes for NaN and for distances above max_distance (it marks them invalid and clamps them
  to max_distance; the backend, sdfdag_backend.py:436-440, marks only non-finite values invalid
  and clamps with clamp(0, max)); the epilogue follows the backend, so only the cases on which
  both agree are mirrored here.
"""

from __future__ import annotations

import math

import numpy as np
import pytest
import torch

from navi_b200.fan import build_spherical_ray_directions
from oracle import oracle as O
from oracle.postprocess_ref import postprocess


def _dir_at(dirs, az_idx, el_idx, el_bins):
    return dirs[az_idx * el_bins + el_idx]


class TestCardinalDirections:
    AZ, EL = 256, 48

    def setup_method(self):
        self.dirs = build_spherical_ray_directions(self.AZ, self.EL)

    @pytest.mark.parametrize("az_frac,expected", [(0, [0.0, 0.0, -1.0]), (1, [1.0, 0.0, 0.0]),
                                                  (2, [0.0, 0.0, 1.0]), (3, [-1.0, 0.0, 0.0])])
    def test_horizontal_quarters(self, az_frac, expected):
        d = _dir_at(self.dirs, az_frac * self.AZ // 4, self.EL // 2, self.EL)
        np.testing.assert_allclose(d, expected, atol=0.07)

    def test_poles(self):
        np.testing.assert_allclose(_dir_at(self.dirs, 0, 0, self.EL), [0.0, 1.0, 0.0], atol=1e-5)
        np.testing.assert_allclose(_dir_at(self.dirs, 0, self.EL - 1, self.EL), [0.0, -1.0, 0.0], atol=1e-5)
        top = np.array([_dir_at(self.dirs, a, 0, self.EL) for a in range(self.AZ)])
        bot = np.array([_dir_at(self.dirs, a, self.EL - 1, self.EL) for a in range(self.AZ)])
        assert np.all(np.ptp(top, axis=0) < 1e-5) and np.all(np.ptp(bot, axis=0) < 1e-5)


@pytest.mark.parametrize("az,el", [(8, 3), (64, 16), (256, 48), (128, 24), (1024, 256), (48, 12)])
def test_unit_norms(az, el):
    dirs = build_spherical_ray_directions(az, el)
    assert dirs.dtype == np.float32 and dirs.shape == (az * el, 3)
    np.testing.assert_allclose(np.linalg.norm(dirs, axis=-1), 1.0, atol=1e-6)


def test_index_mapping():
    az, el = 16, 5
    dirs = build_spherical_ray_directions(az, el)
    grid = dirs.reshape(az, el, 3)
    for a in range(az):
        for e in range(el):
            assert np.array_equal(grid[a, e], dirs[a * el + e])


FORWARD = np.array([[0.0, 0.0, -1.0]], np.float32)
MULTI = np.array([[0.0, 0.0, -1.0], [1.0, 0.0, 0.0], [0.0, 1.0, 0.0], [0.0, 0.0, 1.0]], np.float32)


def _rot(local, yaw):
    return O.rotate_fan(local, np.float32(math.cos(yaw)), np.float32(math.sin(yaw)))[0]


def test_yaw_identity():
    np.testing.assert_allclose(_rot(FORWARD, 0.0), FORWARD, atol=1e-7)
    np.testing.assert_allclose(_rot(MULTI, 0.0), MULTI, atol=1e-7)


def test_yaw_quarter_and_half_turns():
    np.testing.assert_allclose(_rot(FORWARD, math.pi / 2), [[-1.0, 0.0, 0.0]], atol=1e-6)
    np.testing.assert_allclose(_rot(np.array([[1.0, 0.0, 0.0]], np.float32), math.pi / 2), [[0.0, 0.0, -1.0]],
                               atol=1e-6)
    np.testing.assert_allclose(_rot(FORWARD, math.pi), [[0.0, 0.0, 1.0]], atol=1e-6)


@pytest.mark.parametrize("yaw", [0.0, 0.3, 1.0, math.pi / 2, math.pi, 4.0, 2 * math.pi - 0.01])
def test_yaw_preserves_y_and_norm(yaw):
    local = build_spherical_ray_directions(32, 9)
    world = _rot(local, yaw)
    assert np.array_equal(world[:, 1], local[:, 1])
    np.testing.assert_allclose(np.linalg.norm(world, axis=-1), 1.0, atol=1e-6)


def _post(dist, az, el, max_distance):
    d = torch.tensor(dist, dtype=torch.float32).reshape(1, -1)
    s = torch.ones_like(d, dtype=torch.int32)
    obs, stats = postprocess(d, s, az_bins=az, el_bins=el, max_distance=max_distance, structure_band_min_distance=1.0,
                             structure_band_max_distance=2.0, proximity_distance_threshold=0.5)
    return obs[0, 0], obs[0, 2]


def test_post_known_depths_and_validity():
    depth, valid = _post([0.5, 1.0, 5.0, 100.0, float("inf")], 5, 1, 100.0)
    den = math.log1p(100.0)
    for i, want in enumerate([math.log1p(0.5) / den, math.log1p(1.0) / den, math.log1p(5.0) / den, 1.0, 1.0]):
        assert abs(float(depth[i, 0]) - want) < 1e-6
    assert [bool(v) for v in valid[:, 0]] == [True, True, True, True, False]
    depth, valid = _post([0.0], 1, 1, 100.0)
    assert float(depth[0, 0]) == 0.0 and bool(valid[0, 0])
    depth, valid = _post([100.0, 15.0], 2, 1, 100.0)
    assert bool(valid[0, 0]) and bool(valid[1, 0])


def test_post_flat_to_grid_order():
    az, el = 8, 4
    n = az * el
    depth, _ = _post(list(range(n)), az, el, float(n + 1))
    den = math.log1p(float(n + 1))
    for a in range(az):
        for e in range(el):
            assert abs(float(depth[a, e]) - math.log1p(a * el + e) / den) < 1e-6
