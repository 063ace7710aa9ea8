"""Local spherical ray fan (the host-built table the fused generator rotates).

Restates ``build_spherical_ray_directions``
(projects/environment/src/navi_environment/backends/sdfdag_backend.py:205-221):
azimuth = linspace(0, 2pi, Az, endpoint=False), elevation = linspace(+pi/2,
-pi/2, El, endpoint=True), both float32; flat index az * El + el; direction
(cos el * sin az, sin el, -cos el * cos az), computed with numpy float32 so the
table is bit-identical to the reference's.  Built once per fan shape, on the
host, as the reference does at backend init (sdfdag_backend.py:749).
"""

from __future__ import annotations

import math

import numpy as np

__all__ = ["build_spherical_ray_directions"]


def build_spherical_ray_directions(azimuth_bins: int, elevation_bins: int) -> np.ndarray:
    az = np.linspace(0.0, 2.0 * math.pi, azimuth_bins, endpoint=False, dtype=np.float32)
    el = np.linspace(math.pi / 2.0, -math.pi / 2.0, elevation_bins, endpoint=True, dtype=np.float32)
    az_grid, el_grid = np.meshgrid(az, el, indexing="ij")
    az_flat = az_grid.reshape(-1)
    el_flat = el_grid.reshape(-1)
    cos_el = np.cos(el_flat)
    return np.stack(
        [cos_el * np.sin(az_flat), np.sin(el_flat), -cos_el * np.cos(az_flat)],
        axis=-1,
    ).astype(np.float32)
