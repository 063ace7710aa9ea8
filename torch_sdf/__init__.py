"""Import name of the reference package, bound to navi_b200's implementation.

Code written against the reference (``import torch_sdf``,
``torch_sdf.cast_rays(...)``, ``import torch_sdf.backend``) runs unchanged;
``torch_sdf.backend`` is the very module object ``navi_b200.torch_sdf.backend``
so that attributes patched on one are seen by the other.
"""

import sys

from navi_b200.torch_sdf import (  # noqa: F401
    NodePool,
    SceneSet,
    cast_fan,
    cast_rays,
    cast_rays_ex,
    load_gmdag,
    make_poses,
)
from navi_b200.torch_sdf import backend as _backend

sys.modules[__name__ + ".backend"] = _backend
backend = _backend

__all__ = ["cast_rays", "cast_rays_ex", "cast_fan", "load_gmdag", "make_poses", "NodePool", "SceneSet"]
