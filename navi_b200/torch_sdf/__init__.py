"""torch_sdf surface of the B200 tracer (projects/torch-sdf/torch_sdf/__init__.py).

``cast_rays`` is the drop-in batched cast; ``load_gmdag`` / ``cast_rays_ex`` /
``cast_fan`` are the additions (device upload with a node pool, hit epsilon and
step counts, pose-fused fans).
"""

from ..tracer import NodePool, SceneSet, cast_fan, cast_rays_ex, load_gmdag, make_poses
from .backend import cast_rays

__all__ = ["cast_rays", "cast_rays_ex", "cast_fan", "load_gmdag", "make_poses", "NodePool", "SceneSet"]
