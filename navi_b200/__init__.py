"""navi_b200: B200-native batched sphere tracing of spherical ray fans through .gmdag DAGs.

Subpackages and modules:
- navi_b200.torch_sdf  drop-in ``torch_sdf`` API (cast_rays) plus extensions
- navi_b200.tracer     node pools, scene sets, explicit and pose-fused casts
- navi_b200.gmdag      .gmdag load / validate / write / compile
- navi_b200.scenes     seeded synthetic scenes and poses of the benchmark configs
- navi_b200.fan        local spherical fan table
- navi_b200.build      builds the native libraries in-tree
"""

__version__ = "0.1.0"
