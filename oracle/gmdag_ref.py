"""The reference's .gmdag loader and layout validator, restated literally — TEST INFRASTRUCTURE ONLY.

Follows projects/environment/src/navi_environment/integration/voxel_dag.py:
  _validate_gmdag_dag_layout  :29-78   (recursive visit with visited / active sets)
  load_gmdag_asset            :193-259 (header checks, payload, trailing bytes)
The C++ reader and validator (navi_b200/csrc/gmdag_io.cpp) are checked against these:
same outcome and same first message on the same bytes.
"""

from __future__ import annotations

import struct
import sys
from pathlib import Path

import numpy as np

_HEADER_STRUCT = struct.Struct("<4sIIffffI")


def validate_layout(nodes: np.ndarray) -> None:
    node_count = int(nodes.shape[0])
    visited: set[int] = set()
    active_stack: set[int] = set()

    def visit(node_index: int) -> None:
        if node_index in visited:
            return
        if node_index in active_stack:
            raise RuntimeError(f"Invalid gmdag DAG layout: cycle detected at node index {node_index}")
        if node_index < 0 or node_index >= node_count:
            raise RuntimeError(f"Invalid gmdag DAG layout: node index out of range: {node_index}")
        active_stack.add(node_index)
        node_word = int(nodes[node_index])
        if (node_word >> 63) == 0:
            mask = (node_word >> 55) & 0xFF
            if mask == 0:
                raise RuntimeError(f"Invalid gmdag DAG layout: internal node {node_index} has empty child mask")
            child_base = node_word & 0xFFFFFFFF
            child_count = int(mask.bit_count())
            if child_base >= node_count:
                raise RuntimeError(
                    "Invalid gmdag DAG layout: child pointer table starts beyond payload " f"at index {child_base}")
            if child_base + child_count > node_count:
                raise RuntimeError(
                    "Invalid gmdag DAG layout: child pointer table exceeds payload bounds " f"for node {node_index}")
            for offset in range(child_count):
                child_index = int(nodes[child_base + offset])
                if child_index < 0 or child_index >= node_count:
                    raise RuntimeError(
                        "Invalid gmdag DAG layout: child reference out of range "
                        f"({child_index}) from node {node_index}")
                visit(child_index)
        active_stack.remove(node_index)
        visited.add(node_index)

    old = sys.getrecursionlimit()
    sys.setrecursionlimit(max(old, 10000))
    try:
        visit(0)
    finally:
        sys.setrecursionlimit(old)


def load_asset(path: Path, *, validate_layout_flag: bool = True):
    """(version, resolution, bbox_min, bbox_max, voxel_size, nodes) or the reference's exception."""
    path = path.expanduser().resolve()
    if not path.exists():
        raise FileNotFoundError(f"gmdag asset does not exist: {path}")
    with path.open("rb") as handle:
        header_bytes = handle.read(_HEADER_STRUCT.size)
        if len(header_bytes) != _HEADER_STRUCT.size:
            raise RuntimeError(f"Invalid gmdag header in {path}")
        magic, version, resolution, bmin_x, bmin_y, bmin_z, voxel_size, node_count = _HEADER_STRUCT.unpack(header_bytes)
        if magic != b"GDAG":
            raise RuntimeError(f"Unsupported gmdag magic in {path}: {magic!r}")
        if version != 1:
            raise RuntimeError(f"Unsupported gmdag version in {path}: {version}")
        if resolution <= 0:
            raise RuntimeError(f"Invalid gmdag resolution in {path}: {resolution}")
        if not np.isfinite(voxel_size) or voxel_size <= 0.0:
            raise RuntimeError(f"Invalid gmdag voxel size in {path}: {voxel_size}")
        if node_count <= 0:
            raise RuntimeError(f"Invalid gmdag node count in {path}: {node_count}")
        if not all(np.isfinite(value) for value in (bmin_x, bmin_y, bmin_z)):
            raise RuntimeError(f"Invalid gmdag bounds in {path}: non-finite bbox_min values detected")
        nodes = np.fromfile(handle, dtype=np.uint64, count=node_count)
        if nodes.shape[0] != node_count:
            raise RuntimeError(
                f"Invalid gmdag node payload in {path}: expected {node_count} nodes, found {nodes.shape[0]}")
        if handle.read(1):
            raise RuntimeError(f"Invalid gmdag payload in {path}: trailing bytes detected")
    if validate_layout_flag:
        validate_layout(nodes)
    bbox_min = (float(bmin_x), float(bmin_y), float(bmin_z))
    extent = float(voxel_size) * int(resolution)
    bbox_max = (bbox_min[0] + extent, bbox_min[1] + extent, bbox_min[2] + extent)
    return int(version), int(resolution), bbox_min, bbox_max, float(voxel_size), np.ascontiguousarray(nodes)
