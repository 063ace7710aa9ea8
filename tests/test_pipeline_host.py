"""Host-side logic of navi_b200.pipeline: chunk bounds and argument checks (no GPU needed)."""

from __future__ import annotations

import pytest
import torch

from navi_b200 import pipeline


@pytest.mark.parametrize("n,chunks", [(0, 4), (1, 4), (5, 4), (8, 4), (9, 4), (1000, 7), (3, 1000), (12, 1)])
def test_chunk_bounds_cover_every_index_once(n, chunks):
    b = pipeline._bounds(n, chunks)
    covered = [i for lo, hi in b for i in range(lo, hi)]
    assert covered == list(range(n))
    assert all(hi > lo for lo, hi in b)
    assert len(b) <= max(1, chunks)


def test_run_chunks_with_nothing_to_do_is_a_no_op():
    pipeline.run_chunks([], torch.device("cpu"))


def test_host_casts_reject_device_or_strided_tensors():
    class _Pool:  # never reached: the checks come first
        device = torch.device("cpu")

    h = torch.zeros((4, 3))
    strided = torch.zeros((4, 6))[:, ::2]
    out = torch.zeros(4)
    sem = torch.zeros(4, dtype=torch.int32)
    kw = dict(max_steps=8, max_distance=1.0, bbox_min=[0, 0, 0], bbox_max=[1, 1, 1])
    with pytest.raises(RuntimeError, match="origins must be a contiguous host tensor"):
        pipeline.cast_rays_host(_Pool(), strided, h, out, sem, **kw)
    with pytest.raises(RuntimeError, match="out_semantics must be a contiguous host tensor"):
        pipeline.cast_rays_host(_Pool(), h, h, out, torch.zeros(8, dtype=torch.int32)[::2], **kw)
    with pytest.raises(RuntimeError, match="poses must be a contiguous host tensor"):
        pipeline.cast_fan_host(None, torch.zeros((2, 16))[:, ::2], torch.zeros((3, 3)), out, sem, max_steps=8,
                               max_distance=1.0)
