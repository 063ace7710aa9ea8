"""Contract tests of the drop-in torch_sdf API, mirroring the reference's
projects/torch-sdf/tests/test_sphere_tracing.py:294-680: the native backend is
replaced by a fake and the exact error texts are checked.  No GPU needed."""

from __future__ import annotations

import pytest
import torch

import torch_sdf
import torch_sdf.backend as backend_module


class _FakeTensor:
    def __init__(self, *, shape, dtype, is_cuda=True, contiguous=True):
        self.shape = shape
        self.dtype = dtype
        self.is_cuda = is_cuda
        self._contiguous = contiguous

    def dim(self):
        return len(self.shape)

    def size(self, idx):
        return self.shape[idx]

    def is_contiguous(self):
        return self._contiguous


def _fake_cast_inputs(**overrides):
    values = {
        "dag": _FakeTensor(shape=(8,), dtype=torch.int64),
        "origins": _FakeTensor(shape=(2, 3, 3), dtype=torch.float32),
        "dirs": _FakeTensor(shape=(2, 3, 3), dtype=torch.float32),
        "out_distances": _FakeTensor(shape=(2, 3), dtype=torch.float32),
        "out_semantics": _FakeTensor(shape=(2, 3), dtype=torch.int32),
    }
    values.update(overrides)
    return values["dag"], values["origins"], values["dirs"], values["out_distances"], values["out_semantics"]


@pytest.fixture
def fake_cuda(monkeypatch):
    monkeypatch.setattr(backend_module, "HAS_CUDA_BACKEND", True)
    monkeypatch.setattr(backend_module, "torch_sdf_backend", object())
    monkeypatch.setattr(torch.cuda, "is_available", lambda: True)


def test_package_exposes_reference_entry_points():
    assert torch_sdf.cast_rays is backend_module.cast_rays
    assert torch_sdf.backend is backend_module
    import navi_b200.torch_sdf.backend as inner

    assert inner is backend_module


def test_backend_accepts_explicit_max_distance(monkeypatch):
    captured = {}

    class _FakeBackend:
        def cast_rays(self, *args):
            captured["argc"] = len(args)
            captured["max_distance"] = args[6]

    monkeypatch.setattr(backend_module, "HAS_CUDA_BACKEND", True)
    monkeypatch.setattr(backend_module, "torch_sdf_backend", _FakeBackend())
    monkeypatch.setattr(torch.cuda, "is_available", lambda: True)
    dag, o, d, od, os_ = _fake_cast_inputs(origins=_FakeTensor(shape=(1, 1, 3), dtype=torch.float32),
                                           dirs=_FakeTensor(shape=(1, 1, 3), dtype=torch.float32),
                                           out_distances=_FakeTensor(shape=(1, 1), dtype=torch.float32),
                                           out_semantics=_FakeTensor(shape=(1, 1), dtype=torch.int32))
    backend_module.cast_rays(dag, o, d, od, os_, 64, 17.5, [0, 0, 0], [1, 1, 1], 128)
    assert captured["argc"] == 11
    assert captured["max_distance"] == 17.5


def test_extensions_route_to_cast_rays_ex(monkeypatch):
    captured = {}

    class _FakeBackend:
        def cast_rays(self, *args):
            raise AssertionError("default call used for an extended cast")

        def cast_rays_ex(self, *args):
            captured["args"] = args

    monkeypatch.setattr(backend_module, "HAS_CUDA_BACKEND", True)
    monkeypatch.setattr(backend_module, "torch_sdf_backend", _FakeBackend())
    monkeypatch.setattr(torch.cuda, "is_available", lambda: True)
    backend_module.cast_rays(*_fake_cast_inputs(), 64, 30.0, [0, 0, 0], [1, 1, 1], 128,
                             skip_direction_validation=True, hit_epsilon=1e-4)
    assert captured["args"][11] == 1e-4
    assert captured["args"][12] is None


def test_validate_direction_norms_rejects_unnormalized_vectors():
    with pytest.raises(RuntimeError, match="normalized within tolerance"):
        backend_module._validate_direction_norms(torch.tensor([[[1.2, 0.0, 0.0]]]))


def test_validate_direction_norms_rejects_nonfinite_vectors():
    with pytest.raises(RuntimeError, match="finite direction vectors"):
        backend_module._validate_direction_norms(torch.tensor([[[float("nan"), 0.0, 1.0]]]))


def test_validate_direction_norms_accepts_vectors_within_tolerance():
    backend_module._validate_direction_norms(torch.tensor([[[1.0, 5e-5, 0.0]]]))


@pytest.mark.parametrize(
    "overrides,args,match",
    [
        ({"dirs": _FakeTensor(shape=(2, 3, 3), dtype=torch.float32, contiguous=False)}, None, "dirs must be contiguous"),
        ({"dag": _FakeTensor(shape=(8,), dtype=torch.int64, is_cuda=False)}, None, "dag_tensor must be on CUDA"),
        ({"out_semantics": _FakeTensor(shape=(2, 3), dtype=torch.int32, is_cuda=False)}, None,
         "out_semantics must be a CUDA tensor"),
        ({"dirs": _FakeTensor(shape=(2, 3, 3), dtype=torch.float64)}, None, "dirs must have dtype"),
        ({"out_semantics": _FakeTensor(shape=(2, 4), dtype=torch.int32)}, None, "out_semantics must have shape"),
        ({}, (0, 30.0, [0, 0, 0], [1, 1, 1], 128), "max_steps must be a positive integer"),
        ({}, (64, 0.0, [0, 0, 0], [1, 1, 1], 128), "max_distance must be a finite positive float"),
        ({}, (64, 30.0, [1, 0, 0], [1, 1, 1], 128), r"bbox_min\[0\] must be strictly less than bbox_max\[0\]"),
        ({}, (64, 30.0, [0.0, float("nan"), 0.0], [1.0, 1.0, 1.0], 128), "must contain only finite floats"),
        ({}, (64, float("inf"), [0, 0, 0], [1, 1, 1], 128), "max_distance must be a finite positive float"),
        ({}, (64, 30.0, [0, 0, 0], [1, 1, 1], 0), "resolution must be a positive integer"),
        ({"dag": _FakeTensor(shape=(8,), dtype=torch.int32)}, None, "dag_tensor must have dtype"),
        ({"origins": _FakeTensor(shape=(2, 3), dtype=torch.float32)}, None, r"origins must have shape \[batch, rays, 3\]"),
        ({"dirs": _FakeTensor(shape=(2, 4, 3), dtype=torch.float32)}, None, "dirs must match origins shape"),
    ],
)
def test_backend_rejects_invalid_calls(fake_cuda, overrides, args, match):
    tensors = _fake_cast_inputs(**overrides)
    rest = args or (64, 30.0, [0, 0, 0], [1, 1, 1], 128)
    with pytest.raises(RuntimeError, match=match):
        backend_module.cast_rays(*tensors, *rest)


def test_missing_backend_raises(monkeypatch):
    monkeypatch.setattr(backend_module, "HAS_CUDA_BACKEND", False)
    with pytest.raises(RuntimeError, match="torch_sdf_backend is not available"):
        backend_module.cast_rays(*_fake_cast_inputs(), 64, 30.0, [0, 0, 0], [1, 1, 1], 128)


def test_no_cpu_fallback_without_cuda(monkeypatch):
    monkeypatch.setattr(backend_module, "HAS_CUDA_BACKEND", True)
    monkeypatch.setattr(torch.cuda, "is_available", lambda: False)
    with pytest.raises(RuntimeError, match="does not support CPU fallback"):
        backend_module.cast_rays(*_fake_cast_inputs(), 64, 30.0, [0, 0, 0], [1, 1, 1], 128)


def test_native_backend_contract_messages_without_gpu():
    """The native backend object applies the bindings.cpp TORCH_CHECK texts (bindings.cpp:57-89)."""
    be = backend_module._NativeBackend()
    cpu = torch.zeros((1, 1, 3))
    with pytest.raises(RuntimeError, match="^dag_tensor must be a CUDA tensor$"):
        be.cast_rays(torch.zeros(4, dtype=torch.int64), cpu, cpu, torch.zeros((1, 1)),
                     torch.zeros((1, 1), dtype=torch.int32), 8, 1.0, [0, 0, 0], [1, 1, 1], 1)
