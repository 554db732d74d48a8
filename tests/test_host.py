"""CPU checks of the Python mirror of the reference API: argument validation
and error behaviour (no CPU fallback), without a GPU."""

from __future__ import annotations

import math

import pytest
import torch

import sinkhorn_b200 as skb
from sinkhorn_b200 import _tensors as T


def test_exports_mirror_the_reference_package():
    for name in ("sinkhorn", "SinkhornOutput", "sinkhorn_differentiable", "__version__"):
        assert hasattr(skb, name)
    from sinkhorn_b200.cuda import lse_col, lse_row, sinkhorn_forward_cuda  # noqa: F401
    from sinkhorn_b200.cuda.forward import sinkhorn_forward_cuda as s2  # noqa: F401


def test_cost_must_be_3d():
    with pytest.raises(ValueError, match="3D"):
        skb.sinkhorn(torch.zeros(4, 4))


def test_cpu_tensor_raises_instead_of_falling_back():
    with pytest.raises(RuntimeError, match="no CPU fallback"):
        skb.sinkhorn(torch.zeros(1, 4, 4))


def test_unknown_backend_is_rejected():
    with pytest.raises(ValueError, match="backend"):
        skb.sinkhorn(torch.zeros(1, 4, 4), backend="pytorch")


def test_float64_is_rejected_on_cpu_before_device_checks():
    with pytest.raises((TypeError, RuntimeError)):
        T.check_cost(torch.zeros(1, 4, 4, dtype=torch.float64))


def test_tau_encoding():
    assert math.isinf(T.tau_arg(None))
    assert T.tau_arg(2.0) == 2.0


def test_vector_and_mask_shape_checks():
    with pytest.raises(ValueError, match="shape"):
        T.vec(torch.zeros(2, 3), (2, 4), torch.device("cpu"), "a")
    m = T.mask(torch.tensor([[True, False]]), (1, 2), torch.device("cpu"), "mask_a")
    assert m.dtype == torch.uint8 and m.tolist() == [[1, 0]]
    m2 = T.mask(torch.tensor([[2, 0]]), (1, 2), torch.device("cpu"), "mask_a")
    assert m2.tolist() == [[1, 0]]


def test_sinkhorn_output_divergence_is_dual_estimate():
    f = torch.tensor([[1.0, 3.0]])
    g = torch.tensor([[2.0, 2.0, 2.0]])
    out = skb.SinkhornOutput(f=f, g=g, n_iters=1, converged=True)
    assert torch.allclose(out.sinkhorn_divergence(None, 0.1), torch.tensor([4.0]))


def test_missing_library_raises_instead_of_computing(monkeypatch, tmp_path):
    """Without the built library every entry point raises: nothing runs on the
    CPU instead."""
    from sinkhorn_b200 import _lib
    monkeypatch.setattr(_lib, "LIB_PATH", str(tmp_path / "libsinkhorn_b200.so"))
    monkeypatch.setattr(_lib, "_lib", None)
    with pytest.raises(RuntimeError, match="no CPU fallback"):
        _lib.load()
    from sinkhorn_b200.cuda.solver import plan_query
    with pytest.raises(RuntimeError, match="no CPU fallback"):
        plan_query(torch.zeros(1, 4, 4))
