"""torch integration the reference's test-suite checks for this path
(tests/test_chamfer.py:335-358, tests/test_knn.py:389-423 of the reference):
torch.library.opcheck on the operators and torch.compile of the public API."""
import pytest
import torch

import datagen

pytestmark = pytest.mark.gpu
DEV = "cuda"


def test_opcheck_chamfer_forward():
    import torch_point_ops_b200 as tpo  # noqa: F401

    x1 = datagen.uniform(2, 40, 1).to(DEV)
    x2 = datagen.uniform(2, 50, 2).to(DEV)
    # the backward scatters with atomics (summation order free), so like the
    # reference only the forward is checked for autograd registration details
    torch.library.opcheck(torch.ops.torch_point_ops_b200_chamfer.chamfer_forward.default, (x1, x2),
                          test_utils=("test_schema", "test_faketensor"))


def test_opcheck_knn_forward():
    import torch_point_ops_b200 as tpo  # noqa: F401

    p1 = torch.randn(2, 30, 3, device=DEV)
    p2 = torch.randn(2, 40, 3, device=DEV)
    l1 = torch.tensor([30, 20], device=DEV)
    l2 = torch.tensor([40, 11], device=DEV)
    torch.library.opcheck(torch.ops.torch_point_ops_b200_knn.knn_forward.default,
                          (p1, p2, l1, l2, 2, 5, -1), test_utils=("test_schema", "test_faketensor"))


def test_opcheck_knn_gather():
    import torch_point_ops_b200 as tpo  # noqa: F401

    x = torch.randn(2, 40, 3, device=DEV)
    idx = torch.randint(0, 40, (2, 30, 4), device=DEV)
    torch.library.opcheck(torch.ops.torch_point_ops_b200_knn.knn_gather_forward.default,
                          (x, idx, None), test_utils=("test_schema", "test_faketensor"))


def test_torch_compile_chamfer_and_knn():
    import torch_point_ops_b200 as tpo

    x1 = datagen.uniform(2, 300, 3).to(DEV)
    x2 = datagen.uniform(2, 200, 4).to(DEV)

    def f(a, b):
        d1, d2 = tpo.chamfer_distance(a, b)
        i, d = tpo.knn_points(a, b, K=4)
        return d1.sum() + d2.sum() + d.sum()

    eager = f(x1, x2)
    compiled = torch.compile(f, fullgraph=True)(x1, x2)
    assert torch.allclose(eager, compiled, rtol=1e-6)
