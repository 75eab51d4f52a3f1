"""torch_contract (autograd over the GPU contraction) against the reference
binding's own torch tests and torch float64 einsum.

The first group repeats the cases of the reference's
python/ndtensors_rs/tests/test_torch_ops.py (values and assertions as there:
:14-52 forward, :58-124 backward, :130-198 edge cases), once with CPU tensors
(the reference's device) and once with CUDA tensors, which never leave device
memory here.  The second group checks random float64 contractions on CUDA
against torch.einsum at the contraction tolerance (relative Frobenius error
<= 1e-12), and the gradients by torch.autograd.gradcheck.
"""

from __future__ import annotations

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")

RTOL = 1e-12
DEVICES = ["cpu", "cuda"]


def rel_fro(x, y):
    x, y = x.detach().double().cpu(), y.detach().double().cpu()
    return float(torch.linalg.norm((x - y).flatten()) / torch.linalg.norm(y.flatten()))


@pytest.fixture
def tc(gpu):
    from ndtensors_b200.torch_ops import torch_contract

    return torch_contract


@pytest.mark.parametrize("dev", DEVICES)
def test_matrix_multiply(tc, dev):
    c = tc(torch.ones((2, 3), device=dev), (1, -1), torch.ones((3, 4), device=dev), (-1, 2))
    assert c.shape == (2, 4) and c.device.type == dev
    assert c[0, 0].item() == 3.0


@pytest.mark.parametrize("dev", DEVICES)
def test_matrix_multiply_values(tc, dev):
    a = torch.tensor([[1.0, 2.0], [3.0, 4.0]], device=dev)
    b = torch.tensor([[5.0, 6.0], [7.0, 8.0]], device=dev)
    c = tc(a, (1, -1), b, (-1, 2))
    torch.testing.assert_close(c, torch.tensor([[19.0, 22.0], [43.0, 50.0]], dtype=torch.float64, device=dev))


@pytest.mark.parametrize("dev", DEVICES)
def test_inner_product(tc, dev):
    r = tc(torch.tensor([1.0, 2.0, 3.0], device=dev), (-1,), torch.tensor([4.0, 5.0, 6.0], device=dev), (-1,))
    assert r.shape == (1,)
    assert r[0].item() == 32.0


@pytest.mark.parametrize("dev", DEVICES)
def test_outer_product(tc, dev):
    v1, v2 = torch.tensor([1.0, 2.0], device=dev), torch.tensor([3.0, 4.0, 5.0], device=dev)
    r = tc(v1, (1,), v2, (2,))
    assert r.shape == (2, 3)
    torch.testing.assert_close(r, torch.outer(v1, v2).to(torch.float64))


@pytest.mark.parametrize("dev", DEVICES)
def test_backward_values(tc, dev):
    a = torch.ones((2, 3), requires_grad=True, device=dev)
    b = torch.ones((3, 4), requires_grad=True, device=dev)
    tc(a, (1, -1), b, (-1, 2)).sum().backward()
    assert a.grad.shape == (2, 3) and b.grad.shape == (3, 4)
    assert a.grad.device.type == dev and b.grad.device.type == dev
    assert a.grad[0, 0].item() == 4.0  # sum_k B[j, k]
    assert b.grad[0, 0].item() == 2.0  # sum_i A[i, j]


@pytest.mark.parametrize("dev", DEVICES)
def test_backward_chain_rule(tc, dev):
    rng = np.random.default_rng(42)
    a_np, b_np, g_np = rng.random((2, 3)), rng.random((3, 4)), rng.random((2, 4))
    a = torch.tensor(a_np, requires_grad=True, device=dev)
    b = torch.tensor(b_np, requires_grad=True, device=dev)
    (tc(a, (1, -1), b, (-1, 2)) * torch.tensor(g_np, device=dev)).sum().backward()
    np.testing.assert_array_almost_equal(a.grad.cpu().numpy(), g_np @ b_np.T, decimal=10)
    np.testing.assert_array_almost_equal(b.grad.cpu().numpy(), a_np.T @ g_np, decimal=10)


@pytest.mark.parametrize("dev", DEVICES)
def test_autograd_grad(tc, dev):
    a = torch.ones((2, 3), requires_grad=True, device=dev)
    b = torch.ones((3, 4), requires_grad=True, device=dev)
    grads = torch.autograd.grad(tc(a, (1, -1), b, (-1, 2)).sum(), [a, b])
    assert len(grads) == 2 and grads[0].shape == (2, 3) and grads[1].shape == (3, 4)


@pytest.mark.parametrize("dev", DEVICES)
def test_edge_cases(tc, dev):
    v1 = torch.ones((5,), requires_grad=True, device=dev)
    v2 = torch.ones((5,), requires_grad=True, device=dev)
    r = tc(v1, (-1,), v2, (-1,))
    assert r[0].item() == 5.0
    r.sum().backward()
    assert v1.grad is not None and v2.grad is not None
    a = torch.ones((2, 3, 4), requires_grad=True, device=dev)
    b = torch.ones((4, 5), requires_grad=True, device=dev)
    c = tc(a, (1, 2, -1), b, (-1, 3))
    assert c.shape == (2, 3, 5) and c[0, 0, 0].item() == 4.0
    c.sum().backward()
    assert a.grad is not None and b.grad is not None
    a = torch.ones((2, 3, 4), requires_grad=True, device=dev)
    b = torch.ones((3, 4, 5), requires_grad=True, device=dev)
    c = tc(a, (1, -1, -2), b, (-1, -2, 2))
    assert c.shape == (2, 5) and c[0, 0].item() == 12.0
    c.sum().backward()
    assert a.grad is not None and b.grad is not None
    with torch.no_grad():
        c = tc(torch.ones((2, 3), device=dev), (1, -1), torch.ones((3, 4), device=dev), (-1, 2))
    assert c.shape == (2, 4) and not c.requires_grad
    c = tc(torch.ones((2, 3), requires_grad=True, device=dev).detach(), (1, -1),
           torch.ones((3, 4), requires_grad=True, device=dev).detach(), (-1, 2))
    assert c.shape == (2, 4)


EINSUM_CASES = [
    # (shape_a, labels_a, shape_b, labels_b, einsum)
    ((24, 16, 20), (1, 2, -1), (20, 8, 12), (-1, 3, 4), "abk,kcd->abcd"),  # MPS merge shape
    ((10, 6, 7, 9), (-2, 1, -1, 2), (7, 5, 10), (-1, 3, -2), "jakb,kcj->abc"),  # permuted operands
    ((64, 5, 2, 2, 16), (1, -1, -2, 3, 4), (5, 5, 2, 2), (-1, 5, -2, 6), "aijbc,idje->abcde"),  # skinny
    ((300, 7), (1, -1), (7,), (-1,), "ak,k->a"),  # matrix-vector
]


@pytest.mark.parametrize("sa,la,sb,lb,eq", EINSUM_CASES)
def test_cuda_forward_backward_vs_einsum(tc, sa, la, sb, lb, eq):
    g = torch.Generator(device="cuda").manual_seed(len(eq))
    a = torch.randn(sa, dtype=torch.float64, device="cuda", generator=g, requires_grad=True)
    b = torch.randn(sb, dtype=torch.float64, device="cuda", generator=g, requires_grad=True)
    a2, b2 = a.detach().clone().requires_grad_(), b.detach().clone().requires_grad_()
    c = tc(a, la, b, lb)
    ref = torch.einsum(eq, a2, b2)
    assert c.is_cuda and c.shape == ref.shape
    assert rel_fro(c, ref) <= RTOL
    w = torch.randn(ref.shape, dtype=torch.float64, device="cuda", generator=g)
    (c * w).sum().backward()
    (ref * w).sum().backward()
    assert a.grad.is_cuda and b.grad.is_cuda
    assert rel_fro(a.grad, a2.grad) <= RTOL
    assert rel_fro(b.grad, b2.grad) <= RTOL


def test_cuda_gradcheck(tc):
    g = torch.Generator(device="cuda").manual_seed(3)
    a = torch.randn((4, 3, 5), dtype=torch.float64, device="cuda", generator=g, requires_grad=True)
    b = torch.randn((5, 3, 2), dtype=torch.float64, device="cuda", generator=g, requires_grad=True)
    assert torch.autograd.gradcheck(lambda x, y: tc(x, (1, -1, -2), y, (-2, -1, 2)), (a, b), eps=1e-6, atol=1e-4)


def test_mixed_devices_rejected(tc):
    from ndtensors_b200 import NDTensorsError

    with pytest.raises(NDTensorsError):
        tc(torch.ones(3), (-1,), torch.ones(3, device="cuda"), (-1,))
