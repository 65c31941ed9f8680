"""On-device fp64 Cholesky ridge solve vs torch.linalg (fp64) and the CholeskyFit on CUDA vs the CPU EigenFit."""
import pytest
import torch

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("n,R", [(64, 5), (200, 333), (1000, 70)])
def test_ridge_solve(n, R):
    from ridgefill_data_b200.ops.linalg import ridge_solve
    g = torch.Generator(device="cuda").manual_seed(0)
    x = torch.randn(4 * n, n, device="cuda", dtype=torch.float64, generator=g)
    a = x.T @ x / n
    b = torch.randn(n, R, device="cuda", dtype=torch.float64, generator=g)
    shift = 0.03 * a.diagonal().mean().item()
    got = ridge_solve(a, b, shift)
    ref = torch.linalg.solve(a + shift * torch.eye(n, device="cuda", dtype=torch.float64), b)
    assert ((got - ref).norm() / ref.norm()).item() < 1e-10


def test_cholesky_fit_on_device_matches_eigen_fit():
    from ridgefill_data_b200.ridge.fit import CholeskyFit, EigenFit
    from ridgefill_data_b200.ridge.stats import RidgeStats
    g = torch.Generator().manual_seed(1)
    x = torch.randn(3000, 256, generator=g) * 2 + 1
    ys = {i: x @ (0.05 * torch.randn(256, 256, generator=g)) + 0.1 * torch.randn(3000, 256, generator=g)
          for i in (4, 5)}
    st = RidgeStats(4, [4, 5], 256, "cuda")
    st.add(x.cuda().bfloat16(), {i: y.cuda().bfloat16() for i, y in ys.items()})
    state = st.state()
    e = EigenFit(state).layer(5, [0.03])[0.03]
    c = CholeskyFit(state, device="cuda").layer(5, [0.03])[0.03]
    assert ((c[0].cpu() - e[0]).norm() / e[0].norm()).item() < 1e-5
    assert ((c[1].cpu() - e[1]).norm() / e[1].norm().clamp_min(1e-9)).item() < 1e-4
