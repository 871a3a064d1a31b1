"""CPU checks of the batched OCP linearisation (the QP producer) against
finite differences and the reference's conventions."""
import torch

from turbompc_b200.problems.quadrotor import make_obstacle_problem, make_quadrotor_problem
from turbompc_b200.solver import TurboMPCSolver, identify_active_inequalities


def test_dynamics_jacobian_matches_finite_differences():
    ocp, p = make_quadrotor_problem(3, N=4, dtype=torch.float64, device="cpu")
    x = torch.randn(3, 5, 12, dtype=torch.float64) * 0.3
    u = torch.rand(3, 5, 4, dtype=torch.float64) * 5
    An, Bn, A, B, Cs = ocp.get_dynamics_linearized_matrices(x, u, p)
    f0 = ocp.next_states(x, u, p)
    h = 1e-6
    for j in range(16):
        xp, up = x.clone(), u.clone()
        if j < 12:
            xp[:, :4, j] += h
        else:
            up[:, :4, j - 12] += h
        fd = (ocp.next_states(xp, up, p) - f0) / h
        J = A[..., j] if j < 12 else B[..., j - 12]
        assert torch.allclose(fd, J, atol=1e-5)
    # c = -f + A x + B u  and  A_next = -I
    c = Cs[:, 1:]
    assert torch.allclose(c, -f0 + torch.einsum("btij,btj->bti", A, x[:, :4]) +
                          torch.einsum("btij,btj->bti", B, u[:, :4]))
    assert torch.allclose(An, -torch.eye(12, dtype=torch.float64).expand_as(An))


def test_cost_blocks_match_autograd():
    ocp, p = make_quadrotor_problem(2, N=3, dtype=torch.float64, device="cpu")
    p = dict(p, weights_penalization_control_rate=torch.tensor([0.5, 0.2, 0.1, 0.3], dtype=torch.float64))
    x = torch.randn(2, 4, 12, dtype=torch.float64)
    u = torch.randn(2, 4, 4, dtype=torch.float64)
    D, E, q = ocp.get_cost_linearized_blocks(x, u, p)
    z = torch.cat([x, u], -1).reshape(2, -1).requires_grad_(True)

    def total(zf):
        zz = zf.reshape(2, 4, 16)
        return ocp.cost(zz[..., :12], zz[..., 12:], p).sum()

    H = torch.autograd.functional.hessian(total, z)  # (2, 64, 2, 64)
    for b in range(2):
        Hb = H[b, :, b, :]
        for t in range(4):
            assert torch.allclose(Hb[t * 16:(t + 1) * 16, t * 16:(t + 1) * 16], D[b, t], atol=1e-9)
        for t in range(3):
            assert torch.allclose(Hb[t * 16:(t + 1) * 16, (t + 1) * 16:(t + 2) * 16], E[b, t], atol=1e-9)
    g = torch.autograd.grad(total(z), z)[0].reshape(2, 4, 16)
    Pz = torch.einsum("btij,btj->bti", D, z.detach().reshape(2, 4, 16))
    zz = z.detach().reshape(2, 4, 16)
    Pz[:, 1:] += torch.einsum("btij,btj->bti", E.transpose(-1, -2), zz[:, :-1])
    Pz[:, :-1] += torch.einsum("btij,btj->bti", E, zz[:, 1:])
    assert torch.allclose(g - Pz, q, atol=1e-8)


def test_box_and_obstacle_rows():
    ocp, p = make_obstacle_problem(2, N=3, dtype=torch.float64, device="cpu")
    assert ocp.num_inequality_constraints == 4 + 8
    x = torch.randn(2, 4, 12, dtype=torch.float64)
    u = torch.rand(2, 4, 4, dtype=torch.float64)
    G, l, up = ocp.get_inequalities_linearized_matrices(x, u, p)
    assert G.shape == (2, 4, 12, 16)
    assert torch.all(G[:, :, :4, 12:] == torch.eye(4, dtype=torch.float64))
    # linearised obstacle row is exact at the linearisation point
    c, r = p["obstacles_centers"], p["obstacles_radii"]
    g = 1 - (x[:, :, None, :3] - c[:, None]).norm(dim=-1) / (r[:, None] + 0.001)
    gl = torch.einsum("btki,bti->btk", G[:, :, 4:], torch.cat([x, u], -1))
    assert torch.allclose(gl - up[:, :, 4:], g, atol=1e-12)


def test_active_set_rule():
    g = torch.tensor([0.0, 0.5, 1.0])
    lo, hi = identify_active_inequalities(g, torch.zeros(3), torch.ones(3), 1e-9, 1e-9)
    assert lo.tolist() == [True, False, False] and hi.tolist() == [False, False, True]


def test_solver_builds_qp_on_cpu():
    ocp, p = make_quadrotor_problem(2, N=5, dtype=torch.float64, device="cpu")
    s = TurboMPCSolver(ocp, {"num_sqp_iteration_max": 2})
    guess = s.initial_guess(p)
    qp = s._build_qp_data(guess.states, guess.controls, p)
    assert (qp.Nb, qp.T, qp.n, qp.nx, qp.n0, qp.m) == (2, 6, 16, 12, 12, 4)


def test_learned_cost_quadratisation_matches_autograd():
    """Config 5 cost: D and q of the MLP-augmented stage cost equal the
    autograd Hessian / gradient-minus-Hessian-times-point of cost()."""
    import torch
    from turbompc_b200.problems.learned_cost import make_learned_cost_problem
    prog, params = make_learned_cost_problem(2, N=4, hidden=8, seed=1, dtype=torch.float64, device="cpu")
    g = torch.Generator().manual_seed(0)
    xs = torch.randn(2, 5, 6, generator=g, dtype=torch.float64)
    us = 0.05 * torch.randn(2, 5, 3, generator=g, dtype=torch.float64)
    D, E, q = prog.get_cost_linearized_blocks(xs, us, params)
    z = torch.cat([xs, us], -1).reshape(-1).requires_grad_(True)
    f = lambda zz: prog.cost(zz.view(2, 5, 9)[..., :6], zz.view(2, 5, 9)[..., 6:], params).sum()
    Hf = torch.autograd.functional.hessian(f, z).view(2, 5, 9, 2, 5, 9)
    grad = torch.autograd.grad(f(z), z)[0].view(2, 5, 9)
    for b in range(2):
        for t in range(5):
            assert torch.allclose(D[b, t], Hf[b, t, :, b, t, :], atol=1e-10)
    zz = z.detach().view(2, 5, 9)
    Pz = torch.einsum("btij,btj->bti", D, zz)
    Pz[:, 1:] += torch.einsum("btij,btj->bti", E, zz[:, :-1])
    Pz[:, :-1] += torch.einsum("btji,btj->bti", E, zz[:, 1:])
    assert torch.allclose(q, grad - Pz, atol=1e-9)
    assert (torch.linalg.eigvalsh(D) > 0).all()


def test_gradient_accuracy_problem_data_is_stable_and_seeded():
    """benchmarking/linear-system/utils.py:28-62: eigenvalues of A inside the
    unit circle, the legacy NumPy stream seeded by the seed."""
    import numpy as np
    from turbompc_b200.gradient_accuracy import problem_data
    Q, R, A, B, b, x0 = problem_data(16, 3, 8, 4)
    assert np.abs(np.linalg.eigvals(A)).max() < 1.0
    assert x0.shape == (16, 8) and B.shape == (8, 4) and b.shape == (8,)
    rs = np.random.RandomState(3)
    rs.randn(8, 8)  # A's draw comes first, then B's
    assert np.array_equal(B, rs.randn(8, 4))
    Q2, R2, A2, B2, b2, x02 = problem_data(16, 3, 8, 4)
    assert np.array_equal(A, A2) and np.array_equal(x0, x02)
