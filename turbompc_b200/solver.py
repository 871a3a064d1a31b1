"""TurboMPC SQP solver with the B200 backend
(mirrors turbompc/solvers/turbompc_solver.py).

    solver = TurboMPCSolver(program, params=load_solver_params(),
                            forward_backend="b200", backward_backend="b200")
    guess = solver.initial_guess(problem_params)
    sol = solver.solve(guess, problem_params, weights={})

Everything is batched: ``sol.states`` is (Nb, N+1, nx).  Each SQP iteration
builds the QP at the current trajectory on the GPU and solves it with one
launch of the fused ADMM kernel (``tmpc_admm_solve_*``), warm-started from
the previous ADMM state; the per-problem SQP loop stops when the first-order
error is <= tol_convergence (problems that stop early keep their iterate, as
under jax.vmap of the reference's while_loop).
"""
from __future__ import annotations

import copy
import enum
from typing import Any, Dict, NamedTuple, Optional, Union

import torch

from . import ops
from .ops import ADMMState, AdmmConfig
from .qp_data import (QPCostBlocks, QPData, QPEqualityBlocks, QPInequalityBlocks, qpdata_from_ocp_blocks,
                      scale_qp_data)

DEFAULT_SOLVER_PARAMS: Dict[str, Any] = {
    # turbompc/solvers/params/turbompc.yaml:1-23
    "verbose": False,
    "tol_convergence": 1e-6,
    "convergence_criterion": "first_order",
    "num_sqp_iteration_max": 15,
    "linesearch": False,
    "admm": {
        "rho": 0.1, "sigma": 1e-6, "max_iter": 100, "eps_abs": 1e-9, "eps_rel": 1e-9, "rho_min": 1e-6,
        "rho_max": 1e6, "check_termination_every": 25, "adapt_rho_every": 25, "adaptive_rho_tolerance": 5.0,
        "relaxation_parameter": 1.6, "rho_f_factor": 1000.0,
        "pcg": {"max_iter": 10000, "tol_epsilon": 1e-20},
    },
}


def load_solver_params(overrides: Optional[Dict[str, Any]] = None) -> Dict[str, Any]:
    p = copy.deepcopy(DEFAULT_SOLVER_PARAMS)
    if overrides:
        _deep_merge(p, overrides)
    return p


def _deep_merge(dst, src):
    for k, v in src.items():
        if isinstance(v, dict) and isinstance(dst.get(k), dict):
            _deep_merge(dst[k], v)
        else:
            dst[k] = v


class ForwardBackend(enum.IntEnum):
    """Forward QP backends (turbompc_solver.py:56-64) plus the B200 ones."""

    B200 = 100  # fused ADMM + PCG (drop-in for admm_fused_pcg)
    B200_DIRECT = 101  # fused ADMM + block-tridiagonal Cholesky (drop-in for admm_fused_cudss)


class BackwardBackend(enum.IntEnum):
    B200 = 100  # direct adjoint KKT solve on the GPU (drop-in for direct_cudss_ffi)


_FORWARD_NAMES = {"b200": ForwardBackend.B200, "b200_pcg": ForwardBackend.B200,
                  "admm_fused_pcg": ForwardBackend.B200, "b200_direct": ForwardBackend.B200_DIRECT,
                  "admm_fused_cudss": ForwardBackend.B200_DIRECT}
_BACKWARD_NAMES = {"b200": BackwardBackend.B200, "direct_cudss_ffi": BackwardBackend.B200,
                   "direct_jax_dense": BackwardBackend.B200}


def parse_forward_backend(value: Union[str, ForwardBackend]) -> ForwardBackend:
    if isinstance(value, ForwardBackend):
        return value
    if not isinstance(value, str):
        raise TypeError(f"Expected str or ForwardBackend, got {type(value)}")
    try:
        return _FORWARD_NAMES[value.lower()]
    except KeyError as exc:
        raise ValueError(f"Unknown forward backend: {value!r}. Options: {sorted(_FORWARD_NAMES)}") from exc


def parse_backward_backend(value: Union[str, BackwardBackend]) -> BackwardBackend:
    if isinstance(value, BackwardBackend):
        return value
    if not isinstance(value, str):
        raise TypeError(f"Expected str or BackwardBackend, got {type(value)}")
    try:
        return _BACKWARD_NAMES[value.lower()]
    except KeyError as exc:
        raise ValueError(f"Unknown backward backend: {value!r}. Options: {sorted(_BACKWARD_NAMES)}") from exc


class KKTState(NamedTuple):
    """turbompc_solver.py:194-203 (batched)."""

    states: torch.Tensor
    controls: torch.Tensor
    slack: torch.Tensor
    y_f: torch.Tensor  # (Nb, N+1, nx)
    y_ineq: torch.Tensor  # (Nb, N+1, m)
    ineq_active_lower_idx: torch.Tensor
    ineq_active_upper_idx: torch.Tensor


class SolverStats(NamedTuple):
    admm_num_iters: torch.Tensor  # (Nb, max_iter)
    eq_constraints_violations: torch.Tensor
    ineq_constraints_violations: torch.Tensor
    convergence_errors: torch.Tensor
    # Per-problem OR of the fused kernel's status words over the SQP
    # iterations (TMPC_STATUS_SINGULAR_BLOCK = 1, TMPC_STATUS_NONFINITE = 2;
    # 0 = clean).  The reference reports no such field (its top-level status
    # is always STATUS_SUCCESS, turbompc_solver.py:1752); it is an addition.
    kernel_status: Optional[torch.Tensor] = None  # (Nb,) int32


class TurboMPCSolution(NamedTuple):
    """turbompc_solver.py:225-238 (batched over the leading axis)."""

    states: torch.Tensor
    controls: torch.Tensor
    slack: torch.Tensor
    status: int
    num_iter: torch.Tensor  # (Nb,)
    convergence_error: torch.Tensor  # (Nb,)
    admm_iters: torch.Tensor  # (Nb, max_iter)
    linesearch_alphas: Optional[torch.Tensor] = None
    admm_state: Optional[ADMMState] = None
    solver_stats: Optional[SolverStats] = None
    dual_backward_guess: Optional[torch.Tensor] = None
    kkt_state: Optional[KKTState] = None


def identify_active_inequalities(g, l, u, eps_abs, eps_rel):
    """turbompc_solver.py:269-292: min(g-l, u-g) <= eps_abs + eps_rel |bound|."""
    dl = g - l
    du = u - g
    use_upper = du < dl
    bound = torch.where(use_upper, u.abs(), l.abs())
    active = torch.minimum(dl, du) <= eps_abs + eps_rel * bound
    return active & ~use_upper, active & use_upper


def _inf(x):
    return x.reshape(x.shape[0], -1).abs().amax(dim=1) if x.shape[-1] > 0 else torch.zeros(
        x.shape[0], dtype=x.dtype, device=x.device)


class TurboMPCSolver:
    """SQP solver that uses the fused B200 ADMM kernel for each QP."""

    STATUS_SUCCESS = 0
    STATUS_FAILED = -1

    def __init__(self, program, params: Optional[Dict[str, Any]] = None, name: str = "TurboMPCSolver", *,
                 forward_backend: Union[str, ForwardBackend] = "b200",
                 backward_backend: Union[str, BackwardBackend] = "b200", use_full_hessian: bool = True):
        self._program = program
        self._params = load_solver_params(params) if params is not None else load_solver_params()
        self._name = name
        self._forward_backend = parse_forward_backend(forward_backend)
        self._backward_backend = parse_backward_backend(backward_backend)
        self._use_full_hessian = use_full_hessian
        crit = self._params.get("convergence_criterion", "first_order")
        if crit not in ("first_order", "step"):
            raise ValueError(f"Unknown convergence criterion: {crit!r}")
        if self._params.get("linesearch", False):
            raise NotImplementedError("line search is not on the b200 path (turbompc.yaml default: False)")
        a = self._params["admm"]
        self._admm_cfg = AdmmConfig(
            max_iter=int(a["max_iter"]), pcg_max_iter=int(a["pcg"]["max_iter"]),
            check_every=int(a.get("check_termination_every", 1)), adapt_rho_every=int(a.get("adapt_rho_every", 5)),
            eps_abs=float(a.get("eps_abs", 1e-4)), eps_rel=float(a.get("eps_rel", 1e-3)), sigma=float(a["sigma"]),
            rho_f_factor=float(a.get("rho_f_factor", 1000.0)), alpha=float(a.get("relaxation_parameter", 1.0)),
            pcg_eps=float(a["pcg"].get("tol_epsilon", 1e-8)),
            adaptive_rho_tolerance=float(a.get("adaptive_rho_tolerance", 5.0)),
            rho_min=float(a.get("rho_min", 1e-6)), rho_max=float(a.get("rho_max", 1e6)),
            use_slack=bool(program.use_slack_variables),
            linsys=1 if self._forward_backend == ForwardBackend.B200_DIRECT else 0)
        self._workspace = None
        self.solve = self.get_differentiable_solve_function()

    def _side_stream(self, dev):
        """One side stream per device for the overlapped first-order check."""
        ss = self.__dict__.setdefault("_side_streams", {})
        if dev.index not in ss:
            ss[dev.index] = torch.cuda.Stream(device=dev)
        return ss[dev.index]

    # -------------------------------------------------------------- props
    @property
    def program(self):
        return self._program

    @property
    def params(self):
        return self._params

    @property
    def name(self):
        return self._name

    @property
    def forward_backend(self):
        return self._forward_backend

    @property
    def backward_backend(self):
        return self._backward_backend

    @property
    def admm_config(self) -> AdmmConfig:
        return self._admm_cfg

    # --------------------------------------------------------------- API
    def initial_guess(self, params=None) -> TurboMPCSolution:
        params = params if params is not None else self._program.params
        states, controls = self._program.initial_guess(params)
        Nb = states.shape[0]
        mi = int(self._params["num_sqp_iteration_max"])
        m = self._program.num_inequality_constraints
        z = lambda *s: torch.zeros(*s, dtype=states.dtype, device=states.device)
        stats = SolverStats(torch.zeros(Nb, mi, dtype=torch.int64, device=states.device), z(Nb, mi), z(Nb, mi),
                            z(Nb, mi))
        return TurboMPCSolution(states=states, controls=controls, slack=z(Nb, states.shape[1], m),
                                status=self.STATUS_SUCCESS, num_iter=torch.zeros(Nb, dtype=torch.int64,
                                                                                 device=states.device),
                                convergence_error=z(Nb), admm_iters=torch.zeros(Nb, mi, dtype=torch.int64,
                                                                                device=states.device),
                                admm_state=None, solver_stats=stats)

    def make_params_with_weights(self, weights, problem_params=None):
        base = dict(self._program.params if problem_params is None else problem_params)
        out = dict(base)
        for k, v in (weights or {}).items():
            if isinstance(v, dict) and isinstance(out.get(k), dict):
                d = dict(out[k])
                d.update(v)
                out[k] = d
            else:
                out[k] = v
        return out

    def get_differentiable_solve_function(self):
        """solve(guess, params, weights) -> TurboMPCSolution.  Gradients w.r.t.
        tensors in ``weights`` (and initial_state) flow through the adjoint KKT
        backward when the b200 backward path is available."""
        from .backward import make_differentiable_solve

        return make_differentiable_solve(self)

    # ------------------------------------------------------------ QP build
    def _build_qp_data(self, states, controls, params, prev: Optional[QPData] = None,
                       apply_variable_scaling: bool = True) -> QPData:
        """turbompc_solver.py:1098-1156.  With ``prev`` (the previous SQP
        iterate's QP of the same solve) the blocks that do not depend on the
        linearisation point are reused: the tracking cost (D, E, q), the
        initial rows (A0, c0), A_plus = -[I 0] and, without extra nonlinear
        inequalities, the box rows (G, l, u).  The dynamics rows (A_minus, c)
        are recomputed.  With the problem's rescale_optimization_variables
        and apply_variable_scaling, the column scaling z = diag(state_diff,
        control_diff) z_hat is applied (qp_data.py:178-210); the constraint
        rows come row-scaled from the problem either way."""
        prog = self._program
        A_minus, c_dyn = prog.linearized_dynamics_rows(states, controls, params)
        scale = apply_variable_scaling and getattr(prog, "rescale_optimization_variables", False)
        col = None
        if scale:
            sd, cd = prog.rescaling(params, states)
            col = torch.cat([sd, cd])
        if prev is not None and getattr(prog, "state_independent_cost", False):
            ineq = prev.ineq
            if not prog.state_independent_inequalities:
                G, l, u = prog.get_inequalities_linearized_matrices(states, controls, params)
                if col is not None:
                    G = G * col
                ineq = QPInequalityBlocks(G.contiguous(), l.contiguous(), u.contiguous(),
                                          prev.ineq.slack_penalization_weight, prev.ineq.use_slack_variables)
            if col is not None:
                A_minus = (A_minus * col).contiguous()
            return QPData(prev.cost, QPEqualityBlocks(prev.eq.A0, A_minus, prev.eq.A_plus, prev.eq.c0, c_dyn), ineq)
        D, E, q = prog.get_cost_linearized_blocks(states, controls, params)
        G, l, u = prog.get_inequalities_linearized_matrices(states, controls, params)
        A0, c0 = prog.get_initial_equality_linearized_matrices(params, states)
        Nb = states.shape[0]
        if hasattr(prog, "dynamics_plus_rows"):
            A_plus = prog.dynamics_plus_rows(params, states, Nb)
        else:
            nx = states.shape[-1]
            A_plus = torch.zeros_like(A_minus)
            A_plus[..., :nx] = -torch.eye(nx, dtype=states.dtype, device=states.device)
        sw = params.get("slack_penalization_weight", None)
        if sw is not None:
            sw = torch.as_tensor(sw, dtype=states.dtype, device=states.device).expand(states.shape[0]).contiguous()
        c = lambda t: t.contiguous()
        qp = QPData(QPCostBlocks(c(D), c(E), c(q)), QPEqualityBlocks(c(A0), A_minus, A_plus, c(c0), c_dyn),
                    QPInequalityBlocks(c(G), c(l), c(u), sw, prog.use_slack_variables))
        if scale:
            sd, cd = prog.rescaling(params, states)
            qp = scale_qp_data(qp, sd, cd).map(lambda t: t.contiguous())
        return qp

    def _first_order_error(self, qp: QPData, states, controls, slacks, st: ADMMState):
        """turbompc_solver.py:1158-1225 (first_order criterion): the fused CUDA
        kernel on GPU tensors (tmpc_first_order_error_*)."""
        x = torch.cat([states, controls], -1)
        if x.is_cuda:
            return ops.first_order_error(qp, x, st, slacks)
        return self._first_order_error_torch(qp, states, controls, slacks, st)

    def _first_order_error_torch(self, qp: QPData, states, controls, slacks, st: ADMMState):
        """The same measure in PyTorch operations (host tensors; the GPU kernel's test reference)."""
        x = torch.cat([states, controls], -1)
        D, E = qp.cost.D, qp.cost.E
        Px = torch.einsum("btij,btj->bti", D, x)
        Px[:, 1:] += torch.einsum("btij,btj->bti", E, x[:, :-1])
        Px[:, :-1] += torch.einsum("btji,btj->bti", E, x[:, 1:])
        Ct = torch.zeros_like(x)
        Ct[:, 0] += torch.einsum("bki,bk->bi", qp.eq.A0, st.y_f_0)
        Ct[:, :-1] += torch.einsum("btki,btk->bti", qp.eq.A_minus, st.y_f_dyn)
        Ct[:, 1:] += torch.einsum("btki,btk->bti", qp.eq.A_plus, st.y_f_dyn)
        Gt = torch.einsum("btki,btk->bti", qp.ineq.G, st.y_g)
        stat = _inf(Px + qp.cost.q + Ct + Gt)
        Cx0 = torch.einsum("bki,bi->bk", qp.eq.A0, x[:, 0]) - qp.eq.c0
        Cx = (torch.einsum("btki,bti->btk", qp.eq.A_minus, x[:, :-1])
              + torch.einsum("btki,bti->btk", qp.eq.A_plus, x[:, 1:]) - qp.eq.c)
        eq = torch.maximum(_inf(Cx0), _inf(Cx))
        g = torch.einsum("btki,bti->btk", qp.ineq.G, x)
        gb = g + slacks if qp.ineq.use_slack_variables else g
        if qp.m > 0:
            viol = torch.maximum((qp.ineq.l - gb).clamp_min(0), (gb - qp.ineq.u).clamp_min(0))
            ineq = _inf(viol)
        else:
            ineq = torch.zeros_like(stat)
        conv = torch.maximum(stat, torch.maximum(eq, ineq))
        if qp.ineq.use_slack_variables and qp.m > 0:
            sw = qp.ineq.slack_penalization_weight
            conv = torch.maximum(conv, _inf(sw[:, None, None] * slacks + st.y_g))
        return conv, eq, ineq, gb

    @staticmethod
    def _ineq_rows(qp: QPData, xb, slacks=None):
        """g = G z (+ slacks) at the QP's iterate: the CUDA kernel for GPU
        tensors (tmpc_ineq_rows_*)."""
        if xb.is_cuda:
            return ops.ineq_rows(qp.ineq.G, xb, slacks)
        g = torch.einsum("btki,bti->btk", qp.ineq.G, xb)
        return g if slacks is None else g + slacks

    def _build_kkt_state(self, states, controls, st: ADMMState, g, l, u) -> KKTState:
        """turbompc_solver.py:1387-1439."""
        nx = self._program.num_state_variables
        y_f = torch.cat([st.y_f_0[:, None, :nx], st.y_f_dyn], 1)
        y_ineq = st.y_g
        slack = st.xi_g
        a = self._params["admm"]
        if self._program.use_slack_variables:
            lo, up = slack > 1e-12, slack < -1e-12
        else:
            pl, pu = identify_active_inequalities(g, l, u, a["eps_abs"], a["eps_rel"])
            tol = a["eps_abs"]
            dl, du = y_ineq < -tol, y_ineq > tol
            und = ~(dl | du)
            lo, up = dl | (und & pl), du | (und & pu)
        return KKTState(states, controls, slack, y_f, y_ineq, lo, up)

    # --------------------------------------------------------------- solve
    def _solve_impl(self, states, controls, params, admm_state0: Optional[ADMMState] = None) -> TurboMPCSolution:
        """SQP loop (turbompc_solver.py:1519-1760)."""
        max_iter = int(self._params["num_sqp_iteration_max"])
        tol = float(self._params["tol_convergence"])
        crit = self._params.get("convergence_criterion", "first_order")
        Nb = states.shape[0]
        dev, dt = states.device, states.dtype
        qp = self._build_qp_data(states, controls, params)
        cfg = self._admm_cfg
        if admm_state0 is None:
            admm_state0 = ops.admm_initial_state(qp, self._params["admm"]["rho"])
        st = admm_state0
        slacks = st.xi_g
        # The selected iterate (z = [states, controls], unscaled) of every
        # problem: its last active SQP iterate.  The KKT state is elementwise in
        # (iterate, ADMM state, g, l, u), so it is built once after the loop
        # from the selected inputs (equal to selecting the per-iteration states).
        z_cur = torch.cat([states, controls], -1)
        conv = torch.full((Nb,), float("inf"), dtype=dt, device=dev)
        it_count = torch.zeros(Nb, dtype=torch.int64, device=dev)
        admm_iters = torch.zeros(Nb, max_iter, dtype=torch.int64, device=dev)
        eqv = torch.zeros(Nb, max_iter, dtype=dt, device=dev)
        inv = torch.zeros(Nb, max_iter, dtype=dt, device=dev)
        cerr = torch.zeros(Nb, max_iter, dtype=dt, device=dev)
        active = torch.ones(Nb, dtype=torch.bool, device=dev)
        nx = self._program.num_state_variables
        g_sel = l_sel = u_sel = None
        sw = qp.ineq.slack_penalization_weight
        kstatus = torch.zeros(Nb, dtype=torch.int32, device=dev)
        rescale = bool(getattr(self._program, "rescale_optimization_variables", False))
        # With tol_convergence <= 0 no problem stops early, so the first-order
        # check of iteration k (which feeds only the statistics, the selects
        # and the KKT state) runs on a side stream, overlapping the next ADMM
        # call; its results are applied right after that call is launched, in
        # the order the sequential loop applies them.
        cur = torch.cuda.current_stream(dev) if dev.type == "cuda" else None
        side = self._side_stream(dev) if (cur is not None and tol <= 0) else None
        pending = None

        def apply(p):
            nonlocal g_sel, l_sel, u_sel, conv, active
            k_, cv_, ev_, iv_, g_, l_, u_, act_, on_side, _keep = p  # _keep: inputs of the side stream
            if on_side:
                cur.wait_stream(side)
                for t_ in (cv_, ev_, iv_, g_):
                    t_.record_stream(cur)
            if k_ == 0:
                g_sel, l_sel, u_sel, conv = g_, l_, u_, cv_
            else:
                sel = lambda new, old: new if new is old else torch.where(
                    act_.view(-1, *([1] * (new.dim() - 1))), new, old)
                g_sel, l_sel, u_sel, conv = sel(g_, g_sel), sel(l_, l_sel), sel(u_, u_sel), sel(cv_, conv)
            eqv[:, k_], inv[:, k_], cerr[:, k_] = ev_, iv_, cv_
            active = act_ & (conv > tol)

        for k in range(max_iter):
            if k > 0 and tol > 0 and not bool(active.any()):
                break
            st_new, iters, status = ops.admm_solve(qp, st, cfg, slack_weight=sw, workspace=self._workspace)
            if pending is not None:
                apply(pending)
                pending = None
            xb = st_new.x_blocks  # QP (scaled) coordinates
            if rescale:
                s_new, c_new = self._program.unscale_states_controls(xb[..., :nx], xb[..., nx:], params)
                z_new = torch.cat([s_new, c_new], -1)
            else:
                z_new = xb
            sl_new = st_new.xi_g
            step = _inf(z_new - z_cur)
            if sl_new.shape[-1] > 0:
                step = step + _inf(sl_new - slacks)
            # Masked update (problems already converged keep their iterate).
            if k == 0:  # every problem is active: nothing to select
                kstatus = status.clone()
                z_cur, slacks, st = z_new, sl_new, st_new
                admm_iters[:, k] = iters
            else:
                sel = lambda new, old: new if new is old else torch.where(
                    active.view(-1, *([1] * (new.dim() - 1))), new, old)
                kstatus = kstatus | torch.where(active, status, torch.zeros_like(status))
                z_cur, slacks = sel(z_new, z_cur), sel(sl_new, slacks)
                st = ADMMState(*(sel(n_, o_) for n_, o_ in zip(st_new, st)))
                admm_iters[:, k] = torch.where(active, iters, admm_iters[:, k])
            it_count = it_count + active.to(torch.int64)
            on_side = False
            if crit == "first_order":
                if k + 1 < max_iter:
                    qp_next = self._build_qp_data(z_new[..., :nx], z_new[..., nx:], params, prev=qp)
                    if side is not None:
                        side.wait_stream(cur)
                        with torch.cuda.stream(side):
                            cv, ev, iv, g = self._first_order_error(qp_next, xb[..., :nx], xb[..., nx:], sl_new,
                                                                    st_new)
                        on_side = True
                    else:
                        cv, ev, iv, g = self._first_order_error(qp_next, xb[..., :nx], xb[..., nx:], sl_new, st_new)
                else:
                    qp_next = qp
                    cv = step if k == 0 else conv
                    ev = iv = torch.zeros_like(cv)
                    g = self._ineq_rows(qp, xb, sl_new if qp.ineq.use_slack_variables else None)
            else:
                qp_next = self._build_qp_data(z_new[..., :nx], z_new[..., nx:], params, prev=qp) \
                    if k + 1 < max_iter else qp
                cv, ev, iv, g = step, torch.zeros_like(step), torch.zeros_like(step), self._ineq_rows(qp_next, xb)
            # the side stream's inputs stay referenced until the main stream has
            # waited for it (their memory is not handed out again before)
            p = (k, cv, ev, iv, g, qp_next.ineq.l, qp_next.ineq.u, active, on_side, (xb, sl_new, st_new, qp_next))
            if on_side:
                pending = p
            else:
                apply(p)
            if k + 1 < max_iter:
                # Every problem moves on to the QP at its new iterate: a problem
                # that has converged still runs (its results are discarded by
                # the selects), so its QP needs no select and the loop never
                # waits on the device to decide.
                qp = qp_next
        if pending is not None:
            apply(pending)
        states, controls = z_cur[..., :nx].contiguous(), z_cur[..., nx:].contiguous()
        kkt = None if g_sel is None else self._build_kkt_state(states, controls, st, g_sel, l_sel, u_sel)
        return TurboMPCSolution(states=states, controls=controls, slack=st.xi_g, status=self.STATUS_SUCCESS,
                                num_iter=it_count, convergence_error=conv, admm_iters=admm_iters, admm_state=st,
                                solver_stats=SolverStats(admm_iters, eqv, inv, cerr, kstatus), kkt_state=kkt)
