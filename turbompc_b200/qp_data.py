"""Batched stage-blocked QP containers (mirror turbompc/solvers/qp_data.py:13-97).

Every tensor carries a leading batch axis ``Nb`` (the layout the reference's
FFI handlers see after ``vmap_method="broadcast_all"``):

    cost.D (Nb, T, n, n)   cost.E (Nb, N, n, n)   cost.q (Nb, T, n)
    eq.A0 (Nb, n0, n)      eq.A_minus / eq.A_plus (Nb, N, nx, n)
    eq.c0 (Nb, n0)         eq.c (Nb, N, nx)
    ineq.G (Nb, T, m, n)   ineq.l / ineq.u (Nb, T, m)
"""
from __future__ import annotations

from dataclasses import dataclass, field, replace
from typing import Optional

import torch


@dataclass(frozen=True)
class QPCostBlocks:
    D: torch.Tensor
    E: torch.Tensor
    q: torch.Tensor


@dataclass(frozen=True)
class QPEqualityBlocks:
    A0: torch.Tensor
    A_minus: torch.Tensor
    A_plus: torch.Tensor
    c0: torch.Tensor
    c: torch.Tensor


@dataclass(frozen=True)
class QPInequalityBlocks:
    G: torch.Tensor
    l: torch.Tensor
    u: torch.Tensor
    slack_penalization_weight: Optional[torch.Tensor] = None  # (Nb,) or scalar
    use_slack_variables: bool = False


@dataclass(frozen=True)
class QPData:
    cost: QPCostBlocks
    eq: QPEqualityBlocks
    ineq: QPInequalityBlocks

    @property
    def Nb(self) -> int:
        return self.cost.D.shape[0]

    @property
    def T(self) -> int:
        return self.cost.D.shape[1]

    @property
    def n(self) -> int:
        return self.cost.D.shape[2]

    @property
    def nx(self) -> int:
        return self.eq.A_minus.shape[2]

    @property
    def n0(self) -> int:
        return self.eq.A0.shape[1]

    @property
    def m(self) -> int:
        return self.ineq.G.shape[2]

    @property
    def dtype(self) -> torch.dtype:
        return self.cost.D.dtype

    @property
    def device(self) -> torch.device:
        return self.cost.D.device

    def tensors(self):
        return dict(D=self.cost.D, E=self.cost.E, q=self.cost.q, A0=self.eq.A0, A_minus=self.eq.A_minus,
                    A_plus=self.eq.A_plus, c0=self.eq.c0, c=self.eq.c, G=self.ineq.G, l=self.ineq.l,
                    u=self.ineq.u)

    def map(self, fn) -> "QPData":
        """Apply fn to every tensor (e.g. ``lambda t: t.to('cuda')``)."""
        sw = self.ineq.slack_penalization_weight
        return QPData(
            cost=QPCostBlocks(fn(self.cost.D), fn(self.cost.E), fn(self.cost.q)),
            eq=QPEqualityBlocks(fn(self.eq.A0), fn(self.eq.A_minus), fn(self.eq.A_plus), fn(self.eq.c0),
                                fn(self.eq.c)),
            ineq=QPInequalityBlocks(fn(self.ineq.G), fn(self.ineq.l), fn(self.ineq.u),
                                    None if sw is None else fn(sw), self.ineq.use_slack_variables),
        )

    def slice(self, lo: int, hi: int) -> "QPData":
        """Sub-batch [lo, hi) (views)."""
        return self.map(lambda t: t[lo:hi] if t.dim() > 0 else t)


def qpdata_from_ocp_blocks(D, E, q, A0, c0, As_next, Bs_next, As, Bs, c_dyn, ineq_blocks, ineq_l, ineq_u,
                           use_slack_variables=False, slack_penalization_weight=None) -> QPData:
    """qp_data.py:140-175: A_minus = [A B], A_plus = [A_next B_next]."""
    return QPData(
        cost=QPCostBlocks(D, E, q),
        eq=QPEqualityBlocks(A0, torch.cat([As, Bs], dim=-1), torch.cat([As_next, Bs_next], dim=-1), c0, c_dyn),
        ineq=QPInequalityBlocks(ineq_blocks, ineq_l, ineq_u, slack_penalization_weight, use_slack_variables),
    )


def scale_qp_data(qp: QPData, state_scale: torch.Tensor, control_scale: torch.Tensor) -> QPData:
    """Column scaling z = S z_hat (qp_data.py:178-210)."""
    s = torch.cat([state_scale, control_scale], dim=-1)
    col = s[..., None, None, :]
    row = s[..., None, :, None]
    return QPData(
        cost=QPCostBlocks(qp.cost.D * row * col, qp.cost.E * row * col, qp.cost.q * s[..., None, :]),
        eq=QPEqualityBlocks(qp.eq.A0 * s[..., None, :], qp.eq.A_minus * col, qp.eq.A_plus * col, qp.eq.c0,
                            qp.eq.c),
        ineq=replace(qp.ineq, G=qp.ineq.G * col),
    )
