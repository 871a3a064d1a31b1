"""The gradient-accuracy sweep (turbompc_b200.gradient_accuracy, the protocol
of benchmarking/linear-system/benchmark_turbompc_gradient_accuracy.py) on a
small case: at a tight solver tolerance the rollout's automatic gradient with
respect to Q and R agrees with central finite differences."""
import argparse

import pytest

from turbompc_b200 import gradient_accuracy as ga

pytestmark = pytest.mark.gpu


def test_gradient_accuracy_small_sweep():
    args = argparse.Namespace(tolerances=[1e-9], n_seeds=2, batch_size=4, horizon=8, sim_steps=3, n_state=4,
                              n_ctrl=2, umax=1.0, admm_max_iter=4000, fd_eps=1e-5, forward="b200_direct",
                              quiet=True, out="")
    res = ga.run(args)["1e-09"]
    assert res["cos_all"]["min"] > 0.9999, res["cos_all"]
    assert res["rel_l2_all"]["max"] < 1e-3, res["rel_l2_all"]
