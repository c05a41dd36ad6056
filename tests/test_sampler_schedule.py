"""CPU checks of the DPM-Solver++ (2M) schedule restated in the oracle."""
import math

import numpy as np

from oracle import rdt1b_ref


def test_timesteps_and_final_step():
    ts, a, b, c = rdt1b_ref.dpm_schedule(5)
    assert ts == [999, 799, 599, 400, 200]
    assert (a[-1], b[-1], c[-1]) == (0.0, 1.0, 0.0)
    assert c[0] == 0.0


def test_constant_prediction_is_fixed_point_of_the_ode():
    # if the network always predicts x0*, the exact probability-flow solution
    # from x_s = α_s x0* + σ_s ε is x_t = α_t x0* + σ_t ε; every first- and
    # second-order update with a constant x0 reproduces it exactly.
    ts, a, b, c = rdt1b_ref.dpm_schedule(5)
    def abar(t):
        return math.cos((t + 0.008) / 1.008 * math.pi / 2) ** 2
    betas = [min(1 - abar((i + 1) / 1000) / abar(i / 1000), 0.999) for i in range(1000)]
    ac = np.cumprod(1 - np.array(betas))
    x0, eps = 0.7, -1.3
    x = math.sqrt(ac[ts[0]]) * x0 + math.sqrt(1 - ac[ts[0]]) * eps
    for i in range(5):
        x = a[i] * x + b[i] * x0 + c[i] * x0
        if i < 4:
            t = ts[i + 1]
            assert abs(x - (math.sqrt(ac[t]) * x0 + math.sqrt(1 - ac[t]) * eps)) < 1e-9
    assert abs(x - x0) < 1e-12
