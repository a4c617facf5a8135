"""The device denoising loop's Euler schedule (dlm_sdxl_schedule) against the oracle restatement
of the reference's EulerDiscreteScheduler and against the values its own header records for 20
steps (src/infer/scheduler.hpp:19-21: sigmas[0] = 11.028, timesteps 951 ... 1)."""
import numpy as np
import pytest

from dollama_b200.pipeline import euler_schedule
from oracle.sdxl_pipeline import euler_schedule as oracle_schedule


@pytest.mark.parametrize("steps", [1, 4, 20, 30, 50])
def test_schedule_matches_oracle(steps):
    s, t = euler_schedule(steps)
    os_, ot = oracle_schedule(steps)
    assert np.array_equal(np.float32(t), ot)
    assert np.allclose(np.float32(s), os_, rtol=1e-6, atol=0)
    assert s[-1] == 0.0


def test_schedule_reference_values():
    s, t = euler_schedule(20)
    assert abs(s[0] - 11.028) < 5e-4
    assert t[0] == 951.0 and t[-1] == 1.0
    assert all(a > b for a, b in zip(s, s[1:]))
