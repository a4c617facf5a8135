"""The Euler schedule and step arithmetic against the reference's OWN EulerDiscreteScheduler
(src/infer/scheduler.hpp, compiled from its header into oracle/_ref/libref_scheduler.so by
oracle/build_oracle.py): the library's dlm_sdxl_schedule and the denoising oracle's schedule,
scale_model_input and epsilon Euler step must be bit-identical to it (all of them compute in
double and round to fp32 once)."""
import ctypes

import numpy as np
import pytest
import torch

from oracle.build_oracle import build
from oracle.sdxl_pipeline import euler_schedule as oracle_schedule, euler_step, scale_input

STEPS = [1, 2, 3, 7, 20, 25, 30, 50, 999, 1000]


@pytest.fixture(scope="module")
def ref():
    path = build().get("ref_scheduler")
    if path is None:
        pytest.skip("reference tree absent: libref_scheduler.so not built")
    lib = ctypes.CDLL(path)
    f = ctypes.POINTER(ctypes.c_float)
    lib.ref_sched_set_timesteps.argtypes = [ctypes.c_int, f, f]
    lib.ref_sched_scale.argtypes = [ctypes.c_int, ctypes.c_int, f, ctypes.c_size_t]
    lib.ref_sched_step.argtypes = [ctypes.c_int, ctypes.c_int, f, f, f, ctypes.c_size_t]
    return lib


def _fp(a):
    return a.ctypes.data_as(ctypes.POINTER(ctypes.c_float))


def _ref_schedule(lib, steps):
    s = np.zeros(steps + 1, np.float32)
    t = np.zeros(steps, np.float32)
    assert lib.ref_sched_set_timesteps(steps, _fp(s), _fp(t)) == 0
    return s, t


@pytest.mark.parametrize("steps", STEPS)
def test_library_schedule_is_the_reference(ref, steps):
    from dollama_b200 import _lib as L
    s = np.zeros(steps + 1, np.float32)
    t = np.zeros(steps, np.float32)
    L.call("dlm_sdxl_schedule", steps, _fp(s), _fp(t))
    rs, rt = _ref_schedule(ref, steps)
    assert np.array_equal(s, rs) and np.array_equal(t, rt)


@pytest.mark.parametrize("steps", STEPS)
def test_oracle_schedule_is_the_reference(ref, steps):
    s, t = oracle_schedule(steps)
    rs, rt = _ref_schedule(ref, steps)
    assert np.array_equal(s, rs) and np.array_equal(t, rt)


def test_invalid_step_counts(ref):
    from dollama_b200 import _lib as L
    s = np.zeros(2, np.float32)
    assert ref.ref_sched_set_timesteps(0, _fp(s), _fp(s)) == -1
    assert L.lib().dlm_sdxl_schedule(0, _fp(s), _fp(s)) != 0


@pytest.mark.parametrize("steps", [20, 30])
def test_oracle_step_arithmetic_is_the_reference(ref, steps):
    rng = np.random.default_rng(steps)
    sig, _ = oracle_schedule(steps)
    n = 4 * 32 * 32
    for i in range(steps):
        x = rng.standard_normal(n).astype(np.float32) * 3.0
        e = rng.standard_normal(n).astype(np.float32)
        xs = x.copy()
        assert ref.ref_sched_scale(steps, i, _fp(xs), n) == 0
        assert np.array_equal(scale_input(torch.from_numpy(x), sig[i]).numpy(), xs)
        prev = np.zeros(n, np.float32)
        assert ref.ref_sched_step(steps, i, _fp(e), _fp(x), _fp(prev), n) == 0
        got = euler_step(torch.from_numpy(x), torch.from_numpy(e), sig[i], sig[i + 1]).numpy()
        assert np.array_equal(got, prev)
