"""The flow-matching sampler of the Z-Image pipeline (scheduler.cpp:117-135,
pipeline.cpp:229-244): the sigma schedule and the guided Euler update, restated in the
oracle and in the library's host code, pinned bit for bit to the reference's own
FlowMatchScheduler (golden fixture written by tests/golden/make_golden.py, and the
reference library itself where it is built)."""
import numpy as np
import pytest

from conftest import load_golden


@pytest.fixture(scope="module")
def host():
    """The library's host-side entry points (no device needed)."""
    import sdb200

    sdb200.lib()
    return sdb200


def test_flow_sigmas_match_reference_golden(orc, host):
    g = load_golden("flow_sampler")
    for i, steps in enumerate(g["steps"]):
        for j, shift in enumerate(g["shifts"]):
            want = g["sig"][i, j, :steps + 1]
            assert np.array_equal(orc.flow_sigmas(int(steps), float(shift)), want), (steps, shift)
            assert np.array_equal(host.flow_sigmas(int(steps), float(shift)), want), (steps, shift)


def test_flow_step_matches_reference_golden(orc):
    g = load_golden("flow_sampler")
    sig = orc.flow_sigmas(8, 3.0)
    got = orc.flow_step(g["x"], g["out"], None, 0.0, sig[2] - sig[3])
    assert np.array_equal(got, g["x_plain"])
    got = orc.flow_step(g["x"], g["out"], g["neg"], 2.5, sig[5] - sig[6])
    assert np.array_equal(got, g["x_cfg"])


def test_flow_sampler_vs_reference_library(orc, host, ref):
    for steps in (1, 2, 8, 28, 50):
        for shift in (1.0, 3.0, 4.7):
            want = ref.flow_sigmas(steps, shift)
            assert np.array_equal(orc.flow_sigmas(steps, shift), want)
            assert np.array_equal(host.flow_sigmas(steps, shift), want)


def test_flow_sigmas_rejects_zero_steps(host):
    with pytest.raises(host.SdbError):
        host.flow_sigmas(0, 3.0)
