import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)
sys.path.insert(0, os.path.join(ROOT, "oracle"))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (B200, sm_100a)")
    config.addinivalue_line("markers", "slow: full-size model parity (minutes of oracle CPU time)")


@pytest.fixture(scope="session")
def built():
    """Native libraries built in-tree (nvcc cross-compiles without a GPU)."""
    from arm_ai_b200 import build
    build.build()
    import build as oracle_build  # oracle/build.py
    oracle_build.build()
    return True


@pytest.fixture(scope="session")
def tiny_model(built):
    from arm_ai_b200 import synth
    return synth.model_path("tiny", seed=1)


@pytest.fixture(scope="session")
def small_model(built):
    from arm_ai_b200 import synth
    return synth.model_path("small", seed=2)


@pytest.fixture(scope="session")
def tied_model(built):
    from arm_ai_b200 import synth
    return synth.model_path("tiny", seed=3, tie_output=True)


@pytest.fixture(scope="session")
def tp4_model(built):
    from arm_ai_b200 import synth
    return synth.model_path("tp4", seed=5)


@pytest.fixture(scope="session")
def hd128_model(built):
    from arm_ai_b200 import synth
    return synth.model_path("tiny128", seed=4)


# Measured parity figures that tests record (e.g. the benchmarked
# configuration's logit error and greedy-id agreement), printed at the end of
# the run so that the summary of a quiet (-q) run carries them.
PARITY_REPORT: list[str] = []


@pytest.fixture(scope="session")
def parity_report():
    return PARITY_REPORT


def pytest_terminal_summary(terminalreporter, exitstatus, config):
    if PARITY_REPORT:
        terminalreporter.section("parity report")
        for line in PARITY_REPORT:
            terminalreporter.write_line(line)
