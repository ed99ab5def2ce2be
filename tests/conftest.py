import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (sm_100a) and the built CUDA library")
    config.addinivalue_line("markers", "slow: full-size parity cases (minutes of CPU oracle time)")


@pytest.fixture(scope="session")
def golden():
    import numpy as np
    return np.load(os.path.join(ROOT, "tests", "golden", "ref_kernels.npz"))


def pytest_terminal_summary(terminalreporter, exitstatus, config):
    """The model-level parity records (tests/modelcheck.py): per compared sequence its steps, the largest logit error
    against the FP64 oracle as a fraction of the bound 0.05 + 0.003|ref|, the argmax agreement with the
    half-transport oracle, the smallest top-2 margin and any miss with its gap and rounding bound."""
    try:
        from tests import modelcheck as MC
    except Exception:
        return
    if not MC.RECORDS:
        return
    import json
    terminalreporter.write_sep("-", "model-level parity records (every step compared)")
    for r in MC.RECORDS:
        terminalreporter.write_line(json.dumps(r, sort_keys=True))
