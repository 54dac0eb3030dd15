"""The reference simulator's known-answer scenarios on the B200 buffer.

Same scenarios as tests/test_oracle_scenarios.py (restated from the
reference's tests/test_cuda_*.py), run through ataraxos_b200's
StrategoRolloutBuffer, i.e. through libstratego_b200.so's C ABI.
"""

from __future__ import annotations

import pytest

from scenarios import SCENARIOS

pytestmark = pytest.mark.gpu


def _make(n, **kw):
    from ataraxos_b200 import StrategoRolloutBuffer

    return StrategoRolloutBuffer(n, 0, **kw)


@pytest.mark.parametrize("scenario", SCENARIOS, ids=[s.__name__ for s in SCENARIOS])
def test_gpu_scenario(scenario):
    scenario(_make)
