"""The reference simulator's known-answer scenarios on the CPU oracle.

Pins the oracle (oracle/stratego_oracle.c) against the reference's own CUDA
tests (tests/test_cuda_{sim,api,rules,infostate}.py), restated in
tests/scenarios.py.
"""

from __future__ import annotations

import pytest

from _helpers import OracleRolloutBuffer
from scenarios import SCENARIOS


def _make(n, **kw):
    return OracleRolloutBuffer(n, 0, **kw)


@pytest.mark.parametrize("scenario", SCENARIOS, ids=[s.__name__ for s in SCENARIOS])
def test_oracle_scenario(scenario):
    scenario(_make)
