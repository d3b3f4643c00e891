"""The build's smoke entry point (one fused append + one decode on cuda:0,
checked against the oracle inside), run as the round-end check runs it."""

from __future__ import annotations

import sys
from pathlib import Path

import pytest

pytestmark = pytest.mark.gpu

sys.path.insert(0, str(Path(__file__).resolve().parents[1]))


def test_smoke_entry_point(cuda_lib):
    import __graft_entry__

    __graft_entry__.smoke()
