"""Runs after every other GPU test but the no-allocation MoE entry's (which
is collected last and checks its own bits): no kernel's time-bounded wait
gave up and the VQ kernel's shared-memory layout check held
(graft_device_errors)."""
from __future__ import annotations

import pytest

pytestmark = pytest.mark.gpu


def test_no_device_errors_after_the_suite(lib):
    import kernels_b200 as kb
    assert kb.device_errors(clear=True) == {"int4": 0, "vq": 0, "moe": 0}
