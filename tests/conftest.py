import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG = os.path.join(ROOT, "mac-kernels-public_b200")
TESTS = os.path.join(ROOT, "tests")
for p in (ROOT, PKG, TESTS):
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (sm_100a) GPU; parity tests through the C-ABI")
    config.addinivalue_line("markers", "slow: longer CPU test")


@pytest.fixture(autouse=True)
def _poison_uninitialized_memory(request):
    """GPU tests run with every fresh torch allocation poisoned: floating-point tensors from
    torch.empty are filled with NaN and integer tensors with their maximum value (PyTorch's
    deterministic mode with fill_uninitialized_memory).  Outputs, workspaces and caches the
    library is handed therefore never hold an earlier result, so a kernel that skips a store or
    reads a workspace entry it never wrote shows up as a NaN or a wrong value instead of passing on
    a recycled allocation.  warn_only keeps library ops without a deterministic variant usable."""
    if request.node.get_closest_marker("gpu") is None:
        yield
        return
    import torch
    prev = torch.are_deterministic_algorithms_enabled()
    prev_warn = torch.is_deterministic_algorithms_warn_only_enabled()
    prev_fill = torch.utils.deterministic.fill_uninitialized_memory
    torch.use_deterministic_algorithms(True, warn_only=True)
    torch.utils.deterministic.fill_uninitialized_memory = True
    try:
        yield
    finally:
        torch.utils.deterministic.fill_uninitialized_memory = prev_fill
        torch.use_deterministic_algorithms(prev, warn_only=prev_warn)
