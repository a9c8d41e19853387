"""CPU checks of the input-gradient restatement: it is the adjoint of the forward oracle (whose
weight decode and rotation are pinned to the reference's golden vectors), so
<dy, linear(x)> == <grad_input(dy), x> for every x and dy."""
import numpy as np
import pytest

from oracle import qlin_oracle as O


@pytest.mark.parametrize("group", [0, 32, 64, 128, 256])
def test_grad_input_is_the_adjoint_of_the_forward(group):
    rng = np.random.default_rng(group + 1)
    m, n, k = 5, 48, 512
    q = rng.integers(-127, 128, (n, k)).astype(np.int8)
    s = (np.abs(rng.normal(0, 0.02, n)) / 127).astype(np.float32)
    x = rng.normal(size=(m, k))
    dy = rng.normal(size=(m, n))
    w_rot = q.astype(np.float64) * s.astype(np.float64)[:, None]
    y = (O.rotate_rows(x, group) if group else x) @ w_rot.T  # forward: rot(x) . (q * s)^T
    dx = O.int8_grad_input(dy, q, s, group)
    assert dx.shape == (m, k)
    lhs, rhs = float(np.sum(dy * y)), float(np.sum(dx * x))
    assert abs(lhs - rhs) <= 1e-9 * max(1.0, abs(lhs))
