"""Elementwise ops on tensors past one launch's 2^30 vectors.

The kernels index vectors with 32 bits, so a call on a larger tensor runs as
several launches over consecutive ranges (whole tokens / columns where the op
has them). Unaligned starting pointers force one float per vector, so a few GB
cross the boundary. Each result is compared bitwise with the same op run on
pieces that each fit one launch, and the residual add with torch's add (both
are one IEEE rounding per element), all on the device.
"""

import pytest
import torch

from tfx import ops

pytestmark = pytest.mark.gpu

ONE_LAUNCH = 1 << 30  # vectors per launch


@pytest.fixture(autouse=True)
def _free_memory():
    yield
    torch.cuda.synchronize()
    torch.cuda.empty_cache()


def _normal(n, seed, std=1.0):
    g = torch.Generator(device="cuda")
    g.manual_seed(seed)
    return torch.randn(n, generator=g, device="cuda") * std


def test_gelu_past_one_launch_matches_pieces():
    n = ONE_LAUNCH + (1 << 20) + 3
    buf = _normal(n + 1, 11, 1.5)
    x = buf[1:]  # 4-byte offset: one float per vector
    y = ops.gelu_erf(x)
    half = n // 2
    assert torch.equal(y[:half], ops.gelu_erf(x[:half].clone()))
    assert torch.equal(y[half:], ops.gelu_erf(x[half:].clone()))


def test_add_past_two_launches_matches_torch():
    n = 2 * ONE_LAUNCH + 5
    a = _normal(n + 1, 12)[1:]
    b = _normal(n + 1, 13)[1:]
    assert torch.equal(ops.add(a, b), a + b)


def test_geglu_column_chunks_past_one_launch():
    inter = 1153  # odd: one float per vector
    cols = ONE_LAUNCH // inter + 7
    u = _normal(2 * inter * cols, 14, 1.5)
    y = ops.geglu(u, inter).reshape(-1)
    c = cols // 2
    assert torch.equal(y[: c * inter], ops.geglu(u[: 2 * c * inter].clone(), inter).reshape(-1))
    assert torch.equal(y[c * inter:], ops.geglu(u[2 * c * inter:].clone(), inter).reshape(-1))


def test_bias_token_chunks_past_one_launch():
    features = 769  # odd: one float per vector
    tokens = ONE_LAUNCH // features + 11
    x = _normal(features * tokens, 15)
    bias = _normal(features, 16, 0.02)
    y = ops.bias_act(x, bias, features=features)
    assert torch.equal(y.view(tokens, features), x.view(tokens, features) + bias[None, :])
