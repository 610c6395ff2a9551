"""Elementwise ops on tensors past one launch's 2^30 vectors.

The kernels index vectors with 32 bits, so a call on a larger tensor runs as
several launches over consecutive ranges (whole tokens / columns where the op
has them). Unaligned starting pointers force one float per vector, so a few GB
cross the boundary. Each result is compared bitwise with the same op run on
pieces that each fit one launch (the residual add with torch's add: both are
one IEEE rounding per element), and a seeded sample of about 4 million output
elements of each (whole columns / tokens for GeGLU and the bias) is compared
bitwise with the CPU oracle of the reference's arithmetic
(crates/cpu-kernels/src/lib.rs:509-511 GELU, :516-538 GeGLU, :274-288 bias).
"""

import numpy as np
import pytest
import torch

from helpers import assert_bitwise
from tfx import ops

pytestmark = pytest.mark.gpu

ONE_LAUNCH = 1 << 30  # vectors per launch
SAMPLE = 1 << 22      # output elements checked against the oracle


@pytest.fixture(autouse=True)
def _free_memory():
    yield
    torch.cuda.synchronize()
    torch.cuda.empty_cache()


def _normal(n, seed, std=1.0):
    g = torch.Generator(device="cuda")
    g.manual_seed(seed)
    return torch.randn(n, generator=g, device="cuda") * std


def _sample(n, count, seed):
    g = torch.Generator(device="cuda")
    g.manual_seed(seed)
    return torch.randint(0, n, (count,), generator=g, device="cuda")


def _np(t):
    return t.detach().cpu().numpy().reshape(-1)


def test_gelu_past_one_launch_matches_pieces_and_oracle(orc):
    n = ONE_LAUNCH + (1 << 20) + 3
    buf = _normal(n + 1, 11, 1.5)
    x = buf[1:]  # 4-byte offset: one float per vector
    y = ops.gelu_erf(x)
    half = n // 2
    assert torch.equal(y[:half], ops.gelu_erf(x[:half].clone()))
    assert torch.equal(y[half:], ops.gelu_erf(x[half:].clone()))
    idx = _sample(n, SAMPLE, 21)
    idx[:2] = torch.tensor([0, n - 1], device="cuda")  # both ends of the tensor
    assert_bitwise(_np(y[idx]), orc.gelu_erf_f32(_np(x[idx])), "gelu > 2^30 vectors sample")


def test_add_past_two_launches_matches_torch_and_oracle(orc):
    n = 2 * ONE_LAUNCH + 5
    a = _normal(n + 1, 12)[1:]
    b = _normal(n + 1, 13)[1:]
    y = ops.add(a, b)
    assert torch.equal(y, a + b)
    idx = _sample(n, SAMPLE, 22)
    idx[:2] = torch.tensor([0, n - 1], device="cuda")
    assert_bitwise(_np(y[idx]), orc.add_f32(_np(a[idx]), _np(b[idx])), "add sample")


def test_geglu_column_chunks_past_one_launch_and_oracle(orc):
    inter = 1153  # odd: one float per vector
    cols = ONE_LAUNCH // inter + 7
    u = _normal(2 * inter * cols, 14, 1.5)
    y = ops.geglu(u, inter).reshape(-1)
    c = cols // 2
    assert torch.equal(y[: c * inter], ops.geglu(u[: 2 * c * inter].clone(), inter).reshape(-1))
    assert torch.equal(y[c * inter:], ops.geglu(u[2 * c * inter:].clone(), inter).reshape(-1))
    ncol = SAMPLE // inter
    cs = _sample(cols, ncol, 23)
    cs[:2] = torch.tensor([0, cols - 1], device="cuda")
    us = u.view(cols, 2 * inter)[cs]
    ys = y.view(cols, inter)[cs]
    assert_bitwise(_np(ys), orc.geglu_f32(_np(us), inter, ncol), "geglu column sample")


def test_bias_token_chunks_past_one_launch_and_oracle(orc):
    features = 769  # odd: one float per vector
    tokens = ONE_LAUNCH // features + 11
    x = _normal(features * tokens, 15)
    bias = _normal(features, 16, 0.02)
    y = ops.bias_act(x, bias, features=features)
    assert torch.equal(y.view(tokens, features), x.view(tokens, features) + bias[None, :])
    ntok = SAMPLE // features
    ts = _sample(tokens, ntok, 24)
    ts[:2] = torch.tensor([0, tokens - 1], device="cuda")
    xs = x.view(tokens, features)[ts]
    ys = y.view(tokens, features)[ts]
    assert_bitwise(_np(ys), orc.bias_act_f32(_np(xs), _np(bias), features, ntok, 0),
                   "bias token sample")
