"""GPU parity: the residual add fused into the feature-first LayerNorm is
bit-identical to the two ops run separately, and within the f32 tolerance of
the oracle's add then LayerNorm."""

import ctypes

import numpy as np
import pytest
import torch

from gpu_util import P, S, call, dev, empty, host
from helpers import assert_bitwise, assert_close, splitmix_normal, splitmix_uniform, F32_RTOL, F32_ATOL_REL

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("d,cols,with_bias,with_sum,offset", [
    (768, 2048, False, True, 0), (768, 1001, True, True, 0), (1024, 300, False, False, 0),
    (64, 77, True, True, 0), (2048, 40, False, True, 0), (768, 50, False, True, 1),
    (6, 9, True, True, 0)])
def test_add_layernorm_matches_unfused(orc, d, cols, with_bias, with_sum, offset):
    n = d * cols
    a = splitmix_normal(n, 0x7E4F0B00 + d)
    b = splitmix_normal(n, 0x7E4F0B01 + d, std=0.5)
    w = splitmix_uniform(d, 0x7E4F0B02, 0.5, 1.5)
    bias = splitmix_normal(d, 0x7E4F0B03, std=0.1) if with_bias else None
    ad, bd, wd = dev(a, offset), dev(b, offset), dev(w)
    biasd = dev(bias) if with_bias else None
    s_f = empty(n, offset_elems=offset) if with_sum else None
    y_f = empty(n, offset_elems=offset)
    call("tfx_add_layernorm_ff_f32", P(ad), P(bd), P(wd), P(biasd), P(s_f), P(y_f), d, cols,
         ctypes.c_float(1e-5), S())
    s_u, y_u = empty(n, offset_elems=offset), empty(n, offset_elems=offset)
    call("tfx_add_f32", P(ad), P(bd), P(s_u), n, S())
    call("tfx_layernorm_ff_f32", P(s_u), P(wd), P(biasd), P(y_u), d, cols, ctypes.c_float(1e-5),
         S())
    assert_bitwise(host(y_f), host(y_u), "fused y vs add then LayerNorm")
    if with_sum:
        assert_bitwise(host(s_f), host(s_u), "fused sum vs add")
    want = orc.layer_norm_feature_first_f32(orc.add_f32(a, b), d, cols, w, bias, 1e-5)
    assert_close(host(y_f), want, F32_RTOL, F32_ATOL_REL, "fused vs oracle")


def test_add_layernorm_in_place_residual(orc):
    """sum_out == a: the residual stream updated in place (x += attn), y beside it."""
    d, cols = 768, 513
    n = d * cols
    a = splitmix_normal(n, 0x7E4F0B10)
    b = splitmix_normal(n, 0x7E4F0B11)
    w = splitmix_uniform(d, 0x7E4F0B12, 0.5, 1.5)
    ad, bd, wd, y = dev(a), dev(b), dev(w), empty(n)
    call("tfx_add_layernorm_ff_f32", P(ad), P(bd), P(wd), None, P(ad), P(y), d, cols,
         ctypes.c_float(1e-5), S())
    s = orc.add_f32(a, b)
    assert_bitwise(host(ad), s, "in-place sum")
    assert_close(host(y), orc.layer_norm_feature_first_f32(s, d, cols, w, None, 1e-5), F32_RTOL,
                 F32_ATOL_REL, "in-place y")
