"""GPU parity: gated SiLU (two-input and stacked) and the residual add."""

import numpy as np
import pytest

from gpu_util import P, S, call, dev, empty, host
from helpers import assert_bitwise, assert_close, splitmix_normal, F32_RTOL, F32_ATOL_REL

pytestmark = pytest.mark.gpu


def test_gated_silu_config3_full_size(orc):
    """gate, up ~ N(0,1), 16384 x 3584. CUDA expf vs glibc expf
    differ by at most an ulp or two; the tolerance is the f32 bar."""
    n = 16384 * 3584
    g = splitmix_normal(n, 0x7E4F0022)
    u = splitmix_normal(n, 0x7E4F0023)
    gd, ud, yd = dev(g), dev(u), empty(n)
    call("tfx_gated_silu_f32", P(gd), P(ud), P(yd), n, S())
    st = assert_close(host(yd), orc.gated_silu_f32(g, u), F32_RTOL, F32_ATOL_REL, "silu config 3")
    assert st["max_ulp"] <= 8


@pytest.mark.parametrize("n,offset", [(1, 0), (7, 1), (4097, 2), (10001, 3)])
def test_gated_silu_odd(orc, n, offset):
    g = splitmix_normal(n, 0x7E4F0700 + n, std=4.0)
    u = splitmix_normal(n, 0x7E4F0701 + n)
    gd, ud, yd = dev(g, offset), dev(u, offset), empty(n, offset_elems=offset)
    call("tfx_gated_silu_f32", P(gd), P(ud), P(yd), n, S())
    assert_close(host(yd), orc.gated_silu_f32(g, u), F32_RTOL, F32_ATOL_REL, "silu odd")


def test_gated_silu_stacked(orc):
    """FusedScope::gated_silu_stacked: gu (rows, 2*inter) column-major, gate | up."""
    rows, inter = 257, 3584
    gu = splitmix_normal(rows * 2 * inter, 0x7E4F0710)
    gd, yd = dev(gu), empty(rows * inter)
    call("tfx_gated_silu_stacked_f32", P(gd), P(yd), rows, inter, S())
    g, u = gu[:rows * inter], gu[rows * inter:]
    assert_close(host(yd), orc.gated_silu_f32(g, u), F32_RTOL, F32_ATOL_REL, "silu stacked")


def test_gated_silu_in_place(orc):
    n = 1 << 20
    g = splitmix_normal(n, 0x7E4F0720)
    u = splitmix_normal(n, 0x7E4F0721)
    gd, ud = dev(g), dev(u)
    call("tfx_gated_silu_f32", P(gd), P(ud), P(gd), n, S())
    assert_close(host(gd), orc.gated_silu_f32(g, u), F32_RTOL, F32_ATOL_REL, "silu in place")


@pytest.mark.parametrize("n,offset", [(768 * 32768, 0), (5, 1), (1023, 2)])
def test_residual_add_bitwise(orc, n, offset):
    a = splitmix_normal(n, 0x7E4F0730 + n)
    b = splitmix_normal(n, 0x7E4F0731 + n)
    ad, bd, yd = dev(a, offset), dev(b, offset), empty(n, offset_elems=offset)
    call("tfx_add_f32", P(ad), P(bd), P(yd), n, S())
    assert_bitwise(host(yd), orc.add_f32(a, b), "add")
