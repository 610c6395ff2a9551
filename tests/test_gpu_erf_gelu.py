"""GPU parity: erf / exact GELU / GeGLU / bias-GELU against the oracle.

The f32 path computes the reference's own operations (tfx_math.h), so every
comparison here is bitwise (the north-star bar of <= 4 ulp is met at 0 ulp)."""

import numpy as np
import pytest

from gpu_util import P, S, call, dev, empty, host, f32
from helpers import (golden_case, golden_tensor, assert_bitwise, assert_close, splitmix_normal,
                     decode_value, F64_RTOL, F64_ATOL_REL)

pytestmark = pytest.mark.gpu


def gpu_unary(name, x, offset=0):
    xd = dev(x, offset)
    yd = empty(x.size, offset_elems=offset)
    call(name, P(xd), P(yd), x.size, S())
    return host(yd)


def test_known_values(orc):
    c = golden_case("erf_f32_mlx_known_values")
    x, want = golden_tensor(c, "x"), golden_tensor(c, "erf")
    got = gpu_unary("tfx_erf_f32", x)
    assert np.max(np.abs(got - want)) < c["tolerance"]["abs"]
    c = golden_case("gelu_erf_f32_known_values")
    x, want = golden_tensor(c, "x"), golden_tensor(c, "gelu")
    got = gpu_unary("tfx_gelu_erf_f32", x)
    assert np.max(np.abs(got - want)) < c["tolerance"]["abs"]


def test_special_values(orc):
    c = golden_case("erf_f32_special_values")
    x = golden_tensor(c, "x")
    got = gpu_unary("tfx_erf_f32", x)
    assert_bitwise(got, orc.erf_f32(x), "erf specials")
    assert got[1].tobytes() == np.float32(-0.0).tobytes()
    assert np.isnan(got[6])
    g = gpu_unary("tfx_gelu_erf_f32", x)
    assert_bitwise(g, orc.gelu_erf_f32(x), "gelu specials")


def test_reference_sweeps_bitwise(orc):
    """The sweeps of crates/tenferro-ext/tests/erf.rs:57-83, :132-145 and
    erf_cuda.rs:12-79 (which allow 1e-6 / 2e-6 / 4e-6) -- here 0 ulp."""
    c = golden_case("erf_f32_branch_boundary_sweep")
    sw = c["sweep"]
    x = np.arange(sw["start"], sw["stop"] + 1, dtype=np.float32) * np.float32(sw["step"])
    bb = np.float32(c["boundary"]).view(np.uint32)
    edge = np.array([bb - 1, bb, bb + 1], dtype=np.uint32).view(np.float32)
    extra = np.array([decode_value(v) for v in c["extra"]], dtype=np.float32)
    x = np.concatenate([x, edge, -edge, extra])
    assert_bitwise(gpu_unary("tfx_erf_f32", x), orc.erf_f32(x), "erf boundary sweep")
    c = golden_case("gelu_erf_native_composition_sweep")
    sw = c["sweep"]
    x = np.arange(sw["start"], sw["stop"] + 1, dtype=np.float32) * np.float32(sw["step"])
    assert_bitwise(gpu_unary("tfx_gelu_erf_f32", x), orc.gelu_erf_f32(x), "gelu sweep")
    c = golden_case("erf_gelu_cuda_sweep")
    sw = c["sweep"]
    base = np.arange(sw["start"], sw["stop"] + 1, dtype=np.float32) * np.float32(sw["step"])
    for scale in c["scales"]:
        x = (base * np.float32(scale)).astype(np.float32)
        assert_bitwise(gpu_unary("tfx_erf_f32", x), orc.erf_f32(x), f"erf scale {scale}")
        assert_bitwise(gpu_unary("tfx_gelu_erf_f32", x), orc.gelu_erf_f32(x), f"gelu {scale}")


def test_bit_pattern_sample_bitwise(orc):
    """2^26 f32 bit patterns spread over the whole space (every 64th pattern,
    with a per-run offset), through the packed vector path."""
    bits = (np.arange(0, 1 << 32, 64, dtype=np.uint64) + 37).astype(np.uint32)
    x = bits.view(np.float32)
    assert_bitwise(gpu_unary("tfx_erf_f32", x), orc.erf_f32(x), "erf bit sample")
    assert_bitwise(gpu_unary("tfx_gelu_erf_f32", x), orc.gelu_erf_f32(x), "gelu bit sample")


@pytest.mark.parametrize("n,offset", [(1, 0), (3, 0), (5, 1), (1027, 1), (1026, 2), (4099, 3)])
def test_odd_sizes_and_alignment(orc, n, offset):
    x = splitmix_normal(n, 0x7E4F0100 + n, std=1.5)
    assert_bitwise(gpu_unary("tfx_erf_f32", x, offset), orc.erf_f32(x), "erf")
    assert_bitwise(gpu_unary("tfx_gelu_erf_f32", x, offset), orc.gelu_erf_f32(x), "gelu")


def test_gelu_config2_full_size(orc):
    """standalone exact GELU on 2304 x 8192, X ~ N(0, 1.5)."""
    x = splitmix_normal(2304 * 8192, 0x7E4F0010, std=1.5)
    assert_bitwise(gpu_unary("tfx_gelu_erf_f32", x), orc.gelu_erf_f32(x), "gelu config 2")


def test_geglu_config2_full_size(orc):
    """GeGLU (2304, 8192) -> (1152, 8192)."""
    inter, cols = 1152, 8192
    u = splitmix_normal(2 * inter * cols, 0x7E4F0011, std=1.5)
    ud, yd = dev(u), empty(inter * cols)
    call("tfx_geglu_ff_f32", P(ud), P(yd), inter, cols, S())
    assert_bitwise(host(yd), orc.geglu_f32(u, inter, cols), "geglu config 2")


@pytest.mark.parametrize("inter,cols,offset", [(257, 65, 0), (258, 3, 2), (4, 1, 0), (1, 7, 1)])
def test_geglu_odd_shapes(orc, inter, cols, offset):
    """Includes the uneven (257, 65) shape of crates/cpu-kernels/src/lib.rs:1375-1402."""
    if (inter, cols) == (257, 65):
        i = np.arange(2 * inter * cols)
        u = (((i % 103).astype(np.float32) - np.float32(51.0)) / np.float32(7.0)).astype(np.float32)
    else:
        u = splitmix_normal(2 * inter * cols, 0x7E4F0200 + inter, std=1.5)
    ud, yd = dev(u, offset), empty(inter * cols, offset_elems=offset)
    call("tfx_geglu_ff_f32", P(ud), P(yd), inter, cols, S())
    assert_bitwise(host(yd), orc.geglu_f32(u, inter, cols), f"geglu {inter}x{cols}")


def test_geglu_rejects_overlap():
    import tfx
    u = empty(2 * 8 * 4)
    with pytest.raises(tfx.TfxError) as e:
        call("tfx_geglu_ff_f32", P(u), P(u), 8, 4, S())
    assert "overlap" in str(e.value)


@pytest.mark.parametrize("act", [0, 1, 2])
def test_bias_act_config4_full_size(orc, act):
    """bias (768) ~ N(0, 0.02) onto [8192, 768] ~ N(0, 1)."""
    F, T = 768, 8192
    x = splitmix_normal(F * T, 0x7E4F0030)
    b = splitmix_normal(F, 0x7E4F0031, std=0.02)
    xd, bd, yd = dev(x), dev(b), empty(F * T)
    call("tfx_bias_act_ff_f32", P(xd), P(bd), P(yd), F, T, act, S())
    assert_bitwise(host(yd), orc.bias_act_f32(x, b, F, T, act), f"bias act {act}")
    if act == 0:
        assert_bitwise(host(yd), orc.bias_add_f32(x, b, F, T), "bias add")


@pytest.mark.parametrize("F,T,offset,with_bias", [(7, 5, 0, True), (6, 3, 1, True), (8, 9, 0, False),
                                                  (768, 3, 2, True)])
def test_bias_act_odd(orc, F, T, offset, with_bias):
    x = splitmix_normal(F * T, 0x7E4F0300 + F)
    b = splitmix_normal(F, 0x7E4F0301 + F, std=0.02) if with_bias else None
    xd, yd = dev(x, offset), empty(F * T, offset_elems=offset)
    bd = dev(b) if with_bias else None
    call("tfx_bias_act_ff_f32", P(xd), P(bd), P(yd), F, T, 1, S())
    assert_bitwise(host(yd), orc.bias_act_f32(x, b, F, T, 1), "bias gelu odd")


def test_bias_in_place(orc):
    F, T = 768, 64
    x = splitmix_normal(F * T, 0x7E4F0310)
    b = splitmix_normal(F, 0x7E4F0311, std=0.02)
    xd, bd = dev(x), dev(b)
    call("tfx_bias_act_ff_f32", P(xd), P(bd), P(xd), F, T, 0, S())
    assert_bitwise(host(xd), orc.bias_add_f32(x, b, F, T), "bias in place")


def test_erf_f64_matches_oracle(orc):
    """crates/tenferro-ext/tests/erf.rs:106-129 sweep, |diff| <= 5e-16."""
    c = golden_case("erf_f64_native_sweep")
    sw = c["sweep"]
    x = np.arange(sw["start"], sw["stop"] + 1) * sw["step"]
    xd, yd = dev(x), empty(x.size, dtype=__import__("torch").float64)
    call("tfx_erf_f64", P(xd), P(yd), x.size, S())
    got = host(yd)
    assert np.max(np.abs(got - orc.erf_f64(x))) <= c["tolerance"]["abs"]
    call("tfx_gelu_erf_f64", P(xd), P(yd), x.size, S())
    got = host(yd)
    assert_close(got, orc.gelu_erf_f64(x), F64_RTOL, F64_ATOL_REL, "gelu f64")
    assert got[np.argmin(np.abs(x))] == 0.0
