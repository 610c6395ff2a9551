"""GPU parity: feature-first LayerNorm and feature-last RMSNorm (f32, f64).

The GPU sums in a tree, the reference sequentially, so these compare within
the f32 tolerance |a - r| <= 1e-6*max|r| + 1e-5*|r| (f64: 1e-14, 1e-12)."""

import math

import numpy as np
import pytest
import torch

from gpu_util import P, S, call, dev, empty, host, f32, f64
from helpers import (golden_case, golden_tensor, assert_close, lcg_f32, splitmix_normal,
                     splitmix_uniform, F32_RTOL, F32_ATOL_REL, F64_RTOL, F64_ATOL_REL)

pytestmark = pytest.mark.gpu


def gpu_ln(x, w, b, d, cols, eps, offset=0, in_place=False):
    xd = dev(x, offset)
    wd = dev(w)
    bd = dev(b) if b is not None else None
    dtype = torch.float32 if x.dtype == np.float32 else torch.float64
    yd = xd if in_place else empty(d * cols, dtype=dtype, offset_elems=offset)
    fn = "tfx_layernorm_ff_f32" if x.dtype == np.float32 else "tfx_layernorm_ff_f64"
    call(fn, P(xd), P(wd), P(bd), P(yd), d, cols, (f32 if x.dtype == np.float32 else f64)(eps), S())
    return host(yd)


def test_layernorm_config1_full_size(orc):
    """768 x 8192, X ~ N(0,1), gamma ~ U(0.5, 1.5), no bias, eps 1e-5."""
    d, cols = 768, 8192
    x = splitmix_normal(d * cols, 0x7E4F0000)
    w = splitmix_uniform(d, 0x7E4F0001, 0.5, 1.5)
    got = gpu_ln(x, w, None, d, cols, 1e-5)
    st = assert_close(got, orc.layer_norm_feature_first_f32(x, d, cols, w, None, 1e-5),
                      F32_RTOL, F32_ATOL_REL, "layernorm config 1")
    assert st["max_abs"] < 1e-5


def test_layernorm_f64_config1_full_size(orc):
    d, cols = 768, 8192
    x = splitmix_normal(d * cols, 0x7E4F0000, dtype=np.float64)
    w = splitmix_uniform(d, 0x7E4F0001, 0.5, 1.5, dtype=np.float64)
    got = gpu_ln(x, w, None, d, cols, 1e-5)
    assert_close(got, orc.layer_norm_feature_first_f64(x, d, cols, w, None, 1e-5), F64_RTOL,
                 F64_ATOL_REL, "layernorm f64 config 1")


def test_layernorm_reference_lcg_cases(orc):
    """crates/tenferro-ext/src/layernorm.rs:319-376: naive check, diff < 1e-5."""
    c = golden_case("layernorm_ff_matches_naive")
    for d, l, b in c["shapes"]:
        state = c["lcg"]["seed"]
        x, state = lcg_f32(state, d * l * b)
        w, state = lcg_f32(state, d)
        bias, state = lcg_f32(state, d)
        for bias_in in (None, bias):
            got = gpu_ln(x, w, bias_in, d, l * b, c["eps"])
            want = orc.layer_norm_feature_first_f32(x, d, l * b, w, bias_in, c["eps"])
            assert np.max(np.abs(got - want)) < c["tolerance"]["abs"]


def test_layernorm_f64_primitive(orc):
    c = golden_case("layer_norm_f64_primitive")
    rows, cols, eps = c["rows"], c["cols"], c["eps"]
    x = np.ascontiguousarray(golden_tensor(c, "x").reshape(cols, rows).T).ravel()
    w, b = golden_tensor(c, "weight"), golden_tensor(c, "bias")
    got = gpu_ln(x, w, b, cols, rows, eps).reshape(rows, cols)
    xv = x.reshape(rows, cols)
    for i in range(rows):
        mean = sum(xv[i]) / cols
        var = sum((xv[i] - mean) ** 2) / cols
        want = (xv[i] - mean) * (1.0 / math.sqrt(var + eps)) * w + b
        assert np.max(np.abs(got[i] - want)) <= c["tolerance"]["abs"]


@pytest.mark.parametrize("d,cols,offset,bias", [
    (1, 5, 0, True), (2, 3, 0, False), (31, 7, 0, True), (33, 9, 1, True), (64, 1, 0, True),
    (767, 13, 0, True), (769, 11, 0, False), (768, 3, 1, True), (1024, 8, 0, True),
    (1025, 4, 0, True), (2048, 3, 0, False), (4100, 2, 0, True), (8192, 2, 0, True),
    (8196, 2, 0, True), (10000, 2, 0, False)])
def test_layernorm_shapes(orc, d, cols, offset, bias):
    x = splitmix_normal(d * cols, 0x7E4F0400 + d, std=2.0)
    w = splitmix_uniform(d, 0x7E4F0401 + d, 0.5, 1.5)
    b = splitmix_normal(d, 0x7E4F0402 + d, std=0.1) if bias else None
    got = gpu_ln(x, w, b, d, cols, 1e-5, offset)
    assert_close(got, orc.layer_norm_feature_first_f32(x, d, cols, w, b, 1e-5), F32_RTOL,
                 F32_ATOL_REL, f"layernorm d={d}")
    x64, w64 = x.astype(np.float64), w.astype(np.float64)
    b64 = b.astype(np.float64) if bias else None
    got64 = gpu_ln(x64, w64, b64, d, cols, 1e-5, offset)
    assert_close(got64, orc.layer_norm_feature_first_f64(x64, d, cols, w64, b64, 1e-5), F64_RTOL,
                 F64_ATOL_REL, f"layernorm f64 d={d}")


def test_layernorm_in_place(orc):
    d, cols = 768, 100
    x = splitmix_normal(d * cols, 0x7E4F0410)
    w = splitmix_uniform(d, 0x7E4F0411, 0.5, 1.5)
    got = gpu_ln(x, w, None, d, cols, 1e-5, in_place=True)
    assert_close(got, orc.layer_norm_feature_first_f32(x, d, cols, w, None, 1e-5), F32_RTOL,
                 F32_ATOL_REL, "layernorm in place")


def test_layernorm_errors():
    import tfx
    x = empty(16)
    with pytest.raises(tfx.TfxError) as e:
        call("tfx_layernorm_ff_f32", P(x), None, None, P(x), 8, 2, f32(1e-5), S())
    assert "tenferro-ext::layernorm_ff: weight: null pointer" in str(e.value)
    call("tfx_layernorm_ff_f32", None, None, None, None, 0, 2, f32(1e-5), S())  # empty: no-op


# ---- RMSNorm --------------------------------------------------------------------

def gpu_rms(x, w, rows, width, centered, eps, offset=0, in_place=False):
    xd, wd = dev(x, offset), dev(w)
    dtype = torch.float32 if x.dtype == np.float32 else torch.float64
    yd = xd if in_place else empty(rows * width, dtype=dtype, offset_elems=offset)
    fn = "tfx_rmsnorm_last_f32" if x.dtype == np.float32 else "tfx_rmsnorm_last_f64"
    call(fn, P(xd), P(wd), P(yd), rows, width, int(centered),
         (f32 if x.dtype == np.float32 else f64)(eps), S())
    return host(yd)


@pytest.mark.parametrize("centered", [True, False])
def test_rmsnorm_config3_full_size(orc, centered):
    """hidden 1024, 16384 tokens, eps 1e-6, w ~ N(1, 0.1)."""
    rows, width = 16384, 1024
    x = splitmix_normal(rows * width, 0x7E4F0020)
    w = splitmix_normal(width, 0x7E4F0021, mean=1.0, std=0.1)
    eps = float(np.float32(1e-6))  # the ext trait truncates its f64 eps to f32
    got = gpu_rms(x, w, rows, width, centered, eps)
    assert_close(got, orc.rms_norm_last_f32(x, rows, width, w, centered, eps), F32_RTOL,
                 F32_ATOL_REL, "rmsnorm config 3")


@pytest.mark.parametrize("rows,width,offset", [
    (1, 1, 0), (3, 4, 0), (63, 31, 0), (64, 1024, 1), (257, 100, 0), (130, 1025, 0),
    (128, 2048, 0), (100, 4096, 0), (96, 4100, 0), (64, 8192, 0), (10, 9000, 0), (4, 3, 1),
    (4, 3, 0), (100, 200, 0), (1000, 1000, 0), (1600, 1400, 0), (20000, 64, 0), (16, 768, 0),
    (300, 3000, 0), (64, 2500, 0), (3000, 520, 0)])
def test_rmsnorm_shapes(orc, rows, width, offset):
    x = splitmix_normal(rows * width, 0x7E4F0500 + rows + width)
    w = splitmix_normal(width, 0x7E4F0501 + width, mean=1.0, std=0.1)
    for centered in (True, False):
        got = gpu_rms(x, w, rows, width, centered, 1e-6, offset)
        assert_close(got, orc.rms_norm_last_f32(x, rows, width, w, centered, 1e-6), F32_RTOL,
                     F32_ATOL_REL, f"rmsnorm {rows}x{width}")
        x64, w64 = x.astype(np.float64), w.astype(np.float64)
        got64 = gpu_rms(x64, w64, rows, width, centered, 1e-6, offset)
        assert_close(got64, orc.rms_norm_last_f64(x64, rows, width, w64, centered, 1e-6),
                     F64_RTOL, F64_ATOL_REL, f"rmsnorm f64 {rows}x{width}")


def test_rmsnorm_in_place(orc):
    rows, width = 4096, 1024
    x = splitmix_normal(rows * width, 0x7E4F0510)
    w = splitmix_normal(width, 0x7E4F0511, mean=1.0, std=0.1)
    got = gpu_rms(x, w, rows, width, True, 1e-6, in_place=True)
    assert_close(got, orc.rms_norm_last_f32(x, rows, width, w, True, 1e-6), F32_RTOL,
                 F32_ATOL_REL, "rmsnorm in place")


def test_no_wait_gave_up():
    """Every bounded wait of the TMA-pipelined kernels completed in the runs above."""
    import ctypes
    from tfx import _lib
    n = ctypes.c_uint32(99)
    call("tfx_wait_timeouts", ctypes.byref(n))
    assert n.value == 0


def test_rmsnorm_f64_primitives(orc):
    c = golden_case("rms_norm_f64_primitive")
    rows, cols, eps = c["rows"], c["cols"], c["eps"]
    x, w = golden_tensor(c, "x"), golden_tensor(c, "weight")
    for centered in (False, True):
        got = gpu_rms(x, w, rows, cols, centered, eps)
        want = np.empty_like(x)
        for i in range(rows):
            inv = 1.0 / math.sqrt(sum(x[i + j * rows] ** 2 for j in range(cols)) / cols + eps)
            for j in range(cols):
                want[i + j * rows] = x[i + j * rows] * inv * ((1.0 + w[j]) if centered else w[j])
        assert np.max(np.abs(got - want)) <= c["tolerance"]["abs"]
