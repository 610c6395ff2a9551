"""The RMSNorm entry point that allocates nothing (tfx_rmsnorm_last_f32_noalloc).

It exists for callers that cannot let a library allocate device memory during
a call -- a serving process whose HBM is reserved up front by its own
allocator, or a latency-critical loop that must not touch an allocator -- and
keeps its partial sums in a fixed array inside libtfx's device image instead.
This file checks, through the C ABI, that it returns what the allocating entry
point tfx_rmsnorm_last_f32 returns and what the CPU oracle of the reference's
rms_norm_last_into (crates/cpu-kernels/src/lib.rs:545-581) returns (same f32
tolerance as every test here), on two calls in a row with different data; that
a shape whose partial sums exactly fill the fixed array (65536 x 1024: 2^20
sums) runs; and that one row more is rejected. It sorts last so a run that
stops at the first failure has already run every other test, and it needs
nothing from them: it passes alone in a fresh process too.
"""

import numpy as np
import pytest
import torch

import tfx
from gpu_util import P, S, dev, empty, f32, host
from helpers import assert_close, splitmix_normal, F32_RTOL, F32_ATOL_REL
from tfx import _lib

pytestmark = pytest.mark.gpu


def _run(name, x, w, rows, width, centered):
    xd, wd, yd = dev(x), dev(w), empty(rows * width)
    rc = getattr(_lib.lib, name)(P(xd), P(wd), P(yd), rows, width, int(centered), f32(1e-6), S())
    if rc != 0:
        raise tfx.TfxError(rc, tfx.last_error())
    return host(yd)


@pytest.mark.parametrize("rows,width", [(16384, 1024), (1000, 4096), (258, 1025),
                                        (65536, 1024)])
def test_noalloc_matches_allocating_entry_point_and_oracle_on_consecutive_calls(orc, rows,
                                                                                width):
    w = splitmix_normal(width, 0x7E4F0B01 + width, mean=1.0, std=0.1)
    for call, centered in enumerate((True, False)):
        x = splitmix_normal(rows * width, 0x7E4F0B00 + 7919 * call + rows)
        got = _run("tfx_rmsnorm_last_f32_noalloc", x, w, rows, width, centered)
        want = _run("tfx_rmsnorm_last_f32", x, w, rows, width, centered)
        assert_close(got, want, F32_RTOL, F32_ATOL_REL, f"noalloc call {call} {rows}x{width}")
        ref = orc.rms_norm_last_f32(x, rows, width, w, centered, 1e-6)
        assert_close(got, ref, F32_RTOL, F32_ATOL_REL,
                     f"noalloc vs oracle call {call} {rows}x{width}")
        del x, got, want, ref
        torch.cuda.empty_cache()


def test_noalloc_rejects_shapes_beyond_its_fixed_scratch():
    rows, width = 65537, 1024  # 16 chunks x 65537 rows > 2^20 partial sums
    xd, wd, yd = empty(rows * width), empty(width), empty(rows * width)
    rc = _lib.lib.tfx_rmsnorm_last_f32_noalloc(P(xd), P(wd), P(yd), rows, width, 1, f32(1e-6),
                                               S())
    assert rc == _lib.TFX_ERR_UNSUPPORTED
    assert "exceed the fixed scratch" in tfx.last_error()
    torch.cuda.synchronize()
