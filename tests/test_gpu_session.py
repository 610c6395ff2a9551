"""GPU parity of the host-buffer session (tfx_session_*): every op on host
arrays, split into many pipelined chunks (small chunk size), against the
oracle -- the ext-op executor form of the reference (CPU TensorRead in, owned
host tensor out)."""

import numpy as np
import pytest
import torch

from helpers import (assert_bitwise, assert_close, splitmix_normal, splitmix_uniform, F32_RTOL,
                     F32_ATOL_REL, F64_RTOL, F64_ATOL_REL)
from tfx.session import Session

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def sess():
    s = Session(0, chunk_bytes=1 << 20)  # 1 MiB chunks: dozens of chunks per call
    yield s
    s.close()


def test_session_layernorm(orc, sess):
    d, cols = 768, 3001
    x = splitmix_normal(d * cols, 0x7E4F0800)
    w = splitmix_uniform(d, 0x7E4F0801, 0.5, 1.5)
    b = splitmix_normal(d, 0x7E4F0802, std=0.1)
    y = sess.layer_norm_feature_first(x, w, b, 1e-5)
    assert_close(y, orc.layer_norm_feature_first_f32(x, d, cols, w, b, 1e-5), F32_RTOL,
                 F32_ATOL_REL, "session layernorm")
    x64, w64 = x.astype(np.float64), w.astype(np.float64)
    y64 = sess.layer_norm_feature_first(x64, w64, None, 1e-5)
    assert_close(y64, orc.layer_norm_feature_first_f64(x64, d, cols, w64, None, 1e-5), F64_RTOL,
                 F64_ATOL_REL, "session layernorm f64")


def test_session_rmsnorm_strided_row_chunks(orc, sess):
    rows, width = 5003, 1024
    x = splitmix_normal(rows * width, 0x7E4F0810)
    w = splitmix_normal(width, 0x7E4F0811, mean=1.0, std=0.1)
    y = sess.rms_norm_last(x, w, True, 1e-6)
    assert_close(y, orc.rms_norm_last_f32(x, rows, width, w, True, 1e-6), F32_RTOL, F32_ATOL_REL,
                 "session rmsnorm")


def test_session_elementwise_bitwise(orc, sess):
    n = 3_000_001
    x = splitmix_normal(n, 0x7E4F0820, std=1.5)
    assert_bitwise(sess.erf(x), orc.erf_f32(x), "session erf")
    assert_bitwise(sess.gelu_erf(x), orc.gelu_erf_f32(x), "session gelu")
    b = splitmix_normal(n, 0x7E4F0821)
    assert_bitwise(sess.add(x, b), orc.add_f32(x, b), "session add")
    assert_close(sess.gated_silu(x, b), orc.gated_silu_f32(x, b), F32_RTOL, F32_ATOL_REL,
                 "session silu")
    inter, cols = 1152, 777
    u = splitmix_normal(2 * inter * cols, 0x7E4F0822, std=1.5)
    assert_bitwise(sess.geglu(u, inter), orc.geglu_f32(u, inter, cols), "session geglu")
    F, T = 768, 2049
    xb = splitmix_normal(F * T, 0x7E4F0823)
    bias = splitmix_normal(F, 0x7E4F0824, std=0.02)
    assert_bitwise(sess.bias_act(xb, bias), orc.bias_add_f32(xb, bias, F, T), "session bias")
    assert_bitwise(sess.bias_act(xb, bias, act=1), orc.bias_act_f32(xb, bias, F, T, 1),
                   "session bias gelu")


def test_session_softmax_with_host_masks(orc, sess):
    B, H, L = 3, 4, 128
    s = splitmix_normal(B * H * L * L, 0x7E4F0830, std=2.0)
    vl = np.array([128, 90, 17], dtype=np.int32)
    kw = dict(window=16, valid_lens=vl, window_skips_invalid_query=True)
    assert_close(sess.masked_softmax(s, B, H, L, L, **kw),
                 orc.masked_softmax_f32(s, B, H, L, L, **kw), F32_RTOL, F32_ATOL_REL,
                 "session softmax")
    keep = (np.arange(L)[None, :] <= np.arange(L)[:, None]).astype(np.uint8).ravel()  # [q][k]
    kw = dict(keep=keep, keep_strides=(0, L, 1), semantics=1)
    assert_close(sess.masked_softmax(s, B, H, L, L, **kw),
                 orc.masked_softmax_f32(s, B, H, L, L, **kw), F32_RTOL, F32_ATOL_REL,
                 "session softmax keep")


def test_session_rope_chain_layout(orc, sess):
    hidden, hd, L, B = 768, 64, 512, 5
    x = splitmix_normal(3 * hidden * L * B, 0x7E4F0840)
    strides = (hd, 3 * hidden, 3 * hidden * L, 1)
    # elements past the last rotated vector of each item are not written: start from x
    y = sess.rope_pairhalf(x, 160000.0, 24, L, B, hd, hd, strides, out=x.copy())
    c, s = orc.rope_tables_f32(160000.0, L, hd)
    assert_bitwise(y, orc.rope_pairhalf_f32(x, c, s, 24, L, B, hd, hd, strides), "session rope")


def test_session_pinned_torch_tensors(orc, sess):
    n = 1 << 22
    x = torch.from_numpy(splitmix_normal(n, 0x7E4F0850, std=1.5)).pin_memory()
    y = torch.empty(n, dtype=torch.float32).pin_memory()
    sess.gelu_erf(x, out=y)
    assert_bitwise(y.numpy(), orc.gelu_erf_f32(x.numpy()), "session pinned gelu")


def _vector_mask(size, n_vec, L, B, hd, strides):
    sv, sp, sb, sf = strides
    idx = (np.arange(n_vec)[:, None, None, None] * sv + np.arange(L)[None, :, None, None] * sp +
           np.arange(B)[None, None, :, None] * sb + np.arange(hd)[None, None, None, :] * sf)
    mask = np.zeros(size, dtype=bool)
    mask[idx.ravel()] = True
    return mask


def test_session_rope_rows_copy_only_the_vectors(orc, sess):
    # q and k of a feature-first qkv (3h, L, B): only their rows cross PCIe;
    # v is not part of the call and y's v block keeps what it held.
    hidden, hd, L, B = 768, 64, 512, 3
    x = splitmix_normal(3 * hidden * L * B, 0x7E4F0860)
    strides = (hd, 3 * hidden, 3 * hidden * L, 1)
    y0 = np.full_like(x, 7.0)
    y = sess.rope_pairhalf(x, 10000.0, 24, L, B, hd, hd, strides, out=y0.copy())
    c, s = orc.rope_tables_f32(10000.0, L, hd)
    want = orc.rope_pairhalf_f32(x, c, s, 24, L, B, hd, hd, strides)
    m = _vector_mask(x.size, 24, L, B, hd, strides)
    assert_bitwise(y[m], want[m], "session rope vectors")
    assert np.all(y[~m] == 7.0), "session rope wrote outside the vectors"


def test_session_rope_padded_batch_items_take_the_extent_copy(orc, sess):
    # batch items padded apart (stride_batch != seq * stride_pos): whole extents
    hidden, hd, L, B, pad = 256, 32, 100, 4, 96
    strides = (hd, 3 * hidden, 3 * hidden * L + pad, 1)
    x = splitmix_normal(strides[2] * B, 0x7E4F0861)
    y = sess.rope_pairhalf(x, 160000.0, 16, L, B, hd, hd, strides, out=x.copy())
    c, s = orc.rope_tables_f32(160000.0, L, hd)
    assert_bitwise(y, orc.rope_pairhalf_f32(x, c, s, 16, L, B, hd, hd, strides),
                   "session rope padded items")


@pytest.mark.parametrize("cols", [1, 5, 63, 64, 65, 200, 1000])
def test_session_chunk_plan_covers_every_column(orc, cols):
    # 16 KiB chunks of 768-float columns: 2 units per chunk at most, so the
    # ramped plan runs through its small-call and tail branches.
    d = 768
    x = splitmix_normal(d * cols, 0x7E4F0870 + cols)
    w = splitmix_uniform(d, 0x7E4F0871, 0.5, 1.5)
    with Session(0, chunk_bytes=16 * 1024 * 4) as s:
        y = s.layer_norm_feature_first(x, w, None, 1e-5)
        g = s.gelu_erf(x)
    assert_close(y, orc.layer_norm_feature_first_f32(x, d, cols, w, None, 1e-5), F32_RTOL,
                 F32_ATOL_REL, f"chunked layernorm {cols}")
    assert_bitwise(g, orc.gelu_erf_f32(x), f"chunked gelu {cols}")


def test_session_add_layernorm_matches_the_two_ops(orc, sess):
    d, cols = 768, 2999
    a = splitmix_normal(d * cols, 0x7E4F0880)
    b = splitmix_normal(d * cols, 0x7E4F0881)
    w = splitmix_uniform(d, 0x7E4F0882, 0.5, 1.5)
    s_want = orc.add_f32(a, b)
    y_want = sess.layer_norm_feature_first(s_want, w, None, 1e-5)
    s_got, y_got = sess.add_layer_norm_feature_first(a, b, w, None, 1e-5,
                                                     sum_out=np.empty_like(a))
    assert_bitwise(s_got, s_want, "session add+ln sum")
    assert_bitwise(y_got, y_want, "session add+ln y")
    _, y_only = sess.add_layer_norm_feature_first(a, b, w, None, 1e-5)
    assert_bitwise(y_only, y_want, "session add+ln without sum")


def test_session_gemm_geglu_and_bias_act_chunked(orc, sess):
    """The fused GEMM epilogues on host buffers: 1 MiB chunks cut the 3000
    tokens into whole 128-token tiles, so the result is bitwise the device
    call's (each token depends on its own column of x only) and within the f32
    bar of the oracle's projection + epilogue."""
    from tfx import ops
    in_dim, inter, length = 768, 1152, 3000
    x = splitmix_normal(in_dim * length, 0x7E4F0860)
    w = splitmix_normal(in_dim * 2 * inter, 0x7E4F0861, std=in_dim ** -0.5)
    b = splitmix_normal(2 * inter, 0x7E4F0862, std=0.02)
    y = sess.gemm_geglu(x, w, b, inter)
    dev = ops.gemm_geglu(torch.from_numpy(x).cuda(), torch.from_numpy(w).cuda(),
                         torch.from_numpy(b).cuda(), inter).cpu().numpy().reshape(-1)
    assert_bitwise(y, dev, "session gemm_geglu vs device call")
    assert_close(y, orc.gemm_geglu_f32(x, w, b, in_dim, inter, length), F32_RTOL, F32_ATOL_REL,
                 "session gemm_geglu")
    out_dim = 300
    w2 = splitmix_normal(in_dim * out_dim, 0x7E4F0863, std=in_dim ** -0.5)
    y2 = sess.gemm_bias_act(x, w2, None, out_dim, act=2)
    assert_close(y2, orc.gemm_bias_act_f32(x, w2, None, in_dim, out_dim, length, 2), F32_RTOL,
                 F32_ATOL_REL, "session gemm_bias_act relu")
