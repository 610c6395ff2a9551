"""GPU parity over the reference's shape regression list.

docs/agents/specs/docs/05_TESTING_BENCHMARKS.md section 4 of the reference lists
the lengths every kernel is checked at: L in {1, 63, 64, 65, 127, 128, 129, 255,
256, 257, 512}. Each op of the path runs at every L in the role its kernels
tile on (tokens / columns, sequence length, feature width) and is compared with
the oracle: bitwise where the op is bit-exact (GELU, GeGLU, bias, add, RoPE,
embedding), within the f32 bar elsewhere.
"""

import numpy as np
import pytest
import torch

from helpers import (assert_bitwise, assert_close, splitmix_normal, splitmix_uniform, F32_RTOL,
                     F32_ATOL_REL)
from tfx import ops

pytestmark = pytest.mark.gpu

LENGTHS = [1, 63, 64, 65, 127, 128, 129, 255, 256, 257, 512]


def cuda(a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


@pytest.mark.parametrize("L", LENGTHS)
def test_layernorm_tokens_and_width(orc, L):
    for d, cols in ((768, L), (L, 37)):
        x = splitmix_normal(d * cols, 0x7E4F0C00 + L + d)
        w = splitmix_uniform(d, 0x7E4F0C01 + d, 0.5, 1.5)
        b = splitmix_normal(d, 0x7E4F0C02 + d, std=0.1)
        y = ops.layer_norm_feature_first(cuda(x), cuda(w), cuda(b), 1e-5).cpu().numpy()
        assert_close(y, orc.layer_norm_feature_first_f32(x, d, cols, w, b, 1e-5), F32_RTOL,
                     F32_ATOL_REL, f"layernorm d={d} cols={cols}")


@pytest.mark.parametrize("L", LENGTHS)
def test_rmsnorm_tokens_and_width(orc, L):
    for rows, width in ((L, 1024), (L * 4, 1024), (100, L)):
        x = splitmix_normal(rows * width, 0x7E4F0C10 + L + width)
        w = splitmix_normal(width, 0x7E4F0C11 + width, mean=1.0, std=0.1)
        y = ops.rms_norm_last(cuda(x), cuda(w), True, float(np.float32(1e-6))).cpu().numpy()
        assert_close(y, orc.rms_norm_last_f32(x, rows, width, w, True, 1e-6), F32_RTOL,
                     F32_ATOL_REL, f"rmsnorm {rows}x{width}")


@pytest.mark.parametrize("L", LENGTHS)
def test_elementwise_bit_exact(orc, L):
    inter = 1152
    u = splitmix_normal(2 * inter * L, 0x7E4F0C20 + L, std=1.5)
    assert_bitwise(ops.geglu(cuda(u), inter).cpu().numpy().ravel(), orc.geglu_f32(u, inter, L),
                   f"geglu cols={L}")
    g = splitmix_normal(L * 97, 0x7E4F0C21 + L, std=1.5)
    assert_bitwise(ops.gelu_erf(cuda(g)).cpu().numpy(), orc.gelu_erf_f32(g), f"gelu n={g.size}")
    x = splitmix_normal(768 * L, 0x7E4F0C22 + L)
    bias = splitmix_normal(768, 0x7E4F0C23, std=0.02)
    assert_bitwise(ops.bias_act(cuda(x), cuda(bias)).cpu().numpy(),
                   orc.bias_add_f32(x, bias, 768, L), f"bias tokens={L}")
    b = splitmix_normal(L * 97, 0x7E4F0C24 + L)
    assert_bitwise(ops.add(cuda(g), cuda(b)).cpu().numpy(), orc.add_f32(g, b), "add")
    assert_close(ops.gated_silu(cuda(g), cuda(b)).cpu().numpy(), orc.gated_silu_f32(g, b),
                 F32_RTOL, F32_ATOL_REL, "silu")


@pytest.mark.parametrize("L", LENGTHS)
def test_softmax_sequence_length(orc, L):
    B, H = 2, 3
    s = splitmix_normal(B * H * L * L, 0x7E4F0C30 + L, std=2.0)
    for kw in (dict(), dict(window=16, valid_len=max(1, L - 5)), dict(causal=True)):
        want = orc.masked_softmax_f32(s, B, H, L, L, **kw)
        got = ops.masked_softmax(cuda(s), B, H, L, L, **kw).cpu().numpy()
        assert_close(got, want, F32_RTOL, F32_ATOL_REL, f"softmax L={L} {kw}")


@pytest.mark.parametrize("L", LENGTHS)
def test_rope_sequence_length(orc, L):
    hidden, hd, B = 256, 64, 2
    strides = (hd, 3 * hidden, 3 * hidden * L, 1)
    x = splitmix_normal(3 * hidden * L * B, 0x7E4F0C40 + L)
    c, s = orc.rope_tables_f32(160000.0, L, hd)
    y = ops.rope_pairhalf(cuda(x), cuda(c), cuda(s), 2 * hidden // hd, L, B, hd, hd, strides,
                          out=cuda(x)).cpu().numpy()
    assert_bitwise(y, orc.rope_pairhalf_f32(x, c, s, 2 * hidden // hd, L, B, hd, hd, strides),
                   f"rope L={L}")


@pytest.mark.parametrize("L", LENGTHS)
def test_laya_attention_sequence_length(orc, L):
    hd, heads, B = 64, 2, 2
    d = hd * heads
    qkv = splitmix_normal(3 * d * L * B, 0x7E4F0C50 + L)
    valid = np.array([L, max(1, L - 3)])
    q = np.arange(L)[None, None, :]
    k = np.arange(L)[None, :, None]
    keep = ((np.abs(q - k) <= 64) & (k < valid[:, None, None])).astype(np.uint8).ravel()
    c, s = orc.rope_tables_f32(10000.0, L, hd)
    got = ops.laya_attention_block(cuda(qkv), cuda(keep), d, heads, L, B, cuda(c),
                                   cuda(s)).cpu().numpy()
    want = orc.laya_attention_block_f32(qkv, keep, d, heads, L, B, c, s)
    assert_close(got, want, F32_RTOL, F32_ATOL_REL, f"laya attention L={L}")


@pytest.mark.parametrize("L", LENGTHS)
def test_embedding_sequence_length(orc, L):
    hidden, vocab = 768, 5000
    table = splitmix_normal(hidden * vocab, 0x7E4F0C60)
    ids = (np.arange(L, dtype=np.int64) * 7919) % vocab
    for layout in (0, 1):
        got = ops.embedding_gather(cuda(table), cuda(ids), hidden, vocab, L, layout)
        assert_bitwise(got.cpu().numpy(), orc.embedding_f32(table, ids, hidden, vocab, layout),
                       f"embedding L={L} layout={layout}")
