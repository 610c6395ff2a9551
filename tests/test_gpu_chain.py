"""GPU parity of the configs[4] chain at its full size (batch 64 x seq 512).

The bench times `bench.Chain.step`: LayerNorm -> RoPE on q,k -> masked softmax
-> residual add fused into the second LayerNorm -> GeGLU over 32768 tokens
(hidden 768, 12 heads x 64, intermediate 1152). These tests run that same
method, for a sliding-window step (even: window 128, theta 10000) and a global
step (odd: theta 160000), and compare every stage's output with the oracle on
the same inputs (crates/cpu-kernels/src/lib.rs:397-443 LayerNorm, :516-538
GeGLU; crates/tenferro-infer/src/rope.rs:68-113, softmax.rs:26-34).

The chain is fed forward: the GEMMs between the stages are out of scope, so
fp32 torch matmuls with seeded weights stand in for them (test plumbing, not
what is checked): qkv = W_qkv h1, scores = (q k^T) / 4 per head from the
rotated q and k, attn = probs v, u = W_up h3. `Chain.step` is run once per
derived input, so in the last pass every stage consumes what the stage before
it produced, and every kernel output is checked: RoPE, the residual sum and
GeGLU bitwise; LayerNorm and softmax within the f32 bar.
"""

import numpy as np
import pytest
import torch

import bench
from helpers import F32_ATOL_REL, F32_RTOL, assert_bitwise, assert_close
from tfx import ops

pytestmark = pytest.mark.gpu


@pytest.fixture(autouse=True)
def _free_memory():
    yield
    torch.cuda.synchronize()
    torch.cuda.empty_cache()


def _fed_forward_chain(step):
    c = bench.CHAIN
    dev = torch.device("cuda", 0)
    chain = bench.Chain(torch, ops, dev, 0, c["batch"])
    B, L, h, H, hd, I = chain.B, chain.L, chain.h, chain.H, chain.hd, chain.I
    g = torch.Generator(device=dev)
    g.manual_seed(0x7E4F0C00 + step)
    w_qkv = torch.randn(h, 3 * h, generator=g, device=dev) / h ** 0.5
    w_up = torch.randn(h, 2 * I, generator=g, device=dev) / h ** 0.5
    hp = torch.backends.cuda.matmul.allow_tf32
    torch.backends.cuda.matmul.allow_tf32 = False
    try:
        chain.step(step)
        # qkv (3h, L, B) feature-first = torch (B*L, 3h)
        torch.matmul(chain.h1.view(B * L, h), w_qkv, out=chain.qkv.view(B * L, 3 * h))
        chain.step(step)
        qk = chain.qk.view(B, L, 3 * h)
        q = qk[..., :h].reshape(B, L, H, hd).transpose(1, 2)
        k = qk[..., h:2 * h].reshape(B, L, H, hd).transpose(1, 2)
        torch.matmul(q, k.transpose(-1, -2), out=chain.scores.view(B, H, L, L))
        chain.scores.mul_(0.25)
        chain.step(step)
        v = chain.qkv.view(B, L, 3 * h)[..., 2 * h:].reshape(B, L, H, hd).transpose(1, 2)
        o = torch.matmul(chain.probs.view(B, H, L, L), v)           # (B, H, L, hd)
        chain.attn.view(B, L, H, hd).copy_(o.transpose(1, 2))      # (h, L, B) feature-first
        chain.step(step)
        torch.matmul(chain.h3.view(B * L, h), w_up, out=chain.u.view(B * L, 2 * I))
        chain.step(step)
    finally:
        torch.backends.cuda.matmul.allow_tf32 = hp
    torch.cuda.synchronize()
    return chain


@pytest.mark.parametrize("step", [0, 1], ids=["window_theta10000", "global_theta160000"])
def test_chain_config4_batch64_every_stage_against_oracle(orc, step):
    c = bench.CHAIN
    chain = _fed_forward_chain(step)
    B, L, h, H, hd, I = chain.B, chain.L, chain.h, chain.H, chain.hd, chain.I
    T = B * L
    local = step % 2 == 0
    cpu = lambda t: t.detach().cpu().numpy().reshape(-1)  # noqa: E731
    x0, g1, g2 = cpu(chain.x0), cpu(chain.gamma1), cpu(chain.gamma2)

    # 1. LayerNorm (d=768, cols=32768)
    want = orc.layer_norm_feature_first_f32(x0, h, T, g1, None, 1e-5)
    assert_close(cpu(chain.h1), want, F32_RTOL, F32_ATOL_REL, "chain layernorm 1")

    # 2. RoPE on the q and k blocks of qkv (24 vectors of 64 per token)
    qkv = cpu(chain.qkv)
    cos_t, sin_t = orc.rope_tables_f32(c["theta_local" if local else "theta_global"], L, hd)
    want = orc.rope_pairhalf_f32(qkv, cos_t, sin_t, 2 * H, L, B, hd, hd,
                                 (hd, 3 * h, 3 * h * L, 1))
    got = cpu(chain.qk)
    assert_bitwise(got.reshape(T, 3 * h)[:, :2 * h], want.reshape(T, 3 * h)[:, :2 * h],
                   "chain rope q,k")
    del qkv, got, want

    # 3. masked softmax over [64, 12, 512, 512]
    scores = cpu(chain.scores)
    assert 1.0 < float(scores[: 1 << 22].std()) < 4.0  # the configs' N(0, 2) scale
    want = orc.masked_softmax_f32(scores, B, H, L, L, window=c["window"] if local else -1,
                                  valid_len=L - c["pad"])
    got = cpu(chain.probs)
    assert_close(got, want, F32_RTOL, F32_ATOL_REL, "chain masked softmax")
    rows = got.reshape(-1, L)
    assert np.all(rows[:, L - c["pad"]:] == 0.0)  # padded keys are exact zeros
    del scores, got, want, rows

    # 4. residual add (bitwise) fused into the second LayerNorm (f32 bar)
    attn = cpu(chain.attn)
    s_want = orc.add_f32(x0, attn)
    assert_bitwise(cpu(chain.h2), s_want, "chain residual sum")
    want = orc.layer_norm_feature_first_f32(s_want, h, T, g2, None, 1e-5)
    assert_close(cpu(chain.h3), want, F32_RTOL, F32_ATOL_REL, "chain layernorm 2")
    del attn, s_want, want

    # 5. GeGLU (2*1152, 32768) -> (1152, 32768), bitwise
    u = cpu(chain.u)
    assert_bitwise(cpu(chain.g), orc.geglu_f32(u, I, T), "chain geglu")


def test_chain_step_is_deterministic_across_calls():
    """Two calls of the timed step on the same inputs give identical outputs
    (the bench's repeated steps time the same work)."""
    chain = bench.Chain(torch, ops, torch.device("cuda", 0), 0, 8)
    chain.step(1)
    first = [t.clone() for t in (chain.h1, chain.probs, chain.h2, chain.h3, chain.g)]
    chain.step(1)
    for a, b in zip(first, (chain.h1, chain.probs, chain.h2, chain.h3, chain.g)):
        assert torch.equal(a, b)
