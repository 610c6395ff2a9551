"""GPU parity of every feature-last RMSNorm kernel variant. The variant is
picked once per process (TFX_RMS_KERNEL), so each runs in a fresh interpreter
that compares a few shapes against the oracle and prints one verdict line."""

import os
import subprocess
import sys

import pytest

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))

SCRIPT = r"""
import sys
sys.path.insert(0, {root!r}); sys.path.insert(0, {pkg!r}); sys.path.insert(0, {tests!r})
import numpy as np, torch
from oracle import oracle as orc
from tfx import ops
from helpers import assert_close, splitmix_normal, F32_RTOL, F32_ATOL_REL
for rows, width in [(16384, 1024), (4096, 2048), (258, 1025), (63, 31), (1000, 4096), (7, 9),
                   (1000, 1000), (20000, 64), (1004, 1500), (20, 600), (16388, 768)]:
    x = splitmix_normal(rows * width, 0x7E4F0900 + rows)
    w = splitmix_normal(width, 0x7E4F0901 + width, mean=1.0, std=0.1)
    for centered in (True, False):
        y = ops.rms_norm_last(torch.from_numpy(x).cuda(), torch.from_numpy(w).cuda(), centered,
                              1e-6).cpu().numpy()
        assert_close(y, orc.rms_norm_last_f32(x, rows, width, w, centered, 1e-6), F32_RTOL,
                     F32_ATOL_REL, f"rms {{rows}}x{{width}}")
print("variant ok")
"""


@pytest.mark.parametrize("variant", ["cluster", "cluster16", "tile", "split", "stream", "ring",
                                     "pair"])
def test_rms_variant(variant):
    code = SCRIPT.format(root=ROOT, pkg=os.path.join(ROOT, "tenferro-decision-rs_b200"),
                         tests=os.path.join(ROOT, "tests"))
    env = dict(os.environ, TFX_RMS_KERNEL=variant)
    res = subprocess.run([sys.executable, "-c", code], env=env, capture_output=True, text=True,
                         timeout=600)
    assert res.returncode == 0 and "variant ok" in res.stdout, res.stdout + res.stderr


LN_SCRIPT = r"""
import sys
sys.path.insert(0, {root!r}); sys.path.insert(0, {pkg!r}); sys.path.insert(0, {tests!r})
import numpy as np, torch
from oracle import oracle as orc
from tfx import ops
from helpers import assert_close, splitmix_normal, splitmix_uniform, F32_RTOL, F32_ATOL_REL
for d, cols in [(768, 8192), (1024, 100), (512, 33), (4, 9), (132, 17)]:
    x = splitmix_normal(d * cols, 0x7E4F0A00 + d)
    w = splitmix_uniform(d, 0x7E4F0A01 + d, 0.5, 1.5)
    for b in (None, splitmix_normal(d, 0x7E4F0A02 + d, std=0.1)):
        y = ops.layer_norm_feature_first(torch.from_numpy(x).cuda(), torch.from_numpy(w).cuda(),
                                         None if b is None else torch.from_numpy(b).cuda(),
                                         1e-5).cpu().numpy()
        assert_close(y, orc.layer_norm_feature_first_f32(x, d, cols, w, b, 1e-5), F32_RTOL,
                     F32_ATOL_REL, f"ln {{d}}x{{cols}}")
print("variant ok")
"""


@pytest.mark.parametrize("variant", ["regs", "smem", "ring"])
def test_layernorm_variant(variant):
    code = LN_SCRIPT.format(root=ROOT, pkg=os.path.join(ROOT, "tenferro-decision-rs_b200"),
                            tests=os.path.join(ROOT, "tests"))
    env = dict(os.environ, TFX_LN_KERNEL=variant)
    res = subprocess.run([sys.executable, "-c", code], env=env, capture_output=True, text=True,
                         timeout=600)
    assert res.returncode == 0 and "variant ok" in res.stdout, res.stdout + res.stderr


DIGEST_SCRIPT = r"""
import sys, hashlib
sys.path.insert(0, {root!r}); sys.path.insert(0, {pkg!r}); sys.path.insert(0, {tests!r})
import torch
from tfx import ops
from helpers import splitmix_normal, splitmix_uniform
h = hashlib.sha256()
for d, cols in [(768, 8192), (768, 32768), (1024, 2500), (64, 7), (516, 4737)]:
    x = torch.from_numpy(splitmix_normal(d * cols, 0x7E4F0A10 + d)).cuda()
    w = torch.from_numpy(splitmix_uniform(d, 0x7E4F0A11 + d, 0.5, 1.5)).cuda()
    b = torch.from_numpy(splitmix_normal(d, 0x7E4F0A12 + d, std=0.1)).cuda()
    for bias in (None, b):
        h.update(ops.layer_norm_feature_first(x, w, bias, 1e-5).cpu().numpy().tobytes())
    ops.layer_norm_feature_first(x, w, b, 1e-5, out=x)  # in place
    h.update(x.cpu().numpy().tobytes())
print("digest", h.hexdigest())
"""


def test_layernorm_ring_gives_the_one_wave_kernels_bits():
    """The persistent ring kernel (default) and the one-wave shared-memory
    kernel use the same lane mapping and roundings: identical outputs,
    in place included, with several columns per warp (32768 columns)."""
    code = DIGEST_SCRIPT.format(root=ROOT, pkg=os.path.join(ROOT, "tenferro-decision-rs_b200"),
                                tests=os.path.join(ROOT, "tests"))
    digests = []
    for variant in ("ring", "smem"):
        env = dict(os.environ, TFX_LN_KERNEL=variant)
        res = subprocess.run([sys.executable, "-c", code], env=env, capture_output=True,
                             text=True, timeout=600)
        assert res.returncode == 0, res.stdout + res.stderr
        digests.append([ln for ln in res.stdout.splitlines() if ln.startswith("digest")][-1])
    assert digests[0] == digests[1]


def test_attention_f32_variant():
    """The attention tests again with every head on the f32-pipe kernel
    (TFX_ATTN_KERNEL is read once per process)."""
    env = dict(os.environ, TFX_ATTN_KERNEL="f32")
    res = subprocess.run([sys.executable, "-m", "pytest", "-q", "-x", "-m", "gpu", "-p",
                          "no:cacheprovider", os.path.join(ROOT, "tests", "test_gpu_attention.py")],
                         env=env, capture_output=True, text=True, timeout=900, cwd=ROOT)
    assert res.returncode == 0, res.stdout[-3000:] + res.stderr[-3000:]


def test_gemm_one_cta_variant():
    """The GEMM-epilogue and Jeff attention tests again on the one-CTA
    tensor-core GEMM (TFX_GEMM_PAIR=0; by default calls whose batches are whole
    256-token rows run on CTA pairs)."""
    env = dict(os.environ, TFX_GEMM_PAIR="0")
    res = subprocess.run([sys.executable, "-m", "pytest", "-q", "-x", "-m", "gpu", "-p",
                          "no:cacheprovider", "-k", "gemm or jeff",
                          os.path.join(ROOT, "tests", "test_gpu_gemm_epilogue.py"),
                          os.path.join(ROOT, "tests", "test_gpu_attention.py")],
                         env=env, capture_output=True, text=True, timeout=900, cwd=ROOT)
    assert res.returncode == 0, res.stdout[-3000:] + res.stderr[-3000:]
