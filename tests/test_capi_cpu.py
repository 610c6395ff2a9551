"""CPU checks of the C ABI: the library loads, exports every symbol the header
declares, validates arguments before any CUDA call, and its host helpers agree
with the oracle. No kernel is launched here."""

import ctypes
import os
import subprocess

import numpy as np
import pytest

import tfx
from tfx import _lib
from helpers import assert_bitwise

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def test_library_exports_every_header_symbol():
    names = _lib.header_symbols()
    assert len(names) >= 19
    for name in names:
        assert hasattr(_lib.lib, name), name
        assert name in _lib.SIGNATURES, f"{name} has no ctypes signature"
    out = subprocess.run(["nm", "-D", "--defined-only", _lib.LIB_PATH], capture_output=True,
                         text=True, check=True).stdout
    exported = {line.split()[-1] for line in out.splitlines() if " T " in line}
    assert set(names) <= exported
    # Everything else stays hidden (-fvisibility=hidden).
    assert not [s for s in exported if s.startswith("tfx_") and s not in names]


def test_version():
    assert _lib.lib.tfx_version() == 10000


@pytest.mark.parametrize("call,expect", [
    (lambda L: L.tfx_layernorm_ff_f32(None, None, None, None, 8, 2, ctypes.c_float(1e-5), None),
     "tenferro-ext::layernorm_ff: x: null pointer"),
    (lambda L: L.tfx_layernorm_ff_f32(None, None, None, None, -1, 2, ctypes.c_float(1e-5), None),
     "tenferro-ext::layernorm_ff: shape: extents must be non-negative"),
    (lambda L: L.tfx_rmsnorm_last_f32(None, None, None, 4, 4, 1, ctypes.c_float(1e-6), None),
     "tenferro-ext::rms_norm_last: x: null pointer"),
    (lambda L: L.tfx_geglu_ff_f32(None, None, 3, 2, None), "tenferro-ext::geglu: u: null pointer"),
    (lambda L: L.tfx_gated_silu_f32(None, None, None, -5, None),
     "tenferro-ext::gated_silu: n: must be non-negative"),
    (lambda L: L.tfx_bias_act_ff_f32(None, None, None, 4, 4, 7, None),
     "tenferro-ext::gemm_bias: act: unknown activation 7"),
    (lambda L: L.tfx_masked_softmax_f32(None, None, None, None),
     "tenferro-infer::masked_softmax: desc: null pointer"),
])
def test_argument_errors_without_gpu(call, expect):
    rc = call(_lib.lib)
    assert rc == _lib.TFX_ERR_INVALID_ARGUMENT
    assert tfx.last_error() == expect


def test_empty_tensors_are_noops_without_gpu():
    L = _lib.lib
    assert L.tfx_layernorm_ff_f32(None, None, None, None, 0, 5, ctypes.c_float(1e-5), None) == 0
    assert L.tfx_rmsnorm_last_f32(None, None, None, 0, 5, 1, ctypes.c_float(1e-6), None) == 0
    assert L.tfx_erf_f32(None, None, 0, None) == 0
    assert L.tfx_geglu_ff_f32(None, None, 0, 5, None) == 0
    d = _lib.SoftmaxDesc()
    L.tfx_softmax_desc_init(ctypes.byref(d), 0, 4, 8, 8)
    assert L.tfx_masked_softmax_f32(None, None, ctypes.byref(d), None) == 0
    assert tfx.last_error() == ""


def test_softmax_desc_defaults():
    d = _lib.SoftmaxDesc()
    _lib.lib.tfx_softmax_desc_init(ctypes.byref(d), 2, 3, 4, 5)
    assert (d.batch, d.heads, d.q_len, d.k_len) == (2, 3, 4, 5)
    assert d.scale == 1.0 and d.window == -1 and d.valid_len == -1
    assert d.semantics == _lib.TFX_SOFTMAX_EXCLUDE and not d.keep and not d.add_mask


@pytest.mark.parametrize("base,seq,rot", [(160000.0, 512, 64), (10000.0, 512, 64),
                                          (10000.0, 33, 6)])
def test_rope_tables_match_oracle(orc, base, seq, rot):
    half = rot // 2
    c = np.empty(seq * half, np.float32)
    s = np.empty(seq * half, np.float32)
    assert _lib.lib.tfx_rope_tables_f32(ctypes.c_double(base), seq, rot,
                                        c.ctypes.data_as(ctypes.c_void_p),
                                        s.ctypes.data_as(ctypes.c_void_p)) == 0
    oc, os_ = orc.rope_tables_f32(base, seq, rot)
    assert_bitwise(c, oc, "cos")
    assert_bitwise(s, os_, "sin")


def test_rope_tables_reject_odd_width():
    assert _lib.lib.tfx_rope_tables_f32(ctypes.c_double(1e4), 4, 3, None, None) == -1
    assert "positive even number" in tfx.last_error()


def test_product_erf_matches_oracle_over_bit_patterns(tmp_path):
    """The product's branch-free erf / GELU (tfx_math.h, host-compiled) equal the
    oracle's literal restatement bit for bit. Every 31st f32 bit pattern by
    default; TFX_EXHAUSTIVE=1 checks all 2^32."""
    exe = tmp_path / "erf_exhaustive"
    subprocess.run(["g++", "-O2", "-std=c++17", "-ffp-contract=off", "-fno-fast-math",
                    "-I", os.path.join(ROOT, "oracle"),
                    "-I", os.path.join(ROOT, "tenferro-decision-rs_b200", "csrc"),
                    os.path.join(ROOT, "tests", "native", "erf_exhaustive.cpp"),
                    os.path.join(ROOT, "oracle", "oracle.cpp"), "-o", str(exe), "-lpthread"],
                   check=True)
    stride = "1" if os.environ.get("TFX_EXHAUSTIVE") == "1" else "31"
    res = subprocess.run([str(exe), stride], capture_output=True, text=True, timeout=1800)
    assert res.returncode == 0, res.stdout + res.stderr
    assert "erf_mismatch=0 gelu_mismatch=0" in res.stdout


def test_session_create_without_gpu_fails_loudly():
    import torch
    if torch.cuda.is_available():
        pytest.skip("a GPU is present; covered by the GPU session tests")
    h = ctypes.c_void_p()
    rc = _lib.lib.tfx_session_create(0, ctypes.byref(h))
    assert rc == _lib.TFX_ERR_CUDA and not h.value
    assert tfx.last_error().startswith("tfx_session: device:")
    assert _lib.lib.tfx_session_destroy(None) == 0
    assert _lib.lib.tfx_session_gelu_erf_f32(None, None, None, 4) == _lib.TFX_ERR_INVALID_ARGUMENT
    assert tfx.last_error() == "tenferro-ext::gelu_erf: session: null session"
    rc = _lib.lib.tfx_session_add_layernorm_ff_f32(None, None, None, None, None, None, None, 8, 2,
                                                   ctypes.c_float(1e-5))
    assert rc == _lib.TFX_ERR_INVALID_ARGUMENT
    assert tfx.last_error() == "tenferro-ext::add_layernorm_ff: session: null session"


def test_header_is_plain_c_and_links(tmp_path):
    """A C99 translation unit (what a cgo / bindgen / N-API binding compiles)
    includes tfx.h, takes the address of every function and links against
    libtfx.so; the program then calls the host-only entry points."""
    names = _lib.header_symbols()
    src = tmp_path / "use_tfx.c"
    src.write_text(
        "#include <stdio.h>\n#include \"tfx.h\"\n"
        "typedef void (*fn_t)(void);\nstatic fn_t const table[] = {\n" +
        "".join(f"  (fn_t)&{n},\n" for n in names) +
        "};\nint main(void) {\n"
        "  printf(\"%d %d\\n\", tfx_version(), (int)(sizeof(table) / sizeof(table[0])));\n"
        "  return tfx_layernorm_ff_f32(0, 0, 0, 0, 8, 2, 1e-5f, 0) == TFX_ERR_INVALID_ARGUMENT ? 0 : 1;\n"
        "}\n")
    exe = tmp_path / "use_tfx"
    libdir = os.path.dirname(_lib.LIB_PATH)
    subprocess.run(["gcc", "-std=c99", "-Wall", "-Werror", "-pedantic", "-I",
                    os.path.join(ROOT, "include"), str(src), "-o", str(exe), "-L", libdir,
                    "-ltfx", f"-Wl,-rpath,{libdir}"], check=True, capture_output=True)
    out = subprocess.run([str(exe)], capture_output=True, text=True, check=True).stdout.split()
    assert out == ["10000", str(len(names))]


def test_session_chunk_plan_invariants(tmp_path):
    """The host-buffer session's chunk plan (csrc/chunk_plan.h) covers every
    unit once, never exceeds the staging slot, keeps every chunk but the last
    aligned, and starts and ends large calls with short chunks."""
    exe = tmp_path / "chunk_plan_test"
    subprocess.run(["g++", "-O2", "-std=c++17", "-Wall", "-Werror", "-I",
                    os.path.join(ROOT, "tenferro-decision-rs_b200", "csrc"),
                    os.path.join(ROOT, "tests", "native", "chunk_plan_test.cpp"), "-o", str(exe)],
                   check=True)
    res = subprocess.run([str(exe)], capture_output=True, text=True, timeout=120)
    assert res.returncode == 0 and "bad=0" in res.stdout, res.stdout


def test_causal_tile_enumeration(tmp_path):
    """The batched GEMM's causal schedules (causal_tiles.cuh, host-compiled):
    live score tiles and the even split-K of the probability-times-value
    contraction cover every unit once, with pieces and slots in order."""
    exe = tmp_path / "causal_tiles_test"
    subprocess.run(["g++", "-O2", "-std=c++17", "-Wall", "-Werror", "-I",
                    os.path.join(ROOT, "tenferro-decision-rs_b200", "csrc"),
                    os.path.join(ROOT, "tests", "native", "causal_tiles_test.cpp"), "-o", str(exe)],
                   check=True)
    res = subprocess.run([str(exe)], capture_output=True, text=True, timeout=300)
    assert res.returncode == 0 and "bad=0" in res.stdout, res.stdout


# Entry points whose arguments are all checked before any CUDA call: with every
# pointer NULL (the required data pointers among them) and every extent 8 the
# call must fail as invalid argument (a null pointer, or a shape the op cannot
# take), naming "op: field: message".
_NO_CUDA_BEFORE_VALIDATION = [
    "tfx_erf_f32", "tfx_gelu_erf_f32", "tfx_erf_f64", "tfx_gelu_erf_f64", "tfx_geglu_ff_f32",
    "tfx_gated_silu_f32", "tfx_gated_silu_stacked_f32", "tfx_bias_act_ff_f32", "tfx_add_f32",
    "tfx_layernorm_ff_f32", "tfx_layernorm_ff_f64", "tfx_rmsnorm_last_f32",
    "tfx_rmsnorm_last_f64", "tfx_rmsnorm_last_f32_noalloc", "tfx_masked_softmax_f32",
    "tfx_rope_pairhalf_f32", "tfx_add_layernorm_ff_f32", "tfx_embedding_f32",
    "tfx_embedding_gather_f32", "tfx_laya_qkv_prep_f32", "tfx_jeff_qkv_prep_f32",
    "tfx_attention_f32", "tfx_laya_attention_block_f32", "tfx_jeff_attention_f32",
    "tfx_gemm_geglu_ff_f32", "tfx_gemm_bias_act_ff_f32", "tfx_wait_timeouts", "tfx_session_set_chunk_bytes", "tfx_session_layernorm_ff_f32",
    "tfx_session_layernorm_ff_f64", "tfx_session_rmsnorm_last_f32", "tfx_session_erf_f32",
    "tfx_session_gelu_erf_f32", "tfx_session_geglu_ff_f32", "tfx_session_gated_silu_f32",
    "tfx_session_bias_act_ff_f32", "tfx_session_add_f32", "tfx_session_gemm_geglu_ff_f32",
    "tfx_session_gemm_bias_act_ff_f32", "tfx_session_add_layernorm_ff_f32",
    "tfx_session_masked_softmax_f32", "tfx_session_rope_pairhalf_f32",
]


def _args(name, extent):
    out = []
    for t in _lib.SIGNATURES[name][1]:
        if t is _lib._i64:
            out.append(extent)
        elif t is ctypes.c_float or t is ctypes.c_double:
            out.append(t(1e-5))
        elif t is _lib._int or t is ctypes.c_int32:
            out.append(0)
        else:
            out.append(None)  # every pointer, descriptor and stream
    return out


@pytest.mark.parametrize("name", _NO_CUDA_BEFORE_VALIDATION)
def test_null_pointers_are_invalid_arguments(name):
    rc = getattr(_lib.lib, name)(*_args(name, 8))
    msg = tfx.last_error()
    assert rc == _lib.TFX_ERR_INVALID_ARGUMENT, (rc, msg)
    assert msg.count(": ") >= 2 and msg.split(": ")[0].startswith(("tenferro-", "tfx")), msg


def test_every_validated_entry_point_is_listed():
    exempt = {"tfx_last_error_string", "tfx_version", "tfx_softmax_desc_init",
              "tfx_attention_desc_init", "tfx_rope_tables_f32", "tfx_rope_tables_powf_f32",
              "tfx_session_create", "tfx_session_destroy"}
    assert set(_lib.header_symbols()) - exempt == set(_NO_CUDA_BEFORE_VALIDATION)


@pytest.mark.parametrize("name", [n for n in _NO_CUDA_BEFORE_VALIDATION
                                  if _lib._i64 in _lib.SIGNATURES[n][1]
                                  and not n.startswith("tfx_session_")])
def test_negative_extents_are_invalid_arguments(name):
    rc = getattr(_lib.lib, name)(*_args(name, -1))
    assert rc == _lib.TFX_ERR_INVALID_ARGUMENT, (rc, tfx.last_error())
