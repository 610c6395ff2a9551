"""tfx -- host front end of libtfx, the B200 (sm_100a) non-GEMM extension ops
of tenferro-decision (LayerNorm, RMSNorm, erf-GELU / GeGLU, gated SiLU, bias
broadcast, masked softmax, RoPE).

`tfx._lib` declares the C ABI of include/tfx.h over ctypes; `tfx.ops` wraps it
for torch CUDA tensors. Importing raises if libtfx.so is not built.
"""

from ._lib import (LIB_PATH, TfxError, check, header_symbols, last_error, lib)  # noqa: F401

__version__ = "1.0.0"
