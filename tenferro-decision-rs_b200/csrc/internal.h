// internal.h -- entry points shared between libtfx's translation units (not
// part of the C ABI).
#pragma once

#include <cstdint>

#include "causal_tiles.cuh"
#include "common.cuh"

namespace tfx {

// softmax.cu: validation of a softmax call, and the launch over a row range.
int validate_softmax(const float* scores, const float* probs, const tfx_softmax_desc* d,
                     int64_t* rows_out);
int masked_softmax_rows(const float* scores, float* probs, const tfx_softmax_desc* d,
                        int64_t row_begin, int64_t row_count, cudaStream_t stream);

// rms_stream.cu: the TMA-pipelined feature-last RMSNorm; 1 when the shape or
// alignment is not covered (nothing launched), else a status.
int rms_stream(const char* op, const float* x, const float* w, float* y, uint32_t rows,
               uint32_t width, int centered, float eps, float inv_width, cudaStream_t stream);
// rms_stream.cu: the same op with a TMA box ring feeding registers (widths
// 513 .. 2048); 1 when not covered, else a status.
int rms_ring(const char* op, const float* x, const float* w, float* y, uint32_t rows,
             uint32_t width, int centered, float eps, float inv_width, cudaStream_t stream);

// rms_stream.cu: the same op on 32-token tiles shared by a CTA pair (widths
// 513 .. 1024); 1 when not covered, else a status.
int rms_pair(const char* op, const float* x, const float* w, float* y, uint32_t rows,
             uint32_t width, int centered, float eps, float inv_width, cudaStream_t stream);

// attention.cu: the tensor-core attention's count of bounded waits that gave
// up on the current device (cudaMemcpyFromSymbol; synchronous).
int attention_wait_timeouts(uint32_t* count);

// gemm_epilogue.cu: the same count for the tensor-core GEMM-epilogue kernel.
int gemm_wait_timeouts(uint32_t* count);
// Batched y (nout, length) = W_b^T x: token t uses the weight rows of batch
// t / batch_tokens (gemm_epilogue.cu). causal (t_b = t's index in its batch):
// 1 = only outputs o <= t_b are wanted (the others may be left unwritten),
// 2 = x[t][i] is 0 for i > t_b (needs in_dim == batch_tokens, nout <= 256:
// the contraction stops there, and its pieces go to output slots, y + p *
// length * nout, that the consumer adds in slot order); 0 = neither.
// planes (optional): {x hi, x lo, w hi, w lo} already split (tf32 hi, exact
// remainder lo), in_dim % 32 == 0, no non-finite value (x and w unused).
// out_t: y of batch b is (nout, batch_tokens), token-contiguous.
int gemm_batched_f32(const char* op, const float* x, const float* w, float* y, int64_t in_dim,
                     int64_t nout, int64_t length, int64_t batch_tokens, cudaStream_t stream,
                     uint32_t causal = 0, const float* const* planes = nullptr, int out_t = 0);
// The split causal 2 uses for these extents on the current device, for a call
// with pre-split operands (planes).
int gemm_causal_k_split(int64_t length, int64_t batch_tokens, CausalKSplit* split);

}  // namespace tfx
