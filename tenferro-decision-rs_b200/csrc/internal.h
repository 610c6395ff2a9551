// internal.h -- entry points shared between libtfx's translation units (not
// part of the C ABI).
#pragma once

#include <cstdint>

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
// t / batch_tokens (gemm_epilogue.cu).
int gemm_batched_f32(const char* op, const float* x, const float* w, float* y, int64_t in_dim,
                     int64_t nout, int64_t length, int64_t batch_tokens, cudaStream_t stream);

}  // namespace tfx
