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

}  // namespace tfx
