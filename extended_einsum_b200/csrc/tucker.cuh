// Log-space Tucker layer 'bfi,bfj,foij->bfo'.
#pragma once

#include "xe_common.cuh"

static xe_status xe_tucker_impl(const float* l, const float* r, const float* w, float* y, int64_t batch,
                                int64_t folds, int64_t i_dim, int64_t j_dim, int64_t o_dim, int32_t shift_mode,
                                cudaStream_t stream);
