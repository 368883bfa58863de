// Tensor-core (tcgen05) paged prefill: shape support test and launcher.
#pragma once
#include "common.cuh"

namespace bl {

bool prefill_tc_supported(int32_t dtype, int64_t head_dim, int64_t block_size, int64_t hq, int64_t hkv);
int prefill_tc_launch(const bl_prefill_args& a, cudaStream_t s);

}  // namespace bl
