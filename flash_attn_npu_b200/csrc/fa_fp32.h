// Parameters of the fp32 CUDA-core attention kernel (fa_fwd_fp32.cu).
#pragma once

#include <cuda_runtime.h>

#include <cstdint>

namespace fa {

struct Fp32Params {
  int64_t batch, heads;
  int seqlen, head_dim;
  int64_t q_stride[3], k_stride[3], v_stride[3], o_stride[3];  // elements: batch, head, seq
  int causal;
  float scale_log2;
};

int launch_fp32_simt(const float* q, const float* k, const float* v, float* o, float* lse,
                     const Fp32Params& p, cudaStream_t stream);

}  // namespace fa
