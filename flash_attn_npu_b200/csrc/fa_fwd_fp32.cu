// fp32 attention forward on the CUDA cores (fp32 FMA), for float32 inputs.
//
// The tensor-core path for fp32 inputs runs the MMAs in TF32 (10-bit mantissa), which keeps the
// output within the parity tolerance but moves the logsumexp by ~1e-3 -- outside the 1e-4 bar.
// This kernel keeps every product and sum in fp32, so fp32 inputs get fp32 results; the TF32
// tensor-core kernel stays available behind FA_FLAG_FP32_TF32.
//
// Same math as the tensor-core kernel (and the reference's `_attn_fwd_inner_loop` online
// softmax, flash_attention_forward.py:698-724): per 64-key tile, scores in base-2 units, tile
// max, rescale of l and the accumulator, then p = 2^(s - m) accumulated into l and O.
//
// CTA: 64 query rows x 4 threads per row (each thread owns a quarter of the head dimension);
// K and V tiles of 64 keys are staged in shared memory.
#include <cuda_runtime.h>

#include <cstdint>

#include "../../include/fa_fwd_sm100.h"
#include "fa_fp32.h"

namespace fa {
namespace {

constexpr int kRows = 64;
constexpr int kTpr = 4;  // threads per query row
constexpr int kKeys = 64;
constexpr int kThreads = kRows * kTpr;

template <int D>
__global__ void __launch_bounds__(kThreads) fa_fwd_fp32_kernel(const float* __restrict__ q,
                                                               const float* __restrict__ k,
                                                               const float* __restrict__ v,
                                                               float* __restrict__ o,
                                                               float* __restrict__ lse,
                                                               const Fp32Params p) {
  constexpr int DS = D / kTpr;  // head-dim slice per thread
  extern __shared__ float smem[];
  float* ks = smem;              // [kKeys][D]
  float* vs = smem + kKeys * D;  // [kKeys][D]

  const int tid = threadIdx.x;
  const int r = tid / kTpr;
  const int part = tid % kTpr;
  const int bh = blockIdx.y;
  const int64_t b = bh / p.heads, h = bh % p.heads;
  const int q0 = blockIdx.x * kRows;
  const int row = q0 + r;
  const bool row_ok = row < p.seqlen;

  float qr[DS];
  const float* qrow = q + b * p.q_stride[0] + h * p.q_stride[1] +
                      static_cast<int64_t>(row_ok ? row : 0) * p.q_stride[2] + part * DS;
#pragma unroll
  for (int d = 0; d < DS; ++d) qr[d] = row_ok ? qrow[d] : 0.f;

  float acc[DS];
#pragma unroll
  for (int d = 0; d < DS; ++d) acc[d] = 0.f;
  float m = -INFINITY;  // running max, base-2 units (scale applied)
  float l = 0.f;

  const int kv_end = p.causal ? min(p.seqlen, q0 + kRows) : p.seqlen;
  const float* kb = k + b * p.k_stride[0] + h * p.k_stride[1];
  const float* vb = v + b * p.v_stride[0] + h * p.v_stride[1];
  for (int kt = 0; kt < kv_end; kt += kKeys) {
    __syncthreads();
    for (int idx = tid; idx < kKeys * D; idx += kThreads) {
      const int kk = idx / D, d = idx % D;
      const bool in = kt + kk < p.seqlen;
      ks[idx] = in ? kb[static_cast<int64_t>(kt + kk) * p.k_stride[2] + d] : 0.f;
      vs[idx] = in ? vb[static_cast<int64_t>(kt + kk) * p.v_stride[2] + d] : 0.f;
    }
    __syncthreads();

    float sc[kKeys];
    float tmax = -INFINITY;
#pragma unroll
    for (int kk = 0; kk < kKeys; ++kk) {
      const float* kr = ks + kk * D + part * DS;
      float dot = 0.f;
#pragma unroll
      for (int d = 0; d < DS; ++d) dot = fmaf(qr[d], kr[d], dot);
      dot += __shfl_xor_sync(0xffffffffu, dot, 1);
      dot += __shfl_xor_sync(0xffffffffu, dot, 2);
      const int key = kt + kk;
      const bool masked = key >= p.seqlen || (p.causal && key > row);
      sc[kk] = masked ? -INFINITY : dot * p.scale_log2;
      tmax = fmaxf(tmax, sc[kk]);
    }
    const float m_new = fmaxf(m, tmax);
    const float base = (m_new == -INFINITY) ? 0.f : m_new;
    const float alpha = exp2f(m - base);  // m = -inf gives 0
    l *= alpha;
#pragma unroll
    for (int d = 0; d < DS; ++d) acc[d] *= alpha;
#pragma unroll
    for (int kk = 0; kk < kKeys; ++kk) {
      const float pk = exp2f(sc[kk] - base);
      l += pk;
      const float* vr = vs + kk * D + part * DS;
#pragma unroll
      for (int d = 0; d < DS; ++d) acc[d] = fmaf(pk, vr[d], acc[d]);
    }
    m = m_new;
  }

  if (row_ok) {
    const float inv_l = 1.f / l;
    float* orow = o + b * p.o_stride[0] + h * p.o_stride[1] +
                  static_cast<int64_t>(row) * p.o_stride[2] + part * DS;
#pragma unroll
    for (int d = 0; d < DS; ++d) orow[d] = acc[d] * inv_l;
    if (part == 0) lse[static_cast<int64_t>(bh) * p.seqlen + row] = (m + log2f(l)) * 0.6931471805599453f;
  }
}

template <int D>
int launch(const float* q, const float* k, const float* v, float* o, float* lse,
           const Fp32Params& p, cudaStream_t stream) {
  const int smem = 2 * kKeys * D * static_cast<int>(sizeof(float));
  auto kern = fa_fwd_fp32_kernel<D>;
  if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem) != cudaSuccess) {
    (void)cudaGetLastError();
    return FA_ERR_LAUNCH;
  }
  const dim3 grid(static_cast<unsigned>((p.seqlen + kRows - 1) / kRows),
                  static_cast<unsigned>(p.batch * p.heads));
  kern<<<grid, kThreads, smem, stream>>>(q, k, v, o, lse, p);
  return cudaGetLastError() == cudaSuccess ? FA_OK : FA_ERR_LAUNCH;
}

}  // namespace

int launch_fp32_simt(const float* q, const float* k, const float* v, float* o, float* lse,
                     const Fp32Params& p, cudaStream_t stream) {
  if (p.batch * p.heads > 65535) return FA_ERR_INVALID_ARG;  // grid.y limit
  switch (p.head_dim) {
    case 16: return launch<16>(q, k, v, o, lse, p, stream);
    case 32: return launch<32>(q, k, v, o, lse, p, stream);
    case 64: return launch<64>(q, k, v, o, lse, p, stream);
    case 128: return launch<128>(q, k, v, o, lse, p, stream);
    case 256: return launch<256>(q, k, v, o, lse, p, stream);
    default: return FA_ERR_UNSUPPORTED_HEAD_DIM;
  }
}

}  // namespace fa
