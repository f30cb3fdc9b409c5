// Internal launch plan shared by the C-ABI front end (fa_fwd_api.cu) and the per-head-dim
// translation units (fa_fwd_d*.cu) that hold the kernel instantiations.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <cstdint>

#include "fa_fwd_kernel.cuh"
#include "fa_fwd_ws.cuh"

namespace fa {

struct LaunchPlan {
  CUtensorMap tmQ, tmK, tmV, tmO;
  FaParams params;
  int dtype;    // FaDtype
  int block_n;  // 64 / 128
  int qt;       // query tiles per CTA (block_m / 128)
  bool vf8;     // V (and P) in float8 e5m2
  bool ws;      // persistent warp-specialised kernel (fa_fwd_ws.cuh) instead of one CTA per tile
  WsParams ws_params;
  int64_t grid;
  cudaStream_t stream;
};

// Kernel geometry facts the host needs before launching (shared-memory size, TMA boxes).
struct KernelInfo {
  bool exists;
  int swz_bytes;      // swizzle span of Q/K/V/O tiles
  int box_cols;       // TMA box inner extent (elements)
  int q_tile_bytes;   // one 128-row query tile
  int kv_tile_bytes;  // one BLOCK_N-row K or V tile
  int threads;
  int smem_fixed;     // bytes besides the K/V ring
  int v_swz_bytes;    // swizzle span of V tiles (differs from the others for fp8 V)
  int v_box_cols;     // TMA box inner extent of V (elements)
};

KernelInfo kernel_info(int head_dim, int dtype, int block_n, int qt, bool vf8);
KernelInfo info_d16(int dtype, int block_n, int qt, bool vf8);
KernelInfo info_d32(int dtype, int block_n, int qt, bool vf8);
KernelInfo info_d64(int dtype, int block_n, int qt, bool vf8);
KernelInfo info_d128(int dtype, int block_n, int qt, bool vf8);
KernelInfo info_d256(int dtype, int block_n, int qt, bool vf8);

int launch_d16(const LaunchPlan& lp);
int launch_d32(const LaunchPlan& lp);
int launch_d64(const LaunchPlan& lp);
int launch_d128(const LaunchPlan& lp);
int launch_d256(const LaunchPlan& lp);

// Launch one instantiation; returns 0 or FA_ERR_LAUNCH (-7) / FA_ERR_UNSUPPORTED_TILE (-5).
template <typename T, int D, int BN, int QT, bool VF8 = false>
int launch_kernel(const LaunchPlan& lp) {
  using G = Geo<T, D, BN, QT, VF8>;
  auto kern = fa_fwd_sm100_kernel<T, D, BN, QT, VF8>;
  const int smem = G::smem_bytes(lp.params.stages);
  if constexpr (QT == 2) {
    // setmaxnreg redistributes exactly the launch allocation; refuse to launch a build whose
    // per-thread register count differs (the split would not add up).
    static int regs_ok = 0;  // 0 unknown, 1 ok, -1 mismatch
    if (regs_ok == 0) {
      cudaFuncAttributes fattr{};
      regs_ok = (cudaFuncGetAttributes(&fattr, kern) == cudaSuccess &&
                 fattr.numRegs == G::REG_LAUNCH)
                    ? 1
                    : -1;
      (void)cudaGetLastError();
    }
    if (regs_ok != 1) return -7;
  }
  if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem) !=
      cudaSuccess) {
    (void)cudaGetLastError();
    return -7;
  }
  kern<<<dim3(static_cast<unsigned>(lp.grid)), dim3(G::NUM_THREADS), smem, lp.stream>>>(
      lp.tmQ, lp.tmK, lp.tmV, lp.tmO, lp.params);
  return cudaGetLastError() == cudaSuccess ? 0 : -7;
}

// Launch the persistent kernel; lp.grid CTAs loop over lp.ws_params.total_tiles tiles.
template <typename T, int D>
int launch_ws(const LaunchPlan& lp) {
  using G = WsGeo<T, D>;
  auto kern = fa_fwd_ws_kernel<T, D>;
  const int smem = ws_smem_bytes<D>(lp.ws_params.stages);
  // The setmaxnreg split redistributes exactly the launch allocation (128 registers per thread
  // for 512 threads); refuse a build whose per-thread count differs.
  static int regs_ok = 0;  // 0 unknown, 1 ok, -1 mismatch
  if (regs_ok == 0) {
    cudaFuncAttributes fattr{};
    regs_ok = (cudaFuncGetAttributes(&fattr, kern) == cudaSuccess && fattr.numRegs == 128) ? 1 : -1;
    (void)cudaGetLastError();
  }
  if (regs_ok != 1) return -7;
  if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem) !=
      cudaSuccess) {
    (void)cudaGetLastError();
    return -7;
  }
  kern<<<dim3(static_cast<unsigned>(lp.grid)), dim3(G::NUM_THREADS), smem, lp.stream>>>(
      lp.tmQ, lp.tmK, lp.tmV, lp.tmO, lp.ws_params);
  return cudaGetLastError() == cudaSuccess ? 0 : -7;
}

// Shared-memory footprint of the persistent kernel besides its K/V ring, and one ring stage.
template <int D>
constexpr int ws_smem_fixed() {
  return ws_smem_bytes<D>(0);
}
template <int D>
constexpr int ws_stage_bytes() {
  return WsGeo<__nv_bfloat16, D>::KV_TILE_BYTES;
}

template <typename T, int D, int BN, int QT, bool VF8 = false>
constexpr KernelInfo info_of() {
  using G = Geo<T, D, BN, QT, VF8>;
  return KernelInfo{true,           G::SWZ,         G::BLK_COLS,
                    G::Q_TILE_BYTES, G::KV_TILE_BYTES, G::NUM_THREADS,
                    G::smem_bytes(0), G::V_SWZ,      G::V_BLK_COLS};
}

}  // namespace fa
