// Instantiation table for one head dimension.  Each fa_fwd_d<D>.cu includes this file with
// FA_HEAD_DIM defined, so the five head dimensions compile as separate translation units.
//
// Instantiated tiles (block_m = 128 * QT, block_n = BN):
//   fp16 / bf16, D <= 128 : (BN, QT) in {(128,2), (64,2), (128,1), (64,1)}
//   fp16 / bf16, D == 256 : (128,1), (64,1)          (two tiles would need 640 TMEM columns)
//   fp32 (tf32 MMA), D in {32, 64} : (128,1), (64,1), (64,2)
//   fp32 (tf32 MMA), D == 128       : (128,1), (64,1)
//   fp32, D == 16: none (tf32 MN-major V needs 128-byte rows)
//   fp32, D == 256: none (a 128-row fp32 query tile plus two K/V stages exceeds 227 KiB)
//   fp8 V (fp16 / bf16 Q, K), D in {32, 64, 128} : (128,2), (128,1); D == 256 : (128,1), (64,1)
// plus, for fp16 / bf16 at D in {64, 128}, the persistent warp-specialised kernel
// (fa_fwd_ws.cuh) behind (block_m, block_n) = (256, 128).
#pragma once

#include "fa_launch.h"

#ifndef FA_HEAD_DIM
#error "define FA_HEAD_DIM"
#endif

namespace fa {
namespace {

template <typename T>
int dispatch_tile(const LaunchPlan& lp) {
  constexpr int D = FA_HEAD_DIM;
  constexpr bool kF32 = Elt<T>::kTf32;
  if (lp.ws) {
    if constexpr (!kF32 && (D == 64 || D == 128)) return launch_ws<T, D>(lp);
    return -5;
  }
  if (lp.vf8) {
    if constexpr (!kF32 && D >= 32) {
      if (lp.block_n == 128 && lp.qt == 1) return launch_kernel<T, D, 128, 1, true>(lp);
      if constexpr (D <= 128) {
        if (lp.block_n == 128 && lp.qt == 2) return launch_kernel<T, D, 128, 2, true>(lp);
      } else {
        if (lp.block_n == 64 && lp.qt == 1) return launch_kernel<T, D, 64, 1, true>(lp);
      }
    }
    return -5;
  }
  if (lp.block_n == 128 && lp.qt == 1) return launch_kernel<T, D, 128, 1>(lp);
  if (lp.block_n == 64 && lp.qt == 1) return launch_kernel<T, D, 64, 1>(lp);
  if constexpr (!kF32 && D <= 128) {
    if (lp.block_n == 128 && lp.qt == 2) return launch_kernel<T, D, 128, 2>(lp);
    if (lp.block_n == 64 && lp.qt == 2) return launch_kernel<T, D, 64, 2>(lp);
  }
  if constexpr (kF32 && D <= 64) {
    if (lp.block_n == 64 && lp.qt == 2) return launch_kernel<T, D, 64, 2>(lp);
  }
  return -5;
}

template <typename T>
KernelInfo info_tile(int block_n, int qt, bool vf8) {
  constexpr int D = FA_HEAD_DIM;
  constexpr bool kF32 = Elt<T>::kTf32;
  if (vf8) {
    if constexpr (!kF32 && D >= 32) {
      if (block_n == 128 && qt == 1) return info_of<T, D, 128, 1, true>();
      if constexpr (D <= 128) {
        if (block_n == 128 && qt == 2) return info_of<T, D, 128, 2, true>();
      } else {
        if (block_n == 64 && qt == 1) return info_of<T, D, 64, 1, true>();
      }
    }
    return KernelInfo{false, 0, 0, 0, 0, 0, 0, 0, 0};
  }
  if (block_n == 128 && qt == 1) return info_of<T, D, 128, 1>();
  if (block_n == 64 && qt == 1) return info_of<T, D, 64, 1>();
  if constexpr (!kF32 && D <= 128) {
    if (block_n == 128 && qt == 2) return info_of<T, D, 128, 2>();
    if (block_n == 64 && qt == 2) return info_of<T, D, 64, 2>();
  }
  if constexpr (kF32 && D <= 64) {
    if (block_n == 64 && qt == 2) return info_of<T, D, 64, 2>();
  }
  return KernelInfo{false, 0, 0, 0, 0, 0, 0, 0, 0};
}

}  // namespace
}  // namespace fa

#define FA_CAT2(a, b) a##b
#define FA_CAT(a, b) FA_CAT2(a, b)

namespace fa {

int FA_CAT(launch_d, FA_HEAD_DIM)(const LaunchPlan& lp) {
  switch (lp.dtype) {
    case 0:
      return dispatch_tile<__half>(lp);
    case 1:
      return dispatch_tile<__nv_bfloat16>(lp);
    case 2:
#if FA_HEAD_DIM <= 128 && FA_HEAD_DIM >= 32
      return dispatch_tile<float>(lp);
#else
      return -5;
#endif
    default:
      return -3;
  }
}

KernelInfo FA_CAT(info_d, FA_HEAD_DIM)(int dtype, int block_n, int qt, bool vf8) {
  switch (dtype) {
    case 0:
      return info_tile<__half>(block_n, qt, vf8);
    case 1:
      return info_tile<__nv_bfloat16>(block_n, qt, vf8);
    case 2:
#if FA_HEAD_DIM <= 128 && FA_HEAD_DIM >= 32
      return info_tile<float>(block_n, qt, vf8);
#else
      return KernelInfo{false, 0, 0, 0, 0, 0, 0, 0, 0};
#endif
    default:
      return KernelInfo{false, 0, 0, 0, 0, 0, 0, 0, 0};
  }
}

}  // namespace fa
