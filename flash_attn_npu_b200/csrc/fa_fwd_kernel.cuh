// FlashAttention forward for B200 (sm_100a): warp-specialised TMA -> tcgen05 -> TMEM pipeline.
//
// What it computes (same contract as the reference Triton kernel `_attn_fwd`,
// flash_attention_forward.py:1036-1111 and its tile body `_attn_fwd_tile`, :872-1033):
//   O[b,h,i,:]  = sum_j softmax_j(scale * q_i . k_j) v_j      (keys j <= i when causal)
//   LSE[b,h,i]  = log sum_j exp(scale * q_i . k_j)           (natural log, fp32)
// The reference keeps a running max m and sum l (`_attn_fwd_inner_loop`, :698-724) and
// finishes with m += log(l), O = acc / l (:1022-1033).  This kernel keeps the same online
// softmax but works in base 2 (exp2 with scale*log2(e) folded in), applies the scale to the
// fp32 logits instead of pre-rounding q (:977-978), masks with -inf rather than -1e6
// (:694-696), and masks the key tail instead of dropping keys past the last full block (:846-869).
//
// CTA shape (one CTA per SM; TMEM and shared memory sized for that):
//   QT query tiles of 128 rows for one (batch, head); BLOCK_M = 128 * QT.
//   warp 0        : TMA producer (Q once, then K/V tiles into a ring of `stages` slots)
//   warp 1        : TMEM allocator + tcgen05.mma issuer (one thread; with QT == 2, tile 0's)
//   warp 2        : QT == 2: tcgen05.mma issuer of tile 1 (the two issuers take turns)
//   warps 2-3     : otherwise idle (keep the softmax warpgroups aligned to TMEM lane quarters)
//   warps 4+4i..  : softmax warpgroup i (thread r owns query row r of tile i = TMEM lane r)
// TMEM columns: S_i (fp32 logits, BN cols) at i*BN, then O_i (fp32, D cols) at QT*BN + i*D.
// P_i (the probabilities, in the input dtype) is written back over the first columns of S_i
// and consumed from TMEM by the P.V MMA (A operand in tensor memory).
//
// Per KV step j the MMA thread issues, for each tile i in order:
//   O_i (+)= P_i(j) V_j ;  S_i(j+1) = Q_i K_{j+1}^T
// tcgen05 MMAs from one thread complete in issue order, so when softmax warpgroup i sees
// S_i(j+1) complete, O_i already holds P_i(j) V_j: the warpgroup can rescale O_i in TMEM
// before releasing P_i(j+1), with no extra barrier.
//
// Rescaling is conditional: the exponent base m only moves when the row max grows by more
// than RESCALE_LOG2 (p values then stay <= 2^RESCALE_LOG2).  The result is exact because
// l and O are both accumulated against the same base.
//
// Every wait is bounded (FA_WAIT_TIMEOUT_NS); a wait that gives up records
// FA_ERR_DEVICE_TIMEOUT in *status, raises a CTA-wide abort flag and all roles drain to the
// teardown, which waits for in-flight copies and MMAs (bounded separately, FA_DRAIN_TIMEOUT_NS)
// before TMEM is freed.
#pragma once

#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cstdint>
#include <type_traits>

#include "sm100_ptx.cuh"

#ifndef FA_WAIT_TIMEOUT_NS
#define FA_WAIT_TIMEOUT_NS 2000000000ull
#endif
// Limit of the teardown drains: a role that stops early still waits this long for the TMA
// loads and MMAs it has issued (they always complete; the limit only bounds the spin).  It is
// separate from FA_WAIT_TIMEOUT_NS so that a build with a short pipeline limit still drains.
#ifndef FA_DRAIN_TIMEOUT_NS
#define FA_DRAIN_TIMEOUT_NS 4000000000ull
#endif

namespace fa {

constexpr float kLog2e = 1.4426950408889634f;
constexpr float kLn2 = 0.6931471805599453f;
constexpr float RESCALE_LOG2 = 8.0f;
// Every p = 2^(x - base) of a row is <= 2^RESCALE_LOG2 whenever the row's sum is; the bound
// sits just below 256 so that an element at the limit (ex2.approx may round it to 256) still
// sends the row through the exact max check.
constexpr float P_SUM_BOUND = 255.0f;
constexpr int kMaxStages = 8;
constexpr int kStatusTimeout = -9;  // FA_ERR_DEVICE_TIMEOUT

// With two query tiles per CTA the MMAs are issued from two warps, one per tile, which take
// turns through a pair of named barriers (see the MMA issuers in the kernel).  0 keeps the
// single issuing thread.
#ifndef FA_DUAL_ISSUE
#define FA_DUAL_ISSUE 1
#endif

struct FaParams {
  int batch;
  int heads;
  int seqlen;
  int n_qblocks;   // ceil(seqlen / BLOCK_M)
  int causal;
  int stages;      // K/V ring depth
  float scale_log2;
  float* lse;      // [B, H, S] fp32 contiguous
  int* status;     // optional
};

template <typename T>
struct Elt;
template <>
struct Elt<__nv_bfloat16> {
  static constexpr int kBytes = 2;
  static constexpr uint32_t kFmt = 1;
  static constexpr bool kTf32 = false;
};
template <>
struct Elt<__half> {
  static constexpr int kBytes = 2;
  static constexpr uint32_t kFmt = 0;
  static constexpr bool kTf32 = false;
};
template <>
struct Elt<float> {
  static constexpr int kBytes = 4;
  static constexpr uint32_t kFmt = 2;
  static constexpr bool kTf32 = true;
};
// float8 e5m2: the V operand (and P) of the fp8-V variant; kind::f8f6f4 format code 1.
struct E5M2 {};
template <>
struct Elt<E5M2> {
  static constexpr int kBytes = 1;
  static constexpr uint32_t kFmt = 1;
  static constexpr bool kTf32 = false;
};

// Compile-time geometry of one kernel instantiation.  VF8: V (and so P) is float8 e5m2 while
// Q, K and O stay T.
template <typename T, int D, int BN, int QT, bool VF8 = false>
struct Geo {
  static constexpr int EB = Elt<T>::kBytes;
  static constexpr int ROW_BYTES = D * EB;                        // one row of Q/K/V/O
  static constexpr int SWZ = ROW_BYTES >= 128 ? 128 : ROW_BYTES;  // swizzle span (32/64/128 B)
  static constexpr int BLK_COLS = SWZ / EB;                       // TMA box inner extent
  static constexpr int NBLK = ROW_BYTES / SWZ;                    // column blocks per row
  static constexpr int BM = 128;                                  // rows per query tile
  static constexpr int Q_BLK_BYTES = BM * SWZ;
  static constexpr int Q_TILE_BYTES = BM * ROW_BYTES;
  static constexpr int KV_BLK_BYTES = BN * SWZ;
  static constexpr int KV_TILE_BYTES = BN * ROW_BYTES;
  static constexpr int KSTEPS_PER_BLK = SWZ / 32;  // MMA K is always 32 bytes
  static constexpr int MMA_K = 32 / EB;            // 16 (f16/bf16) or 8 (tf32)
  // P and V share one element type: T, or e5m2 for the fp8-V variant.
  using PT = typename std::conditional<VF8, E5M2, T>::type;
  static constexpr int VEB = Elt<PT>::kBytes;
  static constexpr int V_ROW_BYTES = D * VEB;
  static constexpr int V_SWZ = VF8 ? (V_ROW_BYTES >= 128 ? 128 : V_ROW_BYTES) : SWZ;
  static constexpr int V_BLK_COLS = V_SWZ / VEB;   // TMA box inner extent of V
  static constexpr int V_NBLK = V_ROW_BYTES / V_SWZ;
  static constexpr int V_BLK_BYTES = BN * V_SWZ;
  static constexpr int V_TILE_BYTES = BN * V_ROW_BYTES;
  static constexpr int PV_K = 32 / VEB;            // keys per P.V MMA (32 bytes of K)
  static constexpr int P_COLS = BN * VEB / 4;      // TMEM columns holding P
  static constexpr int TMEM_S = 0;
  static constexpr int TMEM_O = QT * BN;
  static constexpr int TMEM_USED = QT * (BN + D);
  static constexpr int TMEM_ALLOC = TMEM_USED <= 32    ? 32
                                    : TMEM_USED <= 64  ? 64
                                    : TMEM_USED <= 128 ? 128
                                    : TMEM_USED <= 256 ? 256
                                                       : 512;
  static constexpr int NUM_THREADS = 128 + 128 * QT;
  // Register split for QT == 2: 128 x 80 + 256 x 208 = 63488 <= 384 threads x 168 = 64512.
  static constexpr int REG_LAUNCH = 168;
  static constexpr int REG_LOW = 80;
  static constexpr int REG_HIGH = 208;
  static_assert(QT != 2 || 128 * REG_LOW + 256 * REG_HIGH <= NUM_THREADS * REG_LAUNCH,
                "register split must fit the launch allocation");
  static constexpr uint32_t LAYOUT = SWZ == 128 ? 2u : (SWZ == 64 ? 4u : 6u);
  // V is the MN-major operand of P.V.  For tf32 that operand needs the 32-byte-atom 128B
  // swizzle (descriptor code 1, 4-row K groups; TMA CU_TENSOR_MAP_SWIZZLE_128B_ATOM_32B).
  static constexpr uint32_t V_LAYOUT =
      Elt<T>::kTf32 ? 1u : (V_SWZ == 128 ? 2u : (V_SWZ == 64 ? 4u : 6u));
  static constexpr int V_SBO = Elt<T>::kTf32 ? 4 * SWZ : 8 * V_SWZ;
  static constexpr uint32_t IDESC_S = make_idesc(Elt<T>::kFmt, false, 128, BN);
  static constexpr uint32_t IDESC_O = make_idesc(Elt<PT>::kFmt, true, 128, D);
  // Shared memory: [Q tiles][K/V ring][barriers]; +1024 for base alignment.
  static constexpr int BAR_BYTES = 256;
  static constexpr int smem_bytes(int stages) {
    return 1024 + QT * Q_TILE_BYTES + stages * KV_TILE_BYTES + BAR_BYTES;
  }
  static_assert(TMEM_USED <= 512, "TMEM budget exceeded");
  static_assert(BN == 64 || BN == 128, "BLOCK_N must be 64 or 128");
  static_assert(QT == 1 || QT == 2, "1 or 2 query tiles per CTA");
  static_assert(D % 16 == 0 && D >= 16 && D <= 256, "head_dim");
  static_assert(ROW_BYTES % SWZ == 0, "row must be whole swizzle spans");
  static_assert(!Elt<T>::kTf32 || SWZ == 128, "tf32 needs rows of >= 128 bytes (head_dim >= 32)");
  static_assert(Q_BLK_BYTES % 1024 == 0 && KV_BLK_BYTES % 1024 == 0, "1 KiB tile alignment");
  static_assert(!VF8 || (!Elt<T>::kTf32 && V_SWZ >= 32 && V_BLK_BYTES % 1024 == 0),
                "fp8 V: 16-bit Q/K and rows of at least 32 bytes");
};

// Physical byte offset of logical byte `off` inside a TMA-swizzled region with span SWZ.
template <int SWZ>
__device__ __forceinline__ uint32_t swizzle(uint32_t off) {
  constexpr uint32_t mask = SWZ / 16 - 1;
  return off ^ (((off >> 7) & mask) << 4);
}

struct Shared {
  uint64_t full[kMaxStages];
  uint64_t empty[kMaxStages];
  uint64_t q_full;
  uint64_t s_full[2];
  uint64_t p_full[2];
  uint64_t o_full[2];
  uint64_t mma_done;
  uint32_t tmem_base;
  volatile uint32_t abort_flag;
};
static_assert(sizeof(Shared) <= 256, "barrier block");

// Polls a pipeline wait makes between looks at the clock and the abort flag.  The test build
// of the bounded waits sets FA_WAIT_POLL_NONBLOCKING, FA_WAIT_SPIN_POLLS = 0 and
// FA_WAIT_TIMEOUT_NS = 0: a wait whose phase is not complete at its first (non-suspending)
// probe gives up at once.
#ifndef FA_WAIT_SPIN_POLLS
#define FA_WAIT_SPIN_POLLS 32
#endif
// FA_WAIT_SUSPEND_HINT_NS > 0: each probe may sleep up to that long for the phase.
#ifndef FA_WAIT_SUSPEND_HINT_NS
#define FA_WAIT_SUSPEND_HINT_NS 0
#endif
__device__ __forceinline__ bool wait_poll(uint32_t bar, uint32_t parity) {
#if defined(FA_WAIT_POLL_NONBLOCKING)
  return mbar_test_wait(bar, parity);
#elif FA_WAIT_SUSPEND_HINT_NS > 0
  return mbar_try_wait_hint(bar, parity, FA_WAIT_SUSPEND_HINT_NS);
#else
  return mbar_try_wait(bar, parity);
#endif
}

// Bounded mbarrier wait.  Returns false on timeout or if another role already aborted
// (`abort_flag` is the CTA's shared abort word).
__device__ __forceinline__ bool wait_bar_flag(volatile uint32_t* abort_flag, uint32_t bar,
                                              uint32_t parity, int* status) {
  if (wait_poll(bar, parity)) return true;
  const uint64_t t0 = globaltimer_ns();
  while (true) {
#pragma unroll 1
    for (int i = 0; i < FA_WAIT_SPIN_POLLS; ++i)
      if (wait_poll(bar, parity)) return true;
    if (*abort_flag) return false;
    if (globaltimer_ns() - t0 >= FA_WAIT_TIMEOUT_NS) {
      *abort_flag = 1u;
      if (status) atomicCAS(status, 0, kStatusTimeout);
      return false;
    }
  }
}

__device__ __forceinline__ bool wait_bar(Shared* sh, uint32_t bar, uint32_t parity, int* status) {
  return wait_bar_flag(&sh->abort_flag, bar, parity, status);
}

// Drain wait: spins on the phase until it completes or FA_DRAIN_TIMEOUT_NS passes, ignoring
// the abort flag (it waits for the role's own copies or MMAs, which complete regardless).
__device__ __forceinline__ void drain_bar(uint32_t bar, uint32_t parity) {
  if (mbar_try_wait(bar, parity)) return;
  const uint64_t t0 = globaltimer_ns();
  while (!mbar_try_wait(bar, parity) && globaltimer_ns() - t0 < FA_DRAIN_TIMEOUT_NS) {
  }
}

// Round two floats to a packed 16-bit pair: `lo` in bits 0-15, `hi` in bits 16-31
// (cvt.rn.{bf16,f16}x2.f32 d, a, b puts a in the upper half).
__device__ __forceinline__ uint32_t pack2(float lo, float hi, __nv_bfloat16*) {
  uint32_t d;
  asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(d) : "f"(hi), "f"(lo));
  return d;
}
__device__ __forceinline__ uint32_t pack2(float lo, float hi, __half*) {
  uint32_t d;
  asm("cvt.rn.f16x2.f32 %0, %1, %2;" : "=r"(d) : "f"(hi), "f"(lo));
  return d;
}

// --------------------------------------------------------------------------------------
// exp2 on the FMA pipe, for a pair of lanes.  2^x = 2^n * 2^f with n = round(x) taken from the
// low mantissa bits of x + 1.5*2^23 and f = x - n in [-0.5, 0.5]; 2^f is a degree-4 polynomial
// minimising the relative error on that interval (coefficients from csrc/exp2_poly_fit.py, max
// relative error 2.7e-6 in fp32 Horner form).  2^n is applied by adding n to the exponent
// field.  x is clamped at -126: with n >= -126 and 2^f >= 2^-0.5 (biased exponent >= 126) the
// exponent field stays >= 0 (at -127 a value 2^f < 1 wrapped into the sign bit and gave a NaN
// pattern); 2^-126 is ~0 here.
#ifndef FA_POLY_PAIRS_OF_8
#define FA_POLY_PAIRS_OF_8 0  // element pairs out of every 8 that use the polynomial
#endif
__device__ __forceinline__ float2 exp2_poly2(float2 x) {
  constexpr float kRound = 12582912.0f;  // 1.5 * 2^23
  constexpr float c0 = 9.999992847e-01f, c1 = 6.931217909e-01f, c2 = 2.402474433e-01f,
                  c3 = 5.591785908e-02f, c4 = 9.570101276e-03f;
  x.x = fmaxf(x.x, -126.f);
  x.y = fmaxf(x.y, -126.f);
  const float2 t = fadd2(x, make_float2(kRound, kRound));
  const float2 n = fadd2(t, make_float2(-kRound, -kRound));
  const float2 f = ffma2(n, make_float2(-1.f, -1.f), x);
  float2 q = ffma2(make_float2(c4, c4), f, make_float2(c3, c3));
  q = ffma2(q, f, make_float2(c2, c2));
  q = ffma2(q, f, make_float2(c1, c1));
  q = ffma2(q, f, make_float2(c0, c0));
  // bits(t) = bits(kRound) + n and bits(kRound) << 23 == 0 (mod 2^32): (bits(t) << 23) == n << 23
  q.x = __int_as_float(__float_as_int(q.x) + (__float_as_int(t.x) << 23));
  q.y = __int_as_float(__float_as_int(q.y) + (__float_as_int(t.y) << 23));
  return q;
}

// Degree-3 variant of the same routine (one FMA pair fewer; max relative error 7.5e-5, from
// csrc/exp2_poly_fit.py with degree 3).  The persistent kernel routes a minority of its exp2s
// here: P is rounded to 16 bits (relative step 2^-8 .. 2^-11) and the row sum l mixes these
// values with ex2.approx ones, which keeps the logsumexp well inside its 1e-4 bar.
__device__ __forceinline__ float2 exp2_poly2_deg3(float2 x) {
  constexpr float kRound = 12582912.0f;  // 1.5 * 2^23
  constexpr float c0 = 9.999280572e-01f, c1 = 6.932609677e-01f, c2 = 2.426111251e-01f,
                  c3 = 5.517166480e-02f;
  x.x = fmaxf(x.x, -126.f);
  x.y = fmaxf(x.y, -126.f);
  const float2 t = fadd2(x, make_float2(kRound, kRound));
  const float2 n = fadd2(t, make_float2(-kRound, -kRound));
  const float2 f = ffma2(n, make_float2(-1.f, -1.f), x);
  float2 q = ffma2(make_float2(c3, c3), f, make_float2(c2, c2));
  q = ffma2(q, f, make_float2(c1, c1));
  q = ffma2(q, f, make_float2(c0, c0));
  q.x = __int_as_float(__float_as_int(q.x) + (__float_as_int(t.x) << 23));
  q.y = __int_as_float(__float_as_int(q.y) + (__float_as_int(t.y) << 23));
  return q;
}

// Row maximum of BN logits with 3-input max, 8 independent chains.
template <int BN>
__device__ __forceinline__ float row_max(const float* s) {
  float e[8];
#pragma unroll
  for (int t = 0; t < 8; ++t) e[t] = fmaxf(s[2 * t], s[2 * t + 1]);
#pragma unroll
  for (int k = 16; k < BN; k += 16) {
#pragma unroll
    for (int t = 0; t < 8; ++t) e[t] = fmax3(e[t], s[k + 2 * t], s[k + 2 * t + 1]);
  }
  return fmax3(fmax3(e[0], e[1], e[2]), fmax3(e[3], e[4], e[5]), fmaxf(e[6], e[7]));
}

// P = 2^(s*sl2 + neg_m) for an unmasked row, written to TMEM at tP in two halves: the store of
// the first half is in flight while the second half is computed (the caller waits once; the
// store reads its source registers asynchronously, so finer chunking would pin more of them).
// Returns the row sum of the unrounded fp32 values.  s is left intact.  A fixed share of the
// element pairs can go through the FMA-pipe polynomial.
template <typename T, int BN>
__device__ __forceinline__ float exp2_row_store(const float* s, float sl2, float neg_m, uint32_t tP) {
  constexpr int HALF = BN / 2;
  constexpr int PW = HALF * Elt<T>::kBytes / 4;  // 32-bit TMEM words per half row
  const float2 sc = make_float2(sl2, sl2);
  const float2 nm = make_float2(neg_m, neg_m);
  float2 acc[4];
#pragma unroll
  for (int t = 0; t < 4; ++t) acc[t] = make_float2(0.f, 0.f);
#pragma unroll
  for (int h = 0; h < 2; ++h) {
    uint32_t pk[PW];
    float2 pend = make_float2(0.f, 0.f);
#pragma unroll
    for (int k = h * HALF; k < (h + 1) * HALF; k += 2) {
      const float2 x = ffma2(make_float2(s[k], s[k + 1]), sc, nm);
      float2 pr;
      if (((k >> 1) & 7) < FA_POLY_PAIRS_OF_8) {
        pr = exp2_poly2(x);
      } else {
        pr.x = ex2_approx(x.x);
        pr.y = ex2_approx(x.y);
      }
      acc[(k >> 1) & 3] = fadd2(acc[(k >> 1) & 3], pr);
      const int w = (k - h * HALF) >> 1;
      if constexpr (Elt<T>::kTf32) {
        pk[2 * w] = __float_as_uint(pr.x);
        pk[2 * w + 1] = __float_as_uint(pr.y);
      } else if constexpr (Elt<T>::kBytes == 1) {
        // four e5m2 per word: the even pair is held until the odd pair completes the word
        if (w & 1)
          pk[w >> 1] = pack4_e5m2(pend.x, pend.y, pr.x, pr.y);
        else
          pend = pr;
      } else {
        pk[w] = pack2(pr.x, pr.y, static_cast<T*>(nullptr));
      }
    }
#pragma unroll
    for (int w = 0; w < PW; w += 32) {
      if constexpr (PW >= 32)
        tmem_st32(tP + h * PW + w, pk + w);
      else if constexpr (PW >= 16)
        tmem_st16(tP + h * PW + w, pk + w);
      else
        tmem_st8(tP + h * PW + w, pk + w);
    }
  }
  const float2 a = fadd2(fadd2(acc[0], acc[1]), fadd2(acc[2], acc[3]));
  return a.x + a.y;
}

template <typename T, int D, int BN, int QT, bool VF8 = false>
__global__ void __launch_bounds__(Geo<T, D, BN, QT, VF8>::NUM_THREADS, 1)
    fa_fwd_sm100_kernel(const __grid_constant__ CUtensorMap tmQ,
                        const __grid_constant__ CUtensorMap tmK,
                        const __grid_constant__ CUtensorMap tmV,
                        const __grid_constant__ CUtensorMap tmO, const FaParams p) {
  using G = Geo<T, D, BN, QT, VF8>;
  using PT = typename G::PT;  // element type of P and V
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  uint8_t* q_smem = smem;
  uint8_t* kv_smem = smem + QT * G::Q_TILE_BYTES;
  Shared* sh = reinterpret_cast<Shared*>(kv_smem + p.stages * G::KV_TILE_BYTES);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int stages = p.stages;
  // Two issuing warps (QT == 2): every K/V slot is released by one arrival per issuer.
  constexpr bool kDual = QT == 2 && FA_DUAL_ISSUE != 0;
  constexpr uint32_t kIssuers = kDual ? 2u : 1u;

  // ---- tile coordinates (causal: longest q-blocks first; non-causal: q-blocks of one head
  //      adjacent so K/V stay in L2 -- the reference's two orders, :915-922)
  const int bh_count = p.batch * p.heads;
  int qblk, bh;
  if (p.causal) {
    qblk = p.n_qblocks - 1 - static_cast<int>(blockIdx.x / bh_count);
    bh = static_cast<int>(blockIdx.x % bh_count);
  } else {
    bh = static_cast<int>(blockIdx.x / p.n_qblocks);
    qblk = static_cast<int>(blockIdx.x % p.n_qblocks);
  }
  const int bi = bh / p.heads;
  const int hi = bh % p.heads;
  const int q0 = qblk * (G::BM * QT);

  // KV steps needed by each query tile (0 = tile lies entirely past the sequence end).
  int n_kv[QT];
  int n_max = 0;
#pragma unroll
  for (int i = 0; i < QT; ++i) {
    const int row0 = q0 + G::BM * i;
    if (row0 >= p.seqlen) {
      n_kv[i] = 0;
    } else {
      const int kv_end = p.causal ? min(p.seqlen, row0 + G::BM) : p.seqlen;
      n_kv[i] = (kv_end + BN - 1) / BN;
    }
    n_max = max(n_max, n_kv[i]);
  }

  // ---- setup
  if (threadIdx.x == 0) {
    for (int s = 0; s < stages; ++s) {
      mbar_init(smem_u32(&sh->full[s]), 1);
      mbar_init(smem_u32(&sh->empty[s]), kIssuers);
    }
    mbar_init(smem_u32(&sh->q_full), 1);
    for (int i = 0; i < 2; ++i) {
      mbar_init(smem_u32(&sh->s_full[i]), 1);
      mbar_init(smem_u32(&sh->p_full[i]), 128);
      mbar_init(smem_u32(&sh->o_full[i]), 1);
    }
    mbar_init(smem_u32(&sh->mma_done), kIssuers);
    sh->abort_flag = 0u;
    fence_mbar_init();
  }
  if (warp == 0 && lane == 0) {
    prefetch_tmap(&tmQ);
    prefetch_tmap(&tmK);
    prefetch_tmap(&tmV);
    prefetch_tmap(&tmO);
  }
  if (warp == 1) {
    tmem_alloc(smem_u32(&sh->tmem_base), G::TMEM_ALLOC);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = sh->tmem_base;

  // QT == 2: the producer/MMA warpgroup (warps 0-3) hands registers to the two softmax
  // warpgroups.  The split sums to the launch allocation (the host refuses to launch a build
  // whose per-thread count is not REG_LAUNCH).  Each setmaxnreg sits at the top of its role's
  // branch so the register limit it sets covers that role's code.
  if (warp < 4) {
    if constexpr (QT == 2) setmaxnreg_dec<G::REG_LOW>();
  if (warp == 0) {
    // ================================================================ TMA producer
    if (lane == 0) {
      int issued = 0;  // K/V ring loads issued
      bool q_issued = false;
      bool ok = true;
      if (n_max > 0) {
        uint32_t qbytes = 0;
#pragma unroll
        for (int i = 0; i < QT; ++i)
          if (n_kv[i] > 0) qbytes += G::Q_TILE_BYTES;
        const uint32_t qbar = smem_u32(&sh->q_full);
        mbar_arrive_expect_tx(qbar, qbytes);
#pragma unroll
        for (int i = 0; i < QT; ++i) {
          if (n_kv[i] == 0) continue;
#pragma unroll
          for (int c = 0; c < G::NBLK; ++c)
            tma_load_4d(smem_u32(q_smem + i * G::Q_TILE_BYTES + c * G::Q_BLK_BYTES), &tmQ, qbar,
                        c * G::BLK_COLS, q0 + G::BM * i, hi, bi);
        }
        q_issued = true;
        int slot = 0;
        uint32_t phase = 0;
        for (int j = 0; j < n_max && ok; ++j) {
#pragma unroll
          for (int kv = 0; kv < 2; ++kv) {
            if (!wait_bar(sh, smem_u32(&sh->empty[slot]), phase ^ 1u, p.status)) {
              ok = false;
              break;
            }
            const uint32_t fbar = smem_u32(&sh->full[slot]);
            uint8_t* dst = kv_smem + slot * G::KV_TILE_BYTES;
            if (kv == 0) {
              mbar_arrive_expect_tx(fbar, G::KV_TILE_BYTES);
#pragma unroll
              for (int c = 0; c < G::NBLK; ++c)
                tma_load_4d(smem_u32(dst + c * G::KV_BLK_BYTES), &tmK, fbar, c * G::BLK_COLS,
                            j * BN, hi, bi);
            } else {
              // V may be narrower than K (fp8); it starts at the slot's base either way.
              mbar_arrive_expect_tx(fbar, G::V_TILE_BYTES);
#pragma unroll
              for (int c = 0; c < G::V_NBLK; ++c)
                tma_load_4d(smem_u32(dst + c * G::V_BLK_BYTES), &tmV, fbar, c * G::V_BLK_COLS,
                            j * BN, hi, bi);
            }
            ++issued;
            if (++slot == stages) {
              slot = 0;
              phase ^= 1u;
            }
          }
        }
      }
      {
        // Drain, on every path (another role may have stopped after the last load was
        // issued): every load issued must land before the CTA's shared memory goes away.  A
        // load older than the last `stages` has landed already (its slot was refilled only
        // after the MMA thread had waited for it); in a run without abort these waits return
        // at once.
        if (q_issued) drain_bar(smem_u32(&sh->q_full), 0);
        const int outstanding = min(issued, stages);
        for (int t = 0; t < outstanding; ++t) {
          const int idx = issued - 1 - t;
          drain_bar(smem_u32(&sh->full[idx % stages]), static_cast<uint32_t>((idx / stages) & 1));
        }
      }
    }
  } else if (warp == 1 || (kDual && warp == 2)) {
    // ================================================================ MMA issuer(s)
    {
      // The issuing thread shares its SM sub-partition with two busy softmax warps, so its
      // instruction stream is kept minimal: descriptors are built once and their start-address
      // field (bits 0-13 = address >> 4) is advanced by adding byte offsets >> 4 (shared memory
      // stays below 256 KiB, so the field never carries into the next one); ring slots and
      // phases advance incrementally.
      const uint64_t q_desc = make_smem_desc(smem_u32(q_smem), 16, 8 * G::SWZ, G::LAYOUT);
      const uint64_t k_desc = make_smem_desc(smem_u32(kv_smem), 16, 8 * G::SWZ, G::LAYOUT);
      const uint64_t v_desc =
          make_smem_desc(smem_u32(kv_smem), G::V_BLK_BYTES, G::V_SBO, G::V_LAYOUT);
      constexpr uint32_t kSlotStep = G::KV_TILE_BYTES >> 4;
      const uint32_t full0 = smem_u32(&sh->full[0]);
      const uint32_t empty0 = smem_u32(&sh->empty[0]);

      // S_i = Q_i K^T : A = Q tile (K-major), B = K tile (K-major), both SWZ-swizzled.
      auto issue_s = [&](int i, int kslot) {
        const uint64_t a0 = q_desc + static_cast<uint64_t>((i * G::Q_TILE_BYTES) >> 4);
        const uint64_t b0 = k_desc + static_cast<uint64_t>(kslot * kSlotStep);
        const uint32_t d = tmem + G::TMEM_S + i * BN;
#pragma unroll
        for (int c = 0; c < G::NBLK; ++c) {
#pragma unroll
          for (int kk = 0; kk < G::KSTEPS_PER_BLK; ++kk) {
            const uint64_t ad = a0 + static_cast<uint64_t>((c * G::Q_BLK_BYTES + kk * 32) >> 4);
            const uint64_t bd = b0 + static_cast<uint64_t>((c * G::KV_BLK_BYTES + kk * 32) >> 4);
            if constexpr (Elt<T>::kTf32)
              mma_tf32_ss(d, ad, bd, G::IDESC_S, (c | kk) ? 1u : 0u);
            else
              mma_f16_ss(d, ad, bd, G::IDESC_S, (c | kk) ? 1u : 0u);
          }
        }
      };
      // O_i (+)= P_i V : A = P_i in TMEM, B = V tile (MN-major: rows = keys, cols = head dim).
      auto issue_pv = [&](int i, int vslot, uint32_t acc0) {
        const uint64_t b0 = v_desc + static_cast<uint64_t>(vslot * kSlotStep);
        const uint32_t d = tmem + G::TMEM_O + i * D;
        const uint32_t a = tmem + G::TMEM_S + i * BN;
#pragma unroll
        for (int kk = 0; kk < BN / G::PV_K; ++kk) {
          // PV_K keys = PV_K rows of V; each TMEM column of P holds 4 bytes
          const uint64_t bd = b0 + static_cast<uint64_t>((kk * G::PV_K * G::V_SWZ) >> 4);
          const uint32_t acol = static_cast<uint32_t>(kk * G::PV_K * G::VEB / 4);
          if constexpr (VF8)
            mma_f8_ts(d, a + acol, bd, G::IDESC_O, kk > 0 ? 1u : acc0);
          else if constexpr (Elt<T>::kTf32)
            mma_tf32_ts(d, a + acol, bd, G::IDESC_O, kk > 0 ? 1u : acc0);
          else
            mma_f16_ts(d, a + acol, bd, G::IDESC_O, kk > 0 ? 1u : acc0);
        }
      };
      auto advance = [&](int& sl, uint32_t& ph) {
        if (++sl == stages) {
          sl = 0;
          ph ^= 1u;
        }
      };

      if constexpr (kDual) {
        // Two issuers: warp 1 issues tile 0's MMAs, warp 2 tile 1's (lane 0 issues, the warp
        // stays converged for the named barriers).  They take turns -- S_0(0), S_1(0), then per
        // step j: P_0(j) V_j + Q_0 K_{j+1}^T, P_1(j) V_j + Q_1 K_{j+1}^T -- so the tensor pipe sees
        // the single issuer's order, but each warp waits for its own operands (V_j, K_{j+1},
        // P_i(j)) while the other warp's MMAs are going out, and picks up the turn with one
        // named-barrier hand-off instead of a chain of mbarrier waits between two MMA runs.
        // Turn passing: barrier kTok0 (tile 0 done -> tile 1 may issue), kTok1 (the reverse);
        // bar.arrive by the passer, bar.sync by the taker.  Both warps run the same number of
        // hand-offs whatever happens (an aborted wait only stops the issuing), so neither is
        // left waiting on a named barrier.
        // A K/V slot's empty barrier counts two arrivals: each tile that reads the slot commits
        // once, and a tile that is the slot's only reader (the other tile has run out of keys,
        // causal, or lies past the sequence end) commits twice.  Every commit follows MMAs that
        // read the slot, so no arrival can land in the slot's previous phase.
        constexpr uint32_t kTok0 = 3, kTok1 = 4;
        const int ti = warp - 1;
        const bool lead = lane == 0;
        auto pass_turn = [&]() {
          __syncwarp();
          named_barrier_arrive(ti == 0 ? kTok0 : kTok1, 64);
        };
        auto take_turn = [&]() {
          __syncwarp();
          named_barrier_sync(ti == 0 ? kTok1 : kTok0, 64);
        };
        auto wait_all = [&](uint32_t bar, uint32_t parity) {
          return __all_sync(0xffffffffu, wait_bar(sh, bar, parity, p.status));
        };
        if (n_max > 0) {
          const int mine = ti == 0 ? n_kv[0] : n_kv[QT - 1];
          const int other = ti == 0 ? n_kv[QT - 1] : n_kv[0];
          bool ok = wait_all(smem_u32(&sh->q_full), 0);
          if (ok) ok = wait_all(full0, 0);  // K_0
          tc_fence_after();
          if (ti == 1) take_turn();
          if (ok && lead && mine > 0) {
            issue_s(ti, 0);
            mma_commit(smem_u32(&sh->s_full[ti]));
            mma_commit(empty0);
            if (other == 0) mma_commit(empty0);
          }
          pass_turn();
          int vs = 0;
          uint32_t vph = 0;
          advance(vs, vph);  // V_0
          for (int j = 0; j < n_max; ++j) {
            int ks = vs;
            uint32_t kph = vph;
            advance(ks, kph);  // K_{j+1}
            const bool act = j < mine;          // P_i(j) V_j
            const bool s_next = j + 1 < mine;   // Q_i K_{j+1}^T
            if (ok && act) ok = wait_all(full0 + 8u * vs, vph);
            if (ok && s_next) ok = wait_all(full0 + 8u * ks, kph);
            if (ok && act) ok = wait_all(smem_u32(&sh->p_full[ti]), static_cast<uint32_t>(j & 1));
            tc_fence_after();
            take_turn();
            if (ok && act && lead) {
              issue_pv(ti, vs, j > 0 ? 1u : 0u);
              if (s_next) {
                issue_s(ti, ks);
                mma_commit(smem_u32(&sh->s_full[ti]));
              } else {
                mma_commit(smem_u32(&sh->o_full[ti]));
              }
              mma_commit(empty0 + 8u * vs);
              if (j >= other) mma_commit(empty0 + 8u * vs);
              if (s_next) {
                mma_commit(empty0 + 8u * ks);
                if (j + 1 >= other) mma_commit(empty0 + 8u * ks);
              }
            }
            pass_turn();
            vs = ks;
            vph = kph;
            advance(vs, vph);  // V_{j+1}
          }
          if (ti == 0) take_turn();  // tile 1's last hand-off
          // All MMAs issued by this warp must finish before TMEM is released.
          if (lead) mma_commit(smem_u32(&sh->mma_done));
          drain_bar(smem_u32(&sh->mma_done), 0);
        }
      } else if (lane == 0 && n_max > 0) {
      bool ok = wait_bar(sh, smem_u32(&sh->q_full), 0, p.status);
      tc_fence_after();

      // ring: K_0, V_0, K_1, V_1, ...  (K_j at position 2j, V_j at 2j+1)
      if (ok) ok = wait_bar(sh, full0, 0, p.status);
      if (ok) {
        tc_fence_after();
#pragma unroll
        for (int i = 0; i < QT; ++i) {
          if (n_kv[i] == 0) continue;
          issue_s(i, 0);
          mma_commit(smem_u32(&sh->s_full[i]));
        }
        mma_commit(empty0);
      }
      int vs = 0;
      uint32_t vph = 0;
      advance(vs, vph);  // V_0
      for (int j = 0; j < n_max && ok; ++j) {
        int ks = vs;
        uint32_t kph = vph;
        advance(ks, kph);  // K_{j+1}
        ok = wait_bar(sh, full0 + 8u * vs, vph, p.status);
        if (!ok) break;
        bool k_ready = false;
#pragma unroll
        for (int i = 0; i < QT; ++i) {
          if (j >= n_kv[i]) continue;
          // Every wait comes before the tile's MMAs: a wait or a branch between two MMA
          // groups idles the tensor pipe (it holds little more than the MMA in flight), so
          // P_i(j) V_j and the next Q_i K_{j+1}^T go out as one straight run.
          const bool s_next = j + 1 < n_kv[i];
          if (s_next && !k_ready) {
            ok = wait_bar(sh, full0 + 8u * ks, kph, p.status);
            if (!ok) break;
            k_ready = true;
          }
          ok = wait_bar(sh, smem_u32(&sh->p_full[i]), static_cast<uint32_t>(j & 1), p.status);
          if (!ok) break;
          tc_fence_after();
          if (s_next) {
            issue_pv(i, vs, j > 0 ? 1u : 0u);
            issue_s(i, ks);
            mma_commit(smem_u32(&sh->s_full[i]));
          } else {
            issue_pv(i, vs, j > 0 ? 1u : 0u);
            mma_commit(smem_u32(&sh->o_full[i]));
          }
        }
        if (!ok) break;
        mma_commit(empty0 + 8u * vs);
        if (k_ready) mma_commit(empty0 + 8u * ks);
        vs = ks;
        vph = kph;
        advance(vs, vph);  // V_{j+1}
      }
      // All MMAs issued by this thread must finish before TMEM is released.
      mma_commit(smem_u32(&sh->mma_done));
      drain_bar(smem_u32(&sh->mma_done), 0);
      }
    }
  }
  } else {
    if constexpr (QT == 2) setmaxnreg_inc<G::REG_HIGH>();
    // ================================================================ softmax warpgroups
    const int i = (warp - 4) >> 2;  // query tile
    const int wq = warp & 3;        // TMEM lane quarter
    const int r = wq * 32 + lane;   // row within the tile
    const int row = q0 + G::BM * i + r;
    const uint32_t lane_off = static_cast<uint32_t>(wq * 32) << 16;
    const uint32_t tS = tmem + lane_off + G::TMEM_S + i * BN;
    const uint32_t tO = tmem + lane_off + G::TMEM_O + i * D;
    const float sl2 = p.scale_log2;
    const bool use_max = sl2 >= 0.f;
    bool ok = true;
    float m_used = -INFINITY;  // exponent base, log2 units
    float l = 0.f;
    const int nk = (QT == 1 || i == 0) ? n_kv[0] : n_kv[QT - 1];

    for (int j = 0; j < nk; ++j) {
      ok = wait_bar(sh, smem_u32(&sh->s_full[i]), static_cast<uint32_t>(j & 1), p.status);
      ok = __all_sync(0xffffffffu, ok);
      if (!ok) break;
      tc_fence_after();
      float s[BN];
#pragma unroll
      for (int c = 0; c < BN / 32; ++c) tmem_ld32(tS + c * 32, reinterpret_cast<uint32_t*>(s) + c * 32);
      tmem_wait_ld();

      const int kv0 = j * BN;
      const bool tail = kv0 + BN > p.seqlen;
      const bool diag = p.causal && (kv0 + BN - 1 > q0 + G::BM * i);
      int lim = BN;  // columns >= lim are masked for this row
      if (tail || diag) {
        lim = p.seqlen - kv0;
        if (p.causal) lim = min(lim, row - kv0 + 1);
        lim = max(0, min(lim, BN));
      }
      const bool masked = tail || diag;
      // With a positive scale a masked step runs the unmasked routines on logits whose masked
      // columns are set to -inf: 2^-inf = 0 and the row max ignores them.  (A zero scale
      // would turn -inf into NaN, a negative one flips the extreme: those keep the
      // per-element path below.)
      const bool mask_inf = masked && sl2 > 0.f;
      if (mask_inf) {
#pragma unroll
        for (int k = 0; k < BN; ++k)
          if (k >= lim) s[k] = -INFINITY;
      }
      const bool fast = use_max && (!masked || mask_inf);
      const float fill = use_max ? -INFINITY : INFINITY;

      // O_i holds the sum over steps < j (S_i(j) completion implies P_i(j-1) V_{j-1} is done),
      // so it can be rescaled here, before P_i(j) is released.  Warp-collective.
      auto rescale_o = [&](float alpha) {
#pragma unroll 1
        for (int c = 0; c < D / 32; ++c) {
          uint32_t o[32];
          tmem_ld32(tO + c * 32, o);
          tmem_wait_ld();
          const float2 a2 = make_float2(alpha, alpha);
#pragma unroll
          for (int t = 0; t < 32; t += 2) {
            const float2 v = fmul2(make_float2(__uint_as_float(o[t]), __uint_as_float(o[t + 1])), a2);
            o[t] = __float_as_uint(v.x);
            o[t + 1] = __float_as_uint(v.y);
          }
          tmem_st32(tO + c * 32, o);
        }
        if constexpr (D % 32 == 16) {
          uint32_t o[16];
          tmem_ld16(tO + (D / 32) * 32, o);
          tmem_wait_ld();
#pragma unroll
          for (int t = 0; t < 16; ++t) o[t] = __float_as_uint(__uint_as_float(o[t]) * alpha);
          tmem_st16(tO + (D / 32) * 32, o);
        }
      };

      if (fast && j > 0) {
        // Optimistic pass: exponentiate against the current base.  The row max is only needed
        // when the row sum exceeds P_SUM_BOUND (rare once the base has settled; a row whose
        // max moved past base + RESCALE_LOG2 always does): then a row that needs it takes the
        // new base, O is rescaled, and the warp recomputes P.  The decisions are those of a
        // max taken every step.
        const float base = (m_used == -INFINITY) ? 0.f : -m_used;
        float lt = exp2_row_store<PT, BN>(s, sl2, base, tS);
        if (__any_sync(0xffffffffu, !(lt <= P_SUM_BOUND) || m_used == -INFINITY)) {
          const float m_tile = row_max<BN>(s) * sl2;
          const bool need = m_tile > m_used + RESCALE_LOG2;
          if (__any_sync(0xffffffffu, need)) {
            float alpha = 1.f;
            if (need) {
              alpha = ex2_approx(m_used - m_tile);  // m_used = -inf gives 0
              l *= alpha;
              m_used = m_tile;
            }
            rescale_o(alpha);
            tmem_wait_st();  // the first pass's P stores land before they are overwritten
            lt = exp2_row_store<PT, BN>(s, sl2, -m_used, tS);
          }
        }
        l += lt;
      } else {
        // row extreme (max for scale >= 0, min for scale < 0), 8 independent chains
        float e8[8];
#pragma unroll
        for (int t = 0; t < 8; ++t) e8[t] = fill;
        if (fast) {
          e8[0] = row_max<BN>(s);
        } else if (masked) {
#pragma unroll
          for (int k = 0; k < BN; ++k) {
            const float v = (k < lim) ? s[k] : fill;
            e8[k & 7] = use_max ? fmaxf(e8[k & 7], v) : fminf(e8[k & 7], v);
          }
        } else {
#pragma unroll
          for (int k = 0; k < BN; ++k) e8[k & 7] = fminf(e8[k & 7], s[k]);
        }
        float ext = e8[0];
#pragma unroll
        for (int t = 1; t < 8; ++t) ext = use_max ? fmaxf(ext, e8[t]) : fminf(ext, e8[t]);

        const float m_tile = ext * sl2;             // NaN only when a row is fully masked and scale == 0
        const float m_new = fmaxf(m_used, m_tile);  // fmaxf drops a NaN operand
        const bool need = m_new > m_used + RESCALE_LOG2;
        float alpha = 1.f;
        if (need) {
          alpha = ex2_approx(m_used - m_new);  // m_used = -inf gives 0
          l *= alpha;
          m_used = m_new;
        }
        if (j > 0 && __any_sync(0xffffffffu, need)) rescale_o(alpha);

        // p = 2^(s*scale_log2 - m_used); masked columns -> 0
        const float neg_m = (m_used == -INFINITY) ? 0.f : -m_used;
        if (fast) {
          l += exp2_row_store<PT, BN>(s, sl2, neg_m, tS);  // also writes P
        } else {
          float l8[8];
#pragma unroll
          for (int t = 0; t < 8; ++t) l8[t] = 0.f;
#pragma unroll
          for (int k = 0; k < BN; ++k) {
            const float x = (k < lim) ? fmaf(s[k], sl2, neg_m) : -INFINITY;
            s[k] = ex2_approx(x);
            l8[k & 7] += s[k];
          }
          l += ((l8[0] + l8[1]) + (l8[2] + l8[3])) + ((l8[4] + l8[5]) + (l8[6] + l8[7]));
          // P back into TMEM (over the first P_COLS columns of S_i)
          if constexpr (Elt<T>::kTf32) {
#pragma unroll
            for (int c = 0; c < BN / 32; ++c)
              tmem_st32(tS + c * 32, reinterpret_cast<const uint32_t*>(s) + c * 32);
          } else if constexpr (VF8) {
            uint32_t pk[BN / 4];
#pragma unroll
            for (int k = 0; k < BN / 4; ++k)
              pk[k] = pack4_e5m2(s[4 * k], s[4 * k + 1], s[4 * k + 2], s[4 * k + 3]);
            if constexpr (BN / 4 >= 32) {
#pragma unroll
              for (int c = 0; c < BN / 128; ++c) tmem_st32(tS + c * 32, pk + c * 32);
            } else {
              tmem_st16(tS, pk);
            }
          } else {
            uint32_t pk[BN / 2];
#pragma unroll
            for (int k = 0; k < BN / 2; ++k)
              pk[k] = pack2(s[2 * k], s[2 * k + 1], static_cast<T*>(nullptr));
#pragma unroll
            for (int c = 0; c < BN / 64; ++c) tmem_st32(tS + c * 32, pk + c * 32);
          }
        }
      }
      tmem_wait_st();
      tc_fence_before();
      mbar_arrive(smem_u32(&sh->p_full[i]));
    }

    // ---------------------------------------------------------------- epilogue
    bool have_out = false;
    if (ok && nk > 0) {
      ok = wait_bar(sh, smem_u32(&sh->o_full[i]), 0, p.status);
      ok = __all_sync(0xffffffffu, ok);
      if (ok) {
        tc_fence_after();
        have_out = true;
        const float inv_l = 1.f / l;
        // Stage the O tile in this tile's Q buffer (every S MMA has completed).
        uint8_t* stage = q_smem + i * G::Q_TILE_BYTES;
        constexpr int CH = (D % 32 == 0) ? 32 : 16;
#pragma unroll 1
        for (int c0 = 0; c0 < D; c0 += CH) {
          uint32_t o[32];
          if constexpr (CH == 32)
            tmem_ld32(tO + c0, o);
          else
            tmem_ld16(tO + c0, o);
          tmem_wait_ld();
          // CH columns -> CH*EB bytes -> CH*EB/16 chunks of 16 bytes
          const int blk = (c0 * G::EB) / G::SWZ;
          const int inblk = (c0 * G::EB) % G::SWZ;
          uint8_t* base = stage + blk * G::Q_BLK_BYTES;
          if constexpr (Elt<T>::kTf32) {
#pragma unroll
            for (int q = 0; q < CH / 4; ++q) {
              uint4 w;
              w.x = __float_as_uint(__uint_as_float(o[4 * q + 0]) * inv_l);
              w.y = __float_as_uint(__uint_as_float(o[4 * q + 1]) * inv_l);
              w.z = __float_as_uint(__uint_as_float(o[4 * q + 2]) * inv_l);
              w.w = __float_as_uint(__uint_as_float(o[4 * q + 3]) * inv_l);
              const uint32_t off = swizzle<G::SWZ>(r * G::SWZ + inblk + q * 16);
              *reinterpret_cast<uint4*>(base + off) = w;
            }
          } else {
#pragma unroll
            for (int q = 0; q < CH / 8; ++q) {
              uint4 w;
              w.x = pack2(__uint_as_float(o[8 * q + 0]) * inv_l, __uint_as_float(o[8 * q + 1]) * inv_l, static_cast<T*>(nullptr));
              w.y = pack2(__uint_as_float(o[8 * q + 2]) * inv_l, __uint_as_float(o[8 * q + 3]) * inv_l, static_cast<T*>(nullptr));
              w.z = pack2(__uint_as_float(o[8 * q + 4]) * inv_l, __uint_as_float(o[8 * q + 5]) * inv_l, static_cast<T*>(nullptr));
              w.w = pack2(__uint_as_float(o[8 * q + 6]) * inv_l, __uint_as_float(o[8 * q + 7]) * inv_l, static_cast<T*>(nullptr));
              const uint32_t off = swizzle<G::SWZ>(r * G::SWZ + inblk + q * 16);
              *reinterpret_cast<uint4*>(base + off) = w;
            }
          }
        }
        if (row < p.seqlen) {
          const float lse = (m_used + log2f(l)) * kLn2;
          p.lse[(static_cast<int64_t>(bh) * p.seqlen) + row] = lse;
        }
        fence_proxy_async_smem();
      }
    }
    // All 128 threads of the warpgroup reach this barrier exactly once.
    named_barrier_sync(1 + i, 128);
    if (have_out && r == 0) {
      uint8_t* stage = q_smem + i * G::Q_TILE_BYTES;
#pragma unroll
      for (int c = 0; c < G::NBLK; ++c)
        tma_store_4d(&tmO, smem_u32(stage + c * G::Q_BLK_BYTES), c * G::BLK_COLS,
                     q0 + G::BM * i, hi, bi);
      bulk_commit_group();
      bulk_wait_group_read0();
    }
  }

  // ---- teardown
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, G::TMEM_ALLOC);
  }
}

}  // namespace fa
