// Persistent, warp-specialised FlashAttention forward for B200 (sm_100a): the kernel behind
// the 256-row query blocks (two 128-row tiles) of 16-bit inputs at head_dim 64 and 128.
//
// What it computes is the reference's `_attn_fwd` (flash_attention_forward.py:1036-1111):
//   O[b,h,i,:] = sum_j softmax_j(scale * q_i . k_j) v_j   (keys j <= i when causal)
//   LSE[b,h,i] = log sum_j exp(scale * q_i . k_j)
// with the reference's persistent driver -- each program loops over tiles
// `for tile in range(pid, total_tiles, num_programs)` (:1071-1076), grid = PERSISTENT_PROGRAMS
// (:616-623, :1125-1127) -- and the reference's tile orders (non-causal: the query blocks of
// one head adjacent; causal: longest query blocks first, :915-922).
//
// Roles (16 warps, one CTA per SM):
//   warps 0-3   softmax, query tile 0   (thread r owns row r = TMEM lane r)
//   warps 4-7   softmax, query tile 1
//   warps 8-11  correction: rescales O_i in TMEM when a row's exponent base moves, and writes
//               the output tile (O / l -> shared memory -> TMA store)
//   warp 12     TMEM allocator; tcgen05.mma issuer of query tile 0 (lane 0)
//   warp 13     TMA producer (Q tiles, then the K/V ring)
//   warp 14     tcgen05.mma issuer of query tile 1 (the two issuers take turns)
//   warp 15     idle (it completes the fourth warpgroup for the register split)
//
// TMEM: S_i (fp32 logits, 128 columns) at 128 i; P_i (16-bit probabilities) over the first 64
// columns of S_i; O_i (fp32, D columns) at 256 + D i.
//
// One KV step j, per tile i, issued by tile i's MMA warp in its turn, once P_i(j) is in TMEM
// and the correction warps have rescaled O_i:
//   O_i (+)= P_i V_j ;  S_i = Q_i K_{j+1}^T  (commit: S_i full)
// The softmax warpgroup of tile i, per step: load S_i (the upper half still loading while the
// lower half is exponentiated), exponentiate against the row's exponent base (ex2.approx,
// packed f32x2 arithmetic) with the row sum in the same pass, store P_i over S_i as packed
// 16-bit pairs and release it.  The base moves only when the row max passes it by more than 8
// in log2 units, so O and l rarely need rescaling; the max is taken only when the row sum
// shows it may have moved (see the softmax), and a move hands the per-row rescale factor to
// the correction warps, which rescale O_i in TMEM before the next P V.
//
// Every wait is bounded (FA_WAIT_TIMEOUT_NS); a wait that gives up records
// FA_ERR_DEVICE_TIMEOUT in the status word and raises the CTA's abort flag, after which every
// role leaves its loop and drains what it has in flight (FA_DRAIN_TIMEOUT_NS) before TMEM is
// freed.  The unbounded synchronisations are the final __syncthreads, which every thread
// reaches exactly once, and the two issuers' turn-taking named barriers, which both pass the
// same number of times on every path (a wait that gives up only stops the issuing).
#pragma once

#include <type_traits>

#include "fa_fwd_kernel.cuh"

namespace fa {

struct WsParams {
  int batch;
  int heads;
  int seqlen;
  int n_qblocks;    // ceil(seqlen / 256)
  int total_tiles;  // n_qblocks * batch * heads
  int causal;
  int stages;       // K/V ring depth
  float scale_log2; // > 0 (the host routes other scales to the one-CTA-per-tile kernel)
  float* lse;
  int* status;
};

// Element pairs (of the 16 in each 32-key chunk) that take the FMA-pipe exp2 in chunks 1 and
// 2; chunk 0 and the last chunk use ex2.approx only.  6 -> 12 of 64 pairs (18.75 %).
#ifndef FA_WS_EMU_PAIRS
#define FA_WS_EMU_PAIRS 0
#endif
// 1: after its first base move past the first key block, a softmax warp takes the row max
// first for the rest of the tile (see the softmax); 0: optimistic throughout.
#ifndef FA_WS_ADAPTIVE
#define FA_WS_ADAPTIVE 1
#endif

template <typename T, int D>
struct WsGeo {
  static_assert(D == 64 || D == 128, "persistent kernel: head_dim 64 or 128");
  static constexpr int BN = 128;                  // keys per step
  static constexpr int BM = 128;                  // rows per query tile
  static constexpr int ROW_BYTES = D * 2;
  static constexpr int SWZ = 128;                 // 128-byte swizzle spans
  static constexpr int BLK_COLS = 64;             // elements per span
  static constexpr int NBLK = ROW_BYTES / SWZ;    // spans per row (1 or 2)
  static constexpr int Q_BLK_BYTES = BM * SWZ;    // 16 KiB
  static constexpr int Q_TILE_BYTES = BM * ROW_BYTES;
  static constexpr int KV_BLK_BYTES = BN * SWZ;
  static constexpr int KV_TILE_BYTES = BN * ROW_BYTES;
  // Output: 128 x 32 boxes (64-byte rows, 64-byte swizzle), double-buffered in shared memory
  // so one box's TMA store drains while the next one is written.
  static constexpr int O_BOX_COLS = 32;
  static constexpr int O_SWZ = 64;
  static constexpr int STAGE_BYTES = BM * O_SWZ;  // 8 KiB
  static constexpr int N_OSTAGE = 2;
  static constexpr int QK_MMAS = NBLK * (SWZ / 32);  // K = 16 elements = 32 bytes per MMA
  static constexpr int PV_MMAS = BN / 16;
  static constexpr int TMEM_S = 0;
  static constexpr int TMEM_O = 2 * BN;
  static constexpr int TMEM_ALLOC = 512;
  static constexpr int NUM_THREADS = 512;
  // Register split: launched at 128 per thread (65536 / 512); the two softmax warpgroups
  // take 192, the correction warpgroup 64, the producer/MMA warpgroup 64:
  // 256 * 192 + 128 * 64 + 128 * 64 = 65536 (the split with the fewest spills; 184/88/56
  // measured 3 % slower on cfg4).
#ifndef FA_WS_REG_SOFTMAX
#define FA_WS_REG_SOFTMAX 192
#define FA_WS_REG_CORR 64
#define FA_WS_REG_OTHER 64
#endif
  static constexpr int REG_SOFTMAX = FA_WS_REG_SOFTMAX;
  static constexpr int REG_CORR = FA_WS_REG_CORR;
  static constexpr int REG_OTHER = FA_WS_REG_OTHER;
  static_assert(256 * REG_SOFTMAX + 128 * REG_CORR + 128 * REG_OTHER <= NUM_THREADS * 128,
                "register split must fit the launch allocation");
  static constexpr uint32_t LAYOUT = 2u;  // SWIZZLE_128B
  static constexpr uint32_t IDESC_S = make_idesc(Elt<T>::kFmt, false, 128, BN);
  static constexpr uint32_t IDESC_O = make_idesc(Elt<T>::kFmt, true, 128, D);
};

struct WsShared {
  uint64_t q_full[2], q_empty[2];
  uint64_t kv_full[kMaxStages], kv_empty[kMaxStages];
  uint64_t s_full[2];   // MMA -> softmax: S_i(j) computed
  uint64_t p_ready[2];  // P_i(j) in TMEM and O_i rescaled -> MMA (see the softmax's release)
  uint64_t stats[2];    // softmax -> correction: acc_scale of step j >= 1 written
  uint64_t stats_free[2];  // correction -> softmax: acc_scale read, it may be overwritten
  uint64_t fin[2];      // softmax -> correction: inv_l of the tile written
  uint64_t fin_free[2]; // correction -> softmax: inv_l read, the next tile may overwrite it
  uint64_t o_full[2];   // MMA -> correction: last P.V of the tile done
  uint64_t o_empty[2];  // correction -> MMA: O_i read out, the next tile may overwrite it
  uint64_t ost_full[2]; // correction warps -> store thread: staging buffer written
  uint64_t ost_free[2]; // store thread -> correction warps: staging buffer read by TMA
  uint64_t mma_done;
  uint32_t tmem_base;
  volatile uint32_t abort_flag;
  float acc_scale[2][128];
  float inv_l[2][128];
};

template <int D>
constexpr int ws_smem_bytes(int stages) {
  using G = WsGeo<__nv_bfloat16, D>;
  return 1024 + 2 * G::Q_TILE_BYTES + stages * G::KV_TILE_BYTES +
         G::N_OSTAGE * G::STAGE_BYTES + static_cast<int>(sizeof(WsShared));
}

// Tile coordinates shared by every role: query block, (batch, head), KV steps per query tile.
struct WsTile {
  int qblk, bh, bi, hi, q0;
  int n[2];
  int n_max;
};

__device__ __forceinline__ WsTile ws_tile(const WsParams& p, int t) {
  WsTile w;
  const int bh_count = p.batch * p.heads;
  if (p.causal) {
    w.qblk = p.n_qblocks - 1 - t / bh_count;
    w.bh = t % bh_count;
  } else {
    w.bh = t / p.n_qblocks;
    w.qblk = t % p.n_qblocks;
  }
  w.bi = w.bh / p.heads;
  w.hi = w.bh % p.heads;
  w.q0 = w.qblk * 256;
  w.n_max = 0;
#pragma unroll
  for (int i = 0; i < 2; ++i) {
    const int row0 = w.q0 + 128 * i;
    if (row0 >= p.seqlen) {
      w.n[i] = 0;
    } else {
      const int kv_end = p.causal ? min(p.seqlen, row0 + 128) : p.seqlen;
      w.n[i] = (kv_end + 127) / 128;
    }
    w.n_max = max(w.n_max, w.n[i]);
  }
  return w;
}

// Bounded wait of one thread, and the warp-collective form (every lane polls, the warp agrees
// on the outcome).
__device__ __forceinline__ bool ws_wait1(WsShared* sh, uint32_t bar, uint32_t parity, int* status) {
  return wait_bar_flag(&sh->abort_flag, bar, parity, status);
}
__device__ __forceinline__ bool ws_wait(WsShared* sh, uint32_t bar, uint32_t parity, int* status) {
  return __all_sync(0xffffffffu, ws_wait1(sh, bar, parity, status));
}


template <typename T, int D>
__global__ void __launch_bounds__(512, 1)
    fa_fwd_ws_kernel(const __grid_constant__ CUtensorMap tmQ,
                     const __grid_constant__ CUtensorMap tmK,
                     const __grid_constant__ CUtensorMap tmV,
                     const __grid_constant__ CUtensorMap tmO, const WsParams p) {
  using G = WsGeo<T, D>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  uint8_t* q_smem = smem;                                   // 2 query tiles
  uint8_t* kv_smem = q_smem + 2 * G::Q_TILE_BYTES;          // K/V ring
  uint8_t* o_stage = kv_smem + p.stages * G::KV_TILE_BYTES;  // output staging
  WsShared* sh = reinterpret_cast<WsShared*>(o_stage + G::N_OSTAGE * G::STAGE_BYTES);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int stages = p.stages;

  if (threadIdx.x == 0) {
    for (int s = 0; s < stages; ++s) {
      mbar_init(smem_u32(&sh->kv_full[s]), 1);
      mbar_init(smem_u32(&sh->kv_empty[s]), 2);  // one commit per MMA-issuing warp
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(smem_u32(&sh->q_full[i]), 1);
      mbar_init(smem_u32(&sh->q_empty[i]), 1);
      mbar_init(smem_u32(&sh->s_full[i]), 1);
      mbar_init(smem_u32(&sh->p_ready[i]), 8);  // 2 per lane quarter (see the softmax's release)
      mbar_init(smem_u32(&sh->stats[i]), 4);
      mbar_init(smem_u32(&sh->stats_free[i]), 4);
      mbar_init(smem_u32(&sh->fin[i]), 4);
      mbar_init(smem_u32(&sh->fin_free[i]), 4);
      mbar_init(smem_u32(&sh->o_full[i]), 1);
      mbar_init(smem_u32(&sh->o_empty[i]), 4);
      mbar_init(smem_u32(&sh->ost_full[i]), 4);
      mbar_init(smem_u32(&sh->ost_free[i]), 1);
    }
    mbar_init(smem_u32(&sh->mma_done), 2);  // one commit per MMA-issuing warp
    sh->abort_flag = 0u;
    fence_mbar_init();
  }
  if (warp == 13 && lane == 0) {
    prefetch_tmap(&tmQ);
    prefetch_tmap(&tmK);
    prefetch_tmap(&tmV);
    prefetch_tmap(&tmO);
  }
  if (warp == 12) {
    tmem_alloc(smem_u32(&sh->tmem_base), G::TMEM_ALLOC);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = sh->tmem_base;
  const int t_first = static_cast<int>(blockIdx.x);
  const int t_step = static_cast<int>(gridDim.x);

  if (warp >= 12) {
    setmaxnreg_dec<G::REG_OTHER>();
    if (warp == 13) {
      // ============================================================ TMA producer
      if (lane == 0) {
        uint32_t qe_ph[2] = {0u, 0u};
        int slot = 0;
        uint32_t ph = 0;
        int issued = 0;       // K/V loads issued
        bool q_pending[2] = {false, false};
        uint32_t q_par[2] = {0u, 0u};  // parity of the last Q load's q_full phase
        bool ok = true;
        for (int t = t_first; t < p.total_tiles && ok; t += t_step) {
          const WsTile w = ws_tile(p, t);
#pragma unroll
          for (int i = 0; i < 2; ++i) {
            if (w.n[i] == 0 || !ok) continue;
            // the previous tile's last Q_i K^T has completed
            if (!ws_wait1(sh, smem_u32(&sh->q_empty[i]), qe_ph[i] ^ 1u, p.status)) {
              ok = false;
              break;
            }
            qe_ph[i] ^= 1u;
            const uint32_t qb = smem_u32(&sh->q_full[i]);
            mbar_arrive_expect_tx(qb, G::Q_TILE_BYTES);
#pragma unroll
            for (int c = 0; c < G::NBLK; ++c)
              tma_load_4d(smem_u32(q_smem + i * G::Q_TILE_BYTES + c * G::Q_BLK_BYTES), &tmQ, qb,
                          c * G::BLK_COLS, w.q0 + 128 * i, w.hi, w.bi);
            q_par[i] = q_pending[i] ? q_par[i] ^ 1u : 0u;
            q_pending[i] = true;
          }
          for (int j = 0; j < w.n_max && ok; ++j) {
#pragma unroll
            for (int kv = 0; kv < 2; ++kv) {
              if (!ws_wait1(sh, smem_u32(&sh->kv_empty[slot]), ph ^ 1u, p.status)) {
                ok = false;
                break;
              }
              const uint32_t fb = smem_u32(&sh->kv_full[slot]);
              uint8_t* dst = kv_smem + slot * G::KV_TILE_BYTES;
              mbar_arrive_expect_tx(fb, G::KV_TILE_BYTES);
#pragma unroll
              for (int c = 0; c < G::NBLK; ++c)
                tma_load_4d(smem_u32(dst + c * G::KV_BLK_BYTES), kv == 0 ? &tmK : &tmV, fb,
                            c * G::BLK_COLS, j * G::BN, w.hi, w.bi);
              ++issued;
              if (++slot == stages) {
                slot = 0;
                ph ^= 1u;
              }
            }
          }
        }
        // Drain, on every path (another role may stop after the last load was issued): the
        // loads this thread issued land before shared memory goes away -- the last Q load of
        // each tile slot and the last `stages` K/V loads (older ones landed before their slots
        // were refilled).  Without an abort these phases have completed already.
#pragma unroll
        for (int i = 0; i < 2; ++i)
          if (q_pending[i]) drain_bar(smem_u32(&sh->q_full[i]), q_par[i]);
        const int outstanding = min(issued, stages);
        for (int u = 0; u < outstanding; ++u) {
          const int idx = issued - 1 - u;
          drain_bar(smem_u32(&sh->kv_full[idx % stages]),
                    static_cast<uint32_t>((idx / stages) & 1));
        }
      }
    } else if (warp == 12 || warp == 14) {
      // ============================================================ MMA issuers
      // Warp 12 issues query tile 0's MMAs, warp 14 tile 1's, taking turns through two named
      // barriers: per tile, S_0(0), S_1(0); then per KV step j, tile 0's P V_j (+ Q K_{j+1}^T)
      // and tile 1's.  The tensor pipe sees one issuer's order, while each warp waits for its
      // own operands (V_j, K_{j+1}, P_i(j), O_i) during the other warp's MMAs -- a satisfied
      // mbarrier wait still costs a few hundred cycles, and the pipe holds little more than the
      // MMA in flight.  Turn passing: barrier kTok0 (tile 0 done -> tile 1 may issue), kTok1
      // (the reverse); bar.arrive by the passer, bar.sync by the taker.  Both warps walk the
      // same tiles and steps and make a hand-off on every turn whatever happens (a wait that
      // gives up only stops the issuing), so neither is left in bar.sync.
      // Shared-memory descriptors as low words (start address >> 4 | leading offset >> 4 << 16)
      // plus one high word: stride 1024 B (8 rows of 128 B), version 1, 128-byte swizzle.  The
      // start-address field never carries (shared memory < 256 KiB), so offsets add to the low
      // word.  Q and K are K-major (leading offset unused), V is MN-major with its two 64-column
      // spans KV_BLK_BYTES apart.
      // A K/V slot's empty barrier counts two arrivals, one commit per issuer per use: each
      // commit follows every MMA its warp issued on the slot, so the slot is refilled only
      // after both tiles' MMAs on it have completed.
      constexpr uint32_t kTok0 = 1, kTok1 = 2;
      const int ti = warp == 12 ? 0 : 1;
      constexpr uint32_t kHi = (1024u >> 4) | (1u << 14) | (G::LAYOUT << 29);
      const uint32_t q_lo = (smem_u32(q_smem + ti * G::Q_TILE_BYTES) >> 4) | (1u << 16);
      const uint32_t k_lo = (smem_u32(kv_smem) >> 4) | (1u << 16);
      const uint32_t v_lo = (smem_u32(kv_smem) >> 4) | (static_cast<uint32_t>(G::KV_BLK_BYTES >> 4) << 16);
      const uint32_t hi = kHi;
      constexpr uint32_t kSlotStep = G::KV_TILE_BYTES >> 4;
      const uint32_t full0 = smem_u32(&sh->kv_full[0]);
      const uint32_t empty0 = smem_u32(&sh->kv_empty[0]);
      const uint32_t s_bar = smem_u32(&sh->s_full[ti]);
      const uint32_t pr_bar = smem_u32(&sh->p_ready[ti]);
      const uint32_t oe_bar = smem_u32(&sh->o_empty[ti]);
      const uint32_t qe_bar = smem_u32(&sh->q_empty[ti]);
      const uint32_t dS = tmem + G::TMEM_S + ti * G::BN;
      const uint32_t dO = tmem + G::TMEM_O + ti * D;
      const bool lead = lane == 0;

      auto issue_s = [&](int kslot) {
        const uint32_t b0 = k_lo + static_cast<uint32_t>(kslot) * kSlotStep;
#pragma unroll
        for (int c = 0; c < G::NBLK; ++c) {
#pragma unroll
          for (int kk = 0; kk < G::SWZ / 32; ++kk)
            mma_f16_ss_lo(dS, q_lo + ((c * G::Q_BLK_BYTES + kk * 32) >> 4),
                          b0 + ((c * G::KV_BLK_BYTES + kk * 32) >> 4), hi, G::IDESC_S,
                          (c | kk) ? 1u : 0u);
        }
      };
      // O (+)= P V for the key groups [k0, k1) of 16 keys
      auto issue_pv = [&](int vslot, int k0, int k1, uint32_t acc_first) {
        const uint32_t b0 = v_lo + static_cast<uint32_t>(vslot) * kSlotStep;
#pragma unroll
        for (int kk = k0; kk < k1; ++kk)
          mma_f16_ts_lo(dO, dS + kk * 8, b0 + ((kk * 16 * G::SWZ) >> 4), hi, G::IDESC_O,
                        kk > 0 ? 1u : acc_first);
      };
      auto pass_turn = [&]() {
        __syncwarp();
        named_barrier_arrive(ti == 0 ? kTok0 : kTok1, 64);
      };
      auto take_turn = [&]() {
        __syncwarp();
        named_barrier_sync(ti == 0 ? kTok1 : kTok0, 64);
      };

      // phase bits of this tile's barriers: q_full (0), p_ready (1), o_empty (3)
      uint32_t phs = 0;
      int slot = 0;
      uint32_t ph = 0;
      bool ok = true;
      bool first_turn = true;  // tile 0's very first turn is the only one without a take
      for (int t = t_first; t < p.total_tiles; t += t_step) {
        const WsTile w = ws_tile(p, t);
        const int mine = ti == 0 ? w.n[0] : w.n[1];
        // ---- turn: S(0) = Q K_0^T
        const int k0slot = slot;
        if (ok) ok = ws_wait(sh, full0 + 8u * slot, ph, p.status);
        if (++slot == stages) { slot = 0; ph ^= 1u; }
        if (ok && mine > 0) {
          ok = ws_wait(sh, smem_u32(&sh->q_full[ti]), phs & 1u, p.status);
          phs ^= 1u;
        }
        tc_fence_after();
        if (ti == 1 || !first_turn) take_turn();
        first_turn = false;
        if (ok && lead) {
          if (mine > 0) {
            issue_s(k0slot);
            mma_commit(s_bar);
            if (mine == 1) mma_commit(qe_bar);
          }
          mma_commit(empty0 + 8u * k0slot);
        }
        pass_turn();
        for (int j = 0; j < w.n_max; ++j) {
          // ---- turn: P V_j (+ Q K_{j+1}^T); ring order K_0, V_0, K_1, V_1, ...
          const bool act = j < mine;
          const bool s_next = j + 1 < mine;
          const int vslot = slot;
          const uint32_t vph = ph;
          if (++slot == stages) { slot = 0; ph ^= 1u; }
          const bool k_next = j + 1 < w.n_max;
          const int kslot = slot;
          const uint32_t kph = ph;
          if (k_next && ++slot == stages) { slot = 0; ph ^= 1u; }
          if (ok && act) ok = ws_wait(sh, full0 + 8u * vslot, vph, p.status);
          if (ok && s_next) ok = ws_wait(sh, full0 + 8u * kslot, kph, p.status);
          if (ok && act) {
            ok = ws_wait(sh, pr_bar, (phs >> 1) & 1u, p.status);
            phs ^= 2u;
          }
          if (ok && act && j == 0) {
            // the previous tile's output has been read out of O
            ok = ws_wait(sh, oe_bar, ((phs >> 3) & 1u) ^ 1u, p.status);
            phs ^= 8u;
          }
          tc_fence_after();
          take_turn();
          if (ok && lead) {
            if (act) {
              issue_pv(vslot, 0, G::PV_MMAS, j > 0 ? 1u : 0u);
              if (s_next) {
                issue_s(kslot);
                mma_commit(s_bar);
                if (j + 2 == mine) mma_commit(qe_bar);
              } else {
                mma_commit(smem_u32(&sh->o_full[ti]));
              }
            }
            mma_commit(empty0 + 8u * vslot);
            if (k_next) mma_commit(empty0 + 8u * kslot);
          }
          pass_turn();
        }
      }
      if (ti == 0) take_turn();  // tile 1's last hand-off
      // every MMA this warp issued completes before TMEM is released
      if (lead) mma_commit(smem_u32(&sh->mma_done));
      __syncwarp();
      drain_bar(smem_u32(&sh->mma_done), 0);
    }
  } else if (warp >= 8) {
    setmaxnreg_dec<G::REG_CORR>();
    // ================================================================ correction
    const int wq = warp & 3;
    const int r = wq * 32 + lane;
    const uint32_t lane_off = static_cast<uint32_t>(wq * 32) << 16;
    const bool store_thread = warp == 8 && lane == 0;
    // phase bits: stats (bit i), o_full (2 + i), fin (4 + i), staging free (6 + b, waited
    // producer-style), staging written (8 + b, store thread)
    uint32_t phs = 0;
    int ostage = 0;
    bool ok = true;
    bool stores_issued = false;

    for (int t = t_first; t < p.total_tiles && ok; t += t_step) {
      const WsTile w = ws_tile(p, t);
      // Steps j >= 1: the softmax warp of this lane quarter hands over each row's rescale
      // factor (1 when its exponent base stayed).  When one of the warp's 32 rows moved, the
      // softmax released P_i(j) with one arrival and this warp adds the second once O_i is
      // rescaled; otherwise the softmax's release already counted for both.
      for (int j = 1; j < w.n_max && ok; ++j) {
#pragma unroll
        for (int i = 0; i < 2; ++i) {
          if (j >= w.n[i] || !ok) continue;
          ok = ws_wait(sh, smem_u32(&sh->stats[i]), (phs >> i) & 1u, p.status);
          if (!ok) break;
          phs ^= 1u << i;
          const float a = sh->acc_scale[i][r];
          __syncwarp();
          if (lane == 0) mbar_arrive(smem_u32(&sh->stats_free[i]));
          if (__any_sync(0xffffffffu, a < 1.f)) {
            // O_i holds P V summed over steps < j (S_i(j) is complete, and the MMAs of one
            // thread complete in order) and P_i(j) V_j waits for this warp: rescale its rows
            tc_fence_after();
            const uint32_t tO = tmem + lane_off + G::TMEM_O + i * D;
#pragma unroll 1
            for (int c = 0; c < D / 32; ++c) {
              uint32_t o[32];
              tmem_ld32(tO + c * 32, o);
              tmem_wait_ld();
#pragma unroll
              for (int u = 0; u < 32; u += 2) {
                const float2 v = fmul2(make_float2(__uint_as_float(o[u]), __uint_as_float(o[u + 1])),
                                       make_float2(a, a));
                o[u] = __float_as_uint(v.x);
                o[u + 1] = __float_as_uint(v.y);
              }
              tmem_st32(tO + c * 32, o);
            }
            tmem_wait_st();
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(smem_u32(&sh->p_ready[i]));
          }
        }
      }
      if (!ok) break;
      // ---- epilogue: O_i / l -> 16-bit -> staging (128 x 32 boxes) -> TMA store
#pragma unroll 1
      for (int i = 0; i < 2; ++i) {
        if ((i == 0 ? w.n[0] : w.n[1]) == 0 || !ok) continue;
        ok = ws_wait(sh, smem_u32(&sh->o_full[i]), (phs >> (2 + i)) & 1u, p.status);
        if (ok) ok = ws_wait(sh, smem_u32(&sh->fin[i]), (phs >> (4 + i)) & 1u, p.status);
        if (!ok) break;
        phs ^= (1u << (2 + i)) | (1u << (4 + i));
        tc_fence_after();
        const float inv = sh->inv_l[i][r];
        __syncwarp();
        if (lane == 0) mbar_arrive(smem_u32(&sh->fin_free[i]));
        const uint32_t tO = tmem + lane_off + G::TMEM_O + i * D;
#pragma unroll 1
        for (int q = 0; q < D / G::O_BOX_COLS; ++q) {
          uint32_t pk[16];
          {
            uint32_t o[32];
            tmem_ld32(tO + q * 32, o);
            tmem_wait_ld();
#pragma unroll
            for (int u = 0; u < 16; ++u)
              pk[u] = pack2(__uint_as_float(o[2 * u]) * inv, __uint_as_float(o[2 * u + 1]) * inv,
                            static_cast<T*>(nullptr));
          }
          if (q == D / G::O_BOX_COLS - 1) {
            // O_i is read out: the next tile's first P V may overwrite it
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(smem_u32(&sh->o_empty[i]));
          }
          // wait until this staging buffer's previous store has been read
          ok = ws_wait(sh, smem_u32(&sh->ost_free[ostage]), ((phs >> (6 + ostage)) & 1u) ^ 1u,
                       p.status);
          if (!ok) break;
          phs ^= 1u << (6 + ostage);
          uint8_t* stg = o_stage + ostage * G::STAGE_BYTES;
#pragma unroll
          for (int c = 0; c < 4; ++c)
            *reinterpret_cast<uint4*>(stg + swizzle<G::O_SWZ>(r * G::O_SWZ + c * 16)) =
                make_uint4(pk[4 * c], pk[4 * c + 1], pk[4 * c + 2], pk[4 * c + 3]);
          fence_proxy_async_smem();
          __syncwarp();
          if (lane == 0) mbar_arrive(smem_u32(&sh->ost_full[ostage]));
          if (store_thread) {
            // all four warps have written the box: store it; once the previous box's store
            // has been read, that buffer is free again
            if (!ws_wait1(sh, smem_u32(&sh->ost_full[ostage]), (phs >> (8 + ostage)) & 1u,
                          p.status)) {
              ok = false;
            } else {
              tma_store_4d(&tmO, smem_u32(stg), q * G::O_BOX_COLS, w.q0 + 128 * i, w.hi, w.bi);
              bulk_commit_group();
              bulk_wait_group_read1();
              if (stores_issued) mbar_arrive(smem_u32(&sh->ost_free[ostage ^ 1]));
              stores_issued = true;
            }
            phs ^= 1u << (8 + ostage);
          }
          ok = __shfl_sync(0xffffffffu, ok ? 1 : 0, 0) != 0 && ok;
          if (!ok) break;
          ostage ^= 1;
        }
      }
    }
    if (store_thread && stores_issued) bulk_wait_group_read0();
  } else {
    setmaxnreg_inc<G::REG_SOFTMAX>();
    // ================================================================ softmax warpgroups
    const int i = warp >> 2;   // query tile
    const int wq = warp & 3;   // TMEM lane quarter
    const int r = wq * 32 + lane;
    const uint32_t lane_off = static_cast<uint32_t>(wq * 32) << 16;
    const uint32_t tS = tmem + lane_off + G::TMEM_S + i * G::BN;
    const uint32_t pr_bar = smem_u32(&sh->p_ready[i]);
    const float sl2 = p.scale_log2;
    const float2 sc = make_float2(sl2, sl2);
    uint32_t sf_ph = 0;  // s_full
    uint32_t xf_ph = 0;  // stats_free (producer-style)
    uint32_t ff_ph = 0;  // fin_free (producer-style)
    bool ok = true;

    // p = 2^(s * scale_log2 - m) for the row, P to TMEM in four 32-key chunks; returns the
    // sum of the fp32 p.  s is left intact.
    // With `upper_in_flight`, the upper 64 logits are still being loaded from TMEM (see
    // load_s_lower) and are waited for once the lower half has been exponentiated.
    auto exp_pass = [&](float* sv, float neg_m, bool upper_in_flight = false) -> float {
      const float2 nm = make_float2(neg_m, neg_m);
      float2 acc4[4];
#pragma unroll
      for (int u = 0; u < 4; ++u) acc4[u] = make_float2(0.f, 0.f);
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        if (c == 2 && upper_in_flight) {
          tmem_wait_ld();
          // the registers the asynchronous load wrote are read only after the wait
#pragma unroll
          for (int k = 64; k < 128; ++k) asm volatile("" : "+f"(sv[k]));
        }
        uint32_t pk[16];
#pragma unroll
        for (int u = 0; u < 16; ++u) {
          const int k = c * 32 + 2 * u;
          const float2 x = ffma2(make_float2(sv[k], sv[k + 1]), sc, nm);
          float2 pr;
          if (c >= 1 && c <= 2 && u >= 16 - FA_WS_EMU_PAIRS) {
            pr = exp2_poly2_deg3(x);
          } else {
            pr.x = ex2_approx(x.x);
            pr.y = ex2_approx(x.y);
          }
          acc4[u & 3] = fadd2(acc4[u & 3], pr);
          pk[u] = pack2(pr.x, pr.y, static_cast<T*>(nullptr));
        }
        tmem_st16(tS + c * 16, pk);
      }
      const float2 a2 = fadd2(fadd2(acc4[0], acc4[1]), fadd2(acc4[2], acc4[3]));
      return a2.x + a2.y;
    };
    // Hands P_i(j) to the MMA warp: `count` arrivals of this warp on p_ready (2 = this lane
    // quarter is complete; 1 = its correction warp adds the second after rescaling O).
    auto release = [&](uint32_t count) {
      tmem_wait_st();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive_cnt(pr_bar, count);
    };
    // Hands this step's per-row rescale factors to the correction warp (once it has read the
    // previous step's).
    // Every step after the first hands its per-row rescale factors to the correction warp
    // exactly once (1 for a row whose base stayed).  The wait for the slot (the correction warp
    // has read the previous step's factors) is taken at the top of the step, while S is still
    // being computed, so giving the factors costs only the store and the arrival.
    auto stats_slot = [&]() {
      if (!ws_wait(sh, smem_u32(&sh->stats_free[i]), xf_ph ^ 1u, p.status)) return false;
      xf_ph ^= 1u;
      return true;
    };
    auto give_stats = [&](float acc) {
      sh->acc_scale[i][r] = acc;
      __syncwarp();
      if (lane == 0) mbar_arrive(smem_u32(&sh->stats[i]));
    };

    for (int t = t_first; t < p.total_tiles && ok; t += t_step) {
      const WsTile w = ws_tile(p, t);
      const int nk = w.n[i];
      if (nk == 0) continue;
      const int row = w.q0 + 128 * i + r;
      float m = -INFINITY;  // exponent base, log2 units
      float l = 0.f;
      float s[128];
      // S_i(j) into registers, keys past the sequence end / above the diagonal at -inf
      auto load_s = [&](int j) -> bool {
        if (!ws_wait(sh, smem_u32(&sh->s_full[i]), sf_ph, p.status)) return false;
        sf_ph ^= 1u;
        tc_fence_after();
#pragma unroll
        for (int c = 0; c < 4; ++c) tmem_ld32(tS + c * 32, reinterpret_cast<uint32_t*>(s) + c * 32);
        tmem_wait_ld();
        const int kv0 = j * 128;
        const bool tail = kv0 + 128 > p.seqlen;
        const bool diag = p.causal && (kv0 + 127 > w.q0 + 128 * i);
        if (tail || diag) {
          int lim = p.seqlen - kv0;
          if (p.causal) lim = min(lim, row - kv0 + 1);
#pragma unroll
          for (int k = 0; k < 128; ++k)
            if (k >= lim) s[k] = -INFINITY;
        }
        return true;
      };
      // S_i(j) for the optimistic pass: on an unmasked step only the lower 64 logits are
      // waited for, the upper 64 load while the lower half is exponentiated (true); a masked
      // step (causal diagonal, sequence tail) loads and masks the whole row (false).  Sets
      // `ok` to false on a timeout.
      auto load_s_lower = [&](int j) -> bool {
        const int kv0 = j * 128;
        const bool tail = kv0 + 128 > p.seqlen;
        const bool diag = p.causal && (kv0 + 127 > w.q0 + 128 * i);
        if (tail || diag) {
          ok = load_s(j);
          return false;
        }
        ok = ws_wait(sh, smem_u32(&sh->s_full[i]), sf_ph, p.status);
        if (!ok) return false;
        sf_ph ^= 1u;
        tc_fence_after();
        tmem_ld32(tS, reinterpret_cast<uint32_t*>(s));
        tmem_ld32(tS + 32, reinterpret_cast<uint32_t*>(s) + 32);
        tmem_wait_ld();
#pragma unroll
        for (int k = 0; k < 64; ++k) asm volatile("" : "+f"(s[k]));
        tmem_ld32(tS + 64, reinterpret_cast<uint32_t*>(s) + 64);
        tmem_ld32(tS + 96, reinterpret_cast<uint32_t*>(s) + 96);
        return true;
      };
      // ---- first key block: the exponent base is the row max (O starts from zero, so nothing
      // is rescaled and the correction warps are not involved)
      ok = load_s(0);
      if (!ok) break;
      m = row_max<128>(s) * sl2;
      l = exp_pass(s, m == -INFINITY ? 0.f : -m);
      release(2u);
      // ---- later blocks, optimistic: exponentiate against the current base with the row sum
      // in the same pass.  Every p <= 2^RESCALE_LOG2 whenever the row's sum is; only a row
      // whose sum exceeds P_SUM_BOUND (always one whose max moved past base + RESCALE_LOG2,
      // rarely any other once the base has settled) takes the row max, and a warp with a row
      // that needs the new base recomputes P.  A warp whose rows all keep their base releases
      // P on its own; otherwise its correction warp rescales O and adds the second arrival.
      // The first base move after the first block ends this loop for the tile: rows whose max
      // keeps moving (outlier-heavy inputs) would otherwise pay a second exponent pass per
      // move, so the rest of the tile takes the max first.
      int j = 1;
      for (; j < nk; ++j) {
        ok = stats_slot();
        if (!ok) break;
        const bool upper_in_flight = load_s_lower(j);
        if (!ok) break;
        float sum = exp_pass(s, m == -INFINITY ? 0.f : -m, upper_in_flight);
        float acc = 1.f;
        bool any_need = false;
        if (__any_sync(0xffffffffu, !(sum <= P_SUM_BOUND) || m == -INFINITY)) {
          const float mx = row_max<128>(s) * sl2;
          const bool need = mx > m + RESCALE_LOG2;
          any_need = __any_sync(0xffffffffu, need);
          if (any_need) {
            if (need) {
              acc = ex2_approx(m - mx);  // m = -inf gives 0
              m = mx;
            }
            give_stats(acc);
            tmem_wait_st();  // the first pass's P stores land before they are overwritten
            sum = exp_pass(s, m == -INFINITY ? 0.f : -m);
          }
        }
        release(any_need ? 1u : 2u);
        l = l * acc + sum;
        if (!any_need) {
          give_stats(1.f);
        } else if (FA_WS_ADAPTIVE) {
          ++j;
          break;
        }
      }
      if (!ok) break;
      // ---- the rest of the tile: row max first, then the exponentials against the chosen
      // base; a base move costs the correction warp's O rescale, overlapped with this pass
      for (; j < nk; ++j) {
        ok = stats_slot();
        if (!ok) break;
        ok = load_s(j);
        if (!ok) break;
        const float mx = row_max<128>(s) * sl2;
        const bool need = mx > m + RESCALE_LOG2;
        float acc = 1.f;
        if (need) {
          acc = ex2_approx(m - mx);  // m = -inf gives 0
          m = mx;
        }
        const bool any_need = __any_sync(0xffffffffu, need);
        if (any_need) give_stats(acc);
        const float sum = exp_pass(s, m == -INFINITY ? 0.f : -m);
        release(any_need ? 1u : 2u);
        l = l * acc + sum;
        if (!any_need) give_stats(1.f);
      }
      if (!ok) break;
      // tile done: logsumexp, and 1/l for the correction warps' epilogue (once they have read
      // the previous tile's)
      if (row < p.seqlen) p.lse[static_cast<int64_t>(w.bh) * p.seqlen + row] = (m + log2f(l)) * kLn2;
      ok = ws_wait(sh, smem_u32(&sh->fin_free[i]), ff_ph ^ 1u, p.status);
      if (!ok) break;
      ff_ph ^= 1u;
      sh->inv_l[i][r] = 1.f / l;
      __syncwarp();
      if (lane == 0) mbar_arrive(smem_u32(&sh->fin[i]));
    }
  }

  // ---- teardown: every thread arrives here exactly once
  tc_fence_before();
  __syncthreads();
  if (warp == 12) {
    tc_fence_after();
    tmem_dealloc(tmem, G::TMEM_ALLOC);
  }
}

}  // namespace fa
