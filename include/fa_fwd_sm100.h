/*
 * C ABI of the B200 (sm_100a) FlashAttention forward.
 *
 * This is the native boundary behind the Python module `flash_attention_forward.py`.
 * In the reference project (ZyEng-Art/flash_attn_npu) the same boundary is the launch of the
 * Triton kernel `_attn_fwd[grid](Q, K, V, M, Out, acc, sm_scale, strides..., Z, H, N_CTX,
 * HEAD_DIM, BLOCK_M, BLOCK_N, STAGE, ...)` at flash_attention_forward.py:1159-1193, reached
 * from `_launch_kernel` (flash_attention_forward.py:1130-1194).  `fa_fwd_sm100` takes the
 * place of that launch: same tensors, same strides, same tile knobs, plus an explicit stream.
 *
 * Conventions
 *   - q, k, v, o: device pointers to [B, H, S, D] tensors of `dtype`, each with its own
 *     element strides for the B, H and S dimensions; the D dimension must be contiguous.
 *     Every pointer must be 16-byte aligned and every stride must be a multiple of
 *     16 bytes (the TMA rule); otherwise FA_ERR_MISALIGNED is returned.
 *   - lse: device pointer to a contiguous fp32 [B, H, S] array; receives the natural-log
 *     logsumexp of every query row (the reference's `M` output, flash_attention_forward.py:1031).
 *   - The caller owns every buffer; the library allocates no device memory.
 *   - The launch is asynchronous on `stream`; errors detected on the host are returned
 *     before anything is enqueued.  Device-side failures (a pipeline wait that timed out)
 *     are written to `*dev_status` when it is non-NULL (0 = success).
 *   - Reentrant: tensor maps are built per call and passed by value to the kernel.
 */
#ifndef FA_FWD_SM100_H_
#define FA_FWD_SM100_H_

#include <stdint.h>

#if defined(__GNUC__)
#define FA_API __attribute__((visibility("default")))
#else
#define FA_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

/* Element types (the reference accepts fp16 and bf16, flash_attention_forward.py:1306-1312).
 * fp32 inputs run on the CUDA cores in fp32 by default, or on the tensor cores in TF32 with
 * FA_FLAG_FP32_TF32 (faster; TF32 rounding moves the logsumexp by ~1e-3). */
enum FaDtype { FA_DTYPE_FP16 = 0, FA_DTYPE_BF16 = 1, FA_DTYPE_FP32 = 2 };

/* FaFwdArgs.flags bits.
 * FA_FLAG_V_FP8_E5M2: `v` holds float8 e5m2 values (one byte per element, strides in elements)
 * while `dtype` (fp16 or bf16, head_dim >= 32) describes q, k and o; P is rounded to e5m2 and
 * P.V runs on the fp8 tensor-core path.  Replaces the reference's fp8_v mode
 * (flash_attention_forward.py:704, :996: taken when V is float8e5). */
/* FA_FLAG_ONE_CTA_PER_TILE: run the one-CTA-per-query-block kernel even where the persistent
 * kernel would serve the call (see FaTileConfig.persistent_ctas); kept for A/B comparisons of
 * the two kernels. */
enum FaFlags { FA_FLAG_FP32_TF32 = 1, FA_FLAG_V_FP8_E5M2 = 2, FA_FLAG_ONE_CTA_PER_TILE = 4 };

/* Return codes. */
enum FaStatus {
  FA_OK = 0,
  FA_ERR_INVALID_ARG = -1,          /* null pointer, non-positive size, bad struct size */
  FA_ERR_UNSUPPORTED_HEAD_DIM = -2, /* head_dim not in {16, 32, 64, 128, 256} (flash_attention_forward.py:1121) */
  FA_ERR_UNSUPPORTED_DTYPE = -3,
  FA_ERR_MISALIGNED = -4,           /* pointer or stride violates the 16-byte TMA rule */
  FA_ERR_UNSUPPORTED_TILE = -5,     /* (block_m, block_n, stages) not available for this head_dim */
  FA_ERR_TENSOR_MAP = -6,           /* cuTensorMapEncodeTiled rejected a descriptor */
  FA_ERR_LAUNCH = -7,               /* the CUDA launch itself failed */
  FA_ERR_DEVICE = -8,               /* current device is not an sm_100 part */
  FA_ERR_DEVICE_TIMEOUT = -9        /* written to *dev_status: a pipeline wait gave up */
};

typedef struct FaTileConfig {
  int32_t block_m;         /* query rows per CTA: 128 or 256 (two 128-row tiles) */
  int32_t block_n;         /* keys per pipeline step: 64 or 128 */
  int32_t num_stages;      /* K/V shared-memory ring depth; 0 = largest that fits */
  int32_t persistent_ctas; /* grid of the persistent kernel, which runs every call it serves
                              (fp16 / bf16, head_dim 64 / 128, block 256 x 128, sm_scale > 0):
                              each CTA loops over tiles (reference PERSISTENT_PROGRAMS); 0 = one
                              CTA per SM.  Non-zero values are refused (FA_ERR_UNSUPPORTED_TILE)
                              for calls that run one CTA per tile. */
} FaTileConfig;

typedef struct FaFwdArgs {
  int32_t struct_size; /* sizeof(FaFwdArgs), checked for ABI drift */
  const void* q;
  const void* k;
  const void* v;
  void* o;
  float* lse;
  int64_t batch;    /* Z in the reference */
  int64_t heads;    /* H */
  int64_t seqlen;   /* N_CTX */
  int64_t head_dim; /* HEAD_DIM */
  int64_t q_stride[3]; /* element strides of q for (batch, head, seq) */
  int64_t k_stride[3];
  int64_t v_stride[3];
  int64_t o_stride[3];
  int32_t dtype;  /* enum FaDtype */
  int32_t causal; /* 0 / 1: query i attends keys <= i (reference STAGE=3) */
  float sm_scale; /* softmax scale applied to q.k */
  FaTileConfig tile;   /* tensor-core kernels only */
  int32_t* dev_status; /* optional device int, 0 on success */
  int32_t flags;       /* FaFlags */
} FaFwdArgs;

/* Launch the forward pass.  Returns FA_OK or a negative FaStatus.
 * Replaces: flash_attention_forward.py:1159-1193 (`_attn_fwd[grid](...)`). */
FA_API int fa_fwd_sm100(const FaFwdArgs* args, void* stream);

/* Fill `cfg` with the tile configuration the library picks when the caller gives none
 * (block_m = 0).  Replaces: `_default_tiling` (flash_attention_forward.py:221-242). */
FA_API int fa_fwd_sm100_default_tile(int64_t head_dim, int32_t dtype, int32_t causal,
                              int64_t seqlen, FaTileConfig* cfg);

/* 1 if the kernel family has an instantiation for these knobs, else 0.  Used by the tuner
 * to build its sweep (replaces the candidate filter at tune_flash_attention_forward.py:76-115). */
FA_API int fa_fwd_sm100_supported(int64_t head_dim, int32_t dtype, int32_t block_m, int32_t block_n,
                           int32_t num_stages);

/* Largest K/V ring depth that fits shared memory for these knobs (0 if unsupported). */
FA_API int fa_fwd_sm100_max_stages(int64_t head_dim, int32_t dtype, int32_t block_m, int32_t block_n);

/* Number of CTAs the launch uses for this problem (reference: `_build_grid`,
 * flash_attention_forward.py:1125-1127). */
FA_API int64_t fa_fwd_sm100_grid_size(const FaFwdArgs* args);

/* Human-readable text for a status code. */
FA_API const char* fa_fwd_sm100_status_string(int code);

/* Library version, e.g. 1000 for 0.1.0. */
FA_API int fa_fwd_sm100_version(void);

#ifdef __cplusplus
}
#endif

#endif /* FA_FWD_SM100_H_ */
