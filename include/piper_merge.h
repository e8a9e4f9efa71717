/*
 * piper_merge.h - C ABI of the B200 (sm_100a) fused quantized LoRA merge.
 *
 * One call merges  W <- requant(dequant(W) + strength * (B @ A))  in place for a
 * packed quantized weight W, recomputing its data-dependent scales, with
 * round-to-nearest or counter-based stochastic rounding. These entry points
 * replace the raw-buffer Triton launchers of Piper Offload 0.2.5:
 *
 *   piper_merge_mx       <- src/piper_offload/_triton_mx_lora.py:333      merge_mx_lora_
 *   piper_merge_nvfp4    <- src/piper_offload/_triton_nvfp4_lora.py:515   merge_nvfp4_lora
 *   piper_merge_float8   <- src/piper_offload/_triton_float8_lora.py:486  merge_float8_lora
 *   piper_merge_int8     <- src/piper_offload/_triton_int8_lora.py:267    merge_int8_lora
 *   piper_merge_gguf     <- (no reference merge; GGUF weights are routed-only in the
 *                            reference, src/piper_offload/lora.py:752-753)
 *   piper_merge_batch    <- several of the above in one launch sequence (the per-weight
 *                            loop of src/piper_offload/merge.py:124)
 *
 * All pointers are device pointers of the current CUDA device, except `descs`
 * and `stream`. `stream` is a cudaStream_t (pass torch.cuda.current_stream()).
 * Every call is asynchronous on `stream`. Buffers are updated IN PLACE: the
 * codes/scales/zero-point pointers keep their addresses (the reference copies
 * its out-of-place results back into the same storage, int8_adapter.py:397-400).
 *
 * Return value: 0 on success, otherwise a PIPER_MERGE_E* code; nothing has been
 * enqueued when an argument error is returned. piper_merge_last_error() gives
 * the message of the calling thread's last failure.
 */
#ifndef PIPER_MERGE_H
#define PIPER_MERGE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- status codes ---- */
#define PIPER_MERGE_OK 0
#define PIPER_MERGE_EINVAL 1      /* bad argument / unsupported layout (ValueError) */
#define PIPER_MERGE_ECUDA 2       /* CUDA launch or runtime failure (RuntimeError) */
#define PIPER_MERGE_EWORKSPACE 3  /* workspace too small */
#define PIPER_MERGE_ETIMEOUT 4    /* a bounded device-side wait gave up */

/* ---- formats ---- */
#define PIPER_FMT_MXFP8_E4M3 0
#define PIPER_FMT_MXFP8_E5M2 1
#define PIPER_FMT_MXFP4 2
#define PIPER_FMT_NVFP4 3
#define PIPER_FMT_FP8_E4M3 4   /* TorchAO scaled FP8, fp32 scales */
#define PIPER_FMT_FP8_E5M2 5
#define PIPER_FMT_INT8 6       /* TorchAO affine INT8 */
#define PIPER_FMT_GGUF_Q8_0 7
#define PIPER_FMT_GGUF_Q4_0 8
#define PIPER_FMT_BNB8 9             /* bitsandbytes LLM.int8: int8 CB, fp32 SCB per row */
#define PIPER_FMT_QUANTO_INT8 10     /* Quanto qint8 qbytes, scales in the compute dtype */
#define PIPER_FMT_QUANTO_FP8_E4M3 11 /* Quanto qfloat8 qbytes */
#define PIPER_FMT_QUANTO_FP8_E5M2 12
#define PIPER_FMT_BNB4_NF4 13        /* bitsandbytes 4-bit, NF4 code selection */
#define PIPER_FMT_BNB4_FP4 14        /* bitsandbytes 4-bit, FP4 code selection */

/* ---- floating dtypes (factors = compute dtype; INT8 scales) ----
 * bf16 / fp16 factors: the rank-r update runs on tcgen05 tensor cores.
 * fp32 factors: the reference's IEEE fp32 dot (one fused multiply-add per rank
 * step, in rank order; _triton_float8_lora.py:53-66) on CUDA cores. */
#define PIPER_DT_BF16 0
#define PIPER_DT_F16 1
#define PIPER_DT_F32 2

/* ---- MX E8M0 scale rounding (mx_adapter.py:55-60) ---- */
#define PIPER_MX_FLOOR 0
#define PIPER_MX_RCEIL 1
#define PIPER_MX_CEIL 2
#define PIPER_MX_EVEN 3

/* ---- flags ---- */
#define PIPER_FLAG_SWIZZLED 1u      /* MX / NVFP4 blocked 128x4 scale layout */
#define PIPER_FLAG_ASYMMETRIC 2u    /* INT8 with zero points recomputed */
#define PIPER_FLAG_REDUCE_RANGE 4u  /* INT8 codes in [-64, 63] */
#define PIPER_FLAG_STOCHASTIC 8u    /* stochastic rounding keyed by `seed` */

/*
 * One weight to merge. Logical shape rows x cols; factors b (rows x rank) and
 * a (rank x cols), contiguous, in `compute_dtype`.
 *
 * qdata   codes: MXFP8/FP8 rows x cols bytes; MXFP4/NVFP4 rows x cols/2 packed
 *         bytes (element 2j in the low nibble of byte j); INT8 rows x cols int8;
 *         GGUF rows x (cols/32)*34 (Q8_0) or (cols/32)*18 (Q4_0) raw block bytes.
 * scale   MX: E8M0 bytes, rows x cols/32 or swizzled ((rows+127)/128*32) x
 *         ((cols+127)/128*16); NVFP4: E4M3 bytes, rows x cols/16 or swizzled
 *         ((rows+127)/128*32) x ((cols+63)/64*16); FP8: fp32, one per
 *         quantization block; INT8: `scale_dtype`, one per block; BNB8: fp32
 *         SCB, one per row; Quanto: `compute_dtype`, one per tensor, row
 *         (block (1, cols)) or column (block (rows, 1)); BNB4: fp32 absmax per 64-value block, or uint8 codes of the
 *         nested quantization; GGUF: unused.
 * zero_point  INT8 only: int8 per block, or NULL (symmetric storage).
 * global_scale NVFP4 only: fp32 per-tensor scale (two-level), or NULL.
 * block_rows, block_cols  FP8/INT8 quantization block: (1, cols) per row,
 *         (rows, cols) per tensor, (1, g) per group with g | cols.
 * codebook BNB4 only: 16 fp32 code values (bitsandbytes QuantState.code).
 * nested_absmax, nested_code, nested_offset  BNB4 nested absmax only: fp32
 *         per 256 blocks (updated), 256 fp32 code values, fp32 offset (updated);
 *         NULL otherwise. The first 4-bit value of byte j is its high nibble.
 * offset_base is added to every logical element offset row*cols+col before it
 *         keys the stochastic stream (0 reproduces the reference; a row shard
 *         passes its first element's global offset to draw the unsharded stream).
 */
typedef struct piper_merge_desc {
  void* qdata;
  void* scale;
  void* zero_point;
  void* global_scale;
  const void* b;
  const void* a;
  int64_t rows;
  int64_t cols;
  int64_t rank;
  int64_t block_rows;
  int64_t block_cols;
  int32_t format;        /* PIPER_FMT_* */
  int32_t compute_dtype; /* PIPER_DT_* (factor dtype) */
  int32_t scale_dtype;   /* PIPER_DT_* (INT8 scale storage dtype) */
  int32_t scale_mode;    /* PIPER_MX_* */
  uint32_t flags;        /* PIPER_FLAG_* */
  float strength;
  uint64_t seed;
  uint64_t offset_base;
  const void* codebook;
  void* nested_absmax;
  const void* nested_code;
  void* nested_offset;
} piper_merge_desc;

/* Bytes of device workspace `piper_merge_batch` needs for these descriptors.
 * 0 means no workspace (NULL may be passed). Per-row FP8 / INT8 weights of a
 * call too small to fill the GPU with whole 128-row strips ask for 16 bytes
 * per row, which lets them split their columns over every SM; given less (or
 * NULL), the call still runs them, with the fused one-launch pass. Returns 0
 * on success. */
int piper_merge_workspace_size(const piper_merge_desc* descs, int32_t count, size_t* bytes);

/* Merge `count` weights, enqueued on `stream`. `workspace` is a device buffer of
 * at least piper_merge_workspace_size() bytes, 256-byte aligned; it is fully
 * (re)initialised by the call. Weights must not alias one another. */
int piper_merge_batch(const piper_merge_desc* descs, int32_t count, void* workspace,
                      size_t workspace_bytes, void* stream);

/* Single-weight conveniences mirroring the reference launchers' arguments. */

/* _triton_mx_lora.py:333 merge_mx_lora_(qdata, scale, elem_dtype, block_size=32,
 * orig_dtype, b, a, strength, *, scaling_mode, swizzled, rounding_seed). */
int piper_merge_mx(void* qdata, void* scale, const void* b, const void* a, int64_t rows,
                   int64_t cols, int64_t rank, int32_t elem_format, int32_t compute_dtype,
                   int32_t scaling_mode, int32_t swizzled, float strength, int32_t has_seed,
                   uint64_t seed, uint64_t offset_base, void* stream);

/* _triton_nvfp4_lora.py:515 merge_nvfp4_lora(qdata, scale, per_tensor_scale, 16,
 * is_swizzled_scales, b, a, strength, *, rounding_seed). `workspace` >= 256 bytes
 * when global_scale != NULL (two-level), else may be NULL. */
int piper_merge_nvfp4(void* qdata, void* scale, void* global_scale, const void* b,
                      const void* a, int64_t rows, int64_t cols, int64_t rank,
                      int32_t compute_dtype, int32_t swizzled, float strength, int32_t has_seed,
                      uint64_t seed, uint64_t offset_base, void* workspace,
                      size_t workspace_bytes, void* stream);

/* _triton_float8_lora.py:486 merge_float8_lora(qdata, scale, block_size, b, a,
 * strength, *, rounding_seed). */
int piper_merge_float8(void* qdata, void* scale, const void* b, const void* a, int64_t rows,
                       int64_t cols, int64_t rank, int64_t block_rows, int64_t block_cols,
                       int32_t e5m2, int32_t compute_dtype, float strength, int32_t has_seed,
                       uint64_t seed, uint64_t offset_base, void* workspace,
                       size_t workspace_bytes, void* stream);

/* piper_merge_float8 without a workspace argument. No counterpart in the
 * reference: an addition for callers that cannot allocate device memory at
 * merge time. Per-tensor scales, groups wider than one tile (more than 256
 * columns) and per-row weights too small to fill the GPU with whole 128-row
 * strips (fewer than two strips per SM) keep 16 bytes per quantization block
 * in a fixed 1 MiB array in device memory (one per device and CUDA context);
 * larger per-row weights need none. Layouts needing more than 65,536 blocks (e.g. 512-column
 * groups over rows x cols/512 > 65,536) are rejected with
 * PIPER_MERGE_EWORKSPACE before anything is enqueued. The first call in each
 * context looks the array up (cudaGetSymbolAddress) and should come before
 * any stream capture. All calls on a device share the array, so overlapping
 * calls race on it. */
int piper_merge_float8_noalloc(void* qdata, void* scale, const void* b, const void* a, int64_t rows,
                               int64_t cols, int64_t rank, int64_t block_rows, int64_t block_cols,
                               int32_t e5m2, int32_t compute_dtype, float strength, int32_t has_seed,
                               uint64_t seed, uint64_t offset_base, void* stream);

/* _triton_int8_lora.py:267 merge_int8_lora(qdata, scale, zero_point, block_size,
 * b, a, strength, *, asymmetric, reduce_range, rounding_seed). */
int piper_merge_int8(void* qdata, void* scale, void* zero_point, const void* b, const void* a,
                     int64_t rows, int64_t cols, int64_t rank, int64_t block_rows,
                     int64_t block_cols, int32_t compute_dtype, int32_t scale_dtype,
                     int32_t asymmetric, int32_t reduce_range, float strength, int32_t has_seed,
                     uint64_t seed, uint64_t offset_base, void* workspace,
                     size_t workspace_bytes, void* stream);

/* GGUF Q8_0 / Q4_0 raw-block merge (new capability; decode follows
 * gguf_dequant.py:57-61 and :107-115, re-encode follows gguf 0.19.0
 * quants.Q8_0/Q4_0.quantize_blocks). quant_type: 8 = Q8_0, 2 = Q4_0. */
int piper_merge_gguf(void* raw, const void* b, const void* a, int64_t rows, int64_t cols,
                     int64_t rank, int32_t quant_type, int32_t compute_dtype, float strength,
                     int32_t has_seed, uint64_t seed, uint64_t offset_base, void* stream);

/* _triton_static_float8_lora.py:174 merge_static_float8_lora(qdata, scale, b, a,
 * strength, *, rounding_seed): per-tensor FP8 with one fp32 scale. `workspace`
 * >= piper_merge_workspace_size() of the equivalent per-tensor descriptor (256 B). */
int piper_merge_static_float8(void* qdata, void* scale, const void* b, const void* a, int64_t rows,
                              int64_t cols, int64_t rank, int32_t e5m2, int32_t compute_dtype,
                              float strength, int32_t has_seed, uint64_t seed, uint64_t offset_base,
                              void* workspace, size_t workspace_bytes, void* stream);

/* _triton_bnb8_lora.py:145 merge_bnb8_lora(cb, scb, b, a, strength, *,
 * rounding_seed): int8 CB rows x cols, fp32 SCB per row, fp16 factors. */
int piper_merge_bnb8(void* cb, void* scb, const void* b, const void* a, int64_t rows, int64_t cols,
                     int64_t rank, float strength, int32_t has_seed, uint64_t seed,
                     uint64_t offset_base, void* stream);

/* _triton_quanto_lora.py:317 / :345 merge_quanto_qint8_lora /
 * merge_quanto_qfloat8_lora(qdata, scale, axis, b, a, strength, *,
 * rounding_seed). storage: 0 = qint8, 1 = qfloat8 e4m3, 2 = qfloat8 e5m2;
 * per_row: 1 for axis 0 (one scale per row), 0 for a scalar scale. Per-column
 * (last-axis) scales go through piper_merge_batch with block (rows, 1). The
 * scalar and per-column layouts need workspace (piper_merge_workspace_size).
 * Scales and factors share `compute_dtype`. */
int piper_merge_quanto(void* qdata, void* scale, const void* b, const void* a, int64_t rows,
                       int64_t cols, int64_t rank, int32_t storage, int32_t per_row,
                       int32_t compute_dtype, float strength, int32_t has_seed, uint64_t seed,
                       uint64_t offset_base, void* workspace, size_t workspace_bytes, void* stream);

/* _triton_bnb4_lora.py:434 merge_bnb4_lora(packed, absmax, code, nested_absmax,
 * nested_code, offset, logical_shape, 64, quant_type, b, a, strength, *,
 * rounding_seed). nf4: 1 for NF4, 0 for FP4. Nested absmax (nested_absmax !=
 * NULL) needs workspace (piper_merge_workspace_size) and round-to-nearest. */
int piper_merge_bnb4(void* packed, void* absmax, const void* code, void* nested_absmax,
                     const void* nested_code, void* nested_offset, const void* b, const void* a,
                     int64_t rows, int64_t cols, int64_t rank, int32_t nf4, int32_t compute_dtype,
                     float strength, int32_t has_seed, uint64_t seed, uint64_t offset_base,
                     void* workspace, size_t workspace_bytes, void* stream);

/* Self-test of the failure path, no counterpart in the reference: enqueues a
 * one-thread kernel that waits on a barrier nothing arrives on. Its bounded
 * wait gives up after the kernels' wait limit (2 s), sets the device status
 * word (read it with piper_merge_device_status) and returns; the context stays
 * usable. */
int piper_merge_selftest_timeout(void* stream);

/* Message of the calling thread's last failed call ("" if none). */
const char* piper_merge_last_error(void);

/* Reads and clears the device-side error word of the current device (nonzero
 * when a bounded wait timed out). Synchronises `stream`. */
int piper_merge_device_status(void* stream, uint32_t* status);

/* Library version string, e.g. "piper-merge 0.1 sm_100a". */
const char* piper_merge_version(void);

/* Number of merge kernels this process has launched so far (all devices).
 * No counterpart in the reference: a measurement aid for benchmarks. */
uint64_t piper_merge_launches(void);

#ifdef __cplusplus
}
#endif

#endif /* PIPER_MERGE_H */
