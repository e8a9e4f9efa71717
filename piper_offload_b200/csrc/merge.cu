// merge.cu - fused quantized LoRA merge for B200 (sm_100a).
//
// merge_kernel is persistent and warp-specialised: one CTA per SM strides over
// work items (a 128-row strip of one weight and a range of its BN-column
// tiles, BN = 256, 128 or 64). Its roles:
//   warp 0      one lane issues 2-D bulk tensor copies (TMA, no multicast):
//               the B strip (128 x r) per item, the A tile (r x BN) and the
//               code tile (128 rows x BN columns, swizzled) per tile, into
//               rings of shared-memory stages with full / empty mbarriers;
//   warp 1      one lane owns the 512 tensor-memory columns and issues the
//               rank-r update D = B @ A as tcgen05.mma (M=128, N=BN, K=16)
//               into one of 512 / BN fp32 accumulators per tile;
//   warps 2-3   cp.async for per-row scale bytes (MX / NVFP4) and for the
//               tiles and factors whose alignment rules out TMA;
//   warps 4..   two or three epilogue warpgroups; tile t goes to warpgroup
//               t mod W, whose thread i owns tile row i (tensor-memory lane i):
//               tcgen05.ld of the accumulator 32 columns at a time, decode,
//               merge with the reference's rounding points, block maxima,
//               new scales, round-to-nearest or Philox stochastic codes keyed
//               by logical element offset, written in place in shared memory
//               and stored back with one bulk tensor copy.
// Pass kinds (enum Pass): kLocal, one sweep where every scale is local to a
// tile (MX, NVFP4 single-level, GGUF, bitsandbytes 4-bit, FP8 / INT8 groups of
// at most 256 columns); kFused, per-row FP8 / INT8 in one launch, each CTA
// sweeping a strip's tiles twice (row maxima, then codes) with the maxima on
// chip; kReduce then kEncode (or kLocal), two launches for per-tensor scales,
// groups wider than a tile and the NVFP4 global scale, with block maxima in a
// workspace and launch groups sized so the second launch re-reads from L2.
// Every wait is bounded; a wait that gives up records a status bit and the
// CTA winds down (ptx.cuh).
//
// Reference kernels restated here (Piper Offload 0.2.5):
//   src/piper_offload/_triton_mx_lora.py:162-295      (MX, in place)
//   src/piper_offload/_triton_nvfp4_lora.py:107-367   (NVFP4)
//   src/piper_offload/_triton_float8_lora.py:26-308   (scaled FP8)
//   src/piper_offload/_triton_int8_lora.py:24-236     (affine INT8)
//   src/piper_offload/_triton_stochastic_quantization.py (SR helpers)
//   src/piper_offload/gguf_dequant.py:57-115 + gguf quants (GGUF Q8_0 / Q4_0)
#include <cuda.h>
#include <cuda_runtime.h>
#include <cudaTypedefs.h>

#include <algorithm>
#include <atomic>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <mutex>
#include <string>
#include <vector>

#include "../../include/piper_merge.h"
#include "numerics.cuh"
#include "ptx.cuh"

namespace pm {

constexpr int kMaxWeights = 48;  // 48 x 640-byte descriptors stay within the 32 KB of kernel parameters
constexpr int kMaxRank = 256;

// kLocal: scales local to a tile, one pass. kReduce / kEncode: the two
// launches of layouts whose scales need a reduction across CTAs (per-tensor,
// wide groups, NVFP4 global scale). kFused: per-row layouts in one launch;
// each CTA reduces, then encodes, whole 128-row strips.
enum Pass : int { kLocal = 0, kReduce = 1, kEncode = 2, kFused = 3 };

// Device-side descriptor of one weight (or a row range of one weight).
struct alignas(64) DevWeight {
  CUtensorMap tmap;    // 2-D map of the code bytes (rows x row_bytes), valid when use_tma
  CUtensorMap tmap_a;  // A factor (r x N), boxes of 64 columns x KP rows, 128-byte swizzle
  CUtensorMap tmap_b;  // B factor (M x r), boxes of kb_row bytes x 128 rows, matching swizzle
  uint8_t* q;
  void* scale;
  int8_t* zp;
  float* gscale;
  const uint16_t* b;
  const uint16_t* a;
  uint32_t* qmax;      // workspace: per-qparam max(|x|) or max(x, 0) as float bits
  uint32_t* qmin;      // workspace: per-qparam -min(x, 0) as float bits (INT8)
  float* old_scale;    // workspace: per-qparam input scale (two-pass)
  int32_t* old_zp;     // workspace: per-qparam input zero point (two-pass)
  int64_t row_bytes;   // code bytes per row
  uint64_t offset_base;
  uint32_t k0, k1;     // Philox key (seed lo / hi)
  float strength;
  uint32_t flags;
  int M, N, r, KP;
  int row_begin;       // first row of this launch's range (multiple of 128)
  int row_blocks;      // 128-row strips in the range
  int col_items;       // work items per strip
  int item_cols;       // columns per work item (multiple of the tile width)
  int item_begin;      // first blockIdx of this weight
  int group;           // FP8/INT8 quantization block width in columns
  int nq_row;          // FP8/INT8 quantization blocks per row (0 = per tensor)
  int scale_cols;      // MX: N/32, NVFP4: N/16
  int scale_mode;      // MX E8M0 rounding
  int scale_dt;        // stored scale dtype (INT8: as given; FP8: fp32, Quanto: the compute dtype)
  const float* code16; // BNB4: 16-entry code table
  const float* ncode;  // BNB4 nested: 256-entry code table of the block maxima (else null)
  const float* nabs;   // BNB4 nested: fp32 maximum per 256 blocks
  const float* noff;   // BNB4 nested: fp32 offset
  int col_axis;        // Quanto last-axis scales: one per column (two-pass, workspace per column)
  int use_tma;         // code tiles move by bulk tensor copies (swizzled rows)
  int use_tma_a;       // A tiles by bulk tensor copies (else cp.async into the same layout)
  int use_tma_b;       // B strips by bulk tensor copies (else cp.async into the same layout)
};

struct LaunchParams {
  DevWeight w[kMaxWeights];
  int n_weights;
  int n_items;  // work items over all weights, in order of decreasing cost
  uint32_t sched_slot;  // this launch's item counter in g_sched_next
  int kp_max;    // shared-memory layout is sized for the largest padded rank
  int c_stages;  // ring of (code tile, scale bytes) stages, freed after the write-back
  int a_stages;  // ring of A tiles, freed when the tensor core has read them
  int b_bufs;    // B strips (1 or 2)
};

// Item counters of concurrent launches: each launch takes the next slot of
// this ring, which the host zeroes on the launch's stream just before it.
constexpr int kSchedSlots = 4096;
__device__ unsigned int g_sched_next[kSchedSlots];

__host__ __device__ constexpr int align_up(int x, int a) { return (x + a - 1) / a * a; }

// Code bytes for `cols` columns of one row.
template <int FMT>
__host__ __device__ constexpr int code_bytes(int cols) {
  if constexpr (FMT == PIPER_FMT_MXFP4 || FMT == PIPER_FMT_NVFP4 || FMT == PIPER_FMT_BNB4_NF4 ||
                FMT == PIPER_FMT_BNB4_FP4)
    return cols / 2;
  else if constexpr (FMT == PIPER_FMT_GGUF_Q8_0) return cols / 32 * 34;
  else if constexpr (FMT == PIPER_FMT_GGUF_Q4_0) return cols / 32 * 18;
  else return cols;
}

// Shared-memory row stride of a code tile: 16-byte multiple plus 16 bytes of
// padding, so 8 consecutive rows start in 8 different 16-byte bank groups.
template <int FMT, int BN>
__host__ __device__ constexpr int row_stride() {
  return align_up(code_bytes<FMT>(BN), 16) + 16;
}

// Per-row scale bytes of one tile in shared memory (MX: BN/32, NVFP4: BN/16).
constexpr int kScaleSlot = 16;

// Blocked 128x4 scale layout (_triton_mx_lora.py:97-112, _triton_nvfp4_lora.py:88-104).
__device__ __forceinline__ int64_t swizzled_index(int row, int col, int scale_cols) {
  const int col_blocks = (scale_cols + 3) / 4;
  const int rin = row & 127;
  return (static_cast<int64_t>(row >> 7) * col_blocks + (col >> 2)) * 512 + (rin & 31) * 16 +
         (rin >> 5) * 4 + (col & 3);
}

__device__ __forceinline__ int64_t scale_index(const DevWeight& W, int row, int col) {
  if (W.flags & PIPER_FLAG_SWIZZLED) return swizzled_index(row, col, W.scale_cols);
  return static_cast<int64_t>(row) * W.scale_cols + col;
}

__device__ __forceinline__ float load_scale_dt(const void* p, int64_t i, int dt) {
  if (dt == kBF16) return __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(p)[i]);
  if (dt == kF16) return __half2float(reinterpret_cast<const __half*>(p)[i]);
  return reinterpret_cast<const float*>(p)[i];
}

__device__ __forceinline__ void store_scale_dt(void* p, int64_t i, int dt, float v) {
  if (dt == kBF16) reinterpret_cast<__nv_bfloat16*>(p)[i] = __float2bfloat16_rn(v);
  else if (dt == kF16) reinterpret_cast<__half*>(p)[i] = __float2half_rn(v);
  else reinterpret_cast<float*>(p)[i] = v;
}

__device__ __forceinline__ void atomic_max_nonneg(uint32_t* p, float v) {
  // fmaxf-based accumulation never carries NaN; non-negative floats order like their bits.
  if (v > 0.0f) atomicMax(p, __float_as_uint(v));
}

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xFFFFFFFFu, v, o));
  return v;
}

// Balanced-tree reductions over a chunk. fmaxf / fminf are exact, commutative
// and associative (NaN operands are ignored, -0 orders below +0), so a tree
// gives the same value as the sequential fold while its dependency depth is
// log2(N) instead of N.
template <int N>
__device__ __forceinline__ float tree_max_abs(const float (&m)[N]) {
  float t[N / 2];
#pragma unroll
  for (int i = 0; i < N / 2; ++i) t[i] = fmaxf(fabsf(m[2 * i]), fabsf(m[2 * i + 1]));
#pragma unroll
  for (int w = N / 4; w >= 1; w /= 2) {
#pragma unroll
    for (int i = 0; i < w; ++i) t[i] = fmaxf(t[2 * i], t[2 * i + 1]);
  }
  return t[0];
}
template <int N>
__device__ __forceinline__ float tree_max(const float (&m)[N]) {
  float t[N / 2];
#pragma unroll
  for (int i = 0; i < N / 2; ++i) t[i] = fmaxf(m[2 * i], m[2 * i + 1]);
#pragma unroll
  for (int w = N / 4; w >= 1; w /= 2) {
#pragma unroll
    for (int i = 0; i < w; ++i) t[i] = fmaxf(t[2 * i], t[2 * i + 1]);
  }
  return t[0];
}
template <int N>
__device__ __forceinline__ float tree_min(const float (&m)[N]) {
  float t[N / 2];
#pragma unroll
  for (int i = 0; i < N / 2; ++i) t[i] = fminf(m[2 * i], m[2 * i + 1]);
#pragma unroll
  for (int w = N / 4; w >= 1; w /= 2) {
#pragma unroll
    for (int i = 0; i < w; ++i) t[i] = fminf(t[2 * i], t[2 * i + 1]);
  }
  return t[0];
}

// Three-source maxima (sm_100 `max` / `min` with three operands, one
// instruction each). The plain forms ignore a NaN operand like fmaxf; the
// .NaN forms return NaN when any operand is NaN. `.abs` compares magnitudes.
__device__ __forceinline__ float max3_abs(float a, float b, float c) {
  float d;
  asm("max.abs.f32 %0, %1, %2, %3;" : "=f"(d) : "f"(a), "f"(b), "f"(c));
  return d;
}
__device__ __forceinline__ float max3_abs_nan(float a, float b, float c) {
  float d;
  asm("max.NaN.abs.f32 %0, %1, %2, %3;" : "=f"(d) : "f"(a), "f"(b), "f"(c));
  return d;
}

// Reduction of N values by a three-operand associative, commutative op
// (exact for maxima in any order): ceil(N / 3) operations per level.
template <int N, class Op3>
__device__ __forceinline__ float tree3(const float (&m)[N], Op3 op) {
  if constexpr (N == 1) {
    return m[0];
  } else if constexpr (N == 2) {
    return op(m[0], m[1], m[1]);
  } else {
    constexpr int M = (N + 2) / 3;
    float t[M];
#pragma unroll
    for (int i = 0; i < M; ++i) {
      const int a = 3 * i;
      t[i] = a + 2 < N ? op(m[a], m[a + 1], m[a + 2]) : (a + 1 < N ? op(m[a], m[a + 1], m[a + 1]) : m[a]);
    }
    return tree3<M>(t, op);
  }
}

__device__ __forceinline__ float max3_nan(float a, float b, float c) {
  float d;
  asm("max.NaN.f32 %0, %1, %2, %3;" : "=f"(d) : "f"(a), "f"(b), "f"(c));
  return d;
}
__device__ __forceinline__ float min3_nan(float a, float b, float c) {
  float d;
  asm("min.NaN.f32 %0, %1, %2, %3;" : "=f"(d) : "f"(a), "f"(b), "f"(c));
  return d;
}
__device__ __forceinline__ float max3f(float a, float b, float c) {
  float d;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(d) : "f"(a), "f"(b), "f"(c));
  return d;
}
__device__ __forceinline__ float min3f(float a, float b, float c) {
  float d;
  asm("min.f32 %0, %1, %2, %3;" : "=f"(d) : "f"(a), "f"(b), "f"(c));
  return d;
}

// ------------------------------------------------------------ MX scales
struct MxScale {
  uint32_t code;
  float inv;
};

// Exact ceil(log2(d)) for d > 0 (finite or +inf).
__device__ __forceinline__ float ceil_log2_exact(float d) {
  const uint32_t bits = __float_as_uint(d);
  const int ex = static_cast<int>((bits >> 23) & 0xFFu);
  const uint32_t man = bits & 0x7FFFFFu;
  if (ex == 0xFF) return __int_as_float(0x7F800000);
  if (ex == 0) {  // subnormal: d = man * 2^-149
    const int fl = 31 - __clz(man);
    return static_cast<float>(fl + ((man & (man - 1u)) ? 1 : 0) - 149);
  }
  return static_cast<float>(ex - 127 + (man ? 1 : 0));
}

__device__ __forceinline__ float exp2_int(float u) {  // 2^u for integral u in [-127, 127]
  const int e = static_cast<int>(u);
  if (e >= -126) return __uint_as_float(static_cast<uint32_t>(e + 127) << 23);
  return __uint_as_float(1u << (22 + (e + 127)));
}

// _calculate_scale (_triton_mx_lora.py:115-159).
__device__ __forceinline__ MxScale mx_scale(float amax, int mode, int target, float maxpos,
                                            int mbits) {
  MxScale s;
  if (mode == PIPER_MX_RCEIL) {
    const float d = __fmul_rn(amax, __frcp_rn(maxpos));  // `/ MAX_POS` (constexpr): x * fp32(1 / MAX_POS) on sm_100
    float u;
    if (d != d) u = __int_as_float(0x7FC00000);
    else if (d == 0.0f) u = __int_as_float(0xFF800000);
    else u = ceil_log2_exact(d);
    u = fminf(fmaxf(u, -127.0f), 127.0f);
    uint32_t code = static_cast<uint32_t>(__float2int_rz(u + 127.0f)) & 0xFFu;
    if (d != d) code = 255u;
    s.code = code;
    s.inv = code == 0u ? 1.0f : exp2_int(-u);
    return s;
  }
  uint32_t bits = __float_as_uint(amax);
  if (mode == PIPER_MX_EVEN) {
    const uint32_t bias = mbits == 3 ? 524288u : (mbits == 2 ? 1048576u : 2097152u);
    bits = (bits + bias) & 0xFF800000u;
  }
  int ex = static_cast<int>((bits >> 23) & 255u) - 127;
  if (mode == PIPER_MX_CEIL) ex += (bits & 0x7FFFFFu) != 0u ? 1 : 0;
  int ub = ex - target;
  ub = ub < -127 ? -127 : (ub > 128 ? 128 : ub);
  uint32_t code = static_cast<uint32_t>(ub + 127) & 0xFFu;
  if (amax != amax) code = 255u;
  float sc = __uint_as_float(code << 23);
  sc = fmaxf(sc, 1.1754943508222875e-38f);
  s.code = code;
  s.inv = div_full(1.0f, sc);
  return s;
}

template <int FMT>
struct MxParams;
template <>
struct MxParams<PIPER_FMT_MXFP8_E4M3> {
  static constexpr int kTarget = 8, kMbits = 3;
  static constexpr float kMax = 448.0f;
};
template <>
struct MxParams<PIPER_FMT_MXFP8_E5M2> {
  static constexpr int kTarget = 15, kMbits = 2;
  static constexpr float kMax = 57344.0f;
};
template <>
struct MxParams<PIPER_FMT_MXFP4> {
  static constexpr int kTarget = 2, kMbits = 1;
  static constexpr float kMax = 6.0f;
};

// ------------------------------------------------------- per-thread context
struct RowCtx {
  int row;               // global row
  bool valid;            // row < M
  uint8_t* srow;         // this row's code segment in shared memory
  uint32_t swz;          // XOR applied to 16-byte chunk indices (swizzled TMA rows)
  int box_shift;         // log2(16-byte chunks per box row)
  int box_stride;        // bytes between consecutive boxes of a tile
  const uint8_t* sscale; // this row's prefetched scale bytes for the tile (MX / NVFP4)
  int blk0;              // scale block index of sscale[0]
  int tile_col0;         // first column of the tile
  int tile_cols;         // valid columns in the tile
};

// 16-byte chunk `c16` of this row: box c16 >> box_shift, swizzled chunk within it.
__device__ __forceinline__ uint8_t* chunk_ptr(const RowCtx& c, int c16) {
  const uint32_t in_box = static_cast<uint32_t>(c16) & ((1u << c.box_shift) - 1u);
  return c.srow + (c16 >> c.box_shift) * c.box_stride + ((in_box ^ c.swz) << 4);
}
__device__ __forceinline__ void load_chunks32(const RowCtx& c, int k, uint32_t (&w)[8]) {
  const uint4 a = *reinterpret_cast<const uint4*>(chunk_ptr(c, 2 * k));
  const uint4 b = *reinterpret_cast<const uint4*>(chunk_ptr(c, 2 * k + 1));
  w[0] = a.x; w[1] = a.y; w[2] = a.z; w[3] = a.w;
  w[4] = b.x; w[5] = b.y; w[6] = b.z; w[7] = b.w;
}
__device__ __forceinline__ void store_chunks32(const RowCtx& c, int k, const uint32_t (&w)[8]) {
  *reinterpret_cast<uint4*>(chunk_ptr(c, 2 * k)) = make_uint4(w[0], w[1], w[2], w[3]);
  *reinterpret_cast<uint4*>(chunk_ptr(c, 2 * k + 1)) = make_uint4(w[4], w[5], w[6], w[7]);
}
__device__ __forceinline__ void load_bytes32(const uint8_t* s, uint32_t (&w)[8]) {
  const uint4 a = *reinterpret_cast<const uint4*>(s);
  const uint4 b = *reinterpret_cast<const uint4*>(s + 16);
  w[0] = a.x; w[1] = a.y; w[2] = a.z; w[3] = a.w;
  w[4] = b.x; w[5] = b.y; w[6] = b.z; w[7] = b.w;
}
__device__ __forceinline__ void store_bytes32(uint8_t* s, const uint32_t (&w)[8]) {
  *reinterpret_cast<uint4*>(s) = make_uint4(w[0], w[1], w[2], w[3]);
  *reinterpret_cast<uint4*>(s + 16) = make_uint4(w[4], w[5], w[6], w[7]);
}
__device__ __forceinline__ uint32_t byte_of(const uint32_t (&w)[8], int i) {
  return (w[i >> 2] >> ((i & 3) * 8)) & 0xFFu;
}

// ------------------------------------------------- fp32 factors (CUDA cores)
// The rank-r update of 32 columns [col, col + 32) of one row for fp32 LoRA
// factors. The reference runs them through `tl.dot(b, a, input_precision=
// "ieee")` (_triton_float8_lora.py:53-66 and the other launchers' rank
// loops), which Triton evaluates on CUDA cores as one fused multiply-add per
// rank step, in rank order, starting from +0 and continuing across its rank
// blocks (`accumulator += tl.dot(...)` becomes the dot's accumulator input).
// This function makes the same chain. The rank is padded to the reference's
// block (16 for rank <= 16, else a multiple of 32) with zero factors; each
// padded step adds an exact +0, which only turns a -0 sum into +0. Rows past
// the weight and columns past its end read no memory and give unused values.
__device__ __forceinline__ void f32_update(const DevWeight& W, int row, bool valid, int col, float (&acc)[32]) {
#pragma unroll
  for (int i = 0; i < 32; ++i) acc[i] = 0.0f;
  const float* __restrict__ brow = reinterpret_cast<const float*>(W.b) + static_cast<int64_t>(row) * W.r;
  const float* __restrict__ acol = reinterpret_cast<const float*>(W.a) + col;
  const int ncols = min(32, W.N - col);
  const bool vec = ncols == 32 && ((reinterpret_cast<uintptr_t>(acol) | (static_cast<uintptr_t>(W.N) * 4u)) & 15u) == 0;
  for (int k = 0; k < W.r; ++k) {
    const float bk = valid ? __ldg(brow + k) : 0.0f;
    const float* __restrict__ ak = acol + static_cast<int64_t>(k) * W.N;
    float av[32];
    if (vec) {
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const float4 v = __ldg(reinterpret_cast<const float4*>(ak) + j);
        av[4 * j] = v.x;
        av[4 * j + 1] = v.y;
        av[4 * j + 2] = v.z;
        av[4 * j + 3] = v.w;
      }
    } else {
#pragma unroll
      for (int j = 0; j < 32; ++j) av[j] = j < ncols ? __ldg(ak + j) : 0.0f;
    }
#pragma unroll
    for (int j = 0; j < 32; ++j) acc[j] = __fmaf_rn(bk, av[j], acc[j]);
  }
  const int rank_block = W.r <= 16 ? 16 : 32;
  if (W.r % rank_block != 0) {
#pragma unroll
    for (int j = 0; j < 32; ++j) acc[j] = __fadd_rn(acc[j], 0.0f);
  }
}

// Stores the new scale bytes of this thread's row for one tile (MX: one per
// 32 columns, NVFP4: one per 16), which the encoders leave in the tile's
// shared-memory scale slot in place of the input bytes: one wide store per row
// and tile instead of a one-byte store per block, whose 32 lanes (32 rows)
// would each touch another sector.
template <int FMT>
__device__ __forceinline__ void flush_tile_scales(const DevWeight& W, const RowCtx& c) {
  if (!c.valid) return;
  constexpr int kBlk = FMT == PIPER_FMT_NVFP4 ? 16 : 32;
  const int nb = (c.tile_cols + kBlk - 1) / kBlk;
  uint8_t* scale8 = reinterpret_cast<uint8_t*>(W.scale);
  const uint8_t* src = c.sscale;
  if (W.flags & PIPER_FLAG_SWIZZLED) {
    // 128x4 blocked layout: blocks 4j .. 4j+3 of a row are 4 contiguous bytes
    // (tiles start on a multiple of 4 blocks).
    int j = 0;
    for (; j + 4 <= nb; j += 4)
      *reinterpret_cast<uint32_t*>(scale8 + swizzled_index(c.row, c.blk0 + j, W.scale_cols)) =
          *reinterpret_cast<const uint32_t*>(src + j);
    for (; j < nb; ++j) scale8[swizzled_index(c.row, c.blk0 + j, W.scale_cols)] = src[j];
    return;
  }
  uint8_t* dst = scale8 + static_cast<int64_t>(c.row) * W.scale_cols + c.blk0;
  const uintptr_t a = reinterpret_cast<uintptr_t>(dst);
  if (nb == 16 && (a & 15u) == 0) {
    *reinterpret_cast<uint4*>(dst) = *reinterpret_cast<const uint4*>(src);
  } else if (nb == 8 && (a & 7u) == 0) {
    *reinterpret_cast<uint2*>(dst) = *reinterpret_cast<const uint2*>(src);
  } else if (nb == 4 && (a & 3u) == 0) {
    *reinterpret_cast<uint32_t*>(dst) = *reinterpret_cast<const uint32_t*>(src);
  } else {
    for (int j = 0; j < nb; ++j) dst[j] = src[j];
  }
}

// ================================================================ MX epilogue
template <int FMT, int CDT>
__device__ __forceinline__ void mx_chunk(const DevWeight& W, const RowCtx& c, int k,
                                         const float (&acc)[32]) {
  using P = MxParams<FMT>;
  const int col = c.tile_col0 + 32 * k;
  const int blk = col >> 5;
  const uint32_t sc = c.valid ? c.sscale[blk - c.blk0] : 127u;
  const float bscale = dec_e8m0(sc);
  // Decode: FP8 / FP4 values are exactly representable in bf16, so the
  // reference's bf16 cast of the element is the identity.
  float merged[32];
  if constexpr (FMT == PIPER_FMT_MXFP4) {
    const uint4 pk = *reinterpret_cast<const uint4*>(chunk_ptr(c, k));
    const uint32_t wv[4] = {pk.x, pk.y, pk.z, pk.w};
#pragma unroll
    for (int j = 0; j < 16; ++j) dec_e2m1x2(wv[j >> 2] >> ((j & 3) * 8), merged[2 * j], merged[2 * j + 1]);
  } else {
    uint32_t wv[8];
    load_chunks32(c, k, wv);
#pragma unroll
    for (int w = 0; w < 8; ++w) {
      float f[4];
      dec_fp8x4<FMT == PIPER_FMT_MXFP8_E4M3>(wv[w], f);
#pragma unroll
      for (int j = 0; j < 4; ++j) merged[4 * w + j] = f[j];
    }
  }
  // base = bf16(elem * bf16(scale)): for scale codes 20..230 every product is
  // an exact bf16 normal, so the rounding is the identity. fp32 compute
  // (float32 weights) keeps the fp32 product (_triton_mx_lora.py:239-245).
  if (CDT == kF32 || (sc >= 20u && sc <= 230u)) {
#pragma unroll
    for (int i = 0; i < 32; ++i) merged[i] = __fmul_rn(merged[i], bscale);
  } else {
    const float bs = bf16r(bscale);
#pragma unroll
    for (int i = 0; i < 32; ++i) merged[i] = bf16r(__fmul_rn(merged[i], bs));
  }
#pragma unroll
  for (int i = 0; i < 32; ++i) merged[i] = fmaf(acc[i], W.strength, merged[i]);
#pragma unroll
  for (int i = 0; i < 32; i += 2) round_dt2<CDT>(merged[i], merged[i + 1]);
  const float amax = tree_max_abs(merged);
  const MxScale s = mx_scale(amax, W.scale_mode, P::kTarget, P::kMax, P::kMbits);
  const bool sr = (W.flags & PIPER_FLAG_STOCHASTIC) != 0u;
  const PhiloxKey key = philox_key(W.k0, W.k1);
  const uint64_t off0 =
      W.offset_base + static_cast<uint64_t>(c.row) * static_cast<uint64_t>(W.N) + col;
#pragma unroll
  for (int i = 0; i < 32; ++i) merged[i] = fminf(fmaxf(__fmul_rn(merged[i], s.inv), -P::kMax), P::kMax);
  if constexpr (FMT == PIPER_FMT_MXFP4) {
    uint32_t out[4] = {0u, 0u, 0u, 0u};
    if (sr) {
#pragma unroll
      for (int w = 0; w < 4; ++w) {
        float v[8];
#pragma unroll
        for (int j = 0; j < 8; ++j) v[j] = merged[8 * w + j];
        uint32_t nib[1];
        sr_e2m1xn<8>(v, key, off0 + 8 * w, nib);
        out[w] = nib[0];
      }
    } else {
#pragma unroll
      for (int j = 0; j < 16; ++j) out[j >> 2] |= enc_e2m1x2(merged[2 * j], merged[2 * j + 1]) << ((j & 3) * 8);
    }
    *reinterpret_cast<uint4*>(chunk_ptr(c, k)) = make_uint4(out[0], out[1], out[2], out[3]);
  } else {
    constexpr bool kE4 = FMT == PIPER_FMT_MXFP8_E4M3;
    uint32_t out[8];
    if (sr) {
#pragma unroll
      for (int w8 = 0; w8 < 4; ++w8) {
        float x[8];
#pragma unroll
        for (int j = 0; j < 8; ++j) x[j] = merged[8 * w8 + j];
        uint32_t wd[2];
        sr_fp8xn<kE4, 8>(x, P::kMax, key, off0 + 8 * w8, wd);
        out[2 * w8] = wd[0];
        out[2 * w8 + 1] = wd[1];
      }
    } else {
#pragma unroll
      for (int w = 0; w < 8; ++w)
        out[w] = enc_fp8x4<kE4>(merged[4 * w], merged[4 * w + 1], merged[4 * w + 2], merged[4 * w + 3]);
    }
    store_chunks32(c, k, out);
  }
  // The new scale byte replaces the input one in the tile's shared-memory slot;
  // flush_tile_scales stores the row's bytes of the tile at once.
  const_cast<uint8_t*>(c.sscale)[blk - c.blk0] = static_cast<uint8_t>(s.code);
}

// Fast path of mx_chunk, same codes and scale, for the common block: scale
// code in [20, 230] (every decoded product exact in bf16), merged values all
// finite with a maximum of 0 or at least 2^-100, and a new inverse scale that
// is an exact power of two. Then
//  * merged = fma(acc, strength, elem * scale) runs two elements per packed
//    instruction and stays unrounded for the block maximum (rounding is
//    monotone: max |bf16(x)| = bf16(max |x|));
//  * bf16(merged) * inv = bf16(merged * inv), so the normalized values take one
//    packed multiply and one packed rounding (a bf16-subnormal merged value
//    scales to below 2^-18 there, which encodes as zero either way);
//  * the satfinite conversions clamp to the largest finite code as the
//    reference's clamp does for finite values.
// Any other block returns false before writing anything and takes mx_chunk.
template <int FMT, int CDT>
__device__ __forceinline__ bool mx_chunk_fast(const DevWeight& W, const RowCtx& c, int k, const float (&acc)[32]) {
  using P = MxParams<FMT>;
  if constexpr (CDT == kF32) return false;  // the shortcuts below rely on bf16 rounding
  const int col = c.tile_col0 + 32 * k;
  const int blk = col >> 5;
  const uint32_t sc = c.valid ? c.sscale[blk - c.blk0] : 127u;
  if (sc < 20u || sc > 230u) {
    return false;
  }
  const float bscale = dec_e8m0(sc);
  float m[32];
  if constexpr (FMT == PIPER_FMT_MXFP4) {
    const uint4 pk = *reinterpret_cast<const uint4*>(chunk_ptr(c, k));
    const uint32_t wv[4] = {pk.x, pk.y, pk.z, pk.w};
#pragma unroll
    for (int j = 0; j < 16; ++j) dec_e2m1x2(wv[j >> 2] >> ((j & 3) * 8), m[2 * j], m[2 * j + 1]);
  } else {
    uint32_t wv[8];
    load_chunks32(c, k, wv);
#pragma unroll
    for (int w = 0; w < 8; ++w) {
      float f[4];
      dec_fp8x4<FMT == PIPER_FMT_MXFP8_E4M3>(wv[w], f);
#pragma unroll
      for (int j = 0; j < 4; ++j) m[4 * w + j] = f[j];
    }
  }
  const float2 b2 = make_float2(bscale, bscale);
  const float2 st2 = make_float2(W.strength, W.strength);
#pragma unroll
  for (int i = 0; i < 32; i += 2) {
    const float2 t = __ffma2_rn(make_float2(acc[i], acc[i + 1]), st2, __fmul2_rn(make_float2(m[i], m[i + 1]), b2));
    m[i] = t.x;
    m[i + 1] = t.y;
  }
  float amax = tree3(m, max3_abs_nan);
  if (!(amax <= 3.40282347e38f) || (amax != 0.0f && amax < 7.888609052210118e-31f /* 2^-100 */)) {
    return false;
  }
  amax = bf16r(amax);
  const MxScale s = mx_scale(amax, W.scale_mode, P::kTarget, P::kMax, P::kMbits);
  if ((__float_as_uint(s.inv) & 0x807FFFFFu) != 0u || s.inv == 0.0f) {
    return false;
  }
  const float2 inv2 = make_float2(s.inv, s.inv);
#pragma unroll
  for (int i = 0; i < 32; i += 2) {
    float2 t = __fmul2_rn(make_float2(m[i], m[i + 1]), inv2);
    bf16r2(t.x, t.y);
    m[i] = t.x;
    m[i + 1] = t.y;
  }
  const bool sr = (W.flags & PIPER_FLAG_STOCHASTIC) != 0u;
  const PhiloxKey key = philox_key(W.k0, W.k1);
  const uint64_t off0 = W.offset_base + static_cast<uint64_t>(c.row) * static_cast<uint64_t>(W.N) + col;
  if constexpr (FMT == PIPER_FMT_MXFP4) {
    uint32_t out[4] = {0u, 0u, 0u, 0u};
    if (sr) {
#pragma unroll
      for (int w = 0; w < 4; ++w) {
        float v[8];
#pragma unroll
        for (int j = 0; j < 8; ++j) v[j] = m[8 * w + j];
        uint32_t nib[1];
        sr_e2m1xn<8>(v, key, off0 + 8 * w, nib);  // |v| < 8: magnitudes from 6 up keep the top code
        out[w] = nib[0];
      }
    } else {
#pragma unroll
      for (int j = 0; j < 16; ++j) out[j >> 2] |= enc_e2m1x2(m[2 * j], m[2 * j + 1]) << ((j & 3) * 8);
    }
    *reinterpret_cast<uint4*>(chunk_ptr(c, k)) = make_uint4(out[0], out[1], out[2], out[3]);
  } else {
    constexpr bool kE4 = FMT == PIPER_FMT_MXFP8_E4M3;
    uint32_t out[8];
    if (sr) {
#pragma unroll
      for (int w8 = 0; w8 < 4; ++w8) {
        float x[8];
#pragma unroll
        for (int j = 0; j < 8; ++j) x[j] = m[8 * w8 + j];
        uint32_t wd[2];
        sr_fp8xn_finite<kE4, 8>(x, key, off0 + 8 * w8, wd);
        out[2 * w8] = wd[0];
        out[2 * w8 + 1] = wd[1];
      }
    } else {
#pragma unroll
      for (int w = 0; w < 8; ++w) out[w] = enc_fp8x4<kE4>(m[4 * w], m[4 * w + 1], m[4 * w + 2], m[4 * w + 3]);
    }
    store_chunks32(c, k, out);
  }
  const_cast<uint8_t*>(c.sscale)[blk - c.blk0] = static_cast<uint8_t>(s.code);  // flushed per tile
  return true;
}

// ============================================================= NVFP4 epilogue
// One 16-element block. `codes` holds its 8 packed bytes (in: input codes,
// out: merged codes). PASS kReduce accumulates |merged| into `amax_acc`.
template <int PASS, int CDT>
__device__ __forceinline__ void nvfp4_block(const DevWeight& W, const RowCtx& c, int col,
                                            const float* acc, float g_in, float g_out,
                                            bool two_level, float& amax_acc, uint2& codes) {
  uint8_t* scale8 = reinterpret_cast<uint8_t*>(W.scale);
  const int blk = col >> 4;
  float bsc = dec_e4m3(c.valid ? c.sscale[blk - c.blk0] : 0u);  // E4M3 values are exact in bf16
  if (two_level) {
    bsc = __fmul_rn(bsc, g_in);
    if (CDT == kBF16) bsc = bf16r(bsc);
  }
  float m[16];
  const uint32_t wv[2] = {codes.x, codes.y};
#pragma unroll
  for (int j = 0; j < 8; ++j) dec_e2m1x2(wv[j >> 2] >> ((j & 3) * 8), m[2 * j], m[2 * j + 1]);
#pragma unroll
  for (int i = 0; i < 16; ++i) m[i] = __fmul_rn(m[i], bsc);
  // Single-level: e2m1 (<= 2 significant bits) x e4m3 (<= 4) is an exact bf16
  // normal, so only the two-level product needs rounding.
  if (CDT == kBF16 && two_level) {
#pragma unroll
    for (int i = 0; i < 16; i += 2) bf16r2(m[i], m[i + 1]);
  }
#pragma unroll
  for (int i = 0; i < 16; ++i) {
    const float upd = __fmul_rn(acc[i], W.strength);
    m[i] = upd == 0.0f ? m[i] : fmaf(acc[i], W.strength, m[i]);
  }
#pragma unroll
  for (int i = 0; i < 16; i += 2) round_dt2<CDT>(m[i], m[i + 1]);
  const float amax = tree_max_abs(m);
  if constexpr (PASS == kReduce) {
    if (c.valid) amax_acc = fmaxf(amax_acc, amax);
  } else {
    float fs = __fmul_rn(amax, 1.0f / 6.0f);  // `/ 6.0` (literal): x * fp32(1 / 6) on sm_100
    if (two_level) fs = div_full(fs, g_out);
    fs = fminf(fmaxf(fs, 0.015625f), 448.0f);
    const uint32_t fcode = enc_e4m3(fs);
    fs = dec_e4m3(fcode);
    const int64_t sidx = scale_index(W, c.row, blk);
    if (c.valid) const_cast<uint8_t*>(c.sscale)[blk - c.blk0] = static_cast<uint8_t>(fcode);  // flushed per tile
    else if (W.flags & PIPER_FLAG_SWIZZLED) scale8[sidx] = 0u;  // swizzle padding rows
    const bool sr = (W.flags & PIPER_FLAG_STOCHASTIC) != 0u;
    if (two_level) {
      const float recip = div_full(div_full(1.0f, g_out), fs);
#pragma unroll
      for (int i = 0; i < 16; ++i) m[i] = __fmul_rn(m[i], recip);
    } else if (sr) {
#pragma unroll
      for (int i = 0; i < 16; ++i) m[i] = div_full(m[i], fs);
    } else {
      // x * RN(1/fs), re-checked with div.full near an E2M1 rounding boundary.
      const float inv = __frcp_rn(fs);
      float q[16];
      bool near = false;
#pragma unroll
      for (int i = 0; i < 16; ++i) {
        q[i] = __fmul_rn(m[i], inv);
        near |= near_e2m1_edge(q[i]);
      }
      if (near) {
#pragma unroll
        for (int i = 0; i < 16; ++i) q[i] = div_full(m[i], fs);
      }
#pragma unroll
      for (int i = 0; i < 16; ++i) m[i] = q[i];
    }
#pragma unroll
    for (int i = 0; i < 16; ++i) m[i] = fminf(fmaxf(m[i], -6.0f), 6.0f);
    uint32_t out[2] = {0u, 0u};
    if (sr) {
      const PhiloxKey key = philox_key(W.k0, W.k1);
      const uint64_t off0 =
          W.offset_base + static_cast<uint64_t>(c.row) * static_cast<uint64_t>(W.N) + col;
#pragma unroll
      for (int w = 0; w < 2; ++w) {
        float v[8];
#pragma unroll
        for (int j = 0; j < 8; ++j) v[j] = m[8 * w + j];
        uint32_t nib[1];
        sr_e2m1xn<8>(v, key, off0 + 8 * w, nib);
        out[w] = nib[0];
      }
    } else {
#pragma unroll
      for (int j = 0; j < 8; ++j) out[j >> 2] |= enc_e2m1x2(m[2 * j], m[2 * j + 1]) << ((j & 3) * 8);
    }
    codes = make_uint2(out[0], out[1]);
  }
}

// Fast path of nvfp4_block, same codes and scales, for a block whose decoded
// scale is a non-negative finite value (so no base value is -0, and
// fma(acc, strength, base) equals the reference's `where(update == 0, base,
// base + update)` for every update, signed zeros included) and whose merged
// values are all finite: the merge runs two elements per packed instruction,
// the block maximum takes three-operand maxima, and the satfinite E2M1
// conversion clamps as the reference's clamp to [-6, 6] does for finite
// values (stochastic codes keep the top code from 6 up). The quotient of a
// single-level block is div.full, as the reference divides. Returns false,
// having written nothing, for any other block.
template <int PASS, int CDT>
__device__ __forceinline__ bool nvfp4_block_fast(const DevWeight& W, const RowCtx& c, int col, const float* acc,
                                                 float g_in, float g_out, bool two_level, float& amax_acc,
                                                 uint2& codes) {
  const int blk = col >> 4;
  float bsc = dec_e4m3(c.valid ? c.sscale[blk - c.blk0] : 0u);
  if (two_level) {
    bsc = __fmul_rn(bsc, g_in);
    if (CDT == kBF16) bsc = bf16r(bsc);
  }
  if (__float_as_uint(bsc) >= 0x7F800000u) return false;  // negative (incl. -0), infinite or NaN
  float m[16];
  const uint32_t wv[2] = {codes.x, codes.y};
#pragma unroll
  for (int j = 0; j < 8; ++j) dec_e2m1x2(wv[j >> 2] >> ((j & 3) * 8), m[2 * j], m[2 * j + 1]);
  const float2 b2 = make_float2(bsc, bsc);
  const float2 st2 = make_float2(W.strength, W.strength);
#pragma unroll
  for (int i = 0; i < 16; i += 2) {
    float2 t = __fmul2_rn(make_float2(m[i], m[i + 1]), b2);
    if (CDT == kBF16 && two_level) bf16r2(t.x, t.y);  // single-level products are exact bf16 values
    t = __ffma2_rn(make_float2(acc[i], acc[i + 1]), st2, t);
    // The maxima pass rounds only the block maximum below (rounding is
    // monotone: max |compute(x)| = compute(max |x|)).
    if constexpr (PASS != kReduce) round_dt2<CDT>(t.x, t.y);
    m[i] = t.x;
    m[i + 1] = t.y;
  }
  const float amax = tree3(m, max3_abs_nan);
  if (!(amax <= 3.40282347e38f)) return false;
  if constexpr (PASS == kReduce) {
    if (c.valid) amax_acc = fmaxf(amax_acc, round_dt<CDT>(amax));
    return true;
  } else {
    uint8_t* scale8 = reinterpret_cast<uint8_t*>(W.scale);
    float fs = __fmul_rn(amax, 1.0f / 6.0f);  // `/ 6.0` (literal): x * fp32(1 / 6) on sm_100
    if (two_level) fs = div_full(fs, g_out);
    fs = fminf(fmaxf(fs, 0.015625f), 448.0f);
    const uint32_t fcode = enc_e4m3(fs);
    fs = dec_e4m3(fcode);
    const int64_t sidx = scale_index(W, c.row, blk);
    if (c.valid) const_cast<uint8_t*>(c.sscale)[blk - c.blk0] = static_cast<uint8_t>(fcode);  // flushed per tile
    else if (W.flags & PIPER_FLAG_SWIZZLED) scale8[sidx] = 0u;  // swizzle padding rows
    if (two_level) {
      const float recip = div_full(div_full(1.0f, g_out), fs);
      const float2 r2 = make_float2(recip, recip);
#pragma unroll
      for (int i = 0; i < 16; i += 2) {
        const float2 t = __fmul2_rn(make_float2(m[i], m[i + 1]), r2);
        m[i] = t.x;
        m[i + 1] = t.y;
      }
    } else {
#pragma unroll
      for (int i = 0; i < 16; ++i) m[i] = div_full(m[i], fs);
    }
    uint32_t out[2] = {0u, 0u};
    if (W.flags & PIPER_FLAG_STOCHASTIC) {
      const PhiloxKey key = philox_key(W.k0, W.k1);
      const uint64_t off0 = W.offset_base + static_cast<uint64_t>(c.row) * static_cast<uint64_t>(W.N) + col;
#pragma unroll
      for (int w = 0; w < 2; ++w) {
        float v[8];
#pragma unroll
        for (int j = 0; j < 8; ++j) v[j] = m[8 * w + j];
        uint32_t nib[1];
        sr_e2m1xn<8>(v, key, off0 + 8 * w, nib);
        out[w] = nib[0];
      }
    } else {
#pragma unroll
      for (int j = 0; j < 8; ++j) out[j >> 2] |= enc_e2m1x2(m[2 * j], m[2 * j + 1]) << ((j & 3) * 8);
    }
    codes = make_uint2(out[0], out[1]);
    return true;
  }
}

template <int PASS, int CDT>
__device__ __forceinline__ void nvfp4_chunk(const DevWeight& W, const RowCtx& c, int k,
                                            const float (&acc)[32], float g_in, float g_out,
                                            bool two_level, float& amax_acc) {
  const int col = c.tile_col0 + 32 * k;
  uint4 pk = *reinterpret_cast<const uint4*>(chunk_ptr(c, k));
  uint2 lo = make_uint2(pk.x, pk.y), hi = make_uint2(pk.z, pk.w);
  if (!nvfp4_block_fast<PASS, CDT>(W, c, col, acc, g_in, g_out, two_level, amax_acc, lo))
    nvfp4_block<PASS, CDT>(W, c, col, acc, g_in, g_out, two_level, amax_acc, lo);
  if (!nvfp4_block_fast<PASS, CDT>(W, c, col + 16, acc + 16, g_in, g_out, two_level, amax_acc, hi))
    nvfp4_block<PASS, CDT>(W, c, col + 16, acc + 16, g_in, g_out, two_level, amax_acc, hi);
  if constexpr (PASS != kReduce)
    *reinterpret_cast<uint4*>(chunk_ptr(c, k)) = make_uint4(lo.x, lo.y, hi.x, hi.y);
}

// ========================================================= FP8 / INT8 helpers
template <int FMT>
struct Int8Range {
  int qmin, qmax;
};

__device__ __forceinline__ int qparam_index(const DevWeight& W, int row, int col) {
  return W.nq_row == 0 ? 0 : row * W.nq_row + col / W.group;
}

// New FP8 scale from the block amax (_reduce_row_scale_kernel, _triton_float8_lora.py:249-271).
// `max_abs / FP8_LIMIT` divides by a constexpr, which Triton evaluates on sm_100
// as a product with the fp32 reciprocal of the constant (measured on a B200).
template <int CDT>
__device__ __forceinline__ float fp8_new_scale(float amax, float limit) {
  const float rcp = limit == 448.0f ? 1.0f / 448.0f : 1.0f / 57344.0f;
  float s = round_dt<CDT>(__fmul_rn(amax, rcp));
  return s == 0.0f ? 1.1920928955078125e-07f : s;
}

// INT8 qparams (_choose_qparams_kernel, _triton_int8_lora.py:122-186).
struct Int8Q {
  float scale;   // value of the stored scale (scale dtype)
  int zp;
};
template <int CDT>
__device__ __forceinline__ Int8Q int8_qparams(float min_v, float max_v, bool asym, int qmin,
                                              int qmax, int scale_dt) {
  min_v = round_dt<CDT>(min_v);
  max_v = round_dt<CDT>(max_v);
  float s;
  if (asym) {
    const float rng = round_dt<CDT>(__fsub_rn(max_v, min_v));
    // Constexpr divisors: a product with the fp32 reciprocal, as Triton evaluates them on sm_100.
    s = __fmul_rn(rng, __frcp_rn(static_cast<float>(qmax - qmin)));
  } else {
    s = __fmul_rn(fmaxf(-min_v, max_v), __frcp_rn(static_cast<float>(qmax - qmin) / 2.0f));
  }
  s = round_dt<CDT>(s);
  s = fmaxf(s, 1.1920928955078125e-07f);
  s = round_dt<CDT>(s);
  int zp = 0;
  if (asym) {
    const float ratio = round_dt<CDT>(div_full(min_v, s));
    long long z = static_cast<long long>(qmin) - __float2ll_rn(ratio);
    z = z < qmin ? qmin : (z > qmax ? qmax : z);
    zp = static_cast<int>(z);
  }
  Int8Q q;
  q.scale = round_dt_rt(s, scale_dt);
  q.zp = zp;
  return q;
}

// _quantize_kernel (_triton_int8_lora.py:189-236) for 32 values sharing one
// quantization block: inverse_scale = scale_dtype(1 / scale) (div.full),
// scaled = scale_dtype(x * inverse_scale), q = rint(scaled) + zp, optional
// stochastic rounding of x / scale + zp, clamp.
__device__ __forceinline__ void round_rt2(float& a, float& b, int dt) {
  if (dt == kBF16) bf16r2(a, b);
  else if (dt == kF16) f16r2(a, b);
}

__device__ __forceinline__ void int8_encode32(const float (&m)[32], const Int8Q& q, int qmin, int qmax,
                                              int scale_dt, bool sr, const PhiloxKey& key, uint64_t off0,
                                              uint32_t (&out)[8]) {
  float inv = div_full(1.0f, q.scale);
  inv = round_dt_rt(inv, scale_dt);
  if (!sr) {
    float x[32];
#pragma unroll
    for (int i = 0; i < 32; ++i) x[i] = __fmul_rn(m[i], inv);
    if (scale_dt == kBF16) {  // one dispatch per chunk
#pragma unroll
      for (int i = 0; i < 32; i += 2) bf16r2(x[i], x[i + 1]);
    } else if (scale_dt == kF16) {
#pragma unroll
      for (int i = 0; i < 32; i += 2) f16r2(x[i], x[i + 1]);
    }
    // Round to nearest in the integer domain: for |x| < 2^22 the bits of
    // x + 1.5 * 2^23 minus those of 1.5 * 2^23 are rint(x); a chunk holding a
    // NaN or a larger value takes the general path below.
    bool big = false;
#pragma unroll
    for (int i = 0; i < 32; ++i) big |= !(fabsf(x[i]) < 4194304.0f);
    if (!big) {
      int qi[32];
#pragma unroll
      for (int i = 0; i < 32; ++i) {
        const int r = static_cast<int>(__float_as_uint(__fadd_rn(x[i], 12582912.0f)) - 0x4B400000u) + q.zp;
        qi[i] = min(max(r, qmin), qmax);
      }
#pragma unroll
      for (int w = 0; w < 8; ++w)
        out[w] = __byte_perm(__byte_perm(qi[4 * w], qi[4 * w + 1], 0x0040), __byte_perm(qi[4 * w + 2], qi[4 * w + 3], 0x0040),
                             0x5410);
      return;
    }
  }
  const float zpf = static_cast<float>(q.zp);
  const float qlo = static_cast<float>(qmin), qhi = static_cast<float>(qmax);
#pragma unroll
  for (int w = 0; w < 8; ++w) {
    float xs[4], qq[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) xs[j] = __fmul_rn(m[4 * w + j], inv);
    round_rt2(xs[0], xs[1], scale_dt);
    round_rt2(xs[2], xs[3], scale_dt);
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      // rint (half to even) of |x| < 2^22 via the 1.5 * 2^23 magic addend;
      // the sum with zp is exact in fp32 there.
      const float xi = xs[j];
      if (fabsf(xi) < 4194304.0f) qq[j] = __fadd_rn(__fsub_rn(__fadd_rn(xi, 12582912.0f), 12582912.0f), zpf);
      else qq[j] = static_cast<float>(__float2ll_rn(xi) + q.zp);
    }
    if (sr) {
      float ss[4];
#pragma unroll
      for (int j = 0; j < 4; ++j) ss[j] = __fadd_rn(div_full(m[4 * w + j], q.scale), zpf);
      sr_int_xn<4>(ss, qq, qlo, qhi, key, off0 + 4 * w);
    }
    // Clamped codes are integers in [-128, 255]: the low byte of the bits of
    // q + 1.5 * 2^23 is q mod 256.
    uint32_t qb[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) qb[j] = __float_as_uint(__fadd_rn(fminf(fmaxf(qq[j], qlo), qhi), 12582912.0f));
    out[w] = __byte_perm(__byte_perm(qb[0], qb[1], 0x0040), __byte_perm(qb[2], qb[3], 0x0040), 0x5410);
  }
}

__device__ __forceinline__ uint32_t int8_encode(float v, const Int8Q& q, int qmin, int qmax,
                                                int scale_dt, bool sr, const PhiloxKey& key,
                                                uint64_t off) {
  const float inv = round_dt_rt(div_full(1.0f, q.scale), scale_dt);
  const float scaled = round_dt_rt(__fmul_rn(v, inv), scale_dt);
  long long qi = __float2ll_rn(scaled) + q.zp;
  float qf = static_cast<float>(qi);
  if (sr) {
    const float ss = __fadd_rn(div_full(v, q.scale), static_cast<float>(q.zp));
    qf = sr_int(ss, qf, static_cast<float>(qmin), static_cast<float>(qmax), key, off);
  }
  qf = fminf(fmaxf(qf, static_cast<float>(qmin)), static_cast<float>(qmax));
  return static_cast<uint32_t>(static_cast<int32_t>(qf)) & 0xFFu;
}

// ------------------------------------------------ bitsandbytes / Quanto flavors
// bitsandbytes LLM.int8 (_triton_bnb8_lora.py) and Quanto qbytes
// (_triton_quanto_lora.py) run on the INT8 / FP8 pipeline with their own
// decode, scale and encode arithmetic, selected per weight at run time.
enum Flavor { kTorchao = 0, kBnb = 1, kQuanto = 2 };

// Kernel formats: the bitsandbytes / Quanto ids instantiate the INT8 / FP8
// kernels with their flavor fixed at compile time.
__host__ __device__ constexpr int base_fmt(int f) {
  return f == PIPER_FMT_BNB8 || f == PIPER_FMT_QUANTO_INT8 ? PIPER_FMT_INT8
         : f == PIPER_FMT_QUANTO_FP8_E4M3                 ? PIPER_FMT_FP8_E4M3
         : f == PIPER_FMT_QUANTO_FP8_E5M2                 ? PIPER_FMT_FP8_E5M2
                                                          : f;
}
__host__ __device__ constexpr int flavor_of(int f) {
  return f == PIPER_FMT_BNB8 ? kBnb
         : (f == PIPER_FMT_QUANTO_INT8 || f == PIPER_FMT_QUANTO_FP8_E4M3 || f == PIPER_FMT_QUANTO_FP8_E5M2) ? kQuanto
                                                                                                             : kTorchao;
}
__host__ __device__ constexpr int kernel_fmt(int base, int flavor) {
  return flavor == kBnb      ? PIPER_FMT_BNB8
         : flavor == kQuanto ? (base == PIPER_FMT_INT8       ? PIPER_FMT_QUANTO_INT8
                                : base == PIPER_FMT_FP8_E4M3 ? PIPER_FMT_QUANTO_FP8_E4M3
                                                             : PIPER_FMT_QUANTO_FP8_E5M2)
                             : base;
}

// New scale of a block from its max |x|. bitsandbytes: SCB = the row's max
// |merged| (_triton_bnb8_lora.py:84-98). Quanto: (amax / qmax).to(dtype), 0 ->
// fp32 eps (_triton_quanto_lora.py:202-217); torch divides a CUDA tensor by a
// host scalar as a multiplication by the scalar's fp32 reciprocal.
template <int CDT>
__device__ __forceinline__ float flavor_scale(int flavor, float amax, float qmax) {
  if (flavor == kBnb) return amax;
  const float s = round_dt<CDT>(__fmul_rn(amax, __frcp_rn(qmax)));
  return s == 0.0f ? 1.1920928955078125e-07f : s;
}

// INT8 codes of 32 merged values of one row for the bitsandbytes and Quanto
// flavors. bitsandbytes (_triton_bnb8_lora.py:101-142): x = (v / SCB) * 127
// (0 where SCB == 0), rint or stochastic, clamp [-127, 127]. Quanto qint8
// (_triton_quanto_lora.py:107-168): s = v / scale, rint(dtype(s)) or
// stochastic on s, clamp [-128, 127].
template <int CDT>
__device__ __forceinline__ void flavor_int8_encode32(int flavor, const float (&m)[32], float s, bool sr,
                                                     const PhiloxKey& key, uint64_t off0, uint32_t (&out)[8]) {
  const float lo = flavor == kBnb ? -127.0f : -128.0f;
  if (!sr) {
    // Round to nearest in the integer domain (see int8_encode32); a chunk
    // holding a NaN or |x| >= 2^22 takes the general loop below.
    float x[32];
    bool big = false;
#pragma unroll
    for (int i = 0; i < 32; ++i) {
      x[i] = flavor == kBnb ? (s == 0.0f ? 0.0f : __fmul_rn(div_full(m[i], s), 127.0f))
                            : round_dt<CDT>(div_full(m[i], s));
      big |= !(fabsf(x[i]) < 4194304.0f);
    }
    if (!big) {
      const int ilo = flavor == kBnb ? -127 : -128;
      int qi[32];
#pragma unroll
      for (int i = 0; i < 32; ++i) {
        const int r = static_cast<int>(__float_as_uint(__fadd_rn(x[i], 12582912.0f)) - 0x4B400000u);
        qi[i] = min(max(r, ilo), 127);
      }
#pragma unroll
      for (int w = 0; w < 8; ++w)
        out[w] = __byte_perm(__byte_perm(qi[4 * w], qi[4 * w + 1], 0x0040), __byte_perm(qi[4 * w + 2], qi[4 * w + 3], 0x0040),
                             0x5410);
      return;
    }
  }
#pragma unroll
  for (int w = 0; w < 8; ++w) {
    float ss[4], qq[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const float mi = m[4 * w + j];
      float x;
      if (flavor == kBnb) {
        ss[j] = s == 0.0f ? 0.0f : __fmul_rn(div_full(mi, s), 127.0f);
        x = ss[j];
      } else {
        ss[j] = div_full(mi, s);
        x = round_dt<CDT>(ss[j]);
      }
      qq[j] = rintf(x);
    }
    if (sr) sr_int_xn<4>(ss, qq, lo, 127.0f, key, off0 + 4 * w);
    uint32_t qb[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) qb[j] = __float_as_uint(__fadd_rn(fminf(fmaxf(qq[j], lo), 127.0f), 12582912.0f));
    out[w] = __byte_perm(__byte_perm(qb[0], qb[1], 0x0040), __byte_perm(qb[2], qb[3], 0x0040), 0x5410);
  }
}

// FP8 codes for Quanto qfloat8 (_triton_quanto_lora.py:124-168): s = v / scale;
// round to nearest: fp8(clamp(dtype(s))); stochastic: on clamp(s).
template <bool E4M3, int CDT>
__device__ __forceinline__ void quanto_fp8_encode32(const float (&m)[32], float s, float limit, bool sr,
                                                    const PhiloxKey& key, uint64_t off0, uint32_t (&out)[8]) {
#pragma unroll
  for (int w8 = 0; w8 < 4; ++w8) {
    float x[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const float q = div_full(m[8 * w8 + j], s);
      x[j] = fminf(fmaxf(sr ? q : round_dt<CDT>(q), -limit), limit);
    }
    if (sr) {
      uint32_t wd[2];
      sr_fp8xn<E4M3, 8>(x, limit, key, off0 + 8 * w8, wd);
      out[2 * w8] = wd[0];
      out[2 * w8 + 1] = wd[1];
    } else {
      out[2 * w8] = enc_fp8x4<E4M3>(x[0], x[1], x[2], x[3]);
      out[2 * w8 + 1] = enc_fp8x4<E4M3>(x[4], x[5], x[6], x[7]);
    }
  }
}

// bitsandbytes decode + merge of 32 columns (_triton_bnb8_lora.py:20-81), fp16:
// base = f16(f16(cb / 127) * f16(SCB)), merged = f16(clamp(base + acc * s, +-65504)).
// `cb / 127.0` is an IEEE division; for every int8 code f16(cb * fp32(1 / 127))
// equals f16(cb / 127) (all 256 codes checked), so the decode multiplies.
__device__ __forceinline__ void bnb8_merged(const uint32_t (&wv)[8], const float (&acc)[32], float s_in,
                                            float strength, float (&merged)[32]) {
  const float s16 = f16r(s_in);
  const float inv127 = __frcp_rn(127.0f);
#pragma unroll
  for (int i = 0; i < 32; ++i) {
    const float qv = static_cast<float>(static_cast<int8_t>(byte_of(wv, i)));
    const float base = f16r(__fmul_rn(f16r(__fmul_rn(qv, inv127)), s16));
    merged[i] = fminf(fmaxf(fmaf(acc[i], strength, base), -65504.0f), 65504.0f);
  }
#pragma unroll
  for (int i = 0; i < 32; i += 2) f16r2(merged[i], merged[i + 1]);
}

// INT8 `base * scale` (_triton_int8_lora.py:80) with one operand bf16 and the
// other fp16 runs in fp16: Triton converts both operands to fp16 and rounds the
// product to fp16 (semantic.computation_type_impl). For fp16 factors with a
// bf16 scale the scale is first rounded to fp16 (int8_f16_scale); for bf16
// factors with an fp16 scale the product is rounded to fp16 before the bf16
// cast (int8_half_product). q - zp is exact in fp16 either way.
template <int CDT>
__device__ __forceinline__ bool int8_f16_scale(int scale_dt) {
  return CDT == kF16 && scale_dt == kBF16;
}

template <int CDT>
__device__ __forceinline__ void int8_half_product(int scale_dt, float (&m)[32]) {
  if constexpr (CDT == kBF16) {
    if (scale_dt == kF16) {
#pragma unroll
      for (int i = 0; i < 32; i += 2) f16r2(m[i], m[i + 1]);
    }
  }
}

// Decode + merge 32 columns of an FP8/INT8 row chunk. Columns >= N are
// garbage and excluded by the callers.
template <int FMT, int CDT>
__device__ __forceinline__ void affine_merged(const DevWeight& W, const RowCtx& c, int k,
                                              const float (&acc)[32], const float* scale_in,
                                              const int* zp_in, float (&merged)[32]) {
  uint32_t wv[8];
  load_chunks32(c, k, wv);
  if constexpr (CDT == kF32 && flavor_of(FMT) == kTorchao) {
    // fp32 compute: fma(q - zp, scale, acc * strength) (see fp8_merged_pk).
    if constexpr (base_fmt(FMT) == PIPER_FMT_INT8) {
#pragma unroll
      for (int i = 0; i < 32; ++i) {
        const float qz = __fsub_rn(static_cast<float>(static_cast<int8_t>(byte_of(wv, i))), static_cast<float>(zp_in[i]));
        merged[i] = fmaf(qz, scale_in[i], __fmul_rn(acc[i], W.strength));
      }
    } else {
#pragma unroll
      for (int w = 0; w < 8; ++w) {
        float f[4];
        dec_fp8x4<base_fmt(FMT) == PIPER_FMT_FP8_E4M3>(wv[w], f);
#pragma unroll
        for (int j = 0; j < 4; ++j)
          merged[4 * w + j] = fmaf(f[j], scale_in[4 * w + j], __fmul_rn(acc[4 * w + j], W.strength));
      }
    }
  } else {
    if constexpr (base_fmt(FMT) == PIPER_FMT_INT8) {
      const bool f16_scale = int8_f16_scale<CDT>(W.scale_dt);
#pragma unroll
      for (int i = 0; i < 32; ++i) {
        const float qv = static_cast<float>(static_cast<int8_t>(byte_of(wv, i)));
        // q - zp is an integer in [-255, 255]: exact in bf16 / fp16.
        const float s = f16_scale ? f16r(scale_in[i]) : scale_in[i];
        merged[i] = __fmul_rn(__fsub_rn(qv, static_cast<float>(zp_in[i])), s);
      }
      int8_half_product<CDT>(W.scale_dt, merged);
    } else {
#pragma unroll
      for (int w = 0; w < 8; ++w) {
        float f[4];
        dec_fp8x4<base_fmt(FMT) == PIPER_FMT_FP8_E4M3>(wv[w], f);
#pragma unroll
        for (int j = 0; j < 4; ++j) merged[4 * w + j] = __fmul_rn(f[j], scale_in[4 * w + j]);
      }
    }
#pragma unroll
    for (int i = 0; i < 32; i += 2) round_dt2<CDT>(merged[i], merged[i + 1]);
#pragma unroll
    for (int i = 0; i < 32; ++i) merged[i] = fmaf(acc[i], W.strength, merged[i]);
#pragma unroll
    for (int i = 0; i < 32; i += 2) round_dt2<CDT>(merged[i], merged[i + 1]);
  }
}

// affine_merged for a chunk inside one quantization block (one scale / zero point).
template <int FMT, int CDT>
__device__ __forceinline__ void affine_merged_u(const DevWeight& W, const RowCtx& c, int k,
                                                const float (&acc)[32], float s_in, int z_in,
                                                float (&merged)[32]) {
  uint32_t wv[8];
  load_chunks32(c, k, wv);
  if constexpr (CDT == kF32 && flavor_of(FMT) == kTorchao) {
    // fp32 compute: fma(q - zp, scale, acc * strength) (see fp8_merged_pk).
    if constexpr (base_fmt(FMT) == PIPER_FMT_INT8) {
      const float zf = static_cast<float>(z_in);
#pragma unroll
      for (int i = 0; i < 32; ++i) {
        const float qz = __fsub_rn(static_cast<float>(static_cast<int8_t>(byte_of(wv, i))), zf);
        merged[i] = fmaf(qz, s_in, __fmul_rn(acc[i], W.strength));
      }
    } else {
#pragma unroll
      for (int w = 0; w < 8; ++w) {
        float f[4];
        dec_fp8x4<base_fmt(FMT) == PIPER_FMT_FP8_E4M3>(wv[w], f);
#pragma unroll
        for (int j = 0; j < 4; ++j) merged[4 * w + j] = fmaf(f[j], s_in, __fmul_rn(acc[4 * w + j], W.strength));
      }
    }
  } else {
    if constexpr (base_fmt(FMT) == PIPER_FMT_INT8) {
      if constexpr (flavor_of(FMT) == kBnb) {
        bnb8_merged(wv, acc, s_in, W.strength, merged);
        return;
      }
      const float zf = static_cast<float>(z_in);
      const float s = int8_f16_scale<CDT>(W.scale_dt) ? f16r(s_in) : s_in;
#pragma unroll
      for (int i = 0; i < 32; ++i) {
        const float qv = static_cast<float>(static_cast<int8_t>(byte_of(wv, i)));
        merged[i] = __fmul_rn(__fsub_rn(qv, zf), s);
      }
      int8_half_product<CDT>(W.scale_dt, merged);
    } else {
#pragma unroll
      for (int w = 0; w < 8; ++w) {
        float f[4];
        dec_fp8x4<base_fmt(FMT) == PIPER_FMT_FP8_E4M3>(wv[w], f);
#pragma unroll
        for (int j = 0; j < 4; ++j) merged[4 * w + j] = __fmul_rn(f[j], s_in);
      }
    }
#pragma unroll
    for (int i = 0; i < 32; i += 2) round_dt2<CDT>(merged[i], merged[i + 1]);
    if constexpr (flavor_of(FMT) == kQuanto) {
      if (s_in == 0.0f) {
        // where(scale == 0, 0, q * scale): Quanto's FP8 codes are NaN under a zero scale (:90-94).
#pragma unroll
        for (int i = 0; i < 32; ++i) merged[i] = 0.0f;
      }
    }
    const float st = W.strength;
#pragma unroll
    for (int i = 0; i < 32; ++i) merged[i] = fmaf(acc[i], st, merged[i]);
#pragma unroll
    for (int i = 0; i < 32; i += 2) round_dt2<CDT>(merged[i], merged[i + 1]);
  }
}

// Stochastic FP8 codes of 32 values: clamp(m / s) (div.full) rounded with
// eight Philox counters per batch, so eight multiply chains are in flight.
template <bool E4M3>
__device__ __forceinline__ void fp8_encode_sr(const float (&m)[32], float s, float limit, const PhiloxKey& key,
                                              uint64_t off0, uint32_t (&out)[8]) {
#pragma unroll
  for (int w8 = 0; w8 < 4; ++w8) {
    float x[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) x[j] = fminf(fmaxf(div_full(m[8 * w8 + j], s), -limit), limit);
    uint32_t wd[2];
    sr_fp8xn<E4M3, 8>(x, limit, key, off0 + 8 * w8, wd);
    out[2 * w8] = wd[0];
    out[2 * w8 + 1] = wd[1];
  }
}

// FP8 codes of 32 merged values for one scale `s` (round to nearest).
// The reference quotient is div.full(x, s); x * RN(1/s) is used unless some
// element lands within 4 ulp of an FP8 rounding boundary.
template <bool E4M3>
__device__ __forceinline__ void fp8_encode_rtn(const float (&m)[32], float s, float limit, uint32_t (&out)[8]) {
  const float inv = __frcp_rn(s);
  float q[32];
  bool near = false;
#pragma unroll
  for (int i = 0; i < 32; ++i) {
    q[i] = __fmul_rn(m[i], inv);
    near |= near_fp8_edge<E4M3>(q[i]);
  }
  if (near) {
#pragma unroll
    for (int i = 0; i < 32; ++i) q[i] = div_full(m[i], s);
  }
#pragma unroll
  for (int i = 0; i < 32; ++i) q[i] = fminf(fmaxf(q[i], -limit), limit);
#pragma unroll
  for (int w = 0; w < 8; ++w) out[w] = enc_fp8x4<E4M3>(q[4 * w], q[4 * w + 1], q[4 * w + 2], q[4 * w + 3]);
}

// ------------------------------------------- packed per-row FP8 (fused pass)
// Decode + merge of 32 FP8 codes of one row (TorchAO scaled FP8,
// _triton_float8_lora.py:70-94): base = compute(fp8 * scale), merged =
// fma(acc, strength, base) in fp32, two elements per packed instruction.
// ROUND rounds the merged values to the compute dtype; the row-maxima sweep
// skips it, since rounding is monotone: max |compute(x)| = compute(max |x|).
template <bool E4M3, int CDT, bool ROUND>
__device__ __forceinline__ void fp8_merged_pk(const uint32_t (&wv)[8], const float (&acc)[32], float s_in,
                                              float strength, float (&m)[32]) {
  const float2 s2 = make_float2(s_in, s_in);
  const float2 st2 = make_float2(strength, strength);
  if constexpr (CDT == kF32) {
    // fp32 compute: the reference's `base = q * scale; merged = base + acc *
    // strength` has no cast in between, and its compilation contracts the
    // first product into the add: fma(q, scale, acc * strength).
#pragma unroll
    for (int w = 0; w < 8; ++w) {
      float f[4];
      dec_fp8x4<E4M3>(wv[w], f);
#pragma unroll
      for (int j = 0; j < 4; ++j) m[4 * w + j] = fmaf(f[j], s_in, __fmul_rn(acc[4 * w + j], strength));
    }
  } else {
#pragma unroll
    for (int w = 0; w < 8; ++w) {
      float f[4];
      dec_fp8x4<E4M3>(wv[w], f);
      float2 b0 = __fmul2_rn(make_float2(f[0], f[1]), s2);
      float2 b1 = __fmul2_rn(make_float2(f[2], f[3]), s2);
      round_dt2<CDT>(b0.x, b0.y);
      round_dt2<CDT>(b1.x, b1.y);
      float2 m0 = __ffma2_rn(make_float2(acc[4 * w], acc[4 * w + 1]), st2, b0);
      float2 m1 = __ffma2_rn(make_float2(acc[4 * w + 2], acc[4 * w + 3]), st2, b1);
      if constexpr (ROUND) {
        round_dt2<CDT>(m0.x, m0.y);
        round_dt2<CDT>(m1.x, m1.y);
      }
      m[4 * w] = m0.x;
      m[4 * w + 1] = m0.y;
      m[4 * w + 2] = m1.x;
      m[4 * w + 3] = m1.y;
    }
  }
}

// Decode + merge of 32 INT8 codes of one row (TorchAO affine INT8,
// _triton_int8_lora.py:70-94): base = compute((q - zp) * scale) with the
// mixed bf16 / fp16 rules of int8_f16_scale / int8_half_product, merged =
// fma(acc, strength, base), two elements per packed instruction. q - zp is
// exact: the code byte with its sign bit flipped, placed under the exponent of
// 2^23, is the float 2^23 + q + 128, and subtracting 2^23 + 128 + zp leaves
// q - zp. ROUND as in fp8_merged_pk.
template <int CDT, bool ROUND>
__device__ __forceinline__ void int8_merged_pk(const uint32_t (&wv)[8], const float (&acc)[32], float s_in, int z_in,
                                               int scale_dt, float strength, float (&m)[32]) {
  const float off = -(8388736.0f + static_cast<float>(z_in));
  const float sc = int8_f16_scale<CDT>(scale_dt) ? f16r(s_in) : s_in;
  const bool half_product = CDT == kBF16 && scale_dt == kF16;
  const float2 off2 = make_float2(off, off);
  const float2 s2 = make_float2(sc, sc);
  const float2 st2 = make_float2(strength, strength);
  if constexpr (CDT == kF32) {
    // fp32 compute: fma(q - zp, scale, acc * strength), as in fp8_merged_pk.
#pragma unroll
    for (int i = 0; i < 32; ++i) {
      const float qz = __fsub_rn(static_cast<float>(static_cast<int8_t>(byte_of(wv, i))), static_cast<float>(z_in));
      m[i] = fmaf(qz, sc, __fmul_rn(acc[i], strength));
    }
  } else {
#pragma unroll
    for (int w = 0; w < 8; ++w) {
      const uint32_t x = wv[w] ^ 0x80808080u;
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        const float2 raw = make_float2(__uint_as_float(__byte_perm(x, 0x4B000000u, 0x7540u + 2u * h)),
                                       __uint_as_float(__byte_perm(x, 0x4B000000u, 0x7541u + 2u * h)));
        float2 b = __fmul2_rn(__fadd2_rn(raw, off2), s2);
        if (half_product) f16r2(b.x, b.y);
        round_dt2<CDT>(b.x, b.y);
        float2 r = __ffma2_rn(make_float2(acc[4 * w + 2 * h], acc[4 * w + 2 * h + 1]), st2, b);
        if constexpr (ROUND) round_dt2<CDT>(r.x, r.y);
        m[4 * w + 2 * h] = r.x;
        m[4 * w + 2 * h + 1] = r.y;
      }
    }
  }
}

// Round-to-nearest INT8 codes of 32 merged values of an all-finite row
// (_quantize_kernel, _triton_int8_lora.py:189-236): x = scale_dtype(m *
// scale_dtype(1 / scale)), q = rint(x) + zp clamped to [qmin, qmax]. In an
// all-finite row |x| <= 128 or so, far below 2^22, so rint(x) is the sum
// x + 1.5 * 2^23 (exact in fp32), whose bits are 0x4B400000 + rint(x); after
// the clamp the zero point is added to those bits, and their low byte is q.
__device__ __forceinline__ void int8_encode_rtn_finite(const float (&m)[32], const Int8Q& q, int qmin, int qmax,
                                                       int scale_dt, uint32_t (&out)[8]) {
  const float inv = round_dt_rt(div_full(1.0f, q.scale), scale_dt);
  const float2 magic2 = make_float2(12582912.0f, 12582912.0f);
  // rint(x) is clamped to [qmin - zp, qmax - zp] in the float domain and the
  // zero point is added to the bits.
  const float lo = 12582912.0f + static_cast<float>(qmin - q.zp);
  const float hi = 12582912.0f + static_cast<float>(qmax - q.zp);
  const uint32_t zpu = static_cast<uint32_t>(q.zp);
#pragma unroll
  for (int w = 0; w < 8; ++w) {
    uint32_t qb[4];
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      // Scalar products: with fp32 scales nothing separates the product from
      // the magic add, and a packed product followed by the packed add was
      // measured to round as one fused multiply-add (codes off by one at
      // x = n + 1/2); __fmul_rn is never fused.
      float2 x = make_float2(__fmul_rn(m[4 * w + 2 * h], inv), __fmul_rn(m[4 * w + 2 * h + 1], inv));
      round_rt2(x.x, x.y, scale_dt);
      const float2 y = __fadd2_rn(x, magic2);
      qb[2 * h] = __float_as_uint(fminf(fmaxf(y.x, lo), hi)) + zpu;
      qb[2 * h + 1] = __float_as_uint(fminf(fmaxf(y.y, lo), hi)) + zpu;
    }
    out[w] = __byte_perm(__byte_perm(qb[0], qb[1], 0x0040u), __byte_perm(qb[2], qb[3], 0x0040u), 0x5410u);
  }
}

// Round-to-nearest FP8 codes of 32 merged values of a row whose values are all
// finite (no NaN or infinity in the row): q = div.full(m, s) as the reference
// divides, then the satfinite RTNE conversion. |q| <= amax / s <= limit *
// (1 + 2^-8) there, which rounds to the largest finite code exactly as the
// reference's clamp to [-limit, limit] followed by RTNE does.
template <bool E4M3>
__device__ __forceinline__ void fp8_encode_rtn_finite(const float (&m)[32], float s, uint32_t (&out)[8]) {
  float q[32];
#pragma unroll
  for (int i = 0; i < 32; ++i) q[i] = div_full(m[i], s);
#pragma unroll
  for (int w = 0; w < 8; ++w) out[w] = enc_fp8x4<E4M3>(q[4 * w], q[4 * w + 1], q[4 * w + 2], q[4 * w + 3]);
}

// Stochastic FP8 codes of 32 merged values of an all-finite row: q =
// div.full(m, s), eight Philox counters per batch (sr_fp8xn_finite).
template <bool E4M3>
__device__ __forceinline__ void fp8_encode_sr_finite(const float (&m)[32], float s, const PhiloxKey& key,
                                                     uint64_t off0, uint32_t (&out)[8]) {
#pragma unroll
  for (int w8 = 0; w8 < 4; ++w8) {
    float x[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) x[j] = div_full(m[8 * w8 + j], s);
    uint32_t wd[2];
    sr_fp8xn_finite<E4M3, 8>(x, key, off0 + 8 * w8, wd);
    out[2 * w8] = wd[0];
    out[2 * w8 + 1] = wd[1];
  }
}

// Stored scale of an FP8 / INT8 weight: TorchAO FP8 scales are fp32; INT8,
// bitsandbytes and Quanto scales have the weight's scale dtype.
template <int FMT>
__device__ __forceinline__ float load_scale(const DevWeight& W, int64_t i) {
  if constexpr (base_fmt(FMT) != PIPER_FMT_INT8 && flavor_of(FMT) == kTorchao)
    return reinterpret_cast<const float*>(W.scale)[i];
  else
    return load_scale_dt(W.scale, i, W.scale_dt);
}
template <int FMT>
__device__ __forceinline__ void store_scale(const DevWeight& W, int64_t i, float v) {
  if constexpr (base_fmt(FMT) != PIPER_FMT_INT8 && flavor_of(FMT) == kTorchao)
    reinterpret_cast<float*>(W.scale)[i] = v;
  else
    store_scale_dt(W.scale, i, W.scale_dt, v);
}

// Quantization parameters of the quantization block a thread is working in,
// kept in registers while consecutive chunks stay in that block (per-row and
// per-tensor layouts: for the whole work item), so the workspace and scale
// loads are issued once per block rather than once per 32 columns.
struct QpCache {
  int qp = -1;
  float s_in = 1.0f;   // input scale (ENCODE: saved by the REDUCE pass)
  int z_in = 0;        // input zero point
  float qmax = 0.0f;   // ENCODE: reduced max(|x|) or max(x, 0)
  float nmin = 0.0f;   // ENCODE (INT8): reduced -min(x, 0)
};

template <int FMT, int PASS>
__device__ __forceinline__ void qp_load(const DevWeight& W, int qp, QpCache& q) {
  if (q.qp == qp) return;
  q.qp = qp;
  if (PASS == kEncode) {
    q.s_in = W.old_scale[qp];
    q.z_in = W.old_zp[qp];
    q.qmax = __uint_as_float(W.qmax[qp]);
    if (base_fmt(FMT) == PIPER_FMT_INT8) q.nmin = __uint_as_float(W.qmin[qp]);
  } else if (base_fmt(FMT) == PIPER_FMT_INT8) {
    q.s_in = load_scale_dt(W.scale, qp, W.scale_dt);
    q.z_in = W.zp != nullptr ? static_cast<int>(W.zp[qp]) : 0;
  } else {
    q.s_in = load_scale<FMT>(W, qp);
  }
}

// Input scale / zero point of each column of a chunk.
template <int FMT, int PASS>
__device__ __forceinline__ void affine_inputs(const DevWeight& W, const RowCtx& c, int col,
                                              float (&scale_in)[32], int (&zp_in)[32], QpCache& qc) {
  if (!c.valid) {
#pragma unroll
    for (int i = 0; i < 32; ++i) {
      scale_in[i] = 1.0f;
      zp_in[i] = 0;
    }
    return;
  }
  const bool uniform = W.nq_row == 0 || W.group >= 32;
  if (uniform && (W.nq_row == 0 || (col % W.group) + 32 <= W.group)) {
    qp_load<FMT, PASS>(W, qparam_index(W, c.row, col), qc);
#pragma unroll
    for (int i = 0; i < 32; ++i) {
      scale_in[i] = qc.s_in;
      zp_in[i] = qc.z_in;
    }
    return;
  }
#pragma unroll
  for (int i = 0; i < 32; ++i) {
    const int cc = min(col + i, W.N - 1);
    const int qp = qparam_index(W, c.row, cc);
    if (PASS == kEncode) {
      scale_in[i] = W.old_scale[qp];
      zp_in[i] = W.old_zp[qp];
    } else if (base_fmt(FMT) == PIPER_FMT_INT8) {
      scale_in[i] = c.valid ? load_scale_dt(W.scale, qp, W.scale_dt) : 1.0f;
      zp_in[i] = (W.zp != nullptr && c.valid) ? static_cast<int>(W.zp[qp]) : 0;
    } else {
      scale_in[i] = c.valid ? reinterpret_cast<const float*>(W.scale)[qp] : 1.0f;
      zp_in[i] = 0;
    }
  }
}

// ================================================ bitsandbytes 4-bit epilogue
// One 64-value block of _merge_quantize_kernel (_triton_bnb4_lora.py:163-313):
// base = compute(code[q] * absmax) (nested absmax: nested_code[c] * nested
// absmax + offset, one fused multiply-add), merged = compute(base + acc * s),
// new absmax = max |merged|, x = clamp(merged / absmax, -1, 1) encoded to the
// nearest table entry (NF4, ties to the lower index; _nearest_sorted_code
// :29-50) or by the FP4 thresholds (_nearest_fp4_code :53-75), or
// stochastically (_stochastic_sorted_code, _stochastic_fp4_code :135-160).
// Per-lane tables (code[lane & 15], FP4 level values) are read with full-warp
// shuffles, so the whole warp runs these helpers together and every lookup is
// evaluated unconditionally (never under a per-lane condition).
__device__ __forceinline__ float lane_lut(float lut, int idx) { return __shfl_sync(0xFFFFFFFFu, lut, idx); }

__device__ __forceinline__ int fp4_level_to_store(int level) {
  return level < 2 ? level : (level < 4 ? level + 4 : (level < 6 ? level : level - 4));
}

// Decode + merge of 32 values (16 code bytes) of one 64-value block.
template <int CDT>
__device__ __forceinline__ void bnb4_merged32(const uint32_t (&wv)[4], float scale, float lut, float strength,
                                              const float (&acc)[32], float (&m)[32]) {
#pragma unroll
  for (int j = 0; j < 16; ++j) {
    const uint32_t byte = (wv[j >> 2] >> ((j & 3) * 8)) & 0xFFu;
    m[2 * j] = lane_lut(lut, static_cast<int>(byte >> 4));
    m[2 * j + 1] = lane_lut(lut, static_cast<int>(byte & 15u));
  }
  if constexpr (CDT == kF32) {
    // fp32 compute: fma(code, scale, acc * strength) (see fp8_merged_pk;
    // _triton_bnb4_lora.py:247-254).
#pragma unroll
    for (int i = 0; i < 32; ++i) m[i] = fmaf(m[i], scale, __fmul_rn(acc[i], strength));
  } else {
#pragma unroll
    for (int i = 0; i < 32; ++i) m[i] = __fmul_rn(m[i], scale);
#pragma unroll
    for (int i = 0; i < 32; i += 2) round_dt2<CDT>(m[i], m[i + 1]);
#pragma unroll
    for (int i = 0; i < 32; ++i) m[i] = fmaf(acc[i], strength, m[i]);
#pragma unroll
    for (int i = 0; i < 32; i += 2) round_dt2<CDT>(m[i], m[i + 1]);
  }
}

// NF4 index of the reference's binary search (_nearest_sorted_code :29-50,
// _stochastic_sorted_code): ui = first index in [0, 15] whose entry is not
// below v. With a non-decreasing table (`tbl`, whole table in registers) that is
// the count of tbl[0..14] below v: 15 independent compares.
template <bool SR>
__device__ __forceinline__ int nf4_code_sorted(float v, float lut, const float (&tbl)[16], const PhiloxKey& key,
                                               uint64_t off) {
  int ui = 0;
#pragma unroll
  for (int j = 0; j < 15; ++j) ui += tbl[j] < v ? 1 : 0;
  const int li = max(ui - 1, 0);
  const float up = lane_lut(lut, ui);
  const float lo = lane_lut(lut, li);
  int code = fabsf(__fsub_rn(v, lo)) <= fabsf(__fsub_rn(v, up)) ? li : ui;
  if constexpr (SR) {
    const bool exact = up == v;
    const int li2 = exact ? ui : li;
    const float lo2 = exact ? up : lo;
    const float width = __fsub_rn(up, lo2);
    const float prob = width > 0.0f ? div_full(__fsub_rn(v, lo2), width) : 0.0f;
    const int chosen = philox_uniform(key, off) < prob ? ui : li2;
    const bool interior = (v > tbl[0]) & (v < tbl[15]) & !exact;
    code = interior ? chosen : code;
  }
  return code;
}

// The same with the table read by the 4-step binary search (any table order).
__device__ __noinline__ int nf4_code_search(float v, const float* __restrict__ code16, bool sr, const PhiloxKey& key,
                                            uint64_t off) {
  int ui = 0, high = 15;
  for (int st = 0; st < 4; ++st) {
    const int mid = (ui + high) >> 1;
    const bool right = __ldg(code16 + mid) < v;
    ui = right ? mid + 1 : ui;
    high = right ? high : mid;
  }
  const int li = max(ui - 1, 0);
  const float up = __ldg(code16 + ui);
  const float lo = __ldg(code16 + li);
  int code = fabsf(__fsub_rn(v, lo)) <= fabsf(__fsub_rn(v, up)) ? li : ui;
  if (sr) {
    const bool exact = up == v;
    const int li2 = exact ? ui : li;
    const float lo2 = __ldg(code16 + li2);
    const float width = __fsub_rn(up, lo2);
    const float prob = width > 0.0f ? div_full(__fsub_rn(v, lo2), width) : 0.0f;
    const int chosen = philox_uniform(key, off) < prob ? ui : li2;
    const bool interior = (v > __ldg(code16)) & (v < __ldg(code16 + 15)) & !exact;
    code = interior ? chosen : code;
  }
  return code;
}

// FP4 code (_nearest_fp4_code :53-75, _stochastic_fp4_code :135-160); `lvl`
// holds the FP4 level value of lane & 7.
template <bool SR>
__device__ __forceinline__ int fp4_code(float v, float lvl, const PhiloxKey& key, uint64_t off) {
  const float mag = fabsf(v);
  const int level = (mag > 0.0026041667442768812f) + (mag > 0.08593750256113708f) + (mag > 0.2083333358168602f) +
                    (mag > 0.2916666716337204f) + (mag > 0.4166666716337204f) + (mag > 0.5833333432674408f) +
                    (mag > 0.8333333432674408f);
  int code = fp4_level_to_store(level) + ((v < 0.0f && level != 0) ? 8 : 0);
  if constexpr (SR) {
    // _fp4_storage_to_level of the nearest code is the level itself.
    const float nearest = lane_lut(lvl, level);
    const bool down = nearest > mag;
    const int lol = down ? level - 1 : level;
    const int upl = down ? level : level + 1;
    const float lo = lane_lut(lvl, max(lol, 0));
    const float up = lane_lut(lvl, min(upl, 7));
    const float prob = up > lo ? div_full(__fsub_rn(mag, lo), __fsub_rn(up, lo)) : 0.0f;
    const int lv = philox_uniform(key, off) < prob ? upl : lol;
    const int chosen = fp4_level_to_store(lv) + ((v < 0.0f && lv != 0) ? 8 : 0);
    const bool interior = (mag > 0.0f) & (mag < 1.0f) & (prob > 0.0f);
    code = interior ? chosen : code;
  }
  return code;
}

// Codes of 32 merged values (x = clamp(m / safe, -1, 1)) into 16 bytes, first
// value of each byte in the high nibble. NF4 uses `lut` = code[lane & 15] and
// the register table; FP4 uses `lut` = its level values.
template <int FMT, bool SR>
__device__ __forceinline__ void bnb4_encode32(const float (&m)[32], float safe, float lut, const float (&tbl)[16],
                                              const PhiloxKey& key, uint64_t off0, uint32_t (&out)[4]) {
#pragma unroll
  for (int w = 0; w < 4; ++w) out[w] = 0u;
#pragma unroll
  for (int i = 0; i < 32; ++i) {
    const float v = fminf(fmaxf(div_full(m[i], safe), -1.0f), 1.0f);
    int code;
    if constexpr (FMT == PIPER_FMT_BNB4_NF4) code = nf4_code_sorted<SR>(v, lut, tbl, key, off0 + i);
    else code = fp4_code<SR>(v, lut, key, off0 + i);
    const int j = i >> 1;
    out[j >> 2] |= static_cast<uint32_t>(code & 15) << ((j & 3) * 8 + ((i & 1) ? 0 : 4));
  }
}

// Nested quantization of the new block maxima (_triton_bnb4_lora.py:316-375,
// :399-431): offset = mean of the maxima; per 256 blocks the maximum of
// |x - offset| and the nearest code of (x - offset) / maximum in the
// 256-entry table. The mean is summed in fp64 in a fixed order (kBnb4Parts
// contiguous ranges, then their partial sums in index order) and rounded once;
// the reference sums in Triton's fp32 reduction order.
constexpr int kBnb4Parts = 64;

__global__ void __launch_bounds__(256) bnb4_partial_kernel(const uint32_t* __restrict__ raw, int64_t n,
                                                           double* __restrict__ part) {
  __shared__ double red[8];
  const int64_t per = (n + gridDim.x - 1) / gridDim.x;
  const int64_t b0 = static_cast<int64_t>(blockIdx.x) * per;
  const int64_t b1 = min(n, b0 + per);
  double s = 0.0;
  for (int64_t i = b0 + threadIdx.x; i < b1; i += blockDim.x) s += static_cast<double>(__uint_as_float(raw[i]));
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) s += __shfl_down_sync(0xFFFFFFFFu, s, o);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = s;
  __syncthreads();
  if (threadIdx.x == 0) {
    double t = 0.0;
    for (int w = 0; w < 8; ++w) t += red[w];
    part[blockIdx.x] = t;
  }
}

// Every CTA folds the partial sums in the same order, so all see the same
// offset; CTA 0 stores it.
__global__ void __launch_bounds__(256) bnb4_nested_kernel(const uint32_t* __restrict__ raw, int64_t n,
                                                          const double* __restrict__ part, float* __restrict__ off,
                                                          const float* __restrict__ ncode, uint8_t* __restrict__ qabs,
                                                          float* __restrict__ nabs) {
  __shared__ float tbl[256];
  __shared__ float s_off;
  tbl[threadIdx.x] = ncode[threadIdx.x];
  if (threadIdx.x == 0) {
    double t = 0.0;
    for (int b = 0; b < kBnb4Parts; ++b) t += part[b];
    s_off = div_full(__double2float_rn(t), static_cast<float>(n));  // `/ TOTAL_VALUES` (runtime divisor: Triton's fp32 division)
    if (blockIdx.x == 0) *off = s_off;
  }
  __syncthreads();
  const int lane = threadIdx.x & 31;
  const int64_t w = static_cast<int64_t>(blockIdx.x) * 8 + (threadIdx.x >> 5);
  const int64_t nblk = (n + 255) / 256;
  if (w >= nblk) return;
  const float o = s_off;
  float cen[8];
  float mx = 0.0f;
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    const int64_t i = w * 256 + lane + 32 * j;
    cen[j] = i < n ? __fsub_rn(__uint_as_float(raw[i]), o) : 0.0f;
    mx = fmaxf(mx, fabsf(cen[j]));
  }
#pragma unroll
  for (int x = 16; x > 0; x >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xFFFFFFFFu, mx, x));
  const float safe = mx == 0.0f ? 1.0f : mx;
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    const int64_t i = w * 256 + lane + 32 * j;
    if (i >= n) continue;
    const float v = fminf(fmaxf(div_full(cen[j], safe), -1.0f), 1.0f);
    int low = 0, high = 255;
#pragma unroll
    for (int st = 0; st < 8; ++st) {
      const int mid = (low + high) >> 1;
      const bool right = tbl[mid] < v;
      low = right ? mid + 1 : low;
      high = right ? high : mid;
    }
    const int li = max(low - 1, 0);
    qabs[i] = static_cast<uint8_t>(fabsf(__fsub_rn(v, tbl[li])) <= fabsf(__fsub_rn(v, tbl[low])) ? li : low);
  }
  if (lane == 0) nabs[w] = mx;
}

// ====================================================== Quanto last-axis scales
// One scale per column (_triton_quanto_lora.py:202-217 with dim=0). REDUCE: each
// column's max |merged| over a warp's 32 rows by one warp reduction, then one
// atomic per column; row 0 saves the input scales. ENCODE: the column scales
// dtype(amax * fp32(1 / qmax)) and the codes of _quantize_qbytes_kernel
// (:107-168). The whole warp runs this together (warp reductions).
template <int FMT, int PASS, int CDT>
__device__ __forceinline__ void quanto_column_chunk(const DevWeight& W, const RowCtx& c, int k, int col, int nvalid,
                                                    const float (&acc)[32], int lane, const PhiloxKey& key) {
  constexpr bool kInt8 = base_fmt(FMT) == PIPER_FMT_INT8;
  constexpr bool kE4 = base_fmt(FMT) == PIPER_FMT_FP8_E4M3;
  constexpr float kQmax = kInt8 ? 127.0f : (kE4 ? 448.0f : 57344.0f);
  uint32_t wv[8];
  load_chunks32(c, k, wv);
  float s_in[32];
#pragma unroll
  for (int i = 0; i < 32; ++i) {
    const int cc = min(col + i, W.N - 1);
    s_in[i] = PASS == kReduce ? load_scale<FMT>(W, cc) : W.old_scale[cc];
  }
  float m[32];
  if constexpr (kInt8) {
#pragma unroll
    for (int i = 0; i < 32; ++i) m[i] = static_cast<float>(static_cast<int8_t>(byte_of(wv, i)));
  } else {
#pragma unroll
    for (int w = 0; w < 8; ++w) {
      float f[4];
      dec_fp8x4<kE4>(wv[w], f);
#pragma unroll
      for (int j = 0; j < 4; ++j) m[4 * w + j] = f[j];
    }
  }
#pragma unroll
  for (int i = 0; i < 32; ++i) m[i] = s_in[i] == 0.0f ? 0.0f : __fmul_rn(m[i], s_in[i]);
#pragma unroll
  for (int i = 0; i < 32; i += 2) round_dt2<CDT>(m[i], m[i + 1]);
#pragma unroll
  for (int i = 0; i < 32; ++i) m[i] = fmaf(acc[i], W.strength, m[i]);
#pragma unroll
  for (int i = 0; i < 32; i += 2) round_dt2<CDT>(m[i], m[i + 1]);
  if constexpr (PASS == kReduce) {
    uint32_t mine = 0u;
#pragma unroll
    for (int i = 0; i < 32; ++i) {
      const uint32_t v = (c.valid && i < nvalid) ? __float_as_uint(fabsf(m[i])) : 0u;
      const uint32_t r = __reduce_max_sync(0xFFFFFFFFu, v);  // non-negative floats order like their bits
      mine = lane == i ? r : mine;
    }
    if (lane < nvalid && mine != 0u) atomicMax(&W.qmax[col + lane], mine);
    if (c.valid && c.row == 0) {
      for (int i = 0; i < nvalid; ++i) W.old_scale[col + i] = s_in[i];
    }
  } else {
    uint32_t out[8] = {0u, 0u, 0u, 0u, 0u, 0u, 0u, 0u};
    if (c.valid) {
      const uint64_t off0 = W.offset_base + static_cast<uint64_t>(c.row) * static_cast<uint64_t>(W.N) + col;
      const bool sr = (W.flags & PIPER_FLAG_STOCHASTIC) != 0u;
      for (int i = 0; i < nvalid; ++i) {
        const float s = flavor_scale<CDT>(kQuanto, __uint_as_float(W.qmax[col + i]), kQmax);
        if (c.row == 0) store_scale<FMT>(W, col + i, s);
        const float ss = div_full(m[i], s);
        uint32_t code;
        if constexpr (kInt8) {
          float qf = rintf(round_dt<CDT>(ss));
          if (sr) qf = sr_int(ss, qf, -128.0f, 127.0f, key, off0 + i);
          qf = fminf(fmaxf(qf, -128.0f), 127.0f);
          code = static_cast<uint32_t>(static_cast<int32_t>(qf)) & 0xFFu;
        } else {
          code = sr ? sr_fp8<kE4>(fminf(fmaxf(ss, -kQmax), kQmax), kQmax, key, off0 + i)
                    : enc_fp8<kE4>(fminf(fmaxf(round_dt<CDT>(ss), -kQmax), kQmax));
        }
        out[i >> 2] |= code << ((i & 3) * 8);
      }
    }
    store_chunks32(c, k, out);
  }
}

// ============================================================ GGUF epilogue
__device__ __forceinline__ float roundf_away(float x) {  // gguf.quants.np_roundf
  const float a = fabsf(x);
  const float fl = floorf(a);
  const float b = __fadd_rn(fl, floorf(__fmul_rn(2.0f, __fsub_rn(a, fl))));
  return x > 0.0f ? b : (x < 0.0f ? -b : 0.0f * x);
}

// Signed byte b of `w` (xor 0x80 already applied) as a float, exactly:
// 2^23 + (b ^ 0x80) assembled by a byte permute, minus 2^23 + 128.
__device__ __forceinline__ float sbyte_to_float(uint32_t wx, int b) {
  return __uint_as_float(__byte_perm(wx, 0x4B000000u, 0x7540u + static_cast<uint32_t>(b))) - 8388736.0f;
}
// Byte b of `w` (a value 0..15) minus 8 as a float, exactly.
__device__ __forceinline__ float nibble_to_float_m8(uint32_t w, int b) {
  return __uint_as_float(__byte_perm(w, 0x4B000000u, 0x7540u + static_cast<uint32_t>(b))) - 8388616.0f;
}
// Low byte of an integer-valued float in [-2^22, 2^22] (two's complement), exactly.
__device__ __forceinline__ uint32_t float_int_bits(float q) { return __float_as_uint(q + 12582912.0f); }
__device__ __forceinline__ uint32_t pack_low_bytes(uint32_t a, uint32_t b, uint32_t c, uint32_t d) {
  return __byte_perm(__byte_perm(a, b, 0x0040u), __byte_perm(c, d, 0x0040u), 0x5410u);
}

// One GGUF block (32 elements) of a tile row. Blocks start at even byte
// offsets, so a block is read and written as the 4-byte words that cover it
// (9 for Q8_0, 5 for Q4_0); the 2 bytes of a neighbouring block that share a
// word are written back unchanged (this thread owns the whole row segment).
template <int FMT, int CDT>
__device__ __forceinline__ void gguf_chunk(const DevWeight& W, const RowCtx& c, int k,
                                           const float (&acc)[32]) {
  constexpr bool kQ8 = FMT == PIPER_FMT_GGUF_Q8_0;
  constexpr int kTS = kQ8 ? 34 : 18;
  constexpr int kWords = kQ8 ? 9 : 5;
  constexpr int kCodeWords = kQ8 ? 8 : 4;
  const int byte0 = kTS * k;
  const bool odd = (byte0 & 2) != 0;  // the block starts in the high half of its first word
  uint32_t* wp = reinterpret_cast<uint32_t*>(c.srow + (byte0 & ~3));
  uint32_t w[kWords];
#pragma unroll
  for (int j = 0; j < kWords; ++j) w[j] = wp[j];
  const uint32_t dbits = odd ? (w[0] >> 16) : (w[0] & 0xFFFFu);
  uint32_t cw[kCodeWords];
#pragma unroll
  for (int j = 0; j < kCodeWords; ++j) cw[j] = odd ? w[j + 1] : __funnelshift_r(w[j], w[j + 1], 16);
  const float d_in = round_dt<CDT>(__half2float(__ushort_as_half(static_cast<unsigned short>(dbits))));
  // Codes as exact floats: a byte (Q8_0: sign bit flipped; Q4_0: nibble)
  // under the exponent of 2^23 is 2^23 + b, and one packed subtraction of 2^23
  // plus the offset (128 or 8) leaves the signed code.
  float merged[32];
  const float2 d2 = make_float2(d_in, d_in);
  const float2 st2 = make_float2(W.strength, W.strength);
  if constexpr (kQ8) {
    const float2 off2 = make_float2(-8388736.0f, -8388736.0f);
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const uint32_t x = cw[j] ^ 0x80808080u;
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        const float2 raw = make_float2(__uint_as_float(__byte_perm(x, 0x4B000000u, 0x7540u + 2u * h)),
                                       __uint_as_float(__byte_perm(x, 0x4B000000u, 0x7541u + 2u * h)));
        const float2 v = __fmul2_rn(d2, __fadd2_rn(raw, off2));
        merged[4 * j + 2 * h] = v.x;
        merged[4 * j + 2 * h + 1] = v.y;
      }
    }
  } else {
    const float2 off2 = make_float2(-8388616.0f, -8388616.0f);
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const uint32_t lo = cw[j] & 0x0F0F0F0Fu;         // elements 4j .. 4j+3
      const uint32_t hi = (cw[j] >> 4) & 0x0F0F0F0Fu;  // elements 16+4j .. 16+4j+3
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        const float2 rl = make_float2(__uint_as_float(__byte_perm(lo, 0x4B000000u, 0x7540u + 2u * h)),
                                      __uint_as_float(__byte_perm(lo, 0x4B000000u, 0x7541u + 2u * h)));
        const float2 rh = make_float2(__uint_as_float(__byte_perm(hi, 0x4B000000u, 0x7540u + 2u * h)),
                                      __uint_as_float(__byte_perm(hi, 0x4B000000u, 0x7541u + 2u * h)));
        const float2 vl = __fmul2_rn(d2, __fadd2_rn(rl, off2));
        const float2 vh = __fmul2_rn(d2, __fadd2_rn(rh, off2));
        merged[4 * j + 2 * h] = vl.x;
        merged[4 * j + 2 * h + 1] = vl.y;
        merged[16 + 4 * j + 2 * h] = vh.x;
        merged[16 + 4 * j + 2 * h + 1] = vh.y;
      }
    }
  }
#pragma unroll
  for (int i = 0; i < 32; i += 2) {
    round_dt2<CDT>(merged[i], merged[i + 1]);
    const float2 m2 = __ffma2_rn(make_float2(acc[i], acc[i + 1]), st2, make_float2(merged[i], merged[i + 1]));
    merged[i] = m2.x;
    merged[i + 1] = m2.y;
    round_dt2<CDT>(merged[i], merged[i + 1]);
  }
  const bool sr = (W.flags & PIPER_FLAG_STOCHASTIC) != 0u;
  const PhiloxKey key = philox_key(W.k0, W.k1);
  const int col = c.tile_col0 + 32 * k;
  const uint64_t off0 =
      W.offset_base + static_cast<uint64_t>(c.row) * static_cast<uint64_t>(W.N) + col;
  uint32_t ow[kCodeWords];
  uint32_t dh;
  if constexpr (kQ8) {
    const float amax = tree3(merged, max3_abs);
    const float d = __fdiv_rn(amax, 127.0f);
    const float id = d == 0.0f ? 0.0f : __fdiv_rn(1.0f, d);
    dh = __half_as_ushort(__float2half_rn(d));
    uint32_t qb[32];
    float x[32];
    bool big = false;
#pragma unroll
    for (int i = 0; i < 32; ++i) {
      x[i] = __fmul_rn(merged[i], id);
      big |= !(fabsf(x[i]) < 4194304.0f);
    }
    if (!sr && !big) {
      // Round half away from zero (roundf is np_roundf exactly); a finite block
      // has |x| <= 127 * (1 + 2^-22), so no clamp is needed, and the low byte
      // of the bits of q + 1.5 * 2^23 is the two's-complement code.
      const float2 magic2 = make_float2(12582912.0f, 12582912.0f);
#pragma unroll
      for (int i = 0; i < 32; i += 2) {
        const float2 y = __fadd2_rn(make_float2(roundf(x[i]), roundf(x[i + 1])), magic2);
        qb[i] = __float_as_uint(y.x);
        qb[i + 1] = __float_as_uint(y.y);
      }
    } else {
      float q[32];
#pragma unroll
      for (int i = 0; i < 32; ++i) q[i] = roundf_away(x[i]);
      if (sr) {
#pragma unroll
        for (int w = 0; w < 4; ++w) {
          float v[8], qq[8];
#pragma unroll
          for (int j = 0; j < 8; ++j) {
            v[j] = x[8 * w + j];
            qq[j] = q[8 * w + j];
          }
          sr_int_xn<8>(v, qq, -127.0f, 127.0f, key, off0 + 8 * w);
#pragma unroll
          for (int j = 0; j < 8; ++j) q[8 * w + j] = qq[j];
        }
      }
#pragma unroll
      for (int i = 0; i < 32; ++i) qb[i] = float_int_bits(fminf(fmaxf(q[i], -128.0f), 127.0f));
    }
#pragma unroll
    for (int j = 0; j < 8; ++j) ow[j] = pack_low_bytes(qb[4 * j], qb[4 * j + 1], qb[4 * j + 2], qb[4 * j + 3]);
  } else {
    // The signed value of the first largest |x| (np.argmax): a pairwise tree
    // that keeps the left value unless the right one is strictly larger gives
    // the first maximum; a chunk holding a NaN scans in order as before.
    bool has_nan = false;
#pragma unroll
    for (int i = 0; i < 32; ++i) has_nan |= merged[i] != merged[i];
    float mx;
    if (!has_nan) {
      float av[32], sv[32];
#pragma unroll
      for (int i = 0; i < 32; ++i) {
        av[i] = fabsf(merged[i]);
        sv[i] = merged[i];
      }
#pragma unroll
      for (int st = 1; st < 32; st <<= 1) {
#pragma unroll
        for (int i = 0; i < 32; i += 2 * st) {
          const bool r = av[i + st] > av[i];
          av[i] = r ? av[i + st] : av[i];
          sv[i] = r ? sv[i + st] : sv[i];
        }
      }
      mx = sv[0];
    } else {
      int imax = 0;
      float best = fabsf(merged[0]);
      for (int i = 1; i < 32; ++i) {
        const float a = fabsf(merged[i]);
        if (a > best) {
          best = a;
          imax = i;
        }
      }
      mx = merged[0];
#pragma unroll
      for (int i = 1; i < 32; ++i) mx = (i == imax) ? merged[i] : mx;
    }
    const float d = __fdiv_rn(mx, -8.0f);
    const float id = d == 0.0f ? 0.0f : __fdiv_rn(1.0f, d);
    dh = __half_as_ushort(__float2half_rn(d));
    uint32_t qb[32];
    float y[32];
    bool bad = false;
#pragma unroll
    for (int i = 0; i < 32; ++i) {
      y[i] = __fadd_rn(__fmul_rn(merged[i], id), 8.5f);
      bad |= !(y[i] >= 0.0f && y[i] < 4194304.0f);
    }
    if (!sr && !bad) {
      // trunc(y) for 0 <= y < 2^22: the bits of y + 2^23 added toward zero.
#pragma unroll
      for (int i = 0; i < 32; ++i)
        qb[i] = min(__float_as_uint(__fadd_rz(y[i], 8388608.0f)) - 0x4B000000u, 15u);
    } else {
      float qf[32];
#pragma unroll
      for (int i = 0; i < 32; ++i) qf[i] = truncf(y[i]);
      if (sr) {
#pragma unroll
        for (int w = 0; w < 4; ++w) {
          float v[8], qq[8];
#pragma unroll
          for (int j = 0; j < 8; ++j) {
            v[j] = __fadd_rn(__fmul_rn(merged[8 * w + j], id), 8.0f);
            qq[j] = qf[8 * w + j];
          }
          sr_int_xn<8>(v, qq, 0.0f, 15.0f, key, off0 + 8 * w);
#pragma unroll
          for (int j = 0; j < 8; ++j) qf[8 * w + j] = qq[j];
        }
      }
#pragma unroll
      for (int i = 0; i < 32; ++i) qb[i] = float_int_bits(fminf(fmaxf(qf[i], 0.0f), 15.0f));
    }
    // byte j = element j (low nibble) | element j+16 (high nibble)
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const uint32_t lo = pack_low_bytes(qb[4 * j], qb[4 * j + 1], qb[4 * j + 2], qb[4 * j + 3]);
      const uint32_t hi = pack_low_bytes(qb[16 + 4 * j], qb[16 + 4 * j + 1], qb[16 + 4 * j + 2], qb[16 + 4 * j + 3]);
      ow[j] = lo | (hi << 4);
    }
  }
  if (odd) {
    wp[0] = (w[0] & 0xFFFFu) | (dh << 16);
#pragma unroll
    for (int j = 0; j < kCodeWords; ++j) wp[j + 1] = ow[j];
  } else {
    wp[0] = dh | (ow[0] << 16);
#pragma unroll
    for (int j = 1; j < kCodeWords; ++j) wp[j] = __funnelshift_l(ow[j - 1], ow[j], 16);
    wp[kCodeWords] = (w[kCodeWords] & 0xFFFF0000u) | (ow[kCodeWords - 1] >> 16);
  }
}

// ================================================================== kernel
// Warp-specialised persistent kernel, one CTA per SM, 128 x (1 + EW) threads:
//   warp 0      (one lane) the B strip of each item, and per tile the A tile
//               and the code tile, by 2-D bulk tensor copies;
//   warp 1      (one lane) TMEM allocation and tcgen05.mma of the rank-r
//               update into one of 512 / BN TMEM accumulators per tile;
//   warps 2-3   per-row scale bytes, and the cp.async fallback for factors or
//               code tiles whose alignment rules out bulk tensor copies;
//   warps 4..   EW epilogue warpgroups; tile t goes to warpgroup t % EW, whose
//               thread i owns tile row i: decode, merge, re-scale and encode
//               in place in shared memory, then one bulk tensor store.
// Code stages, A stages, B strips and accumulators circulate through their own
// full / empty mbarrier pairs. Every wait is bounded (ptx.cuh); a role whose
// wait gives up stops issuing work and the others then give up in turn, so
// the CTA always reaches its exit.
// Epilogue warpgroups per format and tile width (tile t -> warpgroup t % EW).
// Three give the epilogue more warps in flight; GGUF keeps two so that its
// 256-column tiles (the narrowest whose rows are 16-byte multiples) fit two
// accumulators, and bitsandbytes 4-bit keeps two for its per-lane tables.
// NVFP4 runs both: 256-column tiles with two warpgroups for round-to-nearest,
// 128-column tiles with three for stochastic rounding (the host plan picks
// the width by rounding mode; measured 543 vs 476 GB/s RTN, 146 vs 191 SR).
__host__ __device__ constexpr int epi_wgs_rt(int fmt, int bn) {
  if (fmt == PIPER_FMT_NVFP4) return bn >= 256 ? 2 : 3;
  return (fmt == PIPER_FMT_GGUF_Q8_0 || fmt == PIPER_FMT_GGUF_Q4_0 || fmt == PIPER_FMT_BNB4_NF4 ||
          fmt == PIPER_FMT_BNB4_FP4)
             ? 2
             : 3;
}
template <int FMT, int BN>
__host__ __device__ constexpr int epi_wgs() { return epi_wgs_rt(FMT, BN); }
template <int FMT, int BN>
__host__ __device__ constexpr int ws_threads() { return 128 * (1 + epi_wgs<FMT, BN>()); }
constexpr int kLoadThreads = 64;  // warps 2-3
// Dynamic work distribution: warp 0 takes the next item from the launch's
// counter (atomicAdd, items ordered by decreasing cost) and publishes it in a
// ring that every role reads in the same order.
constexpr int kItemRing = 8;
constexpr int kMaxStages = 8;    // code stages
constexpr int kMaxAStages = 4;
constexpr int kMaxAcc = 8;        // accumulator buffers: 512 tensor-memory columns / BN
constexpr uint32_t kCtrlRegs = 56;
// Registers per epilogue thread after the control warpgroup gives up its share
// (launch allocation: threads x (65536 / threads rounded down to 8)).
template <int FMT, int BN>
__host__ __device__ constexpr uint32_t epi_regs() {
  constexpr uint32_t threads = ws_threads<FMT, BN>();
  constexpr uint32_t launch = (65536u / threads) / 8u * 8u;
  return ((threads * launch - 128u * kCtrlRegs) / (128u * epi_wgs<FMT, BN>())) / 8u * 8u;
}
constexpr int kSmemLimit = 232448;  // dynamic shared memory per CTA on sm_100

template <int FMT>
__host__ __device__ constexpr bool is_gguf() {
  return FMT == PIPER_FMT_GGUF_Q8_0 || FMT == PIPER_FMT_GGUF_Q4_0;
}

// Geometry of one code tile (128 rows x BN columns) in shared memory. TMA
// tiles arrive as `kBoxes` boxes of 128 rows x kBoxRow bytes, swizzled in
// 16-byte chunks (128 / 64 / 32-byte rows); GGUF boxes are dense rows.
template <int FMT, int BN>
struct TileGeom {
  static constexpr int kRowBytes = code_bytes<FMT>(BN);
  static constexpr int kBoxRow = is_gguf<FMT>() ? kRowBytes : (kRowBytes >= 128 ? 128 : kRowBytes);
  static constexpr int kBoxes = kRowBytes / kBoxRow;
  static constexpr int kBoxShift = kBoxRow == 128 ? 3 : (kBoxRow == 64 ? 2 : 1);
  static constexpr int kPadRS = row_stride<FMT, BN>();
  static constexpr int kCodeSlot = align_up(128 * (kPadRS > kRowBytes ? kPadRS : kRowBytes), 1024);
};

// Shared memory: code stages, A stages, B strips, then the barriers and the
// TMEM slot (+1 KB of alignment slack for the dynamic shared-memory base).
__host__ __device__ constexpr int ws_code_stage_bytes(int code_slot) {
  return align_up(code_slot + 128 * kScaleSlot, 1024);
}
__host__ __device__ constexpr int ws_a_stage_bytes(int kp, int bn) { return align_up(kp * bn * 2, 1024); }
__host__ __device__ constexpr int ws_b_buf_bytes(int kp) { return 128 * kp * 2; }
// The tail holds the mbarriers, the TMEM slot and the item ring (640 B) and,
// for fused per-row passes, each epilogue warpgroup's partial row maxima for
// two items (2 x 3 x 128 float2).
constexpr int kBarBytes = 640;
constexpr int kTailBytes = kBarBytes + 2 * 3 * 128 * 8;
__host__ __device__ constexpr int ws_smem_bytes(int code_slot, int kp, int bn, int sc, int sa, int nbb) {
  return 1024 + sc * ws_code_stage_bytes(code_slot) + sa * ws_a_stage_bytes(kp, bn) + nbb * ws_b_buf_bytes(kp) +
         kTailBytes;
}

struct ItemGeom {
  int wi, strip, row0, col_begin, col_end, n_tiles;
};

template <int BN>
__device__ __forceinline__ ItemGeom item_geom(const LaunchParams& P, int item) {
  ItemGeom g;
  int wi = 0;
  while (wi + 1 < P.n_weights && P.w[wi + 1].item_begin <= item) ++wi;
  const DevWeight& W = P.w[wi];
  const int local = item - W.item_begin;
  g.wi = wi;
  g.strip = local / W.col_items;
  const int ci = local - g.strip * W.col_items;
  g.row0 = W.row_begin + g.strip * 128;
  g.col_begin = ci * W.item_cols;
  g.col_end = min(W.N, g.col_begin + W.item_cols);
  g.n_tiles = (g.col_end - g.col_begin + BN - 1) / BN;
  return g;
}

// Byte offset of column c0 within a row of codes.
template <int FMT>
__device__ __forceinline__ int64_t code_off(int c0) {
  if constexpr (is_gguf<FMT>()) return code_bytes<FMT>(c0);
  else if constexpr (FMT == PIPER_FMT_MXFP4 || FMT == PIPER_FMT_NVFP4 || FMT == PIPER_FMT_BNB4_NF4 ||
                     FMT == PIPER_FMT_BNB4_FP4)
    return c0 / 2;
  else return c0;
}

// Row bytes of the B strip's swizzle atoms (K-major): the widest of 128 / 64 /
// 32 bytes dividing KP * 2, so a strip is KP*2 / kb boxes of 128 rows x kb bytes.
__host__ __device__ __forceinline__ int kb_row(int kp) {
  return (kp * 2) % 128 == 0 ? 128 : ((kp * 2) % 64 == 0 ? 64 : 32);
}
__host__ __device__ __forceinline__ uint32_t swizzle_layout(int row_bytes) {
  return row_bytes == 128 ? 2u : (row_bytes == 64 ? 4u : 6u);
}
// 16-byte chunk XOR of row r under the swizzle of `row_bytes`-byte rows.
__device__ __forceinline__ uint32_t swizzle_xor(int r, int row_bytes) {
  return row_bytes == 128 ? static_cast<uint32_t>(r & 7)
                          : (row_bytes == 64 ? static_cast<uint32_t>((r >> 1) & 3) : static_cast<uint32_t>((r >> 2) & 1));
}

template <int FMT, int PASS, int BN, int CDT>
__global__ void __launch_bounds__(ws_threads<FMT, BN>(), 1) merge_kernel(const __grid_constant__ LaunchParams P) {
  constexpr int kEpiWGs = epi_wgs<FMT, BN>();
  static_assert(kEpiWGs <= 3, "kTailBytes reserves the row-maxima exchange (rpart) for three epilogue warpgroups");
  // Arrivals that free an item-ring slot: the MMA lane, the two loader warps
  // and every epilogue warp.
  constexpr uint32_t kItemReaders = 1 + 2 + 4 * kEpiWGs;
  using G = TileGeom<FMT, BN>;
  // Per-row TorchAO FP8 and INT8 run the packed fused sweeps.
  constexpr bool kPackedRow = PASS == kFused && flavor_of(FMT) == kTorchao &&
                              (base_fmt(FMT) == PIPER_FMT_FP8_E4M3 || base_fmt(FMT) == PIPER_FMT_FP8_E5M2 ||
                               base_fmt(FMT) == PIPER_FMT_INT8);
  extern __shared__ __align__(1024) uint8_t smem[];
  const int tid = threadIdx.x;
  const int warp = tid >> 5;
  const int lane = tid & 31;
  const int KPL = P.kp_max;
  const int S = P.c_stages;
  const int SA = P.a_stages;
  const int NBB = P.b_bufs;
  constexpr int kCodeStage = ws_code_stage_bytes(G::kCodeSlot);
  const int kAStage = ws_a_stage_bytes(KPL, BN);

  uint8_t* base1k = smem + ((1024u - (smem_u32(smem) & 1023u)) & 1023u);
  uint8_t* sCode = base1k;
  uint8_t* sAst = sCode + S * kCodeStage;
  uint8_t* sB = sAst + SA * kAStage;  // NBB B strips
  uint64_t* bars = reinterpret_cast<uint64_t*>(sB + NBB * ws_b_buf_bytes(KPL));
  uint64_t* full = bars;                  // [kMaxStages] code tile (+ scales) landed
  uint64_t* empty = full + kMaxStages;    // [kMaxStages] code stage written back
  uint64_t* full_a = empty + kMaxStages;  // [kMaxAStages] A tile landed
  uint64_t* empty_a = full_a + kMaxAStages;  // [kMaxAStages] A tile read by the tensor core
  uint64_t* bfull = empty_a + kMaxAStages;   // [2]
  uint64_t* bempty = bfull + 2;           // [2]
  uint64_t* afull = bempty + 2;           // [kMaxAcc]
  uint64_t* aempty = afull + kMaxAcc;     // [kMaxAcc]
  uint64_t* mma_done = aempty + kMaxAcc;
  uint64_t* rmax_bar = mma_done + 1;      // [2] partial row maxima published (fused per-row)
  uint64_t* item_full = rmax_bar + 2;     // [kItemRing] next work item published
  uint64_t* item_empty = item_full + kItemRing;  // [kItemRing] read by every role
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(item_empty + kItemRing);
  int* item_ring = reinterpret_cast<int*>(tmem_slot + 4);  // [kItemRing]
  float2* rpart = reinterpret_cast<float2*>(reinterpret_cast<uint8_t*>(bars) + kBarBytes);  // [2][kEpiWGs][128]
  auto stage_codes = [&](int s) { return sCode + s * kCodeStage; };
  auto stage_scales = [&](int s) { return sCode + s * kCodeStage + G::kCodeSlot; };
  auto stage_a = [&](int x) { return sAst + x * kAStage; };

  if (tid == 0) {
    for (int i = 0; i < SA; ++i) {
      mbar_init(&full_a[i], 1 + kLoadThreads);
      mbar_init(&empty_a[i], 1);  // tcgen05.commit after the MMAs that read it
    }
    for (int i = 0; i < S; ++i) {
      mbar_init(&full[i], 1 + kLoadThreads);
      // REDUCE steps store nothing: each warp of the tile's warpgroup releases
      // the stage (fused passes release stored stages with four arrivals too).
      mbar_init(&empty[i], (PASS == kReduce || PASS == kFused) ? 4 : 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&bfull[i], 1 + kLoadThreads);
      mbar_init(&bempty[i], 1);
    }
    for (int i = 0; i < kMaxAcc; ++i) {
      mbar_init(&afull[i], 1);
      mbar_init(&aempty[i], 4);  // the four warps of the tile's warpgroup
    }
    mbar_init(mma_done, 1);
    for (int i = 0; i < 2; ++i) mbar_init(&rmax_bar[i], kEpiWGs);
    for (int i = 0; i < kItemRing; ++i) {
      mbar_init(&item_full[i], 1);
      mbar_init(&item_empty[i], kItemReaders);
    }
    fence_mbar_init();
  }
  constexpr int NB = 512 / BN;  // accumulator buffers in the 512 tensor-memory columns
  static_assert(NB >= kEpiWGs && NB <= kMaxAcc, "accumulator buffers per warpgroup");
  if (warp == 1) {
    tmem_alloc(tmem_slot, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  // Launch allocation 384 x 168 = 64512 registers: the control warpgroup
  // (warps 0-3) keeps 56 per thread, the two epilogue warpgroups get 224
  // (128 x 56 + 256 x 224 = 64512), which buys the epilogue more independent
  // work in flight per thread.
  if (warp < 4) {
  regs_dec<kCtrlRegs>();
  if (warp == 0) {
    // ------------------------------------------------ code tiles (bulk tensor)
    if (lane == 0) {
      uint32_t t = 0, it = 0;
      bool ok = true;
      // The next item's counter value is fetched one item ahead, so the
      // atomic's round trip overlaps the current item's loads.
      unsigned int next_v = atomicAdd(&g_sched_next[P.sched_slot], 1u);
      for (;; ++it) {
        if (!ok) break;
        // Take the next item (-1 past the last) and publish it to every role.
        const int rs = static_cast<int>(it % kItemRing);
        if (it >= static_cast<uint32_t>(kItemRing)) {
          ok = mbar_wait(&item_empty[rs], ((it / kItemRing) - 1) & 1u, kStatusTimeoutLoad);
          if (!ok) break;
        }
        const unsigned int v = next_v;
        const int item = v < static_cast<unsigned int>(P.n_items) ? static_cast<int>(v) : -1;
        if (item >= 0) next_v = atomicAdd(&g_sched_next[P.sched_slot], 1u);
        item_ring[rs] = item;
        mbar_arrive(&item_full[rs]);
        if (item < 0) break;
        const ItemGeom g = item_geom<BN>(P, item);
        const DevWeight& W = P.w[g.wi];
        const int KP = W.KP;
        if (W.use_tma) prefetch_tmap(&W.tmap);
        // B strip of this item: KP*2 / kb boxes of 128 rows x kb bytes.
        const int jb = it % NBB;
        if (it >= static_cast<uint32_t>(NBB)) {
          ok = mbar_wait(&bempty[jb], ((it / NBB) - 1) & 1u, kStatusTimeoutMma);
          if (!ok) break;
        }
        if (W.use_tma_b) {
          const int kb = kb_row(KP);
          const int nbox = KP * 2 / kb;
          uint8_t* sBj = sB + jb * ws_b_buf_bytes(KPL);
          mbar_arrive_expect_tx(&bfull[jb], static_cast<uint32_t>(nbox * 128 * kb));
          for (int j = 0; j < nbox; ++j) tma_load_2d(sBj + j * 128 * kb, &W.tmap_b, j * (kb / 2), g.row0, &bfull[jb]);
        } else {
          mbar_arrive(&bfull[jb]);
        }
        // Fused per-row passes visit every column tile twice: reduce, then encode.
        const int n_steps = PASS == kFused ? 2 * g.n_tiles : g.n_tiles;
        for (int st = 0; st < n_steps; ++st, ++t) {
          const int tile = st < g.n_tiles ? st : 2 * g.n_tiles - 1 - st;  // encode sweep runs backwards: L2-hot tiles first
          const int c0 = g.col_begin + tile * BN;
          // A tile: BN/64 boxes of 64 columns x KP rows (MN-major, 128-byte swizzle).
          const int x = t % SA;
          if (t >= static_cast<uint32_t>(SA)) {
            ok = mbar_wait(&empty_a[x], ((t / SA) - 1) & 1u, kStatusTimeoutMma);
            if (!ok) break;
          }
          if (W.use_tma_a) {
            mbar_arrive_expect_tx(&full_a[x], static_cast<uint32_t>(BN * KP * 2));
            for (int j = 0; j < BN / 64; ++j)
              tma_load_2d(stage_a(x) + j * KP * 128, &W.tmap_a, c0 + j * 64, 0, &full_a[x]);
          } else {
            mbar_arrive(&full_a[x]);
          }
          // Code tile.
          const int s = t % S;
          if (t >= static_cast<uint32_t>(S)) {
            ok = mbar_wait(&empty[s], ((t / S) - 1) & 1u, kStatusTimeoutLoad);
            if (!ok) break;
          }
          int boxes = 0;
          const int64_t off = code_off<FMT>(c0);
          if (W.use_tma)
            for (int j = 0; j < G::kBoxes; ++j) boxes += (off + j * G::kBoxRow < W.row_bytes) ? 1 : 0;
          if (boxes > 0) mbar_arrive_expect_tx(&full[s], static_cast<uint32_t>(boxes * 128 * G::kBoxRow));
          else mbar_arrive(&full[s]);
          for (int j = 0; j < boxes; ++j) {
            const int xb = static_cast<int>(off + j * G::kBoxRow);
            tma_load_2d(stage_codes(s) + j * 128 * G::kBoxRow, &W.tmap, is_gguf<FMT>() ? xb / 8 : xb, g.row0,
                        &full[s]);
          }
        }
      }
      // Loads still in flight after an early exit land before the CTA retires.
      const uint32_t issued = t;
      for (uint32_t u = issued > static_cast<uint32_t>(S) ? issued - S : 0u; u < issued; ++u)
        mbar_wait(&full[u % S], (u / S) & 1u, kStatusTimeoutLoad);
      for (uint32_t u = issued > static_cast<uint32_t>(SA) ? issued - SA : 0u; u < issued; ++u)
        mbar_wait(&full_a[u % SA], (u / SA) & 1u, kStatusTimeoutLoad);
    }
    __syncwarp();
  } else if (warp == 1) {
    // ------------------------------------------------------------ tensor core
    if (lane == 0) {
      uint32_t t = 0, it = 0;
      bool ok = true;
      constexpr uint32_t idesc = idesc_f16(BN, CDT == kBF16 ? 1u : 0u);
      for (;; ++it) {
        if (!ok) break;
        const int rs = static_cast<int>(it % kItemRing);
        ok = mbar_wait(&item_full[rs], (it / kItemRing) & 1u, kStatusTimeoutLoad);
        if (!ok) break;
        const int item = *reinterpret_cast<volatile int*>(&item_ring[rs]);
        mbar_arrive(&item_empty[rs]);
        if (item < 0) break;
        const ItemGeom g = item_geom<BN>(P, item);
        const int KP = P.w[g.wi].KP;
        const int jb = it % NBB;
        ok = mbar_wait(&bfull[jb], (it / NBB) & 1u, kStatusTimeoutLoad);
        if (!ok) break;
        const uint32_t a_base = smem_u32(sB + jb * ws_b_buf_bytes(KPL));
        const int kb = kb_row(KP);
        const uint32_t a_layout = swizzle_layout(kb);
        // Fused per-row passes visit every column tile twice: reduce, then encode.
        const int n_steps = PASS == kFused ? 2 * g.n_tiles : g.n_tiles;
        for (int st = 0; st < n_steps && ok; ++st, ++t) {  // the MMA needs no column: its A tile is staged
          const int x = t % SA;
          const int ab = t % NB;
          ok = mbar_wait(&full_a[x], (t / SA) & 1u, kStatusTimeoutLoad);
          if (ok && t >= static_cast<uint32_t>(NB)) ok = mbar_wait(&aempty[ab], ((t / NB) - 1) & 1u, kStatusTimeoutMma);
          if (!ok) break;
          if constexpr (CDT == kF32) {
            // fp32 factors: the epilogue forms the update on CUDA cores, so this
            // role only keeps the accumulator and stage rings turning.
            mbar_arrive(&afull[ab]);
            mbar_arrive(&empty_a[x]);
            continue;
          }
          fence_proxy_async_smem();  // cp.async-written operands -> tensor core
          tc_fence_after();
          const uint32_t b_base = smem_u32(stage_a(x));
          for (int ks = 0; ks < KP / 16; ++ks) {
            // B strip, K-major: 16 columns = 32 bytes inside a kb-byte swizzled row.
            const int kbyte = ks * 32;
            const uint64_t adesc =
                smem_desc_sw(a_base + (kbyte / kb) * 128 * kb + (kbyte % kb), 16, 8 * kb, a_layout);
            // A tile, MN-major: 64-column blocks KP*128 bytes apart, 8-row groups 1024 apart.
            const uint64_t bdesc = smem_desc_sw(b_base + ks * 2048, KP * 128, 1024, 2u);
            umma_f16(tmem + ab * BN, adesc, bdesc, idesc, ks > 0 ? 1u : 0u);
          }
          umma_commit(&afull[ab]);
          umma_commit(&empty_a[x]);  // the A stage is free once these MMAs complete
        }
        if constexpr (CDT == kF32) mbar_arrive(&bempty[jb]);
        else umma_commit(&bempty[jb]);  // the strip is free once these MMAs complete
      }
      if constexpr (CDT != kF32) {
        umma_commit(mma_done);
        mbar_wait(mma_done, 0u, kStatusTimeoutMma);
      }
    }
    __syncwarp();
  } else if (warp < 4) {
    // ------------------------------------- A tiles, scales, B strips (cp.async)
    const int lt = tid - 64;
    uint32_t t = 0, it = 0;
    bool ok = true;
    for (;; ++it) {
      if (!__all_sync(0xFFFFFFFFu, ok)) break;
      const int rs = static_cast<int>(it % kItemRing);
      ok = mbar_wait(&item_full[rs], (it / kItemRing) & 1u, kStatusTimeoutLoad);
      ok = __all_sync(0xFFFFFFFFu, ok);  // one decision per warp
      if (!ok) break;
      const int item = *reinterpret_cast<volatile int*>(&item_ring[rs]);
      __syncwarp();
      if (lane == 0) mbar_arrive(&item_empty[rs]);
      if (item < 0) break;
      const ItemGeom g = item_geom<BN>(P, item);
      const DevWeight& W = P.w[g.wi];
      const int KP = W.KP;
      const int rows_here = min(128, W.M - g.row0);
      // B strip (K-major canonical): chunk kc of row t at kc*2048 + (t/8)*128 + (t%8)*16.
      const int jb = it % NBB;
      if (it >= static_cast<uint32_t>(NBB)) {
        ok = mbar_wait(&bempty[jb], ((it / NBB) - 1) & 1u, kStatusTimeoutMma);
        if (!ok) break;
      }
      if (CDT != kF32 && !W.use_tma_b) {  // fp32 factors are read by the epilogue itself
        // Same swizzled K-major layout the bulk tensor copy would produce.
        uint8_t* sBj = sB + jb * ws_b_buf_bytes(KPL);
        const int kb = kb_row(KP);
        const int cpr = kb / 16;  // 16-byte chunks per row
        const bool vec = ((reinterpret_cast<uintptr_t>(W.b) | (W.r * 2)) & 15) == 0;
        for (int idx = lt; idx < 128 * (KP / 8); idx += kLoadThreads) {
          const int rt = idx & 127;
          const int kc = idx >> 7;
          const int row = g.row0 + rt;
          uint8_t* dst = sBj + (kc / cpr) * 128 * kb + rt * kb +
                         (((static_cast<uint32_t>(kc % cpr)) ^ swizzle_xor(rt, kb)) << 4);
          const uint16_t* brow = W.b + static_cast<int64_t>(row) * W.r;
          if (row < W.M && vec && kc * 8 + 8 <= W.r) {
            cp_async16(dst, brow + kc * 8);
          } else {
            uint4 v = make_uint4(0u, 0u, 0u, 0u);
            if (row < W.M) {
              uint16_t e[8];
#pragma unroll
              for (int j = 0; j < 8; ++j) e[j] = (kc * 8 + j < W.r) ? brow[kc * 8 + j] : 0;
              v = make_uint4(e[0] | (e[1] << 16), e[2] | (e[3] << 16), e[4] | (e[5] << 16), e[6] | (e[7] << 16));
            }
            *reinterpret_cast<uint4*>(dst) = v;
          }
        }
      }
      __threadfence_block();  // plain smem stores of ragged rows precede the arrival
      cp_async_mbar_arrive(&bfull[jb]);
      const bool vec_a = ((reinterpret_cast<uintptr_t>(W.a) | (W.N * 2)) & 15) == 0;
      // Fused per-row passes visit every column tile twice: reduce, then encode.
      const int n_steps = PASS == kFused ? 2 * g.n_tiles : g.n_tiles;
      for (int st = 0; st < n_steps; ++st, ++t) {
        const int tile = st < g.n_tiles ? st : 2 * g.n_tiles - 1 - st;  // encode sweep runs backwards: L2-hot tiles first
        const int c0 = g.col_begin + tile * BN;
        const int ncols = min(BN, g.col_end - c0);
        const int x = t % SA;
        if (t >= static_cast<uint32_t>(SA)) {
          ok = mbar_wait(&empty_a[x], ((t / SA) - 1) & 1u, kStatusTimeoutMma);
          if (!ok) break;
        }
        // A tile when it cannot move by bulk tensor copies: the same MN-major
        // layout, 64-column blocks of KP rows x 128 bytes, 128-byte swizzle.
        if (CDT != kF32 && !W.use_tma_a) {
          uint8_t* sA = stage_a(x);
          const int chunks = KP * BN / 8;
          for (int idx = lt; idx < chunks; idx += kLoadThreads) {
            const int ng = idx % (BN / 8);
            const int kr = idx / (BN / 8);
            const int n = c0 + ng * 8;
            uint8_t* dst = sA + (ng >> 3) * KP * 128 + kr * 128 + (((static_cast<uint32_t>(ng & 7)) ^ (kr & 7)) << 4);
            const uint16_t* ap = W.a + static_cast<int64_t>(kr) * W.N + n;
            if (kr < W.r && vec_a && n + 8 <= g.col_end) {
              cp_async16(dst, ap);
            } else {
              uint4 v = make_uint4(0u, 0u, 0u, 0u);
              if (kr < W.r) {
                uint16_t e[8];
#pragma unroll
                for (int j = 0; j < 8; ++j) e[j] = (n + j < g.col_end) ? ap[j] : 0;
                v = make_uint4(e[0] | (e[1] << 16), e[2] | (e[3] << 16), e[4] | (e[5] << 16), e[6] | (e[7] << 16));
              }
              *reinterpret_cast<uint4*>(dst) = v;
            }
          }
        }
        __threadfence_block();
        cp_async_mbar_arrive(&full_a[x]);
        const int s = t % S;
        if (t >= static_cast<uint32_t>(S)) {
          ok = mbar_wait(&empty[s], ((t / S) - 1) & 1u, kStatusTimeoutLoad);
          if (!ok) break;
        }
        if (!W.use_tma) {
          // Codes into the padded row layout (rows of kPadRS bytes).
          const int64_t off = code_off<FMT>(c0);
          const int nbytes = static_cast<int>(code_off<FMT>(c0 + ncols) - off);
          const int64_t m = W.row_bytes | off | nbytes | static_cast<int64_t>(reinterpret_cast<uintptr_t>(W.q));
          const int gran = (m & 15) == 0 ? 16 : ((m & 3) == 0 ? 4 : 1);
          const int per = nbytes / gran;
          const uint8_t* src0 = W.q + static_cast<int64_t>(g.row0) * W.row_bytes + off;
          uint8_t* dst0 = stage_codes(s);
          for (int k = lt; k < rows_here * per; k += kLoadThreads) {
            const int r = k / per;
            const int i = k - r * per;
            uint8_t* dst = dst0 + r * G::kPadRS + i * gran;
            const uint8_t* src = src0 + static_cast<int64_t>(r) * W.row_bytes + i * gran;
            if (gran == 16) cp_async16(dst, src);
            else if (gran == 4) cp_async4(dst, src);
            else *dst = *src;
          }
        }
        // Per-row scale bytes of MX / NVFP4 tiles.
        if constexpr (FMT == PIPER_FMT_MXFP8_E4M3 || FMT == PIPER_FMT_MXFP8_E5M2 || FMT == PIPER_FMT_MXFP4 ||
                      FMT == PIPER_FMT_NVFP4) {
          constexpr int kBlk = FMT == PIPER_FMT_NVFP4 ? 16 : 32;
          const int b0 = c0 / kBlk;
          const int nb = (ncols + kBlk - 1) / kBlk;
          const uint8_t* scale8 = reinterpret_cast<const uint8_t*>(W.scale);
          const bool sw = (W.flags & PIPER_FLAG_SWIZZLED) != 0u;
          const bool vec4 = ((b0 | nb) & 3) == 0 && (sw || (W.scale_cols & 3) == 0) &&
                            (reinterpret_cast<uintptr_t>(W.scale) & 3) == 0;
          for (int rt = lt; rt < rows_here; rt += kLoadThreads) {
            const int row = g.row0 + rt;
            uint8_t* dst = stage_scales(s) + rt * kScaleSlot;
            if (vec4) {
              for (int j = 0; j < nb; j += 4) cp_async4(dst + j, scale8 + scale_index(W, row, b0 + j));
            } else {
              for (int j = 0; j < nb; ++j) dst[j] = scale8[scale_index(W, row, b0 + j)];
            }
          }
        }
        __threadfence_block();
        cp_async_mbar_arrive(&full[s]);
      }
    }
    cp_async_wait_all();
  }
  } else {
    // ---------------------------------------------------------------- epilogue
    regs_inc<epi_regs<FMT, BN>()>();
    const int e = tid - 128;
    const int rt = e & 127;         // tile row / tensor-memory lane of this thread
    const int wg = e >> 7;          // processes tiles t with t % kEpiWGs == wg
    const uint32_t bar_id = 1u + static_cast<uint32_t>(wg);  // this warpgroup's named barrier
    const uint32_t lane_off = static_cast<uint32_t>((e >> 5) & 3) * 32u << 16;
    uint32_t t = 0;
    uint32_t it_e = 0;  // items done by this CTA (fused passes: parity of the row-maxima slot)
    int pending = -1;   // stage whose bulk store may still be reading it
    // Stages are released by four arrivals when warps release them one by one.
    constexpr uint32_t kStoreRelease = PASS == kFused ? 4u : 1u;
    bool ok = true;
    for (;; ++it_e) {
      if (!ok) break;  // decided per warpgroup
      const int rs = static_cast<int>(it_e % kItemRing);
      ok = mbar_wait(&item_full[rs], (it_e / kItemRing) & 1u, kStatusTimeoutLoad);
      ok = named_bar_and(bar_id, 128, ok);  // one decision per warpgroup
      if (!ok) break;
      const int item = *reinterpret_cast<volatile int*>(&item_ring[rs]);
      __syncwarp();
      if (lane == 0) mbar_arrive(&item_empty[rs]);
      if (item < 0) break;
      const ItemGeom g = item_geom<BN>(P, item);
      const DevWeight& W = P.w[g.wi];
      const int local = item - W.item_begin;
      const int row = g.row0 + rt;
      const bool valid = row < W.M;
      const int rows_here = min(128, W.M - g.row0);
      const bool tma = W.use_tma != 0;
      const int owner = static_cast<int>(t % kEpiWGs);  // warpgroup of the item's first tile

      QpCache qc;  // quantization block of this thread's row (FP8 / INT8)
      // Per-thread running reductions for REDUCE passes.
      float red_max = 0.0f, red_nmin = 0.0f;
      // Packed per-row FP8 / INT8: this warpgroup saw a NaN or an infinity in the row
      // (red_special), and so did some warpgroup (f_special, encode sweep).
      bool red_special = false, f_special = false;
      int red_qp = -1;
      // ENCODE passes: qparams of the last quantization block encoded.
      int enc_qp = -1;
      Int8Q enc_q;
      enc_q.scale = 1.0f;
      enc_q.zp = 0;
      float enc_s = 1.0f;
      auto flush_reduce = [&]() {
        if (red_qp >= 0) {
          atomic_max_nonneg(&W.qmax[red_qp], red_max);
          if (base_fmt(FMT) == PIPER_FMT_INT8) atomic_max_nonneg(&W.qmin[red_qp], red_nmin);
        }
        red_max = 0.0f;
        red_nmin = 0.0f;
      };
      // NVFP4 global scales (two-level).
      const bool two_level = (FMT == PIPER_FMT_NVFP4) && W.gscale != nullptr;
      float g_in = 1.0f, g_out = 1.0f;
      if constexpr (FMT == PIPER_FMT_NVFP4) {
        if (two_level) {
          if (PASS == kReduce) {
            g_in = *W.gscale;
            if (local == 0 && rt == 0 && wg == owner) W.old_scale[0] = g_in;
          } else {
            g_in = W.old_scale[0];
            const float amax = __uint_as_float(*W.qmax);
            g_out = fmaxf(__fmul_rn(amax, 1.0f / 2688.0f), 1.1920928955078125e-07f);  // `/ 2688.0`: x * fp32(1 / 2688)
          }
        }
      }

      // Fused per-row passes: the row's input scale / zero point are read once,
      // before any warpgroup can publish (and so before the new scale is
      // written); the new qparams follow from the combined row maxima.
      float f_s_in = 1.0f;
      int f_z_in = 0;
      bool fq_ready = false;
      float f_s = 1.0f;
      Int8Q f_q;
      f_q.scale = 1.0f;
      f_q.zp = 0;
      if constexpr (PASS == kFused) {
        if (valid) {
          qp_load<FMT, kReduce>(W, row, qc);
          f_s_in = qc.s_in;
          f_z_in = qc.z_in;
        }
      }

      // Fused per-row passes visit every column tile twice: reduce, then encode.
      const int n_steps = PASS == kFused ? 2 * g.n_tiles : g.n_tiles;
      for (int st = 0; st < n_steps; ++st, ++t) {
        const int tile = st < g.n_tiles ? st : 2 * g.n_tiles - 1 - st;  // encode sweep runs backwards: L2-hot tiles first
        const bool enc_phase = PASS == kFused && st >= g.n_tiles;
        if constexpr (PASS == kFused) {
          if (st == g.n_tiles) {
            // Publish this warpgroup's partial row maxima (zero when it saw no
            // tile of the strip) for the encode steps of every warpgroup.
            // A row holding a NaN or an infinity is flagged by the sign bit of
            // its (non-negative) maximum.
            rpart[((it_e & 1u) * kEpiWGs + wg) * 128 + rt] =
                make_float2(__int_as_float(__float_as_int(red_max) | (red_special ? 0x80000000 : 0)), red_nmin);
            named_bar_sync(bar_id, 128);
            if (rt == 0) mbar_arrive(&rmax_bar[it_e & 1u]);
          }
        }
        if (static_cast<int>(t % kEpiWGs) != wg) continue;  // another warpgroup's tile
        if (enc_phase && !fq_ready) {
          ok = mbar_wait(&rmax_bar[it_e & 1u], (it_e >> 1) & 1u, kStatusTimeoutLoad);
          float amax = 0.0f, nmin = 0.0f;
#pragma unroll
          for (int w = 0; w < kEpiWGs; ++w) {
            const float2 v = rpart[((it_e & 1u) * kEpiWGs + w) * 128 + rt];
            amax = fmaxf(amax, fabsf(v.x));
            nmin = fmaxf(nmin, v.y);
            f_special |= __float_as_int(v.x) < 0;
          }
          if constexpr (kPackedRow) {  // maxima of unrounded merged values: round them as the values would be
            amax = round_dt<CDT>(amax);
            nmin = round_dt<CDT>(nmin);
          }
          if constexpr (base_fmt(FMT) == PIPER_FMT_INT8) {
            const bool asym = (W.flags & PIPER_FLAG_ASYMMETRIC) != 0u;
            const int qlo = (W.flags & PIPER_FLAG_REDUCE_RANGE) ? -64 : -128;
            const int qhi = (W.flags & PIPER_FLAG_REDUCE_RANGE) ? 63 : 127;
            if constexpr (flavor_of(FMT) == kTorchao) {
              f_q = int8_qparams<CDT>(-nmin, amax, asym, qlo, qhi, W.scale_dt);
            } else {
              f_q.scale = flavor_scale<CDT>(flavor_of(FMT), fmaxf(amax, nmin), 127.0f);
              f_q.zp = 0;
            }
          } else if constexpr (base_fmt(FMT) == PIPER_FMT_FP8_E4M3 || base_fmt(FMT) == PIPER_FMT_FP8_E5M2) {
            const float lim = base_fmt(FMT) == PIPER_FMT_FP8_E4M3 ? 448.0f : 57344.0f;
            if constexpr (flavor_of(FMT) == kQuanto) f_s = flavor_scale<CDT>(kQuanto, amax, lim);
            else f_s = fp8_new_scale<CDT>(amax, lim);
          }
          fq_ready = true;
        }
        if (enc_phase && tile == 0 && valid) {
          // The warpgroup that encodes the row's first tile writes its new qparams.
          if constexpr (base_fmt(FMT) == PIPER_FMT_INT8) {
            store_scale_dt(W.scale, row, W.scale_dt, f_q.scale);
            if (W.zp != nullptr) W.zp[row] = static_cast<int8_t>(f_q.zp);
          } else if constexpr (base_fmt(FMT) == PIPER_FMT_FP8_E4M3 || base_fmt(FMT) == PIPER_FMT_FP8_E5M2) {
            store_scale<FMT>(W, row, f_s);
          }
        }
        const int s = t % S;
        const int ab = t % NB;
        const int c0 = g.col_begin + tile * BN;
        const int tcols = min(BN, g.col_end - c0);
        if (ok) ok = mbar_wait(&full[s], (t / S) & 1u, kStatusTimeoutLoad);
        if (ok) ok = mbar_wait(&afull[ab], (t / NB) & 1u, kStatusTimeoutMma);
        // One decision for all threads that meet at a barrier below: the
        // warpgroup when the tile is stored, each warp alone in REDUCE passes.
        if constexpr (PASS == kReduce) ok = __all_sync(0xFFFFFFFFu, ok);
        else ok = named_bar_and(bar_id, 128, ok);
        if (!ok) break;
        if (rt == 0 && pending >= 0) {
          // The previous tile's bulk store has long finished reading its stage.
          bulk_wait_read_all();
          mbar_arrive_cnt(&empty[pending], kStoreRelease);
          pending = -1;
        }
        tc_fence_after();
        const uint32_t taddr = tmem + lane_off + ab * BN;
        // The update of chunk k (32 columns) of this thread's tile row: the
        // tensor-core accumulator, or for fp32 factors the CUDA-core chain.
        auto acc_at = [&](int k, float (&acc)[32]) {
          if constexpr (CDT == kF32) f32_update(W, row, valid, c0 + 32 * k, acc);
          else tmem_ld32(taddr + 32 * k, acc);
        };
        // Chunks kbeg .. kend-1 of the accumulator, loaded from tensor memory.
        auto chunk_loop = [&](int kbeg, int kend, auto&& body) {
          if constexpr (CDT == kF32) {
            for (int k = kbeg; k < kend; ++k) {
              float acc[32];
              acc_at(k, acc);
              body(k, acc);
            }
          } else {
            // One synchronous load per chunk: keeping the next chunk's load in
            // flight costs 32 registers, which the epilogue's arithmetic uses
            // better (measured 3-16 % faster per format without it).
            for (int k = kbeg; k < kend; ++k) {
              float acc[32];
              tmem_ld32(taddr + 32 * k, acc);
              body(k, acc);
            }
          }
        };

        RowCtx c;
        c.row = row;
        c.valid = valid;
        if (tma) {
          c.srow = stage_codes(s) + rt * G::kBoxRow;
          c.box_stride = 128 * G::kBoxRow;
          c.box_shift = is_gguf<FMT>() ? 16 : G::kBoxShift;
          c.swz = is_gguf<FMT>() ? 0u
                  : (G::kBoxRow == 128 ? static_cast<uint32_t>(rt & 7)
                     : (G::kBoxRow == 64 ? static_cast<uint32_t>((rt >> 1) & 3) : static_cast<uint32_t>((rt >> 2) & 1)));
        } else {
          c.srow = stage_codes(s) + rt * G::kPadRS;
          c.box_stride = 0;
          c.box_shift = 16;
          c.swz = 0u;
        }
        c.sscale = stage_scales(s) + rt * kScaleSlot;
        c.blk0 = (FMT == PIPER_FMT_NVFP4) ? c0 / 16 : c0 / 32;
        c.tile_col0 = c0;
        c.tile_cols = tcols;
        {
      if constexpr (FMT == PIPER_FMT_MXFP8_E4M3 || FMT == PIPER_FMT_MXFP8_E5M2 ||
                    FMT == PIPER_FMT_MXFP4) {
        chunk_loop(0, tcols / 32, [&](int k, const float (&acc)[32]) {
          if (!mx_chunk_fast<FMT, CDT>(W, c, k, acc)) {
            // The accumulator chunk is read again from tensor memory, so the
            // fast path need not keep it live.
            float acc2[32];
            acc_at(k, acc2);
            mx_chunk<FMT, CDT>(W, c, k, acc2);
          }
        });
        flush_tile_scales<FMT>(W, c);
      } else if constexpr (FMT == PIPER_FMT_NVFP4) {
        chunk_loop(0, tcols / 32, [&](int k, const float (&acc)[32]) {
          nvfp4_chunk<PASS, CDT>(W, c, k, acc, g_in, g_out, two_level, red_max);
        });
        if (tcols & 31) {  // trailing 16-column block
          float acc[32];
          const int k = tcols / 32;
          acc_at(k, acc);
          uint2 codes = *reinterpret_cast<const uint2*>(chunk_ptr(c, k));
          nvfp4_block<PASS, CDT>(W, c, c0 + 32 * k, acc, g_in, g_out, two_level, red_max, codes);
          if (PASS != kReduce) *reinterpret_cast<uint2*>(chunk_ptr(c, k)) = codes;
        }
        if constexpr (PASS != kReduce) flush_tile_scales<FMT>(W, c);
      } else if constexpr (FMT == PIPER_FMT_BNB4_NF4 || FMT == PIPER_FMT_BNB4_FP4) {
        // One 64-value block of _merge_quantize_kernel (_triton_bnb4_lora.py:163-313)
        // per pair of 32-column chunks: the block maximum from a first decode,
        // then each chunk decoded again and encoded.
        constexpr bool kNf4 = FMT == PIPER_FMT_BNB4_NF4;
        // Decode table per lane; the encode table: NF4 the same, FP4 its level
        // values (_fp4_level_value :78-105) per lane & 7.
        const float dec = __ldg(W.code16 + (lane & 15));
        const int l7 = lane & 7;
        const float lut = kNf4 ? dec
                               : (l7 == 0   ? 0.0f
                                  : l7 == 1 ? 0.0052083334885537624f
                                  : l7 == 2 ? 0.1666666716337204f
                                  : l7 == 3 ? 0.25f
                                  : l7 == 4 ? 0.3333333432674408f
                                  : l7 == 5 ? 0.5f
                                  : l7 == 6 ? 0.6666666865348816f
                                            : 1.0f);
        float tbl[16];
        bool sorted = true;
#pragma unroll
        for (int j = 0; j < 16; ++j) tbl[j] = __ldg(W.code16 + j);
#pragma unroll
        for (int j = 0; j < 15; ++j) sorted = sorted && !(tbl[j + 1] < tbl[j]);
        const bool sr = (W.flags & PIPER_FLAG_STOCHASTIC) != 0u;
        const PhiloxKey key = philox_key(W.k0, W.k1);
        const int nbr = W.N >> 6;
        for (int k = 0; k < tcols / 32; k += 2) {
          const int col = c0 + 32 * k;
          const int64_t bi = static_cast<int64_t>(row) * nbr + (col >> 6);
          float scale = 0.0f;
          if (valid) {
            if (W.ncode != nullptr) {
              const uint32_t q = reinterpret_cast<const uint8_t*>(W.scale)[bi];
              scale = fmaf(__ldg(W.ncode + q), __ldg(W.nabs + (bi >> 8)), __ldg(W.noff));  // code * absmax + offset
            } else {
              scale = reinterpret_cast<const float*>(W.scale)[bi];
            }
          }
          float amax = 0.0f;
#pragma unroll
          for (int h = 0; h < 2; ++h) {
            const uint4 v4 = *reinterpret_cast<const uint4*>(chunk_ptr(c, k + h));
            const uint32_t wq[4] = {v4.x, v4.y, v4.z, v4.w};
            float acc[32], m[32];
            acc_at((k + h), acc);
            bnb4_merged32<CDT>(wq, scale, dec, W.strength, acc, m);
#pragma unroll
            for (int i = 0; i < 32; ++i) amax = fmaxf(amax, fabsf(m[i]));
          }
          if (valid) {
            if (W.ncode != nullptr) W.qmax[bi] = __float_as_uint(amax);  // raw maxima for the nested pass
            else reinterpret_cast<float*>(W.scale)[bi] = amax;
          }
          const float safe = amax == 0.0f ? 1.0f : amax;
          for (int h = 0; h < 2; ++h) {  // codes still in shared memory: the chunk is rewritten below
            const uint4 v4 = *reinterpret_cast<const uint4*>(chunk_ptr(c, k + h));
            const uint32_t wq[4] = {v4.x, v4.y, v4.z, v4.w};
            float acc[32], m[32];
            acc_at((k + h), acc);
            bnb4_merged32<CDT>(wq, scale, dec, W.strength, acc, m);
            const uint64_t off0 =
                W.offset_base + static_cast<uint64_t>(row) * static_cast<uint64_t>(W.N) + col + 32 * h;
            uint32_t out[4];
            if (kNf4 && !sorted) {  // uniform per item: the reference's binary search, element by element
#pragma unroll
              for (int w = 0; w < 4; ++w) out[w] = 0u;
#pragma unroll
              for (int i = 0; i < 32; ++i) {
                const float v = fminf(fmaxf(div_full(m[i], safe), -1.0f), 1.0f);
                const int code = nf4_code_search(v, W.code16, sr, key, off0 + i);
                const int j = i >> 1;
                out[j >> 2] |= static_cast<uint32_t>(code & 15) << ((j & 3) * 8 + ((i & 1) ? 0 : 4));
              }
            } else if (sr) {
              bnb4_encode32<FMT, true>(m, safe, lut, tbl, key, off0, out);
            } else {
              bnb4_encode32<FMT, false>(m, safe, lut, tbl, key, off0, out);
            }
            *reinterpret_cast<uint4*>(chunk_ptr(c, k + h)) = make_uint4(out[0], out[1], out[2], out[3]);
          }
        }
      } else if constexpr (FMT == PIPER_FMT_GGUF_Q8_0 || FMT == PIPER_FMT_GGUF_Q4_0) {
        chunk_loop(0, tcols / 32, [&](int k, const float (&acc)[32]) { gguf_chunk<FMT, CDT>(W, c, k, acc); });
      } else {
        // ------------------------------------------- FP8 / INT8 (affine) paths
        constexpr bool kInt8 = base_fmt(FMT) == PIPER_FMT_INT8;
        constexpr bool kE4 = base_fmt(FMT) == PIPER_FMT_FP8_E4M3;
        constexpr int kFlv = flavor_of(FMT);
        constexpr float kLimit = kE4 ? 448.0f : 57344.0f;
        const bool asym = (W.flags & PIPER_FLAG_ASYMMETRIC) != 0u;
        const int qmin = (W.flags & PIPER_FLAG_REDUCE_RANGE) ? -64 : -128;
        const int qmax = (W.flags & PIPER_FLAG_REDUCE_RANGE) ? 63 : 127;
        const PhiloxKey key = philox_key(W.k0, W.k1);
        const int nchunks = (tcols + 31) / 32;
        if constexpr (kPackedRow) {
          // Per-row TorchAO FP8 / INT8: packed decode and merge; the maxima
          // sweep keeps the merged values unrounded and flags rows holding a
          // NaN or an infinity, whose encode takes the general clamped path.
          chunk_loop(0, nchunks, [&](int k, const float (&acc)[32]) {
            uint32_t wv[8];
            load_chunks32(c, k, wv);
            float merged[32];
            const int nvalid = min(32, tcols - 32 * k);
            if (!enc_phase) {
              if constexpr (kInt8) int8_merged_pk<CDT, false>(wv, acc, f_s_in, f_z_in, W.scale_dt, W.strength, merged);
              else fp8_merged_pk<kE4, CDT, false>(wv, acc, f_s_in, W.strength, merged);
              if (nvalid < 32) {  // columns past the row end are zero, which leaves the maxima unchanged
#pragma unroll
                for (int i = 0; i < 32; ++i) merged[i] = i < nvalid ? merged[i] : 0.0f;
              }
              if (valid) {
                if constexpr (kInt8) {
                  float hi = tree3(merged, max3_nan), lo = tree3(merged, min3_nan);
                  if (!(hi <= 3.40282347e38f && lo >= -3.40282347e38f)) {  // a NaN or an infinity
                    red_special = true;
                    hi = tree3(merged, max3f);
                    lo = tree3(merged, min3f);
                  }
                  red_max = fmaxf(red_max, hi);
                  red_nmin = fmaxf(red_nmin, -lo);
                } else {
                  float cm = tree3(merged, max3_abs_nan);
                  if (!(cm <= 3.40282347e38f)) {  // a NaN or an infinity
                    red_special = true;
                    cm = tree3(merged, max3_abs);
                  }
                  red_max = fmaxf(red_max, cm);
                }
              }
            } else {
              if constexpr (kInt8) int8_merged_pk<CDT, true>(wv, acc, f_s_in, f_z_in, W.scale_dt, W.strength, merged);
              else fp8_merged_pk<kE4, CDT, true>(wv, acc, f_s_in, W.strength, merged);
              uint32_t out[8] = {0u, 0u, 0u, 0u, 0u, 0u, 0u, 0u};
              if (valid) {
                const uint64_t off0 =
                    W.offset_base + static_cast<uint64_t>(row) * static_cast<uint64_t>(W.N) + c0 + 32 * k;
                const bool sr_on = (W.flags & PIPER_FLAG_STOCHASTIC) != 0u;
                if (!f_special) {
                  if constexpr (kInt8) {
                    if (sr_on) int8_encode32(merged, f_q, qmin, qmax, W.scale_dt, true, key, off0, out);
                    else int8_encode_rtn_finite(merged, f_q, qmin, qmax, W.scale_dt, out);
                  } else {
                    if (sr_on) fp8_encode_sr_finite<kE4>(merged, f_s, key, off0, out);
                    else fp8_encode_rtn_finite<kE4>(merged, f_s, out);
                  }
                } else {
                  if (nvalid < 32) {
#pragma unroll
                    for (int i = 0; i < 32; ++i) merged[i] = i < nvalid ? merged[i] : 0.0f;
                  }
                  if constexpr (kInt8) int8_encode32(merged, f_q, qmin, qmax, W.scale_dt, sr_on, key, off0, out);
                  else if (sr_on) fp8_encode_sr<kE4>(merged, f_s, kLimit, key, off0, out);
                  else fp8_encode_rtn<kE4>(merged, f_s, kLimit, out);
                }
              }
              store_chunks32(c, k, out);
            }
          });
        } else if constexpr (PASS == kFused) {
          // Per-row layout: one quantization block per row, qparams on chip.
          chunk_loop(0, nchunks, [&](int k, const float (&acc)[32]) {
            float merged[32];
            affine_merged_u<FMT, CDT>(W, c, k, acc, f_s_in, f_z_in, merged);
            const int nvalid = min(32, tcols - 32 * k);
            if (nvalid < 32) {
              // Columns past the row end are zero, which leaves the maxima unchanged.
#pragma unroll
              for (int i = 0; i < 32; ++i) merged[i] = i < nvalid ? merged[i] : 0.0f;
            }
            if (!enc_phase) {
              if (valid) {
                if constexpr (kInt8) {
                  red_max = fmaxf(red_max, tree_max(merged));
                  red_nmin = fmaxf(red_nmin, -tree_min(merged));
                } else {
                  red_max = fmaxf(red_max, tree_max_abs(merged));
                }
              }
            } else {
              uint32_t out[8] = {0u, 0u, 0u, 0u, 0u, 0u, 0u, 0u};
              if (valid) {
                const uint64_t off0 =
                    W.offset_base + static_cast<uint64_t>(row) * static_cast<uint64_t>(W.N) + c0 + 32 * k;
                const bool sr_on = (W.flags & PIPER_FLAG_STOCHASTIC) != 0u;
                if constexpr (kInt8) {
                  if constexpr (kFlv != kTorchao) flavor_int8_encode32<CDT>(kFlv, merged, f_q.scale, sr_on, key, off0, out);
                  else int8_encode32(merged, f_q, qmin, qmax, W.scale_dt, sr_on, key, off0, out);
                } else if constexpr (kFlv == kQuanto) {
                  quanto_fp8_encode32<kE4, CDT>(merged, f_s, kLimit, sr_on, key, off0, out);
                } else if (sr_on) {
                  fp8_encode_sr<kE4>(merged, f_s, kLimit, key, off0, out);
                } else {
                  fp8_encode_rtn<kE4>(merged, f_s, kLimit, out);
                }
              }
              store_chunks32(c, k, out);
            }
          });
        } else if constexpr (PASS == kLocal) {
          // Groups of W.group (multiple of 32, dividing the tile width) are local.
          const int gch = W.group / 32;
          for (int g0 = 0; g0 < nchunks; g0 += gch) {
            float gmax = 0.0f, gmin = 0.0f, gabs = 0.0f;
            float s_in = 1.0f;
            int z_in = 0;
            if (valid) {
              qp_load<FMT, PASS>(W, qparam_index(W, row, c0 + 32 * g0), qc);
              s_in = qc.s_in;
              z_in = qc.z_in;
            }
            for (int k = g0; k < g0 + gch; ++k) {
              float acc[32], merged[32];
              acc_at(k, acc);
              affine_merged_u<FMT, CDT>(W, c, k, acc, s_in, z_in, merged);
              if constexpr (kInt8) {
                gmax = fmaxf(gmax, tree_max(merged));
                gmin = fminf(gmin, tree_min(merged));
              } else {
                gabs = fmaxf(gabs, tree_max_abs(merged));
              }
            }
            const int qp = qparam_index(W, row, c0 + 32 * g0);
            if constexpr (kInt8) {
              const Int8Q q = int8_qparams<CDT>(gmin, gmax, asym, qmin, qmax, W.scale_dt);
              if (valid) {
                store_scale_dt(W.scale, qp, W.scale_dt, q.scale);
                if (W.zp != nullptr) W.zp[qp] = static_cast<int8_t>(q.zp);
              }
              for (int k = g0; k < g0 + gch; ++k) {
                float acc[32], merged[32];
                acc_at(k, acc);
                affine_merged_u<FMT, CDT>(W, c, k, acc, s_in, z_in, merged);
                uint32_t out[8];
                const uint64_t off0 = W.offset_base +
                                      static_cast<uint64_t>(row) * static_cast<uint64_t>(W.N) +
                                      c0 + 32 * k;
                int8_encode32(merged, q, qmin, qmax, W.scale_dt, (W.flags & PIPER_FLAG_STOCHASTIC) != 0u,
                              key, off0, out);
                store_chunks32(c, k, out);
              }
            } else {
              const float s = fp8_new_scale<CDT>(gabs, kLimit);
              if (valid) reinterpret_cast<float*>(W.scale)[qp] = s;
              for (int k = g0; k < g0 + gch; ++k) {
                float acc[32], merged[32];
                acc_at(k, acc);
                affine_merged_u<FMT, CDT>(W, c, k, acc, s_in, z_in, merged);
                uint32_t out[8] = {0u, 0u, 0u, 0u, 0u, 0u, 0u, 0u};
                const uint64_t off0 = W.offset_base +
                                      static_cast<uint64_t>(row) * static_cast<uint64_t>(W.N) +
                                      c0 + 32 * k;
                if (W.flags & PIPER_FLAG_STOCHASTIC) {
                  fp8_encode_sr<kE4>(merged, s, kLimit, key, off0, out);
                } else {
                  fp8_encode_rtn<kE4>(merged, s, kLimit, out);
                }
                store_chunks32(c, k, out);
              }
            }
          }
        } else {
          chunk_loop(0, nchunks, [&](int k, const float (&acc)[32]) {
            float merged[32];
            const int col = c0 + 32 * k;
            const int nvalid = min(32, tcols - 32 * k);
            if constexpr (kFlv == kQuanto) {
              if (W.col_axis) {
                quanto_column_chunk<FMT, PASS, CDT>(W, c, k, col, nvalid, acc, lane, key);
                return;
              }
            }
            if constexpr (kFlv == kTorchao) {
              // TorchAO FP8 / INT8, a full chunk inside one quantization block
              // (per-row weights too small for the fused pass, per-tensor,
              // groups wider than a tile): the packed decode and merge of the
              // fused sweeps, block qparams computed once per block.
              if (nvalid == 32 && (W.nq_row == 0 || (W.group >= 32 && (col % W.group) + 32 <= W.group))) {
                uint32_t out[8] = {0u, 0u, 0u, 0u, 0u, 0u, 0u, 0u};
                if (valid) {
                  const int qp = qparam_index(W, row, col);
                  qp_load<FMT, PASS>(W, qp, qc);
                  uint32_t wv[8];
                  load_chunks32(c, k, wv);
                  const bool owner = W.nq_row == 0 ? (row == 0 && col == 0) : (col % W.group == 0);
                  if constexpr (PASS == kReduce) {
                    // Unrounded merged values: rounding is monotone, so the
                    // rounded block maxima are the maxima of the rounded values.
                    if constexpr (kInt8) int8_merged_pk<CDT, false>(wv, acc, qc.s_in, qc.z_in, W.scale_dt, W.strength, merged);
                    else fp8_merged_pk<kE4, CDT, false>(wv, acc, qc.s_in, W.strength, merged);
                    if (qp != red_qp) {
                      flush_reduce();
                      red_qp = qp;
                    }
                    if (owner) {  // first touch of the block saves its input qparams
                      W.old_scale[qp] = qc.s_in;
                      if constexpr (kInt8) W.old_zp[qp] = qc.z_in;
                    }
                    if constexpr (kInt8) {
                      red_max = fmaxf(red_max, round_dt<CDT>(tree3(merged, max3f)));
                      red_nmin = fmaxf(red_nmin, -round_dt<CDT>(tree3(merged, min3f)));
                    } else {
                      red_max = fmaxf(red_max, round_dt<CDT>(tree3(merged, max3_abs)));
                    }
                    return;
                  } else {
                    if (qp != enc_qp) {
                      enc_qp = qp;
                      if constexpr (kInt8) enc_q = int8_qparams<CDT>(-qc.nmin, qc.qmax, asym, qmin, qmax, W.scale_dt);
                      else enc_s = fp8_new_scale<CDT>(qc.qmax, kLimit);
                    }
                    if (owner) {
                      if constexpr (kInt8) {
                        store_scale_dt(W.scale, qp, W.scale_dt, enc_q.scale);
                        if (W.zp != nullptr) W.zp[qp] = static_cast<int8_t>(enc_q.zp);
                      } else {
                        store_scale<FMT>(W, qp, enc_s);
                      }
                    }
                    if constexpr (kInt8) int8_merged_pk<CDT, true>(wv, acc, qc.s_in, qc.z_in, W.scale_dt, W.strength, merged);
                    else fp8_merged_pk<kE4, CDT, true>(wv, acc, qc.s_in, W.strength, merged);
                    const uint64_t off0 =
                        W.offset_base + static_cast<uint64_t>(row) * static_cast<uint64_t>(W.N) + col;
                    const bool sr_on = (W.flags & PIPER_FLAG_STOCHASTIC) != 0u;
                    // Finite values under finite block maxima stay within the
                    // range the shortcut encoders assume (|m| <= the maxima).
                    const bool finite = tree3(merged, max3_abs_nan) <= 3.40282347e38f &&
                                        qc.qmax <= 3.40282347e38f && (!kInt8 || qc.nmin <= 3.40282347e38f);
                    if constexpr (kInt8) {
                      if (!sr_on && finite) int8_encode_rtn_finite(merged, enc_q, qmin, qmax, W.scale_dt, out);
                      else int8_encode32(merged, enc_q, qmin, qmax, W.scale_dt, sr_on, key, off0, out);
                    } else if (finite) {
                      if (sr_on) fp8_encode_sr_finite<kE4>(merged, enc_s, key, off0, out);
                      else fp8_encode_rtn_finite<kE4>(merged, enc_s, out);
                    } else if (sr_on) {
                      fp8_encode_sr<kE4>(merged, enc_s, kLimit, key, off0, out);
                    } else {
                      fp8_encode_rtn<kE4>(merged, enc_s, kLimit, out);
                    }
                  }
                }
                if constexpr (PASS == kEncode) store_chunks32(c, k, out);
                return;
              }
            }
            // A chunk whose valid columns all lie in one quantization block
            // (the tail chunk of a row included) decodes with one scale.
            if (W.nq_row == 0 || (W.group >= 32 && (col % W.group) + nvalid <= W.group)) {
              float s_in = 1.0f;
              int z_in = 0;
              if (valid) {
                qp_load<FMT, PASS>(W, qparam_index(W, row, col), qc);
                s_in = qc.s_in;
                z_in = qc.z_in;
              }
              affine_merged_u<FMT, CDT>(W, c, k, acc, s_in, z_in, merged);
            } else {
              float scale_in[32];
              int zp_in[32];
              affine_inputs<FMT, PASS>(W, c, col, scale_in, zp_in, qc);
              affine_merged<FMT, CDT>(W, c, k, acc, scale_in, zp_in, merged);
            }
            if constexpr (PASS == kReduce) {
              const bool uniform_chunk =
                  W.nq_row == 0 || (W.group >= 32 && (col % W.group) + 32 <= W.group);
              if (valid && uniform_chunk && nvalid == 32) {
                const int qp = qparam_index(W, row, col);
                if (qp != red_qp) {
                  flush_reduce();
                  red_qp = qp;
                }
                // First touch of a quantization block saves its input qparams.
                if (W.nq_row == 0 ? (row == 0 && col == 0) : (col % W.group == 0)) {
                  if (kInt8) {
                    W.old_scale[qp] = load_scale_dt(W.scale, qp, W.scale_dt);
                    W.old_zp[qp] = W.zp != nullptr ? static_cast<int>(W.zp[qp]) : 0;
                  } else {
                    W.old_scale[qp] = load_scale<FMT>(W, qp);
                  }
                }
                if constexpr (kInt8) {
                  red_max = fmaxf(red_max, tree_max(merged));
                  red_nmin = fmaxf(red_nmin, -tree_min(merged));
                } else {
                  red_max = fmaxf(red_max, tree_max_abs(merged));
                }
              } else if (valid) {
#pragma unroll
                for (int i = 0; i < 32; ++i) {
                  if (i < nvalid) {
                    const int qp = qparam_index(W, row, col + i);
                    if (qp != red_qp) {
                      flush_reduce();
                      red_qp = qp;
                      if (W.nq_row == 0 ? (row == 0 && col + i == 0) : ((col + i) % W.group == 0)) {
                        if (kInt8) {
                          W.old_scale[qp] = load_scale_dt(W.scale, qp, W.scale_dt);
                          W.old_zp[qp] = W.zp != nullptr ? static_cast<int>(W.zp[qp]) : 0;
                        } else {
                          W.old_scale[qp] = load_scale<FMT>(W, qp);
                        }
                      }
                    }
                    if (kInt8) {
                      red_max = fmaxf(red_max, merged[i]);
                      red_nmin = fmaxf(red_nmin, -merged[i]);
                    } else {
                      red_max = fmaxf(red_max, fabsf(merged[i]));
                    }
                  }
                }
              }
            } else {  // kEncode
              uint32_t out[8] = {0u, 0u, 0u, 0u, 0u, 0u, 0u, 0u};
              const uint64_t off0 =
                  W.offset_base + static_cast<uint64_t>(row) * static_cast<uint64_t>(W.N) + col;
              const bool sr_on = (W.flags & PIPER_FLAG_STOCHASTIC) != 0u;
              const bool uniform_chunk =
                  W.nq_row == 0 || (W.group >= 32 && (col % W.group) + nvalid <= W.group);
              if (valid && uniform_chunk) {
                // One quantization block covers the whole chunk (per-row / per-tensor).
                const int qp = qparam_index(W, row, col);
                qp_load<FMT, PASS>(W, qp, qc);
                const float qmx = qc.qmax;
                const bool owner = W.nq_row == 0 ? (row == 0 && col == 0) : (col % W.group == 0);
                if constexpr (kInt8) {
                  Int8Q q;
                  if constexpr (kFlv == kTorchao) {
                    q = int8_qparams<CDT>(-qc.nmin, qmx, asym, qmin, qmax, W.scale_dt);
                  } else {
                    q.scale = flavor_scale<CDT>(kFlv, fmaxf(qmx, qc.nmin), 127.0f);
                    q.zp = 0;
                  }
                  if (owner) {
                    store_scale_dt(W.scale, qp, W.scale_dt, q.scale);
                    if (W.zp != nullptr) W.zp[qp] = static_cast<int8_t>(q.zp);
                  }
                  if constexpr (kFlv == kTorchao) int8_encode32(merged, q, qmin, qmax, W.scale_dt, sr_on, key, off0, out);
                  else flavor_int8_encode32<CDT>(kFlv, merged, q.scale, sr_on, key, off0, out);
                } else {
                  const float s = kFlv == kQuanto ? flavor_scale<CDT>(kQuanto, qmx, kLimit)
                                                  : fp8_new_scale<CDT>(qmx, kLimit);
                  if (owner) store_scale<FMT>(W, qp, s);
                  if constexpr (kFlv == kQuanto) {
                    quanto_fp8_encode32<kE4, CDT>(merged, s, kLimit, sr_on, key, off0, out);
                  } else if (sr_on) {
                    fp8_encode_sr<kE4>(merged, s, kLimit, key, off0, out);
                  } else {
                    fp8_encode_rtn<kE4>(merged, s, kLimit, out);
                  }
                }
              } else if (valid) {
                int cur_qp = -1;
                Int8Q q;
                q.scale = 1.0f;
                q.zp = 0;
                float s = 1.0f;
                for (int i = 0; i < nvalid; ++i) {
                  const int qp = qparam_index(W, row, col + i);
                  if (qp != cur_qp) {
                    cur_qp = qp;
                    const float qmx = __uint_as_float(W.qmax[qp]);
                    if (kInt8) {
                      const float qmn = -__uint_as_float(W.qmin[qp]);
                      q = int8_qparams<CDT>(qmn, qmx, asym, qmin, qmax, W.scale_dt);
                    } else {
                      s = fp8_new_scale<CDT>(qmx, kLimit);
                    }
                    const bool owner =
                        W.nq_row == 0 ? (row == 0 && col + i == 0) : ((col + i) % W.group == 0);
                    if (owner) {
                      if (kInt8) {
                        store_scale_dt(W.scale, qp, W.scale_dt, q.scale);
                        if (W.zp != nullptr) W.zp[qp] = static_cast<int8_t>(q.zp);
                      } else {
                        reinterpret_cast<float*>(W.scale)[qp] = s;
                      }
                    }
                  }
                  float mi = merged[0];
#pragma unroll
                  for (int j = 1; j < 32; ++j) mi = (j == i) ? merged[j] : mi;
                  uint32_t code;
                  if (kInt8) {
                    code = int8_encode(mi, q, qmin, qmax, W.scale_dt, sr_on, key, off0 + i);
                  } else {
                    const float x = fminf(fmaxf(div_full(mi, s), -kLimit), kLimit);
                    code = sr_on ? sr_fp8<kE4>(x, kLimit, key, off0 + i) : enc_fp8<kE4>(x);
                  }
                  out[i >> 2] |= code << ((i & 3) * 8);
                }
              }
              store_chunks32(c, k, out);
            }
          });
        }
      }
        }
        // Accumulator drained: hand it back to the tensor core.
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&aempty[ab]);

        // ---- write the tile back (in place) and release the stage.
        const bool stores = PASS == kLocal || PASS == kEncode || enc_phase;
        if (stores && tma) {
          fence_proxy_async_smem();
          named_bar_sync(bar_id, 128);
          if (rt == 0) {
            const int64_t off = code_off<FMT>(c0);
            for (int j = 0; j < G::kBoxes; ++j) {
              if (off + j * G::kBoxRow >= W.row_bytes) break;
              const int x = static_cast<int>(off + j * G::kBoxRow);
              tma_store_2d(&W.tmap, is_gguf<FMT>() ? x / 8 : x, g.row0, stage_codes(s) + j * 128 * G::kBoxRow);
            }
            bulk_commit();
            pending = s;
          }
        } else if (!stores) {
          __syncwarp();
          if (lane == 0) mbar_arrive(&empty[s]);
        } else {
          named_bar_sync(bar_id, 128);
          {
            // Coalesced write-back of the padded layout.
            const int64_t off = code_off<FMT>(c0);
            const int nbytes = static_cast<int>(code_off<FMT>(c0 + tcols) - off);
            const int64_t m = W.row_bytes | off | nbytes | static_cast<int64_t>(reinterpret_cast<uintptr_t>(W.q));
            const int gran = (m & 15) == 0 ? 16 : ((m & 3) == 0 ? 4 : 1);
            const int per = nbytes / gran;
            uint8_t* dst0 = W.q + static_cast<int64_t>(g.row0) * W.row_bytes + off;
            const uint8_t* base = stage_codes(s);
            for (int k = rt; k < rows_here * per; k += 128) {
              const int r = k / per;
              const int i = k - r * per;
              const uint8_t* src = base + r * G::kPadRS + i * gran;
              uint8_t* dst = dst0 + static_cast<int64_t>(r) * W.row_bytes + i * gran;
              if (gran == 16) *reinterpret_cast<uint4*>(dst) = *reinterpret_cast<const uint4*>(src);
              else if (gran == 4) *reinterpret_cast<uint32_t*>(dst) = *reinterpret_cast<const uint32_t*>(src);
              else *dst = *src;
            }
            named_bar_sync(bar_id, 128);
          }
          if (rt == 0) {
            if (pending >= 0) {
              bulk_wait_read_all();
              mbar_arrive_cnt(&empty[pending], kStoreRelease);
              pending = -1;
            }
            mbar_arrive_cnt(&empty[s], kStoreRelease);
          }
        }
      }

      // ---- REDUCE: publish this item's running maxima.
      if constexpr (PASS == kReduce) {
        if constexpr (FMT == PIPER_FMT_NVFP4) {
          const float m = warp_max(red_max);
          if (lane == 0) atomic_max_nonneg(W.qmax, m);
        } else {
          if (W.nq_row == 0) {
            const float m = warp_max(red_max);
            const float n = warp_max(red_nmin);
            if (lane == 0) {
              atomic_max_nonneg(&W.qmax[0], m);
              if (base_fmt(FMT) == PIPER_FMT_INT8) atomic_max_nonneg(&W.qmin[0], n);
            }
          } else {
            flush_reduce();
          }
        }
      }
      // ---- NVFP4: zero swizzle padding columns and publish the new global scale.
      if constexpr (FMT == PIPER_FMT_NVFP4 && PASS == kLocal) {
        if ((W.flags & PIPER_FLAG_SWIZZLED) && g.col_end == W.N && wg == owner) {
          const int padded = align_up(W.scale_cols, 4);
          uint8_t* scale8 = reinterpret_cast<uint8_t*>(W.scale);
          for (int pc = W.scale_cols; pc < padded; ++pc) scale8[swizzled_index(row, pc, W.scale_cols)] = 0u;
        }
        if (two_level && local == 0 && rt == 0 && wg == owner) *W.gscale = g_out;
      }
    }
    if (rt == 0) bulk_wait_all();  // bulk stores complete before the CTA exits
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}



// Self-test of the bounded waits: one thread waits on an mbarrier that nothing
// arrives on. The wait gives up after kWaitLimitNs, records kStatusTimeoutLoad
// in the status word and the kernel returns; nothing faults or hangs.
__global__ void selftest_wait_kernel() {
  __shared__ uint64_t bar;
  if (threadIdx.x == 0) {
    mbar_init(&bar, 1);
    fence_mbar_init();
    mbar_wait(&bar, 0u, kStatusTimeoutLoad);
  }
}
}  // namespace pm


// =================================================================== host side
namespace {

thread_local std::string g_last_error;
std::atomic<uint64_t> g_launches{0};

int fail(int code, const std::string& msg) {
  g_last_error = msg;
  return code;
}

using pm::DevWeight;
using pm::LaunchParams;

// Bytes of codes a two-pass launch group covers, so that its ENCODE launch
// re-reads them from L2 (126 MB on B200).
constexpr int64_t kL2GroupBytes = 96ll << 20;

// Code bytes of `cols` columns (host mirror of code_bytes<FMT>).
int host_code_bytes(int fmt, int cols) {
  switch (fmt) {
    case PIPER_FMT_MXFP4:
    case PIPER_FMT_NVFP4:
    case PIPER_FMT_BNB4_NF4:
    case PIPER_FMT_BNB4_FP4: return cols / 2;
    case PIPER_FMT_GGUF_Q8_0: return cols / 32 * 34;
    case PIPER_FMT_GGUF_Q4_0: return cols / 32 * 18;
    default: return cols;
  }
}

// Shared-memory bytes of one stage's code slot (host mirror of TileGeom::kCodeSlot).
int ws_code_slot(int fmt, int bn) {
  const int rb = host_code_bytes(fmt, bn);
  const int rs = pm::align_up(rb, 16) + 16;
  return pm::align_up(128 * std::max(rs, rb), 1024);
}

// Shared-memory pipeline of one launch: code stages, A stages, B strips.
struct PipeCfg {
  int sc = 0, sa = 0, nbb = 0;
};

// Deepest rings that fit the per-CTA shared-memory limit, in order of
// preference: many code stages (they hold the HBM traffic in flight), then A
// stages (refilled as soon as the tensor core has read them), then a second B
// strip (hides the strip load at item boundaries).
PipeCfg plan_pipe(int fmt, int bn, int kp) {
  const int cs = pm::ws_code_stage_bytes(ws_code_slot(fmt, bn));
  const int as = pm::ws_a_stage_bytes(kp, bn);
  const int bs = pm::ws_b_buf_bytes(kp);
  const int avail = pm::kSmemLimit - 1024 - pm::kTailBytes;
  const int pref[][3] = {{2, 3, 6}, {2, 2, 6}, {1, 2, 6}, {2, 2, 4}, {1, 2, 4}, {1, 2, 3}, {1, 1, 2}};
  for (const auto& q : pref) {
    const int rest = avail - q[0] * bs - q[1] * as;
    if (rest <= 0) continue;
    const int sc = std::min(pm::kMaxStages, rest / cs);
    if (sc >= q[2]) return {sc, q[1], q[0]};
  }
  return {};
}

struct Plan {
  int bn = 128;
  bool two_pass = false;
  bool fused = false;  // per-row FP8 / INT8: one kFused launch, no workspace
  int nq = 0;          // quantization blocks held in the workspace
  int nq_row = 0;      // blocks per row (0 = per tensor)
  int group = 0;
  int flavor = 0;      // pm::Flavor of an FP8 / INT8 weight
  bool col_axis = false;  // Quanto last-axis scales
  size_t ws_off = 0;
};

bool is_fp_dt(int dt) { return dt == PIPER_DT_BF16 || dt == PIPER_DT_F16 || dt == PIPER_DT_F32; }

int64_t row_bytes_of(const piper_merge_desc& d) {
  switch (d.format) {
    case PIPER_FMT_MXFP4:
    case PIPER_FMT_NVFP4:
    case PIPER_FMT_BNB4_NF4:
    case PIPER_FMT_BNB4_FP4: return d.cols / 2;
    case PIPER_FMT_GGUF_Q8_0: return d.cols / 32 * 34;
    case PIPER_FMT_GGUF_Q4_0: return d.cols / 32 * 18;
    default: return d.cols;
  }
}

// bitsandbytes LLM.int8 and Quanto qbytes weights run on the INT8 / FP8
// kernels with their own arithmetic (pm::Flavor); TorchAO FP8 scales are fp32.
// Rewrites `d` to the kernel's format and stored scale dtype.
int normalize(piper_merge_desc& d, int& flavor, bool& col_axis) {
  flavor = pm::kTorchao;
  col_axis = false;
  const bool per_row = d.block_rows == 1 && d.block_cols == d.cols;
  const bool per_tensor = d.block_rows == d.rows && d.block_cols == d.cols;
  const bool per_col = d.block_rows == d.rows && d.block_cols == 1;
  switch (d.format) {
    case PIPER_FMT_FP8_E4M3:
    case PIPER_FMT_FP8_E5M2:
      d.scale_dtype = PIPER_DT_F32;
      break;
    case PIPER_FMT_BNB8:  // _triton_bnb8_lora.py:145-190
      if (d.compute_dtype != PIPER_DT_F16)
        return fail(PIPER_MERGE_EINVAL, "bitsandbytes 8-bit merge expects float16 LoRA factors.");
      if (!per_row) return fail(PIPER_MERGE_EINVAL, "bitsandbytes 8-bit merge expects one SCB value per row.");
      if (d.zero_point != nullptr || (d.flags & (PIPER_FLAG_ASYMMETRIC | PIPER_FLAG_REDUCE_RANGE)))
        return fail(PIPER_MERGE_EINVAL, "bitsandbytes 8-bit storage is symmetric over [-127, 127].");
      d.format = PIPER_FMT_INT8;
      d.scale_dtype = PIPER_DT_F32;
      flavor = pm::kBnb;
      break;
    case PIPER_FMT_QUANTO_INT8:  // _triton_quanto_lora.py:184-200, 220-343
    case PIPER_FMT_QUANTO_FP8_E4M3:
    case PIPER_FMT_QUANTO_FP8_E5M2:
      if (!per_row && !per_tensor && !per_col)
        return fail(PIPER_MERGE_EINVAL, "Quanto qbytes merge expects a scalar scale, one scale per row for axis 0, "
                                        "or one scale per column for the last axis.");
      if (per_col) {  // two passes over the whole weight, one workspace slot per column
        col_axis = true;
        d.block_rows = d.rows;
        d.block_cols = d.cols;
      }
      if (d.zero_point != nullptr || (d.flags & (PIPER_FLAG_ASYMMETRIC | PIPER_FLAG_REDUCE_RANGE)))
        return fail(PIPER_MERGE_EINVAL, "Quanto qbytes storage is symmetric.");
      d.format = d.format == PIPER_FMT_QUANTO_INT8 ? PIPER_FMT_INT8
                 : d.format == PIPER_FMT_QUANTO_FP8_E4M3 ? PIPER_FMT_FP8_E4M3 : PIPER_FMT_FP8_E5M2;
      d.scale_dtype = d.compute_dtype;  // scales share the factors' dtype
      flavor = pm::kQuanto;
      break;
    default:
      break;
  }
  return PIPER_MERGE_OK;
}

// Argument checks mirror the reference launchers (e.g. _triton_mx_lora.py:348-393).
int validate(const piper_merge_desc& d, Plan& p) {
  if (d.rows <= 0 || d.cols <= 0 || d.rank <= 0)
    return fail(PIPER_MERGE_EINVAL, "merge requires non-empty weight and factors.");
  if (d.rows > (1 << 30) || d.cols > (1 << 30) || d.rows * d.cols > (int64_t(1) << 40))
    return fail(PIPER_MERGE_EINVAL, "weight dimensions are too large.");
  if (d.rank > pm::kMaxRank)
    return fail(PIPER_MERGE_EINVAL, "LoRA rank above 256 is not supported by the sm_100a merge (rank " +
                                        std::to_string(d.rank) + ").");
  if (d.qdata == nullptr || d.b == nullptr || d.a == nullptr)
    return fail(PIPER_MERGE_EINVAL, "null qdata or factor pointer.");
  if (!is_fp_dt(d.compute_dtype))
    return fail(PIPER_MERGE_EINVAL, "merge supports float16, bfloat16, and float32 LoRA factors.");
  p = Plan();
  switch (d.format) {
    case PIPER_FMT_MXFP8_E4M3:
    case PIPER_FMT_MXFP8_E5M2:
    case PIPER_FMT_MXFP4:
      if (d.cols % 32 != 0) return fail(PIPER_MERGE_EINVAL, "MX merge requires columns divisible by 32.");
      if (d.compute_dtype != PIPER_DT_BF16 && d.compute_dtype != PIPER_DT_F32)
        return fail(PIPER_MERGE_EINVAL, "MX merge supports bfloat16 and float32 weights and factors.");
      if (d.scale_mode < 0 || d.scale_mode > 3)
        return fail(PIPER_MERGE_EINVAL, "Unsupported MX scaling mode id " + std::to_string(d.scale_mode) + ".");
      if (d.scale == nullptr) return fail(PIPER_MERGE_EINVAL, "MX merge requires E8M0 scales.");
      break;
    case PIPER_FMT_NVFP4:
      if (d.cols % 16 != 0) return fail(PIPER_MERGE_EINVAL, "NVFP4 merge requires columns divisible by 16.");
      if (d.compute_dtype != PIPER_DT_BF16 && d.compute_dtype != PIPER_DT_F32)
        return fail(PIPER_MERGE_EINVAL, "NVFP4 merge supports bfloat16 and float32 LoRA factors.");
      if (d.scale == nullptr) return fail(PIPER_MERGE_EINVAL, "NVFP4 merge requires E4M3 block scales.");
      if (d.global_scale != nullptr) {
        p.two_pass = true;
        p.nq = 1;
      }
      break;
    case PIPER_FMT_FP8_E4M3:
    case PIPER_FMT_FP8_E5M2:
    case PIPER_FMT_INT8: {
      if (d.scale == nullptr) return fail(PIPER_MERGE_EINVAL, "scaled merge requires scales.");
      if (d.format == PIPER_FMT_INT8 && !is_fp_dt(d.scale_dtype))
        return fail(PIPER_MERGE_EINVAL, "INT8 merge supports float16, bfloat16 and float32 scales.");
      const bool per_tensor = d.block_rows == d.rows && d.block_cols == d.cols;
      const bool per_block = d.block_rows == 1 && d.block_cols > 0 && d.block_cols <= d.cols &&
                             d.cols % d.block_cols == 0;
      if (!per_tensor && !per_block)
        return fail(PIPER_MERGE_EINVAL,
                    "supports two-dimensional per-tensor, per-row and per-group layouts, got block size (" +
                        std::to_string(d.block_rows) + ", " + std::to_string(d.block_cols) + ").");
      if (per_tensor) {
        p.two_pass = true;
        p.nq = 1;
        p.nq_row = 0;
        p.group = static_cast<int>(d.cols);
      } else {
        const int g = static_cast<int>(d.block_cols);
        p.group = g;
        p.nq_row = static_cast<int>(d.cols / g);
        if (g < d.cols && (g == 32 || g == 64 || g == 128 || g == 256)) {
          // groups are local to a tile: encoded in one pass
        } else if (g == d.cols) {
          p.fused = true;  // per-row: each CTA reduces then encodes its strips, one launch
        } else {
          p.two_pass = true;
          p.nq = static_cast<int>(d.rows * p.nq_row);
        }
      }
      break;
    }
    case PIPER_FMT_BNB4_NF4:
    case PIPER_FMT_BNB4_FP4:  // _triton_bnb4_lora.py:434-540
      if (d.cols % 64 != 0) return fail(PIPER_MERGE_EINVAL, "BNB4 merge requires row-aligned 64-value blocks.");
      if (d.scale == nullptr || d.codebook == nullptr)
        return fail(PIPER_MERGE_EINVAL, "BNB4 merge requires absmax and a 16-value float32 codebook.");
      if (d.nested_absmax != nullptr) {
        if (d.nested_code == nullptr || d.nested_offset == nullptr)
          return fail(PIPER_MERGE_EINVAL, "Nested BNB4 merge requires its codebook and offset.");
        if (d.flags & PIPER_FLAG_STOCHASTIC)
          return fail(PIPER_MERGE_EINVAL,
                      "BNB4 stochastic merge does not support nested scales because their final effective values "
                      "are unavailable during terminal-code selection.");
        // raw block maxima for the nested pass, then the fp64 partial sums of their mean
        p.nq = static_cast<int>(d.rows * (d.cols / 64)) + 2 * pm::kBnb4Parts + 2;
      }
      break;
    case PIPER_FMT_GGUF_Q8_0:
    case PIPER_FMT_GGUF_Q4_0:
      if (d.cols % 32 != 0) return fail(PIPER_MERGE_EINVAL, "GGUF merge requires columns divisible by 32.");
      break;
    default:
      return fail(PIPER_MERGE_EINVAL, "unknown format id " + std::to_string(d.format) + ".");
  }
  // The widest tile (256, 128 or 64 columns) whose pipeline keeps three
  // stages of (codes, A tile, scales) next to two B strips; 64-column tiles
  // (large ranks) may run with two.
  // fp32 factors are read by the epilogue from global memory: no factor stages.
  const int kp = d.compute_dtype == PIPER_DT_F32 ? 16 : pm::align_up(static_cast<int>(d.rank), 16);
  auto fits = [&](int bn, int min_sc) {
    return 512 / bn >= pm::epi_wgs_rt(d.format, bn) && plan_pipe(d.format, bn, kp).sc >= min_sc;
  };
  // Stochastic NVFP4 prefers three epilogue warpgroups, i.e. 128-column tiles.
  const bool narrow = d.format == PIPER_FMT_NVFP4 && (d.flags & PIPER_FLAG_STOCHASTIC) != 0u;
  // GGUF rows reach the tile by TMA only when a tile row is a multiple of 16
  // bytes, i.e. at 256 columns (Q8_0: 272 bytes, Q4_0: 144); narrower tiles
  // take the cp.async fallback, so GGUF keeps 256 columns down to two stages.
  const bool gguf = d.format == PIPER_FMT_GGUF_Q8_0 || d.format == PIPER_FMT_GGUF_Q4_0;
  if (!narrow && fits(256, gguf ? 2 : 4)) p.bn = 256;
  else if (fits(128, 4)) p.bn = 128;
  else if (fits(64, 2)) p.bn = 64;
  else return fail(PIPER_MERGE_EINVAL, "rank " + std::to_string(d.rank) + " is too large for the merge pipeline.");
  if ((d.format == PIPER_FMT_FP8_E4M3 || d.format == PIPER_FMT_FP8_E5M2 || d.format == PIPER_FMT_INT8) &&
      !p.two_pass && !p.fused && p.group > p.bn) {
    p.two_pass = true;  // the group no longer fits one tile
    p.nq = static_cast<int>(d.rows * p.nq_row);
  }
  return PIPER_MERGE_OK;
}

// Workspace words per quantization block: qmax, qmin, old_scale, old_zp
// (bitsandbytes 4-bit nested: the new block maximum only).
int scratch_words(int format) {
  return format == PIPER_FMT_BNB4_NF4 || format == PIPER_FMT_BNB4_FP4 ? 1 : 4;
}

size_t scratch_bytes(int nq, int words) {
  return nq == 0 ? 0 : (static_cast<size_t>(nq) * 4 * words + 255) / 256 * 256;  // 256-byte aligned
}

// Environment switches, read once per process.
struct EnvFlags {
  bool debug;   // PIPER_MERGE_DEBUG: print each launch's plan to stderr
  bool no_tma;  // PIPER_MERGE_NO_TMA: move every tile by cp.async
};
const EnvFlags& env_flags() {
  static const EnvFlags f{std::getenv("PIPER_MERGE_DEBUG") != nullptr, std::getenv("PIPER_MERGE_NO_TMA") != nullptr};
  return f;
}

constexpr int kMaxDevices = 64;

int sm_count() {
  static std::atomic<int> cached[kMaxDevices] = {};
  int dev = 0, n = 0;
  cudaGetDevice(&dev);
  if (dev >= 0 && dev < kMaxDevices && (n = cached[dev].load(std::memory_order_relaxed)) > 0) return n;
  cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
  n = n > 0 ? n : 148;
  if (dev >= 0 && dev < kMaxDevices) cached[dev].store(n, std::memory_order_relaxed);
  return n;
}

// Identity of the calling thread's current CUDA context: cuCtxGetId, which
// is unique for the life of the process and never reused, plus one; 0 when no
// context is current or the driver lacks the call. Function attributes and
// the addresses of module variables belong to one context (a non-primary
// context, or the primary context re-created after cudaDeviceReset, loads the
// module anew), so host-side caches of either key on this value.
uint64_t current_context_id() {
  static PFN_cuCtxGetCurrent_v4000 get_current = nullptr;
  static PFN_cuCtxGetId_v12000 get_id = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      get_current = reinterpret_cast<PFN_cuCtxGetCurrent_v4000>(p);
    p = nullptr;
    if (cudaGetDriverEntryPoint("cuCtxGetId", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      get_id = reinterpret_cast<PFN_cuCtxGetId_v12000>(p);
    cudaGetLastError();
  });
  if (get_current == nullptr || get_id == nullptr) return 0;
  CUcontext ctx = nullptr;
  if (get_current(&ctx) != CUDA_SUCCESS || ctx == nullptr) return 0;
  unsigned long long id = 0;
  if (get_id(ctx, &id) != CUDA_SUCCESS) return 0;
  return static_cast<uint64_t>(id) + 1u;
}

// Device address of the launch item counters (pm::g_sched_next) in the
// current context, looked up once per context.
unsigned int* sched_counters() {
  static std::mutex mu;
  static uint64_t cached_ctx[kMaxDevices] = {};
  static unsigned int* cached_ptr[kMaxDevices] = {};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return nullptr;
  std::lock_guard<std::mutex> lock(mu);
  uint64_t ctx = current_context_id();
  if (ctx == 0 || cached_ctx[dev] != ctx || cached_ptr[dev] == nullptr) {
    void* ptr = nullptr;
    if (cudaGetSymbolAddress(&ptr, pm::g_sched_next) != cudaSuccess) return nullptr;
    cached_ptr[dev] = static_cast<unsigned int*>(ptr);
    cached_ctx[dev] = current_context_id();
  }
  return cached_ptr[dev];
}

// ------------------------------------------------------------- dispatch
// One CTA per SM: the kernel allocates 2 * BN of the SM's 512 tensor-memory
// columns, and the shared-memory request (at least half the SM's) keeps a
// second CTA off the SM so a tcgen05.alloc never waits on another CTA.
constexpr int kMinSmem = 120 * 1024;

template <int FMT, int PASS, int BN, int CDT>
int launch_t(LaunchParams& lp, int items, int kp_max, cudaStream_t stream) {
  auto kern = pm::merge_kernel<FMT, PASS, BN, CDT>;
  const PipeCfg pc = plan_pipe(pm::base_fmt(FMT), BN, kp_max);
  if (pc.sc < 2)
    return fail(PIPER_MERGE_EINVAL, "rank " + std::to_string(kp_max) + " does not fit the shared-memory pipeline.");
  const int smem =
      std::max(pm::ws_smem_bytes(pm::TileGeom<FMT, BN>::kCodeSlot, kp_max, BN, pc.sc, pc.sa, pc.nbb), kMinSmem);
  // The dynamic shared-memory ceiling is raised to the per-CTA limit once per
  // context and instantiation (every plan's request is below it), not per call.
  static std::atomic<uint64_t> attr_ctx{0};
  const uint64_t ctx = current_context_id();
  cudaError_t e;
  if (ctx == 0 || attr_ctx.load(std::memory_order_acquire) != ctx) {
    e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, pm::kSmemLimit);
    if (e != cudaSuccess)
      return fail(PIPER_MERGE_ECUDA, std::string("cudaFuncSetAttribute: ") + cudaGetErrorString(e));
    attr_ctx.store(ctx, std::memory_order_release);
  }
  lp.n_items = items;
  lp.kp_max = kp_max;
  // This launch's item counter: the next slot of the ring, zeroed on the stream.
  static std::atomic<uint32_t> launch_seq{0};
  lp.sched_slot = launch_seq.fetch_add(1, std::memory_order_relaxed) % pm::kSchedSlots;
  unsigned int* counters = sched_counters();
  if (counters == nullptr) return fail(PIPER_MERGE_ECUDA, "cudaGetSymbolAddress of the item counters failed.");
  e = cudaMemsetAsync(counters + lp.sched_slot, 0, sizeof(unsigned int), stream);
  if (e != cudaSuccess) return fail(PIPER_MERGE_ECUDA, std::string("cudaMemsetAsync: ") + cudaGetErrorString(e));
  lp.c_stages = pc.sc;
  lp.a_stages = pc.sa;
  lp.b_bufs = pc.nbb;
  const int grid = std::min(items, sm_count());
  if (env_flags().debug)
    std::fprintf(stderr, "[piper-merge] fmt=%d pass=%d bn=%d kp=%d stages=%d/%d/%d smem=%d items=%d grid=%d\n", FMT,
                 PASS, BN, kp_max, pc.sc, pc.sa, pc.nbb, smem, items, grid);
  kern<<<grid, pm::ws_threads<FMT, BN>(), smem, stream>>>(lp);
  g_launches.fetch_add(1, std::memory_order_relaxed);
  e = cudaGetLastError();
  if (e != cudaSuccess) return fail(PIPER_MERGE_ECUDA, std::string("kernel launch: ") + cudaGetErrorString(e));
  return PIPER_MERGE_OK;
}

template <int FMT, int PASS, int CDT>
int launch_bn(int bn, LaunchParams& lp, int items, int kp, cudaStream_t s) {
  if (bn == 256) {
    // 256-column tiles leave two accumulator buffers: one per epilogue warpgroup at most.
    if constexpr (512 / 256 >= pm::epi_wgs<FMT, 256>()) return launch_t<FMT, PASS, 256, CDT>(lp, items, kp, s);
    else return fail(PIPER_MERGE_EINVAL, "256-column tiles need at most two epilogue warpgroups.");
  }
  if (bn == 128) return launch_t<FMT, PASS, 128, CDT>(lp, items, kp, s);
  // fp32 factors take no shared-memory factor stages, so the planner never
  // narrows their tiles to 64 columns.
  if constexpr (CDT == pm::kF32) return fail(PIPER_MERGE_EINVAL, "fp32 factors run on 128- or 256-column tiles.");
  else return launch_t<FMT, PASS, 64, CDT>(lp, items, kp, s);
}

// Development builds may compile a subset of the formats: -DPIPER_ONLY_FMTS=<bitmask of PIPER_FMT_* ids>.
#ifdef PIPER_ONLY_FMTS
constexpr bool fmt_on(int f) { return ((PIPER_ONLY_FMTS) >> f) & 1; }
#else
constexpr bool fmt_on(int) { return true; }
#endif

template <int PASS, int CDT>
int launch_fmt(int fmt, int bn, LaunchParams& lp, int items, int kp, cudaStream_t s) {
  if (!fmt_on(fmt)) return fail(PIPER_MERGE_EINVAL, "format not compiled into this build.");
  switch (fmt) {
    case PIPER_FMT_MXFP8_E4M3:
      if constexpr (fmt_on(PIPER_FMT_MXFP8_E4M3) && PASS == pm::kLocal && (CDT == pm::kBF16 || CDT == pm::kF32)) return launch_bn<PIPER_FMT_MXFP8_E4M3, PASS, CDT>(bn, lp, items, kp, s);
      break;
    case PIPER_FMT_MXFP8_E5M2:
      if constexpr (fmt_on(PIPER_FMT_MXFP8_E5M2) && PASS == pm::kLocal && (CDT == pm::kBF16 || CDT == pm::kF32)) return launch_bn<PIPER_FMT_MXFP8_E5M2, PASS, CDT>(bn, lp, items, kp, s);
      break;
    case PIPER_FMT_MXFP4:
      if constexpr (fmt_on(PIPER_FMT_MXFP4) && PASS == pm::kLocal && (CDT == pm::kBF16 || CDT == pm::kF32)) return launch_bn<PIPER_FMT_MXFP4, PASS, CDT>(bn, lp, items, kp, s);
      break;
    case PIPER_FMT_NVFP4:
      if constexpr (fmt_on(PIPER_FMT_NVFP4) && (PASS == pm::kLocal || PASS == pm::kReduce) &&
                    (CDT == pm::kBF16 || CDT == pm::kF32))
        return launch_bn<PIPER_FMT_NVFP4, PASS, CDT>(bn, lp, items, kp, s);
      break;
    case PIPER_FMT_FP8_E4M3:
      if constexpr (fmt_on(PIPER_FMT_FP8_E4M3)) return launch_bn<PIPER_FMT_FP8_E4M3, PASS, CDT>(bn, lp, items, kp, s);
      break;
    case PIPER_FMT_FP8_E5M2:
      if constexpr (fmt_on(PIPER_FMT_FP8_E5M2)) return launch_bn<PIPER_FMT_FP8_E5M2, PASS, CDT>(bn, lp, items, kp, s);
      break;
    case PIPER_FMT_INT8:
      if constexpr (fmt_on(PIPER_FMT_INT8)) return launch_bn<PIPER_FMT_INT8, PASS, CDT>(bn, lp, items, kp, s);
      break;
    case PIPER_FMT_BNB8:  // per-row, fp16 only
      if constexpr (fmt_on(PIPER_FMT_BNB8) && PASS == pm::kFused && CDT == pm::kF16) return launch_bn<PIPER_FMT_BNB8, PASS, CDT>(bn, lp, items, kp, s);
      break;
    case PIPER_FMT_QUANTO_INT8:  // per-row (fused) or per-tensor (reduce + encode)
      if constexpr (fmt_on(PIPER_FMT_QUANTO_INT8) && PASS != pm::kLocal) return launch_bn<PIPER_FMT_QUANTO_INT8, PASS, CDT>(bn, lp, items, kp, s);
      break;
    case PIPER_FMT_QUANTO_FP8_E4M3:
      if constexpr (fmt_on(PIPER_FMT_QUANTO_FP8_E4M3) && PASS != pm::kLocal) return launch_bn<PIPER_FMT_QUANTO_FP8_E4M3, PASS, CDT>(bn, lp, items, kp, s);
      break;
    case PIPER_FMT_QUANTO_FP8_E5M2:
      if constexpr (fmt_on(PIPER_FMT_QUANTO_FP8_E5M2) && PASS != pm::kLocal) return launch_bn<PIPER_FMT_QUANTO_FP8_E5M2, PASS, CDT>(bn, lp, items, kp, s);
      break;
    case PIPER_FMT_BNB4_NF4:
      if constexpr (fmt_on(PIPER_FMT_BNB4_NF4) && PASS == pm::kLocal) return launch_bn<PIPER_FMT_BNB4_NF4, PASS, CDT>(bn, lp, items, kp, s);
      break;
    case PIPER_FMT_BNB4_FP4:
      if constexpr (fmt_on(PIPER_FMT_BNB4_FP4) && PASS == pm::kLocal) return launch_bn<PIPER_FMT_BNB4_FP4, PASS, CDT>(bn, lp, items, kp, s);
      break;
    case PIPER_FMT_GGUF_Q8_0:
      if constexpr (fmt_on(PIPER_FMT_GGUF_Q8_0) && PASS == pm::kLocal) return launch_bn<PIPER_FMT_GGUF_Q8_0, PASS, CDT>(bn, lp, items, kp, s);
      break;
    case PIPER_FMT_GGUF_Q4_0:
      if constexpr (fmt_on(PIPER_FMT_GGUF_Q4_0) && PASS == pm::kLocal) return launch_bn<PIPER_FMT_GGUF_Q4_0, PASS, CDT>(bn, lp, items, kp, s);
      break;
    default: break;
  }
  return fail(PIPER_MERGE_EINVAL, "no kernel for this format / pass / dtype combination.");
}

int launch(int pass, int cdt, int fmt, int bn, LaunchParams& lp, int items, int kp, cudaStream_t s) {
  if (items <= 0) return PIPER_MERGE_OK;
  if (cdt == PIPER_DT_BF16) {
    if (pass == pm::kLocal) return launch_fmt<pm::kLocal, pm::kBF16>(fmt, bn, lp, items, kp, s);
    if (pass == pm::kReduce) return launch_fmt<pm::kReduce, pm::kBF16>(fmt, bn, lp, items, kp, s);
    if (pass == pm::kFused) return launch_fmt<pm::kFused, pm::kBF16>(fmt, bn, lp, items, kp, s);
    return launch_fmt<pm::kEncode, pm::kBF16>(fmt, bn, lp, items, kp, s);
  }
  if (cdt == PIPER_DT_F32) {
    if (pass == pm::kLocal) return launch_fmt<pm::kLocal, pm::kF32>(fmt, bn, lp, items, kp, s);
    if (pass == pm::kReduce) return launch_fmt<pm::kReduce, pm::kF32>(fmt, bn, lp, items, kp, s);
    if (pass == pm::kFused) return launch_fmt<pm::kFused, pm::kF32>(fmt, bn, lp, items, kp, s);
    return launch_fmt<pm::kEncode, pm::kF32>(fmt, bn, lp, items, kp, s);
  }
  if (pass == pm::kLocal) return launch_fmt<pm::kLocal, pm::kF16>(fmt, bn, lp, items, kp, s);
  if (pass == pm::kReduce) return launch_fmt<pm::kReduce, pm::kF16>(fmt, bn, lp, items, kp, s);
  if (pass == pm::kFused) return launch_fmt<pm::kFused, pm::kF16>(fmt, bn, lp, items, kp, s);
  return launch_fmt<pm::kEncode, pm::kF16>(fmt, bn, lp, items, kp, s);
}

// A row range of one weight scheduled in one launch.
struct Segment {
  int desc;
  int row_begin, rows;
};

PFN_cuTensorMapEncodeTiled_v12000 tensor_map_encoder() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static bool tried = false;
  if (!tried) {
    tried = true;
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(ptr);
    cudaGetLastError();
  }
  return fn;
}

int64_t row_bytes_of(const piper_merge_desc& d);

// Code tiles of `bn` columns move by 2-D bulk tensor copies when a row of the
// tile is 64 or 128 bytes (so the 64 B / 128 B swizzle spans it) and rows are
// 16-byte aligned; otherwise by cp.async.
// Tensor map of the code bytes for bulk tensor tiles of 128 rows x bn columns:
// boxes of min(128, tile row) bytes with the matching smem swizzle (a 16-byte
// chunk XOR of 128 / 64 / 32-byte rows), or for GGUF one dense box of the
// whole tile row in 8-byte elements. Requires 16-byte aligned rows and base.
void setup_tma(DevWeight& w, const piper_merge_desc& d, int bn) {
  w.use_tma = 0;
  const bool gguf = d.format == PIPER_FMT_GGUF_Q8_0 || d.format == PIPER_FMT_GGUF_Q4_0;
  const int tile_row = host_code_bytes(d.format, bn);
  const int box_row = gguf ? tile_row : std::min(128, tile_row);
  if (gguf ? (tile_row % 16 != 0 || tile_row / 8 > 256) : (box_row != 32 && box_row != 64 && box_row != 128))
    return;
  const int64_t rb = row_bytes_of(d);
  if ((rb & 15) != 0 || (reinterpret_cast<uintptr_t>(d.qdata) & 15) != 0) return;
  auto enc = tensor_map_encoder();
  if (enc == nullptr) return;
  CUresult r;
  if (gguf) {
    const cuuint64_t dims[2] = {static_cast<cuuint64_t>(rb / 8), static_cast<cuuint64_t>(d.rows)};
    const cuuint64_t strides[1] = {static_cast<cuuint64_t>(rb)};
    const cuuint32_t box[2] = {static_cast<cuuint32_t>(box_row / 8), 128u};
    const cuuint32_t estr[2] = {1u, 1u};
    r = enc(&w.tmap, CU_TENSOR_MAP_DATA_TYPE_UINT64, 2, d.qdata, dims, strides, box, estr,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  } else {
    const cuuint64_t dims[2] = {static_cast<cuuint64_t>(rb), static_cast<cuuint64_t>(d.rows)};
    const cuuint64_t strides[1] = {static_cast<cuuint64_t>(rb)};
    const cuuint32_t box[2] = {static_cast<cuuint32_t>(box_row), 128u};
    const cuuint32_t estr[2] = {1u, 1u};
    const CUtensorMapSwizzle sw = box_row == 128 ? CU_TENSOR_MAP_SWIZZLE_128B
                                  : (box_row == 64 ? CU_TENSOR_MAP_SWIZZLE_64B : CU_TENSOR_MAP_SWIZZLE_32B);
    r = enc(&w.tmap, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, d.qdata, dims, strides, box, estr,
            CU_TENSOR_MAP_INTERLEAVE_NONE, sw, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  }
  if (r != CUDA_SUCCESS) return;
  w.use_tma = 1;
}

// Tensor maps of the LoRA factors for bulk tensor tiles in the swizzled UMMA
// layouts: A (r x N, row-major) in boxes of 64 columns x KP rows with 128-byte
// swizzle (MN-major operand); B (M x r, row-major) in boxes of kb_row(KP)
// bytes x 128 rows with the matching swizzle (K-major operand). Rows past r
// and columns past N read as zeros. Requires 16-byte aligned bases and row
// pitches; otherwise the loader warps copy the same layouts with cp.async.
void setup_tma_factors(DevWeight& w, const piper_merge_desc& d, int kp) {
  w.use_tma_a = 0;
  w.use_tma_b = 0;
  auto enc = tensor_map_encoder();
  if (enc == nullptr) return;
  const cuuint32_t estr[2] = {1u, 1u};
  if ((d.cols * 2) % 16 == 0 && (reinterpret_cast<uintptr_t>(d.a) & 15) == 0 && d.cols >= 64) {
    const cuuint64_t dims[2] = {static_cast<cuuint64_t>(d.cols), static_cast<cuuint64_t>(d.rank)};
    const cuuint64_t strides[1] = {static_cast<cuuint64_t>(d.cols * 2)};
    const cuuint32_t box[2] = {64u, static_cast<cuuint32_t>(kp)};
    if (enc(&w.tmap_a, CU_TENSOR_MAP_DATA_TYPE_UINT16, 2, const_cast<void*>(d.a), dims, strides, box, estr,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS)
      w.use_tma_a = 1;
  }
  if ((d.rank * 2) % 16 == 0 && (reinterpret_cast<uintptr_t>(d.b) & 15) == 0) {
    const int kb = pm::kb_row(kp);
    const cuuint64_t dims[2] = {static_cast<cuuint64_t>(d.rank), static_cast<cuuint64_t>(d.rows)};
    const cuuint64_t strides[1] = {static_cast<cuuint64_t>(d.rank * 2)};
    const cuuint32_t box[2] = {static_cast<cuuint32_t>(kb / 2), 128u};
    const CUtensorMapSwizzle sw = kb == 128 ? CU_TENSOR_MAP_SWIZZLE_128B
                                  : (kb == 64 ? CU_TENSOR_MAP_SWIZZLE_64B : CU_TENSOR_MAP_SWIZZLE_32B);
    if (enc(&w.tmap_b, CU_TENSOR_MAP_DATA_TYPE_UINT16, 2, const_cast<void*>(d.b), dims, strides, box, estr,
            CU_TENSOR_MAP_INTERLEAVE_NONE, sw, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS)
      w.use_tma_b = 1;
  }
}

DevWeight make_dev_weight(const piper_merge_desc& d, const Plan& p, uint8_t* ws, const Segment& seg) {
  DevWeight w;
  std::memset(&w, 0, sizeof(w));
  w.q = static_cast<uint8_t*>(d.qdata);
  w.scale = d.scale;
  w.zp = static_cast<int8_t*>(d.zero_point);
  w.gscale = static_cast<float*>(d.global_scale);
  w.b = static_cast<const uint16_t*>(d.b);
  w.a = static_cast<const uint16_t*>(d.a);
  if (p.nq > 0) {
    uint8_t* base = ws + p.ws_off;
    w.qmax = reinterpret_cast<uint32_t*>(base);
    if (scratch_words(d.format) == 4) {
      w.qmin = reinterpret_cast<uint32_t*>(base + 4 * static_cast<size_t>(p.nq));
      w.old_scale = reinterpret_cast<float*>(base + 8 * static_cast<size_t>(p.nq));
      w.old_zp = reinterpret_cast<int32_t*>(base + 12 * static_cast<size_t>(p.nq));
    }
  }
  w.row_bytes = row_bytes_of(d);
  w.offset_base = d.offset_base;
  w.k0 = static_cast<uint32_t>(d.seed & 0xFFFFFFFFull);
  w.k1 = static_cast<uint32_t>(d.seed >> 32);
  w.strength = d.strength;
  w.flags = d.flags;
  w.M = static_cast<int>(d.rows);
  w.N = static_cast<int>(d.cols);
  w.r = static_cast<int>(d.rank);
  // fp32 factors stay in global memory (the epilogue's CUDA-core update reads
  // them); the smallest factor stages are laid out and left unused.
  const bool f32_factors = d.compute_dtype == PIPER_DT_F32;
  w.KP = f32_factors ? 16 : pm::align_up(static_cast<int>(d.rank), 16);
  w.row_begin = seg.row_begin;
  w.row_blocks = (seg.rows + 127) / 128;
  w.group = p.group;
  w.nq_row = p.nq_row;
  w.scale_cols = d.format == PIPER_FMT_NVFP4 ? static_cast<int>(d.cols / 16) : static_cast<int>(d.cols / 32);
  w.scale_mode = d.scale_mode;
  w.scale_dt = d.scale_dtype;
  w.code16 = static_cast<const float*>(d.codebook);
  w.ncode = static_cast<const float*>(d.nested_code);
  w.nabs = static_cast<const float*>(d.nested_absmax);
  w.noff = static_cast<const float*>(d.nested_offset);
  w.col_axis = p.col_axis ? 1 : 0;
  if (!env_flags().no_tma) {
    setup_tma(w, d, p.bn);
    if (!f32_factors) setup_tma_factors(w, d, w.KP);
  }
  return w;
}

// Launch one group of segments that share a kernel instantiation.
int run_group(const piper_merge_desc* descs, const std::vector<Plan>& plans, uint8_t* ws,
              const std::vector<Segment>& segs, cudaStream_t stream) {
  if (segs.empty()) return PIPER_MERGE_OK;
  const piper_merge_desc& d0 = descs[segs[0].desc];
  const Plan& p0 = plans[segs[0].desc];
  // Items are taken in order by the CTAs (largest first balances the tail):
  // the widest weights, whose items cost the most, come first.
  std::vector<Segment> order(segs);
  std::stable_sort(order.begin(), order.end(),
                   [&](const Segment& x, const Segment& y) { return descs[x.desc].cols > descs[y.desc].cols; });
  LaunchParams lp;
  std::memset(&lp, 0, sizeof(lp));
  lp.n_weights = static_cast<int>(segs.size());
  // Work items: (128-row strip, column range) pairs, taken by the persistent
  // CTAs one at a time; aim for ~32 items per SM so the last wave is short.
  int kp_max = 16;
  int64_t total_tiles = 0;
  for (const Segment& sg : segs) {
    const Plan& p = plans[sg.desc];
    total_tiles += static_cast<int64_t>((sg.rows + 127) / 128) * ((descs[sg.desc].cols + p.bn - 1) / p.bn);
  }
  // Items take at least two column tiles where a strip has them: each item
  // reloads its B strip and takes one atomic from the item counter, and with
  // dynamic distribution a small tail costs little.
  const int64_t target_items = 32ll * sm_count();
  const int tiles_per_item = static_cast<int>(std::max<int64_t>(2, total_tiles / target_items));
  int items = 0;
  for (size_t i = 0; i < order.size(); ++i) {
    const piper_merge_desc& d = descs[order[i].desc];
    const Plan& p = plans[order[i].desc];
    DevWeight w = make_dev_weight(d, p, ws, order[i]);
    const int col_tiles = static_cast<int>((d.cols + p.bn - 1) / p.bn);
    // Fused per-row passes need whole rows in one item.
    const int ci = p.fused ? 1 : std::max(1, (col_tiles + tiles_per_item - 1) / tiles_per_item);
    const int tiles_each = (col_tiles + ci - 1) / ci;
    w.item_cols = tiles_each * p.bn;
    w.col_items = (col_tiles + tiles_each - 1) / tiles_each;
    w.item_begin = items;
    items += w.row_blocks * w.col_items;
    kp_max = std::max(kp_max, w.KP);
    lp.w[i] = w;
  }
  const int kfmt = pm::kernel_fmt(d0.format, p0.flavor);
  int rc;
  if (p0.two_pass) {
    rc = launch(pm::kReduce, d0.compute_dtype, kfmt, p0.bn, lp, items, kp_max, stream);
    if (rc) return rc;
    const int second = d0.format == PIPER_FMT_NVFP4 ? pm::kLocal : pm::kEncode;
    rc = launch(second, d0.compute_dtype, kfmt, p0.bn, lp, items, kp_max, stream);
  } else if (p0.fused) {
    rc = launch(pm::kFused, d0.compute_dtype, kfmt, p0.bn, lp, items, kp_max, stream);
  } else {
    rc = launch(pm::kLocal, d0.compute_dtype, kfmt, p0.bn, lp, items, kp_max, stream);
  }
  if (rc) return rc;
  // bitsandbytes nested absmax: re-quantize the new block maxima.
  for (const Segment& sg : segs) {
    const piper_merge_desc& d = descs[sg.desc];
    const Plan& p = plans[sg.desc];
    if ((d.format != PIPER_FMT_BNB4_NF4 && d.format != PIPER_FMT_BNB4_FP4) || d.nested_absmax == nullptr) continue;
    const uint32_t* raw = reinterpret_cast<const uint32_t*>(ws + p.ws_off);
    const int64_t n = d.rows * (d.cols / 64);
    double* part = reinterpret_cast<double*>(ws + p.ws_off + (static_cast<size_t>(n) * 4 + 7) / 8 * 8);
    pm::bnb4_partial_kernel<<<pm::kBnb4Parts, 256, 0, stream>>>(raw, n, part);
    const int64_t nblk = (n + 255) / 256;
    pm::bnb4_nested_kernel<<<static_cast<unsigned>((nblk + 7) / 8), 256, 0, stream>>>(
        raw, n, part, static_cast<float*>(d.nested_offset), static_cast<const float*>(d.nested_code),
        static_cast<uint8_t*>(d.scale), static_cast<float*>(d.nested_absmax));
    g_launches.fetch_add(2, std::memory_order_relaxed);
    const cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return fail(PIPER_MERGE_ECUDA, std::string("nested BNB4 launch: ") + cudaGetErrorString(e));
  }
  return PIPER_MERGE_OK;
}

bool same_kernel(const piper_merge_desc& a, const Plan& pa, const piper_merge_desc& b, const Plan& pb) {
  return a.format == b.format && a.compute_dtype == b.compute_dtype && pa.bn == pb.bn &&
         pa.two_pass == pb.two_pass && pa.fused == pb.fused && pa.flavor == pb.flavor;  // col_axis is per weight
}

// Per-row FP8 / INT8 weights run the one-launch fused pass, which keeps each
// strip's row maxima on chip but has one work item per 128-row strip. When a
// whole call holds fewer such strips than kSplitStripsPerSm per SM (one small
// weight, e.g. 4096 rows = 32 strips), most SMs would idle, so those weights
// run the reduce / encode launches instead, whose items also split the
// columns, with 16 bytes of workspace per row. A caller that provides no
// workspace still gets the fused pass (piper_merge_batch plans again without
// the split).
constexpr int kSplitStripsPerSm = 2;

int plan_all(const piper_merge_desc* in, int count, std::vector<piper_merge_desc>& descs,
             std::vector<Plan>& plans, size_t& ws_total, bool split_small_rows = true) {
  if (count < 0) return fail(PIPER_MERGE_EINVAL, "negative descriptor count.");
  if (count > 0 && in == nullptr) return fail(PIPER_MERGE_EINVAL, "null descriptor array.");
  descs.assign(in, in + count);
  plans.assign(count, Plan());
  ws_total = 0;
  int64_t fused_strips = 0;
  for (int i = 0; i < count; ++i) {
    int flavor = pm::kTorchao;
    bool col_axis = false;
    int rc = normalize(descs[i], flavor, col_axis);
    if (rc) return rc;
    rc = validate(descs[i], plans[i]);
    if (rc) return rc;
    plans[i].flavor = flavor;
    if (col_axis) {
      plans[i].col_axis = true;
      plans[i].nq = static_cast<int>(descs[i].cols);
    }
    if (plans[i].fused) fused_strips += (descs[i].rows + 127) / 128;
  }
  if (split_small_rows && fused_strips > 0 && fused_strips < static_cast<int64_t>(kSplitStripsPerSm) * sm_count()) {
    for (int i = 0; i < count; ++i) {
      Plan& p = plans[i];
      if (!p.fused || p.flavor == pm::kBnb) continue;  // bitsandbytes 8-bit has the fused pass only
      p.fused = false;
      p.two_pass = true;
      p.nq = static_cast<int>(descs[i].rows) * p.nq_row;
    }
  }
  for (int i = 0; i < count; ++i) {
    plans[i].ws_off = ws_total;
    ws_total += scratch_bytes(plans[i].nq, scratch_words(descs[i].format));
  }
  return PIPER_MERGE_OK;
}

}  // namespace

// ================================================================= C ABI
extern "C" {

int piper_merge_workspace_size(const piper_merge_desc* in, int32_t count, size_t* bytes) {
  std::vector<piper_merge_desc> descs;
  std::vector<Plan> plans;
  size_t total = 0;
  int rc = plan_all(in, count, descs, plans, total);
  if (rc) return rc;
  if (bytes) *bytes = total;
  return PIPER_MERGE_OK;
}

int piper_merge_batch(const piper_merge_desc* in, int32_t count, void* workspace,
                      size_t workspace_bytes, void* stream_ptr) {
  std::vector<piper_merge_desc> descs;
  std::vector<Plan> plans;
  size_t total = 0;
  int rc = plan_all(in, count, descs, plans, total);
  if (rc) return rc;
  if (total > 0 && (workspace == nullptr || workspace_bytes < total)) {
    rc = plan_all(in, count, descs, plans, total, /*split_small_rows=*/false);
    if (rc) return rc;
  }
  if (total > 0 && (workspace == nullptr || workspace_bytes < total))
    return fail(PIPER_MERGE_EWORKSPACE, "workspace of " + std::to_string(workspace_bytes) +
                                             " bytes is smaller than the required " +
                                             std::to_string(total) + ".");
  if (total > 0 && (reinterpret_cast<uintptr_t>(workspace) & 255) != 0)
    return fail(PIPER_MERGE_EINVAL, "workspace must be 256-byte aligned.");
  cudaStream_t stream = static_cast<cudaStream_t>(stream_ptr);
  uint8_t* ws = static_cast<uint8_t*>(workspace);
  if (total > 0) {
    cudaError_t e = cudaMemsetAsync(ws, 0, total, stream);
    if (e != cudaSuccess) return fail(PIPER_MERGE_ECUDA, std::string("cudaMemsetAsync: ") + cudaGetErrorString(e));
  }
  // Cut weights into segments: two-pass per-row/per-block weights by row
  // ranges of about kL2GroupBytes, everything else whole.
  std::vector<Segment> segs;
  for (int i = 0; i < count; ++i) {
    const piper_merge_desc& d = descs[i];
    const Plan& p = plans[i];
    const int rows = static_cast<int>(d.rows);
    if (p.two_pass && p.nq_row > 0) {
      const int64_t rb = row_bytes_of(d);
      int step = static_cast<int>(std::max<int64_t>(128, kL2GroupBytes / std::max<int64_t>(rb, 1) / 128 * 128));
      for (int r0 = 0; r0 < rows; r0 += step) segs.push_back({i, r0, std::min(step, rows - r0)});
    } else {
      segs.push_back({i, 0, rows});
    }
  }
  std::vector<Segment> group;
  int64_t group_bytes = 0;
  for (const Segment& s : segs) {
    const piper_merge_desc& d = descs[s.desc];
    const Plan& p = plans[s.desc];
    const int64_t bytes = row_bytes_of(d) * s.rows;
    bool flush = !group.empty() &&
                 (!same_kernel(descs[group[0].desc], plans[group[0].desc], d, p) ||
                  static_cast<int>(group.size()) >= pm::kMaxWeights ||
                  (p.two_pass && group_bytes + bytes > kL2GroupBytes));
    if (flush) {
      rc = run_group(descs.data(), plans, ws, group, stream);
      if (rc) return rc;
      group.clear();
      group_bytes = 0;
    }
    group.push_back(s);
    group_bytes += bytes;
  }
  return run_group(descs.data(), plans, ws, group, stream);
}

int piper_merge_mx(void* qdata, void* scale, const void* b, const void* a, int64_t rows, int64_t cols,
                   int64_t rank, int32_t elem_format, int32_t compute_dtype, int32_t scaling_mode,
                   int32_t swizzled, float strength, int32_t has_seed, uint64_t seed, uint64_t offset_base,
                   void* stream) {
  piper_merge_desc d;
  std::memset(&d, 0, sizeof(d));
  if (elem_format < 0 || elem_format > 2) return fail(PIPER_MERGE_EINVAL, "MX element format must be 0 (e4m3), 1 (e5m2) or 2 (e2m1).");
  d.format = elem_format == 0 ? PIPER_FMT_MXFP8_E4M3 : (elem_format == 1 ? PIPER_FMT_MXFP8_E5M2 : PIPER_FMT_MXFP4);
  d.qdata = qdata;
  d.scale = scale;
  d.b = b;
  d.a = a;
  d.rows = rows;
  d.cols = cols;
  d.rank = rank;
  d.compute_dtype = compute_dtype;
  d.scale_mode = scaling_mode;
  d.flags = (swizzled ? PIPER_FLAG_SWIZZLED : 0u) | (has_seed ? PIPER_FLAG_STOCHASTIC : 0u);
  d.strength = strength;
  d.seed = seed;
  d.offset_base = offset_base;
  return piper_merge_batch(&d, 1, nullptr, 0, stream);
}

int piper_merge_nvfp4(void* qdata, void* scale, void* global_scale, const void* b, const void* a,
                      int64_t rows, int64_t cols, int64_t rank, int32_t compute_dtype, int32_t swizzled,
                      float strength, int32_t has_seed, uint64_t seed, uint64_t offset_base,
                      void* workspace, size_t workspace_bytes, void* stream) {
  piper_merge_desc d;
  std::memset(&d, 0, sizeof(d));
  d.format = PIPER_FMT_NVFP4;
  d.qdata = qdata;
  d.scale = scale;
  d.global_scale = global_scale;
  d.b = b;
  d.a = a;
  d.rows = rows;
  d.cols = cols;
  d.rank = rank;
  d.compute_dtype = compute_dtype;
  d.flags = (swizzled ? PIPER_FLAG_SWIZZLED : 0u) | (has_seed ? PIPER_FLAG_STOCHASTIC : 0u);
  d.strength = strength;
  d.seed = seed;
  d.offset_base = offset_base;
  return piper_merge_batch(&d, 1, workspace, workspace_bytes, stream);
}

int piper_merge_float8(void* qdata, void* scale, const void* b, const void* a, int64_t rows, int64_t cols,
                       int64_t rank, int64_t block_rows, int64_t block_cols, int32_t e5m2,
                       int32_t compute_dtype, float strength, int32_t has_seed, uint64_t seed,
                       uint64_t offset_base, void* workspace, size_t workspace_bytes, void* stream) {
  piper_merge_desc d;
  std::memset(&d, 0, sizeof(d));
  d.format = e5m2 ? PIPER_FMT_FP8_E5M2 : PIPER_FMT_FP8_E4M3;
  d.qdata = qdata;
  d.scale = scale;
  d.b = b;
  d.a = a;
  d.rows = rows;
  d.cols = cols;
  d.rank = rank;
  d.block_rows = block_rows;
  d.block_cols = block_cols;
  d.compute_dtype = compute_dtype;
  d.flags = has_seed ? PIPER_FLAG_STOCHASTIC : 0u;
  d.strength = strength;
  d.seed = seed;
  d.offset_base = offset_base;
  return piper_merge_batch(&d, 1, workspace, workspace_bytes, stream);
}

// Per-row / per-tensor / wide-group FP8 merges keep 16 bytes of running state
// per quantization block between their two passes. This variant takes that
// scratch from a fixed array in device memory instead of a caller's buffer,
// for callers that cannot allocate device memory at merge time: a C or C++
// host embedding the library without PyTorch's caching allocator (it has no
// device allocator of its own), or a process whose device memory a model cache
// has already reserved, where a merge-time cudaMalloc could fail or force an
// implicit device synchronization. It calls no allocating routine. The array
// exists once per device (every device's copy of the module has its own), so
// overlapping calls on one device, from several host threads or streams, race
// on it. The array's address is looked up (cudaGetSymbolAddress, with the
// device current) by the first call in each CUDA context of a device, and
// again whenever the calling thread's current context changes identity (a
// non-primary context, or the primary context re-created after
// cudaDeviceReset, holds its own copy of the array); make the first call in a
// context before any stream capture. Each call zeroes the blocks it uses on
// the stream before the kernels read them, as the buffer-taking entry point
// does.
namespace {
constexpr size_t kNoAllocScratchBytes = size_t{1} << 20;  // 65,536 quantization blocks
static __device__ __align__(256) uint8_t g_noalloc_scratch[kNoAllocScratchBytes];
std::mutex g_noalloc_mu;
struct NoAllocSlot {
  uint64_t ctx;  // current_context_id() the address belongs to (0: none)
  void* ptr;
};
NoAllocSlot g_noalloc_slot[kMaxDevices] = {};
}  // namespace

int piper_merge_float8_noalloc(void* qdata, void* scale, const void* b, const void* a, int64_t rows, int64_t cols,
                               int64_t rank, int64_t block_rows, int64_t block_cols, int32_t e5m2,
                               int32_t compute_dtype, float strength, int32_t has_seed, uint64_t seed,
                               uint64_t offset_base, void* stream) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return fail(PIPER_MERGE_ECUDA, std::string("cudaGetDevice: ") + cudaGetErrorString(e));
  if (dev < 0 || dev >= kMaxDevices)
    return fail(PIPER_MERGE_EINVAL, "device " + std::to_string(dev) + " is beyond the static scratch table.");
  void* scratch = nullptr;
  {
    std::lock_guard<std::mutex> lock(g_noalloc_mu);
    uint64_t ctx = current_context_id();
    NoAllocSlot& slot = g_noalloc_slot[dev];
    if (ctx == 0 || slot.ctx != ctx || slot.ptr == nullptr) {
      // Looking the symbol up also makes the runtime's context current on a
      // thread that had none, so the context is identified afterwards.
      void* ptr = nullptr;
      e = cudaGetSymbolAddress(&ptr, g_noalloc_scratch);
      if (e != cudaSuccess || ptr == nullptr)
        return fail(PIPER_MERGE_ECUDA, std::string("cudaGetSymbolAddress: ") + cudaGetErrorString(e));
      ctx = current_context_id();
      slot.ctx = ctx;
      slot.ptr = ptr;
    }
    scratch = slot.ptr;
  }
  piper_merge_desc d;
  std::memset(&d, 0, sizeof(d));
  d.format = e5m2 ? PIPER_FMT_FP8_E5M2 : PIPER_FMT_FP8_E4M3;
  d.qdata = qdata;
  d.scale = scale;
  d.b = b;
  d.a = a;
  d.rows = rows;
  d.cols = cols;
  d.rank = rank;
  d.block_rows = block_rows;
  d.block_cols = block_cols;
  d.compute_dtype = compute_dtype;
  d.flags = has_seed ? PIPER_FLAG_STOCHASTIC : 0u;
  d.strength = strength;
  d.seed = seed;
  d.offset_base = offset_base;
  size_t need = 0;
  const int rc = piper_merge_workspace_size(&d, 1, &need);
  if (rc != PIPER_MERGE_OK) return rc;
  if (need > kNoAllocScratchBytes)
    return fail(PIPER_MERGE_EWORKSPACE,
                "this layout needs " + std::to_string(need) + " bytes of scratch; the static scratch of " +
                    "piper_merge_float8_noalloc holds " + std::to_string(kNoAllocScratchBytes) +
                    " bytes (65536 quantization blocks). Use piper_merge_float8 with a workspace.");
  return piper_merge_float8(qdata, scale, b, a, rows, cols, rank, block_rows, block_cols, e5m2, compute_dtype,
                            strength, has_seed, seed, offset_base, scratch, kNoAllocScratchBytes, stream);
}

int piper_merge_int8(void* qdata, void* scale, void* zero_point, const void* b, const void* a, int64_t rows,
                     int64_t cols, int64_t rank, int64_t block_rows, int64_t block_cols, int32_t compute_dtype,
                     int32_t scale_dtype, int32_t asymmetric, int32_t reduce_range, float strength,
                     int32_t has_seed, uint64_t seed, uint64_t offset_base, void* workspace,
                     size_t workspace_bytes, void* stream) {
  piper_merge_desc d;
  std::memset(&d, 0, sizeof(d));
  d.format = PIPER_FMT_INT8;
  d.qdata = qdata;
  d.scale = scale;
  d.zero_point = zero_point;
  d.b = b;
  d.a = a;
  d.rows = rows;
  d.cols = cols;
  d.rank = rank;
  d.block_rows = block_rows;
  d.block_cols = block_cols;
  d.compute_dtype = compute_dtype;
  d.scale_dtype = scale_dtype;
  d.flags = (asymmetric ? PIPER_FLAG_ASYMMETRIC : 0u) | (reduce_range ? PIPER_FLAG_REDUCE_RANGE : 0u) |
            (has_seed ? PIPER_FLAG_STOCHASTIC : 0u);
  d.strength = strength;
  d.seed = seed;
  d.offset_base = offset_base;
  return piper_merge_batch(&d, 1, workspace, workspace_bytes, stream);
}

int piper_merge_static_float8(void* qdata, void* scale, const void* b, const void* a, int64_t rows,
                              int64_t cols, int64_t rank, int32_t e5m2, int32_t compute_dtype,
                              float strength, int32_t has_seed, uint64_t seed, uint64_t offset_base,
                              void* workspace, size_t workspace_bytes, void* stream) {
  return piper_merge_float8(qdata, scale, b, a, rows, cols, rank, rows, cols, e5m2, compute_dtype, strength,
                            has_seed, seed, offset_base, workspace, workspace_bytes, stream);
}

int piper_merge_bnb8(void* cb, void* scb, const void* b, const void* a, int64_t rows, int64_t cols,
                     int64_t rank, float strength, int32_t has_seed, uint64_t seed,
                     uint64_t offset_base, void* stream) {
  piper_merge_desc d;
  std::memset(&d, 0, sizeof(d));
  d.format = PIPER_FMT_BNB8;
  d.qdata = cb;
  d.scale = scb;
  d.b = b;
  d.a = a;
  d.rows = rows;
  d.cols = cols;
  d.rank = rank;
  d.block_rows = 1;
  d.block_cols = cols;
  d.compute_dtype = PIPER_DT_F16;
  d.scale_dtype = PIPER_DT_F32;
  d.flags = has_seed ? PIPER_FLAG_STOCHASTIC : 0u;
  d.strength = strength;
  d.seed = seed;
  d.offset_base = offset_base;
  return piper_merge_batch(&d, 1, nullptr, 0, stream);
}

int piper_merge_quanto(void* qdata, void* scale, const void* b, const void* a, int64_t rows,
                       int64_t cols, int64_t rank, int32_t storage, int32_t per_row,
                       int32_t compute_dtype, float strength, int32_t has_seed, uint64_t seed,
                       uint64_t offset_base, void* workspace, size_t workspace_bytes, void* stream) {
  if (storage < 0 || storage > 2)
    return fail(PIPER_MERGE_EINVAL, "Quanto storage must be 0 (qint8), 1 (qfloat8 e4m3) or 2 (qfloat8 e5m2).");
  piper_merge_desc d;
  std::memset(&d, 0, sizeof(d));
  d.format = storage == 0 ? PIPER_FMT_QUANTO_INT8 : (storage == 1 ? PIPER_FMT_QUANTO_FP8_E4M3 : PIPER_FMT_QUANTO_FP8_E5M2);
  d.qdata = qdata;
  d.scale = scale;
  d.b = b;
  d.a = a;
  d.rows = rows;
  d.cols = cols;
  d.rank = rank;
  d.block_rows = per_row ? 1 : rows;
  d.block_cols = cols;
  d.compute_dtype = compute_dtype;
  d.scale_dtype = compute_dtype;
  d.flags = has_seed ? PIPER_FLAG_STOCHASTIC : 0u;
  d.strength = strength;
  d.seed = seed;
  d.offset_base = offset_base;
  return piper_merge_batch(&d, 1, workspace, workspace_bytes, stream);
}

int piper_merge_bnb4(void* packed, void* absmax, const void* code, void* nested_absmax,
                     const void* nested_code, void* nested_offset, const void* b, const void* a,
                     int64_t rows, int64_t cols, int64_t rank, int32_t nf4, int32_t compute_dtype,
                     float strength, int32_t has_seed, uint64_t seed, uint64_t offset_base,
                     void* workspace, size_t workspace_bytes, void* stream) {
  piper_merge_desc d;
  std::memset(&d, 0, sizeof(d));
  d.format = nf4 ? PIPER_FMT_BNB4_NF4 : PIPER_FMT_BNB4_FP4;
  d.qdata = packed;
  d.scale = absmax;
  d.b = b;
  d.a = a;
  d.rows = rows;
  d.cols = cols;
  d.rank = rank;
  d.compute_dtype = compute_dtype;
  d.flags = has_seed ? PIPER_FLAG_STOCHASTIC : 0u;
  d.strength = strength;
  d.seed = seed;
  d.offset_base = offset_base;
  d.codebook = code;
  d.nested_absmax = nested_absmax;
  d.nested_code = nested_code;
  d.nested_offset = nested_offset;
  return piper_merge_batch(&d, 1, workspace, workspace_bytes, stream);
}

int piper_merge_gguf(void* raw, const void* b, const void* a, int64_t rows, int64_t cols, int64_t rank,
                     int32_t quant_type, int32_t compute_dtype, float strength, int32_t has_seed,
                     uint64_t seed, uint64_t offset_base, void* stream) {
  piper_merge_desc d;
  std::memset(&d, 0, sizeof(d));
  if (quant_type == 8) d.format = PIPER_FMT_GGUF_Q8_0;
  else if (quant_type == 2) d.format = PIPER_FMT_GGUF_Q4_0;
  else return fail(PIPER_MERGE_EINVAL, "GGUF merge supports Q8_0 (8) and Q4_0 (2), got " + std::to_string(quant_type) + ".");
  d.qdata = raw;
  d.b = b;
  d.a = a;
  d.rows = rows;
  d.cols = cols;
  d.rank = rank;
  d.compute_dtype = compute_dtype;
  d.flags = has_seed ? PIPER_FLAG_STOCHASTIC : 0u;
  d.strength = strength;
  d.seed = seed;
  d.offset_base = offset_base;
  return piper_merge_batch(&d, 1, nullptr, 0, stream);
}

const char* piper_merge_last_error(void) { return g_last_error.c_str(); }

int piper_merge_selftest_timeout(void* stream) {
  pm::selftest_wait_kernel<<<1, 32, 0, static_cast<cudaStream_t>(stream)>>>();
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return fail(PIPER_MERGE_ECUDA, std::string("self-test launch: ") + cudaGetErrorString(e));
  return PIPER_MERGE_OK;
}

int piper_merge_device_status(void* stream, uint32_t* status) {
  cudaError_t e = cudaStreamSynchronize(static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return fail(PIPER_MERGE_ECUDA, std::string("cudaStreamSynchronize: ") + cudaGetErrorString(e));
  unsigned int v = 0, zero = 0;
  e = cudaMemcpyFromSymbol(&v, pm::g_status, sizeof(v));
  if (e == cudaSuccess) e = cudaMemcpyToSymbol(pm::g_status, &zero, sizeof(zero));
  if (e != cudaSuccess) return fail(PIPER_MERGE_ECUDA, std::string("status word: ") + cudaGetErrorString(e));
  if (status) *status = v;
  return v == 0 ? PIPER_MERGE_OK : fail(PIPER_MERGE_ETIMEOUT, "a bounded device-side wait timed out.");
}

const char* piper_merge_version(void) { return "piper-merge 0.1 sm_100a"; }

uint64_t piper_merge_launches(void) { return g_launches.load(std::memory_order_relaxed); }

}  // extern "C"
