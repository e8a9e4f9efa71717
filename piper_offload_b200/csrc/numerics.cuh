// numerics.cuh - element-level arithmetic of the merge, kept bit-compatible with
// the reference kernels (src/piper_offload/_triton_*_lora.py):
//   * casts to bf16 / fp16 / e4m3 / e5m2 round to nearest even;
//   * fp32 quotients that the reference writes with `/` use the same
//     `div.full.f32` instruction Triton emits for fp32 division;
//   * `tl.minimum` / `tl.maximum` are IEEE minNum/maxNum (fminf/fmaxf);
//   * `base + acc * strength` is one fused multiply-add, as Triton contracts it.
// The file is compiled with --fmad=false so no other mul+add pair is fused.
#pragma once
#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include <cstdint>

namespace pm {

enum : int { kBF16 = 0, kF16 = 1, kF32 = 2 };

__device__ __forceinline__ float bf16r(float x) { return __bfloat162float(__float2bfloat16_rn(x)); }
__device__ __forceinline__ float f16r(float x) { return __half2float(__float2half_rn(x)); }

template <int DT>
__device__ __forceinline__ float round_dt(float x) {
  if constexpr (DT == kBF16) return bf16r(x);
  else if constexpr (DT == kF16) return f16r(x);
  else return x;
}

__device__ __forceinline__ float round_dt_rt(float x, int dt) {
  return dt == kBF16 ? bf16r(x) : (dt == kF16 ? f16r(x) : x);
}

// fp32 division as emitted by Triton for `a / b` on fp32 tensors.
__device__ __forceinline__ float div_full(float a, float b) {
  float r;
  asm("div.full.f32 %0, %1, %2;" : "=f"(r) : "f"(a), "f"(b));
  return r;
}

// ------------------------------------------------------------------ FP8
__device__ __forceinline__ uint32_t enc_e4m3(float x) {
  uint16_t r;
  asm("cvt.rn.satfinite.e4m3x2.f32 %0, %1, %2;" : "=h"(r) : "f"(0.0f), "f"(x));
  return r & 0xFFu;
}
__device__ __forceinline__ uint32_t enc_e5m2(float x) {
  uint16_t r;
  asm("cvt.rn.satfinite.e5m2x2.f32 %0, %1, %2;" : "=h"(r) : "f"(0.0f), "f"(x));
  return r & 0xFFu;
}
__device__ __forceinline__ float dec_e4m3(uint32_t code) {
  uint32_t h2;
  asm("cvt.rn.f16x2.e4m3x2 %0, %1;" : "=r"(h2) : "h"(static_cast<uint16_t>(code & 0xFFu)));
  return __half2float(__ushort_as_half(static_cast<unsigned short>(h2 & 0xFFFFu)));
}
__device__ __forceinline__ float dec_e5m2(uint32_t code) {
  uint32_t h2;
  asm("cvt.rn.f16x2.e5m2x2 %0, %1;" : "=r"(h2) : "h"(static_cast<uint16_t>(code & 0xFFu)));
  return __half2float(__ushort_as_half(static_cast<unsigned short>(h2 & 0xFFFFu)));
}
template <bool E4M3>
__device__ __forceinline__ uint32_t enc_fp8(float x) {
  if constexpr (E4M3) return enc_e4m3(x);
  else return enc_e5m2(x);
}
template <bool E4M3>
__device__ __forceinline__ float dec_fp8(uint32_t c) {
  if constexpr (E4M3) return dec_e4m3(c);
  else return dec_e5m2(c);
}

// E8M0 code -> fp32 (_e8m0_to_fp32, _triton_mx_lora.py:30-37).
__device__ __forceinline__ float dec_e8m0(uint32_t code) {
  code &= 0xFFu;
  if (code == 255u) return __uint_as_float(0x7FC00000u);
  return __uint_as_float(code == 0u ? (1u << 22) : (code << 23));
}

// ---------------------------------------------------------------- Philox
// Counter-based uniform of the reference's `_random(seed, offset)` =
// Triton `tl.rand`: Philox4x32 with 10 rounds, key = (seed lo, seed hi),
// counter = (offset lo, offset hi, 0, 0); output word 0 folded to a
// non-negative int32 and scaled by the fp32 constant 0x2FFFFFFF.
// Philox4x32-10 key schedule, computed once per chunk: round r uses
// (k0 + r * 0x9E3779B9, k1 + r * 0xBB67AE85). The round keys are the same for
// every element of a weight, so the element loop only multiplies and xors.
struct PhiloxKey {
  uint32_t k0[10], k1[10];
};

__device__ __forceinline__ PhiloxKey philox_key(uint32_t k0, uint32_t k1) {
  PhiloxKey k;
#pragma unroll
  for (int r = 0; r < 10; ++r) {
    k.k0[r] = k0 + static_cast<uint32_t>(r) * 0x9E3779B9u;
    k.k1[r] = k1 + static_cast<uint32_t>(r) * 0xBB67AE85u;
  }
  return k;
}

__device__ __forceinline__ uint32_t philox_word0(const PhiloxKey& key, uint64_t offset) {
  uint32_t c0 = static_cast<uint32_t>(offset);
  uint32_t c1 = static_cast<uint32_t>(offset >> 32);
  uint32_t c2 = 0u, c3 = 0u;
#pragma unroll
  for (int round = 0; round < 10; ++round) {
    const uint32_t hb = __umulhi(0xCD9E8D57u, c2);
    const uint32_t lb = 0xCD9E8D57u * c2;
    const uint32_t ha = __umulhi(0xD2511F53u, c0);
    const uint32_t la = 0xD2511F53u * c0;
    c0 = hb ^ c1 ^ key.k0[round];
    c2 = ha ^ c3 ^ key.k1[round];
    c1 = lb;
    c3 = la;
  }
  return c0;
}

__device__ __forceinline__ float philox_uniform(const PhiloxKey& key, uint64_t offset) {
  const int32_t w = static_cast<int32_t>(philox_word0(key, offset));
  const int32_t x = w ^ (w >> 31);  // x < 0 ? -x - 1 : x
  return __fmul_rn(__int2float_rn(x), __uint_as_float(0x2FFFFFFFu));
}

// ------------------------------------------------- stochastic terminal codes
// The helpers below are branch-free: the uniform draw is computed for every
// element (almost all are interior), so the 32 Philox chains of a chunk are
// independent instruction streams the scheduler can interleave.

// _stochastic_float8 (_triton_stochastic_quantization.py:132-175): `v` is the
// normalized value, already clamped to [-limit, limit] (a NaN became -limit);
// returns the E4M3/E5M2 code.
//
// The reference rounds |v| to nearest, steps one code down when that code is
// above |v|, and so takes lo = the largest code <= |v| and hi = lo + 1, then
// p = (|v| - lo) / (hi - lo). In the normal range lo is |v| with its mantissa
// truncated to 3 (2) bits, the gap is 2^(e-3) (2^(e-2)), and p is exactly the
// dropped mantissa bits scaled by 2^-20 (2^-21); below the smallest normal the
// codes are evenly spaced by 2^-9 (2^-16) and p is the fraction of |v| / gap.
// Where the result is not stochastic (p == 0 or |v| == limit) |v| is on the
// grid, so the reference's round-to-nearest code equals lo.
template <bool E4M3>
__device__ __forceinline__ uint32_t sr_fp8(float v, float limit, const PhiloxKey& key, uint64_t off) {
  constexpr int kMant = E4M3 ? 3 : 2;
  constexpr int kDrop = 23 - kMant;
  constexpr uint32_t kMinNormal = E4M3 ? 0x3C800000u : 0x38800000u;  // 2^-6 / 2^-14
  constexpr uint32_t kBiasFix = (127u - (E4M3 ? 7u : 15u)) << kMant;
  constexpr float kSubScale = E4M3 ? 512.0f : 65536.0f;               // 1 / subnormal gap
  const uint32_t bits = __float_as_uint(v);
  const uint32_t abits = bits & 0x7FFFFFFFu;
  const float mag = __uint_as_float(abits);
  // normal range
  const uint32_t lo_n = (abits >> kDrop) - kBiasFix;
  const float p_n = __uint_as_float(0x3F800000u | ((abits << kMant) & 0x7FFFFFu)) - 1.0f;
  // subnormal range (exact: scaling by a power of two, truncation, subtraction)
  const float t = mag * kSubScale;
  const float fl = truncf(t);
  const uint32_t lo_s = __float_as_uint(fl + 8388608.0f) - 0x4B000000u;
  const float p_s = t - fl;
  const bool normal = abits >= kMinNormal;
  const uint32_t lo = normal ? lo_n : lo_s;
  const float p = normal ? p_n : p_s;
  const float u = philox_uniform(key, off);
  const bool up = mag < limit && p > 0.0f && u < p;
  return (lo + (up ? 1u : 0u)) | ((bits >> 24) & 0x80u);
}

// N consecutive counters advanced round by round, so the N independent
// multiply chains issue back to back.
template <int N>
__device__ __forceinline__ void philox_word0_xn(const PhiloxKey& key, uint64_t offset, uint32_t (&w)[N]) {
  // Round 0 with counter words 2 and 3 zero: the second multiply is zero.
  uint32_t c0[N], c1[N], c2[N], c3[N];
  const uint32_t hi0 = static_cast<uint32_t>(offset >> 32);
  if (static_cast<uint32_t>((offset + static_cast<uint64_t>(N - 1)) >> 32) == hi0) {
    // The N low counter words are lo0 + j with no carry out of 32 bits, so the
    // round-0 products A * (lo0 + j) are A * lo0 + A * j: one wide multiply
    // and N 64-bit additions of constants.
    const uint64_t p0 = static_cast<uint64_t>(0xD2511F53u) * static_cast<uint32_t>(offset);
#pragma unroll
    for (int j = 0; j < N; ++j) {
      const uint64_t p = p0 + static_cast<uint64_t>(0xD2511F53u) * static_cast<uint64_t>(j);
      c0[j] = hi0 ^ key.k0[0];
      c2[j] = static_cast<uint32_t>(p >> 32) ^ key.k1[0];
      c1[j] = 0u;
      c3[j] = static_cast<uint32_t>(p);
    }
  } else {
#pragma unroll
    for (int j = 0; j < N; ++j) {
      const uint64_t o = offset + static_cast<uint64_t>(j);
      const uint32_t lo = static_cast<uint32_t>(o);
      c0[j] = static_cast<uint32_t>(o >> 32) ^ key.k0[0];
      c2[j] = __umulhi(0xD2511F53u, lo) ^ key.k1[0];
      c1[j] = 0u;
      c3[j] = 0xD2511F53u * lo;
    }
  }
  // Round 1: word 0 is (offset >> 32) ^ key, the same for the N counters
  // unless they straddle a multiple of 2^32, so its product is formed once.
  uint32_t ha[N], la[N];
  if (static_cast<uint32_t>((offset + static_cast<uint64_t>(N - 1)) >> 32) == hi0) {
    const uint32_t h = __umulhi(0xD2511F53u, c0[0]);
    const uint32_t l = 0xD2511F53u * c0[0];
#pragma unroll
    for (int j = 0; j < N; ++j) {
      ha[j] = h;
      la[j] = l;
    }
  } else {
#pragma unroll
    for (int j = 0; j < N; ++j) {
      ha[j] = __umulhi(0xD2511F53u, c0[j]);
      la[j] = 0xD2511F53u * c0[j];
    }
  }
#pragma unroll
  for (int j = 0; j < N; ++j) {
    const uint32_t hb = __umulhi(0xCD9E8D57u, c2[j]);
    const uint32_t lb = 0xCD9E8D57u * c2[j];
    c0[j] = hb ^ c1[j] ^ key.k0[1];
    c2[j] = ha[j] ^ c3[j] ^ key.k1[1];
    c1[j] = lb;
    c3[j] = la[j];
  }
#pragma unroll
  for (int round = 2; round < 10; ++round) {
#pragma unroll
    for (int j = 0; j < N; ++j) {
      const uint32_t hb = __umulhi(0xCD9E8D57u, c2[j]);
      const uint32_t lb = 0xCD9E8D57u * c2[j];
      const uint32_t hm = __umulhi(0xD2511F53u, c0[j]);
      const uint32_t lm = 0xD2511F53u * c0[j];
      c0[j] = hb ^ c1[j] ^ key.k0[round];
      c2[j] = hm ^ c3[j] ^ key.k1[round];
      c1[j] = lb;
      c3[j] = lm;
    }
  }
#pragma unroll
  for (int j = 0; j < N; ++j) w[j] = c0[j];
}


// sr_fp8 for N consecutive elements (offsets off .. off+N-1), packed four to
// a word as little-endian bytes; same arithmetic as sr_fp8.
template <bool E4M3, int N>
__device__ __forceinline__ void sr_fp8xn(const float (&v)[N], float limit, const PhiloxKey& key, uint64_t off,
                                         uint32_t (&words)[N / 4]) {
  constexpr int kMant = E4M3 ? 3 : 2;
  constexpr int kDrop = 23 - kMant;
  constexpr uint32_t kMinNormal = E4M3 ? 0x3C800000u : 0x38800000u;
  constexpr uint32_t kBiasFix = (127u - (E4M3 ? 7u : 15u)) << kMant;
  constexpr float kSubScale = E4M3 ? 512.0f : 65536.0f;
  uint32_t r[N];
  philox_word0_xn<N>(key, off, r);
  uint32_t lo[N];
  float p[N];
  bool sub = false;
#pragma unroll
  for (int j = 0; j < N; ++j) {
    const uint32_t abits = __float_as_uint(v[j]) & 0x7FFFFFFFu;
    lo[j] = (abits >> kDrop) - kBiasFix;
    p[j] = __uint_as_float(0x3F800000u | ((abits << kMant) & 0x7FFFFFu)) - 1.0f;
    sub |= abits < kMinNormal;
  }
  // Below the smallest normal (zero included) the codes are evenly spaced;
  // that path runs only when a lane of the active part of the warp needs it.
  if (__any_sync(__activemask(), sub)) {
#pragma unroll
    for (int j = 0; j < N; ++j) {
      const uint32_t abits = __float_as_uint(v[j]) & 0x7FFFFFFFu;
      const float t = __uint_as_float(abits) * kSubScale;
      const float fl = truncf(t);
      if (abits < kMinNormal) {
        lo[j] = __float_as_uint(fl + 8388608.0f) - 0x4B000000u;
        p[j] = t - fl;
      }
    }
  }
#pragma unroll
  for (int w = 0; w < N / 4; ++w) words[w] = 0u;
#pragma unroll
  for (int j = 0; j < N; ++j) {
    const uint32_t bits = __float_as_uint(v[j]);
    const float mag = __uint_as_float(bits & 0x7FFFFFFFu);
    const int32_t x = static_cast<int32_t>(r[j]) ^ (static_cast<int32_t>(r[j]) >> 31);
    const float u = __fmul_rn(__int2float_rn(x), __uint_as_float(0x2FFFFFFFu));
    const bool up = mag < limit && p[j] > 0.0f && u < p[j];
    words[j >> 2] |= ((lo[j] + (up ? 1u : 0u)) | ((bits >> 24) & 0x80u)) << (8 * (j & 3));
  }
}

// _stochastic_e2m1_code (_triton_stochastic_quantization.py:109-129) for N
// consecutive elements (offsets off .. off+N-1) of values already clamped to
// [-6, 6], as nibbles (element j in bits 4j .. 4j+3 of word j / 8).
// The lower code lc (largest magnitude <= |v|) and p = (|v| - lv) / gap follow
// from the fp32 bits: below 0.5 lc = 0 and p = 2|v|; in [0.5, 1) lc = 1 and
// p = 2|v| - 1; from 1 up, (bits >> 22) - 252 is 2e + 2 + the top mantissa bit
// = lc and p is the mantissa below its top bit (all exact, as the reference's
// p is). Where the rounding is not stochastic |v| lies on a code (p == 0) or
// is 6, and the reference's round-to-nearest code is lc there (7 for 6).
template <int N>
__device__ __forceinline__ void sr_e2m1xn(const float (&v)[N], const PhiloxKey& key, uint64_t off,
                                          uint32_t (&out)[(N + 7) / 8]) {
  uint32_t r[N];
  philox_word0_xn<N>(key, off, r);
#pragma unroll
  for (int w = 0; w < (N + 7) / 8; ++w) out[w] = 0u;
#pragma unroll
  for (int j = 0; j < N; ++j) {
    const uint32_t bits = __float_as_uint(v[j]);
    const uint32_t abits = bits & 0x7FFFFFFFu;
    const float mag = __uint_as_float(abits);
    const bool small = abits < 0x3F000000u;  // |v| < 0.5
    const bool below1 = abits < 0x3F800000u;  // |v| < 1
    const uint32_t lc = small ? 0u : min(max((abits >> 22) - 252u, 1u), 7u);
    const float twice = __fmul_rn(mag, 2.0f);
    const float p = small ? twice
                    : below1 ? __fsub_rn(twice, 1.0f)
                             : __fsub_rn(__uint_as_float(0x3F800000u | ((abits << 1) & 0x7FFFFFu)), 1.0f);
    const int32_t x = static_cast<int32_t>(r[j]) ^ (static_cast<int32_t>(r[j]) >> 31);
    const float u = __fmul_rn(__int2float_rn(x), __uint_as_float(0x2FFFFFFFu));
    const bool up = mag < 6.0f && p > 0.0f && u < p;
    out[j >> 3] |= ((lc + (up ? 1u : 0u)) | ((bits >> 28) & 8u)) << (4 * (j & 7));
  }
}

// _stochastic_round_to_int (_triton_stochastic_quantization.py:24-39);
// returns the (possibly) re-rounded value as a float.
__device__ __forceinline__ float sr_int(float v, float det, float qmin, float qmax, const PhiloxKey& key,
                                        uint64_t off) {
  const float lower = floorf(v);
  const float p = __fsub_rn(v, lower);
  const float u = philox_uniform(key, off);
  const bool interior = v > qmin && v < qmax && p > 0.0f;
  return interior ? __fadd_rn(lower, u < p ? 1.0f : 0.0f) : det;
}

// sr_int for N consecutive elements (offsets off .. off+N-1): q[j] holds the
// round-to-nearest value on entry and the result on exit. qmin and qmax lie
// within +-2^22, so an interior v does too, and there floor(v) is the fp32
// sum v + 1.5 * 2^23 rounded down, less 1.5 * 2^23 (both steps exact).
template <int N>
__device__ __forceinline__ void sr_int_xn(const float (&v)[N], float (&q)[N], float qmin, float qmax,
                                          const PhiloxKey& key, uint64_t off) {
  uint32_t r[N];
  philox_word0_xn<N>(key, off, r);
#pragma unroll
  for (int j = 0; j < N; ++j) {
    const float lower = __fsub_rn(__fadd_rd(v[j], 12582912.0f), 12582912.0f);
    const float p = __fsub_rn(v[j], lower);
    const int32_t x = static_cast<int32_t>(r[j]) ^ (static_cast<int32_t>(r[j]) >> 31);
    const float u = __fmul_rn(__int2float_rn(x), __uint_as_float(0x2FFFFFFFu));
    const bool interior = v[j] > qmin && v[j] < qmax && p > 0.0f;
    q[j] = interior ? __fadd_rn(lower, u < p ? 1.0f : 0.0f) : q[j];
  }
}

}  // namespace pm

namespace pm {
// ------------------------------------------------------ packed conversions
// Two fp32 values rounded to bf16 (RTNE) and widened back; one packed cvt.
__device__ __forceinline__ void bf16r2(float& a, float& b) {
  uint32_t d;
  asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(d) : "f"(b), "f"(a));
  // Widen with byte permutes (the ALU pipe), leaving the integer multiply pipe
  // to the Philox multiplies.
  a = __uint_as_float(__byte_perm(d, 0u, 0x1044u));
  b = __uint_as_float(__byte_perm(d, 0u, 0x3244u));
}
__device__ __forceinline__ void f16r2(float& a, float& b) {
  const __half2 h = __floats2half2_rn(a, b);
  const float2 f = __half22float2(h);
  a = f.x;
  b = f.y;
}
template <int DT>
__device__ __forceinline__ void round_dt2(float& a, float& b) {
  if constexpr (DT == kBF16) bf16r2(a, b);
  else if constexpr (DT == kF16) f16r2(a, b);
}

// Four FP8 codes (little-endian bytes of w) to fp32, two per cvt.
template <bool E4M3>
__device__ __forceinline__ void dec_fp8x4(uint32_t w, float (&f)[4]) {
  uint32_t lo, hi;
  if constexpr (E4M3) {
    asm("cvt.rn.f16x2.e4m3x2 %0, %1;" : "=r"(lo) : "h"(static_cast<uint16_t>(w & 0xFFFFu)));
    asm("cvt.rn.f16x2.e4m3x2 %0, %1;" : "=r"(hi) : "h"(static_cast<uint16_t>(w >> 16)));
  } else {
    asm("cvt.rn.f16x2.e5m2x2 %0, %1;" : "=r"(lo) : "h"(static_cast<uint16_t>(w & 0xFFFFu)));
    asm("cvt.rn.f16x2.e5m2x2 %0, %1;" : "=r"(hi) : "h"(static_cast<uint16_t>(w >> 16)));
  }
  const float2 a = __half22float2(*reinterpret_cast<const __half2*>(&lo));
  const float2 b = __half22float2(*reinterpret_cast<const __half2*>(&hi));
  f[0] = a.x;
  f[1] = a.y;
  f[2] = b.x;
  f[3] = b.y;
}

// Four fp32 values to FP8 codes (RTNE, satfinite), packed little-endian.
template <bool E4M3>
__device__ __forceinline__ uint32_t enc_fp8x4(float a, float b, float c, float d) {
  uint16_t lo, hi;
  if constexpr (E4M3) {
    asm("cvt.rn.satfinite.e4m3x2.f32 %0, %1, %2;" : "=h"(lo) : "f"(b), "f"(a));
    asm("cvt.rn.satfinite.e4m3x2.f32 %0, %1, %2;" : "=h"(hi) : "f"(d), "f"(c));
  } else {
    asm("cvt.rn.satfinite.e5m2x2.f32 %0, %1, %2;" : "=h"(lo) : "f"(b), "f"(a));
    asm("cvt.rn.satfinite.e5m2x2.f32 %0, %1, %2;" : "=h"(hi) : "f"(d), "f"(c));
  }
  return __byte_perm(static_cast<uint32_t>(lo), static_cast<uint32_t>(hi), 0x5410u);
}

// Two E2M1 codes (low nibble first) of one byte to fp32. The reference applies
// the sign as `-magnitude`, which Triton lowers to `0.0 - magnitude`, so code 8
// decodes to +0.0 there; the f16x2 add of +0 gives the same (-0 + +0 = +0, every
// other value unchanged).
__device__ __forceinline__ void dec_e2m1x2(uint32_t byte, float& a, float& b) {
  uint32_t h;
  asm("{\n\t.reg .b8 t0, t1;\n\tmov.b16 {t0, t1}, %1;\n\tcvt.rn.f16x2.e2m1x2 %0, t0;\n\t"
      "add.rn.f16x2 %0, %0, %2;\n\t}"
      : "=r"(h)
      : "h"(static_cast<uint16_t>(byte & 0xFFu)), "r"(0u));
  const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&h));
  a = f.x;
  b = f.y;
}

// Two fp32 values to one byte of E2M1 codes (RTNE, satfinite; first value in the low nibble).
__device__ __forceinline__ uint32_t enc_e2m1x2(float lo, float hi) {
  uint16_t r;
  asm("{\n\t.reg .b8 t;\n\tcvt.rn.satfinite.e2m1x2.f32 t, %1, %2;\n\tmov.b16 %0, {t, 0};\n\t}"
      : "=h"(r)
      : "f"(hi), "f"(lo));
  return r & 0xFFu;
}

// ------------------------------------------- quotients near rounding edges
// The reference divides with `div.full.f32`, whose result is within 2 ulp of
// the exact quotient. A quotient computed as x * RN(1/s) is within 1.5 ulp.
// When that approximation is farther than 4 ulp from every rounding boundary
// of the target format, both quotients round to the same code; otherwise the
// caller recomputes with div.full.f32 itself.

// FP8 boundary test: midpoints have the bits below the kept mantissa equal to
// exactly half; values in the subnormal range are always re-checked.
template <bool E4M3>
__device__ __forceinline__ bool near_fp8_edge(float q) {
  const uint32_t a = __float_as_uint(q) & 0x7FFFFFFFu;
  constexpr uint32_t kMinNormal = E4M3 ? 0x3C800000u : 0x38800000u;  // 2^-6 / 2^-14
  constexpr int kDrop = E4M3 ? 20 : 21;
  constexpr uint32_t kMask = (1u << kDrop) - 1u;
  constexpr uint32_t kHalf = 1u << (kDrop - 1);
  const uint32_t low = a & kMask;
  const uint32_t dist = low > kHalf ? low - kHalf : kHalf - low;
  return a < kMinNormal || dist <= 4u;
}

// E2M1 boundary test (0.25, 0.75, 1.25, 1.75, 2.5, 3.5, 5): within 4 ulp of a
// value whose mantissa is a multiple of 2^21 in binades 2^-3 .. 2^2.
__device__ __forceinline__ bool near_e2m1_edge(float q) {
  const uint32_t a = __float_as_uint(q) & 0x7FFFFFFFu;
  const int e = static_cast<int>(a >> 23) - 127;
  const uint32_t low = a & 0x1FFFFFu;
  return e >= -3 && e <= 2 && (low <= 4u || low >= 0x200000u - 4u);
}

// sr_fp8xn for values that are finite with |v| <= limit * (1 + 2^-8), as the
// quotients of an all-finite row are: the same codes with fewer instructions.
//  * Lower neighbour: in the normal range, |v| with the fp32 bits below the
//    kept mantissa cleared is the largest FP8 value <= |v|; the upper one is
//    that plus 2^kDrop in the bits. Both keep v's sign, and the satfinite
//    conversion turns a step past the largest finite value back into it, the
//    reference's non-stochastic result for |v| >= limit.
//  * Draw: the reference's u = fp32(fp32(x) * c), c = 2^-31 (1 - 2^-24), is the
//    float just below z = fp32(x) * 2^-31 for every x >= 1 (the product
//    z - z * 2^-24 lies within half an ulp above that float), so for p > 0,
//    u < p holds exactly when z <= p, i.e. fp32(x) <= p * 2^31; x = 0 gives
//    u = 0 < p as well. p * 2^31 is read off the mantissa bits like p.
//  * Below the smallest normal the grid is uniform (gap 2^-9 / 2^-16); that
//    branch runs only when a lane of the active part of the warp needs it.
template <bool E4M3, int N>
__device__ __forceinline__ void sr_fp8xn_finite(const float (&v)[N], const PhiloxKey& key, uint64_t off,
                                                uint32_t (&words)[N / 4]) {
  constexpr int kMant = E4M3 ? 3 : 2;
  constexpr int kDrop = 23 - kMant;
  constexpr uint32_t kMinNormal = E4M3 ? 0x3C800000u : 0x38800000u;
  constexpr float kSubScale = E4M3 ? 512.0f : 65536.0f;
  constexpr float kSubGap = E4M3 ? 1.0f / 512.0f : 1.0f / 65536.0f;
  uint32_t r[N];
  philox_word0_xn<N>(key, off, r);
  float P[N];      // p * 2^31
  uint32_t y[N];   // fp32 bits of the chosen FP8 value
  bool sub = false;
#pragma unroll
  for (int j = 0; j < N; ++j) {
    const uint32_t bits = __float_as_uint(v[j]);
    const uint32_t abits = bits & 0x7FFFFFFFu;
    sub |= abits < kMinNormal;
    P[j] = __uint_as_float(0x4F000000u | ((abits << kMant) & 0x7FFFFFu)) - 2147483648.0f;
    y[j] = bits & ~((1u << kDrop) - 1u);
  }
  const bool any_sub = __any_sync(__activemask(), sub);
  if (any_sub) {
#pragma unroll
    for (int j = 0; j < N; ++j) {
      const float t = __uint_as_float(__float_as_uint(v[j]) & 0x7FFFFFFFu) * kSubScale;
      const float fl = truncf(t);
      if ((__float_as_uint(v[j]) & 0x7FFFFFFFu) < kMinNormal) P[j] = (t - fl) * 2147483648.0f;
    }
  }
#pragma unroll
  for (int j = 0; j < N; ++j) {
    const int32_t x = static_cast<int32_t>(r[j]) ^ (static_cast<int32_t>(r[j]) >> 31);
    const bool up = P[j] > 0.0f && __int2float_rn(x) <= P[j];
    y[j] += up ? (1u << kDrop) : 0u;
  }
  if (any_sub) {  // the draw is taken again for values below the smallest normal
#pragma unroll
    for (int j = 0; j < N; ++j) {
      const uint32_t bits = __float_as_uint(v[j]);
      const int32_t x = static_cast<int32_t>(r[j]) ^ (static_cast<int32_t>(r[j]) >> 31);
      const bool up = P[j] > 0.0f && __int2float_rn(x) <= P[j];
      const float t = __uint_as_float(bits & 0x7FFFFFFFu) * kSubScale;
      const float fl = truncf(t) + (up ? 1.0f : 0.0f);
      if ((bits & 0x7FFFFFFFu) < kMinNormal) y[j] = __float_as_uint(fl * kSubGap) | (bits & 0x80000000u);
    }
  }
#pragma unroll
  for (int w = 0; w < N / 4; ++w)
    words[w] = enc_fp8x4<E4M3>(__uint_as_float(y[4 * w]), __uint_as_float(y[4 * w + 1]), __uint_as_float(y[4 * w + 2]),
                               __uint_as_float(y[4 * w + 3]));
}

}  // namespace pm
