// Device-side building blocks shared by every sm_100a kernel of the library:
// the counter hash and key derivation, FP32/BF16/FP16/FP8 loads and stores of
// 8-element vectors, and the nearest / stochastic storage rounding rules.
//
// Numerical contract (bit-exact with the reference CPU implementation):
//   hash            sr_states/_hash.py:10-15 and :31-50
//   keys            sr_states/_hash.py:18-28, device mirror sr_states/triton/_keys.py:20-30
//   BF16 stochastic sr_states/_bf16.py:37-74
//   FP16/FP8 rules  sr_states/_minifloat.py:10-70 (24-bit probability grid, saturating FP8)
#pragma once

#include <cstdint>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_fp8.h>
#include <cuda_runtime.h>

#include "srs_b200.h"

namespace srs {

constexpr int kThreads = 256;              // CTA size of every kernel
constexpr int kVec = 8;                    // elements per thread per tile
constexpr int64_t kTile = kThreads * kVec; // elements per tile (row table unit)

// ------------------------------------------------------ packed FP32 math --
//
// Two-lane FP32 arithmetic on sm_100 (add/mul/fma .f32x2 on a 64-bit register
// pair), each lane rounded to nearest once.  Measured on B200 with CUDA 12.9:
// a packed multiply whose only use is a packed add IS fused into one FMA, even
// with the explicit .rn modifier (and so is CUDA's __fadd2_rn(__fmul2_rn())).
// So a product that must be rounded before an addition never goes through
// these helpers: such pairs use mul_add_rn2 below (scalar __fmul_rn/__fadd_rn,
// which CUDA documents as never merged).  A packed product feeding an FMA
// operand, or an FMA result feeding an add, cannot be fused and is safe.

__device__ __forceinline__ float2 mul2_rn(float2 a, float2 b) {
  float2 d;
  asm("{\n\t.reg .b64 pa, pb, pd;\n\t"
      "mov.b64 pa, {%2, %3};\n\tmov.b64 pb, {%4, %5};\n\t"
      "mul.rn.f32x2 pd, pa, pb;\n\tmov.b64 {%0, %1}, pd;\n\t}"
      : "=f"(d.x), "=f"(d.y)
      : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y));
  return d;
}

__device__ __forceinline__ float2 add2_rn(float2 a, float2 b) {
  float2 d;
  asm("{\n\t.reg .b64 pa, pb, pd;\n\t"
      "mov.b64 pa, {%2, %3};\n\tmov.b64 pb, {%4, %5};\n\t"
      "add.rn.f32x2 pd, pa, pb;\n\tmov.b64 {%0, %1}, pd;\n\t}"
      : "=f"(d.x), "=f"(d.y)
      : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y));
  return d;
}

// a*b + c with one rounding per lane.
__device__ __forceinline__ float2 fma2_rn(float2 a, float2 b, float2 c) {
  float2 d;
  asm("{\n\t.reg .b64 pa, pb, pc, pd;\n\t"
      "mov.b64 pa, {%2, %3};\n\tmov.b64 pb, {%4, %5};\n\tmov.b64 pc, {%6, %7};\n\t"
      "fma.rn.f32x2 pd, pa, pb, pc;\n\tmov.b64 {%0, %1}, pd;\n\t}"
      : "=f"(d.x), "=f"(d.y)
      : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y), "f"(c.x), "f"(c.y));
  return d;
}

// a*b + c rounded toward zero, per lane.
__device__ __forceinline__ float2 fma2_rz(float2 a, float2 b, float2 c) {
  float2 d;
  asm("{\n\t.reg .b64 pa, pb, pc, pd;\n\t"
      "mov.b64 pa, {%2, %3};\n\tmov.b64 pb, {%4, %5};\n\tmov.b64 pc, {%6, %7};\n\t"
      "fma.rz.f32x2 pd, pa, pb, pc;\n\tmov.b64 {%0, %1}, pd;\n\t}"
      : "=f"(d.x), "=f"(d.y)
      : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y), "f"(c.x), "f"(c.y));
  return d;
}

// RN(RN(a*b) + c) per lane: the product is rounded before the addition.
__device__ __forceinline__ float2 mul_add_rn2(float2 a, float2 b, float2 c) {
  return make_float2(__fadd_rn(__fmul_rn(a.x, b.x), c.x), __fadd_rn(__fmul_rn(a.y, b.y), c.y));
}

__device__ __forceinline__ float2 splat2(float x) { return make_float2(x, x); }

// ---------------------------------------------------------------- hashing --

__device__ __forceinline__ uint32_t h32(uint32_t x) {
  x ^= x >> 16;
  x *= 0x7FEB352Du;
  x ^= x >> 15;
  x *= 0x846CA68Bu;
  return x ^ (x >> 16);
}

__device__ __forceinline__ uint32_t update_key(const srs_rng& r, uint32_t param_index) {
  uint32_t k = h32(r.seed_lo ^ 0x9E3779B9u);
  k = h32(k ^ r.seed_hi);
  k = h32(k ^ r.step_lo);
  k = h32(k ^ r.step_hi);
  return h32(k ^ param_index);
}

__device__ __forceinline__ uint32_t state_key(uint32_t key, uint32_t index) {
  return h32(key ^ index);
}

// ------------------------------------------------------------ FP8 helpers --

__device__ __forceinline__ float2 e4m3x2_to_float2(uint32_t pair) {
  __half2_raw h = __nv_cvt_fp8x2_to_halfraw2((__nv_fp8x2_storage_t)pair, __NV_E4M3);
  return __half22float2(*reinterpret_cast<__half2*>(&h));
}

// An E5M2 byte is the high byte of the FP16 with the same value.
__device__ __forceinline__ float2 e5m2x2_to_float2(uint32_t pair) {
  const uint32_t w = __byte_perm(pair, 0u, 0x1404u);  // [0, b0, 0, b1]
  return __half22float2(*reinterpret_cast<const __half2*>(&w));
}

__device__ __forceinline__ float2 bf16x2_to_float2(uint32_t w) {
  return make_float2(__uint_as_float(w << 16), __uint_as_float(w & 0xFFFF0000u));
}

__device__ __forceinline__ float2 f16x2_to_float2(uint32_t w) {
  return __half22float2(*reinterpret_cast<const __half2*>(&w));
}

// --------------------------------------------------- stochastic rounding --

// BF16: add the low 16 hash bits to the FP32 encoding and truncate.  Infinities
// survive the addition unchanged; NaN is stored as 0xFFFF, the encoding the
// reference's CPU conversion produces for every NaN.
__device__ __forceinline__ uint32_t bf16_stochastic(float x, uint32_t h) {
  const uint32_t r = (__float_as_uint(x) + (h & 0xFFFFu)) >> 16;
  return (x != x) ? 0xFFFFu : r;
}

// Stochastic rounding of a finite, non-negative FP32 encoding `u` onto a
// minifloat grid with M mantissa bits whose smallest normal power of two has
// FP32 biased exponent EBMIN.  Returns the target magnitude encoding.
//
// The reference evaluates, in exact FP32 arithmetic,
//   e' = max(e, emin); s = |x| * 2^(M-e'); q = floor(s);
//   R = floor((s - q) * 2^24); up = (hash >> 8) < R; result = (q + up) * 2^(e'-M).
// Here the same quantities are taken from the integer encoding: with the
// significand F (implicit bit set) and d = e' - e extra shift bits,
//   q0 = F >> (23-M), r0 = F << (9+M) (the 23-M discarded bits, left-aligned),
//   q = q0 >> d, and floor((s-q) * 2^32) = low word of (q0:r0) >> d.
// Clearing its low 8 bits turns the 32-bit fraction into R * 2^8, so
// (hash >> 8) < R  <=>  hash < (R << 8).  Result encoding = (max(E-EBMIN,0) << M) + q + up,
// which also carries into the next binade (or from subnormal into normal).
// FP32 subnormals (E == 0) get a spurious implicit bit, but then d >= EBMIN - 1
// and every retained bit is shifted out, exactly as the reference's result.
template <int M, int EBMIN>
__device__ __forceinline__ uint32_t grid_stochastic_magnitude(uint32_t u, uint32_t h) {
  const int E = (int)(u >> 23);
  const int ex = max(E - EBMIN, 0);
  const int d = ex - E + EBMIN;  // max(EBMIN - E, 0)
  const uint32_t q0 = ((u >> (23 - M)) & ((1u << M) - 1u)) | (1u << M);
  const uint32_t r0 = u << (9 + M);
  const uint32_t q = __funnelshift_rc(q0, 0u, (uint32_t)d);
  uint32_t frac32;
  if constexpr (M < 8) {
    // q0 < 256: for d >= 32 the clamped shift leaves q0 >> 0 < 256, which the
    // mask below clears, matching the exact (zero) 24-bit threshold.
    frac32 = __funnelshift_rc(r0, q0, (uint32_t)d);
  } else {
    frac32 = (d < 32) ? __funnelshift_rc(r0, q0, (uint32_t)d)
                      : __funnelshift_rc(q0, 0u, (uint32_t)(d - 32));
  }
  const uint32_t up = (h < (frac32 & 0xFFFFFF00u)) ? 1u : 0u;
  return ((uint32_t)ex << M) + q + up;
}

// FP8 E4M3 (torch.float8_e4m3fn): |x| clamped to 448 first, NaN -> sign|0x7F.
__device__ __forceinline__ uint32_t e4m3_stochastic(float x, uint32_t h) {
  const uint32_t b = __float_as_uint(x);
  const uint32_t u = min(b & 0x7FFFFFFFu, 0x43E00000u);  // 448.0f
  uint32_t r = grid_stochastic_magnitude<3, 121>(u, h);
  r = (x != x) ? 0x7Fu : r;
  return r | ((b >> 24) & 0x80u);
}

// FP8 E5M2: |x| clamped to 57344 first, NaN -> sign|0x7F.
__device__ __forceinline__ uint32_t e5m2_stochastic(float x, uint32_t h) {
  const uint32_t b = __float_as_uint(x);
  const uint32_t u = min(b & 0x7FFFFFFFu, 0x47600000u);  // 57344.0f
  uint32_t r = grid_stochastic_magnitude<2, 113>(u, h);
  r = (x != x) ? 0x7Fu : r;
  return r | ((b >> 24) & 0x80u);
}

// FP16: IEEE behaviour.  Finite results at or above 2^16 are infinity; +-Inf
// stays infinite; NaN keeps the F16C encoding (quiet bit, top payload bits).
__device__ __forceinline__ uint32_t f16_stochastic(float x, uint32_t h) {
  const uint32_t b = __float_as_uint(x);
  const uint32_t u = b & 0x7FFFFFFFu;
  uint32_t r = min(grid_stochastic_magnitude<10, 113>(u, h), 0x7C00u);
  if (u >= 0x7F800000u) r = (u == 0x7F800000u) ? 0x7C00u : (0x7E00u | ((u >> 13) & 0x3FFu));
  return r | ((b >> 16) & 0x8000u);
}

// ------------------------------------------------------ round toward zero --
//
// The value of largest magnitude not above |x| in the format, sign kept:
// truncation onto the same grid, i.e. the stochastic rule with a hash that
// never rounds up (h = 0xFFFFFFFF is not below any 24-bit threshold << 8).
// Overflow follows IEEE round-toward-zero where the format has infinities to
// keep (BF16, FP16: finite values end at the largest finite value, +-Inf
// stays infinite) and saturation for FP8 (+-Inf -> +-max finite).  NaN is
// stored as the other rules store it.

__device__ __forceinline__ uint32_t bf16_toward_zero(float x) {
  return (x != x) ? 0xFFFFu : (__float_as_uint(x) >> 16);
}

__device__ __forceinline__ uint32_t e4m3_toward_zero(float x) { return e4m3_stochastic(x, ~0u); }

__device__ __forceinline__ uint32_t e5m2_toward_zero(float x) { return e5m2_stochastic(x, ~0u); }

__device__ __forceinline__ uint32_t f16_toward_zero(float x) {
  const uint32_t b = __float_as_uint(x);
  const uint32_t u = b & 0x7FFFFFFFu;
  if (u < 0x7F800000u) {  // finite: clamp to 65504 (0x477FE000) and truncate
    return grid_stochastic_magnitude<10, 113>(min(u, 0x477FE000u), ~0u) | ((b >> 16) & 0x8000u);
  }
  return f16_stochastic(x, ~0u);  // +-Inf and NaN
}

template <int F>
__device__ __forceinline__ uint32_t toward_zero1(float x) {
  if constexpr (F == SRS_FMT_BF16) return bf16_toward_zero(x);
  else if constexpr (F == SRS_FMT_F16) return f16_toward_zero(x);
  else if constexpr (F == SRS_FMT_E4M3) return e4m3_toward_zero(x);
  else return e5m2_toward_zero(x);
}

// ------------------------------------- stochastic rounding of screened vectors --
//
// Fast forms of the rules above for 8-element vectors that passed a screen (no
// NaN; for the FP16/FP8 grids every |x| < 2^63).  Vectors that fail it use the
// per-element functions above, so results are identical either way.
//
// BF16: the same integer addition as bf16_stochastic, done by the hardware's
// stochastic conversion (cvt_rs_bf16x2) for two elements at a time.
//
// FP16/FP8 grids, in FP32 arithmetic.  With U = 2^(max(e, emin) - M) the grid
// step at |x| and N = (~h) >> 8, the reference's decision
//   up = (h >> 8) < floor(frac * 2^24),  frac = |x|/U - floor(|x|/U),
// is the carry of frac*2^24 + N past 2^24, so the rounded magnitude is
// floor_U(|x| + N*U*2^-24).  Computed as
//   a = RZ(|x| + N*U*2^-24)   (N*U*2^-24 is exact: 24-bit N, power-of-two U)
//   b = RZ(a + U*2^23)        (U*2^23 has unit in the last place U)
//   y = b - U*2^23            (exact)
// Rounding toward zero never carries a sum across a multiple of U, as every
// such multiple in range is an FP32 number, so floor_U(a) is the exact floor;
// adding U*2^23 then keeps whole steps only.  y lies on the target grid or
// beyond its largest finite value, so the hardware round-to-nearest conversion
// stores it exactly (saturating for FP8, overflowing to infinity for FP16), and
// the sign of x is put back on y.  Checked against the CPU oracle for all 2^32
// FP32 inputs, at random hashes and at the hashes on both sides of each
// input's threshold.
template <int F> struct Grid;
template <> struct Grid<SRS_FMT_F16> {
  static constexpr int M = 10;
  static constexpr float kMinNormal = 0x1p-14f;
};
template <> struct Grid<SRS_FMT_E4M3> {
  static constexpr int M = 3;
  static constexpr float kMinNormal = 0x1p-6f;
};
template <> struct Grid<SRS_FMT_E5M2> {
  static constexpr int M = 2;
  static constexpr float kMinNormal = 0x1p-14f;
};

// N * 2^8 for N = (~h) >> 8: the complemented top 24 hash bits, exact as a float.
__device__ __forceinline__ float grid_noise(uint32_t h) {
  return __uint2float_rn(~h & 0xFFFFFF00u);
}

// Rounded values of two screened elements with hashes h0, h1 (still FP32, on
// the target grid).
template <int F>
__device__ __forceinline__ float2 grid_stochastic2(float2 x, uint32_t h0, uint32_t h1) {
  constexpr int M = Grid<F>::M;
  constexpr float kStep = (float)(1 << (23 - M));            // U*2^23 / 2^e'
  constexpr float kNoise = 1.0f / (float)(1ull << (32 + M));  // 2^-(32+M)
  const float ax = fabsf(x.x), ay = fabsf(x.y);
  const float2 s = make_float2(
      __uint_as_float(__float_as_uint(fmaxf(ax, Grid<F>::kMinNormal)) & 0x7F800000u),
      __uint_as_float(__float_as_uint(fmaxf(ay, Grid<F>::kMinNormal)) & 0x7F800000u));
  const float2 n = mul2_rn(make_float2(grid_noise(h0), grid_noise(h1)), splat2(kNoise));
  const float2 a = fma2_rz(n, s, make_float2(ax, ay));
  const float2 b = fma2_rz(s, splat2(kStep), a);
  const float2 y = fma2_rn(s, splat2(-kStep), b);
  return make_float2(__uint_as_float(__float_as_uint(y.x) | (__float_as_uint(x.x) & 0x80000000u)),
                     __uint_as_float(__float_as_uint(y.y) | (__float_as_uint(x.y) & 0x80000000u)));
}

// Screens.  BF16: no NaN among the 8 (a NaN makes the sum NaN).  Grids: the
// sum of squares is below 2^126, so no element is NaN, infinite or >= 2^63.
__device__ __forceinline__ bool screen_bf16(const float (&x)[kVec]) {
  const float2 s = add2_rn(add2_rn(make_float2(x[0], x[1]), make_float2(x[2], x[3])),
                           add2_rn(make_float2(x[4], x[5]), make_float2(x[6], x[7])));
  const float t = s.x + s.y;
  return t == t;
}

__device__ __forceinline__ bool screen_grid(const float (&x)[kVec]) {
  float2 s = mul2_rn(make_float2(x[0], x[1]), make_float2(x[0], x[1]));
  s = fma2_rn(make_float2(x[2], x[3]), make_float2(x[2], x[3]), s);
  s = fma2_rn(make_float2(x[4], x[5]), make_float2(x[4], x[5]), s);
  s = fma2_rn(make_float2(x[6], x[7]), make_float2(x[6], x[7]), s);
  return s.x + s.y < 0x1p126f;
}

// ------------------------------------------------- 8-element vector types --

// Storage traits: bytes per element and 32-bit words per 8-element vector.
template <int F> struct Fmt;
template <> struct Fmt<SRS_FMT_F32> { static constexpr int kBytes = 4; };
template <> struct Fmt<SRS_FMT_BF16> { static constexpr int kBytes = 2; };
template <> struct Fmt<SRS_FMT_F16> { static constexpr int kBytes = 2; };
template <> struct Fmt<SRS_FMT_E4M3> { static constexpr int kBytes = 1; };
template <> struct Fmt<SRS_FMT_E5M2> { static constexpr int kBytes = 1; };

template <int F> constexpr int kWords = kVec * Fmt<F>::kBytes / 4;

// Element offsets (e0) are int64_t or uint32_t: a uint32_t offset, zero-extended,
// lets the address be one wide multiply-add (the staged loops use it).
template <int F, typename I>
__device__ __forceinline__ const char* elem_ptr(const void* base, I e0) {
  return static_cast<const char*>(base) + static_cast<size_t>(e0) * Fmt<F>::kBytes;
}

// Raw 8-element load (16-byte aligned for 2- and 4-byte formats, 8-byte for FP8).
template <int F, typename I>
__device__ __forceinline__ void load_raw8(const void* base, I e0, uint32_t (&w)[kWords<F>]) {
  const char* p = elem_ptr<F>(base, e0);
  if constexpr (kWords<F> == 8) {
    const uint4 a = __ldcs(reinterpret_cast<const uint4*>(p));
    const uint4 b = __ldcs(reinterpret_cast<const uint4*>(p) + 1);
    w[0] = a.x; w[1] = a.y; w[2] = a.z; w[3] = a.w;
    w[4] = b.x; w[5] = b.y; w[6] = b.z; w[7] = b.w;
  } else if constexpr (kWords<F> == 4) {
    const uint4 a = __ldcs(reinterpret_cast<const uint4*>(p));
    w[0] = a.x; w[1] = a.y; w[2] = a.z; w[3] = a.w;
  } else {
    const uint2 a = __ldcs(reinterpret_cast<const uint2*>(p));
    w[0] = a.x; w[1] = a.y;
  }
}

template <int F, typename I>
__device__ __forceinline__ void store_raw8(void* base, I e0, const uint32_t (&w)[kWords<F>]) {
  char* p = const_cast<char*>(elem_ptr<F>(base, e0));
  if constexpr (kWords<F> == 8) {
    __stcs(reinterpret_cast<uint4*>(p), make_uint4(w[0], w[1], w[2], w[3]));
    __stcs(reinterpret_cast<uint4*>(p) + 1, make_uint4(w[4], w[5], w[6], w[7]));
  } else if constexpr (kWords<F> == 4) {
    __stcs(reinterpret_cast<uint4*>(p), make_uint4(w[0], w[1], w[2], w[3]));
  } else {
    __stcs(reinterpret_cast<uint2*>(p), make_uint2(w[0], w[1]));
  }
}

// Element j of a packed vector.
template <int F>
__device__ __forceinline__ uint32_t raw_element(const uint32_t (&w)[kWords<F>], int j) {
  if constexpr (Fmt<F>::kBytes == 4) return w[j];
  else if constexpr (Fmt<F>::kBytes == 2) return (w[j >> 1] >> (16 * (j & 1))) & 0xFFFFu;
  else return (w[j >> 2] >> (8 * (j & 3))) & 0xFFu;
}

// Guarded scalar load of `count` (< 8 or unaligned) elements into packed words.
template <int F, typename I>
__device__ __forceinline__ void load_raw_partial(const void* base, I e0, int count,
                                                 uint32_t (&w)[kWords<F>]) {
#pragma unroll
  for (int i = 0; i < kWords<F>; ++i) w[i] = 0u;
#pragma unroll
  for (int j = 0; j < kVec; ++j) {
    if (j < count) {
      uint32_t v;
      if constexpr (Fmt<F>::kBytes == 4) v = static_cast<const uint32_t*>(base)[e0 + j];
      else if constexpr (Fmt<F>::kBytes == 2) v = static_cast<const uint16_t*>(base)[e0 + j];
      else v = static_cast<const uint8_t*>(base)[e0 + j];
      if constexpr (Fmt<F>::kBytes == 4) w[j] = v;
      else if constexpr (Fmt<F>::kBytes == 2) w[j >> 1] |= v << (16 * (j & 1));
      else w[j >> 2] |= v << (8 * (j & 3));
    }
  }
}

template <int F, typename I>
__device__ __forceinline__ void store_raw_partial(void* base, I e0, int count,
                                                  const uint32_t (&w)[kWords<F>]) {
#pragma unroll
  for (int j = 0; j < kVec; ++j) {
    if (j < count) {
      const uint32_t v = raw_element<F>(w, j);
      if constexpr (Fmt<F>::kBytes == 4) static_cast<uint32_t*>(base)[e0 + j] = v;
      else if constexpr (Fmt<F>::kBytes == 2) static_cast<uint16_t*>(base)[e0 + j] = (uint16_t)v;
      else static_cast<uint8_t*>(base)[e0 + j] = (uint8_t)v;
    }
  }
}

// Decode 8 stored elements to FP32 (exact for every format).
template <int F>
__device__ __forceinline__ void decode8(const uint32_t (&w)[kWords<F>], float (&x)[kVec]) {
  if constexpr (F == SRS_FMT_F32) {
#pragma unroll
    for (int j = 0; j < kVec; ++j) x[j] = __uint_as_float(w[j]);
  } else if constexpr (F == SRS_FMT_BF16 || F == SRS_FMT_F16) {
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float2 f = (F == SRS_FMT_BF16) ? bf16x2_to_float2(w[i]) : f16x2_to_float2(w[i]);
      x[2 * i] = f.x;
      x[2 * i + 1] = f.y;
    }
  } else {
#pragma unroll
    for (int i = 0; i < 2; ++i) {
#pragma unroll
      for (int k = 0; k < 2; ++k) {
        const uint32_t pair = (w[i] >> (16 * k)) & 0xFFFFu;
        const float2 f = (F == SRS_FMT_E4M3) ? e4m3x2_to_float2(pair) : e5m2x2_to_float2(pair);
        x[4 * i + 2 * k] = f.x;
        x[4 * i + 2 * k + 1] = f.y;
      }
    }
  }
}

// Stochastic rounding of 8 values, one element at a time (any input).
template <int F>
__device__ __forceinline__ void encode8_stochastic_exact(const float (&x)[kVec], uint32_t ctr0,
                                                      uint32_t (&w)[kWords<F>]) {
  if constexpr (F == SRS_FMT_BF16 || F == SRS_FMT_F16) {
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const uint32_t h0 = h32(ctr0 + 2 * i), h1 = h32(ctr0 + 2 * i + 1);
      uint32_t lo, hi;
      if constexpr (F == SRS_FMT_BF16) {
        lo = bf16_stochastic(x[2 * i], h0);
        hi = bf16_stochastic(x[2 * i + 1], h1);
      } else {
        lo = f16_stochastic(x[2 * i], h0);
        hi = f16_stochastic(x[2 * i + 1], h1);
      }
      w[i] = lo | (hi << 16);
    }
  } else {
#pragma unroll
    for (int i = 0; i < 2; ++i) {
      uint32_t word = 0u;
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        const uint32_t h = h32(ctr0 + 4 * i + k);
        const uint32_t b = (F == SRS_FMT_E4M3) ? e4m3_stochastic(x[4 * i + k], h)
                                               : e5m2_stochastic(x[4 * i + k], h);
        word |= b << (8 * k);
      }
      w[i] = word;
    }
  }
}

// h32 of counter c + j, one of a vector's 8 consecutive counters, before its
// last xor-shift: h32(c + j) == u ^ (u >> 16) for the returned u.  SHARED: the
// 8 counters do not carry across bit 16, so (c + j) >> 16 == hi for all of
// them and the first xor-shift of h32 reuses that one shift.
template <bool SHARED>
__device__ __forceinline__ uint32_t h32_unmixed_at(uint32_t c, uint32_t j, uint32_t hi) {
  uint32_t x = c + j;
  x ^= SHARED ? hi : (x >> 16);
  x *= 0x7FEB352Du;
  x ^= x >> 15;
  return x * 0x846CA68Bu;
}

template <bool SHARED>
__device__ __forceinline__ uint32_t h32_at(uint32_t c, uint32_t j, uint32_t hi) {
  const uint32_t u = h32_unmixed_at<SHARED>(c, j, hi);
  return u ^ (u >> 16);
}

// The random bits of two BF16 stochastic roundings in the layout of
// cvt_rs_bf16x2: the low 16 bits of h32 are lo16(u) ^ hi16(u), so one byte
// permutation gathers both elements' low halves, another their high halves,
// and one xor mixes them (element `lo` in bits 0-15, element `hi` in 16-31).
__device__ __forceinline__ uint32_t bf16x2_random_bits(uint32_t u_lo, uint32_t u_hi) {
  return __byte_perm(u_lo, u_hi, 0x5410u) ^ __byte_perm(u_lo, u_hi, 0x7632u);
}

// sm_100a's stochastic conversion of two FP32 values to BF16: `hi` is rounded
// with rbits[31:16] into the upper half, `lo` with rbits[15:0] into the lower
// half, each as (FP32 encoding + its 16 random bits) >> 16 -- the rule of
// bf16_stochastic for every input but NaN (no flush of subnormals, overflow
// carries into infinity, infinities stay).  Checked on B200 against that rule
// for every FP32 encoding (the screened-rounding self-test) and on random
// pairs over the whole FP32 range.
__device__ __forceinline__ uint32_t cvt_rs_bf16x2(float hi, float lo, uint32_t rbits) {
  uint32_t d;
  asm("cvt.rs.bf16x2.f32 %0, %1, %2, %3;" : "=r"(d) : "f"(hi), "f"(lo), "r"(rbits));
  return d;
}

template <int F, bool SHARED>
__device__ __forceinline__ void encode8_stochastic_fast_as(const float (&x)[kVec], uint32_t ctr0,
                                                           uint32_t hi,
                                                           uint32_t (&w)[kWords<F>]) {
  if constexpr (F == SRS_FMT_BF16) {
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const uint32_t rbits = bf16x2_random_bits(h32_unmixed_at<SHARED>(ctr0, 2 * i, hi),
                                                h32_unmixed_at<SHARED>(ctr0, 2 * i + 1, hi));
      w[i] = cvt_rs_bf16x2(x[2 * i + 1], x[2 * i], rbits);
    }
  } else if constexpr (F == SRS_FMT_F16) {
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float2 y = grid_stochastic2<F>(make_float2(x[2 * i], x[2 * i + 1]),
                                           h32_at<SHARED>(ctr0, 2 * i, hi),
                                           h32_at<SHARED>(ctr0, 2 * i + 1, hi));
      const __half2 hh = __float22half2_rn(y);
      w[i] = *reinterpret_cast<const uint32_t*>(&hh);
    }
  } else {
    constexpr __nv_fp8_interpretation_t kind = (F == SRS_FMT_E4M3) ? __NV_E4M3 : __NV_E5M2;
#pragma unroll
    for (int i = 0; i < 2; ++i) {
      const float2 y0 = grid_stochastic2<F>(make_float2(x[4 * i], x[4 * i + 1]),
                                            h32_at<SHARED>(ctr0, 4 * i, hi),
                                            h32_at<SHARED>(ctr0, 4 * i + 1, hi));
      const float2 y1 = grid_stochastic2<F>(make_float2(x[4 * i + 2], x[4 * i + 3]),
                                            h32_at<SHARED>(ctr0, 4 * i + 2, hi),
                                            h32_at<SHARED>(ctr0, 4 * i + 3, hi));
      const uint32_t lo = __nv_cvt_float2_to_fp8x2(y0, __NV_SATFINITE, kind);
      const uint32_t up = __nv_cvt_float2_to_fp8x2(y1, __NV_SATFINITE, kind);
      w[i] = __byte_perm(lo, up, 0x5410u);
    }
  }
}

// Stochastic rounding of 8 screened values (see the fast forms above).
template <int F>
__device__ __forceinline__ void encode8_stochastic_fast(const float (&x)[kVec], uint32_t ctr0,
                                                        uint32_t (&w)[kWords<F>]) {
  if ((ctr0 & 0xFFFFu) <= 0xFFF8u) encode8_stochastic_fast_as<F, true>(x, ctr0, ctr0 >> 16, w);
  else encode8_stochastic_fast_as<F, false>(x, ctr0, 0u, w);
}

// Round toward zero, 8 values, one element at a time.
template <int F>
__device__ __forceinline__ void encode8_toward_zero(const float (&x)[kVec],
                                                 uint32_t (&w)[kWords<F>]) {
  constexpr int kPerWord = kVec / kWords<F>;  // 2 (16-bit) or 4 (8-bit) per word
#pragma unroll
  for (int i = 0; i < kWords<F>; ++i) {
    uint32_t word = 0u;
#pragma unroll
    for (int k = 0; k < kPerWord; ++k)
      word |= toward_zero1<F>(x[kPerWord * i + k]) << ((32 / kPerWord) * k);
    w[i] = word;
  }
}

// Round 8 FP32 values into storage format F by `rule` (SRS_RULE_*).  Element j
// of the stochastic rule uses the hash of counter `ctr0 + j` (mod 2^32).  FP32
// storage is the identity under every rule.
template <int F>
__device__ __forceinline__ void encode8(const float (&x)[kVec], uint32_t ctr0, int rule,
                                        uint32_t (&w)[kWords<F>]) {
  if constexpr (F == SRS_FMT_F32) {
#pragma unroll
    for (int j = 0; j < kVec; ++j) w[j] = __float_as_uint(x[j]);
  } else if (rule == SRS_RULE_STOCHASTIC) {
    const bool fast = (F == SRS_FMT_BF16) ? screen_bf16(x) : screen_grid(x);
    if (fast) encode8_stochastic_fast<F>(x, ctr0, w);
    else encode8_stochastic_exact<F>(x, ctr0, w);
  } else if (rule == SRS_RULE_TOWARD_ZERO) {
    encode8_toward_zero<F>(x, w);
  } else if constexpr (F == SRS_FMT_BF16 || F == SRS_FMT_F16) {
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float2 f = make_float2(x[2 * i], x[2 * i + 1]);
      if constexpr (F == SRS_FMT_BF16) {
        const __nv_bfloat162 b = __float22bfloat162_rn(f);
        w[i] = *reinterpret_cast<const uint32_t*>(&b);
      } else {
        const __half2 hh = __float22half2_rn(f);
        w[i] = *reinterpret_cast<const uint32_t*>(&hh);
      }
    }
  } else {
    // Saturating round-to-nearest-even conversion; equal to the reference's
    // clamp-then-grid rounding (verified exhaustively against the CPU oracle).
    constexpr __nv_fp8_interpretation_t kind = (F == SRS_FMT_E4M3) ? __NV_E4M3 : __NV_E5M2;
#pragma unroll
    for (int i = 0; i < 2; ++i) {
      const uint32_t lo =
          __nv_cvt_float2_to_fp8x2(make_float2(x[4 * i], x[4 * i + 1]), __NV_SATFINITE, kind);
      const uint32_t hi =
          __nv_cvt_float2_to_fp8x2(make_float2(x[4 * i + 2], x[4 * i + 3]), __NV_SATFINITE, kind);
      w[i] = (lo & 0xFFFFu) | (hi << 16);
    }
  }
}

// ------------------------------------------------------ parameter dtypes --

// Parameters and gradients are FP32 (P_BF16 == false) or BF16.
template <bool BF16, typename I>
__device__ __forceinline__ void load_param8(const void* base, I e0, int count, bool vec,
                                            float (&x)[kVec]) {
  if constexpr (BF16) {
    uint32_t w[4];
    if (vec) load_raw8<SRS_FMT_BF16>(base, e0, w);
    else load_raw_partial<SRS_FMT_BF16>(base, e0, count, w);
    decode8<SRS_FMT_BF16>(w, x);
  } else {
    uint32_t w[8];
    if (vec) load_raw8<SRS_FMT_F32>(base, e0, w);
    else load_raw_partial<SRS_FMT_F32>(base, e0, count, w);
    decode8<SRS_FMT_F32>(w, x);
  }
}

// One 8-element vector written through an NVLink multicast address: every
// replica bound to the multicast object receives it (16-byte multimem stores;
// two for FP32).  The address must be 16-byte aligned.
template <int F>
__device__ __forceinline__ void multimem_store8(char* mc, const uint32_t (&w)[kWords<F>]) {
#pragma unroll
  for (int i = 0; i < kWords<F>; i += 4)
    asm volatile("multimem.st.relaxed.sys.global.v4.f32 [%0], {%1, %2, %3, %4};"
                 ::"l"(mc + 4 * i), "f"(__uint_as_float(w[i])), "f"(__uint_as_float(w[i + 1])),
                   "f"(__uint_as_float(w[i + 2])), "f"(__uint_as_float(w[i + 3]))
                 : "memory");
}

// Parameter write-back: FP32 as is, BF16 round-to-nearest-even.  With peers,
// the same bytes also reach the same offset of every peer's replica (the fused
// all-gather of a sharded step): plain stores through the peer mappings, or,
// in multicast mode, one multimem store per aligned vector that NVSwitch
// delivers to every replica, this one included (element-wise tails use the
// plain stores, multimem having no 2-byte form).
template <bool BF16, typename I>
__device__ __forceinline__ void store_param8(void* base, I e0, int count, bool vec,
                                             const float (&x)[kVec],
                                             const srs_peers* peers = nullptr) {
  constexpr int F = BF16 ? SRS_FMT_BF16 : SRS_FMT_F32;
  uint32_t w[kWords<F>];
  encode8<F>(x, 0u, SRS_RULE_NEAREST, w);
  if (vec && peers != nullptr && peers->mode == SRS_PEERS_MULTICAST) {
    multimem_store8<F>(const_cast<char*>(elem_ptr<F>(base, e0)) +
                           (BF16 ? peers->mc_delta_bf16 : peers->mc_delta_f32),
                       w);
    return;
  }
  if (vec) store_raw8<F>(base, e0, w);
  else store_raw_partial<F>(base, e0, count, w);
  if (peers != nullptr) {
    for (int i = 0; i < peers->n_peers; ++i) {
      void* replica =
          static_cast<char*>(base) + (BF16 ? peers->delta_bf16[i] : peers->delta_f32[i]);
      if (vec) store_raw8<F>(replica, e0, w);
      else store_raw_partial<F>(replica, e0, count, w);
    }
  }
}

template <int F, typename I>
__device__ __forceinline__ void load_state8(const void* base, I e0, int count, bool vec,
                                            float (&x)[kVec]) {
  uint32_t w[kWords<F>];
  if (vec) load_raw8<F>(base, e0, w);
  else load_raw_partial<F>(base, e0, count, w);
  decode8<F>(w, x);
}

template <int F, typename I>
__device__ __forceinline__ void store_state8(void* base, I e0, int count, bool vec,
                                             const float (&x)[kVec], uint32_t ctr0,
                                             int rule) {
  uint32_t w[kWords<F>];
  encode8<F>(x, ctr0, rule, w);
  if (vec) store_raw8<F>(base, e0, w);
  else store_raw_partial<F>(base, e0, count, w);
}

// store_state8 for values known to pass the screen of their format (no NaN;
// for the FP16/FP8 grids |x| < 2^63): the stochastic rule goes straight to the
// fast form.  Only the stochastic and nearest rules come here (toward-zero
// states take store_state8), which keeps the hot loops free of that code.
template <int F, typename I>
__device__ __forceinline__ void store_state8_screened(void* base, I e0, int count, bool vec,
                                                      const float (&x)[kVec], uint32_t ctr0,
                                                      bool stochastic) {
  uint32_t w[kWords<F>];
  if constexpr (F == SRS_FMT_F32) {
    encode8<F>(x, ctr0, SRS_RULE_NEAREST, w);
  } else {
    if (stochastic) encode8_stochastic_fast<F>(x, ctr0, w);
    else encode8<F>(x, ctr0, SRS_RULE_NEAREST, w);
  }
  if (vec) store_raw8<F>(base, e0, w);
  else store_raw_partial<F>(base, e0, count, w);
}

}  // namespace srs
