// Self-test kernels for the GPU test suite (built into libsrs_selftest.so, never
// loaded by the package).  They check device building blocks of the product
// kernels element by element against CUDA's correctly rounded scalar
// intrinsics, on inputs generated on the device from a counter hash.
#include "srs_kernels.cuh"

namespace {

__device__ __forceinline__ float random_float(uint32_t i, uint32_t seed, uint32_t salt) {
  return __uint_as_float(srs::h32(srs::h32(i ^ salt) + seed));
}

__device__ __forceinline__ bool same(float a, float b) {
  return __float_as_uint(a) == __float_as_uint(b) || (a != a && b != b);
}

// counts[0..2]: mul2, add2, fma2 vs the scalar _rn intrinsics; counts[3]:
// mul_add_rn2 (single-use product, as in the kernels) vs separate rounding;
// counts[4]: add2_rn(mul2_rn()) with a single-use product and counts[5]:
// __fadd2_rn(__fmul2_rn()) -- diagnostics of the packed fusion hazard.
__global__ void packed_math_kernel(uint64_t n, uint32_t seed, unsigned long long* counts) {
  unsigned long long local[6] = {0, 0, 0, 0, 0, 0};
  for (uint64_t i = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; i < n;
       i += (uint64_t)gridDim.x * blockDim.x) {
    const uint32_t k = (uint32_t)i;
    const float2 a = make_float2(random_float(k, seed, 1), random_float(k, seed, 2));
    const float2 b = make_float2(random_float(k, seed, 3), random_float(k, seed, 4));
    const float2 c = make_float2(random_float(k, seed, 5), random_float(k, seed, 6));
    const float2 m = srs::mul2_rn(a, b), s = srs::add2_rn(a, b), f = srs::fma2_rn(a, b, c);
    // Single-use products, distinct operands (c, a) so no product is shared.
    const float2 seq = srs::mul_add_rn2(c, b, a);
    const float2 packed_seq = srs::add2_rn(srs::mul2_rn(c, a), b);
    const float2 cuda_seq = __fadd2_rn(__fmul2_rn(b, c), a);
    local[0] += !same(m.x, __fmul_rn(a.x, b.x)) + !same(m.y, __fmul_rn(a.y, b.y));
    local[1] += !same(s.x, __fadd_rn(a.x, b.x)) + !same(s.y, __fadd_rn(a.y, b.y));
    local[2] += !same(f.x, __fmaf_rn(a.x, b.x, c.x)) + !same(f.y, __fmaf_rn(a.y, b.y, c.y));
    // Reference: the exact product (a double holds it), rounded to float, then one
    // rounded addition.
    const float sx = __fadd_rn(__double2float_rn((double)c.x * b.x), a.x);
    const float sy = __fadd_rn(__double2float_rn((double)c.y * b.y), a.y);
    local[3] += !same(seq.x, sx) + !same(seq.y, sy);
    local[4] += !same(packed_seq.x, __fadd_rn(__double2float_rn((double)c.x * a.x), b.x)) +
                !same(packed_seq.y, __fadd_rn(__double2float_rn((double)c.y * a.y), b.y));
    local[5] += !same(cuda_seq.x, __fadd_rn(__double2float_rn((double)b.x * c.x), a.x)) +
                !same(cuda_seq.y, __fadd_rn(__double2float_rn((double)b.y * c.y), a.y));
  }
  for (int j = 0; j < 6; ++j)
    if (local[j]) atomicAdd(&counts[j], local[j]);
}

// Fast (screened) stochastic rounding against the per-element rules, over every
// FP32 bit pattern: vector k holds the patterns 8k..8k+7 and uses the counter
// base h32(k ^ seed).  counts[0] = vectors that passed the screen and were
// compared, counts[1] = those whose encodings differ, counts[2] = screened out.
template <int F>
__global__ void sr_fast_kernel(uint32_t seed, unsigned long long* counts) {
  unsigned long long local[3] = {0, 0, 0};
  const uint64_t n_vectors = 1ull << 29;
  for (uint64_t k = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; k < n_vectors;
       k += (uint64_t)gridDim.x * blockDim.x) {
    float x[srs::kVec];
#pragma unroll
    for (int j = 0; j < srs::kVec; ++j) x[j] = __uint_as_float((uint32_t)(8 * k + j));
    const uint32_t ctr0 = srs::h32((uint32_t)k ^ seed);
    const bool pass = (F == SRS_FMT_BF16) ? srs::screen_bf16(x) : srs::screen_grid(x);
    if (!pass) {
      ++local[2];
      continue;
    }
    uint32_t fast[srs::kWords<F>], exact[srs::kWords<F>];
    srs::encode8_stochastic_fast<F>(x, ctr0, fast);
    srs::encode8_stochastic_exact<F>(x, ctr0, exact);
    bool differ = false;
#pragma unroll
    for (int i = 0; i < srs::kWords<F>; ++i) differ |= fast[i] != exact[i];
    ++local[0];
    local[1] += differ;
  }
  for (int j = 0; j < 3; ++j)
    if (local[j]) atomicAdd(&counts[j], local[j]);
}

// The facts the screened AdamW arithmetic rests on, for every FP32 input:
// counts[0] = inputs a >= 2^-102 whose corrected rsqrt square root differs
// from __fsqrt_rn; counts[1] = d in [2^-126, 2^126) whose refined negated
// reciprocal differs from -__frcp_rn(d).
__global__ void cr_facts_kernel(unsigned long long* counts) {
  unsigned long long bad_sqrt = 0, bad_rcp = 0;
  for (uint32_t b = 0x00800000u + blockIdx.x * blockDim.x + threadIdx.x; b < 0x7F800000u;
       b += gridDim.x * blockDim.x) {
    const float a = __uint_as_float(b);
    if (b >= 0x0C800000u) {  // 2^-102
      const float y = srs::rsqrt_approx(a);
      const float g = __fmul_rn(a, y), h = __fmul_rn(y, 0.5f);
      const float s = __fmaf_rn(__fmaf_rn(-g, g, a), h, g);
      bad_sqrt += !same(s, __fsqrt_rn(a));
    }
    if (b < 0x7E800000u) {  // 2^126
      const float ny0 = srs::rcp_approx(-a);
      const float ny1 = __fmaf_rn(__fmaf_rn(a, ny0, 1.0f), ny0, ny0);
      bad_rcp += !same(ny1, -__frcp_rn(a));
    }
  }
  if (bad_sqrt) atomicAdd(&counts[0], bad_sqrt);
  if (bad_rcp) atomicAdd(&counts[1], bad_rcp);
}

// Screened AdamW arithmetic (adamw_update_fast) against the per-element IEEE
// operations on random vectors whose exponents range from realistic to
// extreme: counts[0] = vectors that passed the screen, counts[1] = vectors
// whose parameters differ, counts[2] = vectors screened out.
__device__ __forceinline__ float random_scaled(uint32_t h, int lo, int span, bool sign) {
  const int e = lo + (int)((h >> 23) % (uint32_t)span);
  const float mant = __uint_as_float(0x3F800000u | (h & 0x7FFFFFu));
  const float x = ldexpf(mant, e);
  return sign && (h & 0x10000u) ? -x : x;
}

__global__ void adamw_fast_kernel(uint64_t n_vectors, uint32_t seed, srs::ClassScalars k,
                                  const __grid_constant__ srs::AdamWArgs a,
                                  unsigned long long* counts) {
  unsigned long long local[3] = {0, 0, 0};
  for (uint64_t vi = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; vi < n_vectors;
       vi += (uint64_t)gridDim.x * blockDim.x) {
    const uint32_t base = srs::h32((uint32_t)vi ^ seed);
    const bool extreme = (base & 3u) == 0u;
    float p[srs::kVec], m1[srs::kVec], v1[srs::kVec];
#pragma unroll
    for (int j = 0; j < srs::kVec; ++j) {
      const uint32_t h0 = srs::h32(base + 3u * j), h1 = srs::h32(base + 3u * j + 1u),
                     h2 = srs::h32(base + 3u * j + 2u);
      p[j] = random_scaled(h0, extreme ? -140 : -20, extreme ? 270 : 22, true);
      m1[j] = random_scaled(h1, extreme ? -110 : -30, extreme ? 180 : 32, true);
      v1[j] = random_scaled(h2, extreme ? -100 : -50, extreme ? 150 : 55, false);
    }
    float y[srs::kVec];
    if (!srs::adamw_screen(m1, v1, k.m_floor, y)) {
      ++local[2];
      continue;
    }
    float fast[srs::kVec];
#pragma unroll
    for (int j = 0; j < srs::kVec; ++j) fast[j] = p[j];
    srs::adamw_update_fast(fast, m1, v1, y, k, a);
    bool differ = false;
#pragma unroll
    for (int j = 0; j < srs::kVec; ++j) {
      const float root = __fsqrt_rn(v1[j]);
      const float den = __fadd_rn(__fdiv_rn(root, k.c), a.hp.eps);
      const float upd = __fdiv_rn(__fmul_rn(k.nss, m1[j]), den);
      const float want = __fadd_rn(__fmul_rn(p[j], a.hp.decay), upd);
      differ |= !same(fast[j], want);
    }
    ++local[0];
    local[1] += differ;
  }
  for (int j = 0; j < 3; ++j)
    if (local[j]) atomicAdd(&counts[j], local[j]);
}

}  // namespace

extern "C" int srs_selftest_cr_facts(unsigned long long* counts, void* stream) {
  cr_facts_kernel<<<1184, 256, 0, static_cast<cudaStream_t>(stream)>>>(counts);
  return cudaGetLastError() == cudaSuccess ? 0 : -3;
}

// One step class with scalars (c, nss, eps, decay); the host-side eligibility
// rules of the library are the caller's to respect (fast_math must hold).
extern "C" int srs_selftest_adamw_fast(uint64_t n_vectors, uint32_t seed, float c, float inv_c,
                                       float nss, float m_floor, float eps, float decay,
                                       unsigned long long* counts, void* stream) {
  srs::AdamWArgs a{};
  a.hp.eps = eps;
  a.hp.decay = decay;
  srs::ClassScalars k{};
  k.nss = nss;
  k.c = c;
  k.inv_c = inv_c;
  k.fast_math = true;
  k.m_floor = m_floor;
  adamw_fast_kernel<<<1184, 256, 0, static_cast<cudaStream_t>(stream)>>>(n_vectors, seed, k, a,
                                                                        counts);
  return cudaGetLastError() == cudaSuccess ? 0 : -3;
}

extern "C" int srs_selftest_sr_fast(int format, uint32_t seed, unsigned long long* counts,
                                    void* stream) {
  const cudaStream_t s = static_cast<cudaStream_t>(stream);
  switch (format) {
    case SRS_FMT_BF16: sr_fast_kernel<SRS_FMT_BF16><<<1184, 256, 0, s>>>(seed, counts); break;
    case SRS_FMT_F16: sr_fast_kernel<SRS_FMT_F16><<<1184, 256, 0, s>>>(seed, counts); break;
    case SRS_FMT_E4M3: sr_fast_kernel<SRS_FMT_E4M3><<<1184, 256, 0, s>>>(seed, counts); break;
    case SRS_FMT_E5M2: sr_fast_kernel<SRS_FMT_E5M2><<<1184, 256, 0, s>>>(seed, counts); break;
    default: return -1;
  }
  return cudaGetLastError() == cudaSuccess ? 0 : -3;
}

extern "C" int srs_selftest_packed_math(uint64_t n, uint32_t seed, unsigned long long* counts,
                                        void* stream) {
  packed_math_kernel<<<592, 256, 0, static_cast<cudaStream_t>(stream)>>>(n, seed, counts);
  return cudaGetLastError() == cudaSuccess ? 0 : -3;
}
