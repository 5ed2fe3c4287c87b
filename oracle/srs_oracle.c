/*
 * srs_oracle.c — TEST INFRASTRUCTURE ONLY.
 *
 * A plain-C, single-threaded restatement of the reference algorithms of the
 * hot path of sr_states (KristiTopollai/stochastic-rounding-pytorch).  It is
 * the checker of the sm_100a kernels: only tests/, __graft_entry__.smoke() and
 * the CPU legs of bench.py load it.  The product (libsrs_b200.so and the
 * sr_states package) never calls it.
 *
 * Each function follows the reference's own formulation (floating-point grid
 * arithmetic, as in the PyTorch code), not the integer formulation of the CUDA
 * kernels, so agreement between the two is an independent check.  It is
 * pinned against golden vectors produced by the reference itself
 * (tests/golden/make_golden.py).
 *
 * Build: oracle/build_oracle.py (gcc -O2 -ffp-contract=off: every FP32
 * operation is rounded on its own, FMAs appear only as explicit fmaf calls).
 */
#include <math.h>
#include <stdint.h>
#include <string.h>

#define FMT_F32 0
#define FMT_BF16 1
#define FMT_F16 2
#define FMT_E4M3 3
#define FMT_E5M2 4

static inline uint32_t f2u(float f) {
  uint32_t u;
  memcpy(&u, &f, 4);
  return u;
}
static inline float u2f(uint32_t u) {
  float f;
  memcpy(&f, &u, 4);
  return f;
}

/* sr_states/_hash.py:10-15 (_h32) and :31-50 (_u32_hash, mod 2^32). */
uint32_t srs_o_h32(uint32_t v) {
  v ^= v >> 16;
  v *= 0x7FEB352Du;
  v ^= v >> 15;
  v *= 0x846CA68Bu;
  return v ^ (v >> 16);
}

/* sr_states/_hash.py:18-23: low 64 bits of seed and step, 32 of the index. */
uint32_t srs_o_update_key(uint64_t seed, uint64_t step, uint32_t param_index) {
  uint32_t key = srs_o_h32((uint32_t)seed ^ 0x9E3779B9u);
  key = srs_o_h32(key ^ (uint32_t)(seed >> 32));
  key = srs_o_h32(key ^ (uint32_t)step);
  key = srs_o_h32(key ^ (uint32_t)(step >> 32));
  return srs_o_h32(key ^ param_index);
}

/* sr_states/_hash.py:26-28. */
uint32_t srs_o_state_key(uint32_t key, uint32_t index) { return srs_o_h32(key ^ index); }

void srs_o_hash(const uint32_t* counters, uint32_t* out, int64_t n) {
  for (int64_t i = 0; i < n; ++i) out[i] = srs_o_h32(counters[i]);
}

/* ------------------------------------------------------------- formats -- */

/* sr_states/_minifloat.py:10-14: mantissa bits, emin, max finite, saturate. */
typedef struct {
  int mant, emin, bias, width;
  float max;
  int saturate;
} minifmt;

static const minifmt kE4M3 = {3, -6, 7, 8, 448.0f, 1};
static const minifmt kE5M2 = {2, -14, 15, 8, 57344.0f, 1};
static const minifmt kF16 = {10, -14, 15, 16, 65504.0f, 0};

static const minifmt* minifmt_of(int fmt) {
  return fmt == FMT_E4M3 ? &kE4M3 : (fmt == FMT_E5M2 ? &kE5M2 : &kF16);
}

/* Encoding of a value that is exactly representable in the format (or, for
 * FP16, at least 2^16 in magnitude, which is infinity).  NaN encodings are the
 * ones PyTorch's CPU conversions produce: FP8 sign|0x7F, FP16 F16C style. */
static uint32_t encode_exact(float r, const minifmt* f) {
  const uint32_t b = f2u(r);
  const uint32_t sign = (b >> 31) << (f->width - 1);
  const uint32_t u = b & 0x7FFFFFFFu;
  if (u > 0x7F800000u) {
    if (f->width == 8) return sign | 0x7Fu;
    return sign | 0x7E00u | ((u >> 13) & 0x3FFu);
  }
  const float a = fabsf(r);
  if (f->width == 16 && a >= 65536.0f) return sign | 0x7C00u;
  if (a == 0.0f) return sign;
  int e;
  frexpf(a, &e);
  e -= 1; /* a = m * 2^e, m in [1, 2) */
  if (e < f->emin) return sign | (uint32_t)ldexpf(a, f->mant - f->emin);
  const uint32_t frac = (uint32_t)ldexpf(a, f->mant - e) - (1u << f->mant);
  return sign | ((uint32_t)(e + f->bias) << f->mant) | frac;
}

static float decode_minifloat(uint32_t b, int fmt) {
  const minifmt* f = minifmt_of(fmt);
  const int ebits = f->width - 1 - f->mant;
  const uint32_t emax = (1u << ebits) - 1u;
  const uint32_t sign = (b >> (f->width - 1)) & 1u;
  const uint32_t e = (b >> f->mant) & emax;
  const uint32_t m = b & ((1u << f->mant) - 1u);
  float v;
  if (fmt == FMT_E4M3 && e == emax && m == ((1u << f->mant) - 1u)) return NAN; /* e4m3fn: no Inf */
  if (fmt != FMT_E4M3 && e == emax) v = m ? NAN : INFINITY;
  else if (e == 0) v = ldexpf((float)m, 1 - f->bias - f->mant);
  else v = ldexpf((float)(m | (1u << f->mant)), (int)e - f->bias - f->mant);
  return sign ? -v : v;
}

float srs_o_decode(uint32_t bits, int fmt) {
  switch (fmt) {
    case FMT_F32: return u2f(bits);
    case FMT_BF16: return u2f(bits << 16);
    default: return decode_minifloat(bits, fmt);
  }
}

/* sr_states/_minifloat.py:17-26 (_grid): a = q*ulp + remainder*ulp, exact. */
static void grid(float a, const minifmt* f, float* q, float* remainder, float* ulp) {
  int e = (int)((f2u(a) >> 23) & 0xFFu) - 127;
  if (e < f->emin) e = f->emin;
  *ulp = u2f((uint32_t)(e - f->mant + 127) << 23);
  const float reciprocal = u2f((uint32_t)(127 - e + f->mant) << 23);
  const float scaled = a * reciprocal;
  *q = floorf(scaled);
  *remainder = scaled - *q;
}

/* sr_states/_minifloat.py:29-42 (nearest_minifloat); FP16 uses the grid with
 * ties to even and IEEE overflow, which is what x.to(torch.float16) does. */
static uint32_t nearest_minifloat(float x, const minifmt* f) {
  float a = fabsf(x);
  if (f->saturate && a > f->max) a = f->max;
  if (isinf(a)) return encode_exact(x, f); /* FP16 only: Inf stays Inf */
  const float safe = isnan(x) ? 0.0f : a;
  float q, rem, ulp;
  grid(safe, f, &q, &rem, &ulp);
  const int up = (rem > 0.5f) || (rem == 0.5f && (((int32_t)q) & 1));
  float r = (q + (float)up) * ulp;
  r = copysignf(r, x);
  if (isnan(x)) r = x;
  return encode_exact(r, f);
}

/* sr_states/_minifloat.py:45-70 (stochastic_minifloat). */
static uint32_t stochastic_minifloat(float x, const minifmt* f, uint32_t counter) {
  float a = fabsf(x);
  if (f->saturate) a = isnan(a) ? a : fminf(a, f->max);
  const float safe = isfinite(a) ? a : 0.0f;
  float q, rem, ulp;
  grid(safe, f, &q, &rem, &ulp);
  const uint32_t k = srs_o_h32(counter) >> 8;
  const float threshold = floorf(rem * 16777216.0f);
  float r = (q + (((float)k < threshold) ? 1.0f : 0.0f)) * ulp;
  r = copysignf(r, x);
  if (!f->saturate && isinf(x)) r = x;
  if (isnan(x)) r = x;
  return encode_exact(r, f);
}

/* x.to(torch.bfloat16) on the CPU: round to nearest even; every NaN -> 0xFFFF. */
static uint32_t bf16_nearest(float x) {
  const uint32_t u = f2u(x);
  if (isnan(x)) return 0xFFFFu;
  return (u + 0x7FFFu + ((u >> 16) & 1u)) >> 16;
}

/* sr_states/_bf16.py:37-74, then the CPU BF16 conversion (NaN -> 0xFFFF). */
static uint32_t bf16_stochastic(float x, uint32_t counter) {
  const uint32_t bits = f2u(x);
  const uint32_t random_low = srs_o_h32(counter) & 0xFFFFu;
  const uint32_t truncated = bits & 0xFFFF0000u;
  uint32_t rounded = (bits + random_low) & 0xFFFF0000u;
  const int special = (bits & 0x7F800000u) == 0x7F800000u;
  const int nan = special && (bits & 0x007FFFFFu) != 0u;
  if (special) rounded = nan ? (truncated | 0x00400000u) : truncated;
  if (nan) return 0xFFFFu;
  return rounded >> 16;
}

/* Round toward zero: the format's value of largest magnitude not above |x|,
 * sign kept.  Not a reference built-in; it is what a custom rule runs when it
 * is registered with native="toward_zero".  The reference's own tests register
 * a rule of that name for BF16 (tests/test_rounding_registry.py:15-17: clear
 * the low 16 bits of the FP32 encoding, then convert), which this rule equals
 * on every input except NaNs whose payload lies only in those 16 bits (the
 * test's rule turns them into +-Inf; here every NaN is stored as the other
 * BF16 rules store it).  FP16 keeps IEEE round-toward-zero overflow (finite
 * values end at 65504, +-Inf stays infinite); FP8 saturates like the other
 * FP8 rules (sr_states/_minifloat.py:45-70). */
static uint32_t bf16_toward_zero(float x) {
  if (isnan(x)) return 0xFFFFu;
  return f2u(x) >> 16;
}

static uint32_t toward_zero_minifloat(float x, const minifmt* f) {
  if (isnan(x)) return encode_exact(x, f);
  float a = fabsf(x);
  if (isinf(a) && !f->saturate) return encode_exact(x, f);
  if (a > f->max) a = f->max;
  float q, rem, ulp;
  grid(a, f, &q, &rem, &ulp);
  return encode_exact(copysignf(q * ulp, x), f);
}

/* One FP32 value rounded into storage `fmt` by `rule` (0 nearest, 1
 * stochastic, 2 toward zero) with hash counter `counter`; returns the stored
 * bits.  FP32 rules are the identity (sr_states/rounding.py:127-136). */
uint32_t srs_o_round(float x, int fmt, int rule, uint32_t counter) {
  switch (fmt) {
    case FMT_F32: return f2u(x);
    case FMT_BF16:
      if (rule == 2) return bf16_toward_zero(x);
      return rule ? bf16_stochastic(x, counter) : bf16_nearest(x);
    default: {
      const minifmt* f = minifmt_of(fmt);
      if (rule == 2) return toward_zero_minifloat(x, f);
      return rule ? stochastic_minifloat(x, f, counter) : nearest_minifloat(x, f);
    }
  }
}

static int fmt_bytes(int fmt) { return fmt == FMT_F32 ? 4 : (fmt <= FMT_F16 ? 2 : 1); }

static uint32_t load_bits(const void* base, int64_t i, int fmt) {
  switch (fmt_bytes(fmt)) {
    case 4: return ((const uint32_t*)base)[i];
    case 2: return ((const uint16_t*)base)[i];
    default: return ((const uint8_t*)base)[i];
  }
}

static void store_bits(void* base, int64_t i, int fmt, uint32_t v) {
  switch (fmt_bytes(fmt)) {
    case 4: ((uint32_t*)base)[i] = v; break;
    case 2: ((uint16_t*)base)[i] = (uint16_t)v; break;
    default: ((uint8_t*)base)[i] = (uint8_t)v; break;
  }
}

/* sr_states/rounding.py:97-124 with the counter of sr_states/triton/cast.py:25-27:
 * element i uses h32((i + offset + seed) mod 2^32). */
void srs_o_cast(const float* x, void* y, int64_t n, int fmt, int rule, uint32_t seed,
                uint32_t offset) {
  for (int64_t i = 0; i < n; ++i)
    store_bits(y, i, fmt, srs_o_round(x[i], fmt, rule, (uint32_t)i + offset + seed));
}

/* The same cast over the FP32 encodings first_bits + i (exhaustive sweeps). */
void srs_o_cast_bits_range(uint32_t first_bits, int64_t n, void* y, int fmt, int rule,
                           uint32_t seed, uint32_t offset) {
  for (int64_t i = 0; i < n; ++i)
    store_bits(y, i, fmt,
               srs_o_round(u2f(first_bits + (uint32_t)i), fmt, rule, (uint32_t)i + offset + seed));
}

/* Parameter write-back: updated_parameter.to(parameter.dtype). */
static float load_param(const void* base, int64_t i, int bf16) {
  return bf16 ? u2f((uint32_t)((const uint16_t*)base)[i] << 16) : ((const float*)base)[i];
}
static void store_param(void* base, int64_t i, int bf16, float v) {
  if (bf16) ((uint16_t*)base)[i] = (uint16_t)bf16_nearest(v);
  else ((float*)base)[i] = v;
}

/*
 * In-place AdamW on n elements: sr_states/reference/adamw.py:54-105 (op order
 * :79-89, probed on PyTorch's CPU kernels: add(alpha) and addcmul are fused
 * multiply-adds, addcdiv computes (value*t1)/t2) and the state casts with
 * seeds state_key(update_key, 0/1) at `offset` (:91-104).
 * hp = {lr, beta1, beta2, eps, weight_decay}; scalars are rounded from double
 * exactly as PyTorch rounds Python floats.  sqrtf is correctly rounded, while
 * PyTorch's CPU sqrt is not (about 0.7% of inputs differ by one ulp), so the
 * parameter can differ from the reference by one ulp; states cannot.
 */
void srs_o_adamw_scalars(const double* hp, int64_t step, float* s) {
  const double lr = hp[0], beta1 = hp[1], beta2 = hp[2], eps = hp[3], wd = hp[4];
  const double bc1 = 1.0 - pow(beta1, (double)step);
  const double bc2 = 1.0 - pow(beta2, (double)step);
  s[0] = (float)beta1;
  s[1] = (float)beta2;
  s[2] = (float)(1.0 - beta1);
  s[3] = (float)(1.0 - beta2);
  s[4] = (float)eps;
  s[5] = (float)(1.0 - lr * wd);
  s[6] = (float)(-lr / bc1);   /* neg_step_size */
  s[7] = (float)pow(bc2, 0.5); /* bias2_sqrt */
}

/* The same update given the eight FP32 scalars of srs_o_adamw_scalars. */
void srs_o_adamw_core(void* p, int p_bf16, const void* g, int g_bf16, void* m, int m_fmt,
                      int m_rule, void* v, int v_fmt, int v_rule, int64_t n, const float* s,
                      uint32_t update_key, uint32_t offset) {
  const float b1 = s[0], b2 = s[1], omb1 = s[2], omb2 = s[3], epsf = s[4], decay = s[5];
  const float nss = s[6], bc2s = s[7];
  const uint32_t sk0 = srs_o_state_key(update_key, 0), sk1 = srs_o_state_key(update_key, 1);
  for (int64_t i = 0; i < n; ++i) {
    const float p32 = load_param(p, i, p_bf16);
    const float g32 = load_param(g, i, g_bf16);
    const float m32 = srs_o_decode(load_bits(m, i, m_fmt), m_fmt);
    const float v32 = srs_o_decode(load_bits(v, i, v_fmt), v_fmt);
    const float m1 = fmaf(g32, omb1, m32 * b1);
    const float v1 = fmaf(omb2 * g32, g32, v32 * b2);
    const float den = sqrtf(v1) / bc2s + epsf;
    const float p1 = p32 * decay + (nss * m1) / den;
    store_param(p, i, p_bf16, p1);
    const uint32_t ctr = (uint32_t)i + offset;
    store_bits(m, i, m_fmt, srs_o_round(m1, m_fmt, m_rule, ctr + sk0));
    store_bits(v, i, v_fmt, srs_o_round(v1, v_fmt, v_rule, ctr + sk1));
  }
}

void srs_o_adamw(void* p, int p_bf16, const void* g, int g_bf16, void* m, int m_fmt, int m_rule,
                 void* v, int v_fmt, int v_rule, int64_t n, const double* hp, int64_t step,
                 uint32_t update_key, uint32_t offset) {
  float s[8];
  srs_o_adamw_scalars(hp, step, s);
  srs_o_adamw_core(p, p_bf16, g, g_bf16, m, m_fmt, m_rule, v, v_fmt, v_rule, n, s, update_key,
                   offset);
}

/*
 * In-place momentum SGD: sr_states/reference/sgd.py:44-72 (op order :62-64:
 * u' = u*momentum + g, p' = fma(u', -lr, p)); state seed state_key(key, 0).
 */
void srs_o_sgdm_core(void* p, int p_bf16, const void* g, int g_bf16, void* u, int u_fmt,
                     int u_rule, int64_t n, float mf, float nlr, uint32_t update_key,
                     uint32_t offset) {
  const uint32_t sk0 = srs_o_state_key(update_key, 0);
  for (int64_t i = 0; i < n; ++i) {
    const float p32 = load_param(p, i, p_bf16);
    const float g32 = load_param(g, i, g_bf16);
    const float u32 = srs_o_decode(load_bits(u, i, u_fmt), u_fmt);
    const float u1 = u32 * mf + g32;
    const float p1 = fmaf(u1, nlr, p32);
    store_param(p, i, p_bf16, p1);
    store_bits(u, i, u_fmt, srs_o_round(u1, u_fmt, u_rule, (uint32_t)i + offset + sk0));
  }
}

void srs_o_sgdm(void* p, int p_bf16, const void* g, int g_bf16, void* u, int u_fmt, int u_rule,
                int64_t n, double lr, double momentum, uint32_t update_key, uint32_t offset) {
  srs_o_sgdm_core(p, p_bf16, g, g_bf16, u, u_fmt, u_rule, n, (float)momentum, (float)(-lr),
                  update_key, offset);
}

/* Check of the sm_100a kernels' division by a launch-uniform c (Markstein's
 * correction with y = RN(1/c)): over numerators with encodings
 * first, first+stride, ... < last, and inside the kernel's guard
 * lo <= bits(s) < hi, count quotients that differ from the IEEE division s/c. */
uint64_t srs_o_check_uniform_division(float c, float y, uint32_t first, uint32_t last,
                                      uint32_t stride, uint32_t lo, uint32_t hi,
                                      uint64_t* checked) {
  uint64_t bad = 0, n = 0;
  for (uint64_t u = first; u < last; u += stride) {
    if ((uint32_t)u - lo >= hi - lo) continue;
    const float s = u2f((uint32_t)u);
    const float q0 = s * y;
    const float r = fmaf(-c, q0, s);
    const float q1 = fmaf(r, y, q0);
    ++n;
    if (f2u(q1) != f2u(s / c)) ++bad;
  }
  *checked = n;
  return bad;
}
