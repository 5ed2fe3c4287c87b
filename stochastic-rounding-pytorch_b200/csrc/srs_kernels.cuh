// Kernel templates: fused AdamW / momentum-SGD steps over a row table and the
// standalone cast.  Instantiated per storage format in the srs_*.cu units.
//
// Launch shape: a persistent grid (resident CTAs per SM x SM count) walks the
// tile space grid-stride; a tile is 256 threads x 8 consecutive elements of
// one row, loaded and stored as 16-byte vectors.  Each kernel is specialised
// for the parameter/gradient dtype pair the host reports for the launch
// (uniform_kind); rows of another pair, tails and unaligned rows go through
// one generic, out-of-line path.
//
// FP32 arithmetic uses sm_100's packed two-lane instructions (mul2_rn,
// fma2_rn, add2_rn: each lane rounded to nearest on its own, never
// contracted), so the operation order is exactly the reference's.
#pragma once

#include "srs_common.cuh"

namespace srs {

constexpr int kKindMixed = 4;  // template value for launches with mixed dtype pairs

struct AdamWArgs {
  srs_row inline_row;  // the single row of srs_adamw_single (rows == nullptr)
  srs_adamw_hparams hp;
  float inv_bias2_sqrt[SRS_MAX_STEP_CLASSES];  // RN(1 / bias2_sqrt[c]), exact
  // Numerators s with lo <= bits(s) < hi take the reciprocal division path; the
  // host sets lo == hi (empty) for a class whose bias2_sqrt is out of range.
  uint32_t fast_lo[SRS_MAX_STEP_CLASSES];
  uint32_t fast_hi[SRS_MAX_STEP_CLASSES];
  srs_rng rng;
  int32_t m_stochastic;
  int32_t v_stochastic;
};

struct SgdmArgs {
  srs_row inline_row;  // the single row of srs_sgdm_single (rows == nullptr)
  srs_sgdm_hparams hp;
  srs_rng rng;
  int32_t u_stochastic;
};

// A row as held (uniformly) by one CTA while it walks that row's tiles.
struct RowView {
  void* p;
  const void* g;
  void* s0;
  void* s1;
  int64_t numel;
  int64_t tile_begin;
  uint32_t flags;
  uint32_t ctr0;  // offset + state_key(key, 0): counter of element 0 of state 0
  uint32_t ctr1;  // offset + state_key(key, 1)
};

// Step-class scalars of the current row.
struct ClassScalars {
  float nss;         // -lr / bc1
  float c;           // sqrt(bc2)
  float inv_c;       // RN(1 / c)
  uint32_t fast_lo;  // see AdamWArgs::fast_lo
  uint32_t fast_span;
};

__device__ __forceinline__ int64_t ldg_i64(const int64_t* p) {
  return (int64_t)__ldg(reinterpret_cast<const long long*>(p));
}

// Largest r with rows[r].tile_begin <= tile (rows sorted by tile_begin, rows[0].tile_begin == 0).
__device__ __forceinline__ int64_t find_row(const srs_row* rows, int64_t n_rows, int64_t tile) {
  int64_t lo = 0, hi = n_rows - 1;
  while (lo < hi) {
    const int64_t mid = (lo + hi + 1) >> 1;
    if (ldg_i64(&rows[mid].tile_begin) <= tile) lo = mid;
    else hi = mid - 1;
  }
  return lo;
}

__device__ __forceinline__ srs_row load_row(const srs_row* row) {
  const ulonglong2* q = reinterpret_cast<const ulonglong2*>(row);
  const ulonglong2 a = __ldg(q), b = __ldg(q + 1), c = __ldg(q + 2), d = __ldg(q + 3);
  srs_row r;
  r.param = a.x;
  r.grad = a.y;
  r.state[0] = b.x;
  r.state[1] = b.y;
  r.numel = (int64_t)c.x;
  r.tile_begin = (int64_t)c.y;
  r.param_index = (uint32_t)d.x;
  r.offset = (uint32_t)(d.x >> 32);
  r.flags = (uint32_t)d.y;
  r.reserved = (uint32_t)(d.y >> 32);
  return r;
}

template <typename Args>
__device__ __forceinline__ RowView make_view(const srs_row& row, const Args& a) {
  const uint32_t key =
      (a.rng.key_mode == SRS_KEY_GIVEN) ? row.param_index : update_key(a.rng, row.param_index);
  RowView v;
  v.p = reinterpret_cast<void*>(row.param);
  v.g = reinterpret_cast<const void*>(row.grad);
  v.s0 = reinterpret_cast<void*>(row.state[0]);
  v.s1 = reinterpret_cast<void*>(row.state[1]);
  v.numel = row.numel;
  v.tile_begin = row.tile_begin;
  v.flags = row.flags;
  v.ctr0 = row.offset + state_key(key, 0u);
  v.ctr1 = row.offset + state_key(key, 1u);
  return v;
}

// Advance the CTA's row cursor to the row holding `tile`; true if it changed.
template <typename Args>
__device__ __forceinline__ bool seek_row(const srs_row* rows, int64_t n_rows, int64_t tile,
                                         int64_t& r, RowView& rv, const Args& a) {
  int64_t nr = 0;
  if (rows != nullptr) {
    if (r < 0) {
      nr = find_row(rows, n_rows, tile);
    } else {
      nr = r;
      while (nr + 1 < n_rows && ldg_i64(&rows[nr + 1].tile_begin) <= tile) ++nr;
    }
  }
  if (nr == r) return false;
  r = nr;
  rv = make_view(rows != nullptr ? load_row(rows + r) : a.inline_row, a);
  return true;
}

__device__ __forceinline__ float2 splat(float x) { return make_float2(x, x); }

// Correctly rounded s / c for a launch-uniform c with y = RN(1/c): Markstein's
// division step q0 = RN(s*y), r = s - c*q0 (exact through the FMA),
// q1 = RN(q0 + r*y) equals RN(s/c) when nothing underflows or overflows
// (P. Markstein, "Computation of elementary functions on the IBM RISC
// System/6000 processor", IBM J. Res. Dev. 34(1), 1990).  The host enables it
// for 2^-30 <= c <= 2^30 and numerators 2^-59 <= s < 2^60, where q0, r and q1
// stay far from the subnormal and overflow ranges.  Everything else (zero,
// tiny, huge, Inf, NaN numerators) takes the IEEE division.
__device__ __forceinline__ float2 div_by_uniform(float2 s, const ClassScalars& k) {
  const float2 q0 = mul2_rn(s, splat(k.inv_c));
  const float2 r = fma2_rn(splat(-k.c), q0, s);
  const float2 q1 = fma2_rn(r, splat(k.inv_c), q0);
  const uint32_t bx = __float_as_uint(s.x) - k.fast_lo;
  const uint32_t by = __float_as_uint(s.y) - k.fast_lo;
  if (max(bx, by) < k.fast_span) return q1;
  return make_float2(__fdiv_rn(s.x, k.c), __fdiv_rn(s.y, k.c));
}

// --------------------------------------------------------------- AdamW --

// One thread, 8 consecutive elements [e0, e0+count) of a row.  FP32 math in the
// reference CPU operation order (sr_states/reference/adamw.py:79-89): each
// operation rounded once, FMA exactly where PyTorch's CPU kernels use one.
// VEC: aligned 16-byte vector access of 8 elements; else guarded scalar access.
template <bool PB, bool GB, int MF, int VF, bool VEC>
__device__ __forceinline__ void adamw8(const RowView& rv, int64_t e0, int count,
                                       const ClassScalars& k, const AdamWArgs& a) {
  float p[kVec], g[kVec], m[kVec], v[kVec];
  load_param8<PB>(rv.p, e0, count, VEC, p);
  load_param8<GB>(rv.g, e0, count, VEC, g);
  load_state8<MF>(rv.s0, e0, count, VEC, m);
  load_state8<VF>(rv.s1, e0, count, VEC, v);
  const float2 b1 = splat(a.hp.beta1), b2 = splat(a.hp.beta2);
  const float2 omb1 = splat(a.hp.one_minus_beta1), omb2 = splat(a.hp.one_minus_beta2);
  const float2 eps = splat(a.hp.eps), decay = splat(a.hp.decay), nss = splat(k.nss);
#pragma unroll
  for (int i = 0; i < kVec / 2; ++i) {
    const float2 g2 = make_float2(g[2 * i], g[2 * i + 1]);
    const float2 m1 = fma2_rn(g2, omb1, mul2_rn(make_float2(m[2 * i], m[2 * i + 1]), b1));
    const float2 v1 = fma2_rn(mul2_rn(omb2, g2), g2,
                                 mul2_rn(make_float2(v[2 * i], v[2 * i + 1]), b2));
    const float2 root = make_float2(__fsqrt_rn(v1.x), __fsqrt_rn(v1.y));
    const float2 den = add2_rn(div_by_uniform(root, k), eps);
    const float2 num = mul2_rn(nss, m1);
    const float2 upd = make_float2(__fdiv_rn(num.x, den.x), __fdiv_rn(num.y, den.y));
    const float2 p1 = mul_add_rn2(make_float2(p[2 * i], p[2 * i + 1]), decay, upd);
    p[2 * i] = p1.x;
    p[2 * i + 1] = p1.y;
    m[2 * i] = m1.x;
    m[2 * i + 1] = m1.y;
    v[2 * i] = v1.x;
    v[2 * i + 1] = v1.y;
  }
  store_param8<PB>(rv.p, e0, count, VEC, p);
  store_state8<MF>(rv.s0, e0, count, VEC, m, (uint32_t)e0 + rv.ctr0, a.m_stochastic != 0);
  store_state8<VF>(rv.s1, e0, count, VEC, v, (uint32_t)e0 + rv.ctr1, a.v_stochastic != 0);
}

// Any dtype pair, vector or guarded access: tails, unaligned rows and rows
// whose pair differs from the launch's specialisation.  Out of line so the
// specialised loop stays small.
template <int MF, int VF>
__device__ __noinline__ void adamw8_generic(const RowView& rv, int64_t e0, int count, bool vec,
                                            const ClassScalars& k, const AdamWArgs& a) {
  switch ((rv.flags & 3u) | (vec ? 4u : 0u)) {
    case 0: adamw8<false, false, MF, VF, false>(rv, e0, count, k, a); break;
    case 1: adamw8<true, false, MF, VF, false>(rv, e0, count, k, a); break;
    case 2: adamw8<false, true, MF, VF, false>(rv, e0, count, k, a); break;
    case 3: adamw8<true, true, MF, VF, false>(rv, e0, count, k, a); break;
    case 4: adamw8<false, false, MF, VF, true>(rv, e0, count, k, a); break;
    case 5: adamw8<true, false, MF, VF, true>(rv, e0, count, k, a); break;
    case 6: adamw8<false, true, MF, VF, true>(rv, e0, count, k, a); break;
    default: adamw8<true, true, MF, VF, true>(rv, e0, count, k, a); break;
  }
}

#ifndef SRS_ADAMW_MIN_CTAS
#define SRS_ADAMW_MIN_CTAS 4  // resident CTAs per SM the register budget is sized for
#endif

template <int MF, int VF, int KIND>
__global__ void __launch_bounds__(kThreads, SRS_ADAMW_MIN_CTAS)
    adamw_kernel(const srs_row* __restrict__ rows, int64_t n_rows, int64_t n_tiles,
                 const __grid_constant__ AdamWArgs a) {
  int64_t r = -1;
  RowView rv{};
  ClassScalars k{0.f, 1.f, 1.f, 0u, 0u};
  for (int64_t tile = blockIdx.x; tile < n_tiles; tile += gridDim.x) {
    if (seek_row(rows, n_rows, tile, r, rv, a)) {
      const uint32_t cls = (rv.flags >> SRS_ROW_CLASS_SHIFT) & 0xFFu;
      k.nss = a.hp.neg_step_size[cls];
      k.c = a.hp.bias2_sqrt[cls];
      k.inv_c = a.inv_bias2_sqrt[cls];
      k.fast_lo = a.fast_lo[cls];
      k.fast_span = a.fast_hi[cls] - a.fast_lo[cls];
    }
    const int64_t e0 = (tile - rv.tile_begin) * kTile + (int64_t)threadIdx.x * kVec;
    if (e0 < rv.numel) {
      const int count = (int)min((int64_t)kVec, rv.numel - e0);
      const bool vec = (rv.flags & SRS_ROW_VECTOR_OK) != 0u && count == kVec;
      if constexpr (KIND != kKindMixed) {
        if (vec && (rv.flags & 3u) == (uint32_t)KIND) {
          adamw8<(KIND & 1) != 0, (KIND & 2) != 0, MF, VF, true>(rv, e0, count, k, a);
          continue;
        }
      }
      adamw8_generic<MF, VF>(rv, e0, count, vec, k, a);
    }
  }
}

// ----------------------------------------------------------------- SGDM --

// u' = u*mf + g (two roundings); p' = fma(u', -lr, p)  (sr_states/reference/sgd.py:62-64).
template <bool PB, bool GB, int UF, bool VEC>
__device__ __forceinline__ void sgdm8(const RowView& rv, int64_t e0, int count,
                                      const SgdmArgs& a) {
  float p[kVec], g[kVec], u[kVec];
  load_param8<PB>(rv.p, e0, count, VEC, p);
  load_param8<GB>(rv.g, e0, count, VEC, g);
  load_state8<UF>(rv.s0, e0, count, VEC, u);
  const float2 mf = splat(a.hp.momentum), nlr = splat(a.hp.neg_lr);
#pragma unroll
  for (int i = 0; i < kVec / 2; ++i) {
    const float2 u1 = mul_add_rn2(make_float2(u[2 * i], u[2 * i + 1]), mf,
                                  make_float2(g[2 * i], g[2 * i + 1]));
    const float2 p1 = fma2_rn(u1, nlr, make_float2(p[2 * i], p[2 * i + 1]));
    p[2 * i] = p1.x;
    p[2 * i + 1] = p1.y;
    u[2 * i] = u1.x;
    u[2 * i + 1] = u1.y;
  }
  store_param8<PB>(rv.p, e0, count, VEC, p);
  store_state8<UF>(rv.s0, e0, count, VEC, u, (uint32_t)e0 + rv.ctr0, a.u_stochastic != 0);
}

template <int UF>
__device__ __noinline__ void sgdm8_generic(const RowView& rv, int64_t e0, int count, bool vec,
                                           const SgdmArgs& a) {
  switch ((rv.flags & 3u) | (vec ? 4u : 0u)) {
    case 0: sgdm8<false, false, UF, false>(rv, e0, count, a); break;
    case 1: sgdm8<true, false, UF, false>(rv, e0, count, a); break;
    case 2: sgdm8<false, true, UF, false>(rv, e0, count, a); break;
    case 3: sgdm8<true, true, UF, false>(rv, e0, count, a); break;
    case 4: sgdm8<false, false, UF, true>(rv, e0, count, a); break;
    case 5: sgdm8<true, false, UF, true>(rv, e0, count, a); break;
    case 6: sgdm8<false, true, UF, true>(rv, e0, count, a); break;
    default: sgdm8<true, true, UF, true>(rv, e0, count, a); break;
  }
}

template <int UF, int KIND>
__global__ void __launch_bounds__(kThreads)
    sgdm_kernel(const srs_row* __restrict__ rows, int64_t n_rows, int64_t n_tiles,
                const __grid_constant__ SgdmArgs a) {
  int64_t r = -1;
  RowView rv{};
  for (int64_t tile = blockIdx.x; tile < n_tiles; tile += gridDim.x) {
    seek_row(rows, n_rows, tile, r, rv, a);
    const int64_t e0 = (tile - rv.tile_begin) * kTile + (int64_t)threadIdx.x * kVec;
    if (e0 < rv.numel) {
      const int count = (int)min((int64_t)kVec, rv.numel - e0);
      const bool vec = (rv.flags & SRS_ROW_VECTOR_OK) != 0u && count == kVec;
      if constexpr (KIND != kKindMixed) {
        if (vec && (rv.flags & 3u) == (uint32_t)KIND) {
          sgdm8<(KIND & 1) != 0, (KIND & 2) != 0, UF, true>(rv, e0, count, a);
          continue;
        }
      }
      sgdm8_generic<UF>(rv, e0, count, vec, a);
    }
  }
}

// ----------------------------------------------------------------- cast --

// y[e] = round(x[e]); stochastic counter (e + base) mod 2^32 with base = seed + offset.
template <int OF>
__global__ void __launch_bounds__(kThreads)
    cast_kernel(const float* __restrict__ x, void* __restrict__ y, int64_t n, uint32_t base,
                int stochastic, int vec_ok) {
  const int64_t stride = (int64_t)gridDim.x * kThreads * kVec;
  for (int64_t e0 = ((int64_t)blockIdx.x * kThreads + threadIdx.x) * kVec; e0 < n; e0 += stride) {
    const int count = (int)min((int64_t)kVec, n - e0);
    const bool vec = vec_ok != 0 && count == kVec;
    float v[kVec];
    load_state8<SRS_FMT_F32>(x, e0, count, vec, v);
    store_state8<OF>(y, e0, count, vec, v, base + (uint32_t)e0, stochastic != 0);
  }
}

// --------------------------------------------------------------- launch --

// Persistent grid: resident CTAs per SM (occupancy) x SM count, capped by the
// work.  Cached per device and kernel.
int grid_for(const void* kernel, int64_t work_ctas, int grid_ctas, cudaError_t* err);

// kind: 0..3 = the dtype pair shared by all rows, 4 = mixed.
template <int MF, int VF>
cudaError_t launch_adamw(const srs_row* rows, int64_t n_rows, int64_t n_tiles, int kind,
                         const AdamWArgs& a, int grid_ctas, cudaStream_t stream);

template <int UF>
cudaError_t launch_sgdm(const srs_row* rows, int64_t n_rows, int64_t n_tiles, int kind,
                        const SgdmArgs& a, int grid_ctas, cudaStream_t stream);

template <int OF>
cudaError_t launch_cast(const float* x, void* y, int64_t n, uint32_t base, int stochastic,
                        int vec_ok, int grid_ctas, cudaStream_t stream);

}  // namespace srs
