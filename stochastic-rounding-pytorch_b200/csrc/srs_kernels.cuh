// Kernel templates: fused AdamW / momentum-SGD steps over a row table, the
// standalone cast, and device key derivation.  Instantiated per storage
// format in the srs_*.cu translation units.
#pragma once

#include "srs_common.cuh"

namespace srs {

struct AdamWArgs {
  srs_row inline_row;  // the single row of srs_adamw_single (rows == nullptr)
  srs_adamw_hparams hp;
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

// ---------------------------------------------------------------- AdamW --

// One thread, 8 consecutive elements [e0, e0+count) of a row.  FP32 math in the
// reference CPU operation order (sr_states/reference/adamw.py:79-89): each
// operation rounded once, FMA exactly where PyTorch's CPU kernels use one.
template <bool PB, bool GB, int MF, int VF>
__device__ __forceinline__ void adamw8(const RowView& rv, int64_t e0, int count, bool vec,
                                       float nss, float bc2s, const AdamWArgs& a) {
  float p[kVec], g[kVec], m[kVec], v[kVec];
  load_param8<PB>(rv.p, e0, count, vec, p);
  load_param8<GB>(rv.g, e0, count, vec, g);
  load_state8<MF>(rv.s0, e0, count, vec, m);
  load_state8<VF>(rv.s1, e0, count, vec, v);
  const float b1 = a.hp.beta1, b2 = a.hp.beta2, omb1 = a.hp.one_minus_beta1,
              omb2 = a.hp.one_minus_beta2, eps = a.hp.eps, decay = a.hp.decay;
#pragma unroll
  for (int j = 0; j < kVec; ++j) {
    const float m1 = __fmaf_rn(g[j], omb1, __fmul_rn(m[j], b1));
    const float v1 = __fmaf_rn(__fmul_rn(omb2, g[j]), g[j], __fmul_rn(v[j], b2));
    const float den = __fadd_rn(__fdiv_rn(__fsqrt_rn(v1), bc2s), eps);
    p[j] = __fadd_rn(__fmul_rn(p[j], decay), __fdiv_rn(__fmul_rn(nss, m1), den));
    m[j] = m1;
    v[j] = v1;
  }
  store_param8<PB>(rv.p, e0, count, vec, p);
  store_state8<MF>(rv.s0, e0, count, vec, m, (uint32_t)e0 + rv.ctr0, a.m_stochastic != 0);
  store_state8<VF>(rv.s1, e0, count, vec, v, (uint32_t)e0 + rv.ctr1, a.v_stochastic != 0);
}

template <int MF, int VF>
__global__ void __launch_bounds__(kThreads)
    adamw_kernel(const srs_row* __restrict__ rows, int64_t n_rows, int64_t n_tiles,
                 const __grid_constant__ AdamWArgs a) {
  int64_t r = -1;
  RowView rv{};
  float nss = 0.f, bc2s = 1.f;
  for (int64_t tile = blockIdx.x; tile < n_tiles; tile += gridDim.x) {
    int64_t nr = 0;
    if (rows != nullptr) {
      if (r < 0) {
        nr = find_row(rows, n_rows, tile);
      } else {
        nr = r;
        while (nr + 1 < n_rows && ldg_i64(&rows[nr + 1].tile_begin) <= tile) ++nr;
      }
    }
    if (nr != r) {
      r = nr;
      rv = make_view(rows != nullptr ? load_row(rows + r) : a.inline_row, a);
      const uint32_t cls = (rv.flags >> SRS_ROW_CLASS_SHIFT) & 0xFFu;
      nss = a.hp.neg_step_size[cls];
      bc2s = a.hp.bias2_sqrt[cls];
    }
    const int64_t e0 = (tile - rv.tile_begin) * kTile + (int64_t)threadIdx.x * kVec;
    if (e0 < rv.numel) {
      const int count = (int)min((int64_t)kVec, rv.numel - e0);
      const bool vec = (rv.flags & SRS_ROW_VECTOR_OK) != 0u && count == kVec;
      switch (rv.flags & (SRS_ROW_PARAM_BF16 | SRS_ROW_GRAD_BF16)) {
        case 0: adamw8<false, false, MF, VF>(rv, e0, count, vec, nss, bc2s, a); break;
        case 1: adamw8<true, false, MF, VF>(rv, e0, count, vec, nss, bc2s, a); break;
        case 2: adamw8<false, true, MF, VF>(rv, e0, count, vec, nss, bc2s, a); break;
        default: adamw8<true, true, MF, VF>(rv, e0, count, vec, nss, bc2s, a); break;
      }
    }
  }
}

// ----------------------------------------------------------------- SGDM --

// u' = u*mf + g (two roundings); p' = fma(u', -lr, p)  (sr_states/reference/sgd.py:62-64).
template <bool PB, bool GB, int UF>
__device__ __forceinline__ void sgdm8(const RowView& rv, int64_t e0, int count, bool vec,
                                      const SgdmArgs& a) {
  float p[kVec], g[kVec], u[kVec];
  load_param8<PB>(rv.p, e0, count, vec, p);
  load_param8<GB>(rv.g, e0, count, vec, g);
  load_state8<UF>(rv.s0, e0, count, vec, u);
  const float mf = a.hp.momentum, nlr = a.hp.neg_lr;
#pragma unroll
  for (int j = 0; j < kVec; ++j) {
    const float u1 = __fadd_rn(__fmul_rn(u[j], mf), g[j]);
    p[j] = __fmaf_rn(u1, nlr, p[j]);
    u[j] = u1;
  }
  store_param8<PB>(rv.p, e0, count, vec, p);
  store_state8<UF>(rv.s0, e0, count, vec, u, (uint32_t)e0 + rv.ctr0, a.u_stochastic != 0);
}

template <int UF>
__global__ void __launch_bounds__(kThreads)
    sgdm_kernel(const srs_row* __restrict__ rows, int64_t n_rows, int64_t n_tiles,
                const __grid_constant__ SgdmArgs a) {
  int64_t r = -1;
  RowView rv{};
  for (int64_t tile = blockIdx.x; tile < n_tiles; tile += gridDim.x) {
    int64_t nr = 0;
    if (rows != nullptr) {
      if (r < 0) {
        nr = find_row(rows, n_rows, tile);
      } else {
        nr = r;
        while (nr + 1 < n_rows && ldg_i64(&rows[nr + 1].tile_begin) <= tile) ++nr;
      }
    }
    if (nr != r) {
      r = nr;
      rv = make_view(rows != nullptr ? load_row(rows + r) : a.inline_row, a);
    }
    const int64_t e0 = (tile - rv.tile_begin) * kTile + (int64_t)threadIdx.x * kVec;
    if (e0 < rv.numel) {
      const int count = (int)min((int64_t)kVec, rv.numel - e0);
      const bool vec = (rv.flags & SRS_ROW_VECTOR_OK) != 0u && count == kVec;
      switch (rv.flags & (SRS_ROW_PARAM_BF16 | SRS_ROW_GRAD_BF16)) {
        case 0: sgdm8<false, false, UF>(rv, e0, count, vec, a); break;
        case 1: sgdm8<true, false, UF>(rv, e0, count, vec, a); break;
        case 2: sgdm8<false, true, UF>(rv, e0, count, vec, a); break;
        default: sgdm8<true, true, UF>(rv, e0, count, vec, a); break;
      }
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

template <int MF, int VF>
cudaError_t launch_adamw(const srs_row* rows, int64_t n_rows, int64_t n_tiles,
                         const AdamWArgs& a, int grid_ctas, cudaStream_t stream);

template <int UF>
cudaError_t launch_sgdm(const srs_row* rows, int64_t n_rows, int64_t n_tiles, const SgdmArgs& a,
                        int grid_ctas, cudaStream_t stream);

template <int OF>
cudaError_t launch_cast(const float* x, void* y, int64_t n, uint32_t base, int stochastic,
                        int vec_ok, int grid_ctas, cudaStream_t stream);

}  // namespace srs
