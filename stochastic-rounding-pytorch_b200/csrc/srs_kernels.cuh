// Kernel templates: fused AdamW / momentum-SGD steps over a row table and the
// standalone cast.  Instantiated per storage format in the srs_*.cu units.
//
// Launch shape: a persistent grid (resident CTAs per SM x SM count); each CTA
// takes a contiguous range of the tile space and walks it row by row.  A tile
// is 256 threads x 8 consecutive elements of one row.  Full tiles of aligned
// rows are double-buffered through shared memory with per-thread cp.async
// copies; results are stored straight from registers as 16-byte vectors.  Each kernel is specialised
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
  // Nonzero when the class's scalars admit the screened arithmetic path:
  // 2^-10 <= bias2_sqrt <= 1, |neg_step_size| <= 1 and 0 <= eps <= 2^28.
  int32_t fast_math[SRS_MAX_STEP_CLASSES];
  // Smallest |m'| whose numerator nss*m' is >= 2^-90 (Inf when nss == 0).
  float m_floor[SRS_MAX_STEP_CLASSES];
  srs_rng rng;
  int32_t m_rule;  // SRS_RULE_* of the stored first moment
  int32_t v_rule;  // SRS_RULE_* of the stored second moment
  srs_peers peers;  // replicas that receive the updated parameters (n_peers == 0: none)
  int64_t tile_lo, tile_hi;  // the launch covers tiles [tile_lo, tile_hi) of the table
};

struct SgdmArgs {
  srs_row inline_row;  // the single row of srs_sgdm_single (rows == nullptr)
  srs_sgdm_hparams hp;
  srs_rng rng;
  int32_t u_rule;  // SRS_RULE_* of the stored momentum
  srs_peers peers;
  int64_t tile_lo, tile_hi;
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
  bool fast_math;    // see AdamWArgs::fast_math
  float m_floor;     // see AdamWArgs::m_floor
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

// The CTA's share of the tile space: the contiguous range [first, last) of
// tiles, walked row by row.  Rows are entered in table order; a row whose
// tile_begin lies beyond the cursor moves the cursor up to it, so a tile is
// only ever processed by the row that holds it and e0 is never negative.
struct TileRange {
  int64_t tile, last, r;
};

__device__ __forceinline__ TileRange cta_tiles(const srs_row* rows, int64_t n_rows,
                                               int64_t tile_lo, int64_t tile_hi) {
  TileRange t;
  const int64_t span = tile_hi - tile_lo;
  t.tile = tile_lo + span * blockIdx.x / gridDim.x;
  t.last = tile_lo + span * (blockIdx.x + 1) / gridDim.x;
  t.r = (rows != nullptr && t.tile < t.last) ? find_row(rows, n_rows, t.tile) : 0;
  return t;
}

// Tiles of row `rv` within the range: [tile, row_end) after aligning the cursor.
__device__ __forceinline__ int64_t row_end_tile(TileRange& t, const RowView& rv) {
  if (t.tile < rv.tile_begin) t.tile = min(t.last, rv.tile_begin);
  return min(t.last, rv.tile_begin + (rv.numel + kTile - 1) / kTile);
}

// Move to the next row; false when the range (or the table) is exhausted.
__device__ __forceinline__ bool next_row(TileRange& t, int64_t n_rows) {
  if (t.tile >= t.last || t.r + 1 >= n_rows) return false;
  ++t.r;
  return true;
}

// Double-buffered staging of full tiles through shared memory.  While a thread
// computes its 8 elements of tile i, its own asynchronous copies (cp.async,
// global -> shared, 8 or 16 bytes each) of tile i+1 are in flight, so the
// memory latency is hidden behind the arithmetic.  Each thread copies and then
// reads back only its own bytes, so the only waits are cp.async.wait_group on
// the thread's own copies (no barrier, no spin loop).  Used for full tiles of
// rows with SRS_ROW_VECTOR_OK, whose addresses meet cp.async's alignment
// (16 bytes; 8 for FP8 states).
//
// Stage layout: the tile's parameter, gradient and state chunks, one block per
// array, thread t's chunk at t * (bytes per thread).
template <int PBYTES, int GBYTES, int S0, int S1>
struct Stage {
  static constexpr int kP = kVec * PBYTES, kG = kVec * GBYTES;
  static constexpr int kS0 = kVec * Fmt<S0>::kBytes;
  static constexpr int kS1 = S1 >= 0 ? kVec * Fmt<(S1 >= 0 ? S1 : 0)>::kBytes : 0;
  static constexpr int kBytes = kThreads * (kP + kG + kS0 + kS1);
};
#ifndef SRS_STAGES
#define SRS_STAGES 2
#endif
constexpr int kStages = SRS_STAGES;
// Rows the staged loops take: element offsets within them fit in 32 bits (the
// RNG contract limits a parameter to 2^32 elements; longer rows of the C ABI
// run the generic path).
constexpr uint32_t kMaxStagedRow = 0xFFFFFFFFu;

template <int BYTES>
__device__ __forceinline__ void cp_async_chunk(uint32_t s, const void* g) {
  if constexpr (BYTES == 8) {
    asm volatile("cp.async.ca.shared.global [%0], [%1], 8;" ::"r"(s), "l"(g) : "memory");
  } else {
    static_assert(BYTES % 16 == 0, "16-byte chunks");
#pragma unroll
    for (int o = 0; o < BYTES; o += 16)
      asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(s + o),
                   "l"(static_cast<const char*>(g) + o)
                   : "memory");
  }
}

__device__ __forceinline__ void cp_async_commit() {
  asm volatile("cp.async.commit_group;" ::: "memory");
}

// Wait until at most kStages - 1 of this thread's copy groups are pending.
__device__ __forceinline__ void cp_async_wait_stage() {
  asm volatile("cp.async.wait_group %0;" ::"n"(kStages - 1) : "memory");
}

// Copies of this thread's chunks of the tile whose thread-0 element is e0 - threadIdx.x*8.
// e0 is a uint32_t element offset within the row (rows of the staged loops hold
// at most 2^32 elements), so each address is one wide multiply-add.
template <int PBYTES, int GBYTES, int S0, int S1>
__device__ __forceinline__ void stage_issue(const RowView& rv, uint32_t e0, char* stage) {
  using S = Stage<PBYTES, GBYTES, S0, S1>;
  const uint32_t base = (uint32_t)__cvta_generic_to_shared(stage);
  const uint32_t t = threadIdx.x;
  const size_t e = e0;
  cp_async_chunk<S::kP>(base + t * S::kP, static_cast<const char*>(rv.p) + e * PBYTES);
  cp_async_chunk<S::kG>(base + kThreads * S::kP + t * S::kG,
                        static_cast<const char*>(rv.g) + e * GBYTES);
  cp_async_chunk<S::kS0>(base + kThreads * (S::kP + S::kG) + t * S::kS0,
                         static_cast<const char*>(rv.s0) + e * Fmt<S0>::kBytes);
  if constexpr (S1 >= 0)
    cp_async_chunk<S::kS1>(base + kThreads * (S::kP + S::kG + S::kS0) + t * S::kS1,
                           static_cast<const char*>(rv.s1) + e * Fmt<S1>::kBytes);
}

// This thread's chunk of array `block` (0 = parameter, 1 = gradient, 2, 3 = states).
template <int F, int PBYTES, int GBYTES, int S0, int S1>
__device__ __forceinline__ void stage_read(const char* stage, int block, uint32_t (&w)[kWords<F>]) {
  using S = Stage<PBYTES, GBYTES, S0, S1>;
  const int offset = block == 0   ? 0
                     : block == 1 ? kThreads * S::kP
                     : block == 2 ? kThreads * (S::kP + S::kG)
                                  : kThreads * (S::kP + S::kG + S::kS0);
  const uint32_t* s = reinterpret_cast<const uint32_t*>(
      stage + offset + threadIdx.x * (kWords<F> * 4));
  if constexpr (kWords<F> % 4 == 0) {
#pragma unroll
    for (int i = 0; i < kWords<F>; i += 4) {
      const uint4 q = reinterpret_cast<const uint4*>(s)[i / 4];
      w[i] = q.x; w[i + 1] = q.y; w[i + 2] = q.z; w[i + 3] = q.w;
    }
  } else {
    const uint2 q = *reinterpret_cast<const uint2*>(s);
    w[0] = q.x; w[1] = q.y;
  }
}

__device__ __forceinline__ float2 splat(float x) { return make_float2(x, x); }

// End of a step that wrote replicas: order the peer or multicast stores before
// whatever the caller's closing barrier releases (a proxy fence first for
// multicast, whose stores reach this GPU's buffer through another address).
__device__ __forceinline__ void publish_replicas(const srs_peers& peers) {
  if (peers.mode == SRS_PEERS_MULTICAST) asm volatile("fence.proxy.alias;" ::: "memory");
  if (peers.n_peers > 0 || peers.mode == SRS_PEERS_MULTICAST) __threadfence_system();
}

// --------------------------------------------------------------- AdamW --

__device__ __forceinline__ float rcp_approx(float x) {
  float y;
  asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// min(a, b, c) in one instruction (sm_100's three-input min.f32; like fminf,
// a NaN operand is ignored).
__device__ __forceinline__ float fmin3(float a, float b, float c) {
  float d;
  asm("min.f32 %0, %1, %2, %3;" : "=f"(d) : "f"(a), "f"(b), "f"(c));
  return d;
}

__device__ __forceinline__ float rsqrt_approx(float x) {
  float y;
  asm("rsqrt.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// Screened arithmetic of the AdamW update.  For a vector of 8 elements whose
//   m'^2 + v' * 2^88 + rsqrt(v') * 2^86  sums to less than 2^126
// (so |m'| < 2^63, 2^-80 < v' < 2^38, nothing NaN or infinite) and whose
// numerators satisfy |num| >= 2^-90 (|m'| >= the class's m_floor), in a step
// class with 2^-10 <= c <= 1,
// |nss| <= 1 and 0 <= eps <= 2^28, every operation below returns the correctly
// rounded result, i.e. the same bits as __fsqrt_rn / __fdiv_rn:
//  * sqrt(v'): g = v'*y, h = y/2 with y ~ 1/sqrt(v') (MUFU), then one
//    correction s = g + (v' - g^2)*h (P. Markstein, "IA-64 and Elementary
//    Functions", Prentice Hall 2000, ch. 8).  Checked on the GPU against
//    __fsqrt_rn for every FP32 input >= 2^-102.
//  * root / c: Markstein's division step with RN(1/c) (div_by_uniform without
//    its per-element range check: 2^-40 < root < 2^19 here).
//  * num / den: the reciprocal y1 = y0 + y0*(1 - den*y0) of y0 ~ 1/den (MUFU)
//    equals RN(1/den) for every den in [2^-126, 2^126) (checked on the GPU for
//    all of them); then q0 = RN(num*y1), r = num - den*q0 (exact), q = q0 +
//    r*y1 is correctly rounded (Markstein 1990) while num, den and the
//    quotient stay in [2^-90, 2^63), [2^-40, 2^30] and [2^-120, 2^113].  The
//    chain runs on -y0 (the MUFU input negated) so that every step is a plain
//    packed FMA, and the residual is formed as num - den*q0 = num + den*(-q0),
//    which also gives the quotient of a zero numerator its sign.
// Vectors outside the screen take the exact per-element operations instead.
__device__ __forceinline__ bool adamw_screen(const float (&m1)[kVec], const float (&v1)[kVec],
                                             float m_floor, float (&y)[kVec]) {
#pragma unroll
  for (int j = 0; j < kVec; ++j) y[j] = rsqrt_approx(v1[j]);
  float2 acc = mul2_rn(make_float2(m1[0], m1[1]), make_float2(m1[0], m1[1]));
#pragma unroll
  for (int i = 0; i < kVec / 2; ++i) {
    if (i > 0)
      acc = fma2_rn(make_float2(m1[2 * i], m1[2 * i + 1]), make_float2(m1[2 * i], m1[2 * i + 1]),
                    acc);
    acc = fma2_rn(make_float2(v1[2 * i], v1[2 * i + 1]), splat2(0x1p88f), acc);
    acc = fma2_rn(make_float2(y[2 * i], y[2 * i + 1]), splat2(0x1p86f), acc);
  }
  const float lo = fmin3(fmin3(fabsf(m1[0]), fabsf(m1[1]), fabsf(m1[2])),
                         fmin3(fabsf(m1[3]), fabsf(m1[4]), fabsf(m1[5])),
                         fminf(fabsf(m1[6]), fabsf(m1[7])));
  return (acc.x + acc.y < 0x1p126f) && (lo >= m_floor);
}

// Correctly rounded s / c for a launch-uniform c with y = RN(1/c): Markstein's
// division step q0 = RN(s*y), r = s - c*q0 (exact through the FMA),
// q1 = RN(q0 + r*y) equals RN(s/c) when nothing underflows or overflows
// (P. Markstein, "Computation of elementary functions on the IBM RISC
// System/6000 processor", IBM J. Res. Dev. 34(1), 1990).
__device__ __forceinline__ float2 div_by_uniform_unchecked(float2 s, const ClassScalars& k) {
  const float2 q0 = mul2_rn(s, splat(k.inv_c));
  const float2 r = fma2_rn(splat(-k.c), q0, s);
  return fma2_rn(r, splat(k.inv_c), q0);
}

// The same with a range check: the host enables it for 2^-30 <= c <= 2^30 and
// numerators 2^-59 <= s < 2^60, where q0, r and q1 stay far from the subnormal
// and overflow ranges.  Everything else (zero, tiny, huge, Inf, NaN
// numerators) takes the IEEE division.
__device__ __forceinline__ float2 div_by_uniform(float2 s, const ClassScalars& k) {
  const float2 q1 = div_by_uniform_unchecked(s, k);
  const uint32_t bx = __float_as_uint(s.x) - k.fast_lo;
  const uint32_t by = __float_as_uint(s.y) - k.fast_lo;
  if (max(bx, by) < k.fast_span) return q1;
  return make_float2(__fdiv_rn(s.x, k.c), __fdiv_rn(s.y, k.c));
}

// Parameter update of a screened vector (see adamw_screen); p is overwritten.
__device__ __forceinline__ void adamw_update_fast(float (&p)[kVec], const float (&m1)[kVec],
                                                  const float (&v1)[kVec], const float (&y)[kVec],
                                                  const ClassScalars& k, const AdamWArgs& a) {
  const float2 eps = splat(a.hp.eps), decay = splat(a.hp.decay), nss = splat(k.nss);
#pragma unroll
  for (int i = 0; i < kVec / 2; ++i) {
    const float2 v2 = make_float2(v1[2 * i], v1[2 * i + 1]);
    const float2 y2 = make_float2(y[2 * i], y[2 * i + 1]);
    const float2 g = mul2_rn(v2, y2), h = mul2_rn(y2, splat(0.5f));
    const float2 r = make_float2(__fmaf_rn(-g.x, g.x, v2.x), __fmaf_rn(-g.y, g.y, v2.y));
    const float2 root = fma2_rn(r, h, g);
    const float2 den = add2_rn(div_by_uniform_unchecked(root, k), eps);
    const float2 n2 = mul2_rn(nss, make_float2(m1[2 * i], m1[2 * i + 1]));
    const float2 ny0 = make_float2(rcp_approx(-den.x), rcp_approx(-den.y));
    const float2 e = fma2_rn(den, ny0, splat(1.0f));
    const float2 ny1 = fma2_rn(e, ny0, ny0);
    const float2 nq0 = mul2_rn(n2, ny1);
    const float2 res = fma2_rn(den, nq0, n2);
    const float2 nq = fma2_rn(res, ny1, nq0);  // -(num / den)
    // p*decay rounded, then RN(pd - nq) as an FMA with multiplier -1: a packed
    // product feeding a packed add or sub would be contracted into one FMA by
    // ptxas (even written as fma(p, decay, -0)), a product feeding an FMA's
    // addend cannot be.  Checked bit for bit against the oracle.
    const float2 pd = mul2_rn(make_float2(p[2 * i], p[2 * i + 1]), decay);
    const float2 p1 = fma2_rn(nq, splat(-1.0f), pd);
    p[2 * i] = p1.x;
    p[2 * i + 1] = p1.y;
  }
}

// Loads of one thread's 8 elements and the moment updates (every path):
//   m' = fma(g, 1-b1, m*b1); v' = fma((1-b2)*g, g, v*b2).
template <bool PB, bool GB, int MF, int VF, bool VEC, typename I>
__device__ __forceinline__ void adamw_moments(const RowView& rv, I e0, int count,
                                              const AdamWArgs& a, float (&p)[kVec],
                                              float (&m)[kVec], float (&v)[kVec]) {
  float g[kVec];
  load_param8<PB>(rv.p, e0, count, VEC, p);
  load_param8<GB>(rv.g, e0, count, VEC, g);
  load_state8<MF>(rv.s0, e0, count, VEC, m);
  load_state8<VF>(rv.s1, e0, count, VEC, v);
  const float2 b1 = splat(a.hp.beta1), b2 = splat(a.hp.beta2);
  const float2 omb1 = splat(a.hp.one_minus_beta1), omb2 = splat(a.hp.one_minus_beta2);
#pragma unroll
  for (int i = 0; i < kVec / 2; ++i) {
    const float2 g2 = make_float2(g[2 * i], g[2 * i + 1]);
    const float2 m1 = fma2_rn(g2, omb1, mul2_rn(make_float2(m[2 * i], m[2 * i + 1]), b1));
    const float2 v1 = fma2_rn(mul2_rn(omb2, g2), g2,
                                 mul2_rn(make_float2(v[2 * i], v[2 * i + 1]), b2));
    m[2 * i] = m1.x;
    m[2 * i + 1] = m1.y;
    v[2 * i] = v1.x;
    v[2 * i + 1] = v1.y;
  }
}

// The whole element update with the per-element IEEE operations (any input).
// Out of line: it runs for vectors outside the screen, which are rare, and it
// reloads its inputs (nothing is stored before the screen's decision) so that
// the screened path keeps its values in registers.
template <bool PB, bool GB, int MF, int VF, bool VEC, typename I>
__device__ __noinline__ void adamw8_exact(const RowView& rv, I e0, int count,
                                          const ClassScalars& k, const AdamWArgs& a) {
  float p[kVec], m[kVec], v[kVec];
  adamw_moments<PB, GB, MF, VF, VEC>(rv, e0, count, a, p, m, v);
  const float2 eps = splat(a.hp.eps), decay = splat(a.hp.decay), nss = splat(k.nss);
#pragma unroll
  for (int i = 0; i < kVec / 2; ++i) {
    const float2 root = make_float2(__fsqrt_rn(v[2 * i]), __fsqrt_rn(v[2 * i + 1]));
    const float2 den = add2_rn(div_by_uniform(root, k), eps);
    const float2 num = mul2_rn(nss, make_float2(m[2 * i], m[2 * i + 1]));
    const float2 upd = make_float2(__fdiv_rn(num.x, den.x), __fdiv_rn(num.y, den.y));
    const float2 p1 = mul_add_rn2(make_float2(p[2 * i], p[2 * i + 1]), decay, upd);
    p[2 * i] = p1.x;
    p[2 * i + 1] = p1.y;
  }
  const uint32_t ctr_m = (uint32_t)e0 + rv.ctr0, ctr_v = (uint32_t)e0 + rv.ctr1;
  store_param8<PB>(rv.p, e0, count, VEC, p, &a.peers);
  store_state8<MF>(rv.s0, e0, count, VEC, m, ctr_m, a.m_rule);
  store_state8<VF>(rv.s1, e0, count, VEC, v, ctr_v, a.v_rule);
}

// Moments, screen and update of one thread's 8 loaded elements, then the
// stores; vectors outside the screen (or classes without the screened
// arithmetic) are redone by adamw8_exact from global memory.
template <bool PB, bool GB, int MF, int VF, bool VEC, typename I>
__device__ __forceinline__ void adamw8_compute(const RowView& rv, I e0, int count,
                                               const ClassScalars& k, const AdamWArgs& a,
                                               float (&p)[kVec], const float (&g)[kVec],
                                               float (&m)[kVec], float (&v)[kVec]) {
  if (k.fast_math) {
    const float2 b1 = splat(a.hp.beta1), b2 = splat(a.hp.beta2);
    const float2 omb1 = splat(a.hp.one_minus_beta1), omb2 = splat(a.hp.one_minus_beta2);
#pragma unroll
    for (int i = 0; i < kVec / 2; ++i) {
      const float2 g2 = make_float2(g[2 * i], g[2 * i + 1]);
      const float2 m1 = fma2_rn(g2, omb1, mul2_rn(make_float2(m[2 * i], m[2 * i + 1]), b1));
      const float2 v1 = fma2_rn(mul2_rn(omb2, g2), g2,
                                   mul2_rn(make_float2(v[2 * i], v[2 * i + 1]), b2));
      m[2 * i] = m1.x;
      m[2 * i + 1] = m1.y;
      v[2 * i] = v1.x;
      v[2 * i + 1] = v1.y;
    }
    float y[kVec];
    if (adamw_screen(m, v, k.m_floor, y)) {
      adamw_update_fast(p, m, v, y, k, a);
      const uint32_t ctr_m = (uint32_t)e0 + rv.ctr0, ctr_v = (uint32_t)e0 + rv.ctr1;
      store_param8<PB>(rv.p, e0, count, VEC, p, &a.peers);
      store_state8_screened<MF>(rv.s0, e0, count, VEC, m, ctr_m,
                                a.m_rule == SRS_RULE_STOCHASTIC);
      store_state8_screened<VF>(rv.s1, e0, count, VEC, v, ctr_v,
                                a.v_rule == SRS_RULE_STOCHASTIC);
      return;
    }
  }
  adamw8_exact<PB, GB, MF, VF, VEC>(rv, e0, count, k, a);
}

// One thread, 8 consecutive elements [e0, e0+count) of a row.  FP32 math in the
// reference CPU operation order (sr_states/reference/adamw.py:79-89): each
// operation rounded once, FMA exactly where PyTorch's CPU kernels use one:
//   m' = fma(g, 1-b1, m*b1); v' = fma((1-b2)*g, g, v*b2);
//   den = sqrt(v')/c + eps;  p' = p*decay + (nss*m')/den.
// VEC: aligned 16-byte vector access of 8 elements; else guarded scalar access.
template <bool PB, bool GB, int MF, int VF, bool VEC>
__device__ __forceinline__ void adamw8(const RowView& rv, int64_t e0, int count,
                                       const ClassScalars& k, const AdamWArgs& a) {
  float p[kVec], g[kVec], m[kVec], v[kVec];
  load_param8<PB>(rv.p, e0, count, VEC, p);
  load_param8<GB>(rv.g, e0, count, VEC, g);
  load_state8<MF>(rv.s0, e0, count, VEC, m);
  load_state8<VF>(rv.s1, e0, count, VEC, v);
  adamw8_compute<PB, GB, MF, VF, VEC>(rv, e0, count, k, a, p, g, m, v);
}

// The same for a full tile whose inputs were staged in shared memory.
template <bool PB, bool GB, int MF, int VF>
__device__ __forceinline__ void adamw8_staged(const RowView& rv, int64_t e0,
                                              const ClassScalars& k, const AdamWArgs& a,
                                              const char* stage) {
  constexpr int PBYTES = PB ? 2 : 4, GBYTES = GB ? 2 : 4;
  constexpr int PF = PB ? SRS_FMT_BF16 : SRS_FMT_F32, GF = GB ? SRS_FMT_BF16 : SRS_FMT_F32;
  float p[kVec], g[kVec], m[kVec], v[kVec];
  {
    uint32_t wp[kWords<PF>], wg[kWords<GF>], wm[kWords<MF>], wv[kWords<VF>];
    stage_read<PF, PBYTES, GBYTES, MF, VF>(stage, 0, wp);
    stage_read<GF, PBYTES, GBYTES, MF, VF>(stage, 1, wg);
    stage_read<MF, PBYTES, GBYTES, MF, VF>(stage, 2, wm);
    stage_read<VF, PBYTES, GBYTES, MF, VF>(stage, 3, wv);
    decode8<PF>(wp, p);
    decode8<GF>(wg, g);
    decode8<MF>(wm, m);
    decode8<VF>(wv, v);
  }
  adamw8_compute<PB, GB, MF, VF, true>(rv, e0, kVec, k, a, p, g, m, v);
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
// Resident CTAs per SM the register budget is sized for: 3 gives 80 registers
// and no spills; the cp.async double buffer, not the warp count, hides the
// memory latency (measured: as fast as 4 CTAs with spills, slightly faster
// once rsqrt(v') is kept from the screen for the update).
#define SRS_ADAMW_MIN_CTAS 3
#endif

template <int MF, int VF, int KIND>
__global__ void __launch_bounds__(kThreads, SRS_ADAMW_MIN_CTAS)
    adamw_kernel(const srs_row* __restrict__ rows, int64_t n_rows, int64_t n_tiles,
                 const __grid_constant__ AdamWArgs a) {
  TileRange t = cta_tiles(rows, n_rows, a.tile_lo, a.tile_hi);
  if (t.tile >= t.last) return;
  do {
    const RowView rv = make_view(rows != nullptr ? load_row(rows + t.r) : a.inline_row, a);
    const uint32_t cls = (rv.flags >> SRS_ROW_CLASS_SHIFT) & 0xFFu;
    ClassScalars k;
    k.nss = a.hp.neg_step_size[cls];
    k.c = a.hp.bias2_sqrt[cls];
    k.inv_c = a.inv_bias2_sqrt[cls];
    k.fast_lo = a.fast_lo[cls];
    k.fast_span = a.fast_hi[cls] - a.fast_lo[cls];
    k.fast_math = a.fast_math[cls] != 0;
    k.m_floor = a.m_floor[cls];
    const int64_t end = row_end_tile(t, rv);
    if constexpr (KIND != kKindMixed) {
      if ((rv.flags & SRS_ROW_VECTOR_OK) != 0u && (rv.flags & 3u) == (uint32_t)KIND &&
          rv.numel <= (int64_t)kMaxStagedRow) {
        // Tiles whose 2048 elements all lie inside the row, addressed by a 32-bit
        // element offset within the row.
        constexpr bool PB = (KIND & 1) != 0, GB = (KIND & 2) != 0;
        using S = Stage<PB ? 2 : 4, GB ? 2 : 4, MF, VF>;
        extern __shared__ __align__(16) char stage_mem[];
        const int64_t full_end = min(end, rv.tile_begin + rv.numel / kTile);
        const int n_full = t.tile < full_end ? (int)(full_end - t.tile) : 0;
        uint32_t eo = (uint32_t)(t.tile - rv.tile_begin) * (uint32_t)kTile + threadIdx.x * kVec;
        for (int d = 0; d < kStages - 1; ++d) {
          if (d < n_full)
            stage_issue<PB ? 2 : 4, GB ? 2 : 4, MF, VF>(rv, eo + d * (uint32_t)kTile,
                                                        stage_mem + d * S::kBytes);
          cp_async_commit();
        }
        for (int i = 0; i < n_full; ++i, eo += (uint32_t)kTile) {
          if (i + kStages - 1 < n_full)
            stage_issue<PB ? 2 : 4, GB ? 2 : 4, MF, VF>(
                rv, eo + (kStages - 1) * (uint32_t)kTile,
                stage_mem + ((i + kStages - 1) % kStages) * S::kBytes);
          cp_async_commit();
          cp_async_wait_stage();
          adamw8_staged<PB, GB, MF, VF>(rv, (int64_t)eo, k, a, stage_mem + (i % kStages) * S::kBytes);
        }
        t.tile += n_full;
      }
    }
    int64_t e0 = (t.tile - rv.tile_begin) * kTile + (int64_t)threadIdx.x * kVec;
    for (; t.tile < end; ++t.tile, e0 += kTile) {
      if (e0 < rv.numel) {
        const int count = (int)min((int64_t)kVec, rv.numel - e0);
        const bool vec = (rv.flags & SRS_ROW_VECTOR_OK) != 0u && count == kVec;
        adamw8_generic<MF, VF>(rv, e0, count, vec, k, a);
      }
    }
  } while (next_row(t, n_rows));
  publish_replicas(a.peers);
}

// ----------------------------------------------------------------- SGDM --

// u' = u*mf + g (two roundings); p' = fma(u', -lr, p)  (sr_states/reference/sgd.py:62-64).
template <bool PB, int UF, bool VEC, typename I>
__device__ __forceinline__ void sgdm8_compute(const RowView& rv, I e0, int count,
                                              const SgdmArgs& a, float (&p)[kVec],
                                              const float (&g)[kVec], float (&u)[kVec]) {
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
  store_param8<PB>(rv.p, e0, count, VEC, p, &a.peers);
  store_state8<UF>(rv.s0, e0, count, VEC, u, (uint32_t)e0 + rv.ctr0, a.u_rule);
}

template <bool PB, bool GB, int UF, bool VEC>
__device__ __forceinline__ void sgdm8(const RowView& rv, int64_t e0, int count,
                                      const SgdmArgs& a) {
  float p[kVec], g[kVec], u[kVec];
  load_param8<PB>(rv.p, e0, count, VEC, p);
  load_param8<GB>(rv.g, e0, count, VEC, g);
  load_state8<UF>(rv.s0, e0, count, VEC, u);
  sgdm8_compute<PB, UF, VEC>(rv, e0, count, a, p, g, u);
}

template <bool PB, bool GB, int UF>
__device__ __forceinline__ void sgdm8_staged(const RowView& rv, uint32_t e0, const SgdmArgs& a,
                                             const char* stage) {
  constexpr int PBYTES = PB ? 2 : 4, GBYTES = GB ? 2 : 4;
  constexpr int PF = PB ? SRS_FMT_BF16 : SRS_FMT_F32, GF = GB ? SRS_FMT_BF16 : SRS_FMT_F32;
  float p[kVec], g[kVec], u[kVec];
  {
    uint32_t wp[kWords<PF>], wg[kWords<GF>], wu[kWords<UF>];
    stage_read<PF, PBYTES, GBYTES, UF, -1>(stage, 0, wp);
    stage_read<GF, PBYTES, GBYTES, UF, -1>(stage, 1, wg);
    stage_read<UF, PBYTES, GBYTES, UF, -1>(stage, 2, wu);
    decode8<PF>(wp, p);
    decode8<GF>(wg, g);
    decode8<UF>(wu, u);
  }
  sgdm8_compute<PB, UF, true>(rv, e0, kVec, a, p, g, u);
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
  TileRange t = cta_tiles(rows, n_rows, a.tile_lo, a.tile_hi);
  if (t.tile >= t.last) return;
  do {
    const RowView rv = make_view(rows != nullptr ? load_row(rows + t.r) : a.inline_row, a);
    const int64_t end = row_end_tile(t, rv);
    if constexpr (KIND != kKindMixed) {
      if ((rv.flags & SRS_ROW_VECTOR_OK) != 0u && (rv.flags & 3u) == (uint32_t)KIND &&
          rv.numel <= (int64_t)kMaxStagedRow) {
        constexpr bool PB = (KIND & 1) != 0, GB = (KIND & 2) != 0;
        using S = Stage<PB ? 2 : 4, GB ? 2 : 4, UF, -1>;
        extern __shared__ __align__(16) char stage_mem[];
        const int64_t full_end = min(end, rv.tile_begin + rv.numel / kTile);
        const int n_full = t.tile < full_end ? (int)(full_end - t.tile) : 0;
        uint32_t eo = (uint32_t)(t.tile - rv.tile_begin) * (uint32_t)kTile + threadIdx.x * kVec;
        for (int d = 0; d < kStages - 1; ++d) {
          if (d < n_full)
            stage_issue<PB ? 2 : 4, GB ? 2 : 4, UF, -1>(rv, eo + d * (uint32_t)kTile,
                                                        stage_mem + d * S::kBytes);
          cp_async_commit();
        }
        for (int i = 0; i < n_full; ++i, eo += (uint32_t)kTile) {
          if (i + kStages - 1 < n_full)
            stage_issue<PB ? 2 : 4, GB ? 2 : 4, UF, -1>(
                rv, eo + (kStages - 1) * (uint32_t)kTile,
                stage_mem + ((i + kStages - 1) % kStages) * S::kBytes);
          cp_async_commit();
          cp_async_wait_stage();
          sgdm8_staged<PB, GB, UF>(rv, eo, a, stage_mem + (i % kStages) * S::kBytes);
        }
        t.tile += n_full;
      }
    }
    int64_t e0 = (t.tile - rv.tile_begin) * kTile + (int64_t)threadIdx.x * kVec;
    for (; t.tile < end; ++t.tile, e0 += kTile) {
      if (e0 < rv.numel) {
        const int count = (int)min((int64_t)kVec, rv.numel - e0);
        const bool vec = (rv.flags & SRS_ROW_VECTOR_OK) != 0u && count == kVec;
        sgdm8_generic<UF>(rv, e0, count, vec, a);
      }
    }
  } while (next_row(t, n_rows));
  publish_replicas(a.peers);
}

// ----------------------------------------------------------------- cast --

// y[e] = round(x[e]) by `rule`; stochastic counter (e + base) mod 2^32 with
// base = seed + offset.
// Round to nearest (and toward zero) is a plain copy-like stream: a grid-stride
// loop of 8-element vectors reaches the copy bandwidth.  The stochastic rules do more arithmetic
// per byte: each CTA takes a contiguous range of 2048-element tiles and, with
// aligned input and output (vec_ok), double-buffers full tiles through shared
// memory by per-thread cp.async copies of the thread's 32 input bytes, so the
// loads of the next tile are in flight during the hashing and rounding.
constexpr int kCastStageBytes = kThreads * kVec * 4;  // one tile of FP32 input
#ifndef SRS_CAST_STAGES
// Tiles in flight per thread, the current one included.  Measured on B200 at
// 2^30 elements: 3 or 4 stages gain at most 1% on the stochastic casts and
// cost the nearest casts (which share the kernel's shared-memory size, hence
// its occupancy) 10-15%.
#define SRS_CAST_STAGES 2
#endif
constexpr int kCastStages = SRS_CAST_STAGES;

template <int OF, int RULE>
__device__ __forceinline__ void cast_grid_stride(const float* __restrict__ x, void* __restrict__ y,
                                                 int64_t n, int vec_ok) {
  const int64_t stride = (int64_t)gridDim.x * kThreads * kVec;
  for (int64_t e0 = ((int64_t)blockIdx.x * kThreads + threadIdx.x) * kVec; e0 < n;
       e0 += stride) {
    const int count = (int)min((int64_t)kVec, n - e0);
    const bool vec = vec_ok != 0 && count == kVec;
    float v[kVec];
    load_state8<SRS_FMT_F32>(x, e0, count, vec, v);
    store_state8<OF>(y, e0, count, vec, v, 0u, RULE);
  }
}

template <int OF>
__global__ void __launch_bounds__(kThreads)
    cast_kernel(const float* __restrict__ x, void* __restrict__ y, int64_t n, uint32_t base,
                int rule, int vec_ok) {
  if (rule == SRS_RULE_NEAREST) {
    cast_grid_stride<OF, SRS_RULE_NEAREST>(x, y, n, vec_ok);
    return;
  }
  if (rule == SRS_RULE_TOWARD_ZERO) {
    cast_grid_stride<OF, SRS_RULE_TOWARD_ZERO>(x, y, n, vec_ok);
    return;
  }
  extern __shared__ __align__(16) char stage_mem[];
  const int64_t n_tiles = (n + kTile - 1) / kTile;
  int64_t tile = n_tiles * blockIdx.x / gridDim.x;
  const int64_t last = n_tiles * (blockIdx.x + 1) / gridDim.x;
  int64_t e0 = tile * kTile + (int64_t)threadIdx.x * kVec;
  if (vec_ok) {
    const int64_t full_end = min(last, n / kTile);
    const int n_full = tile < full_end ? (int)(full_end - tile) : 0;
    const uint32_t slot = (uint32_t)__cvta_generic_to_shared(stage_mem) + threadIdx.x * kVec * 4;
#pragma unroll
    for (int d = 0; d < kCastStages - 1; ++d) {
      if (d < n_full) cp_async_chunk<kVec * 4>(slot + d * kCastStageBytes, x + e0 + d * kTile);
      cp_async_commit();
    }
    for (int i = 0; i < n_full; ++i, e0 += kTile) {
      const unsigned ahead = (unsigned)i + kCastStages - 1;
      if (ahead < (unsigned)n_full)
        cp_async_chunk<kVec * 4>(slot + (ahead % kCastStages) * kCastStageBytes,
                                 x + e0 + (kCastStages - 1) * kTile);
      cp_async_commit();
      asm volatile("cp.async.wait_group %0;" ::"n"(kCastStages - 1) : "memory");
      const uint4* s = reinterpret_cast<const uint4*>(
          stage_mem + ((unsigned)i % kCastStages) * kCastStageBytes + threadIdx.x * kVec * 4);
      const uint4 a = s[0], b = s[1];
      const float v[kVec] = {__uint_as_float(a.x), __uint_as_float(a.y), __uint_as_float(a.z),
                             __uint_as_float(a.w), __uint_as_float(b.x), __uint_as_float(b.y),
                             __uint_as_float(b.z), __uint_as_float(b.w)};
      store_state8<OF>(y, e0, kVec, true, v, base + (uint32_t)e0, SRS_RULE_STOCHASTIC);
    }
    tile += n_full;
  }
  for (; tile < last; ++tile, e0 += kTile) {
    if (e0 < n) {
      const int count = (int)min((int64_t)kVec, n - e0);
      const bool vec = vec_ok != 0 && count == kVec;
      float v[kVec];
      load_state8<SRS_FMT_F32>(x, e0, count, vec, v);
      store_state8<OF>(y, e0, count, vec, v, base + (uint32_t)e0, SRS_RULE_STOCHASTIC);
    }
  }
}

// --------------------------------------------------------------- launch --

// Dynamic shared memory of a launch: the staging buffers of the specialised
// kernels (none for mixed dtype pairs).
template <int MF, int VF, int KIND>
constexpr int adamw_stage_bytes() {
  return KIND == kKindMixed ? 0
                            : kStages * Stage<(KIND & 1) ? 2 : 4, (KIND & 2) ? 2 : 4, MF, VF>::kBytes;
}

template <int UF, int KIND>
constexpr int sgdm_stage_bytes() {
  return KIND == kKindMixed ? 0
                            : kStages * Stage<(KIND & 1) ? 2 : 4, (KIND & 2) ? 2 : 4, UF, -1>::kBytes;
}


// Persistent grid: resident CTAs per SM (occupancy) x SM count, capped by the
// work.  Cached per device and kernel.
int grid_for(const void* kernel, int64_t work_ctas, int grid_ctas, cudaError_t* err,
             int smem_bytes = 0);

// kind: 0..3 = the dtype pair shared by all rows, 4 = mixed.
template <int MF, int VF>
cudaError_t launch_adamw(const srs_row* rows, int64_t n_rows, int64_t n_tiles, int kind,
                         const AdamWArgs& a, int grid_ctas, cudaStream_t stream);

template <int UF>
cudaError_t launch_sgdm(const srs_row* rows, int64_t n_rows, int64_t n_tiles, int kind,
                        const SgdmArgs& a, int grid_ctas, cudaStream_t stream);

template <int OF>
cudaError_t launch_cast(const float* x, void* y, int64_t n, uint32_t base, int rule,
                        int vec_ok, int grid_ctas, cudaStream_t stream);

}  // namespace srs
