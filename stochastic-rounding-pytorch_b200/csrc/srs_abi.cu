// extern "C" entry points of libsrs_b200.so (declared in include/srs_b200.h):
// argument validation, device capability check, persistent-grid sizing and
// dispatch from runtime formats to the kernel instantiations.
#include <cmath>
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <mutex>
#include <unordered_map>

#include <cuda.h>

#include "srs_kernels.cuh"

namespace srs {
namespace {

thread_local char g_error[512] = "";

int fail(int code, const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_error, sizeof(g_error), fmt, ap);
  va_end(ap);
  return code;
}

int cuda_fail(cudaError_t e, const char* what) {
  return fail(SRS_ERR_CUDA, "%s: %s (%s)", what, cudaGetErrorString(e), cudaGetErrorName(e));
}

constexpr int kMaxDevices = 128;
std::mutex g_mutex;
int g_device_ok[kMaxDevices];  // 0 unknown, 1 usable, -1 unusable
int g_sm_count[kMaxDevices];
std::unordered_map<const void*, int> g_blocks_per_sm[kMaxDevices];

int current_device(int* dev) {
  const cudaError_t e = cudaGetDevice(dev);
  if (e != cudaSuccess) return cuda_fail(e, "cudaGetDevice");
  if (*dev < 0 || *dev >= kMaxDevices) return fail(SRS_ERR_UNSUPPORTED_DEVICE, "device %d", *dev);
  return SRS_OK;
}

int check_device() {
  int dev = 0;
  if (int rc = current_device(&dev)) return rc;
  std::lock_guard<std::mutex> lock(g_mutex);
  if (g_device_ok[dev] == 0) {
    int major = 0, minor = 0, sms = 0;
    cudaError_t e = cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev);
    if (e == cudaSuccess) e = cudaDeviceGetAttribute(&minor, cudaDevAttrComputeCapabilityMinor, dev);
    if (e == cudaSuccess) e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    if (e != cudaSuccess) return cuda_fail(e, "cudaDeviceGetAttribute");
    g_sm_count[dev] = sms;
    g_device_ok[dev] = (major == 10 && minor == 0) ? 1 : -1;
    if (g_device_ok[dev] < 0) {
      return fail(SRS_ERR_UNSUPPORTED_DEVICE,
                  "device %d has compute capability %d.%d; these kernels are built for sm_100a "
                  "(compute capability 10.0, B200)",
                  dev, major, minor);
    }
  } else if (g_device_ok[dev] < 0) {
    return fail(SRS_ERR_UNSUPPORTED_DEVICE,
                "device %d is not compute capability 10.0 (sm_100a kernels)", dev);
  }
  return SRS_OK;
}

bool valid_format(int f) { return f >= SRS_FMT_F32 && f <= SRS_FMT_E5M2; }
bool valid_rule(int r) {
  return r == SRS_RULE_NEAREST || r == SRS_RULE_STOCHASTIC || r == SRS_RULE_TOWARD_ZERO;
}

int check_hp_classes(int n) {
  if (n < 1 || n > SRS_MAX_STEP_CLASSES)
    return fail(SRS_ERR_INVALID_ARGUMENT, "n_step_classes must be in [1, %d], got %d",
                SRS_MAX_STEP_CLASSES, n);
  return SRS_OK;
}

using AdamWLaunch = cudaError_t (*)(const srs_row*, int64_t, int64_t, int, const AdamWArgs&,
                                    int, cudaStream_t);
using SgdmLaunch = cudaError_t (*)(const srs_row*, int64_t, int64_t, int, const SgdmArgs&, int,
                                   cudaStream_t);
using CastLaunch = cudaError_t (*)(const float*, void*, int64_t, uint32_t, int, int, int,
                                   cudaStream_t);

#define SRS_ROW5(M)                                                                     \
  {&launch_adamw<M, 0>, &launch_adamw<M, 1>, &launch_adamw<M, 2>, &launch_adamw<M, 3>, \
   &launch_adamw<M, 4>}
const AdamWLaunch kAdamW[5][5] = {SRS_ROW5(0), SRS_ROW5(1), SRS_ROW5(2), SRS_ROW5(3),
                                  SRS_ROW5(4)};
#undef SRS_ROW5
const SgdmLaunch kSgdm[5] = {&launch_sgdm<0>, &launch_sgdm<1>, &launch_sgdm<2>, &launch_sgdm<3>,
                             &launch_sgdm<4>};
const CastLaunch kCast[5] = {&launch_cast<0>, &launch_cast<1>, &launch_cast<2>, &launch_cast<3>,
                             &launch_cast<4>};

int fmt_bytes(int f) { return f == SRS_FMT_F32 ? 4 : (f <= SRS_FMT_F16 ? 2 : 1); }

int kind_index(uint32_t uniform_kind) { return uniform_kind <= 3u ? (int)uniform_kind : 4; }

float bits_float(uint32_t u) {
  float f;
  memcpy(&f, &u, 4);
  return f;
}

uint32_t float_bits(float f) {
  uint32_t u;
  memcpy(&u, &f, 4);
  return u;
}

// RN(1/c) for a positive normal float c.  The product of two floats is exact
// in double and 1 - c*t is then exact too (Sterbenz), so the neighbour of the
// double-rounded estimate with the smallest |1 - c*t| is the correctly rounded
// reciprocal (no ties: 1/c is never a midpoint unless c is a power of two, and
// then 1/c is exact).  Values outside the normal range are returned as 1/c;
// the kernels use their IEEE division for quotients out of range anyway.
float exact_reciprocal(float c) {
  const float est = (float)(1.0 / (double)c);
  if (!(c > 0.0f) || !std::isfinite(est) || est < 1.1754944e-38f) return est;
  float best = est;
  double best_err = 2.0;
  for (int k = -2; k <= 2; ++k) {
    const float t = bits_float(float_bits(est) + (uint32_t)k);
    const double err = std::fabs(1.0 - (double)c * (double)t);
    if (err < best_err) {
      best_err = err;
      best = t;
    }
  }
  return best;
}

// Smallest float f with RN(|nss| * f) >= 2^-90 for every |m'| >= f (Inf when
// nss is zero or not finite): products are monotone and 2^-90 is a float, so
// |nss| * f >= 2^-90 in exact arithmetic is enough.
float numerator_floor(float nss) {
  const double s = std::fabs((double)nss);
  if (!(s > 0.0) || !std::isfinite(s)) return INFINITY;
  float f = (float)(0x1p-90 / s);
  while (std::isfinite(f) && (double)f * s < 0x1p-90) f = std::nextafter(f, INFINITY);
  return f;
}

// Per step class: the exact reciprocal of bias2_sqrt, the numerator range
// [2^-59, 2^60) of the reciprocal division (empty unless 2^-30 <= c <= 2^30)
// and whether the screened arithmetic path applies (2^-10 <= c <= 1,
// |neg_step_size| <= 1, 0 <= eps <= 2^28; NaN scalars fail every test).  A
// toward-zero state rule also disables it: its stores run on the exact path.
// Needs a.m_rule and a.v_rule set.
void fill_reciprocals(const srs_adamw_hparams& hp, AdamWArgs& a) {
  const bool screen_ok = hp.eps >= 0.0f && hp.eps <= 0x1p28f &&
                         a.m_rule != SRS_RULE_TOWARD_ZERO && a.v_rule != SRS_RULE_TOWARD_ZERO;
  for (int c = 0; c < hp.n_step_classes; ++c) {
    const float b = hp.bias2_sqrt[c];
    a.inv_bias2_sqrt[c] = exact_reciprocal(b);
    const bool ok = b >= 0x1p-30f && b <= 0x1p30f;
    a.fast_lo[c] = ok ? 0x22000000u : 0u;
    a.fast_hi[c] = ok ? 0x5D800000u : 0u;
    const float nss = hp.neg_step_size[c];
    a.fast_math[c] = (b >= 0x1p-10f && b <= 1.0f && nss >= -1.0f && nss <= 1.0f && screen_ok) ? 1 : 0;
    a.m_floor[c] = numerator_floor(nss);
  }
}

__global__ void derive_keys_kernel(const uint32_t* __restrict__ index, uint32_t* __restrict__ out,
                                   int64_t n, const srs_rng rng) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i < n) {
    const uint32_t k = update_key(rng, index[i]);
    out[3 * i] = k;
    out[3 * i + 1] = state_key(k, 0u);
    out[3 * i + 2] = state_key(k, 1u);
  }
}

}  // namespace

int grid_for(const void* kernel, int64_t work_ctas, int grid_ctas, cudaError_t* err,
             int smem_bytes) {
  *err = cudaSuccess;
  int dev = 0;
  *err = cudaGetDevice(&dev);
  if (*err != cudaSuccess) return 0;
  int per_sm = 0, sms = 0;
  {
    std::lock_guard<std::mutex> lock(g_mutex);
    sms = g_sm_count[dev];
    auto it = g_blocks_per_sm[dev].find(kernel);
    if (it != g_blocks_per_sm[dev].end()) per_sm = it->second;
  }
  if (per_sm == 0) {
    // First launch of this kernel on this device: above 48 KB a kernel must
    // opt in to its dynamic shared memory, then the occupancy is measured.
    if (smem_bytes > 48 * 1024) {
      *err = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem_bytes);
      if (*err != cudaSuccess) return 0;
    }
    *err = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kernel, kThreads, smem_bytes);
    if (*err != cudaSuccess) return 0;
    if (per_sm < 1) per_sm = 1;
    std::lock_guard<std::mutex> lock(g_mutex);
    g_blocks_per_sm[dev][kernel] = per_sm;
  }
  if (work_ctas <= 0) return 1;
  if (grid_ctas > 0) return (int)(work_ctas < grid_ctas ? work_ctas : grid_ctas);
  if (sms <= 0) sms = 148;
  const int64_t full = (int64_t)sms * per_sm;
  return (int)(work_ctas < full ? work_ctas : full);
}

}  // namespace srs

using namespace srs;

extern "C" {

int srs_abi_version(void) { return SRS_ABI_VERSION; }

int64_t srs_tile_elems(void) { return kTile; }

const char* srs_last_error(void) { return g_error; }

int srs_check_device(void) {
  g_error[0] = '\0';
  return check_device();
}

int srs_cast(const float* x, void* y, int64_t n, int out_format, int rule, uint32_t seed,
             uint32_t offset, int grid_ctas, void* stream) {
  g_error[0] = '\0';
  if (n < 0) return fail(SRS_ERR_INVALID_ARGUMENT, "n must be non-negative, got %lld", (long long)n);
  if (!valid_format(out_format))
    return fail(SRS_ERR_INVALID_ARGUMENT, "unknown output format %d", out_format);
  if (!valid_rule(rule)) return fail(SRS_ERR_INVALID_ARGUMENT, "unknown rounding rule %d", rule);
  if (n == 0) return SRS_OK;
  if (x == nullptr || y == nullptr)
    return fail(SRS_ERR_INVALID_ARGUMENT, "null input or output pointer");
  if (int rc = check_device()) return rc;
  const uintptr_t xa = reinterpret_cast<uintptr_t>(x), ya = reinterpret_cast<uintptr_t>(y);
  const int yb = fmt_bytes(out_format);
  if (xa % 4 != 0 || ya % yb != 0)
    return fail(SRS_ERR_INVALID_ARGUMENT, "input/output pointers are not element aligned");
  const int ya_need = yb * kVec < 16 ? yb * kVec : 16;
  const int vec_ok = (xa % 16 == 0) && (ya % ya_need == 0);
  const cudaError_t e = kCast[out_format](x, y, n, seed + offset, rule, vec_ok, grid_ctas,
                                          static_cast<cudaStream_t>(stream));
  return e == cudaSuccess ? SRS_OK : cuda_fail(e, "srs_cast launch");
}

static int check_multi(const srs_row* rows, int64_t n_rows, int64_t n_tiles, const void* hp,
                       const srs_rng* rng) {
  if (hp == nullptr || rng == nullptr)
    return fail(SRS_ERR_INVALID_ARGUMENT, "null hyperparameter or rng pointer");
  if (rng->key_mode != SRS_KEY_DERIVE && rng->key_mode != SRS_KEY_GIVEN)
    return fail(SRS_ERR_INVALID_ARGUMENT, "unknown key_mode %d", rng->key_mode);
  if (n_rows < 0 || n_tiles < 0) return fail(SRS_ERR_INVALID_ARGUMENT, "negative row/tile count");
  if (n_tiles > 0 && (rows == nullptr || n_rows == 0))
    return fail(SRS_ERR_INVALID_ARGUMENT, "tiles given without rows");
  if (reinterpret_cast<uintptr_t>(rows) % 16 != 0)
    return fail(SRS_ERR_INVALID_ARGUMENT, "row table must be 16-byte aligned");
  return SRS_OK;
}

static int check_peers(const srs_peers* peers) {
  if (peers == nullptr) return fail(SRS_ERR_INVALID_ARGUMENT, "null peers");
  if (peers->n_peers < 0 || peers->n_peers > SRS_MAX_PEERS)
    return fail(SRS_ERR_INVALID_ARGUMENT, "n_peers must be in [0, %d], got %d", SRS_MAX_PEERS,
                peers->n_peers);
  if (peers->mode != SRS_PEERS_STORE && peers->mode != SRS_PEERS_MULTICAST)
    return fail(SRS_ERR_INVALID_ARGUMENT, "unknown peers mode %d", peers->mode);
  if (peers->mode == SRS_PEERS_MULTICAST &&
      ((peers->mc_delta_bf16 % 16) != 0 || (peers->mc_delta_f32 % 16) != 0))
    return fail(SRS_ERR_INVALID_ARGUMENT,
                "multicast deltas must keep 16-byte alignment (got %lld, %lld)",
                (long long)peers->mc_delta_bf16, (long long)peers->mc_delta_f32);
  return SRS_OK;
}

static int check_range(int64_t n_tiles, int64_t tile_lo, int64_t tile_hi) {
  if (tile_lo < 0 || tile_lo > tile_hi || tile_hi > n_tiles)
    return fail(SRS_ERR_INVALID_ARGUMENT, "tile range [%lld, %lld) is not inside [0, %lld)",
                (long long)tile_lo, (long long)tile_hi, (long long)n_tiles);
  return SRS_OK;
}

static int adamw_multi(const srs_row* rows, int64_t n_rows, int64_t n_tiles, int m_format,
                       int m_rule, int v_format, int v_rule, const srs_adamw_hparams* hp,
                       const srs_rng* rng, uint32_t uniform_kind, const srs_peers* peers,
                       int grid_ctas, void* stream, const char* what, int64_t tile_lo = 0,
                       int64_t tile_hi = -1) {
  g_error[0] = '\0';
  if (!valid_format(m_format) || !valid_format(v_format))
    return fail(SRS_ERR_INVALID_ARGUMENT, "unknown state format (%d, %d)", m_format, v_format);
  if (!valid_rule(m_rule) || !valid_rule(v_rule))
    return fail(SRS_ERR_INVALID_ARGUMENT, "unknown rounding rule (%d, %d)", m_rule, v_rule);
  if (int rc = check_multi(rows, n_rows, n_tiles, hp, rng)) return rc;
  if (int rc = check_hp_classes(hp->n_step_classes)) return rc;
  if (peers != nullptr)
    if (int rc = check_peers(peers)) return rc;
  if (tile_hi < 0) tile_hi = n_tiles;
  if (int rc = check_range(n_tiles, tile_lo, tile_hi)) return rc;
  if (tile_lo == tile_hi) return SRS_OK;
  if (int rc = check_device()) return rc;
  AdamWArgs a{};
  a.tile_lo = tile_lo;
  a.tile_hi = tile_hi;
  a.hp = *hp;
  a.rng = *rng;
  a.m_rule = m_rule;
  a.v_rule = v_rule;
  fill_reciprocals(*hp, a);
  if (peers != nullptr) a.peers = *peers;
  const cudaError_t e = kAdamW[m_format][v_format](rows, n_rows, n_tiles,
                                                   kind_index(uniform_kind), a, grid_ctas,
                                                   static_cast<cudaStream_t>(stream));
  return e == cudaSuccess ? SRS_OK : cuda_fail(e, what);
}

static int sgdm_multi(const srs_row* rows, int64_t n_rows, int64_t n_tiles, int u_format,
                      int u_rule, const srs_sgdm_hparams* hp, const srs_rng* rng,
                      uint32_t uniform_kind, const srs_peers* peers, int grid_ctas, void* stream,
                      const char* what, int64_t tile_lo = 0, int64_t tile_hi = -1) {
  g_error[0] = '\0';
  if (!valid_format(u_format))
    return fail(SRS_ERR_INVALID_ARGUMENT, "unknown state format %d", u_format);
  if (!valid_rule(u_rule)) return fail(SRS_ERR_INVALID_ARGUMENT, "unknown rounding rule %d", u_rule);
  if (int rc = check_multi(rows, n_rows, n_tiles, hp, rng)) return rc;
  if (peers != nullptr)
    if (int rc = check_peers(peers)) return rc;
  if (tile_hi < 0) tile_hi = n_tiles;
  if (int rc = check_range(n_tiles, tile_lo, tile_hi)) return rc;
  if (tile_lo == tile_hi) return SRS_OK;
  if (int rc = check_device()) return rc;
  SgdmArgs a{};
  a.tile_lo = tile_lo;
  a.tile_hi = tile_hi;
  a.hp = *hp;
  a.rng = *rng;
  a.u_rule = u_rule;
  if (peers != nullptr) a.peers = *peers;
  const cudaError_t e = kSgdm[u_format](rows, n_rows, n_tiles, kind_index(uniform_kind), a,
                                        grid_ctas, static_cast<cudaStream_t>(stream));
  return e == cudaSuccess ? SRS_OK : cuda_fail(e, what);
}

int srs_adamw_multi(const srs_row* rows, int64_t n_rows, int64_t n_tiles, int m_format,
                    int m_rule, int v_format, int v_rule, const srs_adamw_hparams* hp,
                    const srs_rng* rng, uint32_t uniform_kind, int grid_ctas, void* stream) {
  return adamw_multi(rows, n_rows, n_tiles, m_format, m_rule, v_format, v_rule, hp, rng,
                     uniform_kind, nullptr, grid_ctas, stream, "srs_adamw_multi launch");
}

int srs_adamw_multi_gather(const srs_row* rows, int64_t n_rows, int64_t n_tiles, int m_format,
                           int m_rule, int v_format, int v_rule, const srs_adamw_hparams* hp,
                           const srs_rng* rng, uint32_t uniform_kind, const srs_peers* peers,
                           int grid_ctas, void* stream) {
  if (peers == nullptr) return fail(SRS_ERR_INVALID_ARGUMENT, "null peers");
  return adamw_multi(rows, n_rows, n_tiles, m_format, m_rule, v_format, v_rule, hp, rng,
                     uniform_kind, peers, grid_ctas, stream, "srs_adamw_multi_gather launch");
}

int srs_sgdm_multi(const srs_row* rows, int64_t n_rows, int64_t n_tiles, int u_format,
                   int u_rule, const srs_sgdm_hparams* hp, const srs_rng* rng,
                   uint32_t uniform_kind, int grid_ctas, void* stream) {
  return sgdm_multi(rows, n_rows, n_tiles, u_format, u_rule, hp, rng, uniform_kind, nullptr,
                    grid_ctas, stream, "srs_sgdm_multi launch");
}

int srs_sgdm_multi_gather(const srs_row* rows, int64_t n_rows, int64_t n_tiles, int u_format,
                          int u_rule, const srs_sgdm_hparams* hp, const srs_rng* rng,
                          uint32_t uniform_kind, const srs_peers* peers, int grid_ctas,
                          void* stream) {
  if (peers == nullptr) return fail(SRS_ERR_INVALID_ARGUMENT, "null peers");
  return sgdm_multi(rows, n_rows, n_tiles, u_format, u_rule, hp, rng, uniform_kind, peers,
                    grid_ctas, stream, "srs_sgdm_multi_gather launch");
}

int srs_adamw_multi_range(const srs_row* rows, int64_t n_rows, int64_t n_tiles, int64_t tile_lo,
                          int64_t tile_hi, int m_format, int m_rule, int v_format, int v_rule,
                          const srs_adamw_hparams* hp, const srs_rng* rng, uint32_t uniform_kind,
                          const srs_peers* peers, int grid_ctas, void* stream) {
  return adamw_multi(rows, n_rows, n_tiles, m_format, m_rule, v_format, v_rule, hp, rng,
                     uniform_kind, peers, grid_ctas, stream, "srs_adamw_multi_range launch",
                     tile_lo, tile_hi);
}

int srs_sgdm_multi_range(const srs_row* rows, int64_t n_rows, int64_t n_tiles, int64_t tile_lo,
                         int64_t tile_hi, int u_format, int u_rule, const srs_sgdm_hparams* hp,
                         const srs_rng* rng, uint32_t uniform_kind, const srs_peers* peers,
                         int grid_ctas, void* stream) {
  return sgdm_multi(rows, n_rows, n_tiles, u_format, u_rule, hp, rng, uniform_kind, peers,
                    grid_ctas, stream, "srs_sgdm_multi_range launch", tile_lo, tile_hi);
}

int srs_copy_async(void* dst, const void* src, uint64_t bytes, void* stream) {
  g_error[0] = '\0';
  if (bytes == 0) return SRS_OK;
  if (dst == nullptr || src == nullptr) return fail(SRS_ERR_INVALID_ARGUMENT, "null pointer");
  const cudaError_t e = cudaMemcpyAsync(dst, src, bytes, cudaMemcpyDeviceToDevice,
                                        static_cast<cudaStream_t>(stream));
  return e == cudaSuccess ? SRS_OK : cuda_fail(e, "srs_copy_async");
}

// Base of the allocation holding a device address, through the driver's
// cuMemGetAddressRange (looked up at run time; the runtime is linked
// statically and the driver is loaded by it).
static int allocation_base(const void* p, CUdeviceptr* base) {
  using AddressRange = CUresult (*)(CUdeviceptr*, size_t*, CUdeviceptr);
  static AddressRange fn = nullptr;
  if (fn == nullptr) {
    void* sym = nullptr;
    cudaDriverEntryPointQueryResult status{};
    const cudaError_t e =
        cudaGetDriverEntryPoint("cuMemGetAddressRange", &sym, cudaEnableDefault, &status);
    if (e != cudaSuccess) return cuda_fail(e, "cudaGetDriverEntryPoint(cuMemGetAddressRange)");
    if (status != cudaDriverEntryPointSuccess || sym == nullptr)
      return fail(SRS_ERR_CUDA, "cuMemGetAddressRange is not available from the driver");
    fn = reinterpret_cast<AddressRange>(sym);
  }
  size_t size = 0;
  const CUresult r = fn(base, &size, reinterpret_cast<CUdeviceptr>(p));
  if (r != CUDA_SUCCESS)
    return fail(SRS_ERR_INVALID_ARGUMENT, "address %p is not in a device allocation (CUresult %d)",
                p, (int)r);
  return SRS_OK;
}

int srs_ipc_export(const void* p, void* handle, uint64_t* offset) {
  g_error[0] = '\0';
  if (p == nullptr || handle == nullptr || offset == nullptr)
    return fail(SRS_ERR_INVALID_ARGUMENT, "null pointer");
  if (int rc = check_device()) return rc;
  CUdeviceptr base = 0;
  if (int rc = allocation_base(p, &base)) return rc;
  static_assert(sizeof(cudaIpcMemHandle_t) == SRS_IPC_HANDLE_BYTES, "IPC handle size");
  cudaIpcMemHandle_t h;
  const cudaError_t e = cudaIpcGetMemHandle(&h, reinterpret_cast<void*>(base));
  if (e != cudaSuccess) return cuda_fail(e, "cudaIpcGetMemHandle");
  memcpy(handle, &h, sizeof(h));
  *offset = (uint64_t)(reinterpret_cast<uintptr_t>(p) - (uintptr_t)base);
  return SRS_OK;
}

int srs_ipc_import(const void* handle, void** base) {
  g_error[0] = '\0';
  if (handle == nullptr || base == nullptr) return fail(SRS_ERR_INVALID_ARGUMENT, "null pointer");
  if (int rc = check_device()) return rc;
  cudaIpcMemHandle_t h;
  memcpy(&h, handle, sizeof(h));
  const cudaError_t e = cudaIpcOpenMemHandle(base, h, cudaIpcMemLazyEnablePeerAccess);
  return e == cudaSuccess ? SRS_OK : cuda_fail(e, "cudaIpcOpenMemHandle");
}

int srs_ipc_close(void* base) {
  g_error[0] = '\0';
  if (base == nullptr) return fail(SRS_ERR_INVALID_ARGUMENT, "null pointer");
  const cudaError_t e = cudaIpcCloseMemHandle(base);
  return e == cudaSuccess ? SRS_OK : cuda_fail(e, "cudaIpcCloseMemHandle");
}

static int check_single_row(const srs_row* row, int64_t* n_tiles) {
  if (row == nullptr) return fail(SRS_ERR_INVALID_ARGUMENT, "null row");
  if (row->numel < 0) return fail(SRS_ERR_INVALID_ARGUMENT, "negative numel");
  *n_tiles = (row->numel + kTile - 1) / kTile;
  if (*n_tiles > 0 && (row->param == 0 || row->grad == 0))
    return fail(SRS_ERR_INVALID_ARGUMENT, "null parameter or gradient address");
  return SRS_OK;
}

int srs_adamw_single(const srs_row* row, int m_format, int m_rule, int v_format, int v_rule,
                     const srs_adamw_hparams* hp, int grid_ctas, void* stream) {
  g_error[0] = '\0';
  if (!valid_format(m_format) || !valid_format(v_format))
    return fail(SRS_ERR_INVALID_ARGUMENT, "unknown state format (%d, %d)", m_format, v_format);
  if (!valid_rule(m_rule) || !valid_rule(v_rule))
    return fail(SRS_ERR_INVALID_ARGUMENT, "unknown rounding rule (%d, %d)", m_rule, v_rule);
  if (hp == nullptr) return fail(SRS_ERR_INVALID_ARGUMENT, "null hyperparameter pointer");
  if (hp->n_step_classes != 1)
    return fail(SRS_ERR_INVALID_ARGUMENT, "a single-tensor step has exactly one step class");
  int64_t n_tiles = 0;
  if (int rc = check_single_row(row, &n_tiles)) return rc;
  if (n_tiles == 0) return SRS_OK;
  if (row->state[0] == 0 || row->state[1] == 0)
    return fail(SRS_ERR_INVALID_ARGUMENT, "null state address");
  if (int rc = check_device()) return rc;
  AdamWArgs a{};
  a.inline_row = *row;
  a.inline_row.tile_begin = 0;
  a.inline_row.flags &= ~(0xFFu << SRS_ROW_CLASS_SHIFT);
  a.tile_lo = 0;
  a.tile_hi = n_tiles;
  a.hp = *hp;
  a.rng.key_mode = SRS_KEY_GIVEN;
  a.m_rule = m_rule;
  a.v_rule = v_rule;
  fill_reciprocals(*hp, a);
  const cudaError_t e = kAdamW[m_format][v_format](nullptr, 1, n_tiles, (int)(row->flags & 3u),
                                                   a, grid_ctas,
                                                   static_cast<cudaStream_t>(stream));
  return e == cudaSuccess ? SRS_OK : cuda_fail(e, "srs_adamw_single launch");
}

int srs_sgdm_single(const srs_row* row, int u_format, int u_rule, const srs_sgdm_hparams* hp,
                    int grid_ctas, void* stream) {
  g_error[0] = '\0';
  if (!valid_format(u_format))
    return fail(SRS_ERR_INVALID_ARGUMENT, "unknown state format %d", u_format);
  if (!valid_rule(u_rule)) return fail(SRS_ERR_INVALID_ARGUMENT, "unknown rounding rule %d", u_rule);
  if (hp == nullptr) return fail(SRS_ERR_INVALID_ARGUMENT, "null hyperparameter pointer");
  int64_t n_tiles = 0;
  if (int rc = check_single_row(row, &n_tiles)) return rc;
  if (n_tiles == 0) return SRS_OK;
  if (row->state[0] == 0) return fail(SRS_ERR_INVALID_ARGUMENT, "null state address");
  if (int rc = check_device()) return rc;
  SgdmArgs a{};
  a.inline_row = *row;
  a.inline_row.tile_begin = 0;
  a.tile_lo = 0;
  a.tile_hi = n_tiles;
  a.hp = *hp;
  a.rng.key_mode = SRS_KEY_GIVEN;
  a.u_rule = u_rule;
  const cudaError_t e = kSgdm[u_format](nullptr, 1, n_tiles, (int)(row->flags & 3u), a,
                                        grid_ctas, static_cast<cudaStream_t>(stream));
  return e == cudaSuccess ? SRS_OK : cuda_fail(e, "srs_sgdm_single launch");
}

int srs_derive_keys(const uint32_t* param_index, uint32_t* out, int64_t n, const srs_rng* rng,
                    void* stream) {
  g_error[0] = '\0';
  if (n < 0 || rng == nullptr) return fail(SRS_ERR_INVALID_ARGUMENT, "bad arguments");
  if (n == 0) return SRS_OK;
  if (param_index == nullptr || out == nullptr)
    return fail(SRS_ERR_INVALID_ARGUMENT, "null pointer");
  if (int rc = check_device()) return rc;
  const int blocks = (int)((n + 255) / 256);
  derive_keys_kernel<<<blocks, 256, 0, static_cast<cudaStream_t>(stream)>>>(param_index, out, n,
                                                                             *rng);
  const cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? SRS_OK : cuda_fail(e, "srs_derive_keys launch");
}

}  // extern "C"

// ---- srs_adamw_multi_noalloc ------------------------------------------------
// The multi-tensor AdamW step for callers that must not allocate device memory
// while stepping: a runtime whose device memory is reserved up front (a
// serving or training process that hands the whole HBM to its own arena), or
// code running where an allocator call could block or fail.  srs_adamw_multi
// needs its row table in device memory that the caller allocated; this entry
// point instead copies a host row table into the fixed table below, which is
// part of the library's device image (one instance per device, loaded with the
// module), and launches the same kernel on it.
//
// The table is the only scratch the step uses.  Every call on a device shares
// it and leaves its own rows in it; nothing in it has to start at zero, as a
// call writes rows [0, n_rows) before its kernel reads them and the kernel
// reads no row beyond n_rows.  Two calls whose copies and kernels can overlap
// in time (different streams, or host threads without ordering) race on it.
static __device__ __align__(256) srs_row g_noalloc_rows[SRS_NOALLOC_MAX_ROWS];

namespace srs {
namespace {

srs_row* g_noalloc_table[kMaxDevices];  // device address of g_noalloc_rows, per device

// Set-up on a device's first call: look up where the module placed the table.
// Module loading is lazy, so this first lookup may load the library's device
// code; it is refused while the stream captures (`capturing`), so the first
// call on each device has to come before any stream capture.
int noalloc_table(srs_row** table, bool capturing) {
  int dev = 0;
  if (int rc = current_device(&dev)) return rc;
  std::lock_guard<std::mutex> lock(g_mutex);
  if (g_noalloc_table[dev] == nullptr) {
    if (capturing)
      return fail(SRS_ERR_INVALID_ARGUMENT,
                  "srs_adamw_multi_noalloc: the first call on device %d was made during stream "
                  "capture; make one call on the device before capturing",
                  dev);
    void* address = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&address, g_noalloc_rows);
    if (e != cudaSuccess) return cuda_fail(e, "cudaGetSymbolAddress(row table)");
    g_noalloc_table[dev] = static_cast<srs_row*>(address);
  }
  *table = g_noalloc_table[dev];
  return SRS_OK;
}

// Alignment SRS_ROW_VECTOR_OK promises for an array of `elem_bytes`-byte
// elements: the 8-element vector accesses and cp.async copies of the kernels
// move 16 bytes at a time (8 for one-byte FP8 states).
uint64_t vector_alignment(int elem_bytes) { return elem_bytes == 1 ? 8u : 16u; }

// Host-side check of a row table: tile_begin prefix sums, n_tiles, step
// classes, addresses, and that every row flagged SRS_ROW_VECTOR_OK has the
// alignment the flag promises (a wrongly flagged row would send the kernel
// into misaligned vector accesses).  Returns the dtype kind the rows share
// (or mixed).
int check_host_rows(const srs_row* rows, int64_t n_rows, int64_t n_tiles, int n_classes,
                    int m_format, int v_format, uint32_t* kind) {
  int64_t tile = 0;
  uint32_t first = rows[0].flags & 3u;
  *kind = first;
  for (int64_t r = 0; r < n_rows; ++r) {
    const srs_row& row = rows[r];
    if (row.numel < 0) return fail(SRS_ERR_INVALID_ARGUMENT, "row %lld: negative numel", (long long)r);
    if (row.tile_begin != tile)
      return fail(SRS_ERR_INVALID_ARGUMENT, "row %lld: tile_begin %lld, expected %lld",
                  (long long)r, (long long)row.tile_begin, (long long)tile);
    const uint32_t cls = (row.flags >> SRS_ROW_CLASS_SHIFT) & 0xFFu;
    if ((int)cls >= n_classes)
      return fail(SRS_ERR_INVALID_ARGUMENT, "row %lld: step class %u, only %d classes",
                  (long long)r, cls, n_classes);
    if (row.numel > 0 && (row.param == 0 || row.grad == 0 || row.state[0] == 0 ||
                          row.state[1] == 0))
      return fail(SRS_ERR_INVALID_ARGUMENT, "row %lld: null address", (long long)r);
    if ((row.flags & SRS_ROW_VECTOR_OK) != 0u) {
      const uint64_t need_p = vector_alignment((row.flags & SRS_ROW_PARAM_BF16) ? 2 : 4);
      const uint64_t need_g = vector_alignment((row.flags & SRS_ROW_GRAD_BF16) ? 2 : 4);
      const uint64_t need_m = vector_alignment(fmt_bytes(m_format));
      const uint64_t need_v = vector_alignment(fmt_bytes(v_format));
      if (row.param % need_p != 0u || row.grad % need_g != 0u || row.state[0] % need_m != 0u ||
          row.state[1] % need_v != 0u)
        return fail(SRS_ERR_INVALID_ARGUMENT,
                    "row %lld: SRS_ROW_VECTOR_OK set but an address is not aligned for vector "
                    "access (param and grad need 16 bytes, states 16 bytes, 8 for FP8)",
                    (long long)r);
    }
    if ((row.flags & 3u) != first) *kind = SRS_KIND_MIXED;
    tile += (row.numel + kTile - 1) / kTile;
  }
  if (tile != n_tiles)
    return fail(SRS_ERR_INVALID_ARGUMENT, "n_tiles is %lld, the rows hold %lld tiles",
                (long long)n_tiles, (long long)tile);
  return SRS_OK;
}

}  // namespace
}  // namespace srs

extern "C" int srs_adamw_multi_noalloc(const srs_row* host_rows, int64_t n_rows, int64_t n_tiles,
                                       int m_format, int m_rule, int v_format, int v_rule,
                                       const srs_adamw_hparams* hp, const srs_rng* rng,
                                       int grid_ctas, void* stream) {
  g_error[0] = '\0';
  if (!valid_format(m_format) || !valid_format(v_format))
    return fail(SRS_ERR_INVALID_ARGUMENT, "unknown state format (%d, %d)", m_format, v_format);
  if (!valid_rule(m_rule) || !valid_rule(v_rule))
    return fail(SRS_ERR_INVALID_ARGUMENT, "unknown rounding rule (%d, %d)", m_rule, v_rule);
  if (hp == nullptr || rng == nullptr)
    return fail(SRS_ERR_INVALID_ARGUMENT, "null hyperparameter or rng pointer");
  if (rng->key_mode != SRS_KEY_DERIVE && rng->key_mode != SRS_KEY_GIVEN)
    return fail(SRS_ERR_INVALID_ARGUMENT, "unknown key_mode %d", rng->key_mode);
  if (int rc = check_hp_classes(hp->n_step_classes)) return rc;
  if (n_rows < 0 || n_tiles < 0) return fail(SRS_ERR_INVALID_ARGUMENT, "negative row/tile count");
  if (n_rows > SRS_NOALLOC_MAX_ROWS)
    return fail(SRS_ERR_INVALID_ARGUMENT,
                "%lld rows exceed the fixed table of srs_adamw_multi_noalloc (at most %d rows); "
                "split the group or use srs_adamw_multi",
                (long long)n_rows, SRS_NOALLOC_MAX_ROWS);
  if (n_rows == 0) {
    if (n_tiles != 0) return fail(SRS_ERR_INVALID_ARGUMENT, "tiles given without rows");
    return SRS_OK;
  }
  if (host_rows == nullptr) return fail(SRS_ERR_INVALID_ARGUMENT, "null row table");
  uint32_t kind = 0;
  if (int rc = check_host_rows(host_rows, n_rows, n_tiles, hp->n_step_classes, m_format,
                               v_format, &kind))
    return rc;
  if (n_tiles == 0) return SRS_OK;
  if (int rc = check_device()) return rc;
  const cudaStream_t s = static_cast<cudaStream_t>(stream);
  cudaStreamCaptureStatus capture = cudaStreamCaptureStatusNone;
  cudaError_t e = cudaStreamIsCapturing(s, &capture);
  if (e != cudaSuccess) return cuda_fail(e, "cudaStreamIsCapturing");
  const bool capturing = capture != cudaStreamCaptureStatusNone;
  if (capturing) {
    // A captured row copy is a graph node that reads host_rows again at every
    // replay: only page-locked rows can be copied that way, and they have to
    // stay valid for as long as the graph can be replayed.
    cudaPointerAttributes where{};
    e = cudaPointerGetAttributes(&where, host_rows);
    if (e != cudaSuccess) return cuda_fail(e, "cudaPointerGetAttributes(host_rows)");
    if (where.type != cudaMemoryTypeHost)
      return fail(SRS_ERR_INVALID_ARGUMENT,
                  "srs_adamw_multi_noalloc under stream capture needs page-locked host_rows "
                  "(every replay copies them again)");
  }
  srs_row* table = nullptr;
  if (int rc = noalloc_table(&table, capturing)) return rc;
  // Stream-ordered: the kernel below (and any later call's copy on this stream)
  // sees exactly these rows.  The copy may read host_rows at any time until it
  // has run on the stream (at every replay, when captured), so the caller keeps
  // them valid until then.
  e = cudaMemcpyAsync(table, host_rows, (size_t)n_rows * sizeof(srs_row),
                      cudaMemcpyHostToDevice, s);
  if (e != cudaSuccess) return cuda_fail(e, "srs_adamw_multi_noalloc row copy");
  AdamWArgs a{};
  a.hp = *hp;
  a.rng = *rng;
  a.m_rule = m_rule;
  a.v_rule = v_rule;
  fill_reciprocals(*hp, a);
  a.tile_lo = 0;
  a.tile_hi = n_tiles;
  e = kAdamW[m_format][v_format](table, n_rows, n_tiles, kind_index(kind), a, grid_ctas, s);
  return e == cudaSuccess ? SRS_OK : cuda_fail(e, "srs_adamw_multi_noalloc launch");
}
