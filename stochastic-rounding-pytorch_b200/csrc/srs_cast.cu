// Standalone FP32 -> {FP32, BF16, FP16, E4M3, E5M2} cast kernels.
#include "srs_kernels.cuh"

namespace srs {

template <int OF>
cudaError_t launch_cast(const float* x, void* y, int64_t n, uint32_t base, int rule,
                        int vec_ok, int grid_ctas, cudaStream_t stream) {
  cudaError_t err = cudaSuccess;
  const int64_t work = (n + kTile - 1) / kTile;
  constexpr int smem = kCastStages * kCastStageBytes;
  const int grid =
      grid_for(reinterpret_cast<const void*>(&cast_kernel<OF>), work, grid_ctas, &err, smem);
  if (err != cudaSuccess) return err;
  cast_kernel<OF><<<grid, kThreads, smem, stream>>>(x, y, n, base, rule, vec_ok);
  return cudaGetLastError();
}

#define SRS_INSTANTIATE(OF)                                                                \
  template cudaError_t launch_cast<OF>(const float*, void*, int64_t, uint32_t, int, int, int, \
                                       cudaStream_t);
SRS_INSTANTIATE(SRS_FMT_F32)
SRS_INSTANTIATE(SRS_FMT_BF16)
SRS_INSTANTIATE(SRS_FMT_F16)
SRS_INSTANTIATE(SRS_FMT_E4M3)
SRS_INSTANTIATE(SRS_FMT_E5M2)
#undef SRS_INSTANTIATE

}  // namespace srs
