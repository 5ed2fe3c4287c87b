// Momentum-SGD step kernels, one per momentum storage format.
#include "srs_kernels.cuh"

namespace srs {

template <int UF, int KIND>
static cudaError_t launch_kind(const srs_row* rows, int64_t n_rows, int64_t n_tiles,
                               const SgdmArgs& a, int grid_ctas, cudaStream_t stream) {
  cudaError_t err = cudaSuccess;
  constexpr int smem = sgdm_stage_bytes<UF, KIND>();
  const void* kernel = reinterpret_cast<const void*>(&sgdm_kernel<UF, KIND>);
  const int grid = grid_for(kernel, a.tile_hi - a.tile_lo, grid_ctas, &err, smem);
  if (err != cudaSuccess) return err;
  sgdm_kernel<UF, KIND><<<grid, kThreads, smem, stream>>>(rows, n_rows, n_tiles, a);
  return cudaGetLastError();
}

template <int UF>
cudaError_t launch_sgdm(const srs_row* rows, int64_t n_rows, int64_t n_tiles, int kind,
                        const SgdmArgs& a, int grid_ctas, cudaStream_t stream) {
  switch (kind) {
    case 0: return launch_kind<UF, 0>(rows, n_rows, n_tiles, a, grid_ctas, stream);
    case 1: return launch_kind<UF, 1>(rows, n_rows, n_tiles, a, grid_ctas, stream);
    case 2: return launch_kind<UF, 2>(rows, n_rows, n_tiles, a, grid_ctas, stream);
    case 3: return launch_kind<UF, 3>(rows, n_rows, n_tiles, a, grid_ctas, stream);
    default: return launch_kind<UF, kKindMixed>(rows, n_rows, n_tiles, a, grid_ctas, stream);
  }
}

#define SRS_INSTANTIATE(UF)                                                                   \
  template cudaError_t launch_sgdm<UF>(const srs_row*, int64_t, int64_t, int, const SgdmArgs&, \
                                       int, cudaStream_t);
SRS_INSTANTIATE(SRS_FMT_F32)
SRS_INSTANTIATE(SRS_FMT_BF16)
SRS_INSTANTIATE(SRS_FMT_F16)
SRS_INSTANTIATE(SRS_FMT_E4M3)
SRS_INSTANTIATE(SRS_FMT_E5M2)
#undef SRS_INSTANTIATE

}  // namespace srs
