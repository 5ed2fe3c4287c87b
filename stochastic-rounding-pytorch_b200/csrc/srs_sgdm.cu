// Momentum-SGD step kernels, one per momentum storage format.
#include "srs_kernels.cuh"

namespace srs {

template <int UF>
cudaError_t launch_sgdm(const srs_row* rows, int64_t n_rows, int64_t n_tiles, const SgdmArgs& a,
                        int grid_ctas, cudaStream_t stream) {
  cudaError_t err = cudaSuccess;
  const int grid =
      grid_for(reinterpret_cast<const void*>(&sgdm_kernel<UF>), n_tiles, grid_ctas, &err);
  if (err != cudaSuccess) return err;
  sgdm_kernel<UF><<<grid, kThreads, 0, stream>>>(rows, n_rows, n_tiles, a);
  return cudaGetLastError();
}

#define SRS_INSTANTIATE(UF)                                                              \
  template cudaError_t launch_sgdm<UF>(const srs_row*, int64_t, int64_t, const SgdmArgs&, \
                                       int, cudaStream_t);
SRS_INSTANTIATE(SRS_FMT_F32)
SRS_INSTANTIATE(SRS_FMT_BF16)
SRS_INSTANTIATE(SRS_FMT_F16)
SRS_INSTANTIATE(SRS_FMT_E4M3)
SRS_INSTANTIATE(SRS_FMT_E5M2)
#undef SRS_INSTANTIATE

}  // namespace srs
