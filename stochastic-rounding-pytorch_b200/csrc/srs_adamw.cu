// AdamW step kernels for one first-moment format (SRS_M_FORMAT, set by the
// build: one object per format) and every second-moment format.
#include "srs_kernels.cuh"

#ifndef SRS_M_FORMAT
#error "compile once per first-moment format with -DSRS_M_FORMAT=<0..4>"
#endif

namespace srs {

template <int MF, int VF, int KIND>
static cudaError_t launch_kind(const srs_row* rows, int64_t n_rows, int64_t n_tiles,
                               const AdamWArgs& a, int grid_ctas, cudaStream_t stream) {
  cudaError_t err = cudaSuccess;
  constexpr int smem = adamw_stage_bytes<MF, VF, KIND>();
  const void* kernel = reinterpret_cast<const void*>(&adamw_kernel<MF, VF, KIND>);
  const int grid = grid_for(kernel, a.tile_hi - a.tile_lo, grid_ctas, &err, smem);
  if (err != cudaSuccess) return err;
  adamw_kernel<MF, VF, KIND><<<grid, kThreads, smem, stream>>>(rows, n_rows, n_tiles, a);
  return cudaGetLastError();
}

template <int MF, int VF>
cudaError_t launch_adamw(const srs_row* rows, int64_t n_rows, int64_t n_tiles, int kind,
                         const AdamWArgs& a, int grid_ctas, cudaStream_t stream) {
  switch (kind) {
    case 0: return launch_kind<MF, VF, 0>(rows, n_rows, n_tiles, a, grid_ctas, stream);
    case 1: return launch_kind<MF, VF, 1>(rows, n_rows, n_tiles, a, grid_ctas, stream);
    case 2: return launch_kind<MF, VF, 2>(rows, n_rows, n_tiles, a, grid_ctas, stream);
    case 3: return launch_kind<MF, VF, 3>(rows, n_rows, n_tiles, a, grid_ctas, stream);
    default: return launch_kind<MF, VF, kKindMixed>(rows, n_rows, n_tiles, a, grid_ctas, stream);
  }
}

#define SRS_INSTANTIATE(VF)                                                                  \
  template cudaError_t launch_adamw<SRS_M_FORMAT, VF>(const srs_row*, int64_t, int64_t, int, \
                                                      const AdamWArgs&, int, cudaStream_t);
SRS_INSTANTIATE(SRS_FMT_F32)
SRS_INSTANTIATE(SRS_FMT_BF16)
SRS_INSTANTIATE(SRS_FMT_F16)
SRS_INSTANTIATE(SRS_FMT_E4M3)
SRS_INSTANTIATE(SRS_FMT_E5M2)
#undef SRS_INSTANTIATE

}  // namespace srs
