// Kernel 3: the histogram path for rows whose candidate set is not bounded by a small
// topK (topK == 0 or topK > GS_MAX_TOP_K).
#include "gs_device.cuh"
#include "gs_block.cuh"
#include "gs_internal.cuh"
#include "../../include/gsampler.h"

namespace gs {

__global__ void large_stub_kernel(const __grid_constant__ FinalizeArgs A) {
  const int row = blockIdx.x;
  const RowPlan* pp = A.plans ? A.plans + row : &A.plan0;
  if (pp->mode != kModeLarge || threadIdx.x != 0) return;
  A.ids[row] = -1;
  if (A.flags) A.flags[row] = GS_FLAG_ERR_UNSUPPORTED | GS_FLAG_LARGE_PATH;
  if (A.cand_count) A.cand_count[row] = 0;
}

size_t large_smem_bytes(int64_t, int) { return 0; }

cudaError_t launch_large(const FinalizeArgs& a, int, int rows, size_t, cudaStream_t st) {
  if (rows == 0) return cudaSuccess;
  large_stub_kernel<<<rows, 32, 0, st>>>(a);
  return cudaGetLastError();
}

}  // namespace gs
