// Lazily built, handle-owned copies of an NVFP4 matrix in the layouts the
// tensor-core GEMM reads.  Freed together with the handle.
#include "common.cuh"
#include "matrix_extras.cuh"

namespace fpb {

void release_matrix_extras(fpb_nvfp4_matrix *m) {
  if (!m || !m->extras) return;
  cudaFree(m->extras->sf_tiled);
  cudaFree(m->extras->packed_folded);
  cudaFree(m->extras->sf_tiled_glu);
  delete m->extras;
  m->extras = nullptr;
}

}  // namespace fpb
