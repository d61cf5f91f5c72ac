// extern "C" wrappers around the reference's own GPU launcher
// (src/gpu/gpu_kernel_launcher.hh), compiled from the reference sources into
// oracle/_ref/libref_gpu.so by oracle/ref.mk.  TEST INFRASTRUCTURE: used only by
// tests/golden/make_golden.py to record the reference kernels' outputs.
#include <cublas_v2.h>
#include <cuda_runtime.h>

#include <cstdint>

#include "gpu/gpu_kernel_launcher.hh"

namespace {
struct Ctx {
  cudaStream_t s = nullptr;
  cudaEvent_t e = nullptr;
  Ctx() {
    cudaStreamCreate(&s);
    cudaEventCreateWithFlags(&e, cudaEventDisableTiming);
  }
  ~Ctx() {
    cudaEventDestroy(e);
    cudaStreamDestroy(s);
  }
  int done() { return cudaStreamSynchronize(s) == cudaSuccess ? 0 : 1; }
};
}  // namespace

extern "C" {

int ref_batch_rabitq_distances(const float* d_rot_query, const void* d_factor, const void* d_records, float* d_dist,
                               uint32_t n, uint32_t dim, uint32_t bits) {
  Ctx c;
  gpu::launch_batch_rabitq_distances(c.s, c.e, d_rot_query, d_factor, d_records, d_dist, n, dim, bits);
  return c.done();
}

int ref_batch_l2_distances(const float* d_query, const float* d_cand, float* d_dist, uint32_t n, uint32_t dim) {
  Ctx c;
  gpu::launch_batch_l2_distances(c.s, c.e, d_query, d_cand, d_dist, n, dim);
  return c.done();
}

int ref_query_prepare(const float* d_query, const float* d_P, const float* d_c, float* d_rot_query, void* d_factor,
                      uint32_t dim, uint32_t bits) {
  Ctx c;
  cublasHandle_t h;
  if (cublasCreate(&h) != CUBLAS_STATUS_SUCCESS) return 2;
  gpu::launch_rabitq_query_prepare(c.s, c.e, h, d_query, d_P, d_c, d_rot_query, d_factor, dim, bits);
  const int r = c.done();
  cublasDestroy(h);
  return r;
}

int ref_quantize_single(const float* d_vector, const float* d_P, const float* d_c, void* d_out, uint32_t dim,
                        uint32_t bits, double t_const) {
  Ctx c;
  cublasHandle_t h;
  if (cublasCreate(&h) != CUBLAS_STATUS_SUCCESS) return 2;
  gpu::launch_rabitq_quantize_single(c.s, c.e, h, d_vector, d_P, d_c, d_out, dim, bits, t_const);
  const int r = c.done();
  cublasDestroy(h);
  return r;
}

int ref_robust_prune(const float* d_src, const float* d_cand, const float* d_dists, const uint32_t* d_order,
                     uint32_t n, uint32_t dim, float alpha, uint32_t R, uint32_t* d_out, uint32_t* d_count) {
  Ctx c;
  gpu::launch_robust_prune(c.s, c.e, d_src, d_cand, d_dists, d_order, n, dim, alpha, R, d_out, d_count);
  return c.done();
}

}  // extern "C"
