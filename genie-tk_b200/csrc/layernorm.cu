// LayerNorm over the last axis: the reference's `_C.layernorm` (kernels/bindings.cpp:93-95,
// declared at :49-55, host code kernels/fused_layernorm/layernorm.cu:17-44):
//   out[r, :] = (x[r, :] - mean_r) / sqrt(var_r + eps) * gamma + beta,
// var the biased variance, fp32 in and out (the reference's tensors are fp32).
// `_C.fused_layernorm_linear` does not use it: gtk_layernorm_linear (general.cu) normalises
// the rows inside its GEMM. The triangle blocks' LayerNorms are fused into their projection
// kernels.
//
// One warp per row, grid-stride over rows. The row is read three times (sum, centred second
// moment, output) from L1/L2 -- rows are short (c_z = 128 floats = 512 B) -- and written
// once, so the kernel is bound by one HBM read and one write per element. In place
// (out == x) is allowed: each element is read and written by the same lane.
#include <cuda_runtime.h>

#include "gtk_host.h"
#include "gtk_sm100.cuh"

namespace gtk {

__device__ __forceinline__ float warp_allsum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

__global__ void __launch_bounds__(256)
    layernorm_rows_kernel(const float* __restrict__ x, const float* __restrict__ gamma, const float* __restrict__ beta,
                          float* out, int64_t rows, int D, float eps) {
  const int lane = threadIdx.x & 31;
  const int64_t nwarps = (static_cast<int64_t>(gridDim.x) * blockDim.x) >> 5;
  const float inv_d = 1.0f / static_cast<float>(D);
  for (int64_t r = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5; r < rows; r += nwarps) {
    const float* xr = x + r * D;
    float s = 0.f;
    for (int c = lane; c < D; c += 32) s += xr[c];
    const float mean = warp_allsum(s) * inv_d;
    float v = 0.f;
    for (int c = lane; c < D; c += 32) {
      const float d = xr[c] - mean;
      v = fmaf(d, d, v);
    }
    const float rstd = rsqrtf(warp_allsum(v) * inv_d + eps);
    float* orow = out + r * D;
    for (int c = lane; c < D; c += 32) orow[c] = fmaf((xr[c] - mean) * rstd, __ldg(gamma + c), __ldg(beta + c));
  }
}

}  // namespace gtk

using namespace gtk;

extern "C" {

int gtk_layernorm(const float* x, const float* gamma, const float* beta, float* out, int64_t rows, int64_t D,
                  float eps, void* stream) {
  if (rows < 1 || !dims_ok(rows, int64_t(1) << 40) || D < 1 || D > (1 << 20))
    return fail(GTK_ERR_INVALID_ARG, "layernorm: bad rows / D");
  if (!(eps >= 0.f)) return fail(GTK_ERR_INVALID_ARG, "layernorm: eps must be >= 0");
  if (int e = check_ptr(x, "x", 4)) return e;
  if (int e = check_ptr(gamma, "gamma", 4)) return e;
  if (int e = check_ptr(beta, "beta", 4)) return e;
  if (int e = check_ptr(out, "out", 4)) return e;
  if (int e = check_device()) return e;
  const int64_t blocks_needed = (rows + 7) / 8;
  const int64_t cap = static_cast<int64_t>(num_sms()) * 16;
  const int blocks = static_cast<int>(blocks_needed < cap ? blocks_needed : cap);
  layernorm_rows_kernel<<<blocks, 256, 0, static_cast<cudaStream_t>(stream)>>>(x, gamma, beta, out, rows,
                                                                               static_cast<int>(D), eps);
  return check_launch("layernorm_rows_kernel");
}

}  // extern "C"
