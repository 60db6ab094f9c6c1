// Internal launch API of the tensor-core attention core (csrc/attn_bwd.cu) for the other
// translation units (the general-shape path runs its attention through it).
#pragma once
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace gtk {
namespace attn {

// head_dim rounded up to the operand planes' 16, 32 or 64 columns.
int padded_head_dim(int d);

// fp32 rows [B*N][N] of pitch `ld` floats, head h's d columns at h * d -> the fp16 plane
// [B*N][H][N][Dp] times `scale` (Dp = padded_head_dim(d), or `Dp` when given: 16, 32 or 64,
// at least d); a clamp to the fp16 range sets the saturation bit in `status`.
int launch_pack(const float* src, int64_t ld, int64_t B, int64_t N, int H, int d, float scale, __half* dst,
                uint32_t* status, cudaStream_t st, int Dp = 0);

// o [B*N][N][H*d] fp32 = softmax(q k^T / sqrt(d) + inf (mask - 1) + tri) v from packed planes,
// without the statistics; mask element (b, i, k) at b*N*N + i*msi + k*msk (or NULL).
int launch_forward(const __half* q, const __half* k, const __half* v, const __half* tri, const float* mask,
                   int64_t msi, int64_t msk, int64_t B, int64_t N, int H, int d, float inf, float* o,
                   cudaStream_t st);

}  // namespace attn
}  // namespace gtk
