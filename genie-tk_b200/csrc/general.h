// The triangle blocks and the pair transition at any channel / head shape (csrc/general.cu).
//
// The tuned kernels of trimul.cu, triatt.cu and transition.cu cover the shapes of the
// benchmark (c_z = c_hidden = 128, 4 heads of 32, a 4x transition). Every other shape the
// reference's modules accept -- its own defaults (c_hidden_tri_att = 32 with 4 heads, so
// head_dim 8), the c_hidden_mul = 64 of its examples, the c_z = 32 / 64 of its tests --
// runs here: fp32 LayerNorms and projections, the per-channel contraction on the tcgen05
// contraction kernel (K2) through fp16 planes, and the attention on the tensor-core
// attention core of attn_bwd.cu through fp16 planes. The
// public entry points of those files dispatch here when the shape is not the tuned one,
// so the C ABI is unchanged.
#pragma once

#include <stddef.h>
#include <stdint.h>

#include "gtk_host.h"
#include "gtk_sm100.cuh"

namespace gtk {
namespace gen {

// Limits of the general path (checked by the *_check functions).
constexpr int kMaxChannels = 512;  // c_z, c_in, c_hidden (TriMul), heads * head_dim
constexpr int kMaxHeads = 32;
constexpr int kMaxHeadDim = 64;

int trimul_check(int c_z, int c_hidden);
size_t trimul_packed_bytes(int c_z, int c_hidden);
int trimul_pack(const gtk_trimul_params* params, int c_z, int c_hidden, void* packed, size_t packed_bytes,
                void* stream);
size_t trimul_workspace_bytes(int64_t B, int64_t N, int c_z, int c_hidden);
int trimul_forward(int outgoing, const float* z, const float* mask, const void* packed, float* out, int add_residual,
                   const DropArgs& drop, void* workspace, size_t workspace_bytes, int64_t B, int64_t N, int c_z,
                   int c_hidden, uint32_t* status, void* stream);

int triatt_check(int c_in, int c_hidden, int heads);
size_t triatt_packed_bytes(int c_in, int c_hidden, int heads);
int triatt_pack(const gtk_triatt_params* params, int c_in, int c_hidden, int heads, void* packed,
                size_t packed_bytes, void* stream);
size_t triatt_workspace_bytes(int64_t B, int64_t N, int c_in, int c_hidden, int heads);
int triatt_forward(int starting, const float* z, const float* mask, const void* packed, float* out,
                   int add_residual, const DropArgs& drop, void* workspace, size_t workspace_bytes, int64_t B,
                   int64_t N, int c_in, int c_hidden, int heads, float inf, uint32_t* status, void* stream);

int transition_check(int c_p, int n);
size_t transition_packed_bytes(int c_p, int n);
int transition_pack(const gtk_transition_params* params, int c_p, int n, void* packed, size_t packed_bytes,
                    void* stream);
size_t transition_workspace_bytes(int64_t B, int64_t N, int c_p, int n);
int transition_forward(const float* z, const float* mask, const void* packed, float* out, int add_residual,
                       void* workspace, size_t workspace_bytes, int64_t B, int64_t N, int c_p, int n,
                       uint32_t* status, void* stream);

}  // namespace gen
}  // namespace gtk
