// Host-side helpers shared by the kernel files: error reporting, TMA tensor-map
// encoding (through the driver entry point, so the library does not link libcuda),
// per-device kernel attribute setup.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <string>

#include "../../include/genie_tk_b200.h"

namespace gtk {

// Thread-local last error message (returned by gtk_last_error_string()).
void set_error(const std::string& msg);
const char* last_error();

// Report a failed check: stores the message and returns `code`.
int fail(int code, const std::string& msg);

// Map a CUDA runtime error after a launch to GTK_ERR_CUDA with the CUDA message.
int check_launch(const char* what);

// Element type of a TMA map.
enum class TmaType { kBF16, kF16, kF32 };

// Encode a tiled tensor map. dims/box are innermost-first; strides_bytes has rank-1
// entries (stride of dims 1..rank-1 in bytes). swizzle_bytes in {0, 32, 64, 128}.
// Returns GTK_OK or GTK_ERR_TMAP (with the message set).
int encode_tmap(CUtensorMap* map, TmaType type, int rank, const void* base, const uint64_t* dims,
                const uint64_t* strides_bytes, const uint32_t* box, int swizzle_bytes);

// Set the dynamic shared memory limit of a kernel once per (kernel, device).
int ensure_smem(const void* kernel, int bytes);

// Current device must be sm_100 (B200 family). Cached per device.
int check_device();

// Streaming multiprocessors of the current device (cached per device).
int num_sms();

inline uint64_t round_up(uint64_t x, uint64_t m) { return (x + m - 1) / m * m; }

// 4D map over a pair tensor [B, R, N, 128] fp32: dims (c, j, r, b), box (32, 128, 1, 1),
// 128-B swizzle. `transposed` walks z[b, j, r] (the ending-node view; requires R == N).
int make_pair_map(CUtensorMap* m, const float* base, int64_t B, int64_t R, int64_t N, bool transposed);

// 4D map over a 16-bit plane buffer [B, R, C, ld]: dims (col, c, r, b).
int make_plane_map(CUtensorMap* m, const void* base, int64_t B, int64_t R, int64_t C, int64_t cols, int64_t ld,
                   uint32_t box_col, uint32_t box_c, uint32_t box_r, int swizzle);

// 2D map over a packed 16-bit weight matrix [rows][128]: box (64, box_rows), 128-B swizzle.
int make_weight_map(CUtensorMap* m, const void* base, int64_t rows, uint32_t box_rows);

int check_ptr(const void* p, const char* name, uintptr_t align = 16);
bool dims_ok(int64_t v, int64_t max_v = (int64_t(1) << 31) - 1);

// Validate a public dropout descriptor (NULL = no dropout) for a [B, N, N] pair problem and
// fill the kernels' DropArgs (defined in gtk_sm100.cuh). `transposed`: the kernel walks the
// pair tensor as z^T (the ending-node attention). `channels`: the block's channel count; its
// keep vectors are ceil(channels / 128) groups of 128 bits.
struct DropArgs;
int drop_args(const gtk_dropout* d, int64_t B, int64_t N, bool transposed, int channels, DropArgs* out);

}  // namespace gtk
