// Data movement for the row-sharded pair stack (one process per GPU, the pair tensor
// [B, N, N, 128] split over its first pair index i into P shards of R = N / P rows).
//
// The collectives themselves are NCCL calls made by the host driver; these kernels
// prepare and scatter the contiguous per-peer chunks those calls exchange:
//
//   gtk_copy_3d            strided block copy (`depth` slabs of `height` rows of `width`
//                          bytes, each side with its own row pitch and slab stride): packs
//                          one slice per peer into the contiguous chunks of an all-to-all,
//                          or scatters the received chunks back into slices, in one launch;
//                          gtk_copy_2d is its one-slab form;
//   gtk_pair_transpose_pack  the pair-grid transpose that turns a row shard into the
//                          per-peer chunks of an all-to-all whose result, after one
//                          gtk_copy_3d over the peers, is the transposed shard (used by the
//                          ending-node attention, which runs as the starting node of z^T).
//
// Both are pure HBM streams: 16-byte vector accesses, every pair vector (128 fp32 =
// 512 B) moved by one warp as one fully coalesced transaction per side.

#include <cuda_runtime.h>
#include <stdint.h>

#include <cstring>
#include <string>

#include "gtk_host.h"
#include "gtk_sm100.cuh"

namespace gtk {

// Rows of 16-byte vectors: grid.y walks the rows (slab k = row / height, row r within it;
// one 32-bit division per row, none per element), grid.x the columns, and every thread keeps
// kVec independent 16-byte loads in flight before its stores.
constexpr int kVec = 4;
constexpr int kRowThreads = 256;

__device__ __forceinline__ void copy_row16(uint4* __restrict__ d, const uint4* __restrict__ s, int64_t w16) {
  for (int64_t c0 = static_cast<int64_t>(blockIdx.x) * (kRowThreads * kVec) + threadIdx.x; c0 < w16;
       c0 += static_cast<int64_t>(gridDim.x) * (kRowThreads * kVec)) {
    uint4 v[kVec];
#pragma unroll
    for (int u = 0; u < kVec; ++u) {
      const int64_t c = c0 + u * kRowThreads;
      if (c < w16) v[u] = __ldg(s + c);
    }
#pragma unroll
    for (int u = 0; u < kVec; ++u) {
      const int64_t c = c0 + u * kRowThreads;
      if (c < w16) d[c] = v[u];
    }
  }
}

__global__ void __launch_bounds__(kRowThreads) copy_3d_kernel(uint8_t* __restrict__ dst, int64_t dpitch, int64_t dslab,
                                                              const uint8_t* __restrict__ src, int64_t spitch,
                                                              int64_t sslab, int64_t w16, int height, int rows) {
  for (int row = blockIdx.y; row < rows; row += gridDim.y) {
    const int k = row / height, r = row - k * height;
    copy_row16(reinterpret_cast<uint4*>(dst + k * dslab + r * dpitch),
               reinterpret_cast<const uint4*>(src + k * sslab + r * spitch), w16);
  }
}

// dst[q][b][x][y][:] = src[b][y][q * (C / P) + x][:] for a pair grid src [B][R][C][128] fp32,
// x in [0, C/P), y in [0, R). One warp moves one 512-B pair vector; warps walk the
// destination in order, so the writes stream and each read is one 512-B segment.
__global__ void __launch_bounds__(256) pair_transpose_pack_kernel(const float4* __restrict__ src,
                                                                  float4* __restrict__ dst, int64_t B, int64_t R,
                                                                  int64_t C, int64_t P) {
  const int lane = threadIdx.x & 31;
  const int64_t CP = C / P;
  const int64_t n_pairs = B * R * C;
  const int64_t warps = static_cast<int64_t>(gridDim.x) * (blockDim.x >> 5);
  for (int64_t w = blockIdx.x * static_cast<int64_t>(blockDim.x >> 5) + (threadIdx.x >> 5); w < n_pairs;
       w += warps) {
    // destination pair index w = ((q * B + b) * CP + x) * R + y
    const int64_t y = w % R;
    int64_t t = w / R;
    const int64_t x = t % CP;
    t /= CP;
    const int64_t b = t % B, q = t / B;
    const int64_t s = (b * R + y) * C + q * CP + x;
    dst[w * 32 + lane] = __ldg(src + s * 32 + lane);
  }
}

// Push form of copy_3d: slab k goes to its own destination base dsts[k] (a peer GPU's
// buffer mapped into this process, or a local buffer), so packing, transfer over NVLink and
// placement are one pass. dsts lives in device memory (P pointers).
__global__ void __launch_bounds__(kRowThreads) push_3d_kernel(const uint64_t* __restrict__ dsts, int64_t doff,
                                                              int64_t dpitch, const uint8_t* __restrict__ src,
                                                              int64_t spitch, int64_t sslab, int64_t w16, int height,
                                                              int rows) {
  for (int row = blockIdx.y; row < rows; row += gridDim.y) {
    const int k = row / height, r = row - k * height;
    uint8_t* d = reinterpret_cast<uint8_t*>(__ldg(dsts + k)) + doff + r * dpitch;
    copy_row16(reinterpret_cast<uint4*>(d), reinterpret_cast<const uint4*>(src + k * sslab + r * spitch), w16);
  }
}

// Push form of the pair-grid transpose: pair (b, y, q*(C/P) + x) of src [B][R][C][128] fp32
// goes to dsts[q] at pair ((b*(C/P) + x)*ndst + row0 + y), i.e. straight into row x,
// column row0 + y of peer q's transposed shard [B][C/P][ndst][128]. grid.y = source row
// (b, y); one warp per 512-B pair vector of that row, two vectors in flight per warp, and
// 32-bit index arithmetic per vector.
__global__ void __launch_bounds__(256) push_pair_transpose_kernel(const float4* __restrict__ src,
                                                                  const uint64_t* __restrict__ dsts, int R, int C,
                                                                  int CP, int64_t ndst, int row0, int n_rows) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  for (int row = blockIdx.y; row < n_rows; row += gridDim.y) {  // row = b * R + y
    const int b = row / R, y = row - b * R;
    const float4* s = src + static_cast<int64_t>(row) * C * 32;
    for (int c0 = (blockIdx.x * 8 + warp) * 2; c0 < C; c0 += gridDim.x * 16) {
      float4 v[2];
#pragma unroll
      for (int u = 0; u < 2; ++u)
        if (c0 + u < C) v[u] = __ldg(s + static_cast<int64_t>(c0 + u) * 32 + lane);
#pragma unroll
      for (int u = 0; u < 2; ++u) {
        const int col = c0 + u;
        if (col >= C) break;
        const int q = col / CP, x = col - q * CP;
        float4* d = reinterpret_cast<float4*>(__ldg(dsts + q)) +
                    ((static_cast<int64_t>(b) * CP + x) * ndst + row0 + y) * 32 + lane;
        *d = v[u];
      }
    }
  }
}

// Stream-ordered barrier over P ranks through flags in peer memory. Thread t publishes
// `epoch` into slot `rank` of rank t's flag array (after a system-scope fence, so the
// writes this rank's earlier kernels made into rank t's memory are visible first), then
// waits until slot t of this rank's own array has reached `epoch`. The wait is bounded:
// after 2 s it sets kStatusTimeoutPeer in the status word and returns.
__global__ void peer_barrier_kernel(const uint64_t* __restrict__ flags, int rank, int P, uint32_t epoch,
                                    uint32_t* status) {
  const int t = threadIdx.x;
  if (t >= P) return;
  __threadfence_system();
  uint32_t* remote = reinterpret_cast<uint32_t*>(flags[t]) + rank;
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(remote), "r"(epoch) : "memory");
  const uint32_t* mine = reinterpret_cast<const uint32_t*>(flags[rank]) + t;
  const uint64_t t0 = global_timer_ns();
  while (true) {
    uint32_t v;
    asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(mine) : "memory");
    if (static_cast<int32_t>(v - epoch) >= 0) break;
    if (global_timer_ns() - t0 > kWaitLimitNs) {
      if (status) atomicOr(status, kStatusTimeoutPeer);
      break;
    }
    __nanosleep(64);
  }
}

// Grid of a row copy: enough x-blocks to cover a row (256 threads x kVec vectors each), and
// rows on y (grid-stride beyond 65535).
static dim3 row_grid(int64_t w16, int64_t rows) {
  const int64_t per_block = static_cast<int64_t>(kRowThreads) * kVec;
  int64_t xb = (w16 + per_block - 1) / per_block;
  if (xb < 1) xb = 1;
  if (xb > 1024) xb = 1024;
  const int64_t yb = rows < 65535 ? (rows > 0 ? rows : 1) : 65535;
  return dim3(static_cast<unsigned>(xb), static_cast<unsigned>(yb));
}

static int grid_for(int64_t work_items, int per_block) {
  const int64_t blocks = (work_items + per_block - 1) / per_block;
  const int64_t cap = static_cast<int64_t>(num_sms()) * 8;
  return static_cast<int>(blocks < cap ? (blocks > 0 ? blocks : 1) : cap);
}

}  // namespace gtk

using namespace gtk;

extern "C" {

int gtk_copy_3d(void* dst, int64_t dpitch, int64_t dslab, const void* src, int64_t spitch, int64_t sslab,
                int64_t width, int64_t height, int64_t depth, void* stream) {
  if (width < 0 || height < 0 || depth < 0 || dpitch < width || spitch < width || dslab < 0 || sslab < 0)
    return fail(GTK_ERR_INVALID_ARG, "copy_3d: bad width/height/depth/pitch");
  if (width == 0 || height == 0 || depth == 0) return GTK_OK;
  if ((width | dpitch | spitch | dslab | sslab) & 15)
    return fail(GTK_ERR_ALIGNMENT, "copy_3d: width, pitches and slab strides must be 16-B multiples");
  if (int e = check_ptr(dst, "dst")) return e;
  if (int e = check_ptr(src, "src")) return e;
  if (int e = check_device()) return e;
  if (height * depth > 2147483647) return fail(GTK_ERR_INVALID_ARG, "copy_3d: too many rows");
  const int64_t w16 = width / 16;
  const dim3 grid = row_grid(w16, height * depth);
  copy_3d_kernel<<<grid, kRowThreads, 0, static_cast<cudaStream_t>(stream)>>>(
      static_cast<uint8_t*>(dst), dpitch, dslab, static_cast<const uint8_t*>(src), spitch, sslab, w16,
      static_cast<int>(height), static_cast<int>(height * depth));
  return check_launch("copy_3d_kernel");
}

int gtk_copy_2d(void* dst, int64_t dpitch, const void* src, int64_t spitch, int64_t width, int64_t height,
                void* stream) {
  return gtk_copy_3d(dst, dpitch, 0, src, spitch, 0, width, height, 1, stream);
}

int gtk_copy_2d_dma(void* dst, int64_t dpitch, const void* src, int64_t spitch, int64_t width, int64_t height,
                    void* stream) {
  if (!dst || !src || width < 0 || height < 0 || dpitch < width || spitch < width)
    return fail(GTK_ERR_INVALID_ARG, "copy_2d_dma: bad arguments");
  if (width == 0 || height == 0) return GTK_OK;
  const cudaError_t e = cudaMemcpy2DAsync(dst, static_cast<size_t>(dpitch), src, static_cast<size_t>(spitch),
                                          static_cast<size_t>(width), static_cast<size_t>(height), cudaMemcpyDefault,
                                          static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return fail(GTK_ERR_CUDA, std::string("copy_2d_dma: ") + cudaGetErrorString(e));
  return GTK_OK;
}

int gtk_peer_alloc(size_t bytes, void** ptr, void* handle) {
  if (!ptr || !handle || bytes == 0) return fail(GTK_ERR_INVALID_ARG, "peer_alloc: bad arguments");
  if (int e = check_device()) return e;
  void* p = nullptr;
  cudaError_t e = cudaMalloc(&p, bytes);
  if (e != cudaSuccess) return fail(GTK_ERR_CUDA, std::string("peer_alloc: cudaMalloc: ") + cudaGetErrorString(e));
  e = cudaMemset(p, 0, bytes);
  cudaIpcMemHandle_t h;
  if (e == cudaSuccess) e = cudaIpcGetMemHandle(&h, p);
  if (e != cudaSuccess) {
    cudaFree(p);
    return fail(GTK_ERR_CUDA, std::string("peer_alloc: ") + cudaGetErrorString(e));
  }
  static_assert(sizeof(h) == GTK_PEER_HANDLE_BYTES, "IPC handle size");
  std::memcpy(handle, &h, sizeof(h));
  *ptr = p;
  return GTK_OK;
}

int gtk_peer_free(void* ptr) {
  if (!ptr) return GTK_OK;
  const cudaError_t e = cudaFree(ptr);
  return e == cudaSuccess ? GTK_OK : fail(GTK_ERR_CUDA, std::string("peer_free: ") + cudaGetErrorString(e));
}

int gtk_peer_open(const void* handle, void** ptr) {
  if (!ptr || !handle) return fail(GTK_ERR_INVALID_ARG, "peer_open: bad arguments");
  if (int e = check_device()) return e;
  cudaIpcMemHandle_t h;
  std::memcpy(&h, handle, sizeof(h));
  const cudaError_t e = cudaIpcOpenMemHandle(ptr, h, cudaIpcMemLazyEnablePeerAccess);
  return e == cudaSuccess ? GTK_OK : fail(GTK_ERR_CUDA, std::string("peer_open: ") + cudaGetErrorString(e));
}

int gtk_peer_close(void* ptr) {
  if (!ptr) return GTK_OK;
  const cudaError_t e = cudaIpcCloseMemHandle(ptr);
  return e == cudaSuccess ? GTK_OK : fail(GTK_ERR_CUDA, std::string("peer_close: ") + cudaGetErrorString(e));
}

int gtk_push_3d(const uint64_t* dsts, int P, int64_t doff, int64_t dpitch, const void* src, int64_t spitch,
                int64_t sslab, int64_t width, int64_t height, void* stream) {
  if (P < 1 || width < 0 || height < 0 || doff < 0 || dpitch < width || spitch < width || sslab < 0)
    return fail(GTK_ERR_INVALID_ARG, "push_3d: bad sizes");
  if (width == 0 || height == 0) return GTK_OK;
  if ((width | dpitch | spitch | sslab | doff) & 15)
    return fail(GTK_ERR_ALIGNMENT, "push_3d: width, pitches, offsets and slab strides must be 16-B multiples");
  if (int e = check_ptr(dsts, "dsts", 8)) return e;
  if (int e = check_ptr(src, "src")) return e;
  if (int e = check_device()) return e;
  if (height * P > 2147483647) return fail(GTK_ERR_INVALID_ARG, "push_3d: too many rows");
  const int64_t w16 = width / 16;
  const dim3 grid = row_grid(w16, height * P);
  push_3d_kernel<<<grid, kRowThreads, 0, static_cast<cudaStream_t>(stream)>>>(
      dsts, doff, dpitch, static_cast<const uint8_t*>(src), spitch, sslab, w16, static_cast<int>(height),
      static_cast<int>(height * P));
  return check_launch("push_3d_kernel");
}

int gtk_push_pair_transpose(const float* src, const uint64_t* dsts, int64_t B, int64_t R, int64_t C, int64_t P,
                            int64_t ndst, int64_t row0, void* stream) {
  if (B < 1 || R < 1 || C < 1 || P < 1 || C % P || row0 < 0 || row0 + R > ndst)
    return fail(GTK_ERR_INVALID_ARG, "push_pair_transpose: need C divisible by P and row0 + R <= ndst");
  if (B * R > 2147483647 || C > 2147483647 || row0 > 2147483647)
    return fail(GTK_ERR_INVALID_ARG, "push_pair_transpose: sizes too large");
  if (int e = check_ptr(src, "src")) return e;
  if (int e = check_ptr(dsts, "dsts", 8)) return e;
  if (int e = check_device()) return e;
  const int n_rows = static_cast<int>(B * R);
  const int64_t xb = (C + 15) / 16;  // 8 warps x 2 vectors per block and row
  const int64_t cap_y = 65535;
  dim3 grid(static_cast<unsigned>(xb < 64 ? xb : 64), static_cast<unsigned>(n_rows < cap_y ? n_rows : cap_y));
  push_pair_transpose_kernel<<<grid, 256, 0, static_cast<cudaStream_t>(stream)>>>(
      reinterpret_cast<const float4*>(src), dsts, static_cast<int>(R), static_cast<int>(C), static_cast<int>(C / P),
      ndst, static_cast<int>(row0), n_rows);
  return check_launch("push_pair_transpose_kernel");
}

int gtk_peer_barrier(const uint64_t* flag_ptrs, int rank, int P, uint32_t epoch, uint32_t* status, void* stream) {
  if (P < 1 || P > 1024 || rank < 0 || rank >= P) return fail(GTK_ERR_INVALID_ARG, "peer_barrier: bad rank/P");
  if (int e = check_ptr(flag_ptrs, "flag_ptrs", 8)) return e;
  if (int e = check_device()) return e;
  peer_barrier_kernel<<<1, ((P + 31) / 32) * 32, 0, static_cast<cudaStream_t>(stream)>>>(flag_ptrs, rank, P, epoch,
                                                                                         status);
  return check_launch("peer_barrier_kernel");
}

int gtk_pair_transpose_pack(const float* src, float* dst, int64_t B, int64_t R, int64_t C, int64_t P, void* stream) {
  if (B < 1 || R < 1 || C < 1 || P < 1 || C % P)
    return fail(GTK_ERR_INVALID_ARG, "pair_transpose_pack: need B, R, C, P >= 1 and C divisible by P");
  if (int e = check_ptr(src, "src")) return e;
  if (int e = check_ptr(dst, "dst")) return e;
  if (src == dst) return fail(GTK_ERR_INVALID_ARG, "pair_transpose_pack: src and dst must not alias");
  if (int e = check_device()) return e;
  const int64_t n_pairs = B * R * C;
  pair_transpose_pack_kernel<<<grid_for(n_pairs, 8), 256, 0, static_cast<cudaStream_t>(stream)>>>(
      reinterpret_cast<const float4*>(src), reinterpret_cast<float4*>(dst), B, R, C, P);
  return check_launch("pair_transpose_pack_kernel");
}

}  // extern "C"
