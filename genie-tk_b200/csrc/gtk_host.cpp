#include "gtk_host.h"

#include <cudaTypedefs.h>

#include <mutex>
#include <set>
#include <utility>

namespace gtk {

namespace {
thread_local std::string g_last_error;
std::mutex g_mu;
}  // namespace

void set_error(const std::string& msg) { g_last_error = msg; }
const char* last_error() { return g_last_error.c_str(); }

int fail(int code, const std::string& msg) {
  set_error(msg);
  return code;
}

int check_launch(const char* what) {
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) {
    return fail(GTK_ERR_CUDA, std::string(what) + ": " + cudaGetErrorString(e));
  }
  return GTK_OK;
}

static PFN_cuTensorMapEncodeTiled_v12000 get_encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static bool tried = false;
  std::lock_guard<std::mutex> lock(g_mu);
  if (!tried) {
    tried = true;
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess) {
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
    }
  }
  return fn;
}

int encode_tmap(CUtensorMap* map, TmaType type, int rank, const void* base, const uint64_t* dims,
                const uint64_t* strides_bytes, const uint32_t* box, int swizzle_bytes) {
  auto fn = get_encode_fn();
  if (!fn) return fail(GTK_ERR_TMAP, "cuTensorMapEncodeTiled is not available from the driver");
  if ((reinterpret_cast<uintptr_t>(base) & 15u) != 0) return fail(GTK_ERR_ALIGNMENT, "TMA base not 16-B aligned");
  cuuint64_t gdim[5];
  cuuint64_t gstride[4];
  cuuint32_t bdim[5];
  cuuint32_t estride[5];
  for (int i = 0; i < rank; ++i) {
    gdim[i] = dims[i];
    bdim[i] = box[i];
    estride[i] = 1;
    if (dims[i] == 0) return fail(GTK_ERR_INVALID_ARG, "TMA dimension of size 0");
  }
  for (int i = 0; i < rank - 1; ++i) {
    gstride[i] = strides_bytes[i];
    if (strides_bytes[i] % 16 != 0) return fail(GTK_ERR_ALIGNMENT, "TMA stride not a multiple of 16 bytes");
  }
  CUtensorMapSwizzle sw = CU_TENSOR_MAP_SWIZZLE_NONE;
  if (swizzle_bytes == 32) sw = CU_TENSOR_MAP_SWIZZLE_32B;
  if (swizzle_bytes == 64) sw = CU_TENSOR_MAP_SWIZZLE_64B;
  if (swizzle_bytes == 128) sw = CU_TENSOR_MAP_SWIZZLE_128B;
  CUtensorMapDataType dt = type == TmaType::kBF16  ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16
                           : type == TmaType::kF16 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16
                                                   : CU_TENSOR_MAP_DATA_TYPE_FLOAT32;
  CUresult r = fn(map, dt, static_cast<cuuint32_t>(rank), const_cast<void*>(base), gdim, gstride, bdim, estride,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, sw, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    return fail(GTK_ERR_TMAP, "cuTensorMapEncodeTiled failed with CUresult " + std::to_string(static_cast<int>(r)));
  }
  return GTK_OK;
}

int ensure_smem(const void* kernel, int bytes) {
  static std::set<std::pair<const void*, int>> done;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return fail(GTK_ERR_CUDA, "cudaGetDevice failed");
  std::lock_guard<std::mutex> lock(g_mu);
  auto key = std::make_pair(kernel, dev);
  if (done.count(key)) return GTK_OK;
  cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
  if (e != cudaSuccess) return fail(GTK_ERR_CUDA, std::string("cudaFuncSetAttribute: ") + cudaGetErrorString(e));
  done.insert(key);
  return GTK_OK;
}

int check_device() {
  static std::set<int> ok_devices;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return fail(GTK_ERR_CUDA, "cudaGetDevice failed");
  {
    std::lock_guard<std::mutex> lock(g_mu);
    if (ok_devices.count(dev)) return GTK_OK;
  }
  int major = 0, minor = 0;
  cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev);
  cudaDeviceGetAttribute(&minor, cudaDevAttrComputeCapabilityMinor, dev);
  if (major != 10 || minor != 0) {
    return fail(GTK_ERR_DEVICE, "genie_tk_b200 kernels are built for sm_100a (B200); device " + std::to_string(dev) +
                                    " is sm_" + std::to_string(major) + std::to_string(minor));
  }
  std::lock_guard<std::mutex> lock(g_mu);
  ok_devices.insert(dev);
  return GTK_OK;
}

int num_sms() {
  static int cache[64] = {0};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 148;
  if (!cache[dev]) {
    int n = 0;
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
    cache[dev] = n > 0 ? n : 148;
  }
  return cache[dev];
}

// 4D map over a pair tensor [B, R, N, 128] (fp32): dims (c, j, r, b), box (32, 128, 1, 1),
// 128-B swizzle. `transposed` walks z[b, j, r] instead (the ending-node view).
int make_pair_map(CUtensorMap* m, const float* base, int64_t B, int64_t R, int64_t N, bool transposed) {
  const uint64_t row = 128 * 4;
  uint64_t dims[4] = {128, static_cast<uint64_t>(N), static_cast<uint64_t>(R), static_cast<uint64_t>(B)};
  uint64_t strides[3] = {row, row * N, row * N * R};
  if (transposed) {
    // pair (r, j) of the transposed problem is z[b, j, r]; requires R == N
    strides[0] = row * N;
    strides[1] = row;
  }
  uint32_t box[4] = {32, 128, 1, 1};
  return encode_tmap(m, TmaType::kF32, 4, base, dims, strides, box, 128);
}

// 4D map over a plane buffer [B, R, C, ld] (fp16): dims (col, c, r, b).
int make_plane_map(CUtensorMap* m, const void* base, int64_t B, int64_t R, int64_t C, int64_t cols, int64_t ld,
                   uint32_t box_col, uint32_t box_c, uint32_t box_r, int swizzle) {
  uint64_t dims[4] = {static_cast<uint64_t>(cols), static_cast<uint64_t>(C), static_cast<uint64_t>(R),
                      static_cast<uint64_t>(B)};
  uint64_t strides[3] = {static_cast<uint64_t>(ld) * 2, static_cast<uint64_t>(ld) * 2 * C,
                         static_cast<uint64_t>(ld) * 2 * C * R};
  uint32_t box[4] = {box_col, box_c, box_r, 1};
  return encode_tmap(m, TmaType::kF16, 4, base, dims, strides, box, swizzle);
}

int make_weight_map(CUtensorMap* m, const void* base, int64_t rows, uint32_t box_rows) {
  uint64_t dims[2] = {128, static_cast<uint64_t>(rows)};
  uint64_t strides[1] = {256};
  uint32_t box[2] = {64, box_rows};
  return encode_tmap(m, TmaType::kF16, 2, base, dims, strides, box, 128);
}

int check_ptr(const void* p, const char* name, uintptr_t align) {
  if (!p) return fail(GTK_ERR_INVALID_ARG, std::string(name) + " is NULL");
  if (reinterpret_cast<uintptr_t>(p) % align) return fail(GTK_ERR_ALIGNMENT, std::string(name) + " is misaligned");
  return GTK_OK;
}

bool dims_ok(int64_t v, int64_t max_v) { return v >= 1 && v <= max_v; }

}  // namespace gtk
