// Library-wide C ABI pieces: version, status strings, the device status
// word, and host helpers (SM count, TMA descriptor encoding, env overrides).
#include <cstdlib>
#include <cstring>
#include <mutex>

#include "common.cuh"
#include "internal.h"

namespace {

__device__ int32_t g_status[4];

constexpr int kMaxDevices = 64;

struct MapKey {
  const void* base;
  uint64_t rows, cols, ld;
  uint32_t box_rows;
  int device;
  bool operator==(const MapKey& o) const {
    return base == o.base && rows == o.rows && cols == o.cols && ld == o.ld && box_rows == o.box_rows &&
           device == o.device;
  }
};

constexpr int kMapCache = 256;
struct MapEntry {
  MapKey key;
  CUtensorMap map;
  bool used;
};
MapEntry g_maps[kMapCache];
int g_map_next = 0;
std::mutex g_map_mu;

typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = []() -> EncodeTiledFn {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) != cudaSuccess ||
        q != cudaDriverEntryPointSuccess)
      return nullptr;
    return reinterpret_cast<EncodeTiledFn>(p);
  }();
  return fn;
}

}  // namespace

namespace fdllm {

int32_t* status_ptr() {
  static int32_t* cache[kMaxDevices] = {nullptr};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return nullptr;
  if (cache[dev] == nullptr) {
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_status) != cudaSuccess) return nullptr;
    cache[dev] = static_cast<int32_t*>(p);
  }
  return cache[dev];
}

int sm_count() {
  static int cache[kMaxDevices] = {0};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return 148;
  if (cache[dev] == 0) {
    int n = 0;
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
    cache[dev] = n > 0 ? n : 148;
  }
  return cache[dev];
}

int env_int(const char* name, int dflt) {
  const char* v = std::getenv(name);
  if (v == nullptr || *v == 0) return dflt;
  return std::atoi(v);
}

int make_tmap_bf16_sw128(CUtensorMap* out, const void* base, uint64_t rows, uint64_t cols, uint64_t ld,
                         uint32_t box_rows) {
  int dev = 0;
  cudaGetDevice(&dev);
  MapKey key{base, rows, cols, ld, box_rows, dev};
  std::lock_guard<std::mutex> lock(g_map_mu);
  for (int i = 0; i < kMapCache; ++i) {
    if (g_maps[i].used && g_maps[i].key == key) {
      *out = g_maps[i].map;
      return FDLLM_OK;
    }
  }
  EncodeTiledFn fn = encode_fn();
  if (fn == nullptr) return FDLLM_ERR_DRIVER;
  if (!aligned16(base) || (ld * 2) % 16 != 0 || box_rows == 0 || box_rows > 256) return FDLLM_ERR_ARG;
  cuuint64_t dims[2] = {cols, rows};
  cuuint64_t strides[1] = {ld * 2};
  cuuint32_t box[2] = {64, box_rows};
  cuuint32_t estr[2] = {1, 1};
  CUtensorMap m;
  CUresult r = fn(&m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return FDLLM_ERR_DRIVER;
  g_maps[g_map_next] = MapEntry{key, m, true};
  g_map_next = (g_map_next + 1) % kMapCache;
  *out = m;
  return FDLLM_OK;
}

}  // namespace fdllm

extern "C" {

const char* fdllm_version(void) { return "flashdllm_b200 0.1.0 (sm_100a)"; }

const char* fdllm_error_string(int code) {
  switch (code) {
    case FDLLM_OK: return "ok";
    case FDLLM_ERR_ARG: return "invalid argument";
    case FDLLM_ERR_CUDA: return "CUDA runtime error";
    case FDLLM_ERR_INDEX: return "index out of range (device)";
    case FDLLM_ERR_TIMEOUT: return "bounded wait timed out (device)";
    case FDLLM_ERR_TABLE: return "malformed block table (device)";
    case FDLLM_ERR_WORKSPACE: return "workspace too small";
    case FDLLM_ERR_DRIVER: return "TMA descriptor encode failed";
    case FDLLM_ERR_SCRATCH_LIMIT: return "request exceeds the fixed scratch of the no-allocation entry point";
    case FDLLM_ERR_RANGE: return "attention-score column sum out of range (device)";
    default: return "unknown status";
  }
}

int fdllm_status_read(int32_t out[4], cudaStream_t stream) {
  int32_t* d = fdllm::status_ptr();
  if (d == nullptr || out == nullptr) return FDLLM_ERR_CUDA;
  if (cudaMemcpyAsync(out, d, 4 * sizeof(int32_t), cudaMemcpyDeviceToHost, stream) != cudaSuccess)
    return FDLLM_ERR_CUDA;
  if (cudaStreamSynchronize(stream) != cudaSuccess) return FDLLM_ERR_CUDA;
  if (cudaMemsetAsync(d, 0, 4 * sizeof(int32_t), stream) != cudaSuccess) return FDLLM_ERR_CUDA;
  return FDLLM_OK;
}

}  // extern "C"
