// Host-side TMA tensor maps. The driver's encoder is fetched once through the runtime's entry-point
// query, so the library does not link libcuda directly. Encoded maps are cached by their full
// description: decode replays the same pointers every step, and weights never move.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>

#include <cstring>
#include <functional>
#include <mutex>
#include <unordered_map>

namespace es {
namespace tmap {

using EncodeFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                              const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                              CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

inline EncodeFn encoder() {
  static EncodeFn fn = [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    cudaError_t e = cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q);
    if (e != cudaSuccess || q != cudaDriverEntryPointSuccess) p = nullptr;
    return reinterpret_cast<EncodeFn>(p);
  }();
  return fn;
}

struct Key {
  uintptr_t ptr;
  int64_t rows, cols, ld;
  int box_rows, box_cols;
  bool operator==(const Key& o) const {
    return ptr == o.ptr && rows == o.rows && cols == o.cols && ld == o.ld && box_rows == o.box_rows &&
           box_cols == o.box_cols;
  }
};
struct KeyHash {
  size_t operator()(const Key& k) const {
    size_t h = std::hash<uintptr_t>()(k.ptr);
    h ^= std::hash<int64_t>()(k.rows) + 0x9e3779b97f4a7c15ull + (h << 6) + (h >> 2);
    h ^= std::hash<int64_t>()(k.cols) + 0x9e3779b97f4a7c15ull + (h << 6) + (h >> 2);
    h ^= std::hash<int64_t>()(k.ld * 131 + k.box_rows * 7 + k.box_cols) + (h << 6) + (h >> 2);
    return h;
  }
};

// A 2-D bf16 map over a row-major [rows, cols] matrix with row stride `ld` elements; the box is
// [box_rows, box_cols] with box_cols * 2 == 128 bytes, swizzled 128B. Out-of-range rows and
// columns read as zero.
inline cudaError_t bf16_2d(CUtensorMap* out, void* base, int64_t rows, int64_t cols, int64_t ld, int box_rows,
                           int box_cols) {
  static std::mutex mu;
  static std::unordered_map<Key, CUtensorMap, KeyHash> cache;
  const Key key{reinterpret_cast<uintptr_t>(base), rows, cols, ld, box_rows, box_cols};
  {
    std::lock_guard<std::mutex> g(mu);
    auto it = cache.find(key);
    if (it != cache.end()) {
      *out = it->second;
      return cudaSuccess;
    }
  }
  if (box_cols * 2 != 128 || reinterpret_cast<uintptr_t>(base) % 16 != 0 || (ld * 2) % 16 != 0)
    return cudaErrorInvalidValue;
  EncodeFn enc = encoder();
  if (enc == nullptr) return cudaErrorNotSupported;
  CUtensorMap m;
  std::memset(&m, 0, sizeof(m));
  const cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
  const cuuint64_t strides[1] = {(cuuint64_t)(ld * 2)};
  const cuuint32_t box[2] = {(cuuint32_t)box_cols, (cuuint32_t)box_rows};
  const cuuint32_t estr[2] = {1, 1};
  CUresult r = enc(&m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, base, dims, strides, box, estr,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return cudaErrorInvalidValue;
  std::lock_guard<std::mutex> g(mu);
  if (cache.size() > 65536) cache.clear();
  cache.emplace(key, m);
  *out = m;
  return cudaSuccess;
}

// A 2-D map of one-byte elements (fp8 tensors) over a row-major [rows, cols] matrix with row stride
// `ld` bytes; the box is [box_rows, box_cols] with box_cols == 128 (one 128-byte swizzle row),
// swizzled 128B. Not cached: callers encode it per launch (a few microseconds on the host).
inline cudaError_t u8_2d(CUtensorMap* out, void* base, int64_t rows, int64_t cols, int64_t ld, int box_rows,
                         int box_cols) {
  if (box_cols != 128 || reinterpret_cast<uintptr_t>(base) % 16 != 0 || ld % 16 != 0) return cudaErrorInvalidValue;
  EncodeFn enc = encoder();
  if (enc == nullptr) return cudaErrorNotSupported;
  std::memset(out, 0, sizeof(*out));
  const cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
  const cuuint64_t strides[1] = {(cuuint64_t)ld};
  const cuuint32_t box[2] = {(cuuint32_t)box_cols, (cuuint32_t)box_rows};
  const cuuint32_t estr[2] = {1, 1};
  CUresult r = enc(out, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, base, dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                   CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? cudaSuccess : cudaErrorInvalidValue;
}

}  // namespace tmap
}  // namespace es
