// Host-side TMA tensor-map encoding with a process-wide cache.
#include <cudaTypedefs.h>

#include <mutex>
#include <unordered_map>

#include "tma_host.h"

namespace cob {
namespace {

PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  });
  return fn;
}

struct MapKey {
  uint64_t ptr, rows, cols, row_bytes;
  uint32_t box_rows, box_cols, bf16;
  bool operator==(const MapKey& o) const {
    return ptr == o.ptr && rows == o.rows && cols == o.cols && row_bytes == o.row_bytes && box_rows == o.box_rows &&
           box_cols == o.box_cols && bf16 == o.bf16;
  }
};
struct MapHash {
  size_t operator()(const MapKey& k) const {
    size_t h = std::hash<uint64_t>()(k.ptr);
    h ^= std::hash<uint64_t>()(k.rows * 1000003ull + k.cols) + 0x9e3779b97f4a7c15ull + (h << 6) + (h >> 2);
    h ^= std::hash<uint64_t>()(k.row_bytes ^ ((uint64_t)k.box_rows << 32) ^ ((uint64_t)k.box_cols << 48) ^ k.bf16);
    return h;
  }
};

}  // namespace

cudaError_t tensor_map_2d(const void* ptr, uint64_t rows, uint64_t cols, uint64_t row_bytes, uint32_t box_rows,
                          uint32_t box_cols, bool bf16, CUtensorMap* out) {
  static std::mutex mu;
  static std::unordered_map<MapKey, CUtensorMap, MapHash> cache;
  const MapKey key{reinterpret_cast<uint64_t>(ptr), rows, cols, row_bytes, box_rows, box_cols, bf16 ? 1u : 0u};
  std::lock_guard<std::mutex> g(mu);
  auto it = cache.find(key);
  if (it != cache.end()) {
    *out = it->second;
    return cudaSuccess;
  }
  auto enc = encode_fn();
  if (!enc) return cudaErrorNotSupported;
  if ((reinterpret_cast<uintptr_t>(ptr) & 15) || row_bytes % 16 || box_cols * 2 != 128) return cudaErrorMisalignedAddress;
  CUtensorMap m;
  cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)row_bytes};
  cuuint32_t box[2] = {box_cols, box_rows};
  cuuint32_t estr[2] = {1, 1};
  const CUresult r = enc(&m, bf16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2,
                         const_cast<void*>(ptr), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                         CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                         CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return cudaErrorInvalidValue;
  if (cache.size() > 16384) cache.clear();
  cache.emplace(key, m);
  *out = m;
  return cudaSuccess;
}

}  // namespace cob
