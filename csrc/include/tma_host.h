// Host-side creation of TMA tensor maps (cuTensorMapEncodeTiled through the runtime's driver
// entry point, so no link against libcuda is needed). Maps are cached by (address, shape, box).
#pragma once
#include <cuda.h>
#include <cuda_runtime.h>

#include <cstdint>
#include <cstring>
#include <mutex>
#include <stdexcept>
#include <string>
#include <unordered_map>

namespace mesh {

using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                   const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                   CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

inline EncodeTiledFn get_encode_fn() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    cudaError_t e = cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q);
    if (e != cudaSuccess || q != cudaDriverEntryPointSuccess || !p)
      throw std::runtime_error("mesh: cuTensorMapEncodeTiled entry point unavailable");
    fn = reinterpret_cast<EncodeTiledFn>(p);
  });
  return fn;
}

struct TmaKey {
  uint64_t addr, inner, outer, pitch;
  uint32_t box_inner, box_outer, swz;
  bool operator==(const TmaKey& o) const {
    return addr == o.addr && inner == o.inner && outer == o.outer && pitch == o.pitch &&
           box_inner == o.box_inner && box_outer == o.box_outer && swz == o.swz;
  }
};
struct TmaKeyHash {
  size_t operator()(const TmaKey& k) const {
    uint64_t h = k.addr * 0x9E3779B97F4A7C15ull;
    h ^= k.inner + 0x632BE59BD9B4E019ull + (h << 6) + (h >> 2);
    h ^= k.outer + (h << 6) + (h >> 2);
    h ^= k.pitch + (h << 6) + (h >> 2);
    h ^= ((uint64_t)k.box_inner << 32 | k.box_outer) + (h << 6) + (h >> 2);
    h ^= k.swz;
    return (size_t)h;
  }
};

// 2D bf16 tensor [outer, inner] with row pitch `pitch_elems`; box [box_outer, box_inner];
// 128-byte swizzle (box_inner * 2 must be 128) unless swizzle128 is false.
inline CUtensorMap tma_map_2d_bf16(const void* base, uint64_t inner, uint64_t outer, uint64_t pitch_elems,
                                   uint32_t box_inner, uint32_t box_outer, bool swizzle128 = true) {
  static std::mutex mu;
  static std::unordered_map<TmaKey, CUtensorMap, TmaKeyHash> cache;
  TmaKey key{(uint64_t)(uintptr_t)base, inner, outer, pitch_elems, box_inner, box_outer, swizzle128 ? 1u : 0u};
  {
    std::lock_guard<std::mutex> lk(mu);
    auto it = cache.find(key);
    if (it != cache.end()) return it->second;
  }
  if (((uintptr_t)base) % 16 != 0) throw std::runtime_error("mesh: TMA base address must be 16-byte aligned");
  if ((pitch_elems * 2) % 16 != 0) throw std::runtime_error("mesh: TMA row pitch must be a multiple of 16 bytes");
  CUtensorMap map;
  std::memset(&map, 0, sizeof(map));
  cuuint64_t dims[2] = {inner, outer};
  cuuint64_t strides[1] = {pitch_elems * 2};
  cuuint32_t box[2] = {box_inner, box_outer};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = get_encode_fn()(&map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides, box,
                               estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                               swizzle128 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_NONE,
                               CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS)
    throw std::runtime_error("mesh: cuTensorMapEncodeTiled failed with code " + std::to_string((int)r));
  std::lock_guard<std::mutex> lk(mu);
  if (cache.size() > 4096) cache.clear();
  cache.emplace(key, map);
  return map;
}

// 3D bf16 tensor: dims {d0, d1, d2} (d0 contiguous), byte strides of dims 1 and 2, box {b0, b1, b2};
// 128-byte swizzle (b0 * 2 must be 128). Cached like the 2D maps.
inline CUtensorMap tma_map_3d_bf16(const void* base, uint64_t d0, uint64_t d1, uint64_t d2, uint64_t stride1_bytes,
                                   uint64_t stride2_bytes, uint32_t b0, uint32_t b1, uint32_t b2) {
  struct Key {
    uint64_t v[8];
    bool operator==(const Key& o) const { return std::memcmp(v, o.v, sizeof(v)) == 0; }
  };
  struct Hash {
    size_t operator()(const Key& k) const {
      uint64_t h = 0x9E3779B97F4A7C15ull;
      for (uint64_t x : k.v) h ^= x + 0x632BE59BD9B4E019ull + (h << 6) + (h >> 2);
      return (size_t)h;
    }
  };
  static std::mutex mu;
  static std::unordered_map<Key, CUtensorMap, Hash> cache;
  Key key{{(uint64_t)(uintptr_t)base, d0, d1, d2, stride1_bytes, stride2_bytes, ((uint64_t)b0 << 32) | b1, b2}};
  {
    std::lock_guard<std::mutex> lk(mu);
    auto it = cache.find(key);
    if (it != cache.end()) return it->second;
  }
  if (((uintptr_t)base) % 16 != 0) throw std::runtime_error("mesh: TMA base address must be 16-byte aligned");
  if (stride1_bytes % 16 != 0 || stride2_bytes % 16 != 0)
    throw std::runtime_error("mesh: TMA strides must be multiples of 16 bytes");
  CUtensorMap map;
  std::memset(&map, 0, sizeof(map));
  cuuint64_t dims[3] = {d0, d1, d2};
  cuuint64_t strides[2] = {stride1_bytes, stride2_bytes};
  cuuint32_t box[3] = {b0, b1, b2};
  cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = get_encode_fn()(&map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void*>(base), dims, strides, box,
                               estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                               CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS)
    throw std::runtime_error("mesh: cuTensorMapEncodeTiled (3d) failed with code " + std::to_string((int)r));
  std::lock_guard<std::mutex> lk(mu);
  if (cache.size() > 4096) cache.clear();
  cache.emplace(key, map);
  return map;
}

}  // namespace mesh
