// Allocation-free C entry point for split-KV paged decode attention (see mesh_noalloc.h).
//
// Declaration: this entry point has no counterpart in the reference project; it is an addition
// of this library for callers that cannot allocate device memory (see the header).
//
// It runs the same kernels as the PyTorch op (attn_decode_kernel + attn_decode_combine_kernel);
// the only difference is where the split-KV scratch lives: a file-scope device array instead of
// a buffer from the caching allocator. No cudaMalloc, cudaFree or allocating library call is
// made here.
#include <cuda_runtime.h>

#include <mutex>

#include "../kernels/attn_decode.cuh"
#include "mesh_noalloc.h"

namespace {

static __device__ __align__(256) float g_noalloc_scratch[MESH_NOALLOC_SCRATCH_FLOATS];

constexpr int kMaxDevices = 64;
float* g_scratch_addr[kMaxDevices] = {nullptr};  // device address of g_noalloc_scratch, per device
std::mutex g_setup_mu;

// In host code `g_noalloc_scratch` names a host-side stand-in, not device memory: the device
// address has to be looked up once per device, with that device current.
float* scratch_for_current_device(int* status) {
  int dev = -1;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) {
    *status = MESH_NOALLOC_ERR_SETUP;
    return nullptr;
  }
  std::lock_guard<std::mutex> lk(g_setup_mu);
  if (g_scratch_addr[dev] == nullptr) {
    void* p = nullptr;
    cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess || p == nullptr) {
      *status = MESH_NOALLOC_ERR_SETUP;
      return nullptr;
    }
    g_scratch_addr[dev] = static_cast<float*>(p);
  }
  return g_scratch_addr[dev];
}

}  // namespace

extern "C" __attribute__((visibility("default"))) int mesh_attn_decode_noalloc(
    const void* q, const void* k_cache, const void* v_cache, const int* block_tables, const int* seq_lens,
    void* out, int B, int num_q_heads, int num_kv_heads, int head_dim, int page_size, int max_pages_per_seq,
    int splits, float scale, int window, void* stream) {
  if (!q || !k_cache || !v_cache || !block_tables || !seq_lens || !out) return MESH_NOALLOC_ERR_ARGUMENT;
  if (B <= 0 || num_kv_heads <= 0 || num_q_heads <= 0 || num_q_heads % num_kv_heads != 0)
    return MESH_NOALLOC_ERR_ARGUMENT;
  const int G = num_q_heads / num_kv_heads;
  if (!(G == 1 || G == 2 || G == 4 || G == 8)) return MESH_NOALLOC_ERR_ARGUMENT;
  if (!(head_dim == 64 || head_dim == 128) || page_size <= 0 || max_pages_per_seq <= 0 || splits < 1 || window < 0)
    return MESH_NOALLOC_ERR_ARGUMENT;
  const unsigned long long need =
      (unsigned long long)B * num_q_heads * (unsigned long long)splits * (unsigned long long)(head_dim + 1);
  if (splits > 1 && need > MESH_NOALLOC_SCRATCH_FLOATS) return MESH_NOALLOC_ERR_TOO_LARGE;

  int status = MESH_NOALLOC_OK;
  float* scratch = scratch_for_current_device(&status);
  if (!scratch) return status;

  mesh::DecodeArgs a;
  a.q = static_cast<const __nv_bfloat16*>(q);
  a.k = static_cast<const __nv_bfloat16*>(k_cache);
  a.v = static_cast<const __nv_bfloat16*>(v_cache);
  a.block_tables = block_tables;
  a.seq_lens = seq_lens;
  a.out = static_cast<__nv_bfloat16*>(out);
  a.ws = scratch;
  a.max_pages = max_pages_per_seq;
  a.hkv = num_kv_heads;
  a.page_size = page_size;
  a.splits = splits;
  a.scale_log2 = scale * 1.4426950408889634f;
  a.window = window;
  // Only this call's own launches are checked (their return codes); an error that some earlier,
  // unrelated launch left pending is neither reported as this call's failure nor cleared here.
  if (mesh::launch_attn_decode(a, B, G, head_dim, static_cast<cudaStream_t>(stream)) != cudaSuccess)
    return MESH_NOALLOC_ERR_LAUNCH;
  return MESH_NOALLOC_OK;
}
