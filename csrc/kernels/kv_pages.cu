// Session KV handoff: gather a session's pages of every layer out of the paged pool into one
// contiguous buffer, and scatter such a buffer into freshly allocated pages of another pool.
//
// Pool layout [layers, pages, kv_heads, page_size, head_dim] bf16 (K and V pools alike); one page of
// one layer is kv_heads * page_size * head_dim contiguous elements, so the buffer keeps that block as
// the unit: buffer [2 (K, V), layers, n_pages, page_elems]. The buffer can then travel to another GPU
// with one peer copy (NVLink) and be scattered there; block tables only need the new page ids.
// The reference moves a session by serialising its host fp32 KVCache into a CBOR checkpoint and
// rebuilding it on the receiver (agent/src/inference/coordinator.rs:1916-1957,
// agent/src/main.rs:2898-3037); here the pages never leave device memory.
#include <ATen/ATen.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/extension.h>

#include "../include/sm100.cuh"

namespace mesh {

// grid (pages, layers, 2): one CTA copies one page block of one layer of K or V, 16 bytes per thread
// step. to_buf: pool -> buffer, else buffer -> pool.
__global__ void __launch_bounds__(256) kv_pages_copy_kernel(uint4* __restrict__ k_pool, uint4* __restrict__ v_pool,
                                                            uint4* __restrict__ buf, const int* __restrict__ pages,
                                                            long pool_pages, int n_pages, long page_vec, bool to_buf) {
  const int p = blockIdx.x, layer = blockIdx.y, which = blockIdx.z;
  uint4* pool = which == 0 ? k_pool : v_pool;
  const long src_page = pages[p];
  uint4* pp = pool + ((long)layer * pool_pages + src_page) * page_vec;
  uint4* bp = buf + (((long)which * gridDim.y + layer) * n_pages + p) * page_vec;
  if (to_buf) {
    for (long i = threadIdx.x; i < page_vec; i += blockDim.x) bp[i] = __ldcs(pp + i);
  } else {
    for (long i = threadIdx.x; i < page_vec; i += blockDim.x) pp[i] = bp[i];
  }
}

// Copies between a pool pair and buf [2, layers, len(pages), page_elems]; pages int32 on the device.
void kv_pages_copy(at::Tensor& k_pool, at::Tensor& v_pool, at::Tensor& buf, const at::Tensor& pages, bool to_buf) {
  TORCH_CHECK(k_pool.dim() == 5 && k_pool.sizes() == v_pool.sizes() && k_pool.is_contiguous() && v_pool.is_contiguous(),
              "kv_pages_copy: pools [layers, pages, kv_heads, page, D]");
  TORCH_CHECK(k_pool.scalar_type() == at::kBFloat16 && v_pool.scalar_type() == at::kBFloat16 &&
                  buf.scalar_type() == at::kBFloat16 && buf.is_contiguous(),
              "kv_pages_copy: bf16 pools and buffer");
  TORCH_CHECK(pages.scalar_type() == at::kInt && pages.is_cuda() && pages.dim() == 1, "kv_pages_copy: int32 page ids");
  const int L = k_pool.size(0);
  const long pool_pages = k_pool.size(1);
  const long page_elems = k_pool.size(2) * k_pool.size(3) * k_pool.size(4);
  TORCH_CHECK(page_elems % 8 == 0, "kv_pages_copy: page block must be a multiple of 16 bytes");
  const int n = pages.size(0);
  TORCH_CHECK(buf.numel() == 2L * L * n * page_elems, "kv_pages_copy: buffer must be [2, layers, pages, page_elems]");
  if (n == 0) return;
  const c10::cuda::CUDAGuard guard(k_pool.device());
  dim3 grid(n, L, 2);
  kv_pages_copy_kernel<<<grid, 256, 0, at::cuda::getCurrentCUDAStream()>>>(
      reinterpret_cast<uint4*>(k_pool.data_ptr()), reinterpret_cast<uint4*>(v_pool.data_ptr()),
      reinterpret_cast<uint4*>(buf.data_ptr()), pages.data_ptr<int>(), pool_pages, n, page_elems / 8, to_buf);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

}  // namespace mesh
