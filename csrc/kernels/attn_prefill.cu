// Paged, causal, varlen GQA prefill attention (flash style) for sm_100a.
//
// A CTA owns 64 query rows = (64/G tokens) x (G query heads of one KV head), so every K/V tile
// fetched from the page pool serves the whole GQA group. K/V tiles of 64 keys (4 pages) are
// double-buffered in XOR-swizzled shared memory with cp.async; S = Q K^T and O += P V use the
// m16n8k16 bf16 tensor-core fragments with an online exp2 softmax kept in registers. Query i of a
// sequence with q_len new tokens and k_len total keys sits at key position k_len - q_len + i, so
// chunked prefill over a cached prefix works unchanged. An optional sliding window restricts
// keys to the last `window` positions (the reference's 4096-token compat window).
//
// Replaces the reference's explicit [heads, T, S] score tensor, host-built causal mask and
// softmax (forward_pass.rs:1096-1125, :2811-2835).
#include <ATen/ATen.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/extension.h>

#include "../include/sm100.cuh"
#include "../include/launch.h"

namespace mesh {

struct PrefillArgs {
  const __nv_bfloat16* q;   // [Tq, hq*D]
  const __nv_bfloat16* k;   // [pages, hkv, ps, D]
  const __nv_bfloat16* v;
  __nv_bfloat16* out;       // [Tq, hq*D]
  const int* cu_q;          // [S+1]
  const int* k_lens;        // [S]
  const int* block_tables;  // [S, max_pages]
  int max_pages, hkv, page_size;
  float scale_log2;
  int window;
};

constexpr int PF_ROWS = 64;
constexpr int PF_KEYS = 64;
constexpr int PF_D = 128;
constexpr int PF_CHUNKS = PF_D / 8;  // 16-byte chunks per row

__device__ __forceinline__ uint32_t swz(int row, int chunk) {
  return (uint32_t)(row * (PF_D * 2) + ((chunk ^ (row & 7)) << 4));
}

__device__ __forceinline__ void cp_async16(uint32_t dst, const void* src, int src_bytes) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst), "l"(src), "r"(src_bytes) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}
__device__ __forceinline__ void mma_bf16(float (&c)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

template <int G>
__global__ void __launch_bounds__(128) attn_prefill_kernel(const PrefillArgs a) {
  constexpr int BQ = PF_ROWS / G;
  extern __shared__ __align__(128) uint8_t smem[];
  griddep_wait();
  griddep_launch_dependents();
  uint8_t* q_sm = smem;
  uint8_t* k_sm = smem + PF_ROWS * PF_D * 2;              // 2 buffers
  uint8_t* v_sm = k_sm + 2 * PF_KEYS * PF_D * 2;          // 2 buffers
  const uint32_t q_base = smem_u32(q_sm), k_base = smem_u32(k_sm), v_base = smem_u32(v_sm);
  constexpr uint32_t KV_TILE = PF_KEYS * PF_D * 2;

  const int seq = blockIdx.z, h = blockIdx.y;
  const int q0 = a.cu_q[seq];
  const int qlen = a.cu_q[seq + 1] - q0;
  const int tok0 = blockIdx.x * BQ;
  if (tok0 >= qlen) return;
  const int klen = a.k_lens[seq];
  const int hq = a.hkv * G;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int pos_base = klen - qlen;  // key position of query token 0

  // ---- Q tile -> smem ----
  for (int i = threadIdx.x; i < PF_ROWS * PF_CHUNKS; i += 128) {
    const int r = i / PF_CHUNKS, c = i - r * PF_CHUNKS;
    const int tok = tok0 + r / G, g = r % G;
    const bool ok = tok < qlen;
    const __nv_bfloat16* src = a.q + (long)(q0 + (ok ? tok : 0)) * hq * PF_D + (h * G + g) * PF_D + c * 8;
    cp_async16(q_base + swz(r, c), src, ok ? 16 : 0);
  }
  cp_async_commit();

  const int last_tok = min(tok0 + BQ, qlen) - 1;
  const int kmax = min(klen, pos_base + last_tok + 1);
  int kmin = 0;
  if (a.window > 0) kmin = max(0, pos_base + tok0 - a.window + 1);
  const int kb_first = kmin / PF_KEYS;
  const int kb_last = (kmax - 1) / PF_KEYS;
  const int* bt = a.block_tables + (long)seq * a.max_pages;
  const long head_stride = (long)a.page_size * PF_D;
  const long page_stride = (long)a.hkv * head_stride;

  auto load_kv = [&](int kb, int buf) {
    for (int i = threadIdx.x; i < PF_KEYS * PF_CHUNKS; i += 128) {
      const int r = i / PF_CHUNKS, c = i - r * PF_CHUNKS;
      const int key = kb * PF_KEYS + r;
      const bool ok = key < klen;
      long off = 0;
      if (ok) {
        const int page = bt[key / a.page_size];
        off = (long)page * page_stride + h * head_stride + (long)(key % a.page_size) * PF_D + c * 8;
      }
      cp_async16(k_base + buf * KV_TILE + swz(r, c), a.k + off, ok ? 16 : 0);
      cp_async16(v_base + buf * KV_TILE + swz(r, c), a.v + off, ok ? 16 : 0);
    }
    cp_async_commit();
  };

  load_kv(kb_first, 0);
  cp_async_wait<1>();  // Q landed
  __syncthreads();

  // Q fragments for this warp's 16 rows, all 8 k-steps of D=128
  uint32_t qf[8][4];
  {
    const int r = warp * 16 + (lane & 15);
#pragma unroll
    for (int kk = 0; kk < 8; ++kk) {
      const int c = kk * 2 + (lane >> 4);
      ldsm_x4(q_base + swz(r, c), qf[kk][0], qf[kk][1], qf[kk][2], qf[kk][3]);
    }
  }
  // per-thread rows: r0 = warp*16 + lane/4, r1 = r0 + 8
  const int rr0 = warp * 16 + (lane >> 2), rr1 = rr0 + 8;
  const int qpos0 = pos_base + tok0 + rr0 / G, qpos1 = pos_base + tok0 + rr1 / G;
  const bool rv0 = tok0 + rr0 / G < qlen, rv1 = tok0 + rr1 / G < qlen;

  float o[16][4];
#pragma unroll
  for (int n = 0; n < 16; ++n) o[n][0] = o[n][1] = o[n][2] = o[n][3] = 0.f;
  float m0 = -INFINITY, m1 = -INFINITY, l0 = 0.f, l1 = 0.f;

  for (int kb = kb_first; kb <= kb_last; ++kb) {
    const int buf = (kb - kb_first) & 1;
    if (kb < kb_last) {
      load_kv(kb + 1, buf ^ 1);
      cp_async_wait<1>();
    } else {
      cp_async_wait<0>();
    }
    __syncthreads();
    const uint32_t kt = k_base + buf * KV_TILE, vt = v_base + buf * KV_TILE;

    // S = Q K^T : 16 x 64 per warp
    float s[8][4];
#pragma unroll
    for (int n = 0; n < 8; ++n) s[n][0] = s[n][1] = s[n][2] = s[n][3] = 0.f;
#pragma unroll
    for (int n = 0; n < 8; ++n) {
#pragma unroll
      for (int kk = 0; kk < 8; kk += 2) {
        uint32_t b0, b1, b2, b3;
        const int r = n * 8 + (lane & 7);
        const int c = kk * 2 + (lane >> 3);
        ldsm_x4(kt + swz(r, c), b0, b1, b2, b3);
        mma_bf16(s[n], qf[kk], b0, b1);
        mma_bf16(s[n], qf[kk + 1], b2, b3);
      }
    }
    // mask + online softmax (exp2 domain)
    const int key_base = kb * PF_KEYS;
    float mx0 = -INFINITY, mx1 = -INFINITY;
#pragma unroll
    for (int n = 0; n < 8; ++n) {
#pragma unroll
      for (int j = 0; j < 2; ++j) {
        const int key = key_base + n * 8 + (lane & 3) * 2 + j;
        const bool kv = key < klen;
        bool ok0 = rv0 && kv && key <= qpos0 && (a.window <= 0 || key > qpos0 - a.window);
        bool ok1 = rv1 && kv && key <= qpos1 && (a.window <= 0 || key > qpos1 - a.window);
        s[n][j] = ok0 ? s[n][j] * a.scale_log2 : -INFINITY;
        s[n][2 + j] = ok1 ? s[n][2 + j] * a.scale_log2 : -INFINITY;
        mx0 = fmaxf(mx0, s[n][j]);
        mx1 = fmaxf(mx1, s[n][2 + j]);
      }
    }
#pragma unroll
    for (int off = 1; off <= 2; off <<= 1) {
      mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, off));
      mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, off));
    }
    const float mn0 = fmaxf(m0, mx0), mn1 = fmaxf(m1, mx1);
    const float c0 = (mn0 == -INFINITY) ? 1.f : exp2f(m0 - mn0);
    const float c1 = (mn1 == -INFINITY) ? 1.f : exp2f(m1 - mn1);
    float ps0 = 0.f, ps1 = 0.f;
    uint32_t pf[4][4];
#pragma unroll
    for (int n = 0; n < 8; ++n) {
      const float p00 = (mn0 == -INFINITY) ? 0.f : exp2f(s[n][0] - mn0);
      const float p01 = (mn0 == -INFINITY) ? 0.f : exp2f(s[n][1] - mn0);
      const float p10 = (mn1 == -INFINITY) ? 0.f : exp2f(s[n][2] - mn1);
      const float p11 = (mn1 == -INFINITY) ? 0.f : exp2f(s[n][3] - mn1);
      ps0 += p00 + p01;
      ps1 += p10 + p11;
      const int kk = n >> 1, hi = n & 1;
      pf[kk][hi * 2 + 0] = pack_bf16x2(p00, p01);
      pf[kk][hi * 2 + 1] = pack_bf16x2(p10, p11);
    }
    l0 = l0 * c0 + ps0;
    l1 = l1 * c1 + ps1;
    m0 = mn0;
    m1 = mn1;
#pragma unroll
    for (int n = 0; n < 16; ++n) {
      o[n][0] *= c0;
      o[n][1] *= c0;
      o[n][2] *= c1;
      o[n][3] *= c1;
    }
    // O += P V : A = P (16 x 64), B = V (64 keys x 128 d) via transposed ldmatrix
#pragma unroll
    for (int kk = 0; kk < 4; ++kk) {
#pragma unroll
      for (int n = 0; n < 16; n += 2) {
        uint32_t b0, b1, b2, b3;
        const int r = kk * 16 + (lane & 7) + ((lane >> 3) & 1) * 8;
        const int c = n + (lane >> 4);
        ldsm_x4_t(vt + swz(r, c), b0, b1, b2, b3);
        mma_bf16(o[n], pf[kk], b0, b1);
        mma_bf16(o[n + 1], pf[kk], b2, b3);
      }
    }
    __syncthreads();  // buffer reuse by the next prefetch
  }

  // finalise: sum l across the 4 lanes of a row, write bf16
#pragma unroll
  for (int off = 1; off <= 2; off <<= 1) {
    l0 += __shfl_xor_sync(0xffffffffu, l0, off);
    l1 += __shfl_xor_sync(0xffffffffu, l1, off);
  }
  const float inv0 = l0 > 0.f ? 1.f / l0 : 0.f, inv1 = l1 > 0.f ? 1.f / l1 : 0.f;
  if (rv0) {
    const int tok = tok0 + rr0 / G, g = rr0 % G;
    __nv_bfloat16* dst = a.out + (long)(q0 + tok) * hq * PF_D + (h * G + g) * PF_D;
#pragma unroll
    for (int n = 0; n < 16; ++n)
      *reinterpret_cast<uint32_t*>(dst + n * 8 + (lane & 3) * 2) = pack_bf16x2(o[n][0] * inv0, o[n][1] * inv0);
  }
  if (rv1) {
    const int tok = tok0 + rr1 / G, g = rr1 % G;
    __nv_bfloat16* dst = a.out + (long)(q0 + tok) * hq * PF_D + (h * G + g) * PF_D;
#pragma unroll
    for (int n = 0; n < 16; ++n)
      *reinterpret_cast<uint32_t*>(dst + n * 8 + (lane & 3) * 2) = pack_bf16x2(o[n][2] * inv1, o[n][3] * inv1);
  }
}

void attn_prefill(const at::Tensor& q, const at::Tensor& kcache, const at::Tensor& vcache, const at::Tensor& cu_q,
                  const at::Tensor& k_lens, const at::Tensor& block_tables, at::Tensor& out, int64_t max_q_len,
                  double scale, int64_t window) {
  TORCH_CHECK(q.scalar_type() == at::kBFloat16 && q.is_contiguous(), "attn_prefill: q bf16 [T, hq*D]");
  TORCH_CHECK(kcache.dim() == 4 && kcache.size(3) == PF_D, "attn_prefill: head_dim 128 only");
  TORCH_CHECK(cu_q.scalar_type() == at::kInt && k_lens.scalar_type() == at::kInt &&
                  block_tables.scalar_type() == at::kInt,
              "attn_prefill: int32 metadata");
  const int S = k_lens.size(0);
  const int hkv = kcache.size(1);
  const int hq = q.size(1) / PF_D;
  const int G = hq / hkv;
  TORCH_CHECK(G == 1 || G == 2 || G == 4 || G == 8, "attn_prefill: group size 1/2/4/8");
  if (S == 0 || max_q_len == 0) return;
  const c10::cuda::CUDAGuard guard(q.device());
  PrefillArgs a;
  a.q = reinterpret_cast<const __nv_bfloat16*>(q.data_ptr());
  a.k = reinterpret_cast<const __nv_bfloat16*>(kcache.data_ptr());
  a.v = reinterpret_cast<const __nv_bfloat16*>(vcache.data_ptr());
  a.out = reinterpret_cast<__nv_bfloat16*>(out.data_ptr());
  a.cu_q = cu_q.data_ptr<int>();
  a.k_lens = k_lens.data_ptr<int>();
  a.block_tables = block_tables.data_ptr<int>();
  a.max_pages = block_tables.size(1);
  a.hkv = hkv;
  a.page_size = kcache.size(2);
  a.scale_log2 = (float)(scale * 1.4426950408889634);
  a.window = (int)window;
  const int BQ = PF_ROWS / G;
  dim3 grid((max_q_len + BQ - 1) / BQ, hkv, S);
  const size_t smem = (PF_ROWS + 4 * PF_KEYS) * PF_D * 2;
  cudaStream_t st = at::cuda::getCurrentCUDAStream();
  auto go = [&](auto kern) {
    cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    launch_k(kern, grid, dim3(128), smem, st, a);
  };
  switch (G) {
    case 1: go(attn_prefill_kernel<1>); break;
    case 2: go(attn_prefill_kernel<2>); break;
    case 4: go(attn_prefill_kernel<4>); break;
    default: go(attn_prefill_kernel<8>); break;
  }
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

}  // namespace mesh
