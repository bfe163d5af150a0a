// Memory-bound kernels of the decoder step (sm_100a):
//  * rmsnorm / add_rmsnorm: residual add fused with RMSNorm (fp32 math, bf16 I/O);
//  * rope_kv_write: half-split RoPE on q and k from a cos/sin table, q written out, k/v written
//    straight into the paged KV pool [pages, kv_heads, page_size, head_dim] via a slot mapping;
//  * embedding gather;
//  * argmax over local vocab logits (fp32) returning (max, index) pairs for the cross-rank merge.
// Reference ops restated: rms_norm (tensor_ops.rs:285), apply_rope (tensor_ops.rs:509-560),
// embed_tokens (tensor_ops.rs:482), sample_greedy (tensor_ops.rs:461), KV append
// (forward_pass.rs:462-521, here a direct page write instead of slice_assign + cat).
#include <ATen/ATen.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/extension.h>

#include "../include/sm100.cuh"
#include "../include/launch.h"

namespace mesh {

template <int NT>
__device__ __forceinline__ float block_sum(float v, float* red) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
  if (l == 0) red[w] = v;
  __syncthreads();
  float t = (threadIdx.x < NT / 32) ? red[threadIdx.x] : 0.f;
  if (w == 0) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) t += __shfl_xor_sync(0xffffffffu, t, o);
    if (l == 0) red[0] = t;
  }
  __syncthreads();
  float r = red[0];
  __syncthreads();
  return r;
}

// One CTA per row. If `delta` is non-null: resid += delta (in place, bf16) first.
// normed = resid * rsqrt(mean(resid^2) + eps) * gamma.
template <int NT>
__global__ void __launch_bounds__(NT) add_rmsnorm_kernel(const __nv_bfloat16* __restrict__ delta,
                                                         __nv_bfloat16* __restrict__ resid,
                                                         const __nv_bfloat16* __restrict__ gamma,
                                                         __nv_bfloat16* __restrict__ normed, int H, float eps) {
  griddep_wait();
  griddep_launch_dependents();
  __shared__ float red[32];
  const long row = blockIdx.x;
  const int nvec = H / 8;
  const uint4* dv = delta ? reinterpret_cast<const uint4*>(delta + row * H) : nullptr;
  uint4* rv = reinterpret_cast<uint4*>(resid + row * H);
  const uint4* gv = reinterpret_cast<const uint4*>(gamma);
  uint4* nv = reinterpret_cast<uint4*>(normed + row * H);
  constexpr int MAXV = 4;  // up to H = 8 * NT * MAXV
  float x[MAXV][8];
  float ss = 0.f;
#pragma unroll
  for (int i = 0; i < MAXV; ++i) {
    int v = threadIdx.x + i * NT;
    if (v < nvec) {
      uint4 r = rv[v];
      const uint32_t* ru = reinterpret_cast<const uint32_t*>(&r);
#pragma unroll
      for (int j = 0; j < 4; ++j) unpack_bf16x2(ru[j], x[i][2 * j], x[i][2 * j + 1]);
      if (dv) {
        uint4 d = dv[v];
        const uint32_t* du = reinterpret_cast<const uint32_t*>(&d);
        uint4 o;
        uint32_t* ou = reinterpret_cast<uint32_t*>(&o);
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          float a, b;
          unpack_bf16x2(du[j], a, b);
          x[i][2 * j] += a;
          x[i][2 * j + 1] += b;
          ou[j] = pack_bf16x2(x[i][2 * j], x[i][2 * j + 1]);
        }
        rv[v] = o;
        // normalise what was stored (bf16-rounded residual), as an unfused add then norm would
#pragma unroll
        for (int j = 0; j < 4; ++j) unpack_bf16x2(ou[j], x[i][2 * j], x[i][2 * j + 1]);
      }
#pragma unroll
      for (int j = 0; j < 8; ++j) ss += x[i][j] * x[i][j];
    }
  }
  const float tot = block_sum<NT>(ss, red);
  const float inv = rsqrtf(tot / (float)H + eps);
#pragma unroll
  for (int i = 0; i < MAXV; ++i) {
    int v = threadIdx.x + i * NT;
    if (v < nvec) {
      uint4 g = gv[v];
      const uint32_t* gu = reinterpret_cast<const uint32_t*>(&g);
      uint4 o;
      uint32_t* ou = reinterpret_cast<uint32_t*>(&o);
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        float g0, g1;
        unpack_bf16x2(gu[j], g0, g1);
        ou[j] = pack_bf16x2(x[i][2 * j] * inv * g0, x[i][2 * j + 1] * inv * g1);
      }
      nv[v] = o;
    }
  }
}

void add_rmsnorm(const c10::optional<at::Tensor>& delta, at::Tensor& resid, const at::Tensor& gamma, at::Tensor& normed,
                 double eps) {
  TORCH_CHECK(resid.is_cuda() && resid.scalar_type() == at::kBFloat16 && resid.is_contiguous(), "add_rmsnorm: resid");
  const int H = resid.size(-1);
  TORCH_CHECK(H % 8 == 0 && H <= 8 * 256 * 4, "add_rmsnorm: H must be a multiple of 8 and <= 8192");
  TORCH_CHECK(gamma.numel() == H && normed.sizes() == resid.sizes(), "add_rmsnorm: shapes");
  const long rows = resid.numel() / H;
  if (rows == 0) return;
  const c10::cuda::CUDAGuard guard(resid.device());
  const __nv_bfloat16* d = nullptr;
  if (delta.has_value()) {
    TORCH_CHECK(delta->sizes() == resid.sizes() && delta->is_contiguous(), "add_rmsnorm: delta");
    d = reinterpret_cast<const __nv_bfloat16*>(delta->data_ptr());
  }
  launch_k(add_rmsnorm_kernel<256>, dim3(rows), dim3(256), 0, at::cuda::getCurrentCUDAStream(), d,
           reinterpret_cast<__nv_bfloat16*>(resid.data_ptr()), reinterpret_cast<const __nv_bfloat16*>(gamma.data_ptr()),
           reinterpret_cast<__nv_bfloat16*>(normed.data_ptr()), H, (float)eps);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

// ----------------------------------------------------------------------------------------------
// RoPE + paged KV write. qkv: [T, (hq + 2*hkv) * D] bf16. cos/sin: [max_pos, D/2] fp32.
// q_out: [T, hq*D]. kcache/vcache: [pages, hkv, page_size, D]. slot: [T] int64 (page*ps + off), <0 skip.
// One CTA per token; each thread rotates 4-element pairs (lo half dims j..j+3 with hi j+D/2..).
// ----------------------------------------------------------------------------------------------
__global__ void rope_kv_write_kernel(const __nv_bfloat16* __restrict__ qkv, const int* __restrict__ pos,
                                     const long* __restrict__ slot, const float* __restrict__ cos_t,
                                     const float* __restrict__ sin_t, __nv_bfloat16* __restrict__ q_out,
                                     __nv_bfloat16* __restrict__ kcache, __nv_bfloat16* __restrict__ vcache, int hq,
                                     int hkv, int D, int page_size) {
  griddep_wait();
  griddep_launch_dependents();
  const long t = blockIdx.x;
  const int width = (hq + 2 * hkv) * D;
  const __nv_bfloat16* row = qkv + t * width;
  const int p = pos[t];
  const long s = slot[t];
  const int half = D / 2;
  const int quads = half / 4;                    // groups of 4 rotated pairs per head
  const int total_rot = (hq + hkv) * quads;
  const float* cr = cos_t + (long)p * half;
  const float* sr = sin_t + (long)p * half;
  for (int i = threadIdx.x; i < total_rot; i += blockDim.x) {
    const int head = i / quads, qd = (i - head * quads) * 4;
    const __nv_bfloat16* src = row + head * D;  // q heads then k heads are contiguous in qkv
    uint2 lo = *reinterpret_cast<const uint2*>(src + qd);
    uint2 hi = *reinterpret_cast<const uint2*>(src + half + qd);
    float l[4], h[4];
    unpack_bf16x2(lo.x, l[0], l[1]);
    unpack_bf16x2(lo.y, l[2], l[3]);
    unpack_bf16x2(hi.x, h[0], h[1]);
    unpack_bf16x2(hi.y, h[2], h[3]);
    float ol[4], oh[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      float c = cr[qd + j], sn = sr[qd + j];
      ol[j] = l[j] * c - h[j] * sn;
      oh[j] = l[j] * sn + h[j] * c;
    }
    uint2 olo = make_uint2(pack_bf16x2(ol[0], ol[1]), pack_bf16x2(ol[2], ol[3]));
    uint2 ohi = make_uint2(pack_bf16x2(oh[0], oh[1]), pack_bf16x2(oh[2], oh[3]));
    if (head < hq) {
      __nv_bfloat16* dst = q_out + t * (long)hq * D + head * D;
      *reinterpret_cast<uint2*>(dst + qd) = olo;
      *reinterpret_cast<uint2*>(dst + half + qd) = ohi;
    } else if (s >= 0) {
      const int kh = head - hq;
      const long page = s / page_size, off = s - page * page_size;
      __nv_bfloat16* dst = kcache + ((page * hkv + kh) * page_size + off) * D;
      *reinterpret_cast<uint2*>(dst + qd) = olo;
      *reinterpret_cast<uint2*>(dst + half + qd) = ohi;
    }
  }
  if (s >= 0) {
    const long page = s / page_size, off = s - page * page_size;
    const int vec = D / 8;
    for (int i = threadIdx.x; i < hkv * vec; i += blockDim.x) {
      const int kh = i / vec, c = (i - kh * vec) * 8;
      uint4 v = *reinterpret_cast<const uint4*>(row + (hq + hkv + kh) * D + c);
      *reinterpret_cast<uint4*>(vcache + ((page * hkv + kh) * page_size + off) * D + c) = v;
    }
  }
}

void rope_kv_write(const at::Tensor& qkv, const at::Tensor& pos, const at::Tensor& slot, const at::Tensor& cos_t,
                   const at::Tensor& sin_t, at::Tensor& q_out, at::Tensor& kcache, at::Tensor& vcache, int64_t hq,
                   int64_t hkv) {
  TORCH_CHECK(qkv.is_contiguous() && qkv.scalar_type() == at::kBFloat16, "rope_kv_write: qkv");
  TORCH_CHECK(pos.scalar_type() == at::kInt && slot.scalar_type() == at::kLong, "rope_kv_write: pos int32, slot int64");
  TORCH_CHECK(kcache.dim() == 4 && kcache.size(1) == hkv, "rope_kv_write: kcache [pages, hkv, ps, D]");
  const int D = kcache.size(3), ps = kcache.size(2);
  TORCH_CHECK(D % 8 == 0 && (D / 2) % 4 == 0, "rope_kv_write: head_dim % 8");
  TORCH_CHECK(qkv.size(1) == (hq + 2 * hkv) * D, "rope_kv_write: qkv width");
  TORCH_CHECK(cos_t.size(1) == D / 2, "rope_kv_write: cos table width");
  const long T = qkv.size(0);
  if (T == 0) return;
  const c10::cuda::CUDAGuard guard(qkv.device());
  launch_k(rope_kv_write_kernel, dim3(T), dim3(128), 0, at::cuda::getCurrentCUDAStream(),
           reinterpret_cast<const __nv_bfloat16*>(qkv.data_ptr()), (const int*)pos.data_ptr<int>(),
           reinterpret_cast<const long*>(slot.data_ptr<int64_t>()), (const float*)cos_t.data_ptr<float>(),
           (const float*)sin_t.data_ptr<float>(), reinterpret_cast<__nv_bfloat16*>(q_out.data_ptr()),
           reinterpret_cast<__nv_bfloat16*>(kcache.data_ptr()), reinterpret_cast<__nv_bfloat16*>(vcache.data_ptr()),
           (int)hq, (int)hkv, D, ps);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

// ----------------------------------------------------------------------------------------------
// embedding gather: out[t] = table[ids[t]] (bf16 rows, 16-byte vectors). Ids outside [0, V) give
// zeros and set the error word (the host validates ids before launch as well).
// ----------------------------------------------------------------------------------------------
__global__ void embed_kernel(const int* __restrict__ ids, const __nv_bfloat16* __restrict__ table,
                             __nv_bfloat16* __restrict__ out, int V, int H, int* err) {
  griddep_wait();
  griddep_launch_dependents();
  const long t = blockIdx.x;
  const int id = ids[t];
  const int nvec = H / 8;
  uint4* o = reinterpret_cast<uint4*>(out + t * H);
  if (id < 0 || id >= V) {
    if (threadIdx.x == 0) record_error(err, ERR_BAD_ARGUMENT);
    for (int i = threadIdx.x; i < nvec; i += blockDim.x) o[i] = make_uint4(0, 0, 0, 0);
    return;
  }
  const uint4* r = reinterpret_cast<const uint4*>(table + (long)id * H);
  for (int i = threadIdx.x; i < nvec; i += blockDim.x) o[i] = r[i];
}

void embedding(const at::Tensor& ids, const at::Tensor& table, at::Tensor& out, at::Tensor& err) {
  TORCH_CHECK(ids.scalar_type() == at::kInt && table.scalar_type() == at::kBFloat16, "embedding: dtypes");
  const int H = table.size(1);
  TORCH_CHECK(H % 8 == 0, "embedding: H % 8");
  const long T = ids.numel();
  if (T == 0) return;
  const c10::cuda::CUDAGuard guard(ids.device());
  launch_k(embed_kernel, dim3(T), dim3(128), 0, at::cuda::getCurrentCUDAStream(), (const int*)ids.data_ptr<int>(),
           reinterpret_cast<const __nv_bfloat16*>(table.data_ptr()), reinterpret_cast<__nv_bfloat16*>(out.data_ptr()),
           (int)table.size(0), H, err.data_ptr<int>());
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

// ----------------------------------------------------------------------------------------------
// argmax over fp32 logits rows [B, Vloc] -> packed (value, global index) pairs [B] as float2
// (index stored as float bits of an int). First maximal index wins, as the reference's strict '>'.
// ----------------------------------------------------------------------------------------------
__global__ void argmax_kernel(const float* __restrict__ logits, int Vloc, long ld, int vocab_offset,
                              float2* __restrict__ out) {
  griddep_wait();
  griddep_launch_dependents();
  __shared__ float sv[32];
  __shared__ int si[32];
  const long b = blockIdx.x;
  const float* row = logits + b * ld;
  float best = -INFINITY;
  int bi = 0x7fffffff;
  for (int i = threadIdx.x; i < Vloc; i += blockDim.x) {
    float v = row[i];
    if (v > best || (v == best && i < bi)) {
      best = v;
      bi = i;
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    float ov = __shfl_xor_sync(0xffffffffu, best, o);
    int oi = __shfl_xor_sync(0xffffffffu, bi, o);
    if (ov > best || (ov == best && oi < bi)) {
      best = ov;
      bi = oi;
    }
  }
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
  if (l == 0) {
    sv[w] = best;
    si[w] = bi;
  }
  __syncthreads();
  if (w == 0) {
    const int nw = blockDim.x >> 5;
    best = l < nw ? sv[l] : -INFINITY;
    bi = l < nw ? si[l] : 0x7fffffff;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      float ov = __shfl_xor_sync(0xffffffffu, best, o);
      int oi = __shfl_xor_sync(0xffffffffu, bi, o);
      if (ov > best || (ov == best && oi < bi)) {
        best = ov;
        bi = oi;
      }
    }
    if (l == 0) out[b] = make_float2(best, __int_as_float(bi + vocab_offset));
  }
}

// Merge per-rank (value, index) candidates [R, B] into token ids [B] (int32): max value, lowest
// index among ties, which equals the first-index argmax over the concatenated vocabulary.
__global__ void argmax_merge_kernel(const float2* __restrict__ cand, int R, int B, int* __restrict__ ids) {
  griddep_wait();
  griddep_launch_dependents();
  int b = blockIdx.x * blockDim.x + threadIdx.x;
  if (b >= B) return;
  float best = -INFINITY;
  int bi = 0x7fffffff;
  for (int r = 0; r < R; ++r) {
    float2 c = cand[(long)r * B + b];
    int ci = __float_as_int(c.y);
    if (c.x > best || (c.x == best && ci < bi)) {
      best = c.x;
      bi = ci;
    }
  }
  ids[b] = bi;
}

// Reduce the LM-head GEMM's per-tile candidates [m_tiles, B] (value, local index) to one
// (value, global index) per token. One CTA per token.
__global__ void argmax_tiles_kernel(const float2* __restrict__ cand, int m_tiles, int B, int vocab_offset,
                                    float2* __restrict__ out) {
  griddep_wait();
  griddep_launch_dependents();
  __shared__ float sv[32];
  __shared__ int si[32];
  const int b = blockIdx.x;
  float best = -INFINITY;
  int bi = 0x7fffffff;
  for (int t = threadIdx.x; t < m_tiles; t += blockDim.x) {
    const float2 c = cand[(long)t * B + b];
    const int ci = __float_as_int(c.y);
    if (c.x > best || (c.x == best && ci < bi)) {
      best = c.x;
      bi = ci;
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    float ov = __shfl_xor_sync(0xffffffffu, best, o);
    int oi = __shfl_xor_sync(0xffffffffu, bi, o);
    if (ov > best || (ov == best && oi < bi)) {
      best = ov;
      bi = oi;
    }
  }
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
  if (l == 0) {
    sv[w] = best;
    si[w] = bi;
  }
  __syncthreads();
  if (w == 0) {
    const int nw = blockDim.x >> 5;
    best = l < nw ? sv[l] : -INFINITY;
    bi = l < nw ? si[l] : 0x7fffffff;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      float ov = __shfl_xor_sync(0xffffffffu, best, o);
      int oi = __shfl_xor_sync(0xffffffffu, bi, o);
      if (ov > best || (ov == best && oi < bi)) {
        best = ov;
        bi = oi;
      }
    }
    if (l == 0) out[b] = make_float2(best, __int_as_float(bi + vocab_offset));
  }
}

void argmax_tiles(const at::Tensor& cand, int64_t vocab_offset, at::Tensor& out) {
  TORCH_CHECK(cand.scalar_type() == at::kFloat && cand.dim() == 3 && cand.size(2) == 2, "argmax_tiles: [T,B,2]");
  const int m_tiles = cand.size(0), B = cand.size(1);
  if (B == 0) return;
  const c10::cuda::CUDAGuard guard(cand.device());
  launch_k(argmax_tiles_kernel, dim3(B), dim3(256), 0, at::cuda::getCurrentCUDAStream(),
           reinterpret_cast<const float2*>(cand.data_ptr<float>()), m_tiles, B, (int)vocab_offset,
           reinterpret_cast<float2*>(out.data_ptr<float>()));
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void argmax_partial(const at::Tensor& logits, int64_t vocab_offset, at::Tensor& out) {
  TORCH_CHECK(logits.scalar_type() == at::kFloat && logits.stride(1) == 1, "argmax_partial: fp32 logits");
  const long B = logits.size(0);
  if (B == 0) return;
  const c10::cuda::CUDAGuard guard(logits.device());
  launch_k(argmax_kernel, dim3(B), dim3(512), 0, at::cuda::getCurrentCUDAStream(),
           (const float*)logits.data_ptr<float>(), (int)logits.size(1), (long)logits.stride(0), (int)vocab_offset,
           reinterpret_cast<float2*>(out.data_ptr<float>()));
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void argmax_merge(const at::Tensor& cand, at::Tensor& ids) {
  TORCH_CHECK(cand.scalar_type() == at::kFloat && cand.dim() == 3 && cand.size(2) == 2, "argmax_merge: [R,B,2] f32");
  const int R = cand.size(0), B = cand.size(1);
  if (B == 0) return;
  const c10::cuda::CUDAGuard guard(cand.device());
  launch_k(argmax_merge_kernel, dim3((B + 127) / 128), dim3(128), 0, at::cuda::getCurrentCUDAStream(),
           reinterpret_cast<const float2*>(cand.data_ptr<float>()), R, B, ids.data_ptr<int>());
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

}  // namespace mesh

namespace mesh {

// Vocabulary-parallel embedding fused with the first RMSNorm: rank r holds rows [start_r, start_r +
// n_r) of the table (near-equal contiguous ranges, larger first) in a symmetric allocation that
// every peer maps; each token's row is read from its owner's table (NVLink peer loads, or local),
// written to `resid` and normalised into `normed`. The tables are written once at load and only
// read afterwards, so no synchronisation between ranks is needed. One CTA per token.
struct EmbedPeerArgs {
  unsigned long long base[8];  // table base of each rank as mapped here
  const int* ids;
  int V, H, world;
  const __nv_bfloat16* gamma;
  float eps;
  __nv_bfloat16* resid;
  __nv_bfloat16* normed;
  int* err;
};

__global__ void __launch_bounds__(256) embed_peer_norm_kernel(const EmbedPeerArgs a) {
  __shared__ float red[8];
  const int t = blockIdx.x;
  griddep_wait();
  griddep_launch_dependents();
  int id = a.ids[t];
  const bool bad = id < 0 || id >= a.V;
  if (bad) {
    if (threadIdx.x == 0) record_error(a.err, ERR_BAD_ARGUMENT);
    id = 0;
  }
  const int base = a.V / a.world, extra = a.V % a.world;
  const int big = extra * (base + 1);
  const int r = id < big ? id / (base + 1) : extra + (id - big) / base;
  const int row = id - (id < big ? r * (base + 1) : big + (r - extra) * base);
  const uint4* src = reinterpret_cast<const uint4*>(a.base[r]) + (long)row * (a.H / 8);
  uint4* res = reinterpret_cast<uint4*>(a.resid + (long)t * a.H);
  const int nvec = a.H / 8;
  uint4 v[4];  // H <= 8192: at most 4 chunks of 16 bytes per thread
  float ss = 0.f;
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const int c = threadIdx.x + 256 * j;
    if (c < nvec) {
      v[j] = bad ? make_uint4(0, 0, 0, 0) : src[c];
      const uint32_t* u = reinterpret_cast<const uint32_t*>(&v[j]);
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        float x0, x1;
        unpack_bf16x2(u[q], x0, x1);
        ss += x0 * x0 + x1 * x1;
      }
      res[c] = v[j];
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
  __syncthreads();
  float tot = 0.f;
#pragma unroll
  for (int w = 0; w < 8; ++w) tot += red[w];
  const float inv = rsqrtf(tot / (float)a.H + a.eps);
  uint4* nrm = reinterpret_cast<uint4*>(a.normed + (long)t * a.H);
  const uint4* g = reinterpret_cast<const uint4*>(a.gamma);
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const int c = threadIdx.x + 256 * j;
    if (c < nvec) {
      const uint4 gv = g[c];
      const uint32_t* u = reinterpret_cast<const uint32_t*>(&v[j]);
      const uint32_t* gu = reinterpret_cast<const uint32_t*>(&gv);
      uint4 o;
      uint32_t* ou = reinterpret_cast<uint32_t*>(&o);
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        float x0, x1, g0, g1;
        unpack_bf16x2(u[q], x0, x1);
        unpack_bf16x2(gu[q], g0, g1);
        ou[q] = pack_bf16x2(x0 * inv * g0, x1 * inv * g1);
      }
      nrm[c] = o;
    }
  }
}

void embed_peer_norm(const at::Tensor& bases, const at::Tensor& ids, int64_t V, const at::Tensor& gamma, double eps,
                     at::Tensor& resid, at::Tensor& normed, at::Tensor& err) {
  TORCH_CHECK(bases.device().is_cpu() && bases.scalar_type() == at::kLong && bases.numel() >= 1 && bases.numel() <= 8,
              "embed_peer_norm: CPU int64 table bases of 1..8 ranks");
  TORCH_CHECK(ids.scalar_type() == at::kInt && ids.is_cuda(), "embed_peer_norm: int32 ids");
  const int T = ids.numel(), H = gamma.numel();
  TORCH_CHECK(H % 8 == 0 && H <= 8192 && resid.size(0) >= T && normed.size(0) >= T && resid.size(1) == H &&
                  resid.is_contiguous() && normed.is_contiguous(),
              "embed_peer_norm: H % 8 == 0, H <= 8192, resid/normed [T, H]");
  if (T == 0) return;
  const c10::cuda::CUDAGuard guard(ids.device());
  EmbedPeerArgs a{};
  a.world = bases.numel();
  for (int i = 0; i < a.world; ++i) a.base[i] = (unsigned long long)bases.data_ptr<int64_t>()[i];
  a.ids = ids.data_ptr<int>();
  a.V = (int)V;
  a.H = H;
  a.gamma = reinterpret_cast<const __nv_bfloat16*>(gamma.data_ptr());
  a.eps = (float)eps;
  a.resid = reinterpret_cast<__nv_bfloat16*>(resid.data_ptr());
  a.normed = reinterpret_cast<__nv_bfloat16*>(normed.data_ptr());
  a.err = err.data_ptr<int>();
  C10_CUDA_CHECK(launch_k(embed_peer_norm_kernel, dim3(T), dim3(256), 0, at::cuda::getCurrentCUDAStream(), a));
}

}  // namespace mesh
