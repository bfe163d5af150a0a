// Paged GQA decode attention kernels (device code + launcher), shared by the torch op and the
// C entry points. See attn_decode.cu for the algorithm.
#pragma once
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include "../include/sm100.cuh"
#include "../include/launch.h"

namespace mesh {

struct DecodeArgs {
  const __nv_bfloat16* q;       // [B, hq*D]
  const __nv_bfloat16* k;       // [pages, hkv, ps, D]
  const __nv_bfloat16* v;
  const int* block_tables;      // [B, max_pages]
  const int* seq_lens;          // [B]
  __nv_bfloat16* out;           // [B, hq*D]
  float* ws;                    // [B, hq, splits, D+1] when splits > 1
  int max_pages, hkv, page_size, splits;
  float scale_log2;             // softmax scale * log2(e)
  int window;                   // 0 = full causal context; else attend the last `window` keys
};

constexpr int DEC_WARPS = 4;

template <int G, int D>
__global__ void __launch_bounds__(DEC_WARPS * 32) attn_decode_kernel(const DecodeArgs a) {
  griddep_wait();
  griddep_launch_dependents();
  constexpr int DPL = D / 32;  // head dims per lane in P.V
  __shared__ float q_s[G][D];
  __shared__ float red_m[DEC_WARPS][G];
  __shared__ float red_l[DEC_WARPS][G];
  __shared__ float red_o[DEC_WARPS][G][D];

  const int seq = blockIdx.x, h = blockIdx.y, split = blockIdx.z;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int hq = a.hkv * G;
  const int L = a.seq_lens[seq];
  const int w0 = (a.window > 0 && L > a.window) ? L - a.window : 0;
  const int n = L - w0;
  int span = (n + a.splits - 1) / a.splits;
  span = (span + 31) & ~31;
  const int t_begin = w0 + split * span;
  const int t_end = min(L, t_begin + span);

  for (int i = threadIdx.x; i < G * D; i += blockDim.x) {
    const int g = i / D, d = i - g * D;
    q_s[g][d] = bf2f(a.q[(long)seq * hq * D + (h * G + g) * D + d]) * a.scale_log2;
  }
  __syncthreads();

  float m[G], l[G], acc[G][DPL];
#pragma unroll
  for (int g = 0; g < G; ++g) {
    m[g] = -INFINITY;
    l[g] = 0.f;
#pragma unroll
    for (int i = 0; i < DPL; ++i) acc[g][i] = 0.f;
  }
  const int* bt = a.block_tables + (long)seq * a.max_pages;
  const long head_stride = (long)a.page_size * D;           // one (page, head) block
  const long page_stride = (long)a.hkv * head_stride;

  for (int blk = t_begin + warp * 32; blk < t_end; blk += DEC_WARPS * 32) {
    const int t = blk + lane;
    const bool valid = t < t_end;
    const int ts = valid ? t : blk;  // lanes past the end reuse a valid key address, weight 0
    const int pg_i = ts / a.page_size;
    const int page = bt[pg_i];
    const long base = (long)page * page_stride + h * head_stride + (long)(ts - pg_i * a.page_size) * D;
    float s[G];
#pragma unroll
    for (int g = 0; g < G; ++g) s[g] = 0.f;
    {
      const uint4* kr = reinterpret_cast<const uint4*>(a.k + base);
      uint4 kv[D / 8];
#pragma unroll
      for (int c = 0; c < D / 8; ++c) kv[c] = __ldg(kr + c);
#pragma unroll
      for (int c = 0; c < D / 8; ++c) {
        const uint32_t* ku = reinterpret_cast<const uint32_t*>(&kv[c]);
        float kf[8];
#pragma unroll
        for (int j = 0; j < 4; ++j) unpack_bf16x2(ku[j], kf[2 * j], kf[2 * j + 1]);
#pragma unroll
        for (int g = 0; g < G; ++g) {
#pragma unroll
          for (int j = 0; j < 8; ++j) s[g] += q_s[g][c * 8 + j] * kf[j];
        }
      }
    }
    float p[G];
#pragma unroll
    for (int g = 0; g < G; ++g) {
      float sv = valid ? s[g] : -INFINITY;
      float mx = sv;
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
      const float mn = fmaxf(m[g], mx);
      const float corr = exp2f(m[g] - mn);  // m = -inf initially -> 0
      p[g] = valid ? exp2f(sv - mn) : 0.f;
      l[g] = l[g] * corr + p[g];
#pragma unroll
      for (int i = 0; i < DPL; ++i) acc[g][i] *= corr;
      m[g] = mn;
    }
    // P.V: lane owns DPL dims; 32 key rows, 8 loads in flight
#pragma unroll 8
    for (int j = 0; j < 32; ++j) {
      const long vb = __shfl_sync(0xffffffffu, base, j);
      const __nv_bfloat16* vr = a.v + vb + lane * DPL;
      float vf[DPL];
      if constexpr (DPL == 4) {
        uint2 vv = __ldg(reinterpret_cast<const uint2*>(vr));
        unpack_bf16x2(vv.x, vf[0], vf[1]);
        unpack_bf16x2(vv.y, vf[2], vf[3]);
      } else {
        uint32_t vv = __ldg(reinterpret_cast<const unsigned int*>(vr));
        unpack_bf16x2(vv, vf[0], vf[1]);
      }
#pragma unroll
      for (int g = 0; g < G; ++g) {
        const float pj = __shfl_sync(0xffffffffu, p[g], j);
#pragma unroll
        for (int i = 0; i < DPL; ++i) acc[g][i] += pj * vf[i];
      }
    }
  }

  // reduce per-lane l, then merge warps through shared memory
#pragma unroll
  for (int g = 0; g < G; ++g) {
    float lv = l[g];
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) lv += __shfl_xor_sync(0xffffffffu, lv, o);
    if (lane == 0) {
      red_m[warp][g] = m[g];
      red_l[warp][g] = lv;
    }
#pragma unroll
    for (int i = 0; i < DPL; ++i) red_o[warp][g][lane * DPL + i] = acc[g][i];
  }
  __syncthreads();
  for (int i = threadIdx.x; i < G * D; i += blockDim.x) {
    const int g = i / D, d = i - g * D;
    float M = -INFINITY;
#pragma unroll
    for (int w = 0; w < DEC_WARPS; ++w) M = fmaxf(M, red_m[w][g]);
    float lsum = 0.f, o = 0.f;
    if (M != -INFINITY) {
#pragma unroll
      for (int w = 0; w < DEC_WARPS; ++w) {
        const float f = exp2f(red_m[w][g] - M);
        lsum += red_l[w][g] * f;
        o += red_o[w][g][d] * f;
      }
    }
    const int qh = h * G + g;
    if (a.splits == 1) {
      a.out[(long)seq * hq * D + qh * D + d] = f2bf(lsum > 0.f ? o / lsum : 0.f);
    } else {
      float* w = a.ws + (((long)seq * hq + qh) * a.splits + split) * (D + 1);
      w[d] = lsum > 0.f ? o / lsum : 0.f;
      if (d == 0) w[D] = lsum > 0.f ? M + log2f(lsum) : -INFINITY;
    }
  }
}

// Merge split partials: out = sum_s o_s * 2^(lse_s - LSE) with LSE = log2(sum 2^lse_s).
template <int D>
__global__ void attn_decode_combine_kernel(const float* __restrict__ ws, __nv_bfloat16* __restrict__ out, int hq,
                                           int splits) {
  griddep_wait();
  griddep_launch_dependents();
  const int seq = blockIdx.x, qh = blockIdx.y;
  const float* w = ws + ((long)seq * hq + qh) * splits * (D + 1);
  float M = -INFINITY;
  for (int s = 0; s < splits; ++s) M = fmaxf(M, w[s * (D + 1) + D]);
  for (int d = threadIdx.x; d < D; d += blockDim.x) {
    float num = 0.f, den = 0.f;
    if (M != -INFINITY) {
      for (int s = 0; s < splits; ++s) {
        const float f = exp2f(w[s * (D + 1) + D] - M);
        num += w[s * (D + 1) + d] * f;
        den += f;
      }
    }
    out[(long)seq * hq * D + qh * D + d] = f2bf(den > 0.f ? num / den : 0.f);
  }
}

// Returns the first launch error; the combine kernel is not enqueued when the split kernel failed
// to launch (it would read scratch that nothing wrote).
template <int G, int D>
inline cudaError_t launch_attn_decode_gd(const DecodeArgs& a, int B, cudaStream_t st) {
  dim3 grid(B, a.hkv, a.splits);
  cudaError_t e = launch_k(attn_decode_kernel<G, D>, grid, dim3(DEC_WARPS * 32), 0, st, a);
  if (e != cudaSuccess || a.splits <= 1) return e;
  return launch_k(attn_decode_combine_kernel<D>, dim3(B, a.hkv * G), dim3(D), 0, st, (const float*)a.ws, a.out,
                  a.hkv * G, a.splits);
}

template <int D>
inline cudaError_t launch_attn_decode_d(const DecodeArgs& a, int B, int G, cudaStream_t st) {
  switch (G) {
    case 1: return launch_attn_decode_gd<1, D>(a, B, st);
    case 2: return launch_attn_decode_gd<2, D>(a, B, st);
    case 4: return launch_attn_decode_gd<4, D>(a, B, st);
    default: return launch_attn_decode_gd<8, D>(a, B, st);
  }
}

inline cudaError_t launch_attn_decode(const DecodeArgs& a, int B, int G, int D, cudaStream_t st) {
  return D == 128 ? launch_attn_decode_d<128>(a, B, G, st) : launch_attn_decode_d<64>(a, B, G, st);
}

}  // namespace mesh
