// Paged GQA decode attention, TMA-streamed (sm_100a).
//
// Decode attention is bound by reading K/V pages (one query token per sequence), so this kernel
// is built around the copy engine: a producer warp streams the pages of one (sequence, KV head)
// into a 3-stage shared-memory ring with 2D TMA loads (128-byte swizzle, no multicast; each
// 16-token page of one head is a [16 x 128] bf16 block = two 16x64 boxes per tensor). Four
// consumer warps each take one page of every 64-key stage: S = Q K^T and O += P V run on
// m16n8k16 tensor-core fragments read with ldmatrix (conflict-free thanks to the swizzle), the G
// query heads of the group padded to 16 rows. Online softmax in the exp2 domain; warps merge
// through shared memory at the end (or write a split partial + log-sum-exp for the combine
// kernel shared with the CUDA-core variant).
#pragma once
#include <cuda.h>
#include <cuda_bf16.h>

#include "../include/launch.h"
#include "../include/sm100.cuh"
#include "attn_decode.cuh"

namespace mesh {

constexpr int DTC_STAGES = 3;
constexpr int DTC_KEYS = 64;               // keys per stage = 4 pages of 16
constexpr int DTC_BOX_BYTES = 16 * 64 * 2; // one [16 x 64] bf16 box
constexpr int DTC_STAGE_BYTES = 4 * 2 * 2 * DTC_BOX_BYTES;  // 4 pages x {K,V} x 2 halves = 32 KB
constexpr int DTC_Q_LD = 136;              // padded bf16 row stride of the Q tile
constexpr uint64_t DTC_WAIT_NS = 2000000000ull;

struct DecodeTcArgs {
  const __nv_bfloat16* q;
  const int* block_tables;
  const int* seq_lens;
  __nv_bfloat16* out;
  float* ws;
  int* err;
  int max_pages, hkv, splits;
  float scale_log2;
  int window;
  // split > 1: per-(sequence, KV head) arrival counters (zero between launches). When set, the
  // last split CTA of a (sequence, KV head) merges the partials itself and resets its counter, so
  // no separate combine launch follows; null keeps the combine kernel.
  int* counters;
};

__device__ __forceinline__ void dtc_ldsm_x4(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}
__device__ __forceinline__ void dtc_ldsm_x4_t(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2,
                                              uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}
__device__ __forceinline__ void dtc_mma(float (&c)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                        uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// byte offset of (row r, 16-byte chunk c) inside a [16 x 64] box written with 128-byte swizzle
__device__ __forceinline__ uint32_t dtc_swz(int r, int c) { return (uint32_t)(r * 128 + ((c ^ (r & 7)) << 4)); }

template <int G>
__global__ void __launch_bounds__(160) attn_decode_tc_kernel(const __grid_constant__ CUtensorMap tmK,
                                                             const __grid_constant__ CUtensorMap tmV,
                                                             const DecodeTcArgs a) {
  constexpr int D = 128;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* sm = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* stages = sm;                                                      // DTC_STAGES x 32 KB
  __nv_bfloat16* q_s = reinterpret_cast<__nv_bfloat16*>(sm + DTC_STAGES * DTC_STAGE_BYTES);  // 16 x 136
  uint64_t* full = reinterpret_cast<uint64_t*>(sm + DTC_STAGES * DTC_STAGE_BYTES + 16 * DTC_Q_LD * 2);
  uint64_t* empty = full + DTC_STAGES;
  __shared__ float red_m[4][8], red_l[4][8];

  const int seq = blockIdx.x, h = blockIdx.y, split = blockIdx.z;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int hq = a.hkv * G;
  // Sequence lengths and block tables are step inputs copied before the step's first kernel; only
  // Q and the newest key/value (position L-1) come from the kernel just before this one. Pages that
  // do not hold position L-1 are streamed before griddepcontrol.wait, overlapping that kernel.
  griddep_launch_dependents();
  const int L = a.seq_lens[seq];
  const int w0 = (a.window > 0 && L > a.window) ? L - a.window : 0;
  const int s0 = (w0 / DTC_KEYS) * DTC_KEYS;  // stage-aligned start
  const int n_stages_total = (L - s0 + DTC_KEYS - 1) / DTC_KEYS;
  const int per_split = (n_stages_total + a.splits - 1) / a.splits;
  const int st_begin = split * per_split;
  const int st_end = min(n_stages_total, st_begin + per_split);
  const int nst = max(0, st_end - st_begin);

  if (threadIdx.x == 0) {
    for (int i = 0; i < DTC_STAGES; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], 4);
    }
    fence_mbar_init();
  }
  __syncthreads();  // barriers initialised

  const int* bt = a.block_tables + (long)seq * a.max_pages;
  if (warp == 4) {
    // ------------------------------- TMA producer -------------------------------
    if (lane == 0) {
      tma_prefetch_desc(&tmK);
      tma_prefetch_desc(&tmV);
      const uint64_t pol = policy_evict_first();
      bool waited = false;
      for (int i = 0; i < nst; ++i) {
        const int s = i % DTC_STAGES;
        const uint32_t ph = (i / DTC_STAGES) & 1;
        if (!mbar_wait_bounded(&empty[s], ph ^ 1, a.err, ERR_MBAR_TIMEOUT_PRODUCER, nullptr, DTC_WAIT_NS)) break;
        const int key0 = s0 + (st_begin + i) * DTC_KEYS;
        if (!waited && key0 + DTC_KEYS > L - 1) {  // this stage holds the newest key/value
          griddep_wait();
          waited = true;
        }
        const int npages = min(4, (L - key0 + 15) / 16);
        mbar_arrive_expect_tx(&full[s], (uint32_t)npages * 4 * DTC_BOX_BYTES);
        uint8_t* st = stages + s * DTC_STAGE_BYTES;
        for (int p = 0; p < npages; ++p) {
          const int page = bt[key0 / 16 + p];
          const int y = (page * a.hkv + h) * 16;
          // layout per page: [K half0][K half1][V half0][V half1], 2 KB each
          uint8_t* pb = st + p * 4 * DTC_BOX_BYTES;
          tma_load_2d(pb, &tmK, &full[s], 0, y, pol);
          tma_load_2d(pb + DTC_BOX_BYTES, &tmK, &full[s], 64, y, pol);
          tma_load_2d(pb + 2 * DTC_BOX_BYTES, &tmV, &full[s], 0, y, pol);
          tma_load_2d(pb + 3 * DTC_BOX_BYTES, &tmV, &full[s], 64, y, pol);
        }
      }
    }
  } else {
    // ------------------------------- consumers -------------------------------
    griddep_wait();  // Q comes from the RoPE kernel just before
    // Q rows 0..G-1 (rows G..15 zero), bf16, padded stride
    for (int i = threadIdx.x; i < 16 * (D / 8); i += 128) {
      const int r = i / (D / 8), c = i - r * (D / 8);
      uint4 v = make_uint4(0, 0, 0, 0);
      if (r < G) v = *reinterpret_cast<const uint4*>(a.q + (long)seq * hq * D + (h * G + r) * D + c * 8);
      *reinterpret_cast<uint4*>(q_s + r * DTC_Q_LD + c * 8) = v;
    }
    named_bar_sync(1, 128);
    // Q fragments (A operand, rows = heads), 8 k-steps of 16
    uint32_t qf[8][4];
    {
      const uint32_t qb = smem_u32(q_s);
      const int r = lane & 15;
#pragma unroll
      for (int kk = 0; kk < 8; ++kk) {
        const int c = kk * 16 + (lane >> 4) * 8;
        dtc_ldsm_x4(qb + (uint32_t)(r * DTC_Q_LD + c) * 2, qf[kk][0], qf[kk][1], qf[kk][2], qf[kk][3]);
      }
    }
    float o[16][4];
#pragma unroll
    for (int n = 0; n < 16; ++n) o[n][0] = o[n][1] = o[n][2] = o[n][3] = 0.f;
    float m_run = -INFINITY, l_run = 0.f;  // row g = lane/4 (rows >= G are padding)
    const int g_row = lane >> 2;
    const bool row_ok = g_row < G;
    for (int i = 0; i < nst; ++i) {
      const int s = i % DTC_STAGES;
      const uint32_t ph = (i / DTC_STAGES) & 1;
      int okw = 1;
      if (lane == 0) okw = mbar_wait_bounded(&full[s], ph, a.err, ERR_MBAR_TIMEOUT_MMA, nullptr, DTC_WAIT_NS);
      okw = __shfl_sync(0xffffffffu, okw, 0);
      if (!okw) break;
      const int key0 = s0 + (st_begin + i) * DTC_KEYS + warp * 16;  // this warp's page
      const uint32_t pb = smem_u32(stages + s * DTC_STAGE_BYTES + warp * 4 * DTC_BOX_BYTES);
      float sc[2][4];
      if (key0 < L) {
#pragma unroll
        for (int n = 0; n < 2; ++n) sc[n][0] = sc[n][1] = sc[n][2] = sc[n][3] = 0.f;
        // S = Q K^T over 16 keys (2 n-tiles of 8)
#pragma unroll
        for (int n = 0; n < 2; ++n) {
#pragma unroll
          for (int kk = 0; kk < 8; kk += 2) {
            const int half = kk >> 2;               // dims 0..63 or 64..127
            const int r = n * 8 + (lane & 7);       // key row inside the page
            const int c = (kk & 3) * 2 + (lane >> 3);  // 16-byte chunk inside the half
            uint32_t b0, b1, b2, b3;
            dtc_ldsm_x4(pb + half * DTC_BOX_BYTES + dtc_swz(r, c), b0, b1, b2, b3);
            dtc_mma(sc[n], qf[kk][0], qf[kk][1], qf[kk][2], qf[kk][3], b0, b1);
            dtc_mma(sc[n], qf[kk + 1][0], qf[kk + 1][1], qf[kk + 1][2], qf[kk + 1][3], b2, b3);
          }
        }
        // mask, online softmax on row g_row (c0, c1 of each n-tile)
        float mx = -INFINITY;
#pragma unroll
        for (int n = 0; n < 2; ++n) {
#pragma unroll
          for (int j = 0; j < 2; ++j) {
            const int key = key0 + n * 8 + (lane & 3) * 2 + j;
            const bool ok = row_ok && key < L && key >= w0;
            sc[n][j] = ok ? sc[n][j] * a.scale_log2 : -INFINITY;
            mx = fmaxf(mx, sc[n][j]);
          }
        }
        mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
        mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
        const float mn = fmaxf(m_run, mx);
        const float corr = (mn == -INFINITY) ? 1.f : exp2f(m_run - mn);
        float p[2][2];
        float ps = 0.f;
#pragma unroll
        for (int n = 0; n < 2; ++n)
#pragma unroll
          for (int j = 0; j < 2; ++j) {
            p[n][j] = (mn == -INFINITY) ? 0.f : exp2f(sc[n][j] - mn);
            ps += p[n][j];
          }
        l_run = l_run * corr + ps;
        m_run = mn;
#pragma unroll
        for (int n = 0; n < 16; ++n) {
          o[n][0] *= corr;
          o[n][1] *= corr;
        }
        const uint32_t pa0 = pack_bf16x2(p[0][0], p[0][1]);
        const uint32_t pa2 = pack_bf16x2(p[1][0], p[1][1]);
        // O += P V : k = 16 keys, n = 128 dims (16 n-tiles), V via transposed ldmatrix
#pragma unroll
        for (int n = 0; n < 16; n += 2) {
          const int half = n >> 3;
          const int r = (lane & 7) + ((lane >> 3) & 1) * 8;      // key row
          const int c = (n & 7) + (lane >> 4);                   // chunk (8 dims)
          uint32_t b0, b1, b2, b3;
          dtc_ldsm_x4_t(pb + (2 + half) * DTC_BOX_BYTES + dtc_swz(r, c), b0, b1, b2, b3);
          dtc_mma(o[n], pa0, 0u, pa2, 0u, b0, b1);
          dtc_mma(o[n + 1], pa0, 0u, pa2, 0u, b2, b3);
        }
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty[s]);
    }
    // l: sum across the 4 lanes of the row
    l_run += __shfl_xor_sync(0xffffffffu, l_run, 1);
    l_run += __shfl_xor_sync(0xffffffffu, l_run, 2);
    if ((lane & 3) == 0 && row_ok) {
      red_m[warp][g_row] = m_run;
      red_l[warp][g_row] = l_run;
    }
    // stash O rows (< G) in the first stage buffer once every warp has finished with the ring
    named_bar_sync(1, 128);
    const uint32_t o_s = smem_u32(stages);  // [4 warps][G][D] fp32
    if (row_ok) {
#pragma unroll
      for (int n = 0; n < 16; ++n) {
        const int d = n * 8 + (lane & 3) * 2;
        sts_f32(o_s + (uint32_t)((warp * G + g_row) * D + d) * 4, o[n][0]);
        sts_f32(o_s + (uint32_t)((warp * G + g_row) * D + d + 1) * 4, o[n][1]);
      }
    }
    named_bar_sync(1, 128);
    for (int i = threadIdx.x; i < G * D; i += 128) {
      const int g = i / D, d = i - g * D;
      float M = -INFINITY;
#pragma unroll
      for (int w = 0; w < 4; ++w) M = fmaxf(M, red_m[w][g]);
      float lsum = 0.f, ov = 0.f;
      if (M != -INFINITY) {
#pragma unroll
        for (int w = 0; w < 4; ++w) {
          const float f = exp2f(red_m[w][g] - M);
          lsum += red_l[w][g] * f;
          ov += lds_f32(o_s + (uint32_t)((w * G + g) * D + d) * 4) * f;
        }
      }
      const int qh = h * G + g;
      if (a.splits == 1) {
        a.out[(long)seq * hq * D + qh * D + d] = f2bf(lsum > 0.f ? ov / lsum : 0.f);
      } else {
        float* w = a.ws + (((long)seq * hq + qh) * a.splits + split) * (D + 1);
        w[d] = lsum > 0.f ? ov / lsum : 0.f;
        if (d == 0) w[D] = lsum > 0.f ? M + log2f(lsum) : -INFINITY;
      }
    }
    if (a.splits > 1 && a.counters != nullptr) {
      // threadfence-reduction: publish this split's partial, count it, and let the last arrival
      // merge all splits (same arithmetic and order as attn_decode_combine_kernel)
      __shared__ int s_last;
      __threadfence();
      named_bar_sync(1, 128);
      int* cnt = a.counters + (long)seq * a.hkv + h;
      if (threadIdx.x == 0) s_last = (atomicAdd(cnt, 1) == a.splits - 1) ? 1 : 0;
      named_bar_sync(1, 128);
      if (s_last) {
        __threadfence();
        for (int i = threadIdx.x; i < G * D; i += 128) {
          const int g = i / D, d = i - g * D;
          const int qh = h * G + g;
          const float* w = a.ws + ((long)seq * hq + qh) * a.splits * (D + 1);
          float M = -INFINITY;
          for (int sp = 0; sp < a.splits; ++sp) M = fmaxf(M, __ldcg(w + sp * (D + 1) + D));
          float num = 0.f, den = 0.f;
          if (M != -INFINITY) {
            for (int sp = 0; sp < a.splits; ++sp) {
              const float f = exp2f(__ldcg(w + sp * (D + 1) + D) - M);
              num += __ldcg(w + sp * (D + 1) + d) * f;
              den += f;
            }
          }
          a.out[(long)seq * hq * D + qh * D + d] = f2bf(den > 0.f ? num / den : 0.f);
        }
        if (threadIdx.x == 0) *cnt = 0;  // ready for the next launch
      }
    }
  }
}

inline size_t attn_decode_tc_smem() { return 1024 + DTC_STAGES * DTC_STAGE_BYTES + 16 * DTC_Q_LD * 2 + 2 * DTC_STAGES * 8; }

template <int G>
inline void launch_attn_decode_tc_g(const CUtensorMap& tk, const CUtensorMap& tv, const DecodeTcArgs& a, int B,
                                    cudaStream_t st) {
  auto kern = attn_decode_tc_kernel<G>;
  static bool configured[64] = {false};
  int dev = 0;
  cudaGetDevice(&dev);
  if (!configured[dev]) {
    cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)attn_decode_tc_smem());
    configured[dev] = true;
  }
  C10_CUDA_CHECK(launch_k(kern, dim3(B, a.hkv, a.splits), dim3(160), attn_decode_tc_smem(), st, tk, tv, a));
  if (a.splits > 1 && a.counters == nullptr)
    C10_CUDA_CHECK(launch_k(attn_decode_combine_kernel<128>, dim3(B, a.hkv * G), dim3(128), 0, st,
                            (const float*)a.ws, a.out, a.hkv * G, a.splits));
}

}  // namespace mesh
