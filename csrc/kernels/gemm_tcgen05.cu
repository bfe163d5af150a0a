// Persistent tcgen05 GEMM for sm_100a: D = A * B^T, A [M,K] and B [N,K] bf16 row-major (K-major).
//
// CTA = 6 warps: warp 0 issues TMA loads (one elected lane), warp 1 owns TMEM and issues
// tcgen05.mma from one thread, warps 2-5 run the epilogue out of TMEM. Tiles are 128 x BN x 64
// (BN a runtime multiple of 16, 16..256), operands staged in a multi-stage smem ring with
// 128-byte swizzle, accumulators double-buffered in TMEM so the epilogue of tile i overlaps the
// main loop of tile i+1.
//
// Two orientations share the kernel:
//  * normal (TRANS=false): out[m][n]; used for prefill (A = activations, B = weights);
//  * swap-AB (TRANS=true): out[n][m]; used for decode (A = weights so the 128-row MMA M dimension
//    runs over output features and the few decode tokens form a narrow N = BN tile).
// Small grids use split-K: every split writes an fp32 partial tile to a workspace, and the last
// CTA to arrive on the tile's counter (atomic ticket, no spinning) sums them and runs the epilogue.
//
// Epilogues: bf16 store, f32 store, and SiLU(gate)*up for gate/up weights interleaved in blocks
// of 64 features (rows g0..63,u0..63,g64..127,...), which writes half as many features.
//
// No TMA multicast is used. All mbarrier waits are bounded (see sm100.cuh).
#include <ATen/ATen.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/extension.h>

#include <mutex>
#include <unordered_map>

#include "../include/sm100.cuh"
#include "../include/tma_host.h"

namespace mesh {

enum EpiKind : int { EPI_STORE_BF16 = 0, EPI_STORE_F32 = 1, EPI_SILU_BF16 = 2 };

constexpr int BM = 128;
constexpr int BK = 64;
constexpr int A_STAGE_BYTES = BM * BK * 2;     // 16 KB
constexpr int EPI_LD = 33;                      // padded fp32 row stride of the epilogue staging tile
constexpr int EPI_SLOT_FLOATS = BM * EPI_LD;
constexpr int NUM_THREADS = 192;
constexpr uint64_t WAIT_LIMIT_NS = 2000000000ull;  // 2 s: far above any legal wait

struct GemmParams {
  int M, N, K;
  int m_tiles, n_tiles, k_blocks, splits;
  int bn, stages;
  void* out;
  long ldo;
  float* workspace;   // [splits][tiles][BM][bn]
  int* counters;      // [tiles], zero on entry, left zero on exit
  int* err;
  uint32_t idesc;
  uint32_t tmem_cols;
};

struct Smem {
  uint8_t* a;
  uint8_t* b;
  float* epi;
  uint64_t* full;
  uint64_t* empty;
  uint64_t* tfull;
  uint64_t* tempty;
  uint32_t* tmem_base;
  int* abort_flag;
  int* epi_flag;
};

__device__ __forceinline__ Smem carve(uint8_t* base, const GemmParams& p) {
  Smem s;
  uintptr_t b = reinterpret_cast<uintptr_t>(base);
  b = (b + 1023) & ~uintptr_t(1023);
  uint8_t* ptr = reinterpret_cast<uint8_t*>(b);
  s.a = ptr;
  ptr += (size_t)p.stages * A_STAGE_BYTES;
  s.b = ptr;
  ptr += (size_t)p.stages * p.bn * BK * 2;
  s.epi = reinterpret_cast<float*>(ptr);
  ptr += 2 * EPI_SLOT_FLOATS * sizeof(float);
  ptr = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(ptr) + 7) & ~uintptr_t(7));
  s.full = reinterpret_cast<uint64_t*>(ptr);
  s.empty = s.full + p.stages;
  s.tfull = s.empty + p.stages;
  s.tempty = s.tfull + 2;
  s.tmem_base = reinterpret_cast<uint32_t*>(s.tempty + 2);
  s.abort_flag = reinterpret_cast<int*>(s.tmem_base + 1);
  s.epi_flag = s.abort_flag + 1;
  return s;
}

__host__ __device__ inline size_t gemm_smem_bytes(int stages, int bn) {
  return 1024 + (size_t)stages * (A_STAGE_BYTES + bn * BK * 2) + 2 * EPI_SLOT_FLOATS * sizeof(float) + 8 +
         (size_t)(2 * stages + 4) * 8 + 16;
}

struct Unit {
  int tm, tn, split, tile, kb0, kb1;
};

__device__ __forceinline__ Unit decode_unit(int u, const GemmParams& p) {
  const int tiles = p.m_tiles * p.n_tiles;
  Unit r;
  r.split = u / tiles;
  int t = u - r.split * tiles;
  // grouped raster: 8 consecutive m-tiles sweep all n-tiles before the next group
  const int G = 8;
  const int group_size = G * p.n_tiles;
  int g = t / group_size;
  int first_m = g * G;
  int gm = min(p.m_tiles - first_m, G);
  int in = t - g * group_size;
  r.tm = first_m + in % gm;
  r.tn = in / gm;
  r.tile = r.tm * p.n_tiles + r.tn;
  r.kb0 = (int)(((long)r.split * p.k_blocks) / p.splits);
  r.kb1 = (int)(((long)(r.split + 1) * p.k_blocks) / p.splits);
  return r;
}

// ----------------------------------------------------------------------------------------------
// epilogue helpers: the epilogue stages 128 x (<=32) fp32 chunks in smem, then writes them with a
// thread mapping chosen for coalescing in each orientation.
// ----------------------------------------------------------------------------------------------
template <int EPI, bool TRANS>
__device__ __forceinline__ void finalize_chunk(const GemmParams& p, const float* slot0, const float* slot1,
                                               int tm, int tn, int c0, int cw, int et) {
  const int m_base = tm * BM;
  if constexpr (EPI == EPI_SILU_BF16) {
    __nv_bfloat16* out = reinterpret_cast<__nv_bfloat16*>(p.out);
    if constexpr (TRANS) {
      // features along M: rows 0..63 gate, 64..127 up; out[n][m_base/2 + r]
      const int m_out_base = tm * (BM / 2);
      const int m_out_lim = p.M / 2;
      for (int idx = et; idx < 32 * cw; idx += 128) {
        int rp = idx & 31, c = idx >> 5;
        int n = tn * p.bn + c0 + c;
        int r = rp * 2;
        if (n >= p.N || m_out_base + r >= m_out_lim) continue;
        float g0 = slot0[r * EPI_LD + c], g1 = slot0[(r + 1) * EPI_LD + c];
        float u0 = slot0[(r + 64) * EPI_LD + c], u1 = slot0[(r + 65) * EPI_LD + c];
        uint32_t v = pack_bf16x2(silu_f(g0) * u0, silu_f(g1) * u1);
        *reinterpret_cast<uint32_t*>(out + (long)n * p.ldo + m_out_base + r) = v;
      }
    } else {
      // features along N: slot0 = gate cols, slot1 = matching up cols; c0 = output column offset
      const int n_out_base = tn * (p.bn / 2) + c0;
      const int n_out_lim = p.N / 2;
      for (int idx = et; idx < BM * 16; idx += 128) {
        int r = idx >> 4, cp = (idx & 15) * 2;
        int m = m_base + r;
        int n = n_out_base + cp;
        if (m >= p.M || n >= n_out_lim) continue;
        float g0 = slot0[r * EPI_LD + cp], g1 = slot0[r * EPI_LD + cp + 1];
        float u0 = slot1[r * EPI_LD + cp], u1 = slot1[r * EPI_LD + cp + 1];
        *reinterpret_cast<uint32_t*>(out + (long)m * p.ldo + n) = pack_bf16x2(silu_f(g0) * u0, silu_f(g1) * u1);
      }
    }
  } else if constexpr (EPI == EPI_STORE_BF16) {
    __nv_bfloat16* out = reinterpret_cast<__nv_bfloat16*>(p.out);
    if constexpr (TRANS) {
      for (int idx = et; idx < 64 * cw; idx += 128) {
        int rp = idx & 63, c = idx >> 6;
        int n = tn * p.bn + c0 + c;
        int m = m_base + rp * 2;
        if (n >= p.N || m >= p.M) continue;
        float a = slot0[(rp * 2) * EPI_LD + c];
        float b = (m + 1 < p.M) ? slot0[(rp * 2 + 1) * EPI_LD + c] : 0.f;
        if (m + 1 < p.M)
          *reinterpret_cast<uint32_t*>(out + (long)n * p.ldo + m) = pack_bf16x2(a, b);
        else
          out[(long)n * p.ldo + m] = f2bf(a);
      }
    } else {
      const int half = cw >> 1;
      for (int idx = et; idx < BM * half; idx += 128) {
        int r = idx / half, cp = (idx - r * half) * 2;
        int m = m_base + r;
        int n = tn * p.bn + c0 + cp;
        if (m >= p.M || n >= p.N) continue;
        float a = slot0[r * EPI_LD + cp], b = slot0[r * EPI_LD + cp + 1];
        if (n + 1 < p.N)
          *reinterpret_cast<uint32_t*>(out + (long)m * p.ldo + n) = pack_bf16x2(a, b);
        else
          out[(long)m * p.ldo + n] = f2bf(a);
      }
    }
  } else {  // EPI_STORE_F32
    float* out = reinterpret_cast<float*>(p.out);
    if constexpr (TRANS) {
      for (int idx = et; idx < BM * cw; idx += 128) {
        int r = idx & 127, c = idx >> 7;
        int n = tn * p.bn + c0 + c;
        int m = m_base + r;
        if (n >= p.N || m >= p.M) continue;
        out[(long)n * p.ldo + m] = slot0[r * EPI_LD + c];
      }
    } else {
      for (int idx = et; idx < BM * cw; idx += 128) {
        int r = idx / cw, c = idx - r * cw;
        int m = m_base + r;
        int n = tn * p.bn + c0 + c;
        if (m >= p.M || n >= p.N) continue;
        out[(long)m * p.ldo + n] = slot0[r * EPI_LD + c];
      }
    }
  }
}

// Chunk plan: for SiLU in normal orientation, each step loads a gate chunk and the matching up
// chunk 64 columns later; everything else walks 32-column chunks.
template <int EPI, bool TRANS>
struct ChunkPlan {
  __device__ static int steps(int bn) {
    if constexpr (EPI == EPI_SILU_BF16 && !TRANS) return (bn / 128) * 2;
    return (bn + 31) / 32;
  }
  // returns (col of slot0, col of slot1 or -1, width, output column offset)
  __device__ static void step(int s, int bn, int& c_a, int& c_b, int& cw, int& c_out) {
    if constexpr (EPI == EPI_SILU_BF16 && !TRANS) {
      int g = s >> 1, h = s & 1;
      c_a = g * 128 + h * 32;
      c_b = c_a + 64;
      cw = 32;
      c_out = g * 64 + h * 32;
    } else {
      c_a = s * 32;
      c_b = -1;
      cw = min(32, bn - c_a);
      c_out = c_a;
    }
  }
};

__device__ __forceinline__ void tmem_chunk_to_smem(uint32_t taddr_row, int col, int cw, float* slot, int row) {
  uint32_t r[16];
  tmem_ld16(taddr_row + col, r);
  tmem_ld_wait();
#pragma unroll
  for (int i = 0; i < 16; ++i) slot[row * EPI_LD + i] = __uint_as_float(r[i]);
  if (cw > 16) {
    tmem_ld16(taddr_row + col + 16, r);
    tmem_ld_wait();
#pragma unroll
    for (int i = 0; i < 16; ++i) slot[row * EPI_LD + 16 + i] = __uint_as_float(r[i]);
  }
}

template <int EPI, bool TRANS>
__global__ void __launch_bounds__(NUM_THREADS, 1)
    gemm_tcgen05_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                        const GemmParams p) {
  extern __shared__ uint8_t smem_raw[];
  Smem s = carve(smem_raw, p);
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int tiles = p.m_tiles * p.n_tiles;
  const int total_units = tiles * p.splits;
  const uint32_t b_stage_bytes = (uint32_t)p.bn * BK * 2;

  if (threadIdx.x == 0) {
    for (int i = 0; i < p.stages; ++i) {
      mbar_init(&s.full[i], 1);
      mbar_init(&s.empty[i], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&s.tfull[i], 1);
      mbar_init(&s.tempty[i], 128);
    }
    *s.abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
  }
  if (warp == 1) {
    tmem_alloc(s.tmem_base, p.tmem_cols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *s.tmem_base;
  volatile int* abort_flag = s.abort_flag;

  if (warp == 0) {
    // ------------------------------- TMA producer -------------------------------
    if (lane == 0) {
      // decode streams weights once (A, evict-first) and reuses the token tile (B); prefill reuses both
      const uint64_t pol_a = TRANS ? policy_evict_first() : policy_evict_last();
      const uint64_t pol_b = policy_evict_last();
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      for (int u = blockIdx.x; u < total_units && ok; u += gridDim.x) {
        Unit un = decode_unit(u, p);
        for (int kb = un.kb0; kb < un.kb1; ++kb) {
          if (!mbar_wait_bounded(&s.empty[stage], phase ^ 1, p.err, ERR_MBAR_TIMEOUT_PRODUCER, abort_flag,
                                 WAIT_LIMIT_NS)) {
            ok = false;
            break;
          }
          mbar_arrive_expect_tx(&s.full[stage], A_STAGE_BYTES + b_stage_bytes);
          tma_load_2d(s.a + (size_t)stage * A_STAGE_BYTES, &tmA, &s.full[stage], kb * BK, un.tm * BM, pol_a);
          tma_load_2d(s.b + (size_t)stage * b_stage_bytes, &tmB, &s.full[stage], kb * BK, un.tn * p.bn, pol_b);
          if (++stage == p.stages) {
            stage = 0;
            phase ^= 1;
          }
        }
      }
      if (!ok) {
        // drain: give copies already in flight a bounded chance to land before the CTA exits
        for (int i = 0; i < p.stages; ++i) {
          uint64_t t0 = globaltimer_ns();
          while (!mbar_try_wait(&s.full[i], 0) && !mbar_try_wait(&s.full[i], 1) &&
                 globaltimer_ns() - t0 < 50000000ull) {
          }
        }
      }
    }
  } else if (warp == 1) {
    // ------------------------------- MMA issuer -------------------------------
    int stage = 0;
    uint32_t phase = 0;
    int it = 0;
    bool ok = true;
    for (int u = blockIdx.x; u < total_units && ok; u += gridDim.x, ++it) {
      Unit un = decode_unit(u, p);
      const int acc = it & 1;
      const uint32_t acc_phase = (it >> 1) & 1;
      int w = 1;
      if (lane == 0)
        w = mbar_wait_bounded(&s.tempty[acc], acc_phase ^ 1, p.err, ERR_MBAR_TIMEOUT_MMA, abort_flag, WAIT_LIMIT_NS);
      w = __shfl_sync(0xffffffffu, w, 0);
      if (!w) {
        ok = false;
        break;
      }
      tc_fence_after();
      const uint32_t d_tmem = tmem_base + (uint32_t)(acc * p.bn);
      for (int kb = un.kb0; kb < un.kb1; ++kb) {
        if (lane == 0)
          w = mbar_wait_bounded(&s.full[stage], phase, p.err, ERR_MBAR_TIMEOUT_MMA, abort_flag, WAIT_LIMIT_NS);
        w = __shfl_sync(0xffffffffu, w, 0);
        if (!w) {
          ok = false;
          break;
        }
        tc_fence_after();
        if (lane == 0) {
          const uint32_t a_addr = smem_u32(s.a + (size_t)stage * A_STAGE_BYTES);
          const uint32_t b_addr = smem_u32(s.b + (size_t)stage * b_stage_bytes);
          const uint64_t a_desc = make_sdesc_sw128(a_addr);
          const uint64_t b_desc = make_sdesc_sw128(b_addr);
#pragma unroll
          for (int k = 0; k < BK / 16; ++k) {
            // advance 16 bf16 = 32 bytes inside the swizzled 128-byte row: +2 in 16-byte units
            umma_bf16(d_tmem, a_desc + 2 * k, b_desc + 2 * k, p.idesc, (kb > un.kb0 || k > 0) ? 1u : 0u);
          }
          umma_commit(&s.empty[stage]);
        }
        __syncwarp();
        if (++stage == p.stages) {
          stage = 0;
          phase ^= 1;
        }
      }
      if (!ok) break;
      if (lane == 0) umma_commit(&s.tfull[acc]);
      __syncwarp();
    }
  } else {
    // ------------------------------- epilogue (warps 2..5) -------------------------------
    const int et = threadIdx.x - 64;            // 0..127
    const int quarter = warp & 3;               // TMEM lane quarter this warp may access
    const int row = quarter * 32 + lane;        // accumulator row (TMEM lane)
    float* slot0 = s.epi;
    float* slot1 = s.epi + EPI_SLOT_FLOATS;
    int it = 0;
    for (int u = blockIdx.x; u < total_units; u += gridDim.x, ++it) {
      Unit un = decode_unit(u, p);
      const int acc = it & 1;
      const uint32_t acc_phase = (it >> 1) & 1;
      if (et == 0)
        *s.epi_flag = mbar_wait_bounded(&s.tfull[acc], acc_phase, p.err, ERR_MBAR_TIMEOUT_EPILOGUE, abort_flag,
                                        WAIT_LIMIT_NS);
      named_bar_sync(1, 128);
      const int ok = *s.epi_flag;
      named_bar_sync(1, 128);
      if (!ok) break;
      tc_fence_after();
      const uint32_t taddr_row = tmem_base + ((uint32_t)(quarter * 32) << 16) + (uint32_t)(acc * p.bn);

      if (p.splits == 1) {
        const int nsteps = ChunkPlan<EPI, TRANS>::steps(p.bn);
        for (int st = 0; st < nsteps; ++st) {
          int ca, cb, cw, cout;
          ChunkPlan<EPI, TRANS>::step(st, p.bn, ca, cb, cw, cout);
          tmem_chunk_to_smem(taddr_row, ca, cw, slot0, row);
          if (cb >= 0) tmem_chunk_to_smem(taddr_row, cb, cw, slot1, row);
          if (st == nsteps - 1) {
            tc_fence_before();
            mbar_arrive(&s.tempty[acc]);
          }
          named_bar_sync(1, 128);
          finalize_chunk<EPI, TRANS>(p, slot0, slot1, un.tm, un.tn, cout, cw, et);
          named_bar_sync(1, 128);
        }
      } else {
        // split-K: write this split's fp32 partial tile, then take a ticket
        float* ws = p.workspace + ((size_t)un.split * tiles + un.tile) * (size_t)BM * p.bn;
        for (int c = 0; c < p.bn; c += 16) {
          uint32_t r[16];
          tmem_ld16(taddr_row + c, r);
          tmem_ld_wait();
          float4* dst = reinterpret_cast<float4*>(ws + (size_t)row * p.bn + c);
#pragma unroll
          for (int i = 0; i < 4; ++i)
            dst[i] = make_float4(__uint_as_float(r[4 * i]), __uint_as_float(r[4 * i + 1]),
                                 __uint_as_float(r[4 * i + 2]), __uint_as_float(r[4 * i + 3]));
        }
        tc_fence_before();
        mbar_arrive(&s.tempty[acc]);
        __threadfence();
        named_bar_sync(1, 128);
        if (et == 0) {
          int ticket = atomicAdd(&p.counters[un.tile], 1);
          int last = (ticket == p.splits - 1);
          if (last) p.counters[un.tile] = 0;
          *s.epi_flag = last;
        }
        named_bar_sync(1, 128);
        const int last = *s.epi_flag;
        named_bar_sync(1, 128);
        if (last) {
          __threadfence();
          const int nsteps = ChunkPlan<EPI, TRANS>::steps(p.bn);
          const size_t split_stride = (size_t)tiles * BM * p.bn;
          const float* ws0 = p.workspace + (size_t)un.tile * BM * p.bn;
          for (int st = 0; st < nsteps; ++st) {
            int ca, cb, cw, cout;
            ChunkPlan<EPI, TRANS>::step(st, p.bn, ca, cb, cw, cout);
            for (int idx = et; idx < BM * cw; idx += 128) {
              int r = idx / cw, c = idx - r * cw;
              float a = 0.f, b = 0.f;
              for (int sp = 0; sp < p.splits; ++sp) {
                const float* w = ws0 + sp * split_stride + (size_t)r * p.bn;
                a += __ldcg(w + ca + c);
                if (cb >= 0) b += __ldcg(w + cb + c);
              }
              slot0[r * EPI_LD + c] = a;
              if (cb >= 0) slot1[r * EPI_LD + c] = b;
            }
            named_bar_sync(1, 128);
            finalize_chunk<EPI, TRANS>(p, slot0, slot1, un.tm, un.tn, cout, cw, et);
            named_bar_sync(1, 128);
          }
        }
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, p.tmem_cols);
  }
}

// ----------------------------------------------------------------------------------------------
// host side
// ----------------------------------------------------------------------------------------------
static int num_sms_cached(int dev) {
  static int cache[64] = {0};
  if (!cache[dev]) {
    cudaDeviceProp prop;
    cudaGetDeviceProperties(&prop, dev);
    cache[dev] = prop.multiProcessorCount;
  }
  return cache[dev];
}

static uint32_t tmem_cols_for(int bn) {
  uint32_t need = 2 * bn, c = 32;
  while (c < need) c <<= 1;
  return c;
}

template <int EPI, bool TRANS>
static void launch_typed(const CUtensorMap& ta, const CUtensorMap& tb, const GemmParams& p, int grid, size_t smem,
                         cudaStream_t stream) {
  auto kern = gemm_tcgen05_kernel<EPI, TRANS>;
  static bool configured[64] = {false};
  int dev;
  cudaGetDevice(&dev);
  if (!configured[dev]) {
    cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, 232448);
    configured[dev] = true;
  }
  kern<<<grid, NUM_THREADS, smem, stream>>>(ta, tb, p);
}

// Choose BN for a problem: decode (swap-AB) uses the token count rounded to 16, prefill 256 (or
// 128 when N is small); SiLU in normal orientation needs BN a multiple of 128.
int gemm_pick_bn(int N, int epi, bool trans) {
  if (trans) {
    int bn = (N + 15) / 16 * 16;
    return bn < 16 ? 16 : (bn > 256 ? 256 : bn);
  }
  if (epi == EPI_SILU_BF16) return N >= 256 ? 256 : 128;
  return N >= 192 ? 256 : (N >= 96 ? 128 : ((N + 15) / 16 * 16));
}

int gemm_pick_splits(int M, int N, int K, int bn, int num_sms) {
  int m_tiles = (M + BM - 1) / BM, n_tiles = (N + bn - 1) / bn;
  int tiles = m_tiles * n_tiles;
  int k_blocks = (K + BK - 1) / BK;
  if (tiles >= num_sms / 2) return 1;
  int splits = num_sms / tiles;
  int max_splits = k_blocks / 2 > 0 ? k_blocks / 2 : 1;  // keep at least two k-blocks per split
  if (splits > max_splits) splits = max_splits;
  if (splits > 32) splits = 32;
  return splits < 1 ? 1 : splits;
}

// out = A @ B^T (normal) or out^T = A @ B^T (trans). Returns nothing; errors go to `err`.
void gemm_tcgen05(const at::Tensor& A, const at::Tensor& B, at::Tensor& out, int64_t epi, bool trans, int64_t bn_req,
                  int64_t splits_req, at::Tensor& workspace, at::Tensor& counters, at::Tensor& err) {
  TORCH_CHECK(A.is_cuda() && B.is_cuda() && out.is_cuda(), "gemm_tcgen05: tensors must be CUDA");
  TORCH_CHECK(A.scalar_type() == at::kBFloat16 && B.scalar_type() == at::kBFloat16, "gemm_tcgen05: bf16 operands");
  TORCH_CHECK(A.dim() == 2 && B.dim() == 2 && A.size(1) == B.size(1), "gemm_tcgen05: A [M,K], B [N,K]");
  TORCH_CHECK(A.stride(1) == 1 && B.stride(1) == 1, "gemm_tcgen05: K must be contiguous");
  TORCH_CHECK((A.stride(0) * 2) % 16 == 0 && (B.stride(0) * 2) % 16 == 0, "gemm_tcgen05: row pitch % 16 bytes");
  TORCH_CHECK(out.stride(-1) == 1, "gemm_tcgen05: out inner dim contiguous");
  const c10::cuda::CUDAGuard guard(A.device());
  int dev = A.get_device();
  const int M = A.size(0), N = B.size(0), K = A.size(1);
  if (M == 0 || N == 0) return;
  GemmParams p{};
  p.M = M;
  p.N = N;
  p.K = K;
  int bn = bn_req > 0 ? (int)bn_req : gemm_pick_bn(N, (int)epi, trans);
  TORCH_CHECK(bn % 16 == 0 && bn >= 16 && bn <= 256, "gemm_tcgen05: BN must be a multiple of 16 in [16,256]");
  if (epi == EPI_SILU_BF16 && !trans) TORCH_CHECK(bn % 128 == 0, "SiLU epilogue needs BN % 128 == 0");
  if (epi == EPI_SILU_BF16) TORCH_CHECK((trans ? M : N) % 128 == 0, "SiLU epilogue: feature dim % 128");
  p.bn = bn;
  p.m_tiles = (M + BM - 1) / BM;
  p.n_tiles = (N + bn - 1) / bn;
  p.k_blocks = (K + BK - 1) / BK;
  const int sms = num_sms_cached(dev);
  int splits = splits_req > 0 ? (int)splits_req : gemm_pick_splits(M, N, K, bn, sms);
  if (splits > p.k_blocks) splits = p.k_blocks;
  p.splits = splits;
  const int tiles = p.m_tiles * p.n_tiles;
  if (splits > 1) {
    TORCH_CHECK(workspace.numel() >= (int64_t)splits * tiles * BM * bn && workspace.scalar_type() == at::kFloat,
                "gemm_tcgen05: workspace too small for split-K (need ", (int64_t)splits * tiles * BM * bn, " floats)");
    TORCH_CHECK(counters.numel() >= tiles && counters.scalar_type() == at::kInt, "gemm_tcgen05: counters too small");
    p.workspace = workspace.data_ptr<float>();
    p.counters = counters.data_ptr<int>();
  }
  const size_t budget = 232448;
  int stages = 8;
  while (stages > 2 && gemm_smem_bytes(stages, bn) > budget) --stages;
  p.stages = stages;
  p.out = out.data_ptr();
  p.ldo = out.stride(0);
  p.err = err.data_ptr<int>();
  p.idesc = make_idesc_bf16(BM, bn);
  p.tmem_cols = tmem_cols_for(bn);

  CUtensorMap ta = tma_map_2d_bf16(A.data_ptr(), K, M, A.stride(0), BK, BM);
  CUtensorMap tb = tma_map_2d_bf16(B.data_ptr(), K, N, B.stride(0), BK, bn);
  const int units = tiles * splits;
  const int grid = units < sms ? units : sms;
  const size_t smem = gemm_smem_bytes(stages, bn);
  cudaStream_t stream = at::cuda::getCurrentCUDAStream();
  switch (epi * 2 + (trans ? 1 : 0)) {
    case EPI_STORE_BF16 * 2 + 0: launch_typed<EPI_STORE_BF16, false>(ta, tb, p, grid, smem, stream); break;
    case EPI_STORE_BF16 * 2 + 1: launch_typed<EPI_STORE_BF16, true>(ta, tb, p, grid, smem, stream); break;
    case EPI_STORE_F32 * 2 + 0: launch_typed<EPI_STORE_F32, false>(ta, tb, p, grid, smem, stream); break;
    case EPI_STORE_F32 * 2 + 1: launch_typed<EPI_STORE_F32, true>(ta, tb, p, grid, smem, stream); break;
    case EPI_SILU_BF16 * 2 + 0: launch_typed<EPI_SILU_BF16, false>(ta, tb, p, grid, smem, stream); break;
    case EPI_SILU_BF16 * 2 + 1: launch_typed<EPI_SILU_BF16, true>(ta, tb, p, grid, smem, stream); break;
    default: TORCH_CHECK(false, "gemm_tcgen05: unknown epilogue ", epi);
  }
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

std::vector<int64_t> gemm_plan(int64_t M, int64_t N, int64_t K, int64_t epi, bool trans, int64_t device) {
  int bn = gemm_pick_bn((int)N, (int)epi, trans);
  int sms = num_sms_cached((int)device);
  int splits = gemm_pick_splits((int)M, (int)N, (int)K, bn, sms);
  int kb = (int)((K + BK - 1) / BK);
  if (splits > kb) splits = kb;
  int tiles = (int)(((M + BM - 1) / BM) * ((N + bn - 1) / bn));
  int stages = 8;
  while (stages > 2 && gemm_smem_bytes(stages, bn) > 232448) --stages;
  return {bn, splits, (int64_t)splits * tiles * BM * bn, tiles, stages};
}

}  // namespace mesh
