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
// Scheduling: whole tiles round-robin over a persistent grid, plus stream-K for the tail waves:
// k-iterations are split evenly over the CTAs; contributors to a tile publish fp32 partials and
// the tile's owner CTA (the one holding its first k-block) adds them to its own TMEM accumulator
// in a fixed order. Swap-AB problems with fewer tiles than SMs (decode, and every tensor-parallel
// shard of it) use cluster split-K instead: a thread-block cluster of C CTAs shares one output
// tile, each CTA accumulates 1/C of the k-range in its own TMEM, stages it in its shared memory,
// and after one cluster barrier every CTA sums its slice of the tile's columns over the C CTAs
// through distributed shared memory (fixed order, deterministic) and runs the epilogue on it.
//
// Epilogues: bf16 store, f32 store, and SiLU(gate)*up for gate/up weights interleaved in blocks
// of 64 features (rows g0..63,u0..63,g64..127,...), which writes half as many features.
//
// No TMA multicast is used. All mbarrier waits are bounded (see sm100.cuh).
#include <ATen/ATen.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/extension.h>

#include <algorithm>
#include <cstdlib>
#include <mutex>
#include <unordered_map>

#include "../include/sm100.cuh"
#include "../include/tma_host.h"
#include "../include/launch.h"

namespace mesh {

enum EpiKind : int { EPI_STORE_BF16 = 0, EPI_STORE_F32 = 1, EPI_SILU_BF16 = 2, EPI_ARGMAX = 3, EPI_QKV_ROPE = 4 };

constexpr int BM = 128;
constexpr int BK = 64;
constexpr int A_STAGE_BYTES = BM * BK * 2;     // 16 KB
constexpr int EPI_LD = 33;                      // padded fp32 row stride of the epilogue staging tile
constexpr int EPI_SLOT_FLOATS = BM * EPI_LD;
constexpr int NUM_THREADS = 192;
constexpr uint64_t WAIT_LIMIT_NS = 2000000000ull;  // 2 s: far above any legal wait

// Fused tensor-parallel all-reduce tail of a decode o_proj / down_proj GEMM (swap-AB, bf16 out).
// The epilogue pushes each token row of the partial product to the rank that owns the row (a
// near-equal split of the T rows over the ranks) over NVLink; the tail then reduces the owned rows
// over the ranks' pushed partials, adds the residual, applies RMSNorm and writes the normed rows
// into every rank (NVLS multicast store, or one peer store per rank), all inside the same launch.
constexpr int AR_TAIL_MAX_RANKS = 8;
// %globaltimer stamps per CTA: 0-15 GEMM phases, 16-21 the fused all-reduce tail
constexpr int TRACE_SLOTS = 32;
struct ArTail {
  int on;
  int rank, world, T, H, t_max;
  unsigned long long ws[AR_TAIL_MAX_RANKS];  // symmetric workspace base of every rank (as mapped here)
  unsigned long long mc;                     // multicast base of the workspace (0: plain peer stores)
  long off_flags;    // uint32 [2 phases][AR_TAIL_MAX_RANKS sources][AR_TAIL_MAX_CTAS], in every rank's workspace
  long off_counts;   // unused (kept so the configuration table keeps its layout)
  long off_push;     // bf16 [world sources][t_max][H] pushed partial rows (this call's parity)
  long off_resid;    // bf16 [t_max][H] residual; a rank keeps its owned rows current
  long off_normed;   // bf16 [t_max][H] normed rows, complete on every rank after the launch
  uint32_t* epoch;   // local epoch word, bumped once per launch
  const __nv_bfloat16* gamma;
  float eps;
  unsigned long long timeout_ns;
};

struct GemmParams {
  int M, N, K;
  int m_tiles, n_tiles, k_blocks;
  int dp_tiles;       // tiles [0, dp_tiles) are owned whole, round-robin over the grid
  int sk_iters_per_cta;  // stream-K share of the remaining tiles' k-iterations (0: none)
  int bn, stages;
  int ck;             // cluster split-K: CTAs per cluster sharing one tile (<= 1: off)
  int epi_bytes;      // shared memory of the epilogue region (staging, or split-K receive buffers)
  int vec_out;        // output rows start 16-byte aligned: whole-tile epilogue may store 16 bytes at once
  int direct_epi;     // whole tiles go TMEM -> registers -> global (else staged through shared memory)
  // EPI_QKV_ROPE (swap-AB qkv projection, one 128-row tile = one head of 128 dims): RoPE on q and k
  // heads from cos/sin tables at each token's position, q heads to `out` [T, hq*128], k and v heads
  // straight into the paged KV pool [pages, hkv, page_size, 128] at each token's slot (< 0: skip)
  const int* rope_pos;
  const long* rope_slot;
  const float* rope_cos;
  const float* rope_sin;
  __nv_bfloat16* rope_k;
  __nv_bfloat16* rope_v;
  int rope_hq, rope_hkv, rope_ps;
  int kbox;           // 64-wide k boxes per pipeline stage (1 or 2); a k-block is 64 * kbox wide
  void* out;
  long ldo;
  float* workspace;   // stream-K partial tiles: slot (sk_tile + cta) x [BM][bn] fp32
  int* counters;      // [stream-K tiles], zero on entry, left zero on exit
  int* err;
  uint32_t idesc;
  uint32_t tmem_cols;
  unsigned long long* trace;  // optional [grid][TRACE_SLOTS] %globaltimer stamps (nullptr: off)
  // Fused reduce-scatter: instead of `out`, bf16 rows go to slot `my_rank` of the destination
  // rank's symmetric buffer over NVLink (1: each token row to its owner rank, 2: to every rank).
  int push_mode, my_rank, world, push_rows;
  long slot_stride;                  // elements between source slots in a destination buffer
  unsigned long long peer_base[8];   // destination buffer base (as mapped here) per rank
  ArTail ar;
};

// owner rank of token row t when `rows` tokens are split into `world` near-equal ranges
__device__ __forceinline__ int row_owner(int t, int rows, int world) {
  const int base = rows / world, extra = rows % world;
  const int big = extra * (base + 1);
  if (t < big) return t / (base + 1);
  return extra + (base > 0 ? (t - big) / base : 0);
}

// store two adjacent bf16 outputs of token row `tok`, feature `f` (f even)
__device__ __forceinline__ void store_out2(const GemmParams& p, int tok, int f, uint32_t v) {
  if (p.push_mode == 0) {
    *reinterpret_cast<uint32_t*>(reinterpret_cast<__nv_bfloat16*>(p.out) + (long)tok * p.ldo + f) = v;
    return;
  }
  const long off = (long)p.my_rank * p.slot_stride + (long)tok * p.ldo + f;
  if (p.push_mode == 1) {
    const int d = row_owner(tok, p.push_rows, p.world);
    *reinterpret_cast<uint32_t*>(reinterpret_cast<__nv_bfloat16*>(p.peer_base[d]) + off) = v;
  } else {
    for (int d = 0; d < p.world; ++d)
      *reinterpret_cast<uint32_t*>(reinterpret_cast<__nv_bfloat16*>(p.peer_base[d]) + off) = v;
  }
}

struct Smem {
  uint8_t* a;
  uint8_t* b;
  float* epi;
  uint64_t* full;
  uint64_t* empty;
  uint64_t* tfull;
  uint64_t* tempty;
  uint64_t* fixbar;   // stream-K owner: partial tiles landed
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
  ptr += (size_t)p.stages * A_STAGE_BYTES * p.kbox;
  s.b = ptr;
  ptr += (size_t)p.stages * p.bn * BK * 2 * p.kbox;
  s.epi = reinterpret_cast<float*>(ptr);
  ptr += p.epi_bytes;
  ptr = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(ptr) + 7) & ~uintptr_t(7));
  s.full = reinterpret_cast<uint64_t*>(ptr);
  s.empty = s.full + p.stages;
  s.tfull = s.empty + p.stages;
  s.tempty = s.tfull + 2;
  s.fixbar = s.tempty + 2;
  s.tmem_base = reinterpret_cast<uint32_t*>(s.fixbar + 1);
  s.abort_flag = reinterpret_cast<int*>(s.tmem_base + 1);
  s.epi_flag = s.abort_flag + 1;
  return s;
}

constexpr int EPI_STAGING_BYTES = 2 * EPI_SLOT_FLOATS * (int)sizeof(float);
constexpr size_t SMEM_BUDGET = 232448;

__host__ __device__ inline size_t gemm_smem_bytes(int stages, int bn, int epi_bytes = EPI_STAGING_BYTES, int kbox = 1) {
  return 1024 + (size_t)stages * (A_STAGE_BYTES + bn * BK * 2) * kbox + (size_t)epi_bytes + 8 +
         (size_t)(2 * stages + 5) * 8 + 16;
}

// columns of the tile each CTA of a C-way cluster split owns, and its receive buffers' size
__host__ __device__ inline int ck_cols(int bn, int C) { return ((bn + C - 1) / C + 3) & ~3; }
__host__ __device__ inline int ck_recv_bytes(int bn, int C) { return C * BM * (ck_cols(bn, C) + 4) * 4; }

// A segment is a contiguous k-range of one output tile processed by one CTA. Data-parallel
// tiles are single segments; stream-K tiles are split across the CTAs whose k-iteration ranges
// cover them ("contributors", fixed by the static partition, so results are deterministic).
struct Seg {
  int tile, tm, tn, kb0, kb1;
  int sk_tile;     // -1 for whole tiles
  int contrib, ncontrib, first_cta;
};

__device__ __forceinline__ void tile_coords(int t, const GemmParams& p, int& tm, int& tn) {
  // grouped raster: 8 consecutive m-tiles sweep all n-tiles before the next group
  const int G = 8;
  const int group_size = G * p.n_tiles;
  const int g = t / group_size;
  const int first_m = g * G;
  const int gm = min(p.m_tiles - first_m, G);
  const int in = t - g * group_size;
  tm = first_m + in % gm;
  tn = in / gm;
}

struct SegIter {
  int i;          // next data-parallel tile ordinal of this CTA
  long g;         // next stream-K global iteration
  long g_end;
  __device__ void init(const GemmParams& p) {
    i = 0;
    g = (long)blockIdx.x * p.sk_iters_per_cta;
    const long sk_total = (long)(p.m_tiles * p.n_tiles - p.dp_tiles) * p.k_blocks;
    g_end = min(g + (long)p.sk_iters_per_cta, sk_total);
    if (p.sk_iters_per_cta == 0) g_end = g;
  }
  __device__ bool next(const GemmParams& p, Seg& s) {
    if (p.ck > 1) {
      // cluster split-K: one segment per CTA, k-range share `rank` of the cluster's tile
      if (i > 0) return false;
      ++i;
      const int C = p.ck;
      const int rank = (int)(blockIdx.x % C);
      s.tile = (int)(blockIdx.x / C);
      tile_coords(s.tile, p, s.tm, s.tn);
      s.kb0 = (int)((long)rank * p.k_blocks / C);
      s.kb1 = (int)((long)(rank + 1) * p.k_blocks / C);
      s.sk_tile = -1;
      s.contrib = rank;
      s.ncontrib = C;
      s.first_cta = 0;
      return true;
    }
    const int t_dp = blockIdx.x + i * gridDim.x;
    if (t_dp < p.dp_tiles) {
      ++i;
      s.tile = t_dp;
      tile_coords(t_dp, p, s.tm, s.tn);
      s.kb0 = 0;
      s.kb1 = p.k_blocks;
      s.sk_tile = -1;
      s.contrib = 0;
      s.ncontrib = 1;
      s.first_cta = 0;
      return true;
    }
    if (g >= g_end) return false;
    const int kb = p.k_blocks;
    const long W = p.sk_iters_per_cta;
    const int st = (int)(g / kb);
    const int k0 = (int)(g - (long)st * kb);
    const long tile_end = (long)(st + 1) * kb;
    const long seg_end = min(tile_end, g_end);
    s.sk_tile = st;
    s.tile = p.dp_tiles + st;
    tile_coords(s.tile, p, s.tm, s.tn);
    s.kb0 = k0;
    s.kb1 = k0 + (int)(seg_end - g);
    const int first = (int)(((long)st * kb) / W);
    const int last = (int)((tile_end - 1) / W);
    s.first_cta = first;
    s.contrib = blockIdx.x - first;
    s.ncontrib = last - first + 1;
    g = seg_end;
    return true;
  }
};

// ----------------------------------------------------------------------------------------------
// epilogue helpers: the epilogue stages 128 x (<=32) fp32 chunks in smem, then writes them with a
// thread mapping chosen for coalescing in each orientation.
// ----------------------------------------------------------------------------------------------
template <int EPI, bool TRANS>
__device__ __forceinline__ void finalize_chunk(const GemmParams& p, uint32_t slot0, uint32_t slot1,
                                               int tm, int tn, int c0, int cw, int et) {
  // slot0/slot1: shared-window addresses of the staged fp32 chunks ([BM][EPI_LD])
  auto S0 = [&](int r, int c) { return lds_f32(slot0 + (uint32_t)(r * EPI_LD + c) * 4); };
  auto S1 = [&](int r, int c) { return lds_f32(slot1 + (uint32_t)(r * EPI_LD + c) * 4); };
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
        float g0 = S0(r, c), g1 = S0((r + 1), c);
        float u0 = S0((r + 64), c), u1 = S0((r + 65), c);
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
        float g0 = S0(r, cp), g1 = S0(r, cp + 1);
        float u0 = S1(r, cp), u1 = S1(r, cp + 1);
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
        float a = S0((rp * 2), c);
        float b = (m + 1 < p.M) ? S0((rp * 2 + 1), c) : 0.f;
        if (m + 1 < p.M)
          store_out2(p, n, m, pack_bf16x2(a, b));
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
        float a = S0(r, cp), b = S0(r, cp + 1);
        if (n + 1 < p.N)
          store_out2(p, m, n, pack_bf16x2(a, b));
        else
          out[(long)m * p.ldo + n] = f2bf(a);
      }
    }
  } else if constexpr (EPI == EPI_ARGMAX) {
    // swap-AB LM head: rows are vocabulary entries, columns tokens. Per token keep the max over
    // this tile's 128 rows (first index on ties); out is float2 [m_tiles][ldo] (value, index bits).
    static_assert(TRANS, "argmax epilogue runs in swap-AB orientation");
    const int c = et >> 2, q = et & 3;
    if (c < cw) {
      const int n = tn * p.bn + c0 + c;
      float best = -INFINITY;
      int bi = 0x7fffffff;
      for (int r = q * 32; r < q * 32 + 32; ++r) {
        const int m = m_base + r;
        if (m < p.M) {
          const float v = S0(r, c);
          if (v > best) {
            best = v;
            bi = m;
          }
        }
      }
#pragma unroll
      for (int o = 1; o <= 2; o <<= 1) {
        const float ov = __shfl_xor_sync(0xffffffffu, best, o);
        const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
        if (ov > best || (ov == best && oi < bi)) {
          best = ov;
          bi = oi;
        }
      }
      if (q == 0 && n < p.N)
        reinterpret_cast<float2*>(p.out)[(long)tm * p.ldo + n] = make_float2(best, __int_as_float(bi));
    }
  } else {  // EPI_STORE_F32
    float* out = reinterpret_cast<float*>(p.out);
    if constexpr (TRANS) {
      for (int idx = et; idx < BM * cw; idx += 128) {
        int r = idx & 127, c = idx >> 7;
        int n = tn * p.bn + c0 + c;
        int m = m_base + r;
        if (n >= p.N || m >= p.M) continue;
        out[(long)n * p.ldo + m] = S0(r, c);
      }
    } else {
      for (int idx = et; idx < BM * cw; idx += 128) {
        int r = idx / cw, c = idx - r * cw;
        int m = m_base + r;
        int n = tn * p.bn + c0 + c;
        if (m >= p.M || n >= p.N) continue;
        out[(long)m * p.ldo + n] = S0(r, c);
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

__device__ __forceinline__ void tmem_chunk_to_smem(uint32_t taddr_row, int col, int cw, uint32_t slot, int row) {
  uint32_t r[16];
  const uint32_t base = slot + (uint32_t)(row * EPI_LD) * 4;
  tmem_ld16(taddr_row + col, r);
  tmem_ld_wait();
#pragma unroll
  for (int i = 0; i < 16; ++i) sts_f32(base + i * 4, __uint_as_float(r[i]));
  if (cw > 16) {
    tmem_ld16(taddr_row + col + 16, r);
    tmem_ld_wait();
#pragma unroll
    for (int i = 0; i < 16; ++i) sts_f32(base + (16 + i) * 4, __uint_as_float(r[i]));
  }
}

// ----------------------------------------------------------------------------------------------
// cluster split-K epilogue (swap-AB orientation only). Every CTA of the cluster holds a partial
// accumulator of the same 128 x bn tile for its share of the k-range. The tile's columns are
// dealt out to the CTAs (CTA k owns columns [k * cpc, k * cpc + cpc), cpc = bn / C rounded up to
// 4). Each thread reads its accumulator row out of TMEM and stores every column group straight
// into the owning CTA's receive buffer through distributed shared memory (remote stores are
// posted, nothing waits on a round trip): owner k's buffer is [C sources][128 rows][cpc + 4]
// fp32 in its epilogue region, which nothing else uses in this mode (the operand ring may still
// be busy in a slower peer). Every thread arrived on the cluster barrier at kernel start and
// waits on it before its first remote store, so no CTA writes into a peer that has not started.
// A second cluster barrier (release/acquire) makes the stores visible; then every CTA sums its
// columns over the C sources in source order (deterministic) from local shared memory and runs
// the epilogue. Both barriers are reached on every path, errors included.
// ----------------------------------------------------------------------------------------------
// Swap-AB bf16 output through shared memory: the tile's rows are output features and its columns
// tokens, so a thread holds one feature of many tokens; written straight to global memory that is
// one 2-byte store per token per thread, which measured ~25 ns each (1.6 us for a 64-token tile).
// Instead each thread puts its values into a [ncols tokens][fw features] bf16 staging tile
// (conflict-free: a warp writes 64 contiguous bytes), and after a named barrier the 128 epilogue
// threads write whole 16-byte chunks of token rows (a warp covers 2-4 rows of 128-256 contiguous
// bytes). `f0` is the first output feature of the tile, `n0` its first token.
__device__ __forceinline__ void stage_put_bf16(uint32_t stage, int fw, int j, int f, float v) {
  __nv_bfloat16 b = f2bf(v);
  sts_u16(stage + (uint32_t)(j * fw + f) * 2, *reinterpret_cast<uint16_t*>(&b));
}
__device__ __forceinline__ void stage_flush_bf16(const GemmParams& p, uint32_t stage, int fw, int ncols, int n0,
                                                 int f0, int f_lim, int et) {
  named_bar_sync(1, 128);
  __nv_bfloat16* out = reinterpret_cast<__nv_bfloat16*>(p.out);
  const int cpr = fw / 8;  // 16-byte chunks per token row
  for (int k = et; k < ncols * cpr; k += 128) {
    const int j = k / cpr, c8 = (k - j * cpr) * 8;
    const int n = n0 + j, f = f0 + c8;
    if (n >= p.N || f >= f_lim) continue;
    const uint4 v = lds_u4(stage + (uint32_t)(j * fw + c8) * 2);
    if (p.push_mode != 0) {
      // fused reduce-scatter: the token row goes to slot `my_rank` of its owner rank (mode 1) or
      // of every rank (mode 2), over NVLink; rows there are 16-byte aligned (H % 8 == 0)
      const long off = (long)p.my_rank * p.slot_stride + (long)n * p.ldo + f;
      if (p.push_mode == 1) {
        const int d = row_owner(n, p.push_rows, p.world);
        *reinterpret_cast<uint4*>(reinterpret_cast<__nv_bfloat16*>(p.peer_base[d]) + off) = v;
      } else {
        for (int d = 0; d < p.world; ++d)
          *reinterpret_cast<uint4*>(reinterpret_cast<__nv_bfloat16*>(p.peer_base[d]) + off) = v;
      }
      continue;
    }
    __nv_bfloat16* dst = out + (long)n * p.ldo + f;
    if (p.vec_out && f + 8 <= f_lim) {
      *reinterpret_cast<uint4*>(dst) = v;
    } else {
      const __nv_bfloat16* e = reinterpret_cast<const __nv_bfloat16*>(&v);
      for (int i = 0; i < 8 && f + i < f_lim; ++i) dst[i] = e[i];
    }
  }
  named_bar_sync(1, 128);  // staging tile free for the next block
}

// One head's worth of rotated (q, k) or plain (v) token rows, staged [ncols][128] bf16, written to
// the q output or the paged KV pool as 16-byte chunks (a token's 128 dims are 256 contiguous bytes
// in both layouts).
__device__ __forceinline__ void stage_flush_qkv(const GemmParams& p, uint32_t stage, int ncols, int n0, int hd,
                                                int et) {
  named_bar_sync(1, 128);
  for (int k = et; k < ncols * 16; k += 128) {
    const int j = k >> 4, c8 = (k & 15) * 8;
    const int n = n0 + j;
    if (n >= p.N) continue;
    __nv_bfloat16* dst;
    if (hd < p.rope_hq) {
      dst = reinterpret_cast<__nv_bfloat16*>(p.out) + (long)n * p.ldo + (long)hd * 128 + c8;
    } else {
      const long sl = p.rope_slot[n];
      if (sl < 0) continue;
      const long page = sl / p.rope_ps, off = sl - page * p.rope_ps;
      const bool is_k = hd < p.rope_hq + p.rope_hkv;
      const int kh = is_k ? hd - p.rope_hq : hd - p.rope_hq - p.rope_hkv;
      dst = (is_k ? p.rope_k : p.rope_v) + ((page * p.rope_hkv + kh) * p.rope_ps + off) * 128 + c8;
    }
    *reinterpret_cast<uint4*>(dst) = lds_u4(stage + (uint32_t)(j * 128 + c8) * 2);
  }
  named_bar_sync(1, 128);
}

// Half-split RoPE of dim d (0..127) of one head at token position `pos`: x is this dim's value,
// y the value of dim d ^ 64 (both already rounded to bf16, as an unfused bf16 qkv buffer would be).
__device__ __forceinline__ float rope_rotate(const GemmParams& p, int d, int pos, float x, float y) {
  const int i = d & 63;
  const float c = p.rope_cos[(long)pos * 64 + i], sn = p.rope_sin[(long)pos * 64 + i];
  return d < 64 ? x * c - y * sn : y * sn + x * c;
}

__device__ __forceinline__ float bf16_round(float v) { return bf2f(f2bf(v)); }

// ----------------------------------------------------------------------------------------------
// Whole-tile epilogue straight from TMEM to global memory (no shared-memory staging): each thread
// owns one accumulator row (TMEM lane). Swap-AB: the row is an output feature and its columns are
// tokens, so for every token the 32 lanes of a warp write 32 consecutive features (64 B bf16).
// Normal orientation: the row is a token and its 16-column groups are 32 contiguous bytes, written
// as 16-byte vectors. SiLU in swap-AB pairs gate row r with up row r + 64, which lives in another
// warp: the up warps hand their columns over in shared memory (double-buffered). The greedy-head
// epilogue reduces (max, first index) per token over the 128 rows with warp shuffles and a
// 4-entry cross-warp step. Columns are read from TMEM up to 64 at a time behind a single
// tcgen05.wait (a wait per 16 columns cost ~2 us per tile); the buffer is released right after
// its last column is read.
// `fetch(col, r, n16)` fills r[0 .. 16*n16) with this thread's row at columns [col, col + 16*n16):
// straight from TMEM for whole tiles, or TMEM plus the other contributors' partials (added in a
// fixed order) for a stream-K tile's owner.
// ----------------------------------------------------------------------------------------------
template <int EPI, bool TRANS, typename Fetch>
__device__ __forceinline__ void direct_epilogue(const GemmParams& p, const Smem& s, Fetch&& fetch, int row,
                                                int lane, int quarter, int tm, int tn, uint64_t* tempty) {
  const int m_base = tm * BM;
  // SiLU hand-over [2][2][64][17] words + output staging [64][64] bf16 / argmax partials [2][4][64] x
  // (value, index) / swap-AB bf16 output staging [64][128]
  float* xbuf = s.epi;
  int blk = 0;
  auto release_if_last = [&](int c_end) {
    if (c_end >= p.bn) {
      tc_fence_before();
      mbar_arrive(tempty);
    }
  };
  if constexpr (EPI == EPI_SILU_BF16 && !TRANS) {
    // gate columns g*128 + [0, 64), up columns g*128 + 64 + [0, 64); output column tn*bn/2 + g*64 + j
    __nv_bfloat16* out = reinterpret_cast<__nv_bfloat16*>(p.out);
    const int m = m_base + row;
    for (int c = 0; c < p.bn / 2; c += 32) {
      const int g = c / 64, j0 = c % 64;
      uint32_t rg[32], ru[32];
      fetch(g * 128 + j0, rg, 2);
      fetch(g * 128 + 64 + j0, ru, 2);
      if (c + 32 >= p.bn / 2) {
        tc_fence_before();
        mbar_arrive(tempty);
      }
      if (m >= p.M) continue;
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        const int n0 = tn * (p.bn / 2) + c + 16 * h;
        uint32_t pk[8];
#pragma unroll
        for (int i = 0; i < 8; ++i)
          pk[i] = pack_bf16x2(silu_f(__uint_as_float(rg[16 * h + 2 * i])) * __uint_as_float(ru[16 * h + 2 * i]),
                              silu_f(__uint_as_float(rg[16 * h + 2 * i + 1])) * __uint_as_float(ru[16 * h + 2 * i + 1]));
        __nv_bfloat16* dst = out + (long)m * p.ldo + n0;
        if (p.vec_out && n0 + 16 <= p.N / 2) {
          reinterpret_cast<uint4*>(dst)[0] = make_uint4(pk[0], pk[1], pk[2], pk[3]);
          reinterpret_cast<uint4*>(dst)[1] = make_uint4(pk[4], pk[5], pk[6], pk[7]);
        } else {
          for (int i = 0; i < 16 && n0 + i < p.N / 2; ++i)
            dst[i] = f2bf(silu_f(__uint_as_float(rg[16 * h + i])) * __uint_as_float(ru[16 * h + i]));
        }
      }
    }
  } else if constexpr (EPI == EPI_SILU_BF16 && TRANS) {
    const bool up = row >= 64;
    const int q = row & 63;
    for (int c = 0; c < p.bn; c += 64, ++blk) {
      const int n16 = min(4, (p.bn - c + 15) / 16);
      uint32_t r[64];
      fetch(c, r, n16);
      release_if_last(c + 64);
      // Balanced exchange: gate thread q keeps columns [0, 32) of the block and receives the matching
      // "up" values; up thread q keeps columns [32, 64) and receives the matching gate values. Values
      // cross as bf16 pairs ([2 dirs][64 features][17 words]); the product is rounded to bf16 anyway.
      uint32_t* xg = reinterpret_cast<uint32_t*>(xbuf) + (blk & 1) * (2 * 64 * 17);  // gate -> up warps
      uint32_t* xu = xg + 64 * 17;                                                 // up -> gate warps
      // (register indices stay compile-time constants in both branches: no local-memory arrays)
      const uint32_t stg = smem_u32(reinterpret_cast<uint32_t*>(xbuf) + 4 * 64 * 17);  // [64 tokens][64] bf16
      if (up) {
#pragma unroll
        for (int j = 0; j < 32; j += 2)
          xu[q * 17 + j / 2] = pack_bf16x2(__uint_as_float(r[j]), __uint_as_float(r[j + 1]));
      } else {
#pragma unroll
        for (int j = 0; j < 32; j += 2)
          xg[q * 17 + j / 2] = pack_bf16x2(__uint_as_float(r[32 + j]), __uint_as_float(r[32 + j + 1]));
      }
      named_bar_sync(1, 128);
      if (up) {  // columns [32, 64): own up values, gate values received
#pragma unroll
        for (int j = 0; j < 32; j += 2) {
          if (32 + j < 16 * n16) {
            float g0, g1;
            unpack_bf16x2(xg[q * 17 + j / 2], g0, g1);
            stage_put_bf16(stg, 64, 32 + j, q, silu_f(g0) * __uint_as_float(r[32 + j]));
            stage_put_bf16(stg, 64, 32 + j + 1, q, silu_f(g1) * __uint_as_float(r[32 + j + 1]));
          }
        }
      } else {   // columns [0, 32): own gate values, up values received
#pragma unroll
        for (int j = 0; j < 32; j += 2) {
          if (j < 16 * n16) {
            float u0, u1;
            unpack_bf16x2(xu[q * 17 + j / 2], u0, u1);
            stage_put_bf16(stg, 64, j, q, silu_f(__uint_as_float(r[j])) * u0);
            stage_put_bf16(stg, 64, j + 1, q, silu_f(__uint_as_float(r[j + 1])) * u1);
          }
        }
      }
      stage_flush_bf16(p, stg, 64, 16 * n16, tn * p.bn + c, tm * (BM / 2), p.M / 2, threadIdx.x - 64);
    }
  } else if constexpr (EPI == EPI_ARGMAX) {
    static_assert(TRANS, "argmax epilogue runs in swap-AB orientation");
    const int m = m_base + row;
    const int et = (threadIdx.x - 64);
    for (int c = 0; c < p.bn; c += 64, ++blk) {
      const int n16 = min(4, (p.bn - c + 15) / 16);
      uint32_t r[64];
      fetch(c, r, n16);
      release_if_last(c + 64);
      float* rv = xbuf + (blk & 1) * 512;  // [4 quarters][64 tokens] values, then indices
      int* ri = reinterpret_cast<int*>(rv + 256);
#pragma unroll
      for (int j = 0; j < 64; ++j) {
        if (j >= 16 * n16) break;
        float best = (m < p.M) ? __uint_as_float(r[j]) : -INFINITY;
        int bi = (m < p.M) ? m : 0x7fffffff;
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
          const float ov = __shfl_xor_sync(0xffffffffu, best, o);
          const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
          if (ov > best || (ov == best && oi < bi)) {
            best = ov;
            bi = oi;
          }
        }
        if (lane == 0) {
          rv[quarter * 64 + j] = best;
          ri[quarter * 64 + j] = bi;
        }
      }
      named_bar_sync(1, 128);
      if (et < 16 * n16) {
        float best = rv[et];
        int bi = ri[et];
        for (int w = 1; w < 4; ++w) {
          const float ov = rv[w * 64 + et];
          const int oi = ri[w * 64 + et];
          if (ov > best || (ov == best && oi < bi)) {
            best = ov;
            bi = oi;
          }
        }
        const int n = tn * p.bn + c + et;
        if (n < p.N) reinterpret_cast<float2*>(p.out)[(long)tm * p.ldo + n] = make_float2(best, __int_as_float(bi));
      }
    }
  } else if constexpr (TRANS && EPI == EPI_QKV_ROPE) {
    const uint32_t xs = smem_u32(xbuf);             // [64 tokens][128 dims] bf16, before RoPE
    const uint32_t stg = xs + 64 * 128 * 2;         // [64 tokens][128 dims] bf16, rotated
    const bool rot = tm < p.rope_hq + p.rope_hkv;  // q and k heads rotate, v heads pass through
    for (int c = 0; c < p.bn; c += 64) {
      const int n16 = min(4, (p.bn - c + 15) / 16);
      uint32_t r[64];
      fetch(c, r, n16);
      release_if_last(c + 64);
#pragma unroll
      for (int j = 0; j < 64; ++j)
        if (j < 16 * n16) stage_put_bf16(xs, 128, j, row, __uint_as_float(r[j]));
      named_bar_sync(1, 128);
#pragma unroll
      for (int j = 0; j < 64; ++j) {
        if (j < 16 * n16) {
          const int n = tn * p.bn + c + j;
          float v = bf16_round(__uint_as_float(r[j]));
          if (rot && n < p.N) {
            const uint16_t y16 = lds_u16(xs + (uint32_t)(j * 128 + (row ^ 64)) * 2);
            v = rope_rotate(p, row, p.rope_pos[n], v, bf2f(*reinterpret_cast<const __nv_bfloat16*>(&y16)));
          }
          stage_put_bf16(stg, 128, j, row, v);
        }
      }
      stage_flush_qkv(p, stg, 16 * n16, tn * p.bn + c, tm, threadIdx.x - 64);
    }
  } else if constexpr (TRANS && EPI == EPI_STORE_BF16) {
    const uint32_t stg = smem_u32(xbuf);  // [64 tokens][128 features] bf16
    for (int c = 0; c < p.bn; c += 64) {
      const int n16 = min(4, (p.bn - c + 15) / 16);
      uint32_t r[64];
      fetch(c, r, n16);
      release_if_last(c + 64);
#pragma unroll
      for (int j = 0; j < 64; ++j)
        if (j < 16 * n16) stage_put_bf16(stg, BM, j, row, __uint_as_float(r[j]));
      stage_flush_bf16(p, stg, BM, 16 * n16, tn * p.bn + c, m_base, p.M, threadIdx.x - 64);
    }
  } else if constexpr (TRANS) {
    const int m = m_base + row;
    for (int c = 0; c < p.bn; c += 64) {
      const int n16 = min(4, (p.bn - c + 15) / 16);
      uint32_t r[64];
      fetch(c, r, n16);
      release_if_last(c + 64);
      if (m >= p.M) continue;
#pragma unroll
      for (int j = 0; j < 64; ++j) {
        const int n = tn * p.bn + c + j;
        if (j >= 16 * n16 || n >= p.N) break;
        if constexpr (EPI == EPI_STORE_F32)
          reinterpret_cast<float*>(p.out)[(long)n * p.ldo + m] = __uint_as_float(r[j]);
        else
          reinterpret_cast<__nv_bfloat16*>(p.out)[(long)n * p.ldo + m] = f2bf(__uint_as_float(r[j]));
      }
    }
  } else {
    const int m = m_base + row;
    for (int c = 0; c < p.bn; c += 32) {
      const int n16 = min(2, (p.bn - c + 15) / 16);
      uint32_t r[32];
      fetch(c, r, n16);
      release_if_last(c + 32);
      if (m >= p.M) continue;
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        if (h >= n16) break;
        const int n0 = tn * p.bn + c + 16 * h;
        if constexpr (EPI == EPI_STORE_F32) {
          float* dst = reinterpret_cast<float*>(p.out) + (long)m * p.ldo + n0;
          if (p.vec_out && n0 + 16 <= p.N) {
#pragma unroll
            for (int i = 0; i < 4; ++i)
              reinterpret_cast<uint4*>(dst)[i] =
                  make_uint4(r[16 * h + 4 * i], r[16 * h + 4 * i + 1], r[16 * h + 4 * i + 2], r[16 * h + 4 * i + 3]);
          } else {
            for (int i = 0; i < 16 && n0 + i < p.N; ++i) dst[i] = __uint_as_float(r[16 * h + i]);
          }
        } else {
          __nv_bfloat16* dst = reinterpret_cast<__nv_bfloat16*>(p.out) + (long)m * p.ldo + n0;
          if (p.vec_out && n0 + 16 <= p.N) {
            uint32_t pk[8];
#pragma unroll
            for (int i = 0; i < 8; ++i)
              pk[i] = pack_bf16x2(__uint_as_float(r[16 * h + 2 * i]), __uint_as_float(r[16 * h + 2 * i + 1]));
            reinterpret_cast<uint4*>(dst)[0] = make_uint4(pk[0], pk[1], pk[2], pk[3]);
            reinterpret_cast<uint4*>(dst)[1] = make_uint4(pk[4], pk[5], pk[6], pk[7]);
          } else {
            for (int i = 0; i < 16 && n0 + i < p.N; ++i) dst[i] = f2bf(__uint_as_float(r[16 * h + i]));
          }
        }
      }
    }
  }
}

template <int EPI, bool TRANS>
__device__ __forceinline__ void ck_epilogue(const GemmParams& p, const Smem& s, uint32_t tmem_base,
                                            volatile int* abort_flag, unsigned long long* trace) {
  static_assert(TRANS, "cluster split-K runs in swap-AB orientation");
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int et = threadIdx.x - 64;      // 0..127
  const int quarter = warp & 3;
  const int row = quarter * 32 + lane;  // TMEM lane this thread may read
  const int C = p.ck;
  const uint32_t rank = cluster_ctarank();
  int tm, tn;
  tile_coords((int)(blockIdx.x / C), p, tm, tn);
  const int cpc = ck_cols(p.bn, C);
  const int ldr = cpc + 4;  // padded row stride of a receive slot (floats)
  const uint32_t recv = smem_u32(s.epi);
  const uint32_t slot_bytes = (uint32_t)(BM * ldr) * 4;

  if (et == 0)
    *s.epi_flag = mbar_wait_bounded(&s.tfull[0], 0, p.err, ERR_MBAR_TIMEOUT_EPILOGUE, abort_flag, WAIT_LIMIT_NS);
  named_bar_sync(1, 128);
  const int ok = *s.epi_flag;
  tc_fence_after();
  if (trace && et == 0) trace[5] = globaltimer_ns();
  const uint32_t taddr_row = tmem_base + ((uint32_t)(quarter * 32) << 16);
  // this CTA's slot in any owner's buffer, at this thread's row
  const uint32_t my_slot_row = recv + rank * slot_bytes + (uint32_t)(row * ldr) * 4;
  cluster_wait_acquire();  // pairs with the arrive at kernel start: every peer CTA is running
  for (int c = 0; c < p.bn; c += 64) {
    const int n16 = min(4, (p.bn - c + 15) / 16);
    uint32_t r[64];
    if (ok) {
#pragma unroll
      for (int k = 0; k < 4; ++k)
        if (k < n16) tmem_ld16(taddr_row + c + 16 * k, *reinterpret_cast<uint32_t(*)[16]>(&r[16 * k]));
      tmem_ld_wait_tied(r);
    } else {
#pragma unroll
      for (int i = 0; i < 64; ++i) r[i] = 0u;
    }
#pragma unroll
    for (int i = 0; i < 64; i += 4) {
      if (i >= 16 * n16) break;
      const int col = c + i;
      const int owner = col / cpc;
      const uint32_t local = my_slot_row + (uint32_t)(col - owner * cpc) * 4;
      st_dsmem_f4(mapa_shared(local, (uint32_t)owner), __uint_as_float(r[i]), __uint_as_float(r[i + 1]),
                  __uint_as_float(r[i + 2]), __uint_as_float(r[i + 3]));
    }
  }
  tc_fence_before();
  cluster_sync();  // every partial slice has landed in its owner's buffer
  if (trace && et == 0) trace[8] = globaltimer_ns();

  const int c_lo = (int)rank * cpc;
  const int c_hi = min(p.bn, c_lo + cpc);
  // v[j] = sum over the C sources of row r, owned columns c + 4j .. c + 4j + 3 (j < nv <= 8)
  auto sum_row = [&](int r, int c, int nv, float4 (&v)[8]) {
    const uint32_t off = (uint32_t)(r * ldr + (c - c_lo)) * 4;
#pragma unroll
    for (int j = 0; j < 8; ++j) v[j] = make_float4(0.f, 0.f, 0.f, 0.f);
    for (int k = 0; k < C; ++k) {
#pragma unroll
      for (int j = 0; j < 8; ++j)
        if (j < nv) {
          const float4 y = lds_f4(recv + (uint32_t)k * slot_bytes + off + 16u * j);
          v[j].x += y.x; v[j].y += y.y; v[j].z += y.z; v[j].w += y.w;
        }
    }
  };
  const int m_base = tm * BM;
  if constexpr (EPI == EPI_SILU_BF16) {
    // rows 0..63 gate, 64..127 up; the two thread halves take alternate 16-column groups
    // staged [cpc tokens][64 features] bf16 in the idle operand ring, written as 16-byte chunks
    const uint32_t stg = smem_u32(s.a);
    const int q = et & 63, half = et >> 6;
    for (int c = c_lo + 16 * half; c < c_hi; c += 32) {
      const int nv = min(4, (c_hi - c) >> 2);
      float4 g[8], u[8];
      sum_row(q, c, nv, g);
      sum_row(q + 64, c, nv, u);
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        if (j >= nv) break;
        const float gv[4] = {g[j].x, g[j].y, g[j].z, g[j].w}, uv[4] = {u[j].x, u[j].y, u[j].z, u[j].w};
#pragma unroll
        for (int e = 0; e < 4; ++e) stage_put_bf16(stg, 64, c - c_lo + 4 * j + e, q, silu_f(gv[e]) * uv[e]);
      }
    }
    if (c_hi > c_lo) stage_flush_bf16(p, stg, 64, c_hi - c_lo, tn * p.bn + c_lo, tm * (BM / 2), p.M / 2, et);
  } else if constexpr (EPI == EPI_ARGMAX) {
    // per token column: max over the tile's 128 rows (first index on ties) -> float2 [m_tiles][ldo]
    float* red_v = reinterpret_cast<float*>(s.a);  // operand ring: idle once this CTA's MMAs completed
    int* red_i = reinterpret_cast<int*>(s.a + 16 * 4);
    const int m = m_base + et;
    for (int c = c_lo; c < c_hi; c += 4) {
      float4 v8[8];
      sum_row(et, c, 1, v8);
      const float vv[4] = {v8[0].x, v8[0].y, v8[0].z, v8[0].w};
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        float best = (m < p.M) ? vv[j] : -INFINITY;
        int bi = (m < p.M) ? m : 0x7fffffff;
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
          const float ov = __shfl_xor_sync(0xffffffffu, best, o);
          const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
          if (ov > best || (ov == best && oi < bi)) {
            best = ov;
            bi = oi;
          }
        }
        if (lane == 0) {
          red_v[(et >> 5) * 4 + j] = best;
          red_i[(et >> 5) * 4 + j] = bi;
        }
      }
      named_bar_sync(1, 128);
      if (et < 4) {
        float best = red_v[et];
        int bi = red_i[et];
        for (int w = 1; w < 4; ++w) {
          const float ov = red_v[w * 4 + et];
          const int oi = red_i[w * 4 + et];
          if (ov > best || (ov == best && oi < bi)) {
            best = ov;
            bi = oi;
          }
        }
        const int n = tn * p.bn + c + et;
        if (n < p.N) reinterpret_cast<float2*>(p.out)[(long)tm * p.ldo + n] = make_float2(best, __int_as_float(bi));
      }
      named_bar_sync(1, 128);
    }
  } else if constexpr (EPI == EPI_QKV_ROPE) {
    // this CTA's tokens of one head: row et and its RoPE partner row et ^ 64 are both summed here
    const uint32_t stg = smem_u32(s.a);
    const bool rot = tm < p.rope_hq + p.rope_hkv;
    for (int c = c_lo; c < c_hi; c += 32) {
      const int nv = min(8, (c_hi - c) >> 2);
      float4 v[8], y[8];
      sum_row(et, c, nv, v);
      if (rot) sum_row(et ^ 64, c, nv, y);
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        if (j >= nv) break;
        const float vv[4] = {v[j].x, v[j].y, v[j].z, v[j].w};
        const float yy[4] = {y[j].x, y[j].y, y[j].z, y[j].w};
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const int n = tn * p.bn + c + 4 * j + e;
          float o = bf16_round(vv[e]);
          if (rot && n < p.N) o = rope_rotate(p, et, p.rope_pos[n], o, bf16_round(yy[e]));
          stage_put_bf16(stg, BM, c - c_lo + 4 * j + e, et, o);
        }
      }
    }
    if (c_hi > c_lo) stage_flush_qkv(p, stg, c_hi - c_lo, tn * p.bn + c_lo, tm, et);
  } else if constexpr (EPI == EPI_STORE_BF16) {
    // staged [cpc tokens][128 features] bf16 in the idle operand ring, written as 16-byte chunks
    const uint32_t stg = smem_u32(s.a);
    for (int c = c_lo; c < c_hi; c += 32) {
      const int nv = min(8, (c_hi - c) >> 2);
      float4 v[8];
      sum_row(et, c, nv, v);
      if (trace && et == 0 && c == c_lo) trace[11] = globaltimer_after(v[0].x);
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        if (j >= nv) break;
        const float vv[4] = {v[j].x, v[j].y, v[j].z, v[j].w};
#pragma unroll
        for (int e = 0; e < 4; ++e) stage_put_bf16(stg, BM, c - c_lo + 4 * j + e, et, vv[e]);
      }
    }
    if (c_hi > c_lo) stage_flush_bf16(p, stg, BM, c_hi - c_lo, tn * p.bn + c_lo, m_base, p.M, et);
  } else {
    const int m = m_base + et;
    for (int c = c_lo; c < c_hi; c += 32) {
      const int nv = min(8, (c_hi - c) >> 2);
      float4 v[8];
      sum_row(et, c, nv, v);
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        if (j >= nv) break;
        const float vv[4] = {v[j].x, v[j].y, v[j].z, v[j].w};
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const int n = tn * p.bn + c + 4 * j + e;
          if (n >= p.N || m >= p.M) continue;
          if constexpr (EPI == EPI_STORE_F32)
            reinterpret_cast<float*>(p.out)[(long)n * p.ldo + m] = vv[e];
          else
            reinterpret_cast<__nv_bfloat16*>(p.out)[(long)n * p.ldo + m] = f2bf(vv[e]);
        }
      }
    }
  }
  if (trace && et == 0) trace[9] = globaltimer_ns();
}

// ----------------------------------------------------------------------------------------------
// Fused all-reduce tail (swap-AB bf16 GEMM with push mode 1; epilogue warps, 128 threads).
//
// Protocol of one launch, epoch e = local epoch word + 1. Flags live in every rank's workspace as
// flag[phase][source rank][source CTA] and only grow, so nothing is reset between launches.
//  phase 0  after the CTA barrier that follows its pushes, one thread of every CTA issues one
//           system-scope fence (cumulative over the barrier: it orders every thread's pushes of
//           the CTA) and stores flag[0][rank][cta] = e into every rank;
//  reduce   CTA i < min(owned rows, grid) waits (bounded) until every rank's every CTA raised its
//           phase-0 flag here, sums its owned rows over the ranks' pushed slots (fp32, source
//           order), adds the residual (stored back rounded to bf16, locally), applies RMSNorm to
//           the rounded value and stores the normed row into every rank;
//  phase 1  the same fence + flag store pattern for flag[1][rank][reducing cta];
//  exit     CTA 0 waits (bounded) for phase 1 of every reducing CTA of every rank (their number
//           follows from T and the row split), then stores e as the new epoch. The next kernel's
//           griddepcontrol.wait therefore sees every normed row.
// A push slot is rewritten only by the next launch, which cannot start its pushes before every rank
// left this one (phase 1), so one set of slots would do; the caller still alternates two. Every
// wait records ERR_PEER_TIMEOUT and gives up after `timeout_ns`.
// ----------------------------------------------------------------------------------------------
constexpr int AR_TAIL_MAX_CTAS = 256;

__device__ __forceinline__ uint32_t* ar_flag(const ArTail& a, int dst, int phase, int src, int cta) {
  return reinterpret_cast<uint32_t*>(a.ws[dst] + a.off_flags) +
         ((long)(phase * AR_TAIL_MAX_RANKS + src) * AR_TAIL_MAX_CTAS + cta);
}

// Called by all 128 epilogue threads right after a barrier that follows their stores.
__device__ __forceinline__ void ar_signal(const ArTail& a, int phase, uint32_t e, int et) {
  if (et == 0) {
    fence_acq_rel_sys();
    for (int d = 0; d < a.world; ++d) st_relaxed_sys(ar_flag(a, d, phase, a.rank, blockIdx.x), e);
  }
}

// rows rank r owns when T rows are split into near-equal ranges (larger ranges first)
__device__ __forceinline__ int ar_rows_of(const ArTail& a, int r) {
  return a.T / a.world + (r < a.T % a.world ? 1 : 0);
}

// Bounded wait until flag[phase][src][c] >= e here for every src and every c < ncta(src) (all 128
// threads poll in parallel); uniform result across the 128 threads.
template <typename NCta>
__device__ __forceinline__ bool ar_wait(const GemmParams& p, int phase, uint32_t e, int et, volatile int* s_ok,
                                        NCta ncta) {
  const ArTail& a = p.ar;
  if (et == 0) *s_ok = 1;
  named_bar_sync(1, 128);
  bool ok = true;
  for (int src = 0; src < a.world && ok; ++src) {
    const int n = ncta(src);
    for (int c = et; c < n && ok; c += 128)
      ok = wait_flag_geq(ar_flag(a, a.rank, phase, src, c), e, a.timeout_ns, p.err);
  }
  if (!ok) *s_ok = 0;
  named_bar_sync(1, 128);
  return *s_ok != 0;
}

// One owned token row: H features, 8 per 16-byte chunk, chunks et + 128 j (j < MAXC), processed
// in groups of G chunks; within a group the residual and every source's chunks are all loaded
// before any is added (one memory round trip per group). The rounded residual of every chunk is
// kept packed for the normalisation pass when MAXC <= 4; wider rows (H > 4096) read back the
// residual they just stored instead, which keeps the register footprint of the tail small.
template <int MAXC, int G, int NSRC>
__device__ __forceinline__ void ar_tail_row(const ArTail& a, long row, int et, volatile float* red) {
  constexpr bool KEEP = MAXC <= 4;
  const int nvec = a.H / 8;
  uint4* resid = reinterpret_cast<uint4*>(a.ws[a.rank] + a.off_resid) + row * nvec;
  const __nv_bfloat16* push0 = reinterpret_cast<const __nv_bfloat16*>(a.ws[a.rank] + a.off_push) + row * a.H;
  uint4 packed[KEEP ? MAXC : 1];
  float ss = 0.f;
#pragma unroll
  for (int g0 = 0; g0 < MAXC; g0 += G) {
    uint4 rv[G];
    uint4 d[NSRC][G];
#pragma unroll
    for (int j = 0; j < G; ++j) {
      const int c = et + 128 * (g0 + j);
      if (c < nvec) rv[j] = resid[c];
    }
#pragma unroll
    for (int src = 0; src < NSRC; ++src) {
      if (src < a.world) {
        const uint4* part = reinterpret_cast<const uint4*>(push0 + (long)src * a.t_max * a.H);
#pragma unroll
        for (int j = 0; j < G; ++j) {
          const int c = et + 128 * (g0 + j);
          if (c < nvec) d[src][j] = __ldcg(part + c);
        }
      }
    }
#pragma unroll
    for (int j = 0; j < G; ++j) {
      const int c = et + 128 * (g0 + j);
      if (c >= nvec) continue;
      float acc[8];
      const uint32_t* ru = reinterpret_cast<const uint32_t*>(&rv[j]);
#pragma unroll
      for (int q = 0; q < 4; ++q) unpack_bf16x2(ru[q], acc[2 * q], acc[2 * q + 1]);
#pragma unroll
      for (int src = 0; src < NSRC; ++src) {  // rank order: deterministic
        if (src < a.world) {
          const uint32_t* du = reinterpret_cast<const uint32_t*>(&d[src][j]);
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            float x0, x1;
            unpack_bf16x2(du[q], x0, x1);
            acc[2 * q] += x0;
            acc[2 * q + 1] += x1;
          }
        }
      }
      // the residual is stored rounded to bf16 and the norm is taken of that stored value
      uint4 pk;
      uint32_t* pu = reinterpret_cast<uint32_t*>(&pk);
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        pu[q] = pack_bf16x2(acc[2 * q], acc[2 * q + 1]);
        float r0, r1;
        unpack_bf16x2(pu[q], r0, r1);
        ss += r0 * r0 + r1 * r1;
      }
      resid[c] = pk;
      if constexpr (KEEP) packed[g0 + j] = pk;
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
  if ((et & 31) == 0) red[et >> 5] = ss;
  named_bar_sync(1, 128);
  const float inv = rsqrtf((red[0] + red[1] + red[2] + red[3]) / (float)a.H + a.eps);
  named_bar_sync(1, 128);  // `red` is reused by the next row
  const uint4* gv = reinterpret_cast<const uint4*>(a.gamma);
#pragma unroll
  for (int j = 0; j < MAXC; ++j) {
    const int c = et + 128 * j;
    if (c < nvec) {
      const uint4 g = gv[c];
      const uint32_t* gu = reinterpret_cast<const uint32_t*>(&g);
      uint4 pk;
      if constexpr (KEEP) pk = packed[j];
      else pk = resid[c];  // written by this thread above
      const uint32_t* pu = reinterpret_cast<const uint32_t*>(&pk);
      uint4 o;
      uint32_t* ou = reinterpret_cast<uint32_t*>(&o);
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        float r0, r1, g0, g1;
        unpack_bf16x2(pu[q], r0, r1);
        unpack_bf16x2(gu[q], g0, g1);
        ou[q] = pack_bf16x2(r0 * inv * g0, r1 * inv * g1);
      }
      const long off = a.off_normed + (row * nvec + c) * 16;
      if (a.mc) {
        multimem_st_16(reinterpret_cast<void*>(a.mc + off), o);
      } else {
        for (int d = 0; d < a.world; ++d) *reinterpret_cast<uint4*>(a.ws[d] + off) = o;
      }
    }
  }
}

template <int MAXC>
__device__ __forceinline__ void ar_tail_rows(const ArTail& a, long r0, int nrows, int et, volatile float* red) {
  for (long row = r0 + blockIdx.x; row < r0 + nrows; row += gridDim.x) {
    if (a.world <= 4)
      ar_tail_row<MAXC, 4, 4>(a, row, et, red);
    else
      ar_tail_row<MAXC, 2, AR_TAIL_MAX_RANKS>(a, row, et, red);
  }
}

// Runs after the CTA barrier that follows the epilogue (every push of this CTA is issued).
__device__ __forceinline__ void ar_tail(const GemmParams& p, const Smem& s, int et, unsigned long long* trace) {
  const ArTail& a = p.ar;
  const bool tr = trace != nullptr && et == 0;
  if (tr) trace[16] = globaltimer_ns();
  volatile uint32_t* s_e = reinterpret_cast<volatile uint32_t*>(s.epi);  // [0] epoch, [1] ok
  volatile float* red = reinterpret_cast<volatile float*>(s.epi) + 4;  // [4] sum-of-squares partials
  if (et == 0) {
    const uint32_t e0 = *reinterpret_cast<volatile uint32_t*>(a.epoch) + 1u;
    s_e[0] = e0;
    ar_signal(a, 0, e0, et);  // the CTA barrier before the tail ordered every push of this CTA
  }
  named_bar_sync(1, 128);
  const uint32_t e = s_e[0];
  if (tr) trace[17] = globaltimer_ns();
  const int grid = (int)gridDim.x;
  const int nrows = ar_rows_of(a, a.rank);
  const long r0 = (long)a.rank * (a.T / a.world) + min(a.rank, a.T % a.world);
  const int nred = min(nrows, grid);
  volatile int* s_ok = reinterpret_cast<volatile int*>(s_e + 1);
  if ((int)blockIdx.x < nred) {
    if (ar_wait(p, 0, e, et, s_ok, [grid](int) { return grid; })) {
      if (tr) trace[18] = globaltimer_ns();
      if (a.H <= 128 * 8 * 4)
        ar_tail_rows<4>(a, r0, nrows, et, red);
      else
        ar_tail_rows<8>(a, r0, nrows, et, red);
      if (tr) trace[19] = globaltimer_ns();
    }
    named_bar_sync(1, 128);  // every normed store of this CTA is issued
    ar_signal(a, 1, e, et);
    if (tr) trace[20] = globaltimer_ns();
  }
  if (blockIdx.x == 0) {
    ar_wait(p, 1, e, et, s_ok, [&a, grid](int src) { return min(ar_rows_of(a, src), grid); });
    if (tr) trace[21] = globaltimer_ns();
    if (et == 0) *a.epoch = e;
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
  const int kbox = p.kbox;
  const uint32_t a_box_bytes = A_STAGE_BYTES, b_box_bytes = (uint32_t)p.bn * BK * 2;
  const uint32_t a_stage_bytes = a_box_bytes * kbox, b_stage_bytes = b_box_bytes * kbox;
  const int bk_eff = BK * kbox;

  if (threadIdx.x == 0) {
    for (int i = 0; i < p.stages; ++i) {
      mbar_init(&s.full[i], 1);
      mbar_init(&s.empty[i], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&s.tfull[i], 1);
      mbar_init(&s.tempty[i], 128);
    }
    mbar_init(s.fixbar, 1);
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
  if (TRANS && p.ck > 1) cluster_arrive_relaxed();  // waited on before any remote shared-memory access
  unsigned long long* trace = p.trace ? p.trace + (size_t)blockIdx.x * TRACE_SLOTS : nullptr;
  if (trace && threadIdx.x == 0) trace[0] = globaltimer_ns();
  // the next kernel may start its prologue on SMs this grid frees up
  griddep_launch_dependents();

  if (warp == 0) {
    // ------------------------------- TMA producer -------------------------------
    if (lane == 0) {
      // decode streams weights once (A, evict-first) and reuses the token tile (B); prefill reuses both
      const uint64_t pol_a = TRANS ? policy_evict_first() : policy_evict_last();
      const uint64_t pol_b = policy_evict_last();
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      SegIter itr;
      itr.init(p);
      Seg sg;
      bool first_seg = true;
      while (ok && itr.next(p, sg)) {
        int kb_start = sg.kb0;
        if (first_seg) {
          // Operand A of the first stages (weights in decode) does not depend on the previous
          // kernel: fetch it before waiting for that kernel's results, then fetch B.
          first_seg = false;
          const int npre = min(p.stages, sg.kb1 - sg.kb0);
          for (int i = 0; i < npre; ++i) {
            mbar_arrive_expect_tx(&s.full[i], a_stage_bytes + b_stage_bytes);
            for (int j = 0; j < kbox; ++j)
              tma_load_2d(s.a + (size_t)i * a_stage_bytes + j * a_box_bytes, &tmA, &s.full[i],
                          (sg.kb0 + i) * bk_eff + j * BK, sg.tm * BM, pol_a);
          }
          griddep_wait();
          if (trace) trace[1] = globaltimer_ns();
          for (int i = 0; i < npre; ++i)
            for (int j = 0; j < kbox; ++j)
              tma_load_2d(s.b + (size_t)i * b_stage_bytes + j * b_box_bytes, &tmB, &s.full[i],
                          (sg.kb0 + i) * bk_eff + j * BK, sg.tn * p.bn, pol_b);
          kb_start = sg.kb0 + npre;
          stage = npre % p.stages;
          phase = (npre == p.stages) ? 1u : 0u;
        }
        for (int kb = kb_start; kb < sg.kb1; ++kb) {
          if (!mbar_wait_bounded(&s.empty[stage], phase ^ 1, p.err, ERR_MBAR_TIMEOUT_PRODUCER, abort_flag,
                                 WAIT_LIMIT_NS)) {
            ok = false;
            break;
          }
          mbar_arrive_expect_tx(&s.full[stage], a_stage_bytes + b_stage_bytes);
          for (int j = 0; j < kbox; ++j) {
            tma_load_2d(s.a + (size_t)stage * a_stage_bytes + j * a_box_bytes, &tmA, &s.full[stage],
                        kb * bk_eff + j * BK, sg.tm * BM, pol_a);
            tma_load_2d(s.b + (size_t)stage * b_stage_bytes + j * b_box_bytes, &tmB, &s.full[stage],
                        kb * bk_eff + j * BK, sg.tn * p.bn, pol_b);
          }
          if (++stage == p.stages) {
            stage = 0;
            phase ^= 1;
          }
        }
      }
      if (first_seg) griddep_wait();  // no work: still order after the previous grid
      if (trace) trace[2] = globaltimer_ns();
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
    __syncwarp();
    if (TRANS && p.ck > 1) {
      cluster_wait_acquire();
      cluster_sync();
    }
  } else if (warp == 1) {
    // ------------------------------- MMA issuer -------------------------------
    int stage = 0;
    uint32_t phase = 0;
    int it = 0;
    bool ok = true;
    SegIter itr;
    itr.init(p);
    Seg sg;
    while (ok && itr.next(p, sg)) {
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
      for (int kb = sg.kb0; kb < sg.kb1; ++kb) {
        if (lane == 0)
          w = mbar_wait_bounded(&s.full[stage], phase, p.err, ERR_MBAR_TIMEOUT_MMA, abort_flag, WAIT_LIMIT_NS);
        w = __shfl_sync(0xffffffffu, w, 0);
        if (!w) {
          ok = false;
          break;
        }
        tc_fence_after();
        if (trace && lane == 0 && it == 0 && kb == sg.kb0) trace[3] = globaltimer_ns();
        if (lane == 0) {
          for (int j = 0; j < kbox; ++j) {
            const uint32_t a_addr = smem_u32(s.a + (size_t)stage * a_stage_bytes + j * a_box_bytes);
            const uint32_t b_addr = smem_u32(s.b + (size_t)stage * b_stage_bytes + j * b_box_bytes);
            const uint64_t a_desc = make_sdesc_sw128(a_addr);
            const uint64_t b_desc = make_sdesc_sw128(b_addr);
#pragma unroll
            for (int k = 0; k < BK / 16; ++k) {
              // advance 16 bf16 = 32 bytes inside the swizzled 128-byte row: +2 in 16-byte units
              umma_bf16(d_tmem, a_desc + 2 * k, b_desc + 2 * k, p.idesc,
                        (kb > sg.kb0 || j > 0 || k > 0) ? 1u : 0u);
            }
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
      ++it;
    }
    if (trace && lane == 0) trace[4] = globaltimer_ns();
    __syncwarp();
    if (TRANS && p.ck > 1) {
      cluster_wait_acquire();
      cluster_sync();
    }
  } else if (TRANS && p.ck > 1) {
    // ------------------------ epilogue, cluster split-K (warps 2..5) ------------------------
    griddep_wait();
    if constexpr (TRANS) ck_epilogue<EPI, TRANS>(p, s, tmem_base, abort_flag, trace);
  } else {
    // ------------------------------- epilogue (warps 2..5) -------------------------------
    griddep_wait();  // output and workspace may still be in use by the previous grid
    const int et = threadIdx.x - 64;            // 0..127
    const int quarter = warp & 3;               // TMEM lane quarter this warp may access
    const int row = quarter * 32 + lane;        // accumulator row (TMEM lane)
    const uint32_t slot0 = smem_u32(s.epi);
    const uint32_t slot1 = slot0 + EPI_SLOT_FLOATS * 4;
    const size_t tile_floats = (size_t)BM * p.bn;
    uint32_t fix_phase = 0;
    int it = 0;
    SegIter itr;
    itr.init(p);
    Seg sg;
    while (itr.next(p, sg)) {
      const int acc = it & 1;
      const uint32_t acc_phase = (it >> 1) & 1;
      ++it;
      if (et == 0)
        *s.epi_flag = mbar_wait_bounded(&s.tfull[acc], acc_phase, p.err, ERR_MBAR_TIMEOUT_EPILOGUE, abort_flag,
                                        WAIT_LIMIT_NS);
      named_bar_sync(1, 128);
      const int ok = *s.epi_flag;
      named_bar_sync(1, 128);
      if (!ok) break;
      if (trace && et == 0 && it == 1) trace[5] = globaltimer_ns();
      tc_fence_after();
      const uint32_t taddr_row = tmem_base + ((uint32_t)(quarter * 32) << 16) + (uint32_t)(acc * p.bn);

      // up to n16 groups of 16 columns behind one wait (r holds 32 or 64 registers)
      auto fetch_tmem = [&](int col, auto& r, int n16) {
        constexpr int W = sizeof(r) / sizeof(r[0]);
#pragma unroll
        for (int k = 0; k < W / 16; ++k)
          if (k < n16) tmem_ld16(taddr_row + col + 16 * k, *reinterpret_cast<uint32_t(*)[16]>(&r[16 * k]));
        tmem_ld_wait_tied(r);
      };
      // the staged swap-AB bf16 store is push-aware; other whole-tile epilogues write `out` only
      constexpr bool kPushDirect = TRANS && EPI == EPI_STORE_BF16;
      const bool direct = p.direct_epi && (p.push_mode == 0 || kPushDirect);
      if (sg.ncontrib == 1 && direct) {
        direct_epilogue<EPI, TRANS>(p, s, fetch_tmem, row, lane, quarter, sg.tm, sg.tn, &s.tempty[acc]);
      } else if (sg.ncontrib > 1 && sg.contrib == 0 && direct) {
        // stream-K owner: wait (bounded) for the other contributors' partials, then run the
        // whole-tile epilogue on own accumulator + partials, read per row straight from the
        // workspace in contributor order (deterministic)
        const bool okw = wait_counter_eq(&p.counters[sg.sk_tile], sg.ncontrib - 1, WAIT_LIMIT_NS, p.err,
                                         ERR_MBAR_TIMEOUT_EPILOGUE);
        (void)okw;
        named_bar_sync(1, 128);
        if (et == 0) p.counters[sg.sk_tile] = 0;
        if (trace && et == 0) trace[10] = globaltimer_ns();
        const float* part_row = p.workspace + (size_t)(sg.sk_tile + sg.first_cta + 1) * tile_floats +
                                (size_t)row * p.bn;
        const int nparts = sg.ncontrib - 1;
        auto fetch_sum = [&](int col, auto& r, int n16) {
          constexpr int W = sizeof(r) / sizeof(r[0]);
          fetch_tmem(col, r, n16);
          for (int k = 0; k < nparts; ++k) {
            const float4* src = reinterpret_cast<const float4*>(part_row + (size_t)k * tile_floats + col);
#pragma unroll
            for (int i = 0; i < W / 4; ++i) {
              if (i < 4 * n16) {
                const float4 y = __ldcg(src + i);
                r[4 * i] = __float_as_uint(__uint_as_float(r[4 * i]) + y.x);
                r[4 * i + 1] = __float_as_uint(__uint_as_float(r[4 * i + 1]) + y.y);
                r[4 * i + 2] = __float_as_uint(__uint_as_float(r[4 * i + 2]) + y.z);
                r[4 * i + 3] = __float_as_uint(__uint_as_float(r[4 * i + 3]) + y.w);
              }
            }
          }
        };
        direct_epilogue<EPI, TRANS>(p, s, fetch_sum, row, lane, quarter, sg.tm, sg.tn, &s.tempty[acc]);
        if (trace && et == 0) trace[11] = globaltimer_ns();
      } else if (sg.ncontrib == 1) {
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
          finalize_chunk<EPI, TRANS>(p, slot0, slot1, sg.tm, sg.tn, cout, cw, et);
          named_bar_sync(1, 128);
        }
      } else {
        // stream-K. The tile's owner is the CTA holding its first k-block (contributor 0); its
        // segment of this tile is the last of its range, while the other contributors reach the
        // tile first. Non-owners publish an fp32 partial and bump the tile counter; the owner waits
        // (bounded) for all of them, adds the partials to its own TMEM accumulator in contributor
        // order (deterministic) and runs the epilogue, then resets the counter for the next launch.
        if (sg.contrib != 0) {
          float* ws = p.workspace + (size_t)(sg.sk_tile + blockIdx.x) * tile_floats;
          for (int c = 0; c < p.bn; c += 16) {
            uint32_t r[16];
            tmem_ld16(taddr_row + c, r);
            tmem_ld_wait();
            float4* dst = reinterpret_cast<float4*>(ws + (size_t)row * p.bn + c);
#pragma unroll
            for (int i = 0; i < 4; ++i)
              __stcg(dst + i, make_float4(__uint_as_float(r[4 * i]), __uint_as_float(r[4 * i + 1]),
                                          __uint_as_float(r[4 * i + 2]), __uint_as_float(r[4 * i + 3])));
          }
          tc_fence_before();
          mbar_arrive(&s.tempty[acc]);
          if (trace && et == 0) trace[8] = globaltimer_ns();
          __threadfence();
          named_bar_sync(1, 128);
          if (et == 0) red_release_gpu_add(&p.counters[sg.sk_tile], 1);
          if (trace && et == 0) trace[9] = globaltimer_ns();
        } else {
          // Owner: its segment of this tile is the last of its range, so the operand ring is idle.
          // Pull the contributors' partial tiles into it with bulk copies (all in flight at once),
          // then add them to the own accumulator chunk by chunk in contributor order.
          const bool okw = wait_counter_eq(&p.counters[sg.sk_tile], sg.ncontrib - 1, WAIT_LIMIT_NS, p.err,
                                           ERR_MBAR_TIMEOUT_EPILOGUE);
          (void)okw;
          named_bar_sync(1, 128);
          if (et == 0) p.counters[sg.sk_tile] = 0;
          if (trace && et == 0) trace[10] = globaltimer_ns();
          const uint32_t tile_bytes = (uint32_t)(tile_floats * 4);
          const size_t ring_bytes = (size_t)p.stages * (a_stage_bytes + b_stage_bytes);
          const int per_batch = (int)(ring_bytes / tile_bytes) < 1 ? 1 : (int)(ring_bytes / tile_bytes);
          const float* part0 = p.workspace + (size_t)(sg.sk_tile + sg.first_cta) * tile_floats;
          const int nsteps = ChunkPlan<EPI, TRANS>::steps(p.bn);
          // own accumulator chunks are kept in TMEM; partial batches accumulate into a running
          // fp32 copy of the tile held in the ring when more than one batch is needed
          const int nparts = sg.ncontrib - 1;
          const int nbatch = (nparts + per_batch - 1) / per_batch;
          for (int st = 0; st < nsteps; ++st) {
            int ca, cb, cw, cout;
            ChunkPlan<EPI, TRANS>::step(st, p.bn, ca, cb, cw, cout);
            tmem_chunk_to_smem(taddr_row, ca, cw, slot0, row);
            if (cb >= 0) tmem_chunk_to_smem(taddr_row, cb, cw, slot1, row);
            if (st == nsteps - 1) {
              tc_fence_before();
              mbar_arrive(&s.tempty[acc]);
            }
            for (int bt_i = 0; bt_i < nbatch; ++bt_i) {
              const int k0 = 1 + bt_i * per_batch;
              const int kn = min(per_batch, nparts - bt_i * per_batch);
              // the whole batch is re-fetched per chunk only when it cannot stay resident
              const bool resident = (nbatch == 1);
              if (!resident || st == 0) {
                named_bar_sync(1, 128);  // ring free of the previous batch's readers
                if (et == 0) {
                  fence_proxy_async();
                  mbar_arrive_expect_tx(s.fixbar, (uint32_t)kn * tile_bytes);
                  for (int k = 0; k < kn; ++k)
                    bulk_load(s.a + (size_t)k * tile_bytes, part0 + (size_t)(k0 + k) * tile_floats, tile_bytes,
                              s.fixbar);
                }
                int okb = 1;
                if (et == 0) {
                  okb = mbar_wait_bounded(s.fixbar, fix_phase, p.err, ERR_MBAR_TIMEOUT_EPILOGUE, abort_flag,
                                          WAIT_LIMIT_NS);
                  *s.epi_flag = okb;
                }
                fix_phase ^= 1;
                if (trace && et == 0 && st == 0) trace[12] = globaltimer_ns();
                named_bar_sync(1, 128);
              } else {
                named_bar_sync(1, 128);
              }
              // add staged partials: a thread owns 4 consecutive columns of one row (16-byte shared
              // loads; a warp covers 4 rows x 32 columns, conflict-free)
              {
                const uint32_t ring = smem_u32(s.a);
                const uint32_t s0 = slot0, s1 = slot1;
                const int q4 = cw >> 2;                 // float4 per row in this chunk (8 or 4)
                const int q4s = (cw == 32) ? 3 : 2;     // log2(q4)
                for (int v = et; v < BM * q4; v += 128) {
                  const int r = v >> q4s, c = (v & (q4 - 1)) * 4;
                  const uint32_t so = (uint32_t)(r * EPI_LD + c) * 4;
                  float4 x0 = make_float4(lds_f32(s0 + so), lds_f32(s0 + so + 4), lds_f32(s0 + so + 8),
                                          lds_f32(s0 + so + 12));
                  float4 x1 = make_float4(0.f, 0.f, 0.f, 0.f);
                  if (cb >= 0)
                    x1 = make_float4(lds_f32(s1 + so), lds_f32(s1 + so + 4), lds_f32(s1 + so + 8),
                                     lds_f32(s1 + so + 12));
                  const uint32_t rowoff = (uint32_t)(r * p.bn) * 4;
#pragma unroll 4
                  for (int k = 0; k < kn; ++k) {
                    const uint32_t pt = ring + (uint32_t)k * tile_bytes + rowoff;
                    const float4 y = lds_f4(pt + (uint32_t)(ca + c) * 4);
                    x0.x += y.x; x0.y += y.y; x0.z += y.z; x0.w += y.w;
                    if (cb >= 0) {
                      const float4 z = lds_f4(pt + (uint32_t)(cb + c) * 4);
                      x1.x += z.x; x1.y += z.y; x1.z += z.z; x1.w += z.w;
                    }
                  }
                  sts_f32(s0 + so, x0.x); sts_f32(s0 + so + 4, x0.y); sts_f32(s0 + so + 8, x0.z);
                  sts_f32(s0 + so + 12, x0.w);
                  if (cb >= 0) {
                    sts_f32(s1 + so, x1.x); sts_f32(s1 + so + 4, x1.y); sts_f32(s1 + so + 8, x1.z);
                    sts_f32(s1 + so + 12, x1.w);
                  }
                }
              }
            }
            named_bar_sync(1, 128);
            if (trace && et == 0 && st == 0) trace[13] = globaltimer_ns();
            finalize_chunk<EPI, TRANS>(p, slot0, slot1, sg.tm, sg.tn, cout, cw, et);
            named_bar_sync(1, 128);
            if (trace && et == 0 && st == 0) trace[14] = globaltimer_ns();
          }
          if (trace && et == 0) trace[11] = globaltimer_ns();
        }
      }
    }
  }

  // pushed tiles visible to the peers: per thread here, or once per CTA in the fused tail's signal
  if (p.push_mode != 0 && !p.ar.on && warp >= 2) __threadfence_system();
  if (trace && threadIdx.x == 64) trace[6] = globaltimer_ns();
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, p.tmem_cols);
  }
  if constexpr (TRANS && EPI == EPI_STORE_BF16) {
    // fused all-reduce tail: TMEM is already released, so cross-GPU waits hold no tensor memory
    if (p.ar.on && warp >= 2) ar_tail(p, s, threadIdx.x - 64, trace);
  }
  if (trace && threadIdx.x == 0) trace[7] = globaltimer_ns();
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
static void configure_kernel() {
  auto kern = gemm_tcgen05_kernel<EPI, TRANS>;
  static bool configured[64] = {false};
  int dev;
  cudaGetDevice(&dev);
  if (!configured[dev]) {
    cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, 232448);
    cudaFuncSetAttribute(kern, cudaFuncAttributeNonPortableClusterSizeAllowed, 1);
    configured[dev] = true;
  }
}

template <int EPI, bool TRANS>
static void launch_typed(const CUtensorMap& ta, const CUtensorMap& tb, const GemmParams& p, int grid, size_t smem,
                         cudaStream_t stream) {
  auto kern = gemm_tcgen05_kernel<EPI, TRANS>;
  configure_kernel<EPI, TRANS>();
  C10_CUDA_CHECK(launch_kc(kern, dim3(grid), dim3(NUM_THREADS), smem, stream, p.ck > 1 ? p.ck : 1, ta, tb, p));
}

// Largest number of co-resident clusters of `C` CTAs of this kernel (every CTA of a cluster split
// must be resident at once, and one wave is the point of the schedule).
template <int EPI, bool TRANS>
static int max_active_clusters(int C, size_t smem) {
  static std::mutex mu;
  static std::unordered_map<long, int> cache;
  int dev;
  cudaGetDevice(&dev);
  const long key = ((long)dev << 40) | ((long)C << 32) | (long)smem;
  std::lock_guard<std::mutex> g(mu);
  auto it = cache.find(key);
  if (it != cache.end()) return it->second;
  configure_kernel<EPI, TRANS>();
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(C * 64);
  cfg.blockDim = dim3(NUM_THREADS);
  cfg.dynamicSmemBytes = smem;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = C;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  int n = 0;
  if (cudaOccupancyMaxActiveClusters(&n, gemm_tcgen05_kernel<EPI, TRANS>, &cfg) != cudaSuccess) {
    cudaGetLastError();
    n = 0;
  }
  cache[key] = n;
  return n;
}

static int max_active_clusters_for(int epi, bool trans, int C, size_t smem) {
  if (!trans) return 0;
  switch (epi) {
    case EPI_STORE_BF16: return max_active_clusters<EPI_STORE_BF16, true>(C, smem);
    case EPI_STORE_F32: return max_active_clusters<EPI_STORE_F32, true>(C, smem);
    case EPI_SILU_BF16: return max_active_clusters<EPI_SILU_BF16, true>(C, smem);
    case EPI_ARGMAX: return max_active_clusters<EPI_ARGMAX, true>(C, smem);
    case EPI_QKV_ROPE: return max_active_clusters<EPI_QKV_ROPE, true>(C, smem);
    default: return 0;
  }
}

static bool ck_enabled() {
  static int v = -1;
  if (v < 0) {
    const char* e = std::getenv("MESH_GEMM_CK");
    v = (e && e[0] == '0') ? 0 : 1;
  }
  return v == 1;
}

// Cluster split-K factor for a swap-AB problem with `tiles` output tiles and `kb` k-blocks: the
// largest C (<= 16, <= kb, tiles * C <= SMs) whose clusters all fit on the GPU at once; 0 if none
// of C >= 2 qualifies.
// shared-memory plan of one CTA: operand stages and epilogue region (receive buffers when C > 1)
struct SmemPlan {
  int stages, epi_bytes;
  size_t bytes;
};
static int max_stages() {
  static int v = -1;
  if (v < 0) {
    const char* e = std::getenv("MESH_GEMM_STAGES");
    v = e ? std::max(2, std::min(8, std::atoi(e))) : 8;
  }
  return v;
}

// 64-wide k boxes per pipeline stage: decode (swap-AB, weight streaming) moves 32 KB of weights
// per stage, which sustains a higher per-SM rate than 16 KB stages (fewer barrier round trips per
// byte); prefill keeps 64-wide stages so that more of them fit next to the 256-wide B tiles.
static int kbox_for(bool trans) {
  static int v = -1;
  if (v < 0) {
    const char* e = std::getenv("MESH_GEMM_KBOX");
    v = e ? std::max(1, std::min(2, std::atoi(e))) : 0;
  }
  return v > 0 ? v : (trans ? 2 : 1);
}

// epilogue region of the whole-tile path: swap-AB SiLU hands bf16 "up" rows across warps
// ([2 blocks][2 directions][64][17] words) and stages its bf16 output ([64][64]); all of it fits
// the staging slots
static int epi_region_bytes(int epi, bool trans) {
  return (trans && epi == EPI_SILU_BF16) ? std::max(EPI_STAGING_BYTES, (4 * 64 * 17) * 4 + 64 * 64 * 2)
                                         : EPI_STAGING_BYTES;
}

static SmemPlan smem_plan(int bn, int C, int kbox, int epi, bool trans) {
  SmemPlan sp;
  const int base = epi_region_bytes(epi, trans);
  sp.epi_bytes = C > 1 ? std::max(base, ck_recv_bytes(bn, C)) : base;
  sp.stages = max_stages();
  while (sp.stages > 2 && gemm_smem_bytes(sp.stages, bn, sp.epi_bytes, kbox) > SMEM_BUDGET) --sp.stages;
  sp.bytes = gemm_smem_bytes(sp.stages, bn, sp.epi_bytes, kbox);
  return sp;
}

static int pick_ck(int tiles, int kb, int num_sms, int epi, int bn, int kbox) {
  int C = std::min(16, std::min(kb, num_sms / std::max(tiles, 1)));
  for (; C >= 2; --C) {
    const SmemPlan sp = smem_plan(bn, C, kbox, epi, true);
    if (sp.bytes <= SMEM_BUDGET && max_active_clusters_for(epi, true, C, sp.bytes) >= tiles) return C;
  }
  return 0;
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

// Schedule: whole tiles round-robin over a persistent grid for all but the last (partial) waves;
// the remaining tiles' k-iterations are spread evenly over the grid (stream-K). Small problems
// (fewer tiles than SMs) become pure stream-K, which replaces classic split-K.
struct Plan {
  int grid, dp_tiles, sk_iters, sk_tiles, tiles;
  size_t ws_floats;
  int ck;
};

// force_mode: 0 auto, 1 data-parallel, 2 stream-K, 3 cluster split-K (swap-AB only).
static Plan make_plan(int M, int N, int K, int bn, int num_sms, int force_mode, int epi, bool trans, bool push,
                      int kbox) {
  Plan pl{};
  const int m_tiles = (M + BM - 1) / BM, n_tiles = (N + bn - 1) / bn;
  const int kb = (K + BK * kbox - 1) / (BK * kbox);
  pl.tiles = m_tiles * n_tiles;
  const long total_iters = (long)pl.tiles * kb;
  int grid = num_sms;
  // Automatic choice for swap-AB (decode) shapes, from measured decode sweeps: one wave of whole
  // tiles when they fill most SMs or each tile is short (<= 8 k-blocks, where a split's fixed
  // cost outweighs its parallelism); cluster split-K when the tiles leave SMs idle.
  if (trans && force_mode == 0 && pl.tiles <= num_sms && (4 * pl.tiles >= 3 * num_sms || kb <= 8)) {
    pl.grid = pl.tiles;
    pl.dp_tiles = pl.tiles;
    return pl;
  }
  if (trans && (!push || epi == EPI_STORE_BF16) &&
      (force_mode == 3 || (force_mode == 0 && ck_enabled() && pl.tiles < num_sms))) {
    const int C = pick_ck(pl.tiles, kb, num_sms, epi, bn, kbox);
    if (C >= 2) {
      pl.ck = C;
      pl.grid = pl.tiles * C;
      pl.dp_tiles = 0;
      pl.sk_iters = 0;
      pl.sk_tiles = 0;
      pl.ws_floats = 0;
      return pl;
    }
  }
  if (force_mode == 1 || (force_mode == 0 && (pl.tiles % grid == 0 || pl.tiles >= 4 * grid))) {
    // pure data-parallel persistent schedule
    pl.grid = pl.tiles < grid ? pl.tiles : grid;
    pl.dp_tiles = pl.tiles;
    pl.sk_iters = 0;
    pl.sk_tiles = 0;
    pl.ws_floats = 0;
    return pl;
  }
  int waves = pl.tiles / grid;
  pl.dp_tiles = waves >= 2 ? (waves - 1) * grid : 0;
  pl.sk_tiles = pl.tiles - pl.dp_tiles;
  const long sk_total = (long)pl.sk_tiles * kb;
  if (sk_total < grid) grid = (int)sk_total;
  long w = (sk_total + grid - 1) / grid;
  if (w < 2 && kb >= 2) {  // keep at least two k-blocks per stream-K share
    w = 2;
    grid = (int)((sk_total + w - 1) / w);
  }
  grid = (int)((sk_total + w - 1) / w);  // every CTA gets a non-empty share
  pl.sk_iters = (int)w;
  pl.grid = grid;
  pl.ws_floats = (size_t)(pl.sk_tiles + grid) * BM * bn;
  (void)total_iters;
  return pl;
}

// out = A @ B^T (normal) or out^T = A @ B^T (trans). Returns nothing; errors go to `err`.
struct RopeArgs {
  const int* pos;
  const long* slot;
  const float* cos;
  const float* sin;
  __nv_bfloat16* k;
  __nv_bfloat16* v;
  int hq, hkv, ps;
};

static void gemm_impl(const at::Tensor& A, const at::Tensor& B, at::Tensor& out, int64_t epi, bool trans,
                      int64_t bn_req, int64_t mode, at::Tensor& workspace, at::Tensor& counters, at::Tensor& err,
                      const c10::optional<at::Tensor>& trace, const std::vector<int64_t>& push, const RopeArgs* rope,
                      const ArTail* ar = nullptr) {
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
  if (epi == EPI_ARGMAX)
    TORCH_CHECK(trans && out.scalar_type() == at::kFloat && out.dim() == 3 && out.size(0) >= (M + BM - 1) / BM &&
                    out.size(1) == N && out.size(2) == 2,
                "argmax epilogue: swap-AB only, out float [m_tiles, N, 2]");
  p.bn = bn;
  p.m_tiles = (M + BM - 1) / BM;
  p.n_tiles = (N + bn - 1) / bn;
  const int kbox = kbox_for(trans);
  p.kbox = kbox;
  p.k_blocks = (K + BK * kbox - 1) / (BK * kbox);
  const int sms = num_sms_cached(dev);
  Plan pl = make_plan(M, N, K, bn, sms, (int)mode, (int)epi, trans, !push.empty(), kbox);
  p.ck = pl.ck;
  TORCH_CHECK(mode != 3 || pl.ck >= 2, "gemm_tcgen05: cluster split-K requested but not possible for this shape");
  TORCH_CHECK(p.ck <= 1 || (trans && (push.empty() || epi == EPI_STORE_BF16)),
              "gemm_tcgen05: cluster split-K needs swap-AB (and the bf16 epilogue when pushing)");
  const SmemPlan sp = smem_plan(bn, p.ck, kbox, (int)epi, trans);
  TORCH_CHECK(sp.bytes <= SMEM_BUDGET, "gemm_tcgen05: shared memory plan exceeds the budget");
  const int stages = sp.stages;
  p.epi_bytes = sp.epi_bytes;
  p.dp_tiles = pl.dp_tiles;
  p.sk_iters_per_cta = pl.sk_iters;
  if (pl.sk_tiles > 0) {
    TORCH_CHECK(workspace.numel() >= (int64_t)pl.ws_floats && workspace.scalar_type() == at::kFloat,
                "gemm_tcgen05: workspace too small for stream-K (need ", (int64_t)pl.ws_floats, " floats)");
    TORCH_CHECK(counters.numel() >= pl.sk_tiles && counters.scalar_type() == at::kInt, "gemm_tcgen05: counters");
    p.workspace = workspace.data_ptr<float>();
    p.counters = counters.data_ptr<int>();
  }
  p.stages = stages;
  p.out = out.data_ptr();
  p.ldo = epi == EPI_ARGMAX ? out.size(1) : out.stride(0);
  p.vec_out = ((reinterpret_cast<uintptr_t>(p.out) & 15) == 0) &&
              ((p.ldo * (epi == EPI_STORE_F32 ? 4 : 2)) % 16 == 0);
  // Swap-AB CTAs that stream many tiles (LM head) keep the staged epilogue, whose cooperative
  // column-at-a-time stores measured faster there; latency-bound few-tile launches and the normal
  // orientation store straight from registers.
  p.direct_epi = (!trans || pl.tiles <= 2 * pl.grid || epi == EPI_QKV_ROPE) ? 1 : 0;
  if (epi == EPI_QKV_ROPE) {
    TORCH_CHECK(rope != nullptr && trans && push.empty(), "qkv+rope epilogue: swap-AB, no push");
    p.rope_pos = rope->pos;
    p.rope_slot = rope->slot;
    p.rope_cos = rope->cos;
    p.rope_sin = rope->sin;
    p.rope_k = rope->k;
    p.rope_v = rope->v;
    p.rope_hq = rope->hq;
    p.rope_hkv = rope->hkv;
    p.rope_ps = rope->ps;
  }
  // push = [mode, my_rank, world, rows, slot_stride, ldo, base_0 .. base_{world-1}]
  if (!push.empty()) {
    TORCH_CHECK(epi == EPI_STORE_BF16 && push.size() >= 6, "fused reduce-scatter needs the bf16 epilogue");
    p.push_mode = (int)push[0];
    p.my_rank = (int)push[1];
    p.world = (int)push[2];
    p.push_rows = (int)push[3];
    p.slot_stride = push[4];
    p.ldo = push[5];
    TORCH_CHECK(p.world >= 1 && p.world <= 8 && (int)push.size() == 6 + p.world, "push: peer table");
    for (int i = 0; i < p.world; ++i) p.peer_base[i] = (unsigned long long)push[6 + i];
  }
  if (ar != nullptr) {
    TORCH_CHECK(trans && epi == EPI_STORE_BF16 && p.push_mode == 1 && ar->world == p.world && ar->rank == p.my_rank &&
                    ar->T == N && ar->H == M,
                "fused all-reduce tail: swap-AB bf16 GEMM pushing rows to their owners");
    TORCH_CHECK(pl.grid <= AR_TAIL_MAX_CTAS, "fused all-reduce tail: at most 256 CTAs");
    p.ar = *ar;
    p.ar.on = 1;
  }
  if (trace.has_value()) {
    TORCH_CHECK(trace->numel() >= (int64_t)pl.grid * TRACE_SLOTS && trace->scalar_type() == at::kLong,
                "gemm trace buffer: int64 [grid * 32]");
    p.trace = reinterpret_cast<unsigned long long*>(trace->data_ptr<int64_t>());
  }
  p.err = err.data_ptr<int>();
  p.idesc = make_idesc_bf16(BM, bn);
  p.tmem_cols = tmem_cols_for(bn);

  CUtensorMap ta = tma_map_2d_bf16(A.data_ptr(), K, M, A.stride(0), BK, BM);
  CUtensorMap tb = tma_map_2d_bf16(B.data_ptr(), K, N, B.stride(0), BK, bn);
  const int grid = pl.grid;
  const size_t smem = sp.bytes;
  cudaStream_t stream = at::cuda::getCurrentCUDAStream();
  switch (epi * 2 + (trans ? 1 : 0)) {
    case EPI_STORE_BF16 * 2 + 0: launch_typed<EPI_STORE_BF16, false>(ta, tb, p, grid, smem, stream); break;
    case EPI_STORE_BF16 * 2 + 1: launch_typed<EPI_STORE_BF16, true>(ta, tb, p, grid, smem, stream); break;
    case EPI_STORE_F32 * 2 + 0: launch_typed<EPI_STORE_F32, false>(ta, tb, p, grid, smem, stream); break;
    case EPI_STORE_F32 * 2 + 1: launch_typed<EPI_STORE_F32, true>(ta, tb, p, grid, smem, stream); break;
    case EPI_SILU_BF16 * 2 + 0: launch_typed<EPI_SILU_BF16, false>(ta, tb, p, grid, smem, stream); break;
    case EPI_SILU_BF16 * 2 + 1: launch_typed<EPI_SILU_BF16, true>(ta, tb, p, grid, smem, stream); break;
    case EPI_ARGMAX * 2 + 1: launch_typed<EPI_ARGMAX, true>(ta, tb, p, grid, smem, stream); break;
    case EPI_QKV_ROPE * 2 + 1: launch_typed<EPI_QKV_ROPE, true>(ta, tb, p, grid, smem, stream); break;
    default: TORCH_CHECK(false, "gemm_tcgen05: unknown epilogue ", epi);
  }
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void gemm_tcgen05(const at::Tensor& A, const at::Tensor& B, at::Tensor& out, int64_t epi, bool trans, int64_t bn_req,
                  int64_t mode, at::Tensor& workspace, at::Tensor& counters, at::Tensor& err,
                  const c10::optional<at::Tensor>& trace, const std::vector<int64_t>& push) {
  TORCH_CHECK(epi != EPI_QKV_ROPE, "gemm_tcgen05: use gemm_qkv_rope for the fused RoPE epilogue");
  gemm_impl(A, B, out, epi, trans, bn_req, mode, workspace, counters, err, trace, push, nullptr);
}

// Decode qkv projection with RoPE and the paged KV write fused into the epilogue (swap-AB):
// w [(hq + 2*hkv) * 128, H] rows = q heads, k heads, v heads; x [T, H]; q_out [T, hq*128];
// kcache / vcache one layer of the pool [pages, hkv, page_size, 128]; pos int32 [T]; slot int64 [T]
// (< 0: padding token, nothing written); cos / sin fp32 [max_pos, 64].
void gemm_qkv_rope(const at::Tensor& w, const at::Tensor& x, at::Tensor& q_out, const at::Tensor& pos,
                   const at::Tensor& slot, const at::Tensor& cos_t, const at::Tensor& sin_t, at::Tensor& kcache,
                   at::Tensor& vcache, int64_t hq, int64_t hkv, int64_t mode, at::Tensor& workspace,
                   at::Tensor& counters, at::Tensor& err) {
  const int64_t T = x.size(0);
  TORCH_CHECK(w.size(0) == (hq + 2 * hkv) * 128, "gemm_qkv_rope: head_dim 128, rows q|k|v");
  TORCH_CHECK(q_out.is_contiguous() && q_out.size(0) == T && q_out.size(1) == hq * 128 &&
                  q_out.scalar_type() == at::kBFloat16,
              "gemm_qkv_rope: q_out [T, hq*128] bf16 contiguous");
  TORCH_CHECK(kcache.is_contiguous() && vcache.is_contiguous() && kcache.dim() == 4 && kcache.size(1) == hkv &&
                  kcache.size(3) == 128 && vcache.sizes() == kcache.sizes() &&
                  kcache.scalar_type() == at::kBFloat16 && vcache.scalar_type() == at::kBFloat16,
              "gemm_qkv_rope: kv pages [pages, hkv, page_size, 128] bf16");
  TORCH_CHECK(pos.is_cuda() && pos.numel() >= T && pos.scalar_type() == at::kInt && slot.is_cuda() &&
                  slot.numel() >= T && slot.scalar_type() == at::kLong,
              "gemm_qkv_rope: pos int32 [T], slot int64 [T] on the device");
  TORCH_CHECK(cos_t.scalar_type() == at::kFloat && sin_t.scalar_type() == at::kFloat && cos_t.size(-1) == 64 &&
                  sin_t.size(-1) == 64 && cos_t.is_contiguous() && sin_t.is_contiguous(),
              "gemm_qkv_rope: cos/sin fp32 [max_pos, 64]");
  RopeArgs r;
  r.pos = pos.data_ptr<int>();
  r.slot = reinterpret_cast<const long*>(slot.data_ptr<int64_t>());
  r.cos = cos_t.data_ptr<float>();
  r.sin = sin_t.data_ptr<float>();
  r.k = reinterpret_cast<__nv_bfloat16*>(kcache.data_ptr());
  r.v = reinterpret_cast<__nv_bfloat16*>(vcache.data_ptr());
  r.hq = (int)hq;
  r.hkv = (int)hkv;
  r.ps = (int)kcache.size(2);
  gemm_impl(w, x, q_out, EPI_QKV_ROPE, true, 0, mode, workspace, counters, err, c10::nullopt, {}, &r);
}

// Decode o_proj / down_proj with the tensor-parallel all-reduce, residual add and RMSNorm fused
// in (see ar_tail): w [H, K] weights, x [T, K] activations; the partial rows go to their owner
// ranks' push slots, and after the launch every rank's `normed` holds RMSNorm(resid + sum) * gamma
// for all T rows while each rank's `resid` holds the updated rows it owns.
// push = [1, my_rank, world, T, slot_stride, H, push slot base of each rank (as mapped here)...]
// cfg  = [t_max, off_flags, off_counts, off_push, off_resid, off_normed, multicast base, timeout ns,
//         workspace base of each rank...]; `part` is this rank's local push slot (shape checks only).
void gemm_allreduce_norm(const at::Tensor& w, const at::Tensor& x, at::Tensor& part, const std::vector<int64_t>& push,
                         const std::vector<int64_t>& cfg, const at::Tensor& gamma, double eps, at::Tensor& epoch,
                         int64_t mode, at::Tensor& workspace, at::Tensor& counters, at::Tensor& err,
                         const c10::optional<at::Tensor>& trace) {
  const int64_t T = x.size(0), H = w.size(0);
  TORCH_CHECK(push.size() >= 6 && push[0] == 1 && push[3] == T && push[5] == H, "gemm_allreduce_norm: push table");
  const int world = (int)push[2];
  TORCH_CHECK(world >= 1 && world <= AR_TAIL_MAX_RANKS && (int64_t)cfg.size() == 8 + world,
              "gemm_allreduce_norm: config table");
  TORCH_CHECK(H % 8 == 0 && H <= 128 * 8 * 8, "gemm_allreduce_norm: H % 8 == 0 and H <= 8192");
  TORCH_CHECK(T <= cfg[0], "gemm_allreduce_norm: T exceeds the workspace rows");
  TORCH_CHECK(gamma.is_cuda() && gamma.scalar_type() == at::kBFloat16 && gamma.numel() == H && gamma.is_contiguous(),
              "gemm_allreduce_norm: gamma bf16 [H]");
  TORCH_CHECK(epoch.is_cuda() && epoch.scalar_type() == at::kInt && epoch.numel() >= 1, "gemm_allreduce_norm: epoch");
  TORCH_CHECK(cfg[6] % 16 == 0, "gemm_allreduce_norm: multicast base must be 16-byte aligned");
  ArTail a{};
  a.rank = (int)push[1];
  a.world = world;
  a.T = (int)T;
  a.H = (int)H;
  a.t_max = (int)cfg[0];
  a.off_flags = cfg[1];
  a.off_counts = cfg[2];
  a.off_push = cfg[3];
  a.off_resid = cfg[4];
  a.off_normed = cfg[5];
  a.mc = (unsigned long long)cfg[6];
  a.timeout_ns = (unsigned long long)cfg[7];
  for (int i = 0; i < world; ++i) a.ws[i] = (unsigned long long)cfg[8 + i];
  a.epoch = reinterpret_cast<uint32_t*>(epoch.data_ptr<int>());
  a.gamma = reinterpret_cast<const __nv_bfloat16*>(gamma.data_ptr());
  a.eps = (float)eps;
  gemm_impl(w, x, part, EPI_STORE_BF16, true, 0, mode, workspace, counters, err, trace, push, nullptr, &a);
}

// [bn, workspace floats, stream-K tiles, stages, grid, dp_tiles, sk_iters, cluster split]
// (the plan of the automatic schedule without a push table)
std::vector<int64_t> gemm_plan(int64_t M, int64_t N, int64_t K, int64_t epi, bool trans, int64_t device) {
  const c10::cuda::CUDAGuard guard((c10::DeviceIndex)device);
  int bn = gemm_pick_bn((int)N, (int)epi, trans);
  const int kbox = kbox_for(trans);
  Plan pl = make_plan((int)M, (int)N, (int)K, bn, num_sms_cached((int)device), 0, (int)epi, trans, false, kbox);
  return {bn, (int64_t)pl.ws_floats, pl.sk_tiles, smem_plan(bn, pl.ck, kbox, (int)epi, trans).stages, pl.grid, pl.dp_tiles, pl.sk_iters,
          pl.ck};
}

}  // namespace mesh
