// Tensor-parallel all-reduce fused with residual add + RMSNorm, over NVLink peer memory.
//
// Each rank's o_proj / down_proj GEMM writes its bf16 partial [T, H] into its own slot of a
// symmetric workspace (one allocation per rank, mapped into every peer). This kernel then
//   one-shot: every rank reads all peers' partials for every row, adds the residual, applies
//             RMSNorm and writes resid/normed locally (latency-optimal for decode-sized T);
//   two-shot: rank r reduces only its 1/n share of the rows, keeps the updated residual rows
//             (only their owner reads them in the later layers of the step), pushes the normed
//             rows into every peer's workspace (P2P or multicast stores) and signals completion
//             (bandwidth-optimal for prefill-sized T).
// Replaces the reference's host-staged TCP ring all-reduce (ring_allreduce.rs:1029-1119 and the
// device->host->device chunk copies of runtime.rs:715-752) and its separate residual add/norm.
//
// Synchronisation: per-block epoch flags in the symmetric workspace. A block raises its flag in
// every peer with st.release.sys and waits (ld.acquire.sys, %globaltimer limit) for the peers'
// flags of the same epoch. Epochs live in a device counter so CUDA-graph replays stay consistent.
// Partial buffers alternate between two slots (parity = call index % 2): the start barrier of
// call i+1 proves every peer finished reading slot (i % 2) in call i, so one barrier per call
// suffices for one-shot. A timed-out wait records ERR_PEER_TIMEOUT and the kernel returns.
#include <ATen/ATen.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/extension.h>

#include <algorithm>
#include <cstdlib>

#include "../include/sm100.cuh"
#include "../include/launch.h"

namespace mesh {

constexpr int AR_MAX_RANKS = 8;
constexpr int AR_MAX_BLOCKS = 256;
constexpr int AR_THREADS = 256;

struct ArArgs {
  uint64_t base[AR_MAX_RANKS];  // symmetric workspace base address of each rank (as mapped here)
  long off_flags;               // uint32 flags: [2 phases][AR_MAX_BLOCKS][AR_MAX_RANKS]
  long off_partial[2];          // bf16 [T_max, H] partial slots
  long off_resid, off_normed;   // bf16 [T_max, H] outputs (symmetric for two-shot)
  int rank, world, T, H, parity;
  const __nv_bfloat16* gamma;
  float eps;
  uint32_t* epoch;              // local [AR_MAX_BLOCKS]
  int* err;
  uint64_t timeout_ns;
  // fused reduce-scatter mode: the GEMMs of all ranks pushed their bf16 partial rows into this
  // rank's slots [world][t_max][H] at off_push; reduction reads local memory only
  int push;
  long off_push;
  int t_max;
  // NVLS multicast base of the symmetric workspace (same offsets as base[]); 0 = plain peer loads
  uint64_t mc;
  uint64_t* trace;  // optional: block 0 records %globaltimer at start / after barrier / rows done / end
  // 1: one sys-scope fence per block, then relaxed flag stores (instead of a release store per peer)
  int single_fence;
};

inline int ar_single_fence() {
  static int v = -1;
  if (v < 0) {
    const char* e = std::getenv("MESH_AR_SINGLE_FENCE");
    v = (e && e[0] == '1') ? 1 : 0;
  }
  return v;
}

__device__ __forceinline__ uint32_t* flag_ptr(const ArArgs& a, int peer, int phase, int block, int src) {
  return reinterpret_cast<uint32_t*>(a.base[peer] + a.off_flags) +
         ((long)phase * AR_MAX_BLOCKS + block) * AR_MAX_RANKS + src;
}

// Returns false (uniformly across the block) if a peer did not arrive in time.
__device__ __forceinline__ bool block_barrier(const ArArgs& a, int phase, uint32_t e, int* s_ok) {
  const int b = blockIdx.x;
  if (threadIdx.x == 0) {
    *s_ok = 1;
    if (a.single_fence) fence_acq_rel_sys();
  }
  __syncthreads();
  if (threadIdx.x < a.world) {
    if (a.single_fence)
      st_relaxed_sys(flag_ptr(a, threadIdx.x, phase, b, a.rank), e);
    else
      st_release_sys(flag_ptr(a, threadIdx.x, phase, b, a.rank), e);
  }
  if (threadIdx.x < a.world) {
    if (!wait_flag_geq(flag_ptr(a, a.rank, phase, b, threadIdx.x), e, a.timeout_ns, a.err)) *s_ok = 0;
  }
  __syncthreads();
  return *s_ok != 0;
}

// Reduce one row over `nsrc` partial sources, add residual, RMSNorm; returns values in x (fp32).
__device__ __forceinline__ const uint4* src_row(const ArArgs& a, int p, long row) {
  const __nv_bfloat16* s =
      a.push ? reinterpret_cast<const __nv_bfloat16*>(a.base[a.rank] + a.off_push) + ((long)p * a.t_max + row) * a.H
             : reinterpret_cast<const __nv_bfloat16*>(a.base[p] + a.off_partial[a.parity]) + row * a.H;
  return reinterpret_cast<const uint4*>(s);
}

template <int MAXV, bool MC>
__device__ __forceinline__ void reduce_norm_row(const ArArgs& a, long row, float (&x)[MAXV][8], float* red,
                                                float& inv) {
  const int nvec = a.H / 8;
  const __nv_bfloat16* resid = reinterpret_cast<const __nv_bfloat16*>(a.base[a.rank] + a.off_resid);
  float ss = 0.f;
  // issue every source's loads before consuming any (one NVLink round trip per row, not one per
  // rank); with NVLS the switch returns the sum over all ranks in a single load
  constexpr int NSRC = MC ? 1 : AR_MAX_RANKS;
  const int nsrc = MC ? 1 : a.world;
  uint4 d[NSRC][MAXV];
  if (MC) {
    const uint4* sr = reinterpret_cast<const uint4*>(a.mc + a.off_partial[a.parity]) + row * nvec;
#pragma unroll
    for (int i = 0; i < MAXV; ++i) {
      const int v = threadIdx.x + i * AR_THREADS;
      if (v < nvec) d[0][i] = multimem_ld_reduce_bf16x8(sr + v);
    }
  }
#pragma unroll
  for (int p = 0; p < NSRC; ++p) {
    if (!MC && p < a.world) {
      const uint4* sr = src_row(a, p, row);
#pragma unroll
      for (int i = 0; i < MAXV; ++i) {
        const int v = threadIdx.x + i * AR_THREADS;
        if (v < nvec) d[p][i] = __ldcg(sr + v);
      }
    }
  }
#pragma unroll
  for (int i = 0; i < MAXV; ++i) {
    const int v = threadIdx.x + i * AR_THREADS;
    if (v < nvec) {
      uint4 r = *reinterpret_cast<const uint4*>(resid + row * a.H + v * 8);
      const uint32_t* ru = reinterpret_cast<const uint32_t*>(&r);
#pragma unroll
      for (int j = 0; j < 4; ++j) unpack_bf16x2(ru[j], x[i][2 * j], x[i][2 * j + 1]);
#pragma unroll
      for (int p = 0; p < NSRC; ++p) {
        if (p < nsrc) {
          const uint32_t* du = reinterpret_cast<const uint32_t*>(&d[p][i]);
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            float u0, u1;
            unpack_bf16x2(du[j], u0, u1);
            x[i][2 * j] += u0;
            x[i][2 * j + 1] += u1;
          }
        }
      }
      // round the new residual to bf16 (what gets stored), normalise that value
#pragma unroll
      for (int j = 0; j < 8; j += 2) {
        uint32_t pk = pack_bf16x2(x[i][j], x[i][j + 1]);
        unpack_bf16x2(pk, x[i][j], x[i][j + 1]);
        ss += x[i][j] * x[i][j] + x[i][j + 1] * x[i][j + 1];
      }
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
  if (l == 0) red[w] = ss;
  __syncthreads();
  float t = (l < AR_THREADS / 32) ? red[l] : 0.f;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) t += __shfl_xor_sync(0xffffffffu, t, o);
  inv = rsqrtf(t / (float)a.H + a.eps);
  __syncthreads();
}

// dst_rank < 0: multicast store into every rank (NVLS)
template <int MAXV>
__device__ __forceinline__ void store_row(const ArArgs& a, int dst_rank, long row, const float (&x)[MAXV][8],
                                          float inv) {
  const int nvec = a.H / 8;
  const uint64_t db = dst_rank < 0 ? a.mc : a.base[dst_rank];
  __nv_bfloat16* resid = reinterpret_cast<__nv_bfloat16*>(db + a.off_resid);
  __nv_bfloat16* normed = reinterpret_cast<__nv_bfloat16*>(db + a.off_normed);
  uint4* resid_l = reinterpret_cast<uint4*>(a.base[a.rank] + a.off_resid);
#pragma unroll
  for (int i = 0; i < MAXV; ++i) {
    const int v = threadIdx.x + i * AR_THREADS;
    if (v < nvec) {
      uint4 g = *reinterpret_cast<const uint4*>(a.gamma + v * 8);
      const uint32_t* gu = reinterpret_cast<const uint32_t*>(&g);
      uint4 ro, no;
      uint32_t* rou = reinterpret_cast<uint32_t*>(&ro);
      uint32_t* nou = reinterpret_cast<uint32_t*>(&no);
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        float g0, g1;
        unpack_bf16x2(gu[j], g0, g1);
        rou[j] = pack_bf16x2(x[i][2 * j], x[i][2 * j + 1]);
        nou[j] = pack_bf16x2(x[i][2 * j] * inv * g0, x[i][2 * j + 1] * inv * g1);
      }
      // the residual row stays with the rank that reduced it (only that rank reads it in later
      // layers of the same step); the normed row goes wherever the next GEMM runs
      if (dst_rank < 0) {
        resid_l[row * a.H / 8 + v] = ro;
        multimem_st_16(normed + row * a.H + v * 8, no);
      } else {
        if (dst_rank == a.rank) *reinterpret_cast<uint4*>(resid + row * a.H + v * 8) = ro;
        *reinterpret_cast<uint4*>(normed + row * a.H + v * 8) = no;
      }
    }
  }
}

// Warp-per-row reduction: each warp owns one token row at a time. Pass 1 sums the residual and the
// sources chunk by chunk (two 16-byte chunks per lane in flight per source), stores the bf16 residual
// (locally, and into every rank for two-shot) and accumulates the sum of squares; pass 2 re-reads the
// residual it just wrote and stores the normalised row. No block-wide synchronisation per row, so
// thousands of rows are in flight and remote-load latency overlaps.
template <bool TWO_SHOT, bool MC>
__device__ __forceinline__ void warp_reduce_norm_row(const ArArgs& a, long row, int lane) {
  const int nvec = a.H / 8;
  uint4* resid_l = reinterpret_cast<uint4*>(reinterpret_cast<__nv_bfloat16*>(a.base[a.rank] + a.off_resid) + row * a.H);
  const uint4* gv = reinterpret_cast<const uint4*>(a.gamma);
  float ss = 0.f;
  constexpr int U = 4;
  for (int c0 = lane; c0 < nvec; c0 += 32 * U) {
    float acc[U][8];
    bool ok[U];
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int c = c0 + u * 32;
      ok[u] = c < nvec;
      if (ok[u]) {
        uint4 r = resid_l[c];
        const uint32_t* ru = reinterpret_cast<const uint32_t*>(&r);
#pragma unroll
        for (int j = 0; j < 4; ++j) unpack_bf16x2(ru[j], acc[u][2 * j], acc[u][2 * j + 1]);
      }
    }
    constexpr int NSRC = MC ? 1 : AR_MAX_RANKS;
    const int nsrc = MC ? 1 : a.world;
    uint4 d[NSRC][U];
    if (MC) {
      const uint4* sr = reinterpret_cast<const uint4*>(a.mc + a.off_partial[a.parity]) + row * nvec;
#pragma unroll
      for (int u = 0; u < U; ++u)
        if (ok[u]) d[0][u] = multimem_ld_reduce_bf16x8(sr + c0 + u * 32);
    }
#pragma unroll
    for (int p = 0; p < NSRC; ++p) {
      if (!MC && p < a.world) {
        const uint4* sr = src_row(a, p, row);
#pragma unroll
        for (int u = 0; u < U; ++u)
          if (ok[u]) d[p][u] = __ldcg(sr + c0 + u * 32);
      }
    }
#pragma unroll
    for (int p = 0; p < NSRC; ++p) {
      if (p >= nsrc) continue;
#pragma unroll
      for (int u = 0; u < U; ++u) {
        if (!ok[u]) continue;
        const uint32_t* du = reinterpret_cast<const uint32_t*>(&d[p][u]);
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          float x0, x1;
          unpack_bf16x2(du[j], x0, x1);
          acc[u][2 * j] += x0;
          acc[u][2 * j + 1] += x1;
        }
      }
    }
#pragma unroll
    for (int u = 0; u < U; ++u) {
      if (!ok[u]) continue;
      uint4 o;
      uint32_t* ou = reinterpret_cast<uint32_t*>(&o);
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        ou[j] = pack_bf16x2(acc[u][2 * j], acc[u][2 * j + 1]);
        float r0, r1;
        unpack_bf16x2(ou[j], r0, r1);  // normalise the stored (bf16-rounded) residual
        ss += r0 * r0 + r1 * r1;
      }
      const int c = c0 + u * 32;
      // two-shot too: the residual row stays local (only its owner reads it in later layers of
      // the same step), so only the normed rows are all-gathered
      resid_l[c] = o;
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
  const float inv = rsqrtf(ss / (float)a.H + a.eps);
  for (int c = lane; c < nvec; c += 32) {
    uint4 r = resid_l[c];
    uint4 g = gv[c];
    const uint32_t* ru = reinterpret_cast<const uint32_t*>(&r);
    const uint32_t* gu = reinterpret_cast<const uint32_t*>(&g);
    uint4 o;
    uint32_t* ou = reinterpret_cast<uint32_t*>(&o);
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      float r0, r1, g0, g1;
      unpack_bf16x2(ru[j], r0, r1);
      unpack_bf16x2(gu[j], g0, g1);
      ou[j] = pack_bf16x2(r0 * inv * g0, r1 * inv * g1);
    }
    if (TWO_SHOT && MC) {
      multimem_st_16(reinterpret_cast<uint4*>(reinterpret_cast<__nv_bfloat16*>(a.mc + a.off_normed) + row * a.H) + c, o);
    } else if (TWO_SHOT) {
      for (int q = 0; q < a.world; ++q)
        reinterpret_cast<uint4*>(reinterpret_cast<__nv_bfloat16*>(a.base[q] + a.off_normed) + row * a.H)[c] = o;
    } else {
      reinterpret_cast<uint4*>(reinterpret_cast<__nv_bfloat16*>(a.base[a.rank] + a.off_normed) + row * a.H)[c] = o;
    }
  }
}

// ROW_BLOCK: one 256-thread block per row (every 16-byte chunk of the row loaded at once; best when
// a rank reduces few rows, e.g. decode); otherwise one warp per row (best for prefill-sized T).
// MC: partial sums come from NVLS multicast loads (the switch adds the ranks' rows) and two-shot
// results leave through multicast stores; otherwise plain peer loads / stores.
template <int MAXV, bool TWO_SHOT, bool ROW_BLOCK, bool MC>
__global__ void __launch_bounds__(AR_THREADS) ar_norm_kernel(const ArArgs a) {
  __shared__ float red[32];
  __shared__ int s_ok;
  __shared__ uint32_t s_epoch;
  const int b = blockIdx.x;
  const bool tr = a.trace != nullptr && b == 0 && threadIdx.x == 0;
  griddep_wait();  // partials come from the GEMM just before
  griddep_launch_dependents();
  if (tr) a.trace[0] = globaltimer_ns();
  if (threadIdx.x == 0) s_epoch = a.epoch[b] + 1;
  __syncthreads();
  const uint32_t e = s_epoch;
  // No proxy fences around the multicast accesses: the partials were written by earlier kernels
  // in stream order and the sys-scope release/acquire flags order them for every rank (the same
  // contract as the multicast all-reduce kernels of torch symmetric memory).
  const bool ok = block_barrier(a, 0, e, &s_ok);
  if (threadIdx.x == 0) a.epoch[b] = e;
  if (!ok) return;
  if (tr) a.trace[1] = globaltimer_ns();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const long gw = (long)b * (AR_THREADS / 32) + warp;
  const long nw = (long)gridDim.x * (AR_THREADS / 32);
  long r0 = 0, r1 = a.T;
  if (TWO_SHOT) {
    const int base_rows = a.T / a.world, extra = a.T % a.world;
    r0 = (long)a.rank * base_rows + min(a.rank, extra);
    r1 = r0 + base_rows + (a.rank < extra ? 1 : 0);
  }
  if (ROW_BLOCK) {
    float x[MAXV][8];
    float inv;
    for (long row = r0 + b; row < r1; row += gridDim.x) {
      reduce_norm_row<MAXV, MC>(a, row, x, red, inv);
      if (TWO_SHOT && MC) {
        store_row<MAXV>(a, -1, row, x, inv);
      } else if (TWO_SHOT) {
        for (int p = 0; p < a.world; ++p) store_row<MAXV>(a, (a.rank + p) % a.world, row, x, inv);
      } else {
        store_row<MAXV>(a, a.rank, row, x, inv);
      }
    }
  } else {
    for (long row = r0 + gw; row < r1; row += nw) warp_reduce_norm_row<TWO_SHOT, MC>(a, row, lane);
  }
  if (tr) a.trace[2] = globaltimer_ns();
  if (TWO_SHOT) {
    __threadfence_system();
    block_barrier(a, 1, e, &s_ok);
  }
  if (tr) a.trace[3] = globaltimer_ns();
}

// Rows this rank reduces; block-per-row up to 255 rows, warp-per-row (8 rows per block) above.
template <bool MC>
inline void launch_ar_t(const ArArgs& a, bool two_shot, cudaStream_t st) {
  const long rows = two_shot ? (a.T + a.world - 1) / a.world : a.T;
  const bool row_block = rows < AR_MAX_BLOCKS;
  const int nb = row_block ? (int)std::max<long>(1, rows) : (int)std::min<long>((rows + 7) / 8, AR_MAX_BLOCKS - 1);
  if (two_shot) {
    if (row_block)
      launch_k(ar_norm_kernel<4, true, true, MC>, dim3(nb), dim3(AR_THREADS), 0, st, a);
    else
      launch_k(ar_norm_kernel<4, true, false, MC>, dim3(nb), dim3(AR_THREADS), 0, st, a);
  } else {
    if (row_block)
      launch_k(ar_norm_kernel<4, false, true, MC>, dim3(nb), dim3(AR_THREADS), 0, st, a);
    else
      launch_k(ar_norm_kernel<4, false, false, MC>, dim3(nb), dim3(AR_THREADS), 0, st, a);
  }
}

inline void launch_ar(const ArArgs& a_in, bool two_shot, cudaStream_t st) {
  ArArgs a = a_in;
  a.single_fence = ar_single_fence();
  if (a.mc != 0 && !a.push)
    launch_ar_t<true>(a, two_shot, st);
  else
    launch_ar_t<false>(a, two_shot, st);
}

// One rank's view of the symmetric workspace and where its regions sit.
void ar_fused_norm(const at::Tensor& bases, int64_t off_flags, int64_t off_p0, int64_t off_p1, int64_t off_resid,
                   int64_t off_normed, int64_t rank, int64_t world, int64_t T, int64_t H, int64_t parity,
                   const at::Tensor& gamma, double eps, at::Tensor& epoch, at::Tensor& err, int64_t nblocks,
                   bool two_shot, double timeout_s, int64_t mc_base, const at::Tensor& trace) {
  TORCH_CHECK(world >= 1 && world <= AR_MAX_RANKS, "ar_fused_norm: world size 1..8");
  TORCH_CHECK(mc_base % 16 == 0, "ar_fused_norm: multicast base must be 16-byte aligned");
  TORCH_CHECK(!trace.defined() || trace.numel() == 0 || (trace.is_cuda() && trace.numel() >= 4 &&
                                                         trace.scalar_type() == at::kLong),
              "ar_fused_norm: trace must be a CUDA int64 tensor of >= 4 elements");
  TORCH_CHECK(bases.numel() == world && bases.scalar_type() == at::kLong && bases.device().is_cpu(),
              "ar_fused_norm: bases must be a CPU int64 tensor of peer addresses");
  TORCH_CHECK(H % 8 == 0 && H <= 8 * AR_THREADS * 4, "ar_fused_norm: H % 8 and H <= 8192");
  TORCH_CHECK(nblocks >= 1 && nblocks < AR_MAX_BLOCKS, "ar_fused_norm: nblocks must be < 256 (last flag row is the setup barrier)");
  TORCH_CHECK(epoch.numel() >= AR_MAX_BLOCKS && epoch.scalar_type() == at::kInt, "ar_fused_norm: epoch counters");
  if (T == 0) return;
  const c10::cuda::CUDAGuard guard(gamma.device());
  ArArgs a{};
  auto bp = bases.data_ptr<int64_t>();
  for (int i = 0; i < world; ++i) a.base[i] = (uint64_t)bp[i];
  a.off_flags = off_flags;
  a.off_partial[0] = off_p0;
  a.off_partial[1] = off_p1;
  a.off_resid = off_resid;
  a.off_normed = off_normed;
  a.rank = (int)rank;
  a.world = (int)world;
  a.T = (int)T;
  a.H = (int)H;
  a.parity = (int)(parity & 1);
  a.gamma = reinterpret_cast<const __nv_bfloat16*>(gamma.data_ptr());
  a.eps = (float)eps;
  a.epoch = reinterpret_cast<uint32_t*>(epoch.data_ptr<int>());
  a.err = err.data_ptr<int>();
  a.timeout_ns = (uint64_t)(timeout_s * 1e9);
  a.mc = (uint64_t)mc_base;
  a.trace = (trace.defined() && trace.numel() > 0) ? reinterpret_cast<uint64_t*>(trace.data_ptr<int64_t>()) : nullptr;
  cudaStream_t st = at::cuda::getCurrentCUDAStream();
  launch_ar(a, two_shot, st);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

// Bare barrier across ranks (used at setup and by tests of the bounded-wait error path).
__global__ void ar_barrier_kernel(const ArArgs a) {
  __shared__ int s_ok;
  __shared__ uint32_t s_epoch;
  griddep_wait();
  if (threadIdx.x == 0) s_epoch = a.epoch[AR_MAX_BLOCKS - 1] + 1;
  __syncthreads();
  block_barrier(a, 0, s_epoch, &s_ok);
  if (threadIdx.x == 0) a.epoch[AR_MAX_BLOCKS - 1] = s_epoch;
}

void ar_barrier(const at::Tensor& bases, int64_t off_flags, int64_t rank, int64_t world, at::Tensor& epoch,
                at::Tensor& err, double timeout_s, const at::Tensor& device_ref) {
  TORCH_CHECK(bases.numel() == world && bases.device().is_cpu(), "ar_barrier: bases");
  const c10::cuda::CUDAGuard guard(device_ref.device());
  ArArgs a{};
  auto bp = bases.data_ptr<int64_t>();
  for (int i = 0; i < world; ++i) a.base[i] = (uint64_t)bp[i];
  a.off_flags = off_flags;
  a.rank = (int)rank;
  a.world = (int)world;
  a.epoch = reinterpret_cast<uint32_t*>(epoch.data_ptr<int>());
  a.err = err.data_ptr<int>();
  a.timeout_ns = (uint64_t)(timeout_s * 1e9);
  // uses block slot AR_MAX_BLOCKS-1 of phase 0; launched with one block whose id is 0, so
  // remap through a dedicated flag row by offsetting the flags base
  a.off_flags = off_flags + (long)(AR_MAX_BLOCKS - 1) * AR_MAX_RANKS * 4;
  a.epoch = reinterpret_cast<uint32_t*>(epoch.data_ptr<int>());
  ar_barrier_kernel<<<1, 32, 0, at::cuda::getCurrentCUDAStream()>>>(a);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

int64_t ar_flags_bytes() { return 2L * AR_MAX_BLOCKS * AR_MAX_RANKS * 4; }

// Second half of the fused GEMM -> reduce-scatter: the o_proj / down GEMMs of all ranks already
// pushed their partial rows into this rank's slots over NVLink (two-shot: only the rows this rank
// owns; one-shot: every row). Wait for the peers, sum the slots from local memory, add the
// residual, RMSNorm, and (two-shot) all-gather the resulting rows into every rank.
void ar_push_reduce_norm(const at::Tensor& bases, int64_t off_flags, int64_t off_push, int64_t off_resid,
                         int64_t off_normed, int64_t rank, int64_t world, int64_t T, int64_t t_max, int64_t H,
                         const at::Tensor& gamma, double eps, at::Tensor& epoch, at::Tensor& err, int64_t nblocks,
                         bool two_shot, double timeout_s) {
  TORCH_CHECK(world >= 1 && world <= AR_MAX_RANKS && bases.numel() == world && bases.device().is_cpu(),
              "ar_push_reduce_norm: bases");
  TORCH_CHECK(H % 8 == 0 && H <= 8 * AR_THREADS * 4 && T <= t_max, "ar_push_reduce_norm: shapes");
  TORCH_CHECK(nblocks >= 1 && nblocks < AR_MAX_BLOCKS, "ar_push_reduce_norm: nblocks");
  if (T == 0) return;
  const c10::cuda::CUDAGuard guard(gamma.device());
  ArArgs a{};
  auto bp = bases.data_ptr<int64_t>();
  for (int i = 0; i < world; ++i) a.base[i] = (uint64_t)bp[i];
  a.off_flags = off_flags;
  a.off_resid = off_resid;
  a.off_normed = off_normed;
  a.rank = (int)rank;
  a.world = (int)world;
  a.T = (int)T;
  a.H = (int)H;
  a.gamma = reinterpret_cast<const __nv_bfloat16*>(gamma.data_ptr());
  a.eps = (float)eps;
  a.epoch = reinterpret_cast<uint32_t*>(epoch.data_ptr<int>());
  a.err = err.data_ptr<int>();
  a.timeout_ns = (uint64_t)(timeout_s * 1e9);
  a.push = 1;
  a.off_push = off_push;
  a.t_max = (int)t_max;
  cudaStream_t st = at::cuda::getCurrentCUDAStream();
  launch_ar(a, two_shot, st);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

}  // namespace mesh
