// Prefill-sized GEMM on SM pairs: out[M, N] = A[M, K] * B[N, K]^T with tcgen05.mma.cta_group::2.
//
// A cluster of two CTAs (two SMs) owns a 256 x 256 output tile. Each CTA stages its own 128 rows of A
// (activations) and its own 128 rows of B (weights, half of N) in shared memory; the leader CTA
// (cluster rank 0) issues one 256 x 256 x 16 MMA per k step that reads both CTAs' tiles, and each
// CTA's TMEM receives its 128 output rows x 256 columns. Per SM and k step this moves 32 KB through
// shared memory for 128 x 256 x 64 multiply-adds, where a one-SM 128 x 256 tile moves 48 KB: the
// operand traffic that bounds the one-SM kernel at large M drops by a third.
//
// Roles per CTA (192 threads): warp 0 TMA producer (both CTAs; every load completes on the leader's
// "full" barrier of the stage), warp 1 MMA issuer (leader only), warps 2..5 epilogue (both CTAs:
// TMEM -> registers -> bf16 global stores; SiLU(gate) * up for the interleaved gate/up weights).
// Accumulators are double-buffered (2 x 256 TMEM columns) so the epilogue of one tile overlaps the
// mainloop of the next. Persistent: clusters walk the tiles in groups of 8 M-tiles for L2 reuse.
// Every wait is bounded; on a timeout the kernel records an error code and unwinds. No TMA load here
// uses cluster multicast.
#include <ATen/ATen.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/extension.h>

#include <algorithm>
#include <cstdlib>

#include "../include/launch.h"
#include "../include/sm100.cuh"
#include "../include/tma_host.h"

namespace mesh {
namespace g2sm {

constexpr int TM = 256;                        // output rows per SM pair (128 per CTA)
constexpr int BK = 64;                         // k elements per stage (one 128-byte swizzle atom)
constexpr uint32_t A_BYTES = 128 * BK * 2;     // one CTA's 128 rows of A for one stage
// Tile width TN (128, 256 or 512 output columns per pair). Up to 256 columns one MMA of N = TN per
// 16-wide k step and two accumulators (the epilogue of a tile overlaps the next mainloop); 512
// columns issue two N = 256 MMAs that share the A stage (a quarter less operand traffic per FLOP)
// into one accumulator that fills TMEM, so the epilogue does not overlap.
template <int TN>
struct Tile {
  static constexpr int NSUB = TN == 512 ? 2 : 1;                // MMAs per 16-wide k step
  static constexpr int MMA_N = TN / NSUB;
  static constexpr int BROWS = MMA_N / 2;                       // rows of B per CTA per MMA
  static constexpr uint32_t B_SUB_BYTES = BROWS * BK * 2;
  static constexpr uint32_t B_BYTES = NSUB * B_SUB_BYTES;
  static constexpr uint32_t STAGE_BYTES = A_BYTES + B_BYTES;
  static constexpr int NACC = TN == 512 ? 1 : 2;                // accumulators in TMEM
  static constexpr uint32_t TMEM_COLS = NACC * TN;
};
constexpr int MAX_STAGES = 9;                  // 24 KB stages (TN = 128) fit 9 times
constexpr int NUM_THREADS = 192;
constexpr uint64_t WAIT_LIMIT_NS = 2000000000ull;
enum Epi : int { STORE_BF16 = 0, SILU_BF16 = 2 };

struct Params {
  __nv_bfloat16* out;
  int M, N, K;        // N = columns of the product (before SiLU halving)
  int ldo;            // out row stride (elements)
  int m_tiles, n_tiles, k_blocks;
  int spin;  // 1: waits poll the barrier; 0: waits sleep inside try_wait between polls
  int stages;
  int* err;
  unsigned long long* trace;  // optional: cluster 0's first 128 k-steps, %globaltimer stamps
};

struct Bars {
  uint64_t full[MAX_STAGES];   // leader: both CTAs' loads of the stage landed
  uint64_t empty[MAX_STAGES];  // each CTA: the stage's MMAs are done with its shared memory (leader:
                           // MMA commit; peer: relayed by the leader's producer)
  uint64_t tfull[2];       // each CTA: accumulator complete (peer: relayed by the leader's epilogue)
  uint64_t tempty[2];      // leader: both CTAs' epilogues finished reading the accumulator
  uint64_t mma_done;       // leader: every issued MMA completed
  uint32_t tmem_base;
  int abort;
  int epi_ok;
};

template <int TN>
constexpr size_t smem_bytes(int stages) { return 1024 + (size_t)stages * Tile<TN>::STAGE_BYTES + sizeof(Bars); }

__device__ __forceinline__ uint32_t leader_addr(const void* p) { return mapa_shared(smem_u32(p), 0); }

// 2D TMA load into this CTA's shared memory whose completion is counted on a barrier that may live
// in the peer CTA of the pair (cluster address).
__device__ __forceinline__ void tma_load_2d_pair(void* dst, const CUtensorMap* map, uint32_t bar_cluster, int x, int y,
                                                 uint64_t hint) {
  asm volatile(
      "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint"
      " [%0], [%1, {%3, %4}], [%2], %5;" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(bar_cluster), "r"(x), "r"(y), "l"(hint)
      : "memory");
}
__device__ __forceinline__ void mbar_arrive_cluster(uint32_t bar_cluster) {
  asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(bar_cluster) : "memory");
}
// Signal-only remote arrive (orders nothing): the stage release the leader relays to its peer, whose
// ordering against the MMA's reads the leader already obtained from the MMA commit.
__device__ __forceinline__ void mbar_arrive_cluster_relaxed(uint32_t bar_cluster) {
  asm volatile("mbarrier.arrive.relaxed.cluster.shared::cluster.b64 _, [%0];" ::"r"(bar_cluster) : "memory");
}
// D[tmem] (+)= A * B^T over the SM pair (issued by the leader; descriptors address both CTAs' tiles).
__device__ __forceinline__ void umma_pair(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                          uint32_t accumulate) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
      " tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p;\n}\n" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}
// Arrive on a barrier of the leader CTA once the prior MMAs of the pair are done.
__device__ __forceinline__ void umma_commit_pair(uint32_t bar_cluster) {
  asm volatile("tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar_cluster)
               : "memory");
}
__device__ __forceinline__ bool wait_bar(uint64_t* bar, uint32_t parity, int* err, int code, volatile int* abort_flag,
                                         int spin) {
  return spin ? mbar_wait_bounded(bar, parity, err, code, abort_flag, WAIT_LIMIT_NS)
              : mbar_wait_bounded_sleep(bar, parity, err, code, abort_flag, WAIT_LIMIT_NS);
}

// grouped raster: 8 consecutive M-tiles sweep all N-tiles before the next group
__device__ __forceinline__ void tile_mn(int t, const Params& p, int& tm, int& tn) {
  const int G = 8;
  const int gsz = G * p.n_tiles;
  const int g = t / gsz;
  const int first = g * G;
  const int gm = min(p.m_tiles - first, G);
  const int in = t - g * gsz;
  tm = first + in % gm;
  tn = in / gm;
}

template <int EPI, int TN>
__global__ void __launch_bounds__(NUM_THREADS, 1)
    gemm_2sm_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB, const Params p) {
  constexpr uint32_t STAGE_BYTES = Tile<TN>::STAGE_BYTES;
  constexpr uint32_t TMEM_COLS = Tile<TN>::TMEM_COLS;
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw = smem_u32(smem_raw);
  uint8_t* stages = smem_raw + (((raw + 1023u) & ~1023u) - raw);
  Bars* bars = reinterpret_cast<Bars*>(stages + (size_t)p.stages * STAGE_BYTES);
  const int STAGES = p.stages;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t rank = cluster_ctarank();  // 0 = leader of the pair
  const int cluster = blockIdx.x >> 1, nclusters = gridDim.x >> 1;
  const int tiles = p.m_tiles * p.n_tiles;

  if (threadIdx.x == 0) {
    for (int i = 0; i < MAX_STAGES; ++i) {
      mbar_init(&bars->full[i], 1);
      mbar_init(&bars->empty[i], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&bars->tfull[i], 1);
      mbar_init(&bars->tempty[i], 2);
    }
    mbar_init(&bars->mma_done, 1);
    bars->abort = 0;
    fence_mbar_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(&bars->tmem_base)),
                 "r"(TMEM_COLS)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
  }
  tc_fence_before();
  // both CTAs' barriers are initialised before any remote arrive or load targets them
  cluster_sync();
  tc_fence_after();
  const uint32_t tmem = bars->tmem_base;
  volatile int* abort_flag = &bars->abort;
  griddep_launch_dependents();

  if (warp == 0) {
    // -------------------------------- TMA producer (both CTAs) --------------------------------
    if (lane == 0) {
      const uint64_t pol_a = policy_evict_last(), pol_b = policy_evict_last();
      griddep_wait();
      int stage = 0;
      uint32_t phase = 0;
      long kb_seq = 0;  // stages filled so far (the first STAGES need no release)
      bool ok = true;
      for (int t = cluster; t < tiles && ok; t += nclusters) {
        int tm, tn;
        tile_mn(t, p, tm, tn);
        const int arow = tm * TM + (int)rank * 128, brow = tn * TN + (int)rank * Tile<TN>::BROWS;
        for (int kb = 0; kb < p.k_blocks; ++kb) {
          // the leader learns from its MMA commit that both CTAs' copies of the stage were consumed
          // and passes that on to the peer's producer (a plain remote arrive)
          if (!wait_bar(&bars->empty[stage], phase ^ 1u, p.err, ERR_MBAR_TIMEOUT_PRODUCER, abort_flag, p.spin)) {
            ok = false;
            break;
          }
          if (rank == 0 && (kb_seq >= STAGES)) mbar_arrive_cluster_relaxed(mapa_shared(smem_u32(&bars->empty[stage]), 1));
          if (p.trace && cluster == 0 && kb_seq < 128) p.trace[(rank ? 128 : 0) + kb_seq] = globaltimer_ns();
          ++kb_seq;
          const uint32_t full = leader_addr(&bars->full[stage]);
          // the leader's barrier counts both CTAs' bytes; one arrival (the leader's, on its own
          // barrier through the CTA-local form) per phase
          if (rank == 0) mbar_arrive_expect_tx(&bars->full[stage], 2 * STAGE_BYTES);
          uint8_t* st = stages + (size_t)stage * STAGE_BYTES;
          tma_load_2d_pair(st, &tmA, full, kb * BK, arow, pol_a);
#pragma unroll
          for (int h = 0; h < Tile<TN>::NSUB; ++h)
            tma_load_2d_pair(st + A_BYTES + h * Tile<TN>::B_SUB_BYTES, &tmB, full, kb * BK,
                             brow + h * Tile<TN>::MMA_N, pol_b);
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
      }
      if (!ok) {
        // give copies already in flight a bounded time to land before the CTA leaves
        const uint64_t t0 = globaltimer_ns();
        while (globaltimer_ns() - t0 < 2000000ull) {
        }
      }
    }
    __syncwarp();
  } else if (warp == 1) {
    // -------------------------------- MMA issuer (leader only) --------------------------------
    if (rank == 0) {
      constexpr uint32_t IDESC = make_idesc_bf16(TM, Tile<TN>::MMA_N);
      long mma_seq = 0;
      int stage = 0;
      uint32_t phase = 0;
      int it = 0;
      bool ok = true;
      for (int t = cluster; t < tiles && ok; t += nclusters, ++it) {
        const int acc = it % Tile<TN>::NACC;
        const uint32_t acc_phase = (uint32_t)(it / Tile<TN>::NACC) & 1u;
        int w = 1;
        if (lane == 0) w = wait_bar(&bars->tempty[acc], acc_phase ^ 1u, p.err, ERR_MBAR_TIMEOUT_MMA, abort_flag, p.spin);
        if (!__shfl_sync(0xffffffffu, w, 0)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t d = tmem + (uint32_t)(acc * TN);
        for (int kb = 0; kb < p.k_blocks; ++kb) {
          if (lane == 0) w = wait_bar(&bars->full[stage], phase, p.err, ERR_MBAR_TIMEOUT_MMA, abort_flag, p.spin);
          if (!__shfl_sync(0xffffffffu, w, 0)) {
            ok = false;
            break;
          }
          if (p.trace && cluster == 0 && lane == 0 && mma_seq < 128) p.trace[256 + mma_seq] = globaltimer_ns();
          ++mma_seq;
          tc_fence_after();
          if (lane == 0) {
            const uint32_t a_addr = smem_u32(stages + (size_t)stage * STAGE_BYTES);
            const uint64_t ad = make_sdesc_sw128(a_addr);
#pragma unroll
            for (int k = 0; k < BK / 16; ++k)
#pragma unroll
              for (int h = 0; h < Tile<TN>::NSUB; ++h)
                umma_pair(d + (uint32_t)(h * Tile<TN>::MMA_N), ad + 2 * k,
                          make_sdesc_sw128(a_addr + A_BYTES + h * Tile<TN>::B_SUB_BYTES) + 2 * k, IDESC,
                          (kb > 0 || k > 0) ? 1u : 0u);
            // the stage is free once these MMAs are done (the producer relays it to the peer)
            umma_commit_pair(smem_u32(&bars->empty[stage]));
          }
          __syncwarp();
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
        if (!ok) break;
        if (lane == 0) umma_commit_pair(smem_u32(&bars->tfull[acc]));
        __syncwarp();
      }
      // every MMA issued above has completed before TMEM is released
      if (lane == 0) {
        umma_commit_pair(smem_u32(&bars->mma_done));
        const uint64_t t0 = globaltimer_ns();
        while (!mbar_try_wait(&bars->mma_done, 0) && globaltimer_ns() - t0 < 50000000ull) {
        }
      }
      __syncwarp();
    }
  } else {
    // -------------------------------- epilogue (warps 2..5, both CTAs) --------------------------------
    griddep_wait();  // `out` may still be read by the previous kernel
    const int quarter = warp & 3;
    const int row = quarter * 32 + lane;  // accumulator row = TMEM lane
    const uint32_t lane_off = (uint32_t)(quarter * 32) << 16;
    const uint32_t tempty = leader_addr(&bars->tempty[0]);
    const int et = threadIdx.x - 64;
    int it = 0;
    for (int t = cluster; t < tiles; t += nclusters, ++it) {
      const int acc = it % Tile<TN>::NACC;
      if (et == 0) {
        // the leader sees the MMA commit and passes the accumulator on to the peer's epilogue
        const bool w = wait_bar(&bars->tfull[acc], (uint32_t)(it / Tile<TN>::NACC) & 1u, p.err,
                                ERR_MBAR_TIMEOUT_EPILOGUE, abort_flag, p.spin);
        if (w && rank == 0) mbar_arrive_cluster(mapa_shared(smem_u32(&bars->tfull[acc]), 1));
        bars->epi_ok = w ? 1 : 0;
      }
      named_bar_sync(1, 128);
      const int ok = *reinterpret_cast<volatile int*>(&bars->epi_ok);
      named_bar_sync(1, 128);
      if (!ok) break;
      tc_fence_after();
      int tm, tn;
      tile_mn(t, p, tm, tn);
      const int m = tm * TM + (int)rank * 128 + row;
      const uint32_t taddr = tmem + lane_off + (uint32_t)(acc * TN);
      if constexpr (EPI == SILU_BF16) {
        // columns [128 b, 128 b + 64) gate and [128 b + 64, 128 b + 128) up of output block b
#pragma unroll 1
        for (int c = 0; c < TN / 2; c += 16) {
          const int b = c / 64, off = c % 64;
          uint32_t g[16], u[16];
          tmem_ld16(taddr + (uint32_t)(b * 128 + off), g);
          tmem_ld16(taddr + (uint32_t)(b * 128 + 64 + off), u);
          tmem_ld_wait_tied(g);
          tmem_ld_wait_tied(u);
          const int n = tn * (TN / 2) + c;
          if (m < p.M && n < p.N / 2) {
            uint32_t pk[8];
#pragma unroll
            for (int e = 0; e < 8; ++e)
              pk[e] = pack_bf16x2(silu_f(__uint_as_float(g[2 * e])) * __uint_as_float(u[2 * e]),
                                  silu_f(__uint_as_float(g[2 * e + 1])) * __uint_as_float(u[2 * e + 1]));
            uint4* dst = reinterpret_cast<uint4*>(p.out + (long)m * p.ldo + n);
            dst[0] = make_uint4(pk[0], pk[1], pk[2], pk[3]);
            dst[1] = make_uint4(pk[4], pk[5], pk[6], pk[7]);
          }
        }
      } else {
#pragma unroll 1
        for (int c = 0; c < TN; c += 32) {
          uint32_t v[32];
          tmem_ld16(taddr + (uint32_t)c, *reinterpret_cast<uint32_t(*)[16]>(&v[0]));
          tmem_ld16(taddr + (uint32_t)c + 16, *reinterpret_cast<uint32_t(*)[16]>(&v[16]));
          tmem_ld_wait_tied(v);
          const int n = tn * TN + c;
          if (m < p.M && n < p.N) {
            uint32_t pk[16];
#pragma unroll
            for (int e = 0; e < 16; ++e) pk[e] = pack_bf16x2(__uint_as_float(v[2 * e]), __uint_as_float(v[2 * e + 1]));
            uint4* dst = reinterpret_cast<uint4*>(p.out + (long)m * p.ldo + n);
#pragma unroll
            for (int q = 0; q < 4; ++q) dst[q] = make_uint4(pk[4 * q], pk[4 * q + 1], pk[4 * q + 2], pk[4 * q + 3]);
          }
        }
      }
      // this CTA is done with the accumulator: one arrival on the leader's barrier per CTA
      tc_fence_before();
      named_bar_sync(1, 128);
      if (et == 0) mbar_arrive_cluster(tempty + (uint32_t)(acc * sizeof(uint64_t)));
    }
  }
  tc_fence_before();
  __syncthreads();
  // no CTA leaves while its peer may still read its shared memory or arrive on its barriers
  cluster_sync();
  tc_fence_after();
  if (warp == 1) asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(TMEM_COLS) : "memory");
}

}  // namespace g2sm
}  // namespace mesh

namespace mesh {

// Shapes the pair kernel serves: bf16, K-contiguous operands, 16-byte aligned rows, N a multiple of 32
// (of 128 with the SiLU epilogue).
bool gemm_2sm_supported(int64_t M, int64_t N, int64_t K, int64_t epi) {
  if (epi != g2sm::STORE_BF16 && epi != g2sm::SILU_BF16) return false;
  if (K % 8 != 0 || N % (epi == g2sm::SILU_BF16 ? 128 : 32) != 0) return false;
  return M >= 1 && N >= 1 && K >= 1;
}

void gemm_2sm(const at::Tensor& A, const at::Tensor& B, at::Tensor& out, int64_t epi, at::Tensor& err,
              const c10::optional<at::Tensor>& trace, int64_t tn) {
  using namespace g2sm;
  TORCH_CHECK(A.scalar_type() == at::kBFloat16 && B.scalar_type() == at::kBFloat16 && out.scalar_type() == at::kBFloat16,
              "gemm_2sm: bf16 operands");
  TORCH_CHECK(A.dim() == 2 && B.dim() == 2 && A.stride(1) == 1 && B.stride(1) == 1 && A.size(1) == B.size(1),
              "gemm_2sm: A [M, K], B [N, K], K contiguous");
  const int M = A.size(0), N = B.size(0), K = A.size(1);
  TORCH_CHECK(gemm_2sm_supported(M, N, K, epi), "gemm_2sm: unsupported shape or epilogue");
  const int n_out = epi == SILU_BF16 ? N / 2 : N;
  TORCH_CHECK(out.dim() == 2 && out.size(0) == M && out.size(1) >= n_out && out.stride(1) == 1 && out.stride(0) % 8 == 0 &&
                  reinterpret_cast<uintptr_t>(out.data_ptr()) % 16 == 0,
              "gemm_2sm: out [M, N'] with 16-byte aligned rows");
  TORCH_CHECK((A.stride(0) * 2) % 16 == 0 && (B.stride(0) * 2) % 16 == 0, "gemm_2sm: 16-byte row pitch");
  const c10::cuda::CUDAGuard guard(A.device());
  Params p;
  p.out = reinterpret_cast<__nv_bfloat16*>(out.data_ptr());
  p.M = M;
  p.N = N;
  p.K = K;
  p.ldo = out.stride(0);
  p.m_tiles = (M + TM - 1) / TM;
  // tile width: 128-column tiles (argument or MESH_PAIR_TN=128) fill a short last wave better but
  // move half again as many operand bytes per FLOP and measured 37-46 % slower than 256.
  static const int force_tn = [] {
    const char* e = std::getenv("MESH_PAIR_TN");
    return e ? std::atoi(e) : 0;
  }();
  auto valid_tn = [&](int v) { return (v == 128 || v == 256 || v == 512) && !(v == 128 && epi == SILU_BF16); };
  // default: 512-column tiles wherever N fills them (measured 1.35-1.51 PFLOP/s on the Llama-3-8B
  // prefill shapes at T=4096 against 1.19-1.30 with 256 columns)
  int tn_sel = N >= 1024 ? 512 : 256;
  if (valid_tn((int)tn))
    tn_sel = (int)tn;
  else if (valid_tn(force_tn))
    tn_sel = force_tn;
  p.n_tiles = (N + tn_sel - 1) / tn_sel;
  p.k_blocks = (K + BK - 1) / BK;
  p.err = err.data_ptr<int>();
  static const int spin = [] {
    const char* e = std::getenv("MESH_WAIT_SPIN");
    return (e && e[0] == '0') ? 0 : 1;
  }();
  p.spin = spin;
  p.trace = nullptr;
  if (trace.has_value() && trace->defined()) {
    TORCH_CHECK(trace->is_cuda() && trace->scalar_type() == at::kLong && trace->numel() >= 384, "gemm_2sm: trace");
    p.trace = reinterpret_cast<unsigned long long*>(trace->data_ptr<int64_t>());
  }
  int sms = 0;
  C10_CUDA_CHECK(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, A.get_device()));
  const int pairs = std::max(1, sms / 2);
  const int clusters = std::max(1, std::min(p.m_tiles * p.n_tiles, pairs));
  // stages: about 192 KB of operands (6 x 32 KB at TN=256, 8 x 24 KB at TN=128) unless overridden
  static const int stages_env = [] {
    const char* e = std::getenv("MESH_PAIR_STAGES");
    return e ? std::atoi(e) : 0;
  }();
  const int max_st = tn_sel == 512 ? 4 : MAX_STAGES;  // 48 KB stages at 512 columns
  const int def_st = tn_sel == 512 ? 4 : (tn_sel == 256 ? 6 : 8);
  const int stages = std::max(2, std::min(stages_env ? stages_env : def_st, max_st));
  p.stages = stages;
  CUtensorMap ta = tma_map_2d_bf16(A.data_ptr(), K, M, A.stride(0), BK, 128);
  CUtensorMap tb = tma_map_2d_bf16(B.data_ptr(), K, N, B.stride(0), BK, tn_sel == 512 ? 128 : tn_sel / 2);
  cudaStream_t st = at::cuda::getCurrentCUDAStream();
  auto go = [&](auto kern, size_t smem) {
    TORCH_CHECK(smem <= 232448, "gemm_2sm: too many stages for shared memory");
    C10_CUDA_CHECK(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
    C10_CUDA_CHECK(launch_kc(kern, dim3(2 * clusters), dim3(NUM_THREADS), smem, st, 2, ta, tb, p));
  };
  if (epi == SILU_BF16 && tn_sel == 512)
    go(gemm_2sm_kernel<SILU_BF16, 512>, smem_bytes<512>(stages));
  else if (epi == SILU_BF16)
    go(gemm_2sm_kernel<SILU_BF16, 256>, smem_bytes<256>(stages));
  else if (tn_sel == 512)
    go(gemm_2sm_kernel<STORE_BF16, 512>, smem_bytes<512>(stages));
  else if (tn_sel == 128)
    go(gemm_2sm_kernel<STORE_BF16, 128>, smem_bytes<128>(stages));
  else
    go(gemm_2sm_kernel<STORE_BF16, 256>, smem_bytes<256>(stages));
}

}  // namespace mesh
