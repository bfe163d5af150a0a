// Paged, causal, varlen GQA prefill attention on the 5th-generation tensor cores (sm_100a).
//
// Persistent: one CTA per SM walks the work items, each a pair of 128-row query tiles (t = 0, 1) of
// one sequence and KV head, heaviest (latest) tile pairs first. A row is (token, query head of the KV
// group), so a tile is 128 / G tokens x the G query heads of one KV head and every K/V block fetched
// from the page pool serves the whole GQA group and both tiles. The K/V ring, the barrier phases and
// TMEM carry over from item to item: the next item's query tiles load as soon as the last QK of the
// current one is done, and its first QK runs while the current item's output is read out of TMEM.
// Roles (320 threads):
//   warp 0      TMA producer: the two query tiles (3D boxes, one per 64-dim half) and, per 128-key
//               block, the 8 pages of K and of V (16x64 boxes, 128-byte swizzle) into a 2-stage ring;
//   warp 1      tcgen05.mma issuer (one thread): S_t = Q_t K_j^T into the TMEM score buffer of
//               tile t, then O_t += P_t V_j with P read from TMEM (the bf16 probabilities overwrite
//               the first 64 columns of S_t) and V read MN-major straight from the page layout;
//   warps 2..5  softmax of tile 0, warps 6..9 softmax of tile 1: a thread owns one row (one TMEM
//               lane): it reads the row's 128 scores with tcgen05.ld, applies the causal / window /
//               length mask, keeps the running maximum and sum, writes P back with tcgen05.st,
//               and at the end normalises O and stores it.
// The tiles ping-pong: while the softmax of one tile runs, the tensor core multiplies for the
// other. The running maximum only moves (and O is rescaled in TMEM) when it grows by more than
// 2^8; numerator and denominator use the same maximum, so the result is exact and most blocks
// skip the rescale.
//
// TMEM columns (512): S0 [0,128) S1 [128,256) O0 [256,384) O1 [384,512).
//
// Query i of a sequence with q_len new tokens and k_len keys sits at key position k_len - q_len + i,
// so chunked prefill over a cached prefix works unchanged. Every wait is bounded (%globaltimer);
// on a timeout the kernel records an error code, drains its copies and MMAs, frees TMEM and exits.
//
// Replaces the reference's explicit [heads, T, S] score tensor, host-built causal mask and softmax
// (agent/src/inference/forward_pass.rs:1096-1125, :2811-2835).
#include <ATen/ATen.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/extension.h>

#include <cstdlib>

#include "../include/launch.h"
#include "../include/sm100.cuh"
#include "../include/tma_host.h"

namespace mesh {
namespace pftc {

constexpr int BM = 128;                       // query rows per tile
constexpr int NT = 2;                         // query tiles per CTA
constexpr int BK = 128;                       // keys per block
constexpr int D = 128;                        // head dim
constexpr int PAGE = 16;                      // KV page tokens
constexpr int PAGES_PER_BLOCK = BK / PAGE;    // 8
constexpr int STAGES = 2;
constexpr uint32_t ATOM_BYTES = 128 * 128;    // 128 rows x 128 B: one 64-element slice of a tile
constexpr uint32_t TILE_BYTES = 2 * ATOM_BYTES;
constexpr uint32_t BOX_BYTES = PAGE * 128;    // one 16 x 64 page box
constexpr int NUM_THREADS = 64 + NT * 128;
constexpr uint32_t TMEM_COLS = 512;
constexpr uint32_t O_COL = NT * BK;           // O_t at O_COL + t * D
constexpr uint64_t WAIT_LIMIT_NS = 2000000000ull;
constexpr float RESCALE_THRESHOLD = 8.0f;     // log2 units

struct Args {
  const int* cu_q;          // [S+1]
  const int* k_lens;        // [S]
  const int* block_tables;  // [S, max_pages]
  __nv_bfloat16* out;       // [T, hq*D]
  int max_pages, hkv, hq, n_ctas, nseq;
  float scale_log2;
  int window;
  int spin;     // 1: waits poll the barrier; 0: waits sleep inside try_wait between polls
  int pv_wait;  // 1: QK_t(j+1) waits for PV_t(j) to complete (P shares S's TMEM columns)
  int* err;
};

struct Bars {
  uint64_t q_full, q_empty;
  uint64_t k_full[STAGES], v_full[STAGES], kv_empty[STAGES];
  uint64_t s_full[NT], p_full[NT], o_done[NT], o_free[NT];
  uint64_t mma_done;
  uint32_t tmem_base;
  int abort;
};

constexpr size_t smem_bytes() { return 1024 + NT * TILE_BYTES + 2 * STAGES * TILE_BYTES + sizeof(Bars); }

__device__ __forceinline__ bool wait_warp(uint64_t* bar, uint32_t parity, int* err, int code, volatile int* abort_flag,
                                          int spin) {
  int ok = 1;
  if (lane_id() == 0)
    ok = spin ? mbar_wait_bounded(bar, parity, err, code, abort_flag, WAIT_LIMIT_NS)
              : mbar_wait_bounded_sleep(bar, parity, err, code, abort_flag, WAIT_LIMIT_NS);
  return __shfl_sync(0xffffffffu, ok, 0) != 0;
}

__device__ __forceinline__ bool wait_one(uint64_t* bar, uint32_t parity, int* err, int code, volatile int* abort_flag,
                                         int spin) {
  return spin ? mbar_wait_bounded(bar, parity, err, code, abort_flag, WAIT_LIMIT_NS)
              : mbar_wait_bounded_sleep(bar, parity, err, code, abort_flag, WAIT_LIMIT_NS);
}

// Per-CTA geometry shared by every role.
template <int G>
struct Geo {
  static constexpr int BQT = BM / G;  // tokens per tile
  int q0, qlen, tok0, klen, pos_base, kb_first;
  int nblk[NT];  // key blocks each tile takes part in (0: tile has no valid row)
  __device__ __forceinline__ bool init(const Args& a, int seq, int cta) {
    q0 = a.cu_q[seq];
    qlen = a.cu_q[seq + 1] - q0;
    tok0 = cta * NT * BQT;
    if (tok0 >= qlen) return false;
    klen = a.k_lens[seq];
    pos_base = klen - qlen;
    const int kmin = a.window > 0 ? max(0, pos_base + tok0 - a.window + 1) : 0;
    kb_first = kmin / BK;
#pragma unroll
    for (int t = 0; t < NT; ++t) {
      const int first = tok0 + t * BQT;
      if (first >= qlen) {
        nblk[t] = 0;
        continue;
      }
      const int last = min(first + BQT, qlen) - 1;
      const int kmax = min(klen, pos_base + last + 1);
      nblk[t] = (kmax - 1) / BK - kb_first + 1;
    }
    return true;
  }
  __device__ __forceinline__ int nblk_all() const { return max(nblk[0], nblk[1]); }
};

template <int G>
__global__ void __launch_bounds__(NUM_THREADS, 1)
    attn_prefill_tc_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                           const __grid_constant__ CUtensorMap tmV, const Args a) {
  constexpr int BQT = Geo<G>::BQT;
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw = smem_u32(smem_raw);
  uint8_t* q_sm = smem_raw + (((raw + 1023u) & ~1023u) - raw);
  uint8_t* k_sm = q_sm + NT * TILE_BYTES;
  uint8_t* v_sm = k_sm + STAGES * TILE_BYTES;
  Bars* bars = reinterpret_cast<Bars*>(v_sm + STAGES * TILE_BYTES);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  // Work item w -> (query tile pair counted from the end, KV head, sequence): every head and
  // sequence of the latest (longest) tile pair first, so the heaviest items start first.
  const int per = a.hkv * a.nseq;
  const int W = a.n_ctas * per;
  auto item = [&](int w, Geo<G>& g, int& h, int& seq) -> bool {
    const int x = w / per, r = w - x * per;
    h = r % a.hkv;
    seq = r / a.hkv;
    return g.init(a, seq, a.n_ctas - 1 - x);
  };

  if (threadIdx.x == 0) {
    mbar_init(&bars->q_full, 1);
    mbar_init(&bars->q_empty, 1);
    for (int i = 0; i < STAGES; ++i) {
      mbar_init(&bars->k_full[i], 1);
      mbar_init(&bars->v_full[i], 1);
      mbar_init(&bars->kv_empty[i], 1);
    }
    for (int t = 0; t < NT; ++t) {
      mbar_init(&bars->s_full[t], 1);
      mbar_init(&bars->p_full[t], 128);
      mbar_init(&bars->o_done[t], 1);
      mbar_init(&bars->o_free[t], 128);
    }
    mbar_init(&bars->mma_done, 1);
    bars->abort = 0;
    fence_mbar_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tmQ);
    tma_prefetch_desc(&tmK);
    tma_prefetch_desc(&tmV);
  }
  if (warp == 1) {
    tmem_alloc(&bars->tmem_base, TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = bars->tmem_base;
  volatile int* abort_flag = &bars->abort;
  // dependents may launch once every CTA of this grid holds its TMEM
  griddep_launch_dependents();

  if (warp == 0) {
    // ------------------------------------ TMA producer ------------------------------------
    if (lane == 0) {
      const uint64_t pol = policy_evict_last();  // K/V pages are re-read by the other query tiles
      griddep_wait();  // Q and the K/V pages come from the previous kernel
      uint32_t kvc = 0;  // key blocks loaded so far (ring position)
      int ic = 0;        // items started
      bool ok = true;
      for (int w = blockIdx.x; w < W && ok; w += gridDim.x) {
        Geo<G> g;
        int h, seq;
        if (!item(w, g, h, seq)) continue;
        // the query buffers are free once every QK of the previous item is done
        if (ic > 0 && !wait_one(&bars->q_empty, (uint32_t)(ic - 1) & 1u, a.err, ERR_MBAR_TIMEOUT_PRODUCER, abort_flag, a.spin)) {
          ok = false;
          break;
        }
        const int ntiles = g.nblk[1] > 0 ? 2 : 1;
        mbar_arrive_expect_tx(&bars->q_full, ntiles * TILE_BYTES);
        for (int t = 0; t < ntiles; ++t) {
          uint8_t* qd = q_sm + t * TILE_BYTES;
          const int tok = g.q0 + g.tok0 + t * BQT;
          tma_load_3d(qd, &tmQ, &bars->q_full, 0, h * G, tok, pol);
          tma_load_3d(qd + ATOM_BYTES, &tmQ, &bars->q_full, 64, h * G, tok, pol);
        }
        ++ic;
        const int* bt = a.block_tables + (long)seq * a.max_pages;
        const int npages = (g.klen + PAGE - 1) / PAGE;
        const int nblk = g.nblk_all();
        for (int j = 0; j < nblk; ++j, ++kvc) {
          const int s = kvc % STAGES;
          const uint32_t ph = (kvc / STAGES) & 1u;
          if (!wait_one(&bars->kv_empty[s], ph ^ 1u, a.err, ERR_MBAR_TIMEOUT_PRODUCER, abort_flag, a.spin)) {
            ok = false;
            break;
          }
          const int kb = g.kb_first + j;
          int rows[PAGES_PER_BLOCK];
#pragma unroll
          for (int p = 0; p < PAGES_PER_BLOCK; ++p) {
            // pages past the sequence end repeat its last page: finite data under masked scores
            const int pg = min(kb * PAGES_PER_BLOCK + p, npages - 1);
            rows[p] = (bt[pg] * a.hkv + h) * PAGE;
          }
          uint8_t* kd = k_sm + s * TILE_BYTES;
          uint8_t* vd = v_sm + s * TILE_BYTES;
          mbar_arrive_expect_tx(&bars->k_full[s], TILE_BYTES);
#pragma unroll
          for (int p = 0; p < PAGES_PER_BLOCK; ++p) {
            tma_load_2d(kd + p * BOX_BYTES, &tmK, &bars->k_full[s], 0, rows[p], pol);
            tma_load_2d(kd + ATOM_BYTES + p * BOX_BYTES, &tmK, &bars->k_full[s], 64, rows[p], pol);
          }
          mbar_arrive_expect_tx(&bars->v_full[s], TILE_BYTES);
#pragma unroll
          for (int p = 0; p < PAGES_PER_BLOCK; ++p) {
            tma_load_2d(vd + p * BOX_BYTES, &tmV, &bars->v_full[s], 0, rows[p], pol);
            tma_load_2d(vd + ATOM_BYTES + p * BOX_BYTES, &tmV, &bars->v_full[s], 64, rows[p], pol);
          }
        }
      }
      if (!ok) {
        // let copies already in flight land before the CTA exits (bounded)
        const uint64_t t0 = globaltimer_ns();
        for (uint32_t k = kvc > STAGES ? kvc - STAGES : 0; k < kvc; ++k) {
          const int s = k % STAGES;
          const uint32_t ph = (k / STAGES) & 1u;
          while (!(mbar_try_wait(&bars->k_full[s], ph) && mbar_try_wait(&bars->v_full[s], ph)) &&
                 globaltimer_ns() - t0 < 50000000ull) {
          }
        }
        if (ic > 0)
          while (!mbar_try_wait(&bars->q_full, (uint32_t)(ic - 1) & 1u) && globaltimer_ns() - t0 < 50000000ull) {
          }
      }
    }
    __syncwarp();
  } else if (warp == 1) {
    // ------------------------------------ MMA issuer ------------------------------------
    constexpr uint32_t IDESC_QK = make_idesc_bf16(BM, BK);
    constexpr uint32_t IDESC_PV = make_idesc_bf16(BM, D) | IDESC_B_MN_MAJOR;
    const uint32_t q_addr = smem_u32(q_sm), k_addr = smem_u32(k_sm), v_addr = smem_u32(v_sm);
    auto wait = [&](uint64_t* bar, uint32_t parity) {
      return wait_warp(bar, parity, a.err, ERR_MBAR_TIMEOUT_MMA, abort_flag, a.spin);
    };
    int qk_left = 0;  // QKs of the current item still to issue (the last one frees the query buffers)
    auto issue_qk = [&](int t, int s) {
      if (lane == 0) {
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk) {
          const uint64_t ad = make_sdesc_sw128(q_addr + t * TILE_BYTES + (kk >> 2) * ATOM_BYTES) + 2 * (kk & 3);
          const uint64_t bd = make_sdesc_sw128(k_addr + s * TILE_BYTES + (kk >> 2) * ATOM_BYTES) + 2 * (kk & 3);
          umma_bf16(tmem + (uint32_t)(t * BK), ad, bd, IDESC_QK, kk > 0 ? 1u : 0u);
        }
        umma_commit(&bars->s_full[t]);
        if (--qk_left == 0) umma_commit(&bars->q_empty);
      }
      __syncwarp();
    };
    auto issue_pv = [&](int t, int s, bool first) {
      if (lane == 0) {
#pragma unroll
        for (int kk = 0; kk < BK / 16; ++kk) {
          // A = P_t: 16 keys = 8 packed columns of the score buffer; B = V: 16 keys = 2048 bytes
          // of the page layout, the two 64-dim halves ATOM_BYTES apart
          const uint64_t bd = make_sdesc_sw128_mn(v_addr + s * TILE_BYTES + kk * 2048, ATOM_BYTES, 1024);
          umma_bf16_ts(tmem + O_COL + (uint32_t)(t * D), tmem + (uint32_t)(t * BK + kk * 8), bd, IDESC_PV,
                       (!first || kk > 0) ? 1u : 0u);
        }
        umma_commit(&bars->o_done[t]);
      }
      __syncwarp();
    };
    uint32_t kvc = 0;
    int ic = 0;
    int tcnt[NT] = {0, 0};  // blocks each tile has gone through (phase of s_full / p_full / o_done)
    int tuse[NT] = {0, 0};  // items each tile has finished (phase of o_free)
    bool ok = true;
    for (int w = blockIdx.x; w < W && ok; w += gridDim.x) {
      Geo<G> g;
      int h, seq;
      if (!item(w, g, h, seq)) continue;
      const int nblk = g.nblk_all();
      qk_left = g.nblk[0] + g.nblk[1];
      if (!wait(&bars->q_full, (uint32_t)ic & 1u) ||
          !wait(&bars->k_full[kvc % STAGES], (kvc / STAGES) & 1u)) {
        ok = false;
        break;
      }
      ++ic;
      tc_fence_after();
      for (int t = 0; t < NT && ok; ++t) {
        if (g.nblk[t] == 0) continue;
        // S_t / P_t of the previous item are free once its last PV_t is done
        if (a.pv_wait && tcnt[t] > 0 && !wait(&bars->o_done[t], (uint32_t)(tcnt[t] - 1) & 1u)) {
          ok = false;
          break;
        }
        tc_fence_after();
        issue_qk(t, kvc % STAGES);
      }
      for (int j = 0; j < nblk && ok; ++j) {
        const uint32_t k = kvc + j;
        const int s = k % STAGES;
        if (!wait(&bars->v_full[s], (k / STAGES) & 1u)) {
          ok = false;
          break;
        }
        if (j + 1 < nblk && !wait(&bars->k_full[(k + 1) % STAGES], ((k + 1) / STAGES) & 1u)) {
          ok = false;
          break;
        }
        for (int t = 0; t < NT && ok; ++t) {
          if (j >= g.nblk[t]) continue;
          // softmax of tile t wrote P_t(j) into TMEM and rescaled O_t
          if (!wait(&bars->p_full[t], (uint32_t)tcnt[t] & 1u)) {
            ok = false;
            break;
          }
          // O_t was read out by the previous item's epilogue
          if (j == 0 && tuse[t] > 0 && !wait(&bars->o_free[t], (uint32_t)(tuse[t] - 1) & 1u)) {
            ok = false;
            break;
          }
          tc_fence_after();
          issue_pv(t, s, j == 0);
          ++tcnt[t];
          if (j + 1 < g.nblk[t]) {
            // S_t(j+1) overwrites the columns P_t(j) is read from. With pv_wait the thread waits until
            // PV_t(j) is done; otherwise it relies on the tensor core executing one thread's MMAs in
            // issue order (PV_t(j) reads its operands before QK_t(j+1), issued after it, writes)
            if (a.pv_wait && !wait(&bars->o_done[t], (uint32_t)(tcnt[t] - 1) & 1u)) {
              ok = false;
              break;
            }
            tc_fence_after();
            issue_qk(t, (k + 1) % STAGES);
          }
        }
        if (ok && lane == 0) umma_commit(&bars->kv_empty[s]);
        __syncwarp();
      }
      kvc += nblk;
      for (int t = 0; t < NT; ++t)
        if (g.nblk[t] > 0) ++tuse[t];
    }
    // every MMA issued above has completed before TMEM is released
    if (lane == 0) {
      umma_commit(&bars->mma_done);
      const uint64_t t0 = globaltimer_ns();
      while (!mbar_try_wait(&bars->mma_done, 0) && globaltimer_ns() - t0 < 50000000ull) {
      }
    }
    __syncwarp();
  } else {
    // ------------------------------------ softmax (warps 2..9) ------------------------------------
    const int t = (warp - 2) >> 2;  // query tile of this warp
    const int quarter = warp & 3;   // TMEM lane quarter this warp may access
    const int row = quarter * 32 + lane;
    const uint32_t lane_off = (uint32_t)(quarter * 32) << 16;
    const uint32_t s_addr = tmem + lane_off + (uint32_t)(t * BK);
    const uint32_t o_addr = tmem + lane_off + O_COL + (uint32_t)(t * D);
    int tcnt = 0;
    bool ok = true;
    for (int w = blockIdx.x; w < W && ok; w += gridDim.x) {
      Geo<G> g;
      int h, seq;
      if (!item(w, g, h, seq)) continue;
      const int nb = g.nblk[t];
      if (nb == 0) continue;
      const int ttok0 = g.tok0 + t * BQT;            // first token of this tile
      const int tq = ttok0 + row / G;
      const int qpos = g.pos_base + tq;
      const int lim = min(qpos, g.klen - 1);                       // last key this row may attend
      const int low = a.window > 0 ? qpos - a.window + 1 : 0;      // first key this row may attend
      const int tlast = min(ttok0 + BQT, g.qlen) - 1;
      const int lim_min = min(g.pos_base + ttok0, g.klen - 1);     // smallest `lim` of the tile
      const int low_max = a.window > 0 ? g.pos_base + tlast - a.window + 1 : 0;
      float m_used = -INFINITY, l = 0.f;
      for (int j = 0; j < nb; ++j, ++tcnt) {
        if (!wait_warp(&bars->s_full[t], (uint32_t)tcnt & 1u, a.err, ERR_MBAR_TIMEOUT_EPILOGUE, abort_flag, a.spin)) {
          ok = false;
          break;
        }
        tc_fence_after();
        uint32_t sv[BK];
#pragma unroll
        for (int c = 0; c < BK / 16; ++c)
          tmem_ld16(s_addr + (uint32_t)(16 * c), *reinterpret_cast<uint32_t(*)[16]>(&sv[16 * c]));
        tmem_ld_wait_tied(sv);

        const int key0 = (g.kb_first + j) * BK;
        if (key0 + BK - 1 > lim_min || key0 < low_max) {
#pragma unroll
          for (int c = 0; c < BK; ++c)
            if (key0 + c > lim || key0 + c < low) sv[c] = __float_as_uint(-INFINITY);
        }
        // row maximum (raw scores; the scale is folded into the exponent below)
        float mx[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) mx[i] = __uint_as_float(sv[i]);
#pragma unroll
        for (int c = 8; c < BK; ++c) mx[c & 7] = fmaxf(mx[c & 7], __uint_as_float(sv[c]));
        const float mraw = fmaxf(fmaxf(fmaxf(mx[0], mx[1]), fmaxf(mx[2], mx[3])),
                                 fmaxf(fmaxf(mx[4], mx[5]), fmaxf(mx[6], mx[7])));
        const float m_new = fmaxf(m_used, mraw * a.scale_log2);
        const bool resc = m_new > m_used + RESCALE_THRESHOLD;
        float alpha = 1.f;
        if (resc) {
          alpha = ex2_ftz(m_used - m_new);  // 0 when m_used is -inf
          m_used = m_new;
        }
        const bool dead = m_used == -INFINITY;  // nothing attended yet (window / padding rows)
        const float mb = dead ? 0.f : m_used;
        float sum[4] = {0.f, 0.f, 0.f, 0.f};
        // P_t(j) overwrites the first 64 columns of the score buffer, 16 packed columns at a time
#pragma unroll
        for (int c = 0; c < BK / 32; ++c) {
          uint32_t pk[16];
#pragma unroll
          for (int e = 0; e < 16; ++e) {
            const float p0 = ex2_ftz(fmaf(__uint_as_float(sv[32 * c + 2 * e]), a.scale_log2, -mb));
            const float p1 = ex2_ftz(fmaf(__uint_as_float(sv[32 * c + 2 * e + 1]), a.scale_log2, -mb));
            sum[e & 3] += p0 + p1;
            pk[e] = pack_bf16x2(p0, p1);
          }
          tmem_st16(s_addr + (uint32_t)(16 * c), pk);
        }
        l = l * alpha + ((sum[0] + sum[1]) + (sum[2] + sum[3]));
        // PV_t(j-1) finished before QK_t(j) was issued, so O_t is stable here
        if (j > 0 && __any_sync(0xffffffffu, resc)) {
#pragma unroll 1
          for (int c = 0; c < D / 16; ++c) {
            uint32_t ov[16];
            tmem_ld16(o_addr + 16 * c, ov);
            tmem_ld_wait_tied(ov);
#pragma unroll
            for (int e = 0; e < 16; ++e) ov[e] = __float_as_uint(__uint_as_float(ov[e]) * alpha);
            tmem_st16(o_addr + 16 * c, ov);
          }
        }
        tmem_st_wait();
        tc_fence_before();
        mbar_arrive(&bars->p_full[t]);
      }
      if (!ok || !wait_warp(&bars->o_done[t], (uint32_t)(tcnt - 1) & 1u, a.err, ERR_MBAR_TIMEOUT_EPILOGUE,
                            abort_flag, a.spin)) {
        ok = false;
        break;
      }
      tc_fence_after();
      const float inv = l > 0.f ? 1.f / l : 0.f;
      const bool valid = tq < g.qlen;
      __nv_bfloat16* dst = a.out + (long)(g.q0 + (valid ? tq : 0)) * a.hq * D + (long)(h * G + row % G) * D;
#pragma unroll 1
      for (int c = 0; c < D / 16; ++c) {
        uint32_t ov[16];
        tmem_ld16(o_addr + 16 * c, ov);
        tmem_ld_wait_tied(ov);
        uint4 w0, w1;
        w0.x = pack_bf16x2(__uint_as_float(ov[0]) * inv, __uint_as_float(ov[1]) * inv);
        w0.y = pack_bf16x2(__uint_as_float(ov[2]) * inv, __uint_as_float(ov[3]) * inv);
        w0.z = pack_bf16x2(__uint_as_float(ov[4]) * inv, __uint_as_float(ov[5]) * inv);
        w0.w = pack_bf16x2(__uint_as_float(ov[6]) * inv, __uint_as_float(ov[7]) * inv);
        w1.x = pack_bf16x2(__uint_as_float(ov[8]) * inv, __uint_as_float(ov[9]) * inv);
        w1.y = pack_bf16x2(__uint_as_float(ov[10]) * inv, __uint_as_float(ov[11]) * inv);
        w1.z = pack_bf16x2(__uint_as_float(ov[12]) * inv, __uint_as_float(ov[13]) * inv);
        w1.w = pack_bf16x2(__uint_as_float(ov[14]) * inv, __uint_as_float(ov[15]) * inv);
        if (valid) {
          reinterpret_cast<uint4*>(dst + 16 * c)[0] = w0;
          reinterpret_cast<uint4*>(dst + 16 * c)[1] = w1;
        }
      }
      // O_t may take the next item's first PV
      tc_fence_before();
      mbar_arrive(&bars->o_free[t]);
    }
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1) tmem_dealloc(tmem, TMEM_COLS);
}

}  // namespace pftc

// True when the tcgen05 kernel serves this shape (head_dim 128, 16-token pages, GQA group 1/2/4/8).
bool attn_prefill_tc_supported(int64_t head_dim, int64_t page_size, int64_t group) {
  return head_dim == pftc::D && page_size == pftc::PAGE &&
         (group == 1 || group == 2 || group == 4 || group == 8);
}

void attn_prefill_tc(const at::Tensor& q, const at::Tensor& kcache, const at::Tensor& vcache, const at::Tensor& cu_q,
                     const at::Tensor& k_lens, const at::Tensor& block_tables, at::Tensor& out, int64_t max_q_len,
                     double scale, int64_t window, at::Tensor& err) {
  using namespace pftc;
  TORCH_CHECK(q.scalar_type() == at::kBFloat16 && q.is_contiguous() && q.dim() == 2, "attn_prefill_tc: q bf16 [T, hq*D]");
  TORCH_CHECK(out.scalar_type() == at::kBFloat16 && out.is_contiguous() && out.sizes() == q.sizes(),
              "attn_prefill_tc: out like q");
  TORCH_CHECK(kcache.dim() == 4 && kcache.is_contiguous() && vcache.is_contiguous() && kcache.sizes() == vcache.sizes() &&
                  kcache.scalar_type() == at::kBFloat16 && vcache.scalar_type() == at::kBFloat16,
              "attn_prefill_tc: k/v cache bf16 [pages, hkv, page, D]");
  TORCH_CHECK(cu_q.scalar_type() == at::kInt && k_lens.scalar_type() == at::kInt &&
                  block_tables.scalar_type() == at::kInt && block_tables.is_contiguous(),
              "attn_prefill_tc: int32 metadata");
  const int hkv = kcache.size(1);
  const int hq = q.size(1) / D;
  TORCH_CHECK(q.size(1) == (int64_t)hq * D && hq % hkv == 0, "attn_prefill_tc: q heads");
  const int G = hq / hkv;
  TORCH_CHECK(attn_prefill_tc_supported(kcache.size(3), kcache.size(2), G),
              "attn_prefill_tc: head_dim 128, 16-token pages, group 1/2/4/8");
  const int S = k_lens.size(0);
  const int64_t T = q.size(0);
  if (S == 0 || max_q_len == 0 || T == 0) return;
  const c10::cuda::CUDAGuard guard(q.device());
  const int64_t rows = kcache.size(0) * hkv * PAGE;
  TORCH_CHECK(rows < (1ll << 31), "attn_prefill_tc: KV pool too large for 32-bit TMA rows");
  const int BQT = BM / G;
  CUtensorMap tq = tma_map_3d_bf16(q.data_ptr(), D, hq, T, (uint64_t)D * 2, (uint64_t)hq * D * 2, 64, G, BQT);
  CUtensorMap tk = tma_map_2d_bf16(kcache.data_ptr(), D, rows, D, 64, PAGE);
  CUtensorMap tv = tma_map_2d_bf16(vcache.data_ptr(), D, rows, D, 64, PAGE);
  Args a;
  a.cu_q = cu_q.data_ptr<int>();
  a.k_lens = k_lens.data_ptr<int>();
  a.block_tables = block_tables.data_ptr<int>();
  a.out = reinterpret_cast<__nv_bfloat16*>(out.data_ptr());
  a.max_pages = block_tables.size(1);
  a.hkv = hkv;
  a.hq = hq;
  a.n_ctas = (int)((max_q_len + NT * BQT - 1) / (NT * BQT));
  a.nseq = S;
  a.scale_log2 = (float)(scale * 1.4426950408889634);
  a.window = (int)window;
  a.err = err.data_ptr<int>();
  static const int spin = [] {
    const char* e = std::getenv("MESH_WAIT_SPIN");
    return (e && e[0] == '0') ? 0 : 1;
  }();
  a.spin = spin;
  static const int pv_wait = [] {
    const char* e = std::getenv("MESH_ATTN_PV_WAIT");
    return (e && e[0] == '1') ? 1 : 0;
  }();
  a.pv_wait = pv_wait;
  // persistent: one CTA per SM walks the work items (tile pair, KV head, sequence)
  int sms = 0;
  C10_CUDA_CHECK(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, q.get_device()));
  const long items = (long)a.n_ctas * hkv * S;
  TORCH_CHECK(items < (1l << 31), "attn_prefill_tc: too many work items");
  dim3 grid((unsigned)std::min<long>(items, sms));
  const size_t smem = smem_bytes();
  cudaStream_t st = at::cuda::getCurrentCUDAStream();
  auto go = [&](auto kern) {
    C10_CUDA_CHECK(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
    C10_CUDA_CHECK(launch_k(kern, grid, dim3(NUM_THREADS), smem, st, tq, tk, tv, a));
  };
  switch (G) {
    case 1: go(attn_prefill_tc_kernel<1>); break;
    case 2: go(attn_prefill_tc_kernel<2>); break;
    case 4: go(attn_prefill_tc_kernel<4>); break;
    default: go(attn_prefill_tc_kernel<8>); break;
  }
}

}  // namespace mesh
