// On-device temperature / top-p sampling over vocabulary-parallel logits (sm_100a).
//
// Semantics of the reference's device sampler (agent/src/inference/runtime.rs:534-601,
// tensor_ops.rs:394-458): y = logits / T, p = softmax(y); with top_p >= 1 the token is the first
// index (vocabulary order) whose running CDF reaches the row's threshold r in [0, 1); with top_p < 1
// the tokens are ordered by descending p (ties by index), the kept prefix is every token whose mass
// before it is below top_p, and the token is the first of the kept prefix whose renormalised running
// CDF reaches r. Greedy rows (T <= 0 or top_p <= 0) take the argmax.
//
// Each rank holds a contiguous slice of the vocabulary. Probability masses e^(y - M) (M = the global
// row maximum) are accumulated in unsigned 64-bit fixed point (2^-40 units): integer sums do not
// depend on the order of accumulation, so every result is bitwise reproducible run to run and the
// same at every TP degree, and the cross-rank sums are exact integer all-reduces. The descending
// order is never materialised: the crossing element of a mass target is found by a radix select
// over the order-preserving 32-bit keys of y, one 8-bit digit per pass, each pass a 256-bin mass
// histogram summed over the ranks. Two selections (the top-p cut, then the sample) cost 8 passes.
//
// Kernels (one CTA per row, 512 threads):
//   samp_max      local row maximum of y                    -> (all-reduce MAX over ranks)
//   samp_mass     local fixed-point mass of the row          -> (all-gather over ranks)
//   samp_hist     256-bin mass histogram of one key digit among keys matching the digits chosen
//                 so far                                      -> (all-reduce SUM over ranks)
//   samp_select   per row: pick the digit whose descending cumulative mass reaches the target
//   samp_find     per row: this rank's lowest index holding the selected key (top-p), or the first
//                 index where the vocabulary-order CDF reaches the target (top-p >= 1)
//                                                             -> (all-reduce MIN over ranks)
#include <ATen/ATen.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/extension.h>

#include <climits>

#include "../include/sm100.cuh"

namespace mesh {
namespace samp {

constexpr int NT = 512;
constexpr double FIX = 1099511627776.0;  // 2^40

// order-preserving map of a float to uint32 (larger float -> larger key)
__device__ __forceinline__ uint32_t fkey(float y) {
  const uint32_t u = __float_as_uint(y);
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}
__device__ __forceinline__ unsigned long long fix_mass(float y, float m) {
  // e^(y - m) in [0, 1] -> round-down 2^-40 fixed point; exp of the difference in fp32
  const float e = __expf(y - m);
  return (unsigned long long)((double)e * FIX);
}

// Row parameters: inv_t = 1/T (0 for greedy rows), top_p, threshold r.
struct Rows {
  const float* logits;  // [B, V_loc]
  int B, V, ld;         // V = local vocabulary size, ld = row stride
  const float* inv_t;   // [B]
};

__device__ __forceinline__ float row_y(const Rows& r, int b, int i) { return r.logits[(long)b * r.ld + i] * r.inv_t[b]; }

__global__ void __launch_bounds__(NT) samp_max_kernel(const Rows r, float* mx) {
  __shared__ float red[NT / 32];
  const int b = blockIdx.x;
  float m = -INFINITY;
  if (r.inv_t[b] > 0.f)
    for (int i = threadIdx.x; i < r.V; i += NT) m = fmaxf(m, row_y(r, b, i));
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = m;
  __syncthreads();
  if (threadIdx.x == 0) {
    float t = red[0];
    for (int w = 1; w < NT / 32; ++w) t = fmaxf(t, red[w]);
    mx[b] = t;
  }
}

__global__ void __launch_bounds__(NT) samp_mass_kernel(const Rows r, const float* gmax, unsigned long long* mass) {
  __shared__ unsigned long long red[NT / 32];
  const int b = blockIdx.x;
  unsigned long long s = 0;
  if (r.inv_t[b] > 0.f) {
    const float m = gmax[b];
    for (int i = threadIdx.x; i < r.V; i += NT) s += fix_mass(row_y(r, b, i), m);
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = s;
  __syncthreads();
  if (threadIdx.x == 0) {
    unsigned long long t = 0;
    for (int w = 0; w < NT / 32; ++w) t += red[w];
    mass[b] = t;
  }
}

// Per-row selection state: the key digits chosen so far, the mass strictly above the current key
// range, the mass target, and (after the last pass) the mass held by the selected key.
struct Sel {
  uint32_t* prefix;
  unsigned long long* above;
  unsigned long long* target;
  unsigned long long* key_mass;
  const int* active;  // [B] 1: this row takes part in the selection
};

__global__ void __launch_bounds__(NT) samp_hist_kernel(const Rows r, const float* gmax, const Sel s, int shift,
                                                       unsigned long long* hist) {
  __shared__ unsigned long long h[256];
  const int b = blockIdx.x;
  for (int i = threadIdx.x; i < 256; i += NT) h[i] = 0;
  __syncthreads();
  if (s.active[b]) {
    const float m = gmax[b];
    const uint32_t want = s.prefix[b];
    for (int i = threadIdx.x; i < r.V; i += NT) {
      const float y = row_y(r, b, i);
      const uint32_t k = fkey(y);
      if (shift < 24 && (k >> (shift + 8)) != (want >> (shift + 8))) continue;
      const unsigned long long w = fix_mass(y, m);
      if (w) atomicAdd(&h[(k >> shift) & 255u], w);
    }
  }
  __syncthreads();
  for (int i = threadIdx.x; i < 256; i += NT) hist[(long)b * 256 + i] = h[i];
}

// One thread per row: walk the (rank-summed) bins from the top and keep the digit whose descending
// cumulative mass reaches the target (the highest non-empty one when the target is 0).
__global__ void samp_select_kernel(int B, const Sel s, int shift, const unsigned long long* hist) {
  const int b = blockIdx.x * blockDim.x + threadIdx.x;
  if (b >= B || !s.active[b]) return;
  const unsigned long long* hb = hist + (long)b * 256;
  unsigned long long cum = s.above[b];
  const unsigned long long tgt = s.target[b];
  int pick = -1, last = -1;
  for (int bin = 255; bin >= 0; --bin) {
    const unsigned long long v = hb[bin];
    if (!v) continue;
    last = bin;
    if (cum + v >= tgt) {
      pick = bin;
      break;
    }
    cum += v;
  }
  if (pick < 0) {  // target above the remaining mass (fixed-point truncation): the lowest key
    pick = last < 0 ? 0 : last;
    cum -= last < 0 ? 0 : hb[pick];
  }
  s.prefix[b] |= (uint32_t)pick << shift;
  s.above[b] = cum;
  if (shift == 0) s.key_mass[b] = hb[pick];
}

// Per-row set-up of a selection. stage 0: the top-p cut (target = ceil(top_p * Z)); stage 1: the
// sample inside the kept prefix (target = ceil(r * kept mass), kept mass = mass above the cut key
// plus the cut key's own mass). Z and this rank's vocabulary-order offset P come from the
// all-gathered per-rank masses [world, B].
__global__ void samp_init_kernel(int B, int world, int rank, int stage, const float* inv_t, const float* top_p,
                                 const float* thr, const unsigned long long* masses, Sel s, int* active,
                                 unsigned long long* z, unsigned long long* pre) {
  const int b = blockIdx.x * blockDim.x + threadIdx.x;
  if (b >= B) return;
  const bool nucleus = inv_t[b] > 0.f && top_p[b] > 0.f && top_p[b] < 1.f;
  if (stage == 0) {
    unsigned long long tot = 0, p = 0;
    for (int q = 0; q < world; ++q) {
      if (q == rank) p = tot;
      tot += masses[(long)q * B + b];
    }
    z[b] = tot;
    pre[b] = p;
    active[b] = nucleus ? 1 : 0;
    s.prefix[b] = 0;
    s.above[b] = 0;
    s.target[b] = nucleus ? (unsigned long long)ceil((double)top_p[b] * (double)tot) : 0ull;
  } else if (nucleus) {
    const unsigned long long kept = s.above[b] + s.key_mass[b];
    s.prefix[b] = 0;
    s.above[b] = 0;
    s.target[b] = (unsigned long long)ceil((double)thr[b] * (double)kept);
  }
}

// Candidate of this rank per row (INT_MAX: none). Nucleus rows: the lowest local index whose key is
// the selected one. Rows with top_p >= 1: the first local index where the vocabulary-order CDF
// (this rank's offset P plus the running local mass) reaches ceil(r * Z). Greedy rows: none.
__global__ void __launch_bounds__(NT) samp_find_kernel(const Rows r, const float* gmax, const float* top_p,
                                                       const float* thr, const Sel s, const unsigned long long* z,
                                                       const unsigned long long* pre, int vocab_offset, int* cand) {
  __shared__ unsigned long long part[NT];
  __shared__ int best;
  const int b = blockIdx.x;
  if (threadIdx.x == 0) best = INT_MAX;
  __syncthreads();
  if (r.inv_t[b] > 0.f && top_p[b] > 0.f) {
    const float m = gmax[b];
    if (s.active[b]) {
      const uint32_t want = s.prefix[b];
      for (int i = threadIdx.x; i < r.V; i += NT)
        if (fkey(row_y(r, b, i)) == want) atomicMin(&best, i);
    } else {
      // contiguous chunk per thread, block-wide exclusive scan of the chunk masses
      const int chunk = (r.V + NT - 1) / NT;
      const int i0 = min(r.V, threadIdx.x * chunk), i1 = min(r.V, i0 + chunk);
      unsigned long long cs = 0;
      for (int i = i0; i < i1; ++i) cs += fix_mass(row_y(r, b, i), m);
      part[threadIdx.x] = cs;
      __syncthreads();
      for (int o = 1; o < NT; o <<= 1) {  // Hillis-Steele inclusive scan
        const unsigned long long v = threadIdx.x >= o ? part[threadIdx.x - o] : 0ull;
        __syncthreads();
        part[threadIdx.x] += v;
        __syncthreads();
      }
      const unsigned long long tgt = (unsigned long long)ceil((double)thr[b] * (double)z[b]);
      unsigned long long acc = pre[b] + part[threadIdx.x] - cs;  // mass before this chunk
      if (acc + cs >= tgt && i1 > i0) {
        for (int i = i0; i < i1; ++i) {
          acc += fix_mass(row_y(r, b, i), m);
          if (acc >= tgt) {
            atomicMin(&best, i);
            break;
          }
        }
      }
    }
  }
  __syncthreads();
  if (threadIdx.x == 0) cand[b] = best == INT_MAX ? INT_MAX : vocab_offset + best;
}

// ids = greedy ids for greedy rows (and rows without a candidate), the sampled candidate otherwise.
__global__ void samp_merge_kernel(int B, const float* inv_t, const float* top_p, const int* cand, const int* greedy,
                                  int* ids) {
  const int b = blockIdx.x * blockDim.x + threadIdx.x;
  if (b >= B) return;
  const bool sampled = inv_t[b] > 0.f && top_p[b] > 0.f;
  ids[b] = (sampled && cand[b] != INT_MAX) ? cand[b] : greedy[b];
}

}  // namespace samp
}  // namespace mesh

namespace mesh {
namespace {

// State workspace st: int64 [6, B] = prefix, above, target, key mass, Z, this rank's offset P;
// active: int32 [B].
samp::Sel sel_of(at::Tensor& st, at::Tensor& active) {
  const int B = st.size(1);
  auto* base = reinterpret_cast<unsigned long long*>(st.data_ptr<int64_t>());
  samp::Sel s;
  s.prefix = reinterpret_cast<uint32_t*>(base);  // low words of row 0 (uint32 per row)
  s.above = base + B;
  s.target = base + 2 * B;
  s.key_mass = base + 3 * B;
  s.active = active.data_ptr<int>();
  return s;
}
samp::Rows rows_of(const at::Tensor& logits, const at::Tensor& inv_t) {
  TORCH_CHECK(logits.is_cuda() && logits.scalar_type() == at::kFloat && logits.dim() == 2 && logits.stride(1) == 1,
              "sampling: fp32 logits [B, V_loc]");
  TORCH_CHECK(inv_t.scalar_type() == at::kFloat && inv_t.numel() == logits.size(0), "sampling: inv_t [B] fp32");
  samp::Rows r;
  r.logits = logits.data_ptr<float>();
  r.B = logits.size(0);
  r.V = logits.size(1);
  r.ld = logits.stride(0);
  r.inv_t = inv_t.data_ptr<float>();
  return r;
}

}  // namespace

// step: 0 max -> out (fp32 [B]); 1 fixed-point mass -> out (int64 [B]) given the global max `gmax`.
void samp_stats(const at::Tensor& logits, const at::Tensor& inv_t, const at::Tensor& gmax, at::Tensor& out,
                int64_t step) {
  const c10::cuda::CUDAGuard guard(logits.device());
  samp::Rows r = rows_of(logits, inv_t);
  if (r.B == 0) return;
  cudaStream_t st = at::cuda::getCurrentCUDAStream();
  if (step == 0)
    samp::samp_max_kernel<<<r.B, samp::NT, 0, st>>>(r, out.data_ptr<float>());
  else
    samp::samp_mass_kernel<<<r.B, samp::NT, 0, st>>>(
        r, gmax.data_ptr<float>(), reinterpret_cast<unsigned long long*>(out.data_ptr<int64_t>()));
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void samp_init(int64_t stage, int64_t world, int64_t rank, const at::Tensor& inv_t, const at::Tensor& top_p,
               const at::Tensor& thr, const at::Tensor& masses, at::Tensor& st, at::Tensor& active) {
  const c10::cuda::CUDAGuard guard(st.device());
  const int B = st.size(1);
  TORCH_CHECK(st.dim() == 2 && st.size(0) == 6 && masses.numel() == world * B, "samp_init: shapes");
  samp::Sel s = sel_of(st, active);
  auto* base = reinterpret_cast<unsigned long long*>(st.data_ptr<int64_t>());
  samp::samp_init_kernel<<<(B + 127) / 128, 128, 0, at::cuda::getCurrentCUDAStream()>>>(
      B, (int)world, (int)rank, (int)stage, inv_t.data_ptr<float>(), top_p.data_ptr<float>(), thr.data_ptr<float>(),
      reinterpret_cast<const unsigned long long*>(masses.data_ptr<int64_t>()), s, active.data_ptr<int>(), base + 4 * B,
      base + 5 * B);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

// pass with digit shift (24, 16, 8, 0): phase 0 builds this rank's histogram into hist [B, 256];
// phase 1 (after the cross-rank sum) selects the digit.
void samp_radix(const at::Tensor& logits, const at::Tensor& inv_t, const at::Tensor& gmax, at::Tensor& st,
                at::Tensor& active, at::Tensor& hist, int64_t shift, int64_t phase) {
  const c10::cuda::CUDAGuard guard(st.device());
  const int B = st.size(1);
  TORCH_CHECK(hist.numel() == (int64_t)B * 256 && hist.scalar_type() == at::kLong, "samp_radix: hist [B, 256] int64");
  samp::Sel s = sel_of(st, active);
  auto* h = reinterpret_cast<unsigned long long*>(hist.data_ptr<int64_t>());
  cudaStream_t stream = at::cuda::getCurrentCUDAStream();
  if (phase == 0)
    samp::samp_hist_kernel<<<B, samp::NT, 0, stream>>>(rows_of(logits, inv_t), gmax.data_ptr<float>(), s, (int)shift, h);
  else
    samp::samp_select_kernel<<<(B + 127) / 128, 128, 0, stream>>>(B, s, (int)shift, h);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void samp_find(const at::Tensor& logits, const at::Tensor& inv_t, const at::Tensor& gmax, const at::Tensor& top_p,
               const at::Tensor& thr, at::Tensor& st, at::Tensor& active, int64_t vocab_offset, at::Tensor& cand) {
  const c10::cuda::CUDAGuard guard(st.device());
  const int B = st.size(1);
  samp::Sel s = sel_of(st, active);
  auto* base = reinterpret_cast<unsigned long long*>(st.data_ptr<int64_t>());
  samp::samp_find_kernel<<<B, samp::NT, 0, at::cuda::getCurrentCUDAStream()>>>(
      rows_of(logits, inv_t), gmax.data_ptr<float>(), top_p.data_ptr<float>(), thr.data_ptr<float>(), s, base + 4 * B,
      base + 5 * B, (int)vocab_offset, cand.data_ptr<int>());
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void samp_merge(const at::Tensor& inv_t, const at::Tensor& top_p, const at::Tensor& cand, const at::Tensor& greedy,
                at::Tensor& ids) {
  const c10::cuda::CUDAGuard guard(ids.device());
  const int B = ids.numel();
  samp::samp_merge_kernel<<<(B + 127) / 128, 128, 0, at::cuda::getCurrentCUDAStream()>>>(
      B, inv_t.data_ptr<float>(), top_p.data_ptr<float>(), cand.data_ptr<int>(), greedy.data_ptr<int>(),
      ids.data_ptr<int>());
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

}  // namespace mesh
