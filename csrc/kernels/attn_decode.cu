// Paged GQA decode attention (flash-decoding) for sm_100a.
//
// One query token per sequence. Grid (seq, kv_head, split); a CTA handles one KV head and all of
// its G query heads, so each K/V page of that head is read from HBM once for the whole group.
// Keys are assigned one per lane (32-token blocks, 4 warps stride over blocks); scores for the G
// heads are computed from a q copy in shared memory; P.V assigns 4 head dims per lane so each
// V row is read as one coalesced 256-byte line. Softmax is online in the exp2 domain.
// With split > 1 each CTA writes a normalised partial and its log2-sum-exp into a scratch buffer
// and the combine kernel merges them.
//
// Replaces the reference's per-session K/V materialisation, GQA index_select expansion, masked
// softmax and two batched GEMMs (forward_pass.rs:633-680, :783-828, :2703-2737, :2811-2835).
// KV layout: [pages, kv_heads, page_size, D] bf16; block_tables [B, max_pages] int32;
// seq_lens [B] int32 = number of valid keys (including the token being decoded).
#include <ATen/ATen.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/extension.h>

#include "../include/sm100.cuh"
#include "attn_decode.cuh"
#include "attn_decode_tc.cuh"
#include "../include/tma_host.h"

namespace mesh {

void attn_decode(const at::Tensor& q, const at::Tensor& kcache, const at::Tensor& vcache,
                 const at::Tensor& block_tables, const at::Tensor& seq_lens, at::Tensor& out, at::Tensor& ws,
                 int64_t splits, double scale, int64_t window) {
  TORCH_CHECK(q.scalar_type() == at::kBFloat16 && q.is_contiguous(), "attn_decode: q bf16 [B, hq*D]");
  TORCH_CHECK(kcache.dim() == 4 && kcache.sizes() == vcache.sizes(), "attn_decode: cache [pages, hkv, ps, D]");
  TORCH_CHECK(block_tables.scalar_type() == at::kInt && seq_lens.scalar_type() == at::kInt, "attn_decode: int32 tables");
  const int B = q.size(0);
  const int hkv = kcache.size(1), ps = kcache.size(2), D = kcache.size(3);
  TORCH_CHECK(D == 128 || D == 64, "attn_decode: head_dim 64 or 128");
  const int hq = q.size(1) / D;
  TORCH_CHECK(hq % hkv == 0, "attn_decode: hq % hkv");
  const int G = hq / hkv;
  TORCH_CHECK(G == 1 || G == 2 || G == 4 || G == 8, "attn_decode: group size 1/2/4/8");
  if (B == 0) return;
  if (splits < 1) splits = 1;
  if (splits > 1) {
    TORCH_CHECK(ws.scalar_type() == at::kFloat && ws.numel() >= (int64_t)B * hq * splits * (D + 1),
                "attn_decode: scratch too small");
  }
  const c10::cuda::CUDAGuard guard(q.device());
  DecodeArgs a;
  a.q = reinterpret_cast<const __nv_bfloat16*>(q.data_ptr());
  a.k = reinterpret_cast<const __nv_bfloat16*>(kcache.data_ptr());
  a.v = reinterpret_cast<const __nv_bfloat16*>(vcache.data_ptr());
  a.block_tables = block_tables.data_ptr<int>();
  a.seq_lens = seq_lens.data_ptr<int>();
  a.out = reinterpret_cast<__nv_bfloat16*>(out.data_ptr());
  a.ws = splits > 1 ? ws.data_ptr<float>() : nullptr;
  a.max_pages = block_tables.size(1);
  a.hkv = hkv;
  a.page_size = ps;
  a.splits = (int)splits;
  a.scale_log2 = (float)(scale * 1.4426950408889634);
  a.window = (int)window;
  const cudaError_t e = launch_attn_decode(a, B, G, D, at::cuda::getCurrentCUDAStream());
  TORCH_CHECK(e == cudaSuccess, "attn_decode launch failed: ", cudaGetErrorString(e));
}

// TMA-streamed tensor-core variant (head_dim 128, 16-token pages).
void attn_decode_tc(const at::Tensor& q, const at::Tensor& kcache, const at::Tensor& vcache,
                    const at::Tensor& block_tables, const at::Tensor& seq_lens, at::Tensor& out, at::Tensor& ws,
                    at::Tensor& err, int64_t splits, double scale, int64_t window,
                    const c10::optional<at::Tensor>& counters) {
  TORCH_CHECK(q.scalar_type() == at::kBFloat16 && q.is_contiguous(), "attn_decode_tc: q bf16 [B, hq*D]");
  TORCH_CHECK(kcache.dim() == 4 && kcache.sizes() == vcache.sizes() && kcache.is_contiguous() && vcache.is_contiguous(),
              "attn_decode_tc: cache [pages, hkv, 16, 128] contiguous");
  TORCH_CHECK(kcache.size(2) == 16 && kcache.size(3) == 128, "attn_decode_tc: page 16, head_dim 128");
  const int B = q.size(0), hkv = kcache.size(1);
  const int hq = q.size(1) / 128;
  const int G = hq / hkv;
  TORCH_CHECK(hq % hkv == 0 && (G == 1 || G == 2 || G == 4 || G == 8), "attn_decode_tc: group size 1/2/4/8");
  if (B == 0) return;
  if (splits < 1) splits = 1;
  if (splits > 1)
    TORCH_CHECK(ws.scalar_type() == at::kFloat && ws.numel() >= (int64_t)B * hq * splits * 129, "attn_decode_tc: scratch");
  const c10::cuda::CUDAGuard guard(q.device());
  const uint64_t rows = (uint64_t)kcache.size(0) * hkv * 16;
  CUtensorMap tk = tma_map_2d_bf16(kcache.data_ptr(), 128, rows, 128, 64, 16);
  CUtensorMap tv = tma_map_2d_bf16(vcache.data_ptr(), 128, rows, 128, 64, 16);
  DecodeTcArgs a;
  a.q = reinterpret_cast<const __nv_bfloat16*>(q.data_ptr());
  a.block_tables = block_tables.data_ptr<int>();
  a.seq_lens = seq_lens.data_ptr<int>();
  a.out = reinterpret_cast<__nv_bfloat16*>(out.data_ptr());
  a.ws = splits > 1 ? ws.data_ptr<float>() : nullptr;
  a.err = err.data_ptr<int>();
  a.max_pages = block_tables.size(1);
  a.hkv = hkv;
  a.splits = (int)splits;
  a.scale_log2 = (float)(scale * 1.4426950408889634);
  a.window = (int)window;
  a.counters = nullptr;
  if (splits > 1 && counters.has_value() && counters->defined() && counters->numel() > 0) {
    TORCH_CHECK(counters->is_cuda() && counters->scalar_type() == at::kInt && counters->is_contiguous() &&
                    counters->numel() >= (int64_t)B * hkv,
                "attn_decode_tc: counters int32 [>= B * hkv], zero between launches");
    a.counters = counters->data_ptr<int>();
  }
  cudaStream_t st = at::cuda::getCurrentCUDAStream();
  switch (G) {
    case 1: launch_attn_decode_tc_g<1>(tk, tv, a, B, st); break;
    case 2: launch_attn_decode_tc_g<2>(tk, tv, a, B, st); break;
    case 4: launch_attn_decode_tc_g<4>(tk, tv, a, B, st); break;
    default: launch_attn_decode_tc_g<8>(tk, tv, a, B, st); break;
  }
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

int64_t attn_decode_pick_splits(int64_t B, int64_t hkv, int64_t max_len, int64_t num_sms) {
  // Measured on B200 (64 sequences x 576 keys): splitting pays only while the (sequence, KV head)
  // CTAs leave most SMs idle; beyond that each split adds a CTA start-up and the combine pass
  // (8 KV heads: 29 us unsplit vs 41 us with 2 splits; 1 KV head: 12.2 us unsplit, 9.5 us with 4).
  const int64_t ctas = B * hkv;
  if (4 * ctas >= 3 * num_sms) return 1;
  int64_t s = (3 * num_sms + ctas) / (2 * ctas);  // about 1.5 waves of CTAs
  int64_t max_s = (max_len + 127) / 128;           // keep >= 128 keys per split
  if (s > max_s) s = max_s;
  if (s > 64) s = 64;
  return s < 1 ? 1 : s;
}

}  // namespace mesh
