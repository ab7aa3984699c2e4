// hcu_ops._C: torch-tensor wrappers over the C ABI of libhcu_indexer.so.
//
// Op names, argument order and meaning, output allocation (torch::empty on the
// input's device and current stream) and TORCH_CHECK messages follow the
// reference binding hcu_ops/csrc/bind.cpp:3-10,36-44,47-51,76-80 and the host
// checks of hcu_ops/csrc/mqa_hist.cu:329-357 / sparse_mask_topk.cu:846-870.
// The additional ops (dequant, ragged logits, keys, CP merge) keep the same
// conventions.
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/extension.h>

#include "../../include/hcu_indexer.h"

namespace {

constexpr int64_t kTopK = 2048;
constexpr int64_t kBins = 4096;

hcu_stream_t cur_stream() { return reinterpret_cast<hcu_stream_t>(at::cuda::getCurrentCUDAStream().stream()); }

void check_status(int st, const char* op) {
  TORCH_CHECK(st == HCU_OK, op, " failed: status ", st,
              st == HCU_ERR_ARG           ? " (invalid argument)"
              : st == HCU_ERR_UNSUPPORTED ? " (unsupported shape/option)"
              : st == HCU_ERR_LAUNCH      ? " (launch error)"
                                          : "",
              " ", hcu_last_error_string());
}

template <typename T>
T* ptr(const torch::Tensor& t) {
  return reinterpret_cast<T*>(t.data_ptr());
}

void check_topk_inputs(const torch::Tensor& score, const torch::Tensor& nonzero_mask, const torch::Tensor& lengths,
                       const torch::Tensor& page_table_size_1, const torch::Tensor& cu_seqlens_q, int64_t topk) {
  TORCH_CHECK(topk == kTopK, "sparse-mask TopK requires topk=2048");
  TORCH_CHECK(score.is_cuda() && score.scalar_type() == at::kFloat && score.dim() == 2 && score.stride(1) == 1,
              "score must be row-contiguous float32 [rows, width]");
  const int64_t rows = score.size(0);
  TORCH_CHECK(nonzero_mask.scalar_type() == at::kShort && nonzero_mask.dim() == 2 && nonzero_mask.stride(1) == 1 &&
                  nonzero_mask.size(0) == rows && nonzero_mask.size(1) == (score.size(1) + 15) / 16,
              "nonzero_mask must be row-contiguous int16 [rows, ceil(width/16)]");
  TORCH_CHECK(lengths.scalar_type() == at::kInt && lengths.dim() == 1 && lengths.is_contiguous() &&
                  lengths.size(0) == rows,
              "lengths must be contiguous int32 [rows]");
  TORCH_CHECK(page_table_size_1.scalar_type() == at::kInt && page_table_size_1.dim() == 2 &&
                  page_table_size_1.stride(1) == 1 && page_table_size_1.size(0) == rows,
              "page_table_size_1 must be row-contiguous int32 [rows, *]");
  TORCH_CHECK(cu_seqlens_q.size(0) == rows + 1,
              "only the decode layout (one page-table row per score row) is supported");
  TORCH_CHECK(rows == 0 || page_table_size_1.size(1) >= std::min<int64_t>(score.size(1), 1),
              "page_table_size_1 must cover the score width");
  TORCH_CHECK(nonzero_mask.device() == score.device() && lengths.device() == score.device() &&
                  page_table_size_1.device() == score.device(),
              "all tensors must be on the score's device");
}

torch::Tensor sparse_mask_topk_transform(const torch::Tensor& score, const torch::Tensor& nonzero_mask,
                                         const torch::Tensor& lengths, const torch::Tensor& page_table_size_1,
                                         const torch::Tensor& cu_seqlens_q, int64_t topk) {
  check_topk_inputs(score, nonzero_mask, lengths, page_table_size_1, cu_seqlens_q, topk);
  const c10::cuda::CUDAGuard guard(score.device());
  const int64_t rows = score.size(0);
  auto dst = torch::empty({rows, kTopK}, score.options().dtype(at::kInt));
  if (rows == 0) return dst;
  check_status(hcu_sparse_mask_topk_transform(ptr<const float>(score), rows, score.size(1), score.stride(0),
                                              ptr<const int16_t>(nonzero_mask), nonzero_mask.stride(0),
                                              ptr<const int32_t>(lengths), ptr<const int32_t>(page_table_size_1),
                                              page_table_size_1.stride(0), topk, ptr<int32_t>(dst), cur_stream()),
               "sparse_mask_topk_transform");
  return dst;
}

// List strategy for many rows (a warp streams each row into a short candidate list; same result).
torch::Tensor sparse_mask_topk_transform_lists(const torch::Tensor& score, const torch::Tensor& nonzero_mask,
                                               const torch::Tensor& lengths, const torch::Tensor& page_table_size_1,
                                               const torch::Tensor& cu_seqlens_q, int64_t topk) {
  check_topk_inputs(score, nonzero_mask, lengths, page_table_size_1, cu_seqlens_q, topk);
  TORCH_CHECK(score.size(1) <= 131072, "sparse_mask_topk_transform_lists: width above 131072");
  const c10::cuda::CUDAGuard guard(score.device());
  const int64_t rows = score.size(0);
  auto dst = torch::empty({rows, kTopK}, score.options().dtype(at::kInt));
  if (rows == 0) return dst;
  const int64_t wsb = hcu_sparse_mask_topk_transform_lists_workspace_bytes(rows, score.size(1));
  TORCH_CHECK(wsb > 0, "sparse_mask_topk_transform_lists: bad shape");
  auto ws = torch::empty({wsb}, score.options().dtype(at::kByte));
  check_status(hcu_sparse_mask_topk_transform_lists(ptr<const float>(score), rows, score.size(1), score.stride(0),
                                                    ptr<const int16_t>(nonzero_mask), nonzero_mask.stride(0),
                                                    ptr<const int32_t>(lengths),
                                                    ptr<const int32_t>(page_table_size_1),
                                                    page_table_size_1.stride(0), topk, ws.data_ptr(), wsb,
                                                    ptr<int32_t>(dst), cur_stream()),
               "sparse_mask_topk_transform_lists");
  return dst;
}

torch::Tensor sparse_mask_topk_transform_split(const torch::Tensor& score, const torch::Tensor& nonzero_mask,
                                               const torch::Tensor& lengths, const torch::Tensor& page_table_size_1,
                                               const torch::Tensor& cu_seqlens_q, int64_t topk, int64_t max_splits) {
  check_topk_inputs(score, nonzero_mask, lengths, page_table_size_1, cu_seqlens_q, topk);
  const c10::cuda::CUDAGuard guard(score.device());
  const int64_t rows = score.size(0);
  auto dst = torch::empty({rows, kTopK}, score.options().dtype(at::kInt));
  if (rows == 0) return dst;
  const int64_t wsb = hcu_topk_workspace_bytes(rows, score.size(1), max_splits);
  auto ws = torch::empty({std::max<int64_t>(wsb, 1)}, score.options().dtype(at::kByte));
  check_status(hcu_sparse_mask_topk_transform_split(
                   ptr<const float>(score), rows, score.size(1), score.stride(0), ptr<const int16_t>(nonzero_mask),
                   nonzero_mask.stride(0), ptr<const int32_t>(lengths), ptr<const int32_t>(page_table_size_1),
                   page_table_size_1.stride(0), topk, max_splits, ws.data_ptr(), wsb, ptr<int32_t>(dst),
                   cur_stream()),
               "sparse_mask_topk_transform_split");
  return dst;
}

torch::Tensor sparse_mask_topk_transform_split_pre(const torch::Tensor& score, const torch::Tensor& nonzero_mask,
                                                   const torch::Tensor& lengths,
                                                   const torch::Tensor& page_table_size_1,
                                                   const torch::Tensor& cu_seqlens_q, int64_t topk,
                                                   int64_t max_splits, const torch::Tensor& zws) {
  check_topk_inputs(score, nonzero_mask, lengths, page_table_size_1, cu_seqlens_q, topk);
  const c10::cuda::CUDAGuard guard(score.device());
  const int64_t rows = score.size(0);
  auto dst = torch::empty({rows, kTopK}, score.options().dtype(at::kInt));
  if (rows == 0) return dst;
  TORCH_CHECK(zws.scalar_type() == at::kInt && zws.is_contiguous() && zws.numel() == rows * (2 * kBins + 2),
              "zws must be the int32 [rows * (2 * 4096 + 2)] pass-1 workspace");
  const int64_t wsb = hcu_topk_workspace_bytes(rows, score.size(1), max_splits);
  auto ws = torch::empty({std::max<int64_t>(wsb, 1)}, score.options().dtype(at::kByte));
  check_status(hcu_sparse_mask_topk_transform_split_pre(
                   ptr<const float>(score), rows, score.size(1), score.stride(0), ptr<const int16_t>(nonzero_mask),
                   nonzero_mask.stride(0), ptr<const int32_t>(lengths), ptr<const int32_t>(page_table_size_1),
                   page_table_size_1.stride(0), topk, max_splits, ptr<int32_t>(zws), ws.data_ptr(), wsb,
                   ptr<int32_t>(dst), cur_stream()),
               "sparse_mask_topk_transform_split_pre");
  return dst;
}

std::vector<torch::Tensor> topk_keys(const torch::Tensor& score, const torch::Tensor& nonzero_mask,
                                     const torch::Tensor& lengths, const torch::Tensor& page_table) {
  check_topk_inputs(score, nonzero_mask, lengths, page_table,
                    torch::empty({score.size(0) + 1}, lengths.options()), kTopK);
  const c10::cuda::CUDAGuard guard(score.device());
  const int64_t rows = score.size(0);
  auto dst = torch::empty({rows, kTopK}, score.options().dtype(at::kInt));
  auto keys = torch::empty({rows, kTopK}, score.options().dtype(at::kInt));
  if (rows == 0) return {dst, keys};
  check_status(hcu_topk_keys(ptr<const float>(score), rows, score.size(1), score.stride(0),
                             ptr<const int16_t>(nonzero_mask), nonzero_mask.stride(0), ptr<const int32_t>(lengths),
                             ptr<const int32_t>(page_table), page_table.stride(0), ptr<int32_t>(dst),
                             ptr<uint32_t>(keys), cur_stream()),
               "topk_keys");
  return {dst, keys};
}

std::vector<torch::Tensor> mqa_logits_hist(const torch::Tensor& q, const torch::Tensor& kv_cache,
                                           const torch::Tensor& weights, const torch::Tensor& context_lens,
                                           const torch::Tensor& block_table, int64_t max_context_len,
                                           int64_t group_size, int64_t persistent_ctas, int64_t rows_per_cta,
                                           const c10::optional<torch::Tensor>& hist_lens) {
  TORCH_CHECK(q.is_cuda() && q.scalar_type() == at::kFloat8_e4m3fn && q.dim() == 4 && q.size(1) == 1 &&
                  (q.size(2) == 32 || q.size(2) == 64) && q.size(3) == 128 && q.is_contiguous(),
              "q must be contiguous fp8 e4m3fn [B, 1, 32|64, 128]");
  const int64_t B = q.size(0);
  const int64_t H = q.size(2);
  TORCH_CHECK(kv_cache.scalar_type() == at::kByte && kv_cache.dim() == 4 && kv_cache.size(1) == 64 &&
                  kv_cache.size(2) == 1 && kv_cache.size(3) == 132 && kv_cache.stride(1) == 132 &&
                  kv_cache.stride(3) == 1 && kv_cache.stride(0) % 16 == 0,
              "kv_cache must be packed fp8+scale uint8 [blocks, 64, 1, 132]");
  TORCH_CHECK(weights.scalar_type() == at::kFloat && weights.dim() == 2 && weights.size(0) == B &&
                  weights.size(1) == H && weights.is_contiguous(),
              "weights must be contiguous float32 [B, heads]");
  TORCH_CHECK(context_lens.scalar_type() == at::kInt && context_lens.dim() == 1 && context_lens.size(0) == B &&
                  context_lens.is_contiguous(),
              "context_lens must be contiguous int32 [B]");
  TORCH_CHECK(block_table.scalar_type() == at::kInt && block_table.dim() == 2 && block_table.size(0) == B &&
                  block_table.stride(1) == 1,
              "block_table must be row-contiguous int32 [B, pages]");
  TORCH_CHECK(max_context_len > 0 && max_context_len == block_table.size(1) * 64,
              "max_context_len must equal block_table capacity");
  TORCH_CHECK(B > 0 && group_size > 0 && B % group_size == 0, "batch must be a positive multiple of group_size");
  const bool hist = hist_lens.has_value();
  if (hist) {
    TORCH_CHECK(hist_lens->scalar_type() == at::kInt && hist_lens->dim() == 1 && hist_lens->size(0) == B &&
                    hist_lens->is_contiguous(),
                "hist_lens must be contiguous int32 [B]");
  }
  const c10::cuda::CUDAGuard guard(q.device());
  auto logits = torch::empty({B, max_context_len}, q.options().dtype(at::kFloat));
  const int64_t mask_stride = (max_context_len + 15) / 16;
  auto mask = torch::empty({B, mask_stride}, q.options().dtype(at::kShort));
  torch::Tensor zws = hist ? torch::empty({B * (2 * kBins + 2)}, q.options().dtype(at::kInt))
                           : torch::empty({0}, q.options().dtype(at::kInt));
  check_status(hcu_mqa_logits_hist(ptr<const uint8_t>(q), B, H, ptr<const uint8_t>(kv_cache), kv_cache.size(0),
                                   kv_cache.stride(0), ptr<const float>(weights), ptr<const int32_t>(context_lens),
                                   ptr<const int32_t>(block_table), block_table.stride(0), max_context_len,
                                   group_size, persistent_ctas, rows_per_cta,
                                   hist ? ptr<const int32_t>(*hist_lens) : nullptr, ptr<float>(logits),
                                   ptr<int16_t>(mask), hist ? ptr<int32_t>(zws) : nullptr, cur_stream()),
               "mqa_logits_hist");
  return {logits, mask, zws};
}

std::vector<torch::Tensor> mqa_logits_ragged(const torch::Tensor& q, const torch::Tensor& k_fp8,
                                             const torch::Tensor& k_scale, const torch::Tensor& weights,
                                             const torch::Tensor& row_start, const torch::Tensor& row_end) {
  TORCH_CHECK(q.is_cuda() && q.scalar_type() == at::kFloat8_e4m3fn && q.dim() == 3 &&
                  (q.size(1) == 32 || q.size(1) == 64) && q.size(2) == 128 && q.is_contiguous(),
              "q must be contiguous fp8 e4m3fn [rows, 32|64, 128]");
  const int64_t R = q.size(0);
  const int64_t H = q.size(1);
  TORCH_CHECK(k_fp8.scalar_type() == at::kFloat8_e4m3fn && k_fp8.dim() == 2 && k_fp8.size(1) == 128 &&
                  k_fp8.is_contiguous(),
              "k_fp8 must be contiguous fp8 e4m3fn [tokens, 128]");
  const int64_t N = k_fp8.size(0);
  TORCH_CHECK(k_scale.scalar_type() == at::kFloat && k_scale.numel() == N && k_scale.is_contiguous(),
              "k_scale must be contiguous float32 [tokens]");
  TORCH_CHECK(weights.scalar_type() == at::kFloat && weights.dim() == 2 && weights.size(0) == R &&
                  weights.size(1) == H && weights.is_contiguous(),
              "weights must be contiguous float32 [rows, heads]");
  TORCH_CHECK(row_start.scalar_type() == at::kInt && row_start.numel() == R && row_start.is_contiguous() &&
                  row_end.scalar_type() == at::kInt && row_end.numel() == R && row_end.is_contiguous(),
              "row_start / row_end must be contiguous int32 [rows]");
  const c10::cuda::CUDAGuard guard(q.device());
  const int64_t stride = (N + 63) / 64 * 64;
  auto logits = torch::empty({R, stride}, q.options().dtype(at::kFloat));
  auto mask = torch::empty({R, stride / 16}, q.options().dtype(at::kShort));
  if (R > 0)
    check_status(hcu_mqa_logits_ragged(ptr<const uint8_t>(q), R, H, ptr<const uint8_t>(k_fp8),
                                       ptr<const float>(k_scale), N, ptr<const float>(weights),
                                       ptr<const int32_t>(row_start), ptr<const int32_t>(row_end),
                                       ptr<float>(logits), stride, ptr<int16_t>(mask), cur_stream()),
                 "mqa_logits_ragged");
  return {logits.narrow(1, 0, N), mask.narrow(1, 0, (N + 15) / 16)};
}

// Fused prefill logits -> top-2048 (hcu_mqa_topk_ragged); fallback_flag (optional int32 [1]) is set
// to 1 when the exact path ran.
torch::Tensor mqa_topk_ragged(const torch::Tensor& q, const torch::Tensor& k_fp8, const torch::Tensor& k_scale,
                              const torch::Tensor& weights, const torch::Tensor& row_end,
                              const torch::Tensor& page_table, const c10::optional<torch::Tensor>& fallback_flag) {
  TORCH_CHECK(q.is_cuda() && q.scalar_type() == at::kFloat8_e4m3fn && q.dim() == 3 &&
                  (q.size(1) == 32 || q.size(1) == 64) && q.size(2) == 128 && q.is_contiguous(),
              "q must be contiguous fp8 e4m3fn [rows, 32|64, 128]");
  const int64_t R = q.size(0);
  const int64_t H = q.size(1);
  TORCH_CHECK(k_fp8.scalar_type() == at::kFloat8_e4m3fn && k_fp8.dim() == 2 && k_fp8.size(1) == 128 &&
                  k_fp8.is_contiguous(),
              "k_fp8 must be contiguous fp8 e4m3fn [tokens, 128]");
  const int64_t N = k_fp8.size(0);
  TORCH_CHECK(N <= 131072, "mqa_topk_ragged supports at most 131072 tokens");
  TORCH_CHECK(k_scale.scalar_type() == at::kFloat && k_scale.numel() == N && k_scale.is_contiguous(),
              "k_scale must be contiguous float32 [tokens]");
  TORCH_CHECK(weights.scalar_type() == at::kFloat && weights.dim() == 2 && weights.size(0) == R &&
                  weights.size(1) == H && weights.is_contiguous(),
              "weights must be contiguous float32 [rows, heads]");
  TORCH_CHECK(row_end.scalar_type() == at::kInt && row_end.numel() == R && row_end.is_contiguous(),
              "row_end must be contiguous int32 [rows]");
  TORCH_CHECK(page_table.scalar_type() == at::kInt && page_table.dim() == 2 && page_table.size(0) == R &&
                  page_table.size(1) >= N && page_table.stride(1) == 1,
              "page_table must be int32 [rows, >= tokens] with unit last stride");
  if (fallback_flag.has_value())
    TORCH_CHECK(fallback_flag->scalar_type() == at::kInt && fallback_flag->numel() >= 1 && fallback_flag->is_cuda(),
                "fallback_flag must be a CUDA int32 tensor of at least one element");
  const c10::cuda::CUDAGuard guard(q.device());
  auto out = torch::empty({R, kTopK}, q.options().dtype(at::kInt));
  if (R == 0) return out;
  const int64_t wsb = hcu_mqa_topk_ragged_workspace_bytes(R, N);
  auto ws = torch::empty({wsb}, q.options().dtype(at::kByte));
  check_status(hcu_mqa_topk_ragged(ptr<const uint8_t>(q), R, H, ptr<const uint8_t>(k_fp8), ptr<const float>(k_scale), N,
                                   ptr<const float>(weights), ptr<const int32_t>(row_end),
                                   ptr<const int32_t>(page_table), page_table.stride(0), ptr<int32_t>(out),
                                   ws.data_ptr(), wsb,
                                   fallback_flag.has_value() ? fallback_flag->data_ptr<int32_t>() : nullptr,
                                   cur_stream()),
               "mqa_topk_ragged");
  return out;
}

torch::Tensor dequantize_k_cache_paged(const torch::Tensor& quant_k_cache, const torch::Tensor& page_table_1) {
  TORCH_CHECK(quant_k_cache.is_cuda() && quant_k_cache.element_size() == 1 && quant_k_cache.size(-1) == 656 &&
                  quant_k_cache.stride(-1) == 1,
              "quant_k_cache must be a byte tensor [..., 656] with unit last stride");
  TORCH_CHECK(page_table_1.scalar_type() == at::kInt && page_table_1.dim() == 1 && page_table_1.is_contiguous(),
              "page_table_1_flattened must be contiguous int32 [n]");
  const c10::cuda::CUDAGuard guard(quant_k_cache.device());
  auto qk = quant_k_cache.view({-1, 656});
  const int64_t n = page_table_1.size(0);
  auto out = torch::empty({n, 1, 576}, quant_k_cache.options().dtype(at::kBFloat16));
  check_status(hcu_dequant_k_cache_paged(ptr<const uint8_t>(qk), qk.size(0), qk.stride(0),
                                         ptr<const int32_t>(page_table_1), n, ptr<uint16_t>(out), cur_stream()),
               "dequantize_k_cache_paged");
  return out;
}

torch::Tensor dequant_index_k_paged(const torch::Tensor& kv_cache, const torch::Tensor& token_loc) {
  TORCH_CHECK(kv_cache.is_cuda() && kv_cache.scalar_type() == at::kByte && kv_cache.dim() == 4 &&
                  kv_cache.size(1) == 64 && kv_cache.size(2) == 1 && kv_cache.size(3) == 132 &&
                  kv_cache.stride(1) == 132 && kv_cache.stride(3) == 1 && kv_cache.stride(0) % 16 == 0,
              "kv_cache must be packed fp8+scale uint8 [blocks, 64, 1, 132]");
  TORCH_CHECK(token_loc.scalar_type() == at::kInt && token_loc.dim() == 1 && token_loc.is_contiguous(),
              "token_loc must be contiguous int32 [n]");
  const c10::cuda::CUDAGuard guard(kv_cache.device());
  const int64_t n = token_loc.size(0);
  auto out = torch::empty({n, 128}, kv_cache.options().dtype(at::kBFloat16));
  check_status(hcu_dequant_index_k_paged(ptr<const uint8_t>(kv_cache), kv_cache.size(0), kv_cache.stride(0),
                                         ptr<const int32_t>(token_loc), n, ptr<uint16_t>(out), cur_stream()),
               "dequant_index_k_paged");
  return out;
}

torch::Tensor quant_store_index_k(const torch::Tensor& k, const torch::Tensor& token_loc, torch::Tensor kv_cache) {
  TORCH_CHECK(kv_cache.is_cuda() && kv_cache.scalar_type() == at::kByte && kv_cache.dim() == 4 &&
                  kv_cache.size(1) == 64 && kv_cache.size(2) == 1 && kv_cache.size(3) == 132 &&
                  kv_cache.stride(1) == 132 && kv_cache.stride(3) == 1 && kv_cache.stride(0) % 16 == 0,
              "kv_cache must be packed fp8+scale uint8 [blocks, 64, 1, 132]");
  TORCH_CHECK(k.device() == kv_cache.device() && (k.scalar_type() == at::kFloat || k.scalar_type() == at::kBFloat16) &&
                  k.dim() == 2 && k.size(1) == 128 && k.stride(1) == 1,
              "k must be float32 or bfloat16 [n, 128] with unit last stride");
  TORCH_CHECK(token_loc.scalar_type() == at::kInt && token_loc.dim() == 1 && token_loc.is_contiguous() &&
                  token_loc.size(0) == k.size(0),
              "token_loc must be contiguous int32 [n]");
  const c10::cuda::CUDAGuard guard(kv_cache.device());
  const int32_t dt = k.scalar_type() == at::kBFloat16 ? HCU_DTYPE_BF16 : HCU_DTYPE_F32;
  check_status(hcu_quant_store_index_k_paged(k.data_ptr(), dt, k.stride(0), ptr<const int32_t>(token_loc), k.size(0),
                                             ptr<uint8_t>(kv_cache), kv_cache.size(0), kv_cache.stride(0),
                                             cur_stream()),
               "quant_store_index_k");
  return kv_cache;
}

// kv_c [T, 512] / [T, 1, 512] and k_pe [T, 64] / [T, 1, 64]: the row stride of dim 0.
int64_t row_stride(const torch::Tensor& x, int64_t width) {
  TORCH_CHECK(x.size(-1) == width && x.stride(-1) == 1 && (x.dim() == 2 || (x.dim() == 3 && x.size(1) == 1)),
              "expected [T, ", width, "] or [T, 1, ", width, "] with a unit last stride");
  return x.stride(0);
}

void rope_qout_kv_store(const torch::Tensor& positions, const torch::Tensor& q_pe, torch::Tensor& q_out,
                        torch::Tensor& kv_c, const torch::Tensor& kv_weight, double norm_eps, torch::Tensor& k_pe,
                        const torch::Tensor& cos_sin_cache, bool is_neox, torch::Tensor& kv_buffer,
                        const torch::Tensor& loc, double store_eps, int64_t rsqrt_mode) {
  const int64_t T = positions.numel();
  TORCH_CHECK(positions.is_cuda() && positions.is_contiguous() &&
                  (positions.scalar_type() == at::kLong || positions.scalar_type() == at::kInt),
              "rope_qout_kv_store: positions must be contiguous int32/int64");
  const auto bf = at::kBFloat16;
  TORCH_CHECK(q_pe.scalar_type() == bf && q_out.scalar_type() == bf && kv_c.scalar_type() == bf &&
                  kv_weight.scalar_type() == bf && k_pe.scalar_type() == bf && cos_sin_cache.scalar_type() == bf,
              "rope_qout_kv_store: bf16 only");
  TORCH_CHECK(q_pe.dim() == 3 && q_pe.size(0) == T && q_pe.size(2) == 64 && q_pe.stride(2) == 1 &&
                  q_out.sizes() == q_pe.sizes() && q_out.stride(2) == 1,
              "rope_qout_kv_store: q_pe / q_out must be [T, nq, 64] with a unit last stride");
  TORCH_CHECK(cos_sin_cache.is_contiguous() && cos_sin_cache.dim() == 2 && cos_sin_cache.size(1) == 64,
              "rope_qout_kv_store: cos_sin_cache must be a contiguous [max_pos, 64]");
  TORCH_CHECK(kv_c.size(0) == T && k_pe.size(0) == T, "rope_qout_kv_store: kv_c / k_pe must have T rows");
  const int64_t kv_tok = row_stride(kv_c, 512), k_tok = row_stride(k_pe, 64);
  TORCH_CHECK(kv_weight.is_contiguous() && kv_weight.numel() == 512, "rope_qout_kv_store: weight must be [512]");
  TORCH_CHECK(kv_buffer.scalar_type() == at::kByte && kv_buffer.dim() >= 2 &&
                  kv_buffer.numel() / std::max<int64_t>(kv_buffer.size(0), 1) >= 656,
              "rope_qout_kv_store: kv_buffer must be uint8 with >= 656 bytes a slot");
  TORCH_CHECK(loc.scalar_type() == at::kLong && loc.is_contiguous() && loc.numel() <= T,
              "rope_qout_kv_store: loc must be a contiguous int64 of at most T slots");
  const c10::cuda::CUDAGuard guard(q_pe.device());
  check_status(hcu_rope_qout_kv_store(positions.data_ptr(), positions.scalar_type() == at::kLong ? 1 : 0, T,
                                      ptr<const uint16_t>(q_pe), q_pe.size(1), q_pe.stride(0), q_pe.stride(1),
                                      ptr<uint16_t>(q_out), q_out.stride(0), q_out.stride(1), ptr<uint16_t>(kv_c),
                                      kv_tok, ptr<const uint16_t>(kv_weight), static_cast<float>(norm_eps),
                                      ptr<uint16_t>(k_pe), k_tok, ptr<const uint16_t>(cos_sin_cache),
                                      cos_sin_cache.size(0), is_neox ? 1 : 0, ptr<uint8_t>(kv_buffer),
                                      kv_buffer.size(0), kv_buffer.stride(0), ptr<const int64_t>(loc), loc.numel(),
                                      static_cast<float>(store_eps), static_cast<int32_t>(rsqrt_mode), cur_stream()),
               "rope_qout_kv_store");
}

torch::Tensor cp_topk_merge(const torch::Tensor& keys, const torch::Tensor& gidx, const torch::Tensor& lengths) {
  TORCH_CHECK(keys.is_cuda() && keys.scalar_type() == at::kInt && keys.dim() == 3 && keys.size(2) == kTopK &&
                  keys.is_contiguous(),
              "keys must be contiguous int32 (uint32 bits) [parts, rows, 2048]");
  TORCH_CHECK(gidx.scalar_type() == at::kInt && gidx.sizes() == keys.sizes() && gidx.is_contiguous(),
              "gidx must be contiguous int32 [parts, rows, 2048]");
  TORCH_CHECK(lengths.scalar_type() == at::kInt && lengths.dim() == 1 && lengths.size(0) == keys.size(1) &&
                  lengths.is_contiguous(),
              "lengths must be contiguous int32 [rows]");
  const c10::cuda::CUDAGuard guard(keys.device());
  const int64_t rows = keys.size(1);
  auto dst = torch::empty({rows, kTopK}, keys.options());
  if (rows == 0) return dst;
  check_status(hcu_cp_topk_merge(ptr<const uint32_t>(keys), ptr<const int32_t>(gidx), keys.size(0), rows,
                                 ptr<const int32_t>(lengths), ptr<int32_t>(dst), cur_stream()),
               "cp_topk_merge");
  return dst;
}

torch::Tensor cp_local_bound(const torch::Tensor& score, const torch::Tensor& nonzero_mask, const torch::Tensor& lengths,
                             const torch::Tensor& totals) {
  check_topk_inputs(score, nonzero_mask, lengths, torch::empty({score.size(0), 1}, lengths.options()),
                    torch::empty({score.size(0) + 1}, lengths.options()), kTopK);
  TORCH_CHECK(totals.scalar_type() == at::kInt && totals.dim() == 1 && totals.size(0) == score.size(0) &&
                  totals.is_contiguous() && totals.device() == score.device(),
              "totals must be contiguous int32 [rows]");
  const c10::cuda::CUDAGuard guard(score.device());
  auto bounds = torch::empty({score.size(0)}, lengths.options());
  if (score.size(0) == 0) return bounds;
  check_status(hcu_cp_local_bound(ptr<const float>(score), score.size(0), score.size(1), score.stride(0),
                                  ptr<const int16_t>(nonzero_mask), nonzero_mask.stride(0), ptr<const int32_t>(lengths),
                                  ptr<const int32_t>(totals), ptr<int32_t>(bounds), cur_stream()),
               "cp_local_bound");
  return bounds;
}

// Writes the filtered lists into send [P, 2, rps, C] (keys then global indices per destination).
void cp_filter(const torch::Tensor& score, const torch::Tensor& nonzero_mask, const torch::Tensor& lengths,
               const torch::Tensor& page_table, const torch::Tensor& bounds, torch::Tensor& send, torch::Tensor& flag) {
  check_topk_inputs(score, nonzero_mask, lengths, page_table, torch::empty({score.size(0) + 1}, lengths.options()),
                    kTopK);
  TORCH_CHECK(bounds.scalar_type() == at::kInt && bounds.dim() == 1 && bounds.size(0) == score.size(0) &&
                  bounds.is_contiguous(),
              "bounds must be contiguous int32 [rows]");
  TORCH_CHECK(send.scalar_type() == at::kInt && send.dim() == 4 && send.size(1) == 2 && send.is_contiguous() &&
                  send.size(0) * send.size(2) >= score.size(0),
              "send must be contiguous int32 [P, 2, rows per rank, C] covering the rows");
  TORCH_CHECK(flag.scalar_type() == at::kInt && flag.numel() >= 1 && flag.is_contiguous(), "flag must be int32 [1]");
  const c10::cuda::CUDAGuard guard(score.device());
  if (score.size(0) == 0) return;
  const int64_t rps = send.size(2), cap = send.size(3);
  int32_t* base = ptr<int32_t>(send);
  check_status(hcu_cp_filter(ptr<const float>(score), score.size(0), score.size(1), score.stride(0),
                             ptr<const int16_t>(nonzero_mask), nonzero_mask.stride(0), ptr<const int32_t>(lengths),
                             ptr<const int32_t>(page_table), page_table.stride(0), ptr<const int32_t>(bounds), cap,
                             reinterpret_cast<uint32_t*>(base), base + rps * cap, rps, 2 * rps * cap, nullptr,
                             ptr<int32_t>(flag), cur_stream()),
               "cp_filter");
}

// Merges recv [P, 2, rows, C] (the exchanged lists of this rank's rows).
torch::Tensor cp_topk_merge_lists(const torch::Tensor& recv, const torch::Tensor& lengths,
                                  const c10::optional<torch::Tensor>& flag, bool short_identity) {
  TORCH_CHECK(recv.is_cuda() && recv.scalar_type() == at::kInt && recv.dim() == 4 && recv.size(1) == 2 &&
                  recv.is_contiguous(),
              "recv must be contiguous int32 [P, 2, rows, C]");
  const int64_t rows = recv.size(2), cap = recv.size(3);
  TORCH_CHECK(lengths.scalar_type() == at::kInt && lengths.dim() == 1 && lengths.size(0) == rows &&
                  lengths.is_contiguous(),
              "lengths must be contiguous int32 [rows]");
  const c10::cuda::CUDAGuard guard(recv.device());
  auto dst = torch::empty({rows, kTopK}, recv.options());
  if (rows == 0) return dst;
  const int32_t* base = ptr<const int32_t>(recv);
  check_status(hcu_cp_topk_merge_lists(reinterpret_cast<const uint32_t*>(base), base + rows * cap, recv.size(0), cap,
                                       2 * rows * cap, rows, ptr<const int32_t>(lengths),
                                       flag ? ptr<int32_t>(*flag) : nullptr, short_identity ? 1 : 0,
                                       ptr<int32_t>(dst), cur_stream()),
               "cp_topk_merge_lists");
  return dst;
}

// ---- context-parallel exchange over peer memory
// peers: int64 CPU tensor [7 + 5 * HCU_CP_MAX_PARTS] = parts, rank, rows, rows_per_rank, list_len, epoch,
// ws pointer, then the per-rank pointers of bounds, lists, lists_exact, out and sig (HCU_CP_MAX_PARTS each).
hcu_cp_peers_t unpack_peers(const torch::Tensor& t) {
  TORCH_CHECK(t.device().is_cpu() && t.scalar_type() == at::kLong && t.dim() == 1 && t.is_contiguous() &&
                  t.numel() == 7 + 5 * HCU_CP_MAX_PARTS,
              "peers must be a contiguous int64 CPU tensor of 7 + 5 x ", HCU_CP_MAX_PARTS, " entries");
  const int64_t* v = t.data_ptr<int64_t>();
  hcu_cp_peers_t p{};
  p.parts = static_cast<int32_t>(v[0]);
  p.rank = static_cast<int32_t>(v[1]);
  p.rows = static_cast<int32_t>(v[2]);
  p.rows_per_rank = static_cast<int32_t>(v[3]);
  p.list_len = static_cast<int32_t>(v[4]);
  p.epoch = static_cast<uint32_t>(v[5]);
  p.ws = reinterpret_cast<int32_t*>(v[6]);
  for (int i = 0; i < HCU_CP_MAX_PARTS; ++i) {
    p.bounds[i] = reinterpret_cast<int32_t*>(v[7 + i]);
    p.lists[i] = reinterpret_cast<int32_t*>(v[7 + HCU_CP_MAX_PARTS + i]);
    p.lists_exact[i] = reinterpret_cast<int32_t*>(v[7 + 2 * HCU_CP_MAX_PARTS + i]);
    p.out[i] = reinterpret_cast<int32_t*>(v[7 + 3 * HCU_CP_MAX_PARTS + i]);
    p.sig[i] = reinterpret_cast<uint32_t*>(v[7 + 4 * HCU_CP_MAX_PARTS + i]);
  }
  return p;
}

void cp_peer_bound(const torch::Tensor& score, const torch::Tensor& nonzero_mask, const torch::Tensor& lengths,
                   const torch::Tensor& totals, const torch::Tensor& peers) {
  const hcu_cp_peers_t p = unpack_peers(peers);
  TORCH_CHECK(score.is_cuda() && score.scalar_type() == at::kFloat && score.dim() == 2 && score.stride(1) == 1 &&
                  score.size(0) == p.rows,
              "score must be row-contiguous float32 [rows, width]");
  TORCH_CHECK(nonzero_mask.scalar_type() == at::kShort && nonzero_mask.dim() == 2 && nonzero_mask.stride(1) == 1 &&
                  nonzero_mask.size(0) == p.rows,
              "nonzero_mask must be row-contiguous int16 [rows, ceil(width/16)]");
  TORCH_CHECK(lengths.scalar_type() == at::kInt && lengths.is_contiguous() && lengths.numel() == p.rows &&
                  totals.scalar_type() == at::kInt && totals.is_contiguous() && totals.numel() == p.rows,
              "lengths and totals must be contiguous int32 [rows]");
  const c10::cuda::CUDAGuard guard(score.device());
  check_status(hcu_cp_peer_bound(ptr<const float>(score), score.size(1), score.stride(0),
                                 ptr<const int16_t>(nonzero_mask), nonzero_mask.stride(0), ptr<const int32_t>(lengths),
                                 ptr<const int32_t>(totals), &p, cur_stream()),
               "cp_peer_bound");
}

void cp_peer_filter(const torch::Tensor& score, const torch::Tensor& nonzero_mask, const torch::Tensor& lengths,
                    const torch::Tensor& page_table, const torch::Tensor& peers) {
  const hcu_cp_peers_t p = unpack_peers(peers);
  check_topk_inputs(score, nonzero_mask, lengths, page_table, torch::empty({score.size(0) + 1}, lengths.options()),
                    kTopK);
  TORCH_CHECK(score.size(0) == p.rows, "score rows must equal the exchange's rows");
  const c10::cuda::CUDAGuard guard(score.device());
  check_status(hcu_cp_peer_filter(ptr<const float>(score), score.size(1), score.stride(0),
                                  ptr<const int16_t>(nonzero_mask), nonzero_mask.stride(0),
                                  ptr<const int32_t>(lengths), ptr<const int32_t>(page_table), page_table.stride(0),
                                  &p, cur_stream()),
               "cp_peer_filter");
}

void cp_peer_merge(const torch::Tensor& totals, bool exact, const torch::Tensor& peers) {
  const hcu_cp_peers_t p = unpack_peers(peers);
  TORCH_CHECK(totals.is_cuda() && totals.scalar_type() == at::kInt && totals.is_contiguous() &&
                  totals.numel() == p.rows_per_rank,
              "totals must be contiguous int32 [rows_per_rank] (this rank's rows)");
  const c10::cuda::CUDAGuard guard(totals.device());
  check_status(hcu_cp_peer_merge(ptr<const int32_t>(totals), exact ? 1 : 0, &p, cur_stream()), "cp_peer_merge");
}

void cp_peer_scatter_exact(const torch::Tensor& keys, const torch::Tensor& entries, const torch::Tensor& peers) {
  const hcu_cp_peers_t p = unpack_peers(peers);
  TORCH_CHECK(keys.is_cuda() && keys.scalar_type() == at::kInt && keys.is_contiguous() && keys.dim() == 2 &&
                  keys.size(0) == p.rows && keys.size(1) == kTopK && entries.sizes() == keys.sizes() &&
                  entries.scalar_type() == at::kInt && entries.is_contiguous(),
              "keys and entries must be contiguous int32 [rows, 2048]");
  const c10::cuda::CUDAGuard guard(keys.device());
  check_status(hcu_cp_peer_scatter_exact(ptr<const uint32_t>(keys), ptr<const int32_t>(entries), &p, cur_stream()),
               "cp_peer_scatter_exact");
}

void cp_peer_finish(bool exact, const torch::Tensor& peers) {
  const hcu_cp_peers_t p = unpack_peers(peers);
  check_status(hcu_cp_peer_finish(exact ? 1 : 0, &p, cur_stream()), "cp_peer_finish");
}

std::vector<torch::Tensor> topk_keys_if(const torch::Tensor& score, const torch::Tensor& nonzero_mask,
                                        const torch::Tensor& lengths, const torch::Tensor& page_table,
                                        const torch::Tensor& run_if) {
  check_topk_inputs(score, nonzero_mask, lengths, page_table,
                    torch::empty({score.size(0) + 1}, lengths.options()), kTopK);
  TORCH_CHECK(run_if.is_cuda() && run_if.scalar_type() == at::kInt && run_if.numel() >= 1,
              "run_if must be an int32 device word");
  const c10::cuda::CUDAGuard guard(score.device());
  const int64_t rows = score.size(0);
  auto dst = torch::empty({rows, kTopK}, score.options().dtype(at::kInt));
  auto keys = torch::empty({rows, kTopK}, score.options().dtype(at::kInt));
  if (rows == 0) return {dst, keys};
  check_status(hcu_topk_keys_if(ptr<const float>(score), rows, score.size(1), score.stride(0),
                                ptr<const int16_t>(nonzero_mask), nonzero_mask.stride(0), ptr<const int32_t>(lengths),
                                ptr<const int32_t>(page_table), page_table.stride(0), ptr<int32_t>(dst),
                                ptr<uint32_t>(keys), ptr<const int32_t>(run_if), cur_stream()),
               "topk_keys_if");
  return {dst, keys};
}

void set_wait_limit_ns(int64_t ns) {
  TORCH_CHECK(ns >= 0, "the wait limit must be >= 0 (0: the default)");
  check_status(hcu_set_wait_limit_ns(static_cast<uint64_t>(ns)), "set_wait_limit_ns");
}

int64_t read_device_status(bool clear) {
  uint32_t s = 0;
  check_status(hcu_read_device_status(&s, clear ? 1 : 0), "read_device_status");
  return static_cast<int64_t>(s);
}

}  // namespace

PYBIND11_MODULE(TORCH_EXTENSION_NAME, m) {
  m.def("sparse_mask_topk_transform", &sparse_mask_topk_transform,
        "Exact top-2048 + page-table transform over sparse-mask MQA logits");
  m.def("sparse_mask_topk_transform_lists", &sparse_mask_topk_transform_lists,
        "top-2048 + page-table transform through per-row candidate lists (many rows)");
  m.def("sparse_mask_topk_transform_split", &sparse_mask_topk_transform_split,
        "Same as sparse_mask_topk_transform; few rows may be split over several CTAs");
  m.def("sparse_mask_topk_transform_split_pre", &sparse_mask_topk_transform_split_pre,
        "sparse_mask_topk_transform_split with pass 1 (histogram) taken from mqa_logits_hist's workspace");
  m.def("mqa_logits_hist", &mqa_logits_hist,
        "paged fp8 indexer logits -> {logits, mask, zws}; with hist_lens also top-k pass 1 into zws");
  m.def("rope_qout_kv_store", &rope_qout_kv_store,
        "MLA decode front end: q rope, kv_a RMS norm in place, k rope, fp8 656-byte KV slot store");
  m.def("cp_local_bound", &cp_local_bound, "context-parallel: per-row sampled bound of the global top-2048 threshold");
  m.def("cp_filter", &cp_filter, "context-parallel: tokens at or above the bound into the exchange buffer");
  m.def("cp_topk_merge_lists", &cp_topk_merge_lists, "context-parallel: merge of the exchanged bounded lists");
  m.def("mqa_logits_ragged", &mqa_logits_ragged,
        "prefill fp8 indexer logits over a contiguous K with per-row [start, end) -> {logits, mask}");
  m.def("mqa_topk_ragged", &mqa_topk_ragged,
        "fused prefill indexer: ragged logits (rows from token 0) -> exact top-2048 through the page table, "
        "without materialising the logits",
        py::arg("q"), py::arg("k_fp8"), py::arg("k_scale"), py::arg("weights"), py::arg("row_end"),
        py::arg("page_table"), py::arg("fallback_flag") = py::none());
  m.def("topk_keys", &topk_keys, "top-2048 indices through a page table plus the selected uint32 keys");
  m.def("dequantize_k_cache_paged", &dequantize_k_cache_paged,
        "MLA 656-byte slot paged dequant -> bf16 [n, 1, 576] (sglang dequantize_k_cache_paged drop-in)");
  m.def("dequant_index_k_paged", &dequant_index_k_paged, "indexer-K page dequant -> bf16 [n, 128]");
  m.def("quant_store_index_k", &quant_store_index_k,
        "quantise K rows per token to fp8 e4m3 + fp32 scale into indexer-K pages (in place)");
  m.def("cp_topk_merge", &cp_topk_merge, "merge per-range (key, global index) top-2048 lists");
  m.def("read_device_status", &read_device_status, "sticky device status bits of the library (synchronises)");
  m.def("cp_peer_bound", &cp_peer_bound, "context-parallel over peer memory: bounds to every rank");
  m.def("cp_peer_filter", &cp_peer_filter, "context-parallel over peer memory: lists to the rows' owners");
  m.def("cp_peer_merge", &cp_peer_merge, "context-parallel over peer memory: merge, rows to every rank");
  m.def("cp_peer_scatter_exact", &cp_peer_scatter_exact, "context-parallel over peer memory: the redo's lists");
  m.def("cp_peer_finish", &cp_peer_finish, "context-parallel over peer memory: wait for every rank's rows");
  m.def("topk_keys_if", &topk_keys_if, "topk_keys predicated on a device word (does nothing when it is 0)");
  m.def("set_wait_limit_ns", &set_wait_limit_ns, "limit of the library's bounded waits (0: default 2 s)");
  m.def("version", []() { return std::string(hcu_version()); });
}
