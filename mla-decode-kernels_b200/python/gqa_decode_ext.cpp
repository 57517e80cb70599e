// PyTorch binding of the C ABI in include/gqa_decode.h.
//
// Mirrors the reference extension (python/gqa_decode_ext.cpp of
// yuqiz7/mla-decode-kernels): the same three functions with the same
// argument names, the same default num_splits = 8 and the same validation
// messages (reference lines 16-62, 102-103), launching on the current torch
// stream.  Everything below the tensor checks goes through the extern "C"
// entry points of libgqa_decode_b200.so.
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/extension.h>

#include <algorithm>
#include <vector>

#include "gqa_decode.h"
#include "mla_decode.h"
#include "dsa_decode.h"

namespace {

struct GqaDims {
  int64_t B, Hq, Hkv, block_size, max_blocks, num_blocks;
};

GqaDims check_inputs(const torch::Tensor& q, const torch::Tensor& k_cache,
                     const torch::Tensor& v_cache, const torch::Tensor& block_table,
                     const torch::Tensor& seq_lens) {
  TORCH_CHECK(q.is_cuda(), "q must be a CUDA tensor");
  TORCH_CHECK(q.scalar_type() == torch::kBFloat16, "q must be bf16");
  TORCH_CHECK(q.is_contiguous(), "q must be contiguous");
  TORCH_CHECK(q.dim() == 3 && q.size(2) == 128, "q must be [B, Hq, 128]");

  TORCH_CHECK(k_cache.is_cuda() && v_cache.is_cuda(), "k_cache/v_cache must be CUDA tensors");
  TORCH_CHECK(k_cache.scalar_type() == torch::kBFloat16 &&
                  v_cache.scalar_type() == torch::kBFloat16,
              "k_cache/v_cache must be bf16");
  TORCH_CHECK(k_cache.is_contiguous() && v_cache.is_contiguous(),
              "k_cache/v_cache must be contiguous");
  TORCH_CHECK(k_cache.dim() == 4 && k_cache.size(3) == 128,
              "k_cache must be [num_blocks, block_size, Hkv, 128]");
  TORCH_CHECK(k_cache.sizes() == v_cache.sizes(), "k_cache and v_cache must have the same shape");

  TORCH_CHECK(block_table.is_cuda(), "block_table must be a CUDA tensor");
  TORCH_CHECK(block_table.scalar_type() == torch::kInt32, "block_table must be int32");
  TORCH_CHECK(block_table.is_contiguous(), "block_table must be contiguous");
  TORCH_CHECK(block_table.dim() == 2, "block_table must be [B, max_blocks]");

  TORCH_CHECK(seq_lens.is_cuda(), "seq_lens must be a CUDA tensor");
  TORCH_CHECK(seq_lens.scalar_type() == torch::kInt32, "seq_lens must be int32");
  TORCH_CHECK(seq_lens.is_contiguous(), "seq_lens must be contiguous");
  TORCH_CHECK(seq_lens.dim() == 1, "seq_lens must be [B]");

  const int64_t B = q.size(0);
  const int64_t Hq = q.size(1);
  const int64_t Hkv = k_cache.size(2);
  const int64_t block_size = k_cache.size(1);
  const int64_t max_blocks = block_table.size(1);
  TORCH_CHECK(Hq % Hkv == 0, "Hq must be divisible by Hkv");
  TORCH_CHECK(block_table.size(0) == B, "block_table batch dim must match q");
  TORCH_CHECK(seq_lens.size(0) == B, "seq_lens batch dim must match q");
  TORCH_CHECK(q.device() == k_cache.device() && q.device() == v_cache.device() &&
                  q.device() == block_table.device() && q.device() == seq_lens.device(),
              "all tensors must be on the same device");
  // Limits of this engine (not in the reference): the group fits 16 MMA
  // column tiles, and the bulk-copy engine needs 16-byte aligned bases.
  TORCH_CHECK(Hq / Hkv <= 128, "Hq / Hkv must be at most 128");
  TORCH_CHECK(max_blocks >= 1, "block_table must have at least one column");
  TORCH_CHECK(reinterpret_cast<uintptr_t>(q.data_ptr()) % 16 == 0 &&
                  reinterpret_cast<uintptr_t>(k_cache.data_ptr()) % 16 == 0 &&
                  reinterpret_cast<uintptr_t>(v_cache.data_ptr()) % 16 == 0,
              "q/k_cache/v_cache must be 16-byte aligned");
  TORCH_CHECK(B <= INT32_MAX && k_cache.size(0) <= INT32_MAX, "dimension too large");
  return {B, Hq, Hkv, block_size, max_blocks, k_cache.size(0)};
}

const gqa_bf16* bf16_ptr(const torch::Tensor& t) {
  return reinterpret_cast<const gqa_bf16*>(t.data_ptr());
}

void check_launch(cudaError_t e, const char* what) {
  TORCH_CHECK(e == cudaSuccess, what, " failed: ", cudaGetErrorString(e));
}

using launch_fn_t = void (*)(const gqa_bf16*, const gqa_bf16*, const gqa_bf16*, const int*,
                             const int*, gqa_bf16*, int, int, int, int, int, float, cudaStream_t);

torch::Tensor gqa_decode_run(launch_fn_t launch, const char* name, torch::Tensor q,
                             torch::Tensor k_cache, torch::Tensor v_cache,
                             torch::Tensor block_table, torch::Tensor seq_lens, double scale) {
  const GqaDims d = check_inputs(q, k_cache, v_cache, block_table, seq_lens);
  const c10::cuda::CUDAGuard guard(q.device());
  auto out = torch::empty_like(q);
  cudaStream_t stream = at::cuda::getCurrentCUDAStream();
  launch(bf16_ptr(q), bf16_ptr(k_cache), bf16_ptr(v_cache), block_table.data_ptr<int>(),
         seq_lens.data_ptr<int>(), reinterpret_cast<gqa_bf16*>(out.data_ptr()),
         static_cast<int>(d.B), static_cast<int>(d.Hq), static_cast<int>(d.Hkv),
         static_cast<int>(d.block_size), static_cast<int>(d.max_blocks),
         static_cast<float>(scale), stream);
  check_launch(gqa_decode_last_error(), name);
  return out;
}

}  // namespace

torch::Tensor gqa_decode_v0(torch::Tensor q, torch::Tensor k_cache, torch::Tensor v_cache,
                            torch::Tensor block_table, torch::Tensor seq_lens, double scale) {
  return gqa_decode_run(gqa_decode_v0_launch, "gqa_decode_v0", q, k_cache, v_cache, block_table,
                        seq_lens, scale);
}

torch::Tensor gqa_decode_v1(torch::Tensor q, torch::Tensor k_cache, torch::Tensor v_cache,
                            torch::Tensor block_table, torch::Tensor seq_lens, double scale) {
  return gqa_decode_run(gqa_decode_v1_launch, "gqa_decode_v1", q, k_cache, v_cache, block_table,
                        seq_lens, scale);
}

torch::Tensor gqa_decode_v2(torch::Tensor q, torch::Tensor k_cache, torch::Tensor v_cache,
                            torch::Tensor block_table, torch::Tensor seq_lens, double scale,
                            int64_t num_splits) {
  const GqaDims d = check_inputs(q, k_cache, v_cache, block_table, seq_lens);
  TORCH_CHECK(num_splits >= 1 && num_splits <= 512, "num_splits must be in [1, 512]");
  const c10::cuda::CUDAGuard guard(q.device());
  auto out = torch::empty_like(q);
  auto f32 = torch::TensorOptions().dtype(torch::kFloat32).device(q.device());
  // Same per-call workspace as the reference extension (lines 106-109).
  auto ws_acc = torch::empty({d.B, d.Hq, num_splits, 128}, f32);
  auto ws_m = torch::empty({d.B, d.Hq, num_splits}, f32);
  auto ws_l = torch::empty({d.B, d.Hq, num_splits}, f32);
  cudaStream_t stream = at::cuda::getCurrentCUDAStream();
  gqa_decode_v2_launch(bf16_ptr(q), bf16_ptr(k_cache), bf16_ptr(v_cache),
                       block_table.data_ptr<int>(), seq_lens.data_ptr<int>(),
                       reinterpret_cast<gqa_bf16*>(out.data_ptr()), static_cast<int>(d.B),
                       static_cast<int>(d.Hq), static_cast<int>(d.Hkv),
                       static_cast<int>(d.block_size), static_cast<int>(d.max_blocks),
                       static_cast<float>(scale), static_cast<int>(num_splits),
                       ws_acc.data_ptr<float>(), ws_m.data_ptr<float>(), ws_l.data_ptr<float>(),
                       stream);
  check_launch(gqa_decode_last_error(), "gqa_decode_v2");
  return out;
}

// Balanced (num_splits == 0) or fixed-split decode into `out` with a caller
// workspace (uint8 CUDA tensor, zeroed once).  check_blocks validates every
// block id against k_cache.size(0).
torch::Tensor gqa_decode(torch::Tensor q, torch::Tensor k_cache, torch::Tensor v_cache,
                         torch::Tensor block_table, torch::Tensor seq_lens, double scale,
                         int64_t num_splits, torch::Tensor workspace, bool check_blocks,
                         c10::optional<torch::Tensor> out_opt) {
  const GqaDims d = check_inputs(q, k_cache, v_cache, block_table, seq_lens);
  TORCH_CHECK(num_splits >= 0 && num_splits <= 512, "num_splits must be in [0, 512]");
  TORCH_CHECK(workspace.is_cuda() && workspace.device() == q.device() && workspace.is_contiguous(),
              "workspace must be a contiguous CUDA tensor on q's device");
  const c10::cuda::CUDAGuard guard(q.device());
  torch::Tensor out;
  if (out_opt.has_value()) {
    out = *out_opt;
    TORCH_CHECK(out.sizes() == q.sizes() && out.scalar_type() == torch::kBFloat16 &&
                    out.is_contiguous() && out.device() == q.device(),
                "out must be a contiguous bf16 tensor shaped like q on q's device");
  } else {
    out = torch::empty_like(q);
  }
  cudaStream_t stream = at::cuda::getCurrentCUDAStream();
  const size_t ws_bytes = static_cast<size_t>(workspace.numel()) * workspace.element_size();
  check_launch(
      gqa_decode_launch(bf16_ptr(q), bf16_ptr(k_cache), bf16_ptr(v_cache),
                        block_table.data_ptr<int>(), seq_lens.data_ptr<int>(),
                        reinterpret_cast<gqa_bf16*>(out.data_ptr()), static_cast<int>(d.B),
                        static_cast<int>(d.Hq), static_cast<int>(d.Hkv),
                        static_cast<int>(d.block_size), static_cast<int>(d.max_blocks),
                        check_blocks ? static_cast<int>(d.num_blocks) : 0,
                        static_cast<float>(scale), static_cast<int>(num_splits),
                        workspace.data_ptr(), ws_bytes, stream),
      "gqa_decode");
  return out;
}

// Unnormalised per-(request, q head) softmax states (m, l, acc) for KV-range
// sharding; see gqa_decode_partial_launch.
std::vector<torch::Tensor> gqa_decode_partial(torch::Tensor q, torch::Tensor k_cache,
                                              torch::Tensor v_cache, torch::Tensor block_table,
                                              torch::Tensor seq_lens, double scale,
                                              torch::Tensor workspace, bool check_blocks) {
  const GqaDims d = check_inputs(q, k_cache, v_cache, block_table, seq_lens);
  TORCH_CHECK(workspace.is_cuda() && workspace.device() == q.device() && workspace.is_contiguous(),
              "workspace must be a contiguous CUDA tensor on q's device");
  const c10::cuda::CUDAGuard guard(q.device());
  auto f32 = torch::TensorOptions().dtype(torch::kFloat32).device(q.device());
  auto m = torch::empty({d.B, d.Hq}, f32);
  auto l = torch::empty({d.B, d.Hq}, f32);
  auto acc = torch::empty({d.B, d.Hq, 128}, f32);
  cudaStream_t stream = at::cuda::getCurrentCUDAStream();
  const size_t ws_bytes = static_cast<size_t>(workspace.numel()) * workspace.element_size();
  check_launch(gqa_decode_partial_launch(
                   bf16_ptr(q), bf16_ptr(k_cache), bf16_ptr(v_cache), block_table.data_ptr<int>(),
                   seq_lens.data_ptr<int>(), m.data_ptr<float>(), l.data_ptr<float>(),
                   acc.data_ptr<float>(), static_cast<int>(d.B), static_cast<int>(d.Hq),
                   static_cast<int>(d.Hkv), static_cast<int>(d.block_size),
                   static_cast<int>(d.max_blocks), check_blocks ? static_cast<int>(d.num_blocks) : 0,
                   static_cast<float>(scale), workspace.data_ptr(), ws_bytes, stream),
               "gqa_decode_partial");
  return {m, l, acc};
}

// KV-range sharded decode with the cross-rank merge over peer memory; see
// gqa_decode_kvshard_launch.  peer_ptrs[r] = rank r's exchange buffer as
// mapped in this process.
torch::Tensor gqa_decode_kvshard(torch::Tensor q, torch::Tensor k_cache, torch::Tensor v_cache,
                                 torch::Tensor block_table, torch::Tensor seq_lens, double scale,
                                 int64_t rank, int64_t world, std::vector<int64_t> peer_ptrs,
                                 int64_t epoch, torch::Tensor workspace, bool check_blocks,
                                 c10::optional<torch::Tensor> out_opt) {
  const GqaDims d = check_inputs(q, k_cache, v_cache, block_table, seq_lens);
  TORCH_CHECK(world >= 1 && world <= 8 && rank >= 0 && rank < world,
              "rank/world must satisfy 0 <= rank < world <= 8");
  TORCH_CHECK(static_cast<int64_t>(peer_ptrs.size()) == world, "need one exchange buffer per rank");
  TORCH_CHECK(epoch > 0 && epoch <= 0xffffffffLL, "epoch must be in [1, 2^32)");
  TORCH_CHECK(workspace.is_cuda() && workspace.device() == q.device() && workspace.is_contiguous(),
              "workspace must be a contiguous CUDA tensor on q's device");
  const c10::cuda::CUDAGuard guard(q.device());
  void* peers[8] = {nullptr};
  for (int64_t r = 0; r < world; ++r) peers[r] = reinterpret_cast<void*>(peer_ptrs[r]);
  torch::Tensor out;
  if (out_opt.has_value()) {
    out = *out_opt;
    TORCH_CHECK(out.is_cuda() && out.device() == q.device() && out.scalar_type() == torch::kBFloat16 &&
                    out.is_contiguous() && out.sizes() == q.sizes(),
                "out must be a contiguous bf16 CUDA tensor shaped like q on q's device");
  } else {
    out = torch::empty_like(q);
  }
  cudaStream_t stream = at::cuda::getCurrentCUDAStream();
  const size_t ws_bytes = static_cast<size_t>(workspace.numel()) * workspace.element_size();
  check_launch(gqa_decode_kvshard_launch(
                   bf16_ptr(q), bf16_ptr(k_cache), bf16_ptr(v_cache), block_table.data_ptr<int>(),
                   seq_lens.data_ptr<int>(), reinterpret_cast<gqa_bf16*>(out.data_ptr()),
                   static_cast<int>(d.B), static_cast<int>(d.Hq), static_cast<int>(d.Hkv),
                   static_cast<int>(d.block_size), static_cast<int>(d.max_blocks),
                   check_blocks ? static_cast<int>(d.num_blocks) : 0, static_cast<float>(scale),
                   static_cast<int>(rank), static_cast<int>(world), peers,
                   static_cast<unsigned>(epoch), workspace.data_ptr(), ws_bytes, stream),
               "gqa_decode_kvshard");
  return out;
}

int64_t kvshard_buffer_bytes(int64_t B, int64_t Hq, int64_t Hkv, int64_t world) {
  return static_cast<int64_t>(gqa_decode_kvshard_buffer_bytes(
      static_cast<int>(B), static_cast<int>(Hq), static_cast<int>(Hkv), static_cast<int>(world)));
}

// Merge states [nshards, rows] (+ acc [nshards, rows, 128]) into bf16 [rows, 128].
torch::Tensor merge_states(torch::Tensor m, torch::Tensor l, torch::Tensor acc) {
  TORCH_CHECK(m.is_cuda() && l.is_cuda() && acc.is_cuda(), "states must be CUDA tensors");
  TORCH_CHECK(m.scalar_type() == torch::kFloat32 && l.scalar_type() == torch::kFloat32 &&
                  acc.scalar_type() == torch::kFloat32,
              "states must be fp32");
  TORCH_CHECK(m.is_contiguous() && l.is_contiguous() && acc.is_contiguous(),
              "states must be contiguous");
  TORCH_CHECK(m.dim() == 2 && l.sizes() == m.sizes() && acc.dim() == 3 &&
                  acc.size(0) == m.size(0) && acc.size(1) == m.size(1) && acc.size(2) == 128,
              "states must be m, l [n, rows] and acc [n, rows, 128]");
  const c10::cuda::CUDAGuard guard(m.device());
  auto out = torch::empty({m.size(1), 128},
                          torch::TensorOptions().dtype(torch::kBFloat16).device(m.device()));
  cudaStream_t stream = at::cuda::getCurrentCUDAStream();
  check_launch(gqa_decode_merge_states(m.data_ptr<float>(), l.data_ptr<float>(),
                                       acc.data_ptr<float>(), static_cast<int>(m.size(0)),
                                       static_cast<int>(m.size(1)),
                                       reinterpret_cast<gqa_bf16*>(out.data_ptr()), stream),
               "merge_states");
  return out;
}

// ---- CSR front end and plan/run ---------------------------------------------

namespace {

void check_i32(const torch::Tensor& t, const torch::Tensor& like, const char* what) {
  TORCH_CHECK(t.is_cuda() && t.device() == like.device(), what, " must be on q's device");
  TORCH_CHECK(t.scalar_type() == torch::kInt32 && t.is_contiguous(), what,
              " must be a contiguous int32 tensor");
}

gqa_decode_pages dense_pages(const torch::Tensor& block_table, const torch::Tensor& seq_lens,
                             int64_t page_size, int64_t num_blocks) {
  gqa_decode_pages pg{};
  pg.block_table = block_table.data_ptr<int>();
  pg.seq_lens = seq_lens.data_ptr<int>();
  pg.max_blocks = static_cast<int>(block_table.size(1));
  pg.block_size = static_cast<int>(page_size);
  pg.num_blocks = static_cast<int>(num_blocks);
  return pg;
}

gqa_decode_pages csr_pages(const torch::Tensor& indptr, const torch::Tensor& indices,
                           const torch::Tensor& last, int64_t page_size, int64_t num_blocks) {
  gqa_decode_pages pg{};
  pg.kv_indptr = indptr.data_ptr<int>();
  pg.kv_indices = indices.data_ptr<int>();
  pg.kv_last_page_len = last.data_ptr<int>();
  pg.block_size = static_cast<int>(page_size);
  pg.num_blocks = static_cast<int>(num_blocks);
  return pg;
}

}  // namespace

// block_table / seq_lens -> (kv_indptr [B+1], kv_indices [B*max_blocks]
// (the first kv_indptr[B] are valid), kv_last_page_len [B]).
std::vector<torch::Tensor> block_table_to_csr(torch::Tensor block_table, torch::Tensor seq_lens,
                                              int64_t page_size) {
  TORCH_CHECK(block_table.is_cuda() && block_table.scalar_type() == torch::kInt32 &&
                  block_table.is_contiguous() && block_table.dim() == 2,
              "block_table must be a contiguous int32 CUDA tensor [B, max_blocks]");
  check_i32(seq_lens, block_table, "seq_lens");
  TORCH_CHECK(seq_lens.dim() == 1 && seq_lens.size(0) == block_table.size(0),
              "seq_lens must be [B]");
  TORCH_CHECK(page_size >= 1, "page_size must be positive");
  const c10::cuda::CUDAGuard guard(block_table.device());
  const int64_t B = block_table.size(0), mb = block_table.size(1);
  auto i32 = torch::TensorOptions().dtype(torch::kInt32).device(block_table.device());
  auto indptr = torch::empty({B + 1}, i32);
  auto indices = torch::empty({std::max<int64_t>(1, B * mb)}, i32);
  auto last = torch::empty({B}, i32);
  check_launch(gqa_decode_block_table_to_csr(
                   block_table.data_ptr<int>(), seq_lens.data_ptr<int>(), static_cast<int>(B),
                   static_cast<int>(std::max<int64_t>(1, mb)), static_cast<int>(page_size),
                   indptr.data_ptr<int>(), indices.data_ptr<int>(), last.data_ptr<int>(),
                   at::cuda::getCurrentCUDAStream()),
               "gqa_decode_block_table_to_csr");
  return {indptr, indices, last};
}

void plan_csr(torch::Tensor indptr, torch::Tensor indices, torch::Tensor last, int64_t Hq,
              int64_t Hkv, int64_t page_size, int64_t num_blocks, torch::Tensor workspace) {
  check_i32(indptr, workspace, "kv_indptr");
  check_i32(indices, workspace, "kv_indices");
  check_i32(last, workspace, "kv_last_page_len");
  TORCH_CHECK(indptr.dim() == 1 && indptr.size(0) >= 1 && last.size(0) == indptr.size(0) - 1,
              "kv_indptr must be [B + 1] and kv_last_page_len [B]");
  const c10::cuda::CUDAGuard guard(workspace.device());
  const gqa_decode_pages pg = csr_pages(indptr, indices, last, page_size, num_blocks);
  const size_t ws_bytes = static_cast<size_t>(workspace.numel()) * workspace.element_size();
  check_launch(gqa_decode_plan(&pg, static_cast<int>(last.size(0)), static_cast<int>(Hq),
                               static_cast<int>(Hkv), workspace.data_ptr(), ws_bytes,
                               at::cuda::getCurrentCUDAStream()),
               "gqa_decode_plan");
}

void plan_dense(torch::Tensor block_table, torch::Tensor seq_lens, int64_t Hq, int64_t Hkv,
                int64_t page_size, int64_t num_blocks, torch::Tensor workspace) {
  check_i32(block_table, workspace, "block_table");
  check_i32(seq_lens, workspace, "seq_lens");
  TORCH_CHECK(block_table.dim() == 2 && seq_lens.dim() == 1 &&
                  seq_lens.size(0) == block_table.size(0),
              "block_table must be [B, max_blocks] and seq_lens [B]");
  const c10::cuda::CUDAGuard guard(workspace.device());
  const gqa_decode_pages pg = dense_pages(block_table, seq_lens, page_size, num_blocks);
  const size_t ws_bytes = static_cast<size_t>(workspace.numel()) * workspace.element_size();
  check_launch(gqa_decode_plan(&pg, static_cast<int>(seq_lens.size(0)), static_cast<int>(Hq),
                               static_cast<int>(Hkv), workspace.data_ptr(), ws_bytes,
                               at::cuda::getCurrentCUDAStream()),
               "gqa_decode_plan");
}

torch::Tensor run_pages(const gqa_decode_pages& pg, const torch::Tensor& q,
                        const torch::Tensor& k_cache, const torch::Tensor& v_cache, double scale,
                        torch::Tensor workspace, c10::optional<torch::Tensor> out_opt) {
  TORCH_CHECK(q.is_cuda() && q.scalar_type() == torch::kBFloat16 && q.is_contiguous() &&
                  q.dim() == 3 && q.size(2) == 128,
              "q must be a contiguous bf16 CUDA tensor [B, Hq, 128]");
  TORCH_CHECK(k_cache.sizes() == v_cache.sizes() && k_cache.dim() == 4 && k_cache.size(3) == 128 &&
                  k_cache.scalar_type() == torch::kBFloat16 &&
                  v_cache.scalar_type() == torch::kBFloat16 && k_cache.is_contiguous() &&
                  v_cache.is_contiguous() && k_cache.device() == q.device() &&
                  v_cache.device() == q.device(),
              "k_cache/v_cache must be contiguous bf16 [num_blocks, block_size, Hkv, 128] on q's device");
  TORCH_CHECK(k_cache.size(1) == pg.block_size, "page_size must match k_cache.size(1)");
  TORCH_CHECK(workspace.is_cuda() && workspace.device() == q.device() && workspace.is_contiguous(),
              "workspace must be a contiguous CUDA tensor on q's device");
  const c10::cuda::CUDAGuard guard(q.device());
  torch::Tensor out = out_opt.has_value() ? *out_opt : torch::empty_like(q);
  TORCH_CHECK(out.sizes() == q.sizes() && out.scalar_type() == torch::kBFloat16 &&
                  out.is_contiguous() && out.device() == q.device(),
              "out must be a contiguous bf16 tensor shaped like q on q's device");
  const size_t ws_bytes = static_cast<size_t>(workspace.numel()) * workspace.element_size();
  check_launch(gqa_decode_run(bf16_ptr(q), bf16_ptr(k_cache), bf16_ptr(v_cache), &pg,
                              reinterpret_cast<gqa_bf16*>(out.data_ptr()),
                              static_cast<int>(q.size(0)), static_cast<int>(q.size(1)),
                              static_cast<int>(k_cache.size(2)), static_cast<float>(scale),
                              workspace.data_ptr(), ws_bytes, at::cuda::getCurrentCUDAStream()),
               "gqa_decode_run");
  return out;
}

torch::Tensor run_csr(torch::Tensor q, torch::Tensor k_cache, torch::Tensor v_cache,
                      torch::Tensor indptr, torch::Tensor indices, torch::Tensor last,
                      double scale, torch::Tensor workspace, bool check_blocks,
                      c10::optional<torch::Tensor> out) {
  check_i32(indptr, q, "kv_indptr");
  check_i32(indices, q, "kv_indices");
  check_i32(last, q, "kv_last_page_len");
  TORCH_CHECK(indptr.dim() == 1 && indptr.size(0) == q.size(0) + 1 && last.size(0) == q.size(0),
              "kv_indptr must be [B + 1] and kv_last_page_len [B]");
  const gqa_decode_pages pg = csr_pages(indptr, indices, last, k_cache.size(1),
                                        check_blocks ? k_cache.size(0) : 0);
  return run_pages(pg, q, k_cache, v_cache, scale, workspace, out);
}

torch::Tensor run_dense(torch::Tensor q, torch::Tensor k_cache, torch::Tensor v_cache,
                        torch::Tensor block_table, torch::Tensor seq_lens, double scale,
                        torch::Tensor workspace, bool check_blocks,
                        c10::optional<torch::Tensor> out) {
  check_inputs(q, k_cache, v_cache, block_table, seq_lens);
  const gqa_decode_pages pg = dense_pages(block_table, seq_lens, k_cache.size(1),
                                          check_blocks ? k_cache.size(0) : 0);
  return run_pages(pg, q, k_cache, v_cache, scale, workspace, out);
}

int64_t workspace_bytes(int64_t B, int64_t Hq, int64_t Hkv, int64_t num_splits) {
  return static_cast<int64_t>(gqa_decode_workspace_bytes(
      static_cast<int>(B), static_cast<int>(Hq), static_cast<int>(Hkv), static_cast<int>(num_splits)));
}

int64_t get_status(bool clear) {
  int s = 0;
  check_launch(gqa_decode_get_status(&s, clear ? 1 : 0), "gqa_decode_get_status");
  return s;
}

int64_t pick_splits(int64_t B, int64_t Hq, int64_t Hkv, int64_t seq_len, int64_t num_sms) {
  return gqa_decode_pick_splits(static_cast<int>(B), static_cast<int>(Hq), static_cast<int>(Hkv),
                                static_cast<int>(seq_len), static_cast<int>(num_sms));
}

// ---- MLA latent-cache decode (include/mla_decode.h) ------------------------

// q [B, s_q, h_q, 576] bf16, kv_cache [num_blocks, 64, 1, 576] bf16 ->
// (out [B, s_q, h_q, 512] bf16, lse [B, h_q, s_q] fp32).
std::vector<torch::Tensor> mla_decode(torch::Tensor q, torch::Tensor kv_cache,
                                      torch::Tensor block_table, torch::Tensor seq_lens,
                                      double softmax_scale, bool causal, int64_t num_splits,
                                      torch::Tensor workspace) {
  // (block ids are always range-checked: the TMA tensor map spans exactly
  // kv_cache's num_blocks pages)
  TORCH_CHECK(q.is_cuda() && kv_cache.is_cuda() && block_table.is_cuda() && seq_lens.is_cuda(),
              "all tensors must be CUDA tensors");
  TORCH_CHECK(q.scalar_type() == torch::kBFloat16 && kv_cache.scalar_type() == torch::kBFloat16,
              "q and kv_cache must be bf16");
  TORCH_CHECK(block_table.scalar_type() == torch::kInt32 && seq_lens.scalar_type() == torch::kInt32,
              "block_table and seq_lens must be int32");
  TORCH_CHECK(q.is_contiguous() && kv_cache.is_contiguous() && block_table.is_contiguous() &&
                  seq_lens.is_contiguous(),
              "all tensors must be contiguous");
  TORCH_CHECK(q.dim() == 4 && q.size(3) == 576, "q must be [B, s_q, h_q, 576]");
  TORCH_CHECK(kv_cache.dim() == 4 && kv_cache.size(2) == 1 && kv_cache.size(3) == 576,
              "kv_cache must be [num_blocks, page, 1, 576]");
  TORCH_CHECK(kv_cache.size(1) == 64, "page size must be 64");
  TORCH_CHECK(block_table.dim() == 2 && block_table.size(0) == q.size(0) &&
                  seq_lens.dim() == 1 && seq_lens.size(0) == q.size(0),
              "block_table [B, max_blocks] and seq_lens [B] must match q's batch");
  TORCH_CHECK(kv_cache.device() == q.device() && block_table.device() == q.device() &&
                  seq_lens.device() == q.device(),
              "all tensors must be on the same device");
  TORCH_CHECK(num_splits >= 1 && num_splits <= 64, "num_splits must be in [1, 64]");
  const c10::cuda::CUDAGuard guard(q.device());
  const int64_t B = q.size(0), s_q = q.size(1), h_q = q.size(2);
  auto out = torch::empty({B, s_q, h_q, 512}, q.options());
  auto lse = torch::empty({B, h_q, s_q}, q.options().dtype(torch::kFloat32));
  const size_t need = mla_decode_workspace_bytes(static_cast<int>(B), static_cast<int>(s_q),
                                                 static_cast<int>(h_q), static_cast<int>(num_splits));
  const size_t ws_bytes = static_cast<size_t>(workspace.numel()) * workspace.element_size();
  TORCH_CHECK(need == 0 || (workspace.is_cuda() && workspace.device() == q.device() &&
                            workspace.is_contiguous() && ws_bytes >= need),
              "workspace must be a contiguous CUDA tensor of at least ", need, " bytes");
  cudaStream_t stream = at::cuda::getCurrentCUDAStream();
  check_launch(mla_decode_launch(reinterpret_cast<const gqa_bf16*>(q.data_ptr()),
                                 reinterpret_cast<const gqa_bf16*>(kv_cache.data_ptr()),
                                 block_table.data_ptr<int>(), seq_lens.data_ptr<int>(),
                                 reinterpret_cast<gqa_bf16*>(out.data_ptr()), lse.data_ptr<float>(),
                                 static_cast<int>(B), static_cast<int>(s_q), static_cast<int>(h_q),
                                 64, static_cast<int>(block_table.size(1)),
                                 static_cast<int>(kv_cache.size(0)),
                                 static_cast<float>(softmax_scale), causal ? 1 : 0,
                                 static_cast<int>(num_splits), need ? workspace.data_ptr() : nullptr,
                                 ws_bytes, stream),
               "mla_decode");
  return {out, lse};
}

// Sparse attention over selected tokens: indices [B, s_q, topk] int32 token
// positions, counts [B, s_q] int32 -> (out [B, s_q, h_q, 512] bf16, lse [B, h_q, s_q]).
std::vector<torch::Tensor> mla_decode_sparse(torch::Tensor q, torch::Tensor kv_cache,
                                             torch::Tensor block_table, torch::Tensor indices,
                                             torch::Tensor counts, double softmax_scale,
                                             int64_t num_splits, torch::Tensor workspace) {
  TORCH_CHECK(q.is_cuda() && kv_cache.is_cuda() && block_table.is_cuda() && indices.is_cuda() &&
                  counts.is_cuda(),
              "all tensors must be CUDA tensors");
  TORCH_CHECK(q.scalar_type() == torch::kBFloat16 && kv_cache.scalar_type() == torch::kBFloat16,
              "q and kv_cache must be bf16");
  TORCH_CHECK(block_table.scalar_type() == torch::kInt32 && indices.scalar_type() == torch::kInt32 &&
                  counts.scalar_type() == torch::kInt32,
              "block_table, indices and counts must be int32");
  TORCH_CHECK(q.is_contiguous() && kv_cache.is_contiguous() && block_table.is_contiguous() &&
                  indices.is_contiguous() && counts.is_contiguous(),
              "all tensors must be contiguous");
  TORCH_CHECK(q.dim() == 4 && q.size(3) == 576, "q must be [B, s_q, h_q, 576]");
  TORCH_CHECK(q.size(2) % 128 == 0, "the fused sparse decode takes h_q a multiple of 128");
  TORCH_CHECK(kv_cache.dim() == 4 && kv_cache.size(1) == 64 && kv_cache.size(2) == 1 &&
                  kv_cache.size(3) == 576,
              "kv_cache must be [num_blocks, 64, 1, 576]");
  const int64_t B = q.size(0), s_q = q.size(1), h_q = q.size(2);
  TORCH_CHECK(block_table.dim() == 2 && block_table.size(0) == B,
              "block_table must be [B, max_blocks]");
  TORCH_CHECK(indices.dim() == 3 && indices.size(0) == B && indices.size(1) == s_q,
              "indices must be [B, s_q, topk]");
  TORCH_CHECK(counts.dim() == 2 && counts.size(0) == B && counts.size(1) == s_q,
              "counts must be [B, s_q]");
  TORCH_CHECK(kv_cache.device() == q.device() && block_table.device() == q.device() &&
                  indices.device() == q.device() && counts.device() == q.device(),
              "all tensors must be on the same device");
  TORCH_CHECK(num_splits >= 1 && num_splits <= 64, "num_splits must be in [1, 64]");
  const c10::cuda::CUDAGuard guard(q.device());
  auto out = torch::empty({B, s_q, h_q, 512}, q.options());
  auto lse = torch::empty({B, h_q, s_q}, q.options().dtype(torch::kFloat32));
  const size_t need = mla_decode_workspace_bytes(static_cast<int>(B), static_cast<int>(s_q),
                                                 static_cast<int>(h_q), static_cast<int>(num_splits));
  const size_t ws_bytes = static_cast<size_t>(workspace.numel()) * workspace.element_size();
  TORCH_CHECK(need == 0 || (workspace.is_cuda() && workspace.device() == q.device() &&
                            workspace.is_contiguous() && ws_bytes >= need),
              "workspace must be a contiguous CUDA tensor of at least ", need, " bytes");
  check_launch(mla_decode_sparse_launch(
                   reinterpret_cast<const gqa_bf16*>(q.data_ptr()),
                   reinterpret_cast<const gqa_bf16*>(kv_cache.data_ptr()),
                   block_table.data_ptr<int>(), indices.data_ptr<int>(), counts.data_ptr<int>(),
                   static_cast<int>(indices.size(2)), reinterpret_cast<gqa_bf16*>(out.data_ptr()),
                   lse.data_ptr<float>(), static_cast<int>(B), static_cast<int>(s_q),
                   static_cast<int>(h_q), 64, static_cast<int>(block_table.size(1)),
                   static_cast<int>(kv_cache.size(0)), static_cast<float>(softmax_scale),
                   static_cast<int>(num_splits), need ? workspace.data_ptr() : nullptr, ws_bytes,
                   at::cuda::getCurrentCUDAStream()),
               "mla_decode_sparse");
  return {out, lse};
}

// Sparse attention over selected cache rows: rows [B, s_q, topk] int32
// physical rows (block id * 64 + slot, -1 padded) as dsa_topk_rows resolves
// them, counts [B, s_q] -> (out [B, s_q, h_q, 512] bf16, lse [B, h_q, s_q]).
std::vector<torch::Tensor> mla_decode_sparse_rows(torch::Tensor q, torch::Tensor kv_cache,
                                                  torch::Tensor rows, torch::Tensor counts,
                                                  double softmax_scale, int64_t num_splits,
                                                  torch::Tensor workspace) {
  TORCH_CHECK(q.is_cuda() && kv_cache.is_cuda() && rows.is_cuda() && counts.is_cuda(),
              "all tensors must be CUDA tensors");
  TORCH_CHECK(q.scalar_type() == torch::kBFloat16 && kv_cache.scalar_type() == torch::kBFloat16,
              "q and kv_cache must be bf16");
  TORCH_CHECK(rows.scalar_type() == torch::kInt32 && counts.scalar_type() == torch::kInt32,
              "rows and counts must be int32");
  TORCH_CHECK(q.is_contiguous() && kv_cache.is_contiguous() && rows.is_contiguous() &&
                  counts.is_contiguous(),
              "all tensors must be contiguous");
  TORCH_CHECK(q.dim() == 4 && q.size(3) == 576, "q must be [B, s_q, h_q, 576]");
  TORCH_CHECK(q.size(2) % 128 == 0, "the fused sparse decode takes h_q a multiple of 128");
  TORCH_CHECK(kv_cache.dim() == 4 && kv_cache.size(1) == 64 && kv_cache.size(2) == 1 &&
                  kv_cache.size(3) == 576,
              "kv_cache must be [num_blocks, 64, 1, 576]");
  const int64_t B = q.size(0), s_q = q.size(1), h_q = q.size(2);
  TORCH_CHECK(rows.dim() == 3 && rows.size(0) == B && rows.size(1) == s_q,
              "rows must be [B, s_q, topk]");
  TORCH_CHECK(counts.dim() == 2 && counts.size(0) == B && counts.size(1) == s_q,
              "counts must be [B, s_q]");
  TORCH_CHECK(kv_cache.device() == q.device() && rows.device() == q.device() &&
                  counts.device() == q.device(),
              "all tensors must be on the same device");
  TORCH_CHECK(num_splits >= 1 && num_splits <= 64, "num_splits must be in [1, 64]");
  const c10::cuda::CUDAGuard guard(q.device());
  auto out = torch::empty({B, s_q, h_q, 512}, q.options());
  auto lse = torch::empty({B, h_q, s_q}, q.options().dtype(torch::kFloat32));
  const size_t need = mla_decode_workspace_bytes(static_cast<int>(B), static_cast<int>(s_q),
                                                 static_cast<int>(h_q), static_cast<int>(num_splits));
  const size_t ws_bytes = static_cast<size_t>(workspace.numel()) * workspace.element_size();
  TORCH_CHECK(need == 0 || (workspace.is_cuda() && workspace.device() == q.device() &&
                            workspace.is_contiguous() && ws_bytes >= need),
              "workspace must be a contiguous CUDA tensor of at least ", need, " bytes");
  check_launch(mla_decode_sparse_rows_launch(
                   reinterpret_cast<const gqa_bf16*>(q.data_ptr()),
                   reinterpret_cast<const gqa_bf16*>(kv_cache.data_ptr()), rows.data_ptr<int>(),
                   counts.data_ptr<int>(), static_cast<int>(rows.size(2)),
                   reinterpret_cast<gqa_bf16*>(out.data_ptr()), lse.data_ptr<float>(),
                   static_cast<int>(B), static_cast<int>(s_q), static_cast<int>(h_q), 64,
                   static_cast<int>(kv_cache.size(0)), static_cast<float>(softmax_scale),
                   static_cast<int>(num_splits), need ? workspace.data_ptr() : nullptr, ws_bytes,
                   at::cuda::getCurrentCUDAStream()),
               "mla_decode_sparse_rows");
  return {out, lse};
}

int64_t mla_workspace_bytes(int64_t B, int64_t s_q, int64_t h_q, int64_t num_splits) {
  return static_cast<int64_t>(mla_decode_workspace_bytes(static_cast<int>(B), static_cast<int>(s_q),
                                                         static_cast<int>(h_q),
                                                         static_cast<int>(num_splits)));
}

int64_t mla_pick_splits(int64_t B, int64_t s_q, int64_t h_q, int64_t max_pages, int64_t num_sms) {
  return mla_decode_pick_splits(static_cast<int>(B), static_cast<int>(s_q), static_cast<int>(h_q),
                                static_cast<int>(max_pages), static_cast<int>(num_sms));
}

int64_t mla_get_status(bool clear) { return mla_decode_get_status(clear ? 1 : 0); }

// ---- DSA sparse decode: indexer, top-k, gather (include/dsa_decode.h) --------

void check_paged(const torch::Tensor& t, const char* name, int64_t dim) {
  TORCH_CHECK(t.is_cuda() && t.scalar_type() == torch::kBFloat16 && t.is_contiguous(), name,
              " must be a contiguous bf16 CUDA tensor");
  const bool shape4 = t.dim() == 4 && t.size(2) == 1 && t.size(3) == dim;
  const bool shape3 = t.dim() == 3 && t.size(2) == dim;
  TORCH_CHECK((shape4 || shape3) && t.size(1) == 64, name, " must be [num_blocks, 64, 1, ", dim,
              "] or [num_blocks, 64, ", dim, "]");
}

void check_table(const torch::Tensor& block_table, const torch::Tensor& seq_lens, int64_t B,
                 const torch::Device& dev) {
  TORCH_CHECK(block_table.is_cuda() && seq_lens.is_cuda() && block_table.device() == dev &&
                  seq_lens.device() == dev,
              "block_table and seq_lens must be CUDA tensors on the query's device");
  TORCH_CHECK(block_table.scalar_type() == torch::kInt32 && seq_lens.scalar_type() == torch::kInt32,
              "block_table and seq_lens must be int32");
  TORCH_CHECK(block_table.is_contiguous() && seq_lens.is_contiguous(),
              "block_table and seq_lens must be contiguous");
  TORCH_CHECK(block_table.dim() == 2 && block_table.size(0) == B && seq_lens.dim() == 1 &&
                  seq_lens.size(0) == B,
              "block_table [B, max_blocks] and seq_lens [B] must match the batch");
}

// q_idx [B, s_q, H, 128] bf16, w_idx [B, s_q, H] fp32, k_idx [num_blocks, 64, (1,) 128]
// bf16 -> scores [B, s_q, max_blocks * 64] fp32 (columns past S_b unwritten).
torch::Tensor dsa_indexer(torch::Tensor q_idx, torch::Tensor w_idx, torch::Tensor k_idx,
                          torch::Tensor block_table, torch::Tensor seq_lens, bool causal) {
  TORCH_CHECK(q_idx.is_cuda() && q_idx.scalar_type() == torch::kBFloat16 && q_idx.is_contiguous(),
              "q_idx must be a contiguous bf16 CUDA tensor");
  TORCH_CHECK(q_idx.dim() == 4 && q_idx.size(3) == 128, "q_idx must be [B, s_q, H, 128]");
  const int64_t B = q_idx.size(0), s_q = q_idx.size(1), H = q_idx.size(2);
  TORCH_CHECK(w_idx.is_cuda() && w_idx.scalar_type() == torch::kFloat32 && w_idx.is_contiguous() &&
                  w_idx.device() == q_idx.device(),
              "w_idx must be a contiguous fp32 CUDA tensor on q_idx's device");
  TORCH_CHECK(w_idx.dim() == 3 && w_idx.size(0) == B && w_idx.size(1) == s_q && w_idx.size(2) == H,
              "w_idx must be [B, s_q, H]");
  check_paged(k_idx, "k_idx", 128);
  TORCH_CHECK(k_idx.device() == q_idx.device(), "k_idx must be on q_idx's device");
  check_table(block_table, seq_lens, B, q_idx.device());
  TORCH_CHECK(s_q >= 1 && s_q <= 2 && (s_q * H == 64 || s_q * H == 128),
              "the indexer takes s_q in {1, 2} and s_q * H in {64, 128}");
  const c10::cuda::CUDAGuard guard(q_idx.device());
  const int64_t stride = block_table.size(1) * 64;
  auto scores = torch::empty({B, s_q, stride}, w_idx.options());
  check_launch(dsa_indexer_launch(reinterpret_cast<const gqa_bf16*>(q_idx.data_ptr()),
                                  w_idx.data_ptr<float>(),
                                  reinterpret_cast<const gqa_bf16*>(k_idx.data_ptr()),
                                  block_table.data_ptr<int>(), seq_lens.data_ptr<int>(),
                                  scores.data_ptr<float>(), stride, static_cast<int>(B),
                                  static_cast<int>(s_q), static_cast<int>(H), 64,
                                  static_cast<int>(block_table.size(1)),
                                  static_cast<int>(k_idx.size(0)), causal ? 1 : 0,
                                  at::cuda::getCurrentCUDAStream()),
               "dsa_indexer");
  return scores;
}

// scores [B, s_q, stride] fp32 -> (indices [B, s_q, k] int32, counts [B, s_q] int32).
std::vector<torch::Tensor> dsa_topk(torch::Tensor scores, torch::Tensor seq_lens, int64_t k,
                                    bool causal) {
  TORCH_CHECK(scores.is_cuda() && scores.scalar_type() == torch::kFloat32 &&
                  scores.is_contiguous() && scores.dim() == 3,
              "scores must be a contiguous fp32 CUDA tensor [B, s_q, S]");
  TORCH_CHECK(seq_lens.is_cuda() && seq_lens.scalar_type() == torch::kInt32 &&
                  seq_lens.is_contiguous() && seq_lens.dim() == 1 &&
                  seq_lens.size(0) == scores.size(0) && seq_lens.device() == scores.device(),
              "seq_lens must be a contiguous int32 CUDA tensor [B] on scores' device");
  TORCH_CHECK(k >= 1 && k <= (1 << 20), "k must be in [1, 2^20]");
  const c10::cuda::CUDAGuard guard(scores.device());
  const int64_t B = scores.size(0), s_q = scores.size(1), S = scores.size(2);
  auto opts = scores.options().dtype(torch::kInt32);
  auto indices = torch::empty({B, s_q, k}, opts);
  auto counts = torch::empty({B, s_q}, opts);
  check_launch(dsa_topk_launch(scores.data_ptr<float>(), S, seq_lens.data_ptr<int>(),
                               static_cast<int>(B), static_cast<int>(s_q), static_cast<int>(k),
                               static_cast<int>(S), causal ? 1 : 0, indices.data_ptr<int>(),
                               counts.data_ptr<int>(), at::cuda::getCurrentCUDAStream()),
               "dsa_topk");
  return {indices, counts};
}

// dsa_topk plus the selected tokens' physical cache rows through block_table
// -> (indices, counts, rows [B, s_q, k] int32, -1 padded).
std::vector<torch::Tensor> dsa_topk_rows(torch::Tensor scores, torch::Tensor seq_lens, int64_t k,
                                         bool causal, torch::Tensor block_table,
                                         int64_t num_blocks) {
  TORCH_CHECK(scores.is_cuda() && scores.scalar_type() == torch::kFloat32 &&
                  scores.is_contiguous() && scores.dim() == 3,
              "scores must be a contiguous fp32 CUDA tensor [B, s_q, S]");
  TORCH_CHECK(seq_lens.is_cuda() && seq_lens.scalar_type() == torch::kInt32 &&
                  seq_lens.is_contiguous() && seq_lens.dim() == 1 &&
                  seq_lens.size(0) == scores.size(0) && seq_lens.device() == scores.device(),
              "seq_lens must be a contiguous int32 CUDA tensor [B] on scores' device");
  TORCH_CHECK(block_table.is_cuda() && block_table.scalar_type() == torch::kInt32 &&
                  block_table.is_contiguous() && block_table.dim() == 2 &&
                  block_table.size(0) == scores.size(0) && block_table.device() == scores.device(),
              "block_table must be a contiguous int32 CUDA tensor [B, max_blocks] on scores' device");
  TORCH_CHECK(k >= 1 && k <= (1 << 20), "k must be in [1, 2^20]");
  TORCH_CHECK(num_blocks >= 1, "num_blocks must be positive");
  const c10::cuda::CUDAGuard guard(scores.device());
  const int64_t B = scores.size(0), s_q = scores.size(1), S = scores.size(2);
  const int64_t max_tokens = std::min<int64_t>(S, block_table.size(1) * 64);
  auto opts = scores.options().dtype(torch::kInt32);
  auto indices = torch::empty({B, s_q, k}, opts);
  auto counts = torch::empty({B, s_q}, opts);
  auto rows = torch::empty({B, s_q, k}, opts);
  check_launch(dsa_topk_rows_launch(scores.data_ptr<float>(), S, seq_lens.data_ptr<int>(),
                                    static_cast<int>(B), static_cast<int>(s_q),
                                    static_cast<int>(k), static_cast<int>(max_tokens),
                                    causal ? 1 : 0, block_table.data_ptr<int>(),
                                    static_cast<int>(block_table.size(1)),
                                    static_cast<int>(num_blocks), indices.data_ptr<int>(),
                                    counts.data_ptr<int>(), rows.data_ptr<int>(),
                                    at::cuda::getCurrentCUDAStream()),
               "dsa_topk_rows");
  return {indices, counts, rows};
}

// kv_cache [num_blocks, 64, 1, 576] bf16, indices [B, s_q, k] int32 ->
// pages [B * s_q * kpad / 64, 64, 1, 576] bf16, kpad = k rounded up to 64.
torch::Tensor dsa_gather(torch::Tensor kv_cache, torch::Tensor block_table, torch::Tensor indices) {
  check_paged(kv_cache, "kv_cache", 576);
  TORCH_CHECK(indices.is_cuda() && indices.scalar_type() == torch::kInt32 &&
                  indices.is_contiguous() && indices.dim() == 3 &&
                  indices.device() == kv_cache.device(),
              "indices must be a contiguous int32 CUDA tensor [B, s_q, k] on kv_cache's device");
  TORCH_CHECK(block_table.is_cuda() && block_table.scalar_type() == torch::kInt32 &&
                  block_table.is_contiguous() && block_table.dim() == 2 &&
                  block_table.size(0) == indices.size(0) &&
                  block_table.device() == kv_cache.device(),
              "block_table must be a contiguous int32 CUDA tensor [B, max_blocks]");
  const c10::cuda::CUDAGuard guard(kv_cache.device());
  const int64_t B = indices.size(0), s_q = indices.size(1), k = indices.size(2);
  const int64_t kpad = (k + 63) / 64 * 64;
  auto pages = torch::empty({B * s_q * kpad / 64, 64, 1, 576}, kv_cache.options());
  check_launch(dsa_gather_launch(reinterpret_cast<const gqa_bf16*>(kv_cache.data_ptr()),
                                 block_table.data_ptr<int>(), indices.data_ptr<int>(),
                                 static_cast<int>(B), static_cast<int>(s_q), static_cast<int>(k),
                                 static_cast<int>(block_table.size(1)),
                                 static_cast<int>(kv_cache.size(0)),
                                 reinterpret_cast<gqa_bf16*>(pages.data_ptr()),
                                 at::cuda::getCurrentCUDAStream()),
               "dsa_gather");
  return pages;
}

int64_t dsa_get_status(bool clear) { return dsa_decode_get_status(clear ? 1 : 0); }

PYBIND11_MODULE(TORCH_EXTENSION_NAME, m) {
  m.def("mla_decode", &mla_decode, "MLA latent-cache paged decode (tcgen05)", py::arg("q"),
        py::arg("kv_cache"), py::arg("block_table"), py::arg("seq_lens"),
        py::arg("softmax_scale"), py::arg("causal"), py::arg("num_splits"), py::arg("workspace"));
  m.def("mla_decode_sparse", &mla_decode_sparse,
        "MLA decode over selected tokens, rows gathered by TMA (tcgen05)", py::arg("q"),
        py::arg("kv_cache"), py::arg("block_table"), py::arg("indices"), py::arg("counts"),
        py::arg("softmax_scale"), py::arg("num_splits"), py::arg("workspace"));
  m.def("mla_decode_sparse_rows", &mla_decode_sparse_rows,
        "MLA decode over selected cache rows resolved by dsa_topk_rows (tcgen05)", py::arg("q"),
        py::arg("kv_cache"), py::arg("rows"), py::arg("counts"), py::arg("softmax_scale"),
        py::arg("num_splits"), py::arg("workspace"));
  m.def("mla_workspace_bytes", &mla_workspace_bytes, "MLA split workspace bytes");
  m.def("mla_pick_splits", &mla_pick_splits, "MLA split count heuristic");
  m.def("mla_get_status", &mla_get_status, "MLA device status word", py::arg("clear") = false);
  m.def("dsa_indexer", &dsa_indexer, "DSA lightning-indexer scores (tcgen05)", py::arg("q_idx"),
        py::arg("w_idx"), py::arg("k_idx"), py::arg("block_table"), py::arg("seq_lens"),
        py::arg("causal"));
  m.def("dsa_topk", &dsa_topk, "DSA top-k token selection", py::arg("scores"),
        py::arg("seq_lens"), py::arg("k"), py::arg("causal"));
  m.def("dsa_topk_rows", &dsa_topk_rows, "DSA top-k with the selected tokens' cache rows",
        py::arg("scores"), py::arg("seq_lens"), py::arg("k"), py::arg("causal"),
        py::arg("block_table"), py::arg("num_blocks"));
  m.def("dsa_gather", &dsa_gather, "DSA gather of the selected latent rows", py::arg("kv_cache"),
        py::arg("block_table"), py::arg("indices"));
  m.def("dsa_get_status", &dsa_get_status, "DSA device status word", py::arg("clear") = false);
  m.def("gqa_decode_v0", &gqa_decode_v0, "GQA decode v0: CUDA-core grouped scan (paged KV, bf16)");
  m.def("gqa_decode_v1", &gqa_decode_v1,
        "GQA decode v1: pipelined TMA + tensor-core scan, unsplit (paged KV, bf16)");
  m.def("gqa_decode_v2", &gqa_decode_v2, "GQA decode v2: split-KV scan + merge (paged KV, bf16)",
        py::arg("q"), py::arg("k_cache"), py::arg("v_cache"), py::arg("block_table"),
        py::arg("seq_lens"), py::arg("scale"), py::arg("num_splits") = 8);
  m.def("gqa_decode", &gqa_decode, "GQA decode, balanced (num_splits=0) or fixed splits",
        py::arg("q"), py::arg("k_cache"), py::arg("v_cache"), py::arg("block_table"),
        py::arg("seq_lens"), py::arg("scale"), py::arg("num_splits"), py::arg("workspace"),
        py::arg("check_blocks") = true, py::arg("out") = py::none());
  m.def("gqa_decode_partial", &gqa_decode_partial, "unnormalised softmax states (m, l, acc)",
        py::arg("q"), py::arg("k_cache"), py::arg("v_cache"), py::arg("block_table"),
        py::arg("seq_lens"), py::arg("scale"), py::arg("workspace"),
        py::arg("check_blocks") = true);
  m.def("gqa_decode_kvshard", &gqa_decode_kvshard,
        "KV-range sharded decode, cross-rank merge over peer memory", py::arg("q"),
        py::arg("k_cache"), py::arg("v_cache"), py::arg("block_table"), py::arg("seq_lens"),
        py::arg("scale"), py::arg("rank"), py::arg("world"), py::arg("peer_ptrs"),
        py::arg("epoch"), py::arg("workspace"), py::arg("check_blocks") = true,
        py::arg("out") = py::none());
  m.def("kvshard_buffer_bytes", &kvshard_buffer_bytes, "exchange buffer bytes per rank");
  m.def("merge_states", &merge_states, "merge per-shard softmax states into bf16 output");
  m.def("block_table_to_csr", &block_table_to_csr, "dense page table -> CSR (GPU)");
  m.def("plan_csr", &plan_csr, "balanced-schedule plan for a CSR page table");
  m.def("plan_dense", &plan_dense, "balanced-schedule plan for a dense page table");
  m.def("run_csr", &run_csr, "planned decode, CSR page table", py::arg("q"), py::arg("k_cache"),
        py::arg("v_cache"), py::arg("kv_indptr"), py::arg("kv_indices"),
        py::arg("kv_last_page_len"), py::arg("scale"), py::arg("workspace"),
        py::arg("check_blocks") = true, py::arg("out") = py::none());
  m.def("run_dense", &run_dense, "planned decode, dense page table", py::arg("q"),
        py::arg("k_cache"), py::arg("v_cache"), py::arg("block_table"), py::arg("seq_lens"),
        py::arg("scale"), py::arg("workspace"), py::arg("check_blocks") = true,
        py::arg("out") = py::none());
  m.def("workspace_bytes", &workspace_bytes, "workspace bytes for gqa_decode on this device");
  m.def("get_status", &get_status, "device status word", py::arg("clear") = false);
  m.def("pick_splits", &pick_splits, "fixed split count heuristic");
}
