// extern "C" entry points of libblut.so (declared in include/blut.h).
#include "blut_common.cuh"
#include "blut_internal.h"
#include "blut_mm.cuh"

#include <atomic>

using namespace blut;

static inline cudaStream_t S(void* s) { return reinterpret_cast<cudaStream_t>(s); }

// Process-wide limit of the bounded device waits (blut_debug_set_wait_limit).
static std::atomic<uint64_t> g_wait_limit_ns{kWaitLimitNs};
uint64_t blut::wait_limit_ns() { return g_wait_limit_ns.load(std::memory_order_relaxed); }

extern "C" {

const char* blut_status_string(int status) {
  switch (status) {
    case BLUT_OK: return "ok";
    case BLUT_ERR_INVALID: return "invalid argument (null pointer, size or alignment)";
    case BLUT_ERR_UNSUPPORTED: return "unsupported format or shape";
    case BLUT_ERR_WORKSPACE: return "workspace too small";
    case BLUT_ERR_LAUNCH: return "kernel launch failed";
    case BLUT_ERR_TIMEOUT: return "a device-side wait timed out";
    case BLUT_ERR_CUDA: return "CUDA runtime error";
    default: return "unknown status";
  }
}

int blut_debug_set_wait_limit(uint64_t ns) {
  g_wait_limit_ns.store(ns ? ns : kWaitLimitNs, std::memory_order_relaxed);
  return BLUT_OK;
}

int blut_dequant(const blut_mat_desc* desc, const blut_canon* src, void* out, void* stream) {
  if (!desc || !src) return BLUT_ERR_INVALID;
  return dequant(*desc, *src, out, S(stream));
}

int blut_blocklut_decompress(void* out_bf16, const void* idx_u8, const void* absmax_bf16, const void* codebook_bf16,
                             int64_t n, int32_t block_size, void* stream) {
  if (n <= 0 || block_size <= 0) return BLUT_ERR_INVALID;
  const int64_t nb = (n + block_size - 1) / block_size;
  return blocklut_decompress(out_bf16, idx_u8, absmax_bf16, codebook_bf16, 1, n, nb, block_size, S(stream));
}

int blut_batch_blocklut_decompress(void* out_bf16, const void* idx_u8, const void* absmax_bf16,
                                   const void* codebook_bf16, int64_t num_experts, int64_t elements_per_expert,
                                   int64_t blocks_per_expert, int32_t block_size, void* stream) {
  return blocklut_decompress(out_bf16, idx_u8, absmax_bf16, codebook_bf16, num_experts, elements_per_expert,
                             blocks_per_expert, block_size, S(stream));
}

int blut_lut_recover(void* out_u16, const void* idx_u8, const void* lut_u16, int64_t n, void* stream) {
  return lut_recover(out_u16, idx_u8, lut_u16, n, S(stream));
}

int64_t blut_bitplane_bytes(int64_t n, int32_t tier) { return bitplane_bytes(n, tier); }

int blut_bitplane_pack(void* planes_u8, const void* idx_u8, int64_t n, void* stream) {
  return bitplane_pack(planes_u8, idx_u8, n, S(stream));
}

int blut_bitplane_recover(void* out_bf16, const void* planes_u8, const void* absmax_bf16, const void* table_bf16,
                          int64_t n, int32_t tier, int32_t block_size, void* stream) {
  return bitplane_recover(out_bf16, planes_u8, absmax_bf16, table_bf16, n, tier, block_size, S(stream));
}

int64_t blut_tiled_bytes(const blut_mat_desc* desc) {
  TiledLayout L;
  if (!desc || !make_layout(*desc, L)) return BLUT_ERR_UNSUPPORTED;
  return L.total;
}

int blut_pack_tiled(const blut_mat_desc* desc, const blut_canon* src, void* tiled, void* stream) {
  if (!desc || !src) return BLUT_ERR_INVALID;
  return pack_tiled(*desc, *src, tiled, S(stream));
}

int blut_dequant_tiled(const blut_mat_desc* desc, const void* tiled, const void* lut_table, void* out,
                       void* stream) {
  if (!desc) return BLUT_ERR_INVALID;
  return dequant_tiled(*desc, tiled, lut_table, out, S(stream));
}

int blut_encode(const blut_mat_desc* desc, const float* w, void* codes, void* tables, void* codes2, void* tables2,
                void* stream) {
  if (!desc) return BLUT_ERR_INVALID;
  return encode(*desc, w, codes, tables, codes2, tables2, S(stream));
}

int blut_encode_r(const void* w_bf16, int64_t n, const void* codebook_bf16, int32_t block_size, void* idx_u8,
                  void* absmax_bf16, void* stream) {
  return encode_r(w_bf16, n, codebook_bf16, block_size, idx_u8, absmax_bf16, false, S(stream));
}

int blut_encode_lut_f32(const void* w_bf16, int64_t n, const float* codebook_f32, int32_t block_size, void* idx_u8,
                        void* absmax_bf16, void* stream) {
  return encode_r(w_bf16, n, codebook_f32, block_size, idx_u8, absmax_bf16, true, S(stream));
}

int blut_lut_gemv(const void* x_bf16, const void* idx_u8, const void* codebook_bf16, const void* absmax_bf16,
                  void* y_bf16, int64_t m, int64_t k, int64_t num_blocks, void* stream) {
  return lut_gemv(x_bf16, idx_u8, codebook_bf16, absmax_bf16, y_bf16, m, k, num_blocks, S(stream));
}

int blut_router(const void* x, const void* w_router, int32_t num_tokens, int32_t hidden, int32_t num_experts,
                int32_t top_k, int32_t renorm, int32_t has_shared_gate, int32_t dtype, int32_t* topk_ids,
                float* topk_weights, float* shared_gate, float* logits, void* stream) {
  return router(x, w_router, num_tokens, hidden, num_experts, top_k, renorm, has_shared_gate, dtype, topk_ids,
                topk_weights, shared_gate, logits, S(stream));
}

size_t blut_moe_workspace_size(const blut_moe_args* args) {
  if (!args || validate_moe(*args) != BLUT_OK) return 0;
  return moe_workspace(*args, nullptr, nullptr);
}

int blut_moe_forward(const blut_moe_args* args, void* workspace, size_t workspace_bytes, void* stream) {
  if (!args) return BLUT_ERR_INVALID;
  return moe_forward(*args, workspace, workspace_bytes, S(stream));
}

int blut_moe_check_status(void* workspace, void* stream) {
  // NULL: the status of blut_moe_forward_noalloc, in its scratch on the current device
  if (!workspace && noalloc_scratch(&workspace) != BLUT_OK) return BLUT_ERR_CUDA;
  int st = 0;
  if (cudaMemcpyAsync(&st, workspace, sizeof(int), cudaMemcpyDeviceToHost, S(stream)) != cudaSuccess)
    return BLUT_ERR_CUDA;
  if (cudaStreamSynchronize(S(stream)) != cudaSuccess) return BLUT_ERR_CUDA;
  if (cudaMemsetAsync(workspace, 0, sizeof(int), S(stream)) != cudaSuccess) return BLUT_ERR_CUDA;
  if (st & kDevTimeout) return BLUT_ERR_TIMEOUT;
  if (st & kDevBadExpert) return BLUT_ERR_INVALID;
  return BLUT_OK;
}

int blut_moe_launch_count(const blut_moe_args* args) {
  if (!args) return BLUT_ERR_INVALID;
  return moe_launch_count(*args);
}

size_t blut_matmul_workspace_size(const blut_mat_desc* desc, int64_t m) {
  return desc ? matmul_workspace(*desc, m) : 0;
}

int blut_matmul(const blut_mat_desc* desc, const void* w_tiled, const void* lut_table, const void* x, int64_t m,
                void* y, int32_t y_f32, void* workspace, size_t workspace_bytes, void* stream) {
  if (!desc) return BLUT_ERR_INVALID;
  return matmul(*desc, w_tiled, lut_table, x, m, y, y_f32, workspace, workspace_bytes, S(stream));
}

int blut_matmul_launch_count(const blut_mat_desc* desc, int64_t m) {
  if (!desc) return BLUT_ERR_INVALID;
  return matmul_launch_count(*desc, m);
}

}  // extern "C"
