/* C++ integration of libblut for the HF offload engine of block_lut (its
 * csrc/ tree: the expert dispatcher's recover-then-matmul path).
 *
 * Header-only, over the C ABI of blut.h: include it, link -lblut -lcudart.
 *
 *  - lut_moe_launch_blocklut_recover: the same signature as the engine's
 *    recover launcher (csrc/kernels/tensor_recover.hpp:31-38, called from
 *    csrc/topology/model_topology.cpp:597-618), on blut_blocklut_decompress;
 *    it returns a status where the reference prints and continues.
 *  - blut_hf::LutExpertModule: the expert module of the dispatcher
 *    (DeepSeekMoEDenseActDense, csrc/dispatcher/expert_module.cpp:22-50:
 *    down(silu(gate x) * up x) by three torch::matmul on recovered bf16
 *    weights), computed straight from the expert's BlockLUT indices by the
 *    fused LUT matmuls (blut_moe_forward with one expert), so no bf16 copy
 *    of the expert is recovered.  SetTensorsFromBlob packs the expert once
 *    (the engine's load of an expert to the GPU); forward runs per token
 *    batch.
 *
 * Errors throw std::runtime_error with blut_status_string's text, as the
 * engine's torch calls throw.
 */
#ifndef BLUT_HF_HPP_
#define BLUT_HF_HPP_

#include <cuda_runtime.h>

#include <cstddef>
#include <cstdint>
#include <cstring>
#include <stdexcept>
#include <string>
#include <vector>

#include "blut.h"

/* Replaces lut_moe_launch_blocklut_recover (csrc/kernels/tensor_recover.hpp:31-38):
 * out[i] = lut[idx[i]] * absmax[i / 128] in bf16 (absmax per 128 elements, the
 * engine's BlockLUT block). */
static inline int lut_moe_launch_blocklut_recover(uint16_t* gpu_output_tensor, const uint8_t* gpu_indices_ptr,
                                                  const uint16_t* gpu_absmax_ptr, const uint16_t* gpu_lut_ptr,
                                                  size_t num_elements, cudaStream_t tensor_stream) {
  return blut_blocklut_decompress(gpu_output_tensor, gpu_indices_ptr, gpu_absmax_ptr, gpu_lut_ptr,
                                  (int64_t)num_elements, 128, tensor_stream);
}

namespace blut_hf {

inline void check(int rc, const char* what) {
  if (rc != BLUT_OK) throw std::runtime_error(std::string("libblut ") + what + ": " + blut_status_string(rc));
}
inline void check_cuda(cudaError_t e, const char* what) {
  if (e != cudaSuccess) throw std::runtime_error(std::string(what) + ": " + cudaGetErrorString(e));
}

/* One expert's BlockLUT tensors on the GPU, as the engine's tensor index holds
 * them after a load: gate_proj and up_proj [inter][hidden], down_proj
 * [hidden][inter], each as uint8 indices and bf16 absmax per 128 elements. */
struct ExpertBlob {
  const uint8_t* gate_idx;
  const uint16_t* gate_absmax;
  const uint8_t* up_idx;
  const uint16_t* up_absmax;
  const uint8_t* down_idx;
  const uint16_t* down_absmax;
};

/* The fused expert module: y [T][hidden] = down(silu(gate x) * up x), bf16
 * in and out, fp32 accumulation.  `lut_bf16` is the tier's 256-entry table
 * (the engine's get_lut_device_for_tier); `tier` masks the indices to 8, 6
 * or 4 bits as the engine's tiers read them. */
class LutExpertModule {
 public:
  LutExpertModule(int hidden, int inter, const uint16_t* lut_bf16, int tier = 0)
      : hidden_(hidden), inter_(inter), lut_(lut_bf16) {
    std::memset(&w13_, 0, sizeof w13_);
    std::memset(&w2_, 0, sizeof w2_);
    w13_.format = w2_.format = BLUT_FMT_R8;
    w13_.bits = w2_.bits = 8;
    w13_.group = w2_.group = 128;
    w13_.tier = w2_.tier = tier;
    w13_.dtype = w2_.dtype = BLUT_BF16;
    w13_.layout = BLUT_LAYOUT_TC | BLUT_LAYOUT_PAIRED;
    w2_.layout = BLUT_LAYOUT_TC;
    w13_.rows = 2LL * inter;
    w13_.cols = hidden;
    w2_.rows = hidden;
    w2_.cols = inter;
    const int64_t b13 = blut_tiled_bytes(&w13_), b2 = blut_tiled_bytes(&w2_);
    if (b13 < 0 || b2 < 0) check(BLUT_ERR_UNSUPPORTED, "expert shape has no tiled layout");
    s13_ = (size_t)((b13 + 255) & ~255LL);
    s2_ = (size_t)((b2 + 255) & ~255LL);
  }
  LutExpertModule(const LutExpertModule&) = delete;
  LutExpertModule& operator=(const LutExpertModule&) = delete;
  ~LutExpertModule() {
    cudaFree(w_);
    cudaFree(ws_);
    cudaFree(route_);
  }

  /* Packs the expert into the tiled layout of the fused matmuls (replaces
   * the recover of SetModuleMemoryFromDiskGrouped plus SetTensorsFromBlob). */
  void SetTensorsFromBlob(const ExpertBlob& b, cudaStream_t stream) {
    const size_t n = (size_t)inter_ * hidden_;  // elements of gate (= up = down)
    if (!w_) check_cuda(cudaMalloc(&w_, s13_ + s2_), "cudaMalloc(expert)");
    void* stage = nullptr;
    check_cuda(cudaMalloc(&stage, 2 * n + 2 * (2 * n / 128)), "cudaMalloc(staging)");
    // w13 = [gate rows; up rows]: contiguous indices and absmax (n is a multiple of 128)
    uint8_t* idx13 = static_cast<uint8_t*>(stage);
    uint16_t* am13 = reinterpret_cast<uint16_t*>(idx13 + 2 * n);
    cudaError_t e = cudaMemcpyAsync(idx13, b.gate_idx, n, cudaMemcpyDeviceToDevice, stream);
    if (e == cudaSuccess) e = cudaMemcpyAsync(idx13 + n, b.up_idx, n, cudaMemcpyDeviceToDevice, stream);
    if (e == cudaSuccess) e = cudaMemcpyAsync(am13, b.gate_absmax, n / 128 * 2, cudaMemcpyDeviceToDevice, stream);
    if (e == cudaSuccess)
      e = cudaMemcpyAsync(am13 + n / 128, b.up_absmax, n / 128 * 2, cudaMemcpyDeviceToDevice, stream);
    int rc = BLUT_OK;
    if (e == cudaSuccess) {
      blut_canon c13{idx13, nullptr, lut_, nullptr, am13};
      rc = blut_pack_tiled(&w13_, &c13, w_, stream);
      if (rc == BLUT_OK) {
        blut_canon c2{b.down_idx, nullptr, lut_, nullptr, b.down_absmax};
        rc = blut_pack_tiled(&w2_, &c2, static_cast<uint8_t*>(w_) + s13_, stream);
      }
    }
    const cudaError_t es = cudaStreamSynchronize(stream);  // the staging buffer goes away below
    cudaFree(stage);
    check_cuda(e, "copy expert");
    check(rc, "pack expert");
    check_cuda(es, "pack");
  }

  /* y [tokens][hidden] = down(silu(gate x) * up x); x and y bf16 on the device. */
  void forward(const void* x_bf16, int tokens, void* y_bf16, cudaStream_t stream) {
    if (!w_) check(BLUT_ERR_INVALID, "forward before SetTensorsFromBlob");
    if (tokens <= 0) return;
    if (tokens > cap_) grow(tokens, stream);
    blut_moe_args a;
    std::memset(&a, 0, sizeof a);
    a.num_tokens = tokens;
    a.hidden = hidden_;
    a.inter = inter_;
    a.num_experts = 1;
    a.top_k = 1;
    a.dtype = BLUT_BF16;
    a.w13 = w13_;
    a.w2 = w2_;
    a.w13_tiled = w_;
    a.w2_tiled = static_cast<uint8_t*>(w_) + s13_;
    a.w13_stride = (int64_t)s13_;
    a.w2_stride = (int64_t)s2_;
    a.lut_table = lut_;
    a.x = x_bf16;
    a.topk_ids = static_cast<const int32_t*>(route_);                                          // expert 0
    a.topk_weights = reinterpret_cast<const float*>(static_cast<const int32_t*>(route_) + cap_);  // weight 1
    a.out = y_bf16;
    const size_t need = blut_moe_workspace_size(&a);
    if (need == 0) check(BLUT_ERR_INVALID, "expert forward arguments");
    if (need > ws_bytes_) {
      check_cuda(cudaStreamSynchronize(stream), "sync before workspace growth");
      cudaFree(ws_);
      ws_ = nullptr;
      check_cuda(cudaMalloc(&ws_, need), "cudaMalloc(workspace)");
      ws_bytes_ = need;
    }
    check(blut_moe_forward(&a, ws_, ws_bytes_, stream), "expert forward");
  }

  /* Device status of the last forward (a bounded wait that timed out); synchronises. */
  void check_status(cudaStream_t stream) { check(blut_moe_check_status(ws_, stream), "device status"); }

 private:
  void grow(int tokens, cudaStream_t stream) {
    check_cuda(cudaStreamSynchronize(stream), "sync before routing growth");
    cudaFree(route_);
    route_ = nullptr;
    check_cuda(cudaMalloc(&route_, (size_t)tokens * 8), "cudaMalloc(routing)");
    // [tokens] int32 ids 0, then [tokens] float weights 1.0: one expert per token, unscaled
    std::vector<int32_t> host(2 * (size_t)tokens, 0);
    const float one = 1.0f;
    for (int i = 0; i < tokens; ++i) std::memcpy(&host[(size_t)tokens + i], &one, 4);
    check_cuda(cudaMemcpy(route_, host.data(), host.size() * 4, cudaMemcpyHostToDevice), "routing");
    cap_ = tokens;
  }

  int hidden_, inter_;
  const uint16_t* lut_;
  blut_mat_desc w13_, w2_;
  size_t s13_ = 0, s2_ = 0;
  void* w_ = nullptr;      // tiled w13 then w2
  void* ws_ = nullptr;
  size_t ws_bytes_ = 0;
  void* route_ = nullptr;  // [cap] int32 zeros, then [cap] float ones
  int cap_ = 0;
};

}  // namespace blut_hf

#endif /* BLUT_HF_HPP_ */
