// Internal declarations shared by the libblut translation units.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include "../../include/blut.h"

namespace blut {

constexpr int kMaxExperts = 1024;
constexpr int kMaxSlots = 1 << 22;  // T * top_k
constexpr int kWideGroupTok = 128;  // token groups of the tcgen05 prefill regime
constexpr int kPlanTopkTokens = 256;  // above this many tokens the top-k runs as its own launch
constexpr int kDevBadExpert = 2;  // device status bit: an expert id was out of range

struct MMParams;

// Routing plan in the workspace.
struct PlanPtrs {
  int* status;
  int* meta;  // [0] groups, [1] n-tiles, [2] shared groups, [3] shared n-tiles
  int *g_expert, *g_slot0, *g_ntok, *g_nt0;
  int *nt_slot0, *nt_cnt;
  int *sg_expert, *sg_slot0, *sg_ntok, *sg_nt0;
  int* tk_slot;   // [T*k] slot of (token, j), -1 if the id was invalid
  int* slot_tok;  // [T*k] token of each slot
  int* counters;  // [kNumCounters] work-item counters of the tcgen05 launches
};

// K slices of the four matmul passes: 0 routed gate/up, 1 routed down,
// 2 shared gate/up, 3 shared down (tcgen05 passes only; 1 = no split).
struct MoESplit {
  int ks[4], bps[4], units[4];
  int64_t groups[4];  // bound on token groups of the pass
  int gtok[2];        // tokens per group: routed, shared (32, or kWideGroupTok for prefill)
  bool gemv[2];       // routed, shared passes run the small-batch GEMV instead of tcgen05
};

// Batches of at most this many tokens run the tcgen05-layout matrices
// through the small-batch GEMV (tc_gemv_kernel).  Measured on config 1
// (Qwen1.5-MoE, 24 layers): one token 529 tokens/s against 495 on the
// tcgen05 matmul; two and four tokens are faster on the tcgen05 matmul.
constexpr int kGemvMaxTokens = 1;

constexpr int kNumCounters = 4;  // routed gate/up, routed down, shared gate/up, shared down

struct MoEWs {
  int* status;
  int32_t* ids;
  float* tw;
  float* sg;
  float* logits;  // [T][E (+1)] router logits (fp32)
  PlanPtrs pp;
  uint8_t *xf, *af, *xfs, *afs;
  float *y, *ys;               // expert outputs, ks[1] / ks[3] slices
  int64_t y_sstride, ys_sstride;
  float *part_r, *part_s;      // gate/up partial sums of split K
  int64_t ntmax, sntmax;
  MoESplit split;
  // single-token path (blut_tok1.cuh); set when tok1_applies
  bool tok1;
  int t1_ks[4], t1_bps[4];     // K slices of routed gate/up, routed down, shared gate/up, shared down
  int* t1_groups;              // [0] routed groups, [1 + g] expert of group g
  float* t1_gw;                // [g] routing weight
  int* t1_cnt;                 // gate/up counters [top_k][units] + [shared units], then down [hidden / 128]
  int t1_ncnt_pair, t1_ncnt;
  float *t1_part_r, *t1_part_s;  // gate/up slices [group][unit][ks][2][128]
  uint16_t *t1_act_r, *t1_act_s; // SiLU * up rows [group][inter]
  float *t1_y_r, *t1_y_s;        // down slices [ks][group][hidden]
};

// The single-token path applies: one token, every projection in the TC layout.
bool tok1_applies(const blut_moe_args& a, const MoESplit& s);

int num_sms();
// Limit of the tcgen05 kernels' bounded device-side waits, in nanoseconds
// (2 s unless blut_debug_set_wait_limit changed it).
uint64_t wait_limit_ns();
// Device address of the current device's blut_moe_forward_noalloc scratch.
int noalloc_scratch(void** out);
// Progressive bit-plane storage of Format R indices (blut_bitplane.cu).
int64_t bitplane_bytes(int64_t n, int tier);
int bitplane_pack(void* planes, const void* idx, int64_t n, cudaStream_t stream);
int bitplane_recover(void* out, const void* planes, const void* absmax, const void* table, int64_t n, int tier,
                     int bs, cudaStream_t stream);
// Consumer warps (units) per work item of the mma.sync matmul for the expected
// number of token groups.
int choose_units_per_item(double est_groups, int units, int sms);
// Error check after a launch stage (synchronises with BLUT_DEBUG_SYNC set).
int stage_done(const char* stage, cudaStream_t s);
size_t moe_workspace(const blut_moe_args& a, uint8_t* base, MoEWs* ws);
void moe_split(const blut_moe_args& a, MoESplit& s);
int validate_moe(const blut_moe_args& a);
int moe_forward(const blut_moe_args& a, void* workspace, size_t ws_bytes, cudaStream_t stream);
int moe_launch_count(const blut_moe_args& a);
int router(const void* x, const void* w, int T, int H, int E, int K, int renorm, int has_sg, int dtype,
           int32_t* ids, float* tw, float* sg, float* logits, cudaStream_t stream);

// LUT matmul dispatch over formats (blut_mm_inst_*.cu).
cudaError_t launch_lut_mm(const blut_mat_desc& d, bool pair, const MMParams& p, int sms, cudaStream_t stream);
cudaError_t launch_mm_b4(int group, bool pair, const MMParams& p, int sms, cudaStream_t stream);
cudaError_t launch_mm_b3(int group, bool pair, const MMParams& p, int sms, cudaStream_t stream);
cudaError_t launch_mm_b2(int group, bool pair, const MMParams& p, int sms, cudaStream_t stream);
cudaError_t launch_mm_nested(int group, bool pair, const MMParams& p, int sms, cudaStream_t stream);
cudaError_t launch_mm_r8(bool pair, const MMParams& p, int sms, cudaStream_t stream);
cudaError_t launch_mm_dense(bool bf16, bool pair, const MMParams& p, int sms, cudaStream_t stream);

bool mm_planes(const blut_mat_desc& d, bool pair, MMParams& p);

// tcgen05 matmul for BLUT_LAYOUT_TC matrices (blut_tc_inst.cu).
struct TcParams;
bool tc_planes(const blut_mat_desc& d, bool pair, TcParams& p);
cudaError_t launch_tc_mm(const blut_mat_desc& d, const TcParams& p, int group_tokens, int sms, cudaStream_t stream);
int tc_gemv_blocks(const blut_mat_desc& d);
int dequant_tiled_tc(const blut_mat_desc& d, const void* tiled, const void* r8_table, void* out,
                     cudaStream_t stream);
int dequant_tiled(const blut_mat_desc& d, const void* tiled, const void* table, void* out, cudaStream_t stream);

// Single-matrix matmul y = W x on either path (blut_matmul.cu).
size_t matmul_workspace(const blut_mat_desc& d, int64_t m);
int matmul(const blut_mat_desc& d, const void* w, const void* lut_table, const void* x, int64_t m, void* y,
           int y_f32, void* workspace, size_t ws_bytes, cudaStream_t stream);
int matmul_launch_count(const blut_mat_desc& d, int64_t m);

// Canonical-layout kernels (blut_pack.cu, blut_gemv.cu).
int dequant(const blut_mat_desc& d, const blut_canon& c, void* out, cudaStream_t stream);
int pack_tiled(const blut_mat_desc& d, const blut_canon& c, void* tiled, cudaStream_t stream);
int encode(const blut_mat_desc& d, const float* w, void* codes, void* tables, void* codes2, void* tables2,
           cudaStream_t stream);
int encode_r(const void* w, int64_t n, const void* cb, int block_size, void* idx, void* absmax, bool f32,
             cudaStream_t stream);
int blocklut_decompress(void* out, const void* idx, const void* absmax, const void* cb, int64_t num_experts,
                        int64_t elems, int64_t blocks_per_expert, int block_size, cudaStream_t stream);
int lut_recover(void* out, const void* idx, const void* lut, int64_t n, cudaStream_t stream);
int lut_gemv(const void* x, const void* idx, const void* cb, const void* absmax, void* y, int64_t m, int64_t k,
             int64_t nb, cudaStream_t stream);

}  // namespace blut
