/*
 * blut.h -- C ABI of libblut.so, the B200 (sm_100a) LUT-dequantised MoE
 * expert forward of block_lut.
 *
 * Every entry point takes plain device pointers, sizes and a cudaStream_t
 * (passed as void*), launches asynchronously on that stream, never allocates,
 * never synchronises the device and returns an int status (0 = ok, < 0 =
 * error, see blut_status_string); the exceptions are the set-up and
 * diagnostic calls that say so (the expert-parallel window set-up, the
 * status reads).  No C++ exceptions cross this boundary.
 *
 * Each declaration names the reference interface it replaces
 * (paths inside the hu-jinzhao/block_lut project).
 */
#ifndef BLUT_H_
#define BLUT_H_

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define BLUT_API __attribute__((visibility("default")))
#else
#define BLUT_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

/* ---------------------------------------------------------------- status -- */
enum {
  BLUT_OK = 0,
  BLUT_ERR_INVALID = -1,     /* null pointer, bad size or misaligned buffer   */
  BLUT_ERR_UNSUPPORTED = -2, /* format / shape combination not implemented    */
  BLUT_ERR_WORKSPACE = -3,   /* caller workspace smaller than required        */
  BLUT_ERR_LAUNCH = -4,      /* a kernel launch failed                        */
  BLUT_ERR_TIMEOUT = -5,     /* a device-side wait gave up (device status)    */
  BLUT_ERR_CUDA = -6         /* another CUDA runtime error                    */
};

/* Human-readable text of a status code (static storage). */
BLUT_API const char* blut_status_string(int status);

/* ---------------------------------------------------------------- formats -- */
enum {
  BLUT_FMT_R8 = 1,     /* reference BlockLUT: uint8 index per weight, one global
                          256-entry bf16 table, bf16 absmax per `group` flat
                          elements (vllm_lut/quant_method.py:117-163)            */
  BLUT_FMT_B = 2,      /* packed b-bit codes (b = 2, 3, 4), one sorted fp16
                          table of 2^b entries per (row, block of `group` along K) */
  BLUT_FMT_NESTED = 3, /* NestedLUT 2+2: 2-bit coarse code into a 4-entry fp16
                          table per block plus a 2-bit residual code into a 4x4
                          refinement table; w = fp16(coarse[c] + refine[c][r])   */
  BLUT_FMT_DENSE = 4   /* plain fp16 / bf16 weights (shared expert)             */
};

enum { BLUT_F16 = 0, BLUT_BF16 = 1, BLUT_F32 = 2 };

/* Tiled layout flags (blut_mat_desc.layout).
 *  BLUT_LAYOUT_PAIRED  row tile t of the first half (gate) and tile t of the
 *                      second half (up) are stored next to each other.
 *  BLUT_LAYOUT_TC      128-row tiles with one row's codes and tables per
 *                      thread, for the tcgen05 (tensor memory) matmuls and
 *                      the single-token GEMV; every format (rows % 128, 256
 *                      paired; cols % 64, % 128 for g128 and FMT_R8).
 *                      Without it: 16-row tiles in mma.sync fragment order,
 *                      every format (cols % 128). */
enum { BLUT_LAYOUT_PAIRED = 1, BLUT_LAYOUT_TC = 2 };

/* Description of one weight matrix W [rows, cols] (y = W x, cols = K). */
typedef struct {
  int32_t format; /* BLUT_FMT_*                                                  */
  int32_t bits;   /* FMT_B: 2, 3, 4.  FMT_R8: 8.  FMT_NESTED: 4.  DENSE: 16      */
  int32_t group;  /* FMT_B / NESTED: table block along K (32, 64, 128).
                     FMT_R8: absmax block in flat elements (the reference: 128)  */
  int32_t tier;   /* FMT_R8: 0 full table (idx), 1 mapped64 (idx & 0x3F),
                     2 mapped16 (idx & 0x0F) -- runtime/model_offload.py:751-758.
                     FMT_NESTED: 0 full (coarse + residual), 1 coarse only       */
  int32_t dtype;  /* compute dtype of weights and activations: BLUT_F16 / BF16.
                     FMT_R8 computes in bf16, FMT_B / NESTED in fp16             */
  int32_t layout; /* tiled layout flags (BLUT_LAYOUT_*); blut_moe_forward needs
                     BLUT_LAYOUT_PAIRED on w13 / s13 and the same
                     BLUT_LAYOUT_TC choice on w13 and w2 (and on s13, s2)     */
  int64_t rows;   /* N: output features                                        */
  int64_t cols;   /* K: input features                                         */
} blut_mat_desc;

/* Canonical (checkpoint) layout of one matrix.  Unused pointers are NULL.
 *  FMT_R8    codes  u8   [rows*cols] (row-major, as the reference's uint8 params)
 *            tables bf16 [256]       (the tier's 256-entry table)
 *            scales bf16 [ceil(rows*cols/group)] (flat absmax blocks)
 *  FMT_B     codes  u8   [rows][cols*bits/8]: element k at bits [k*b, k*b+b)
 *                        of the row's little-endian bit stream (element 0 in
 *                        the low bits, as the reference's bit-plane packing)
 *            tables f16  [rows][cols/group][2^bits] (sorted)
 *  FMT_NESTED codes u8   [rows][cols/4] coarse codes (2-bit stream)
 *            codes2 u8   [rows][cols/4] residual codes (2-bit stream)
 *            tables f16  [rows][cols/group][4]  coarse tables
 *            tables2 f16 [rows][cols/group][16] refinement tables (refine[c*4+r])
 *  FMT_DENSE codes  f16/bf16 [rows][cols]                                     */
typedef struct {
  const void* codes;
  const void* codes2;
  const void* tables;
  const void* tables2;
  const void* scales;
} blut_canon;

/* ------------------------------------------------------------ dequantise -- */

/* Dequantise one matrix from the canonical layout into out [rows][cols]
 * (bf16 for FMT_R8, fp16 for FMT_B / NESTED).  Bit-exact pure table lookup:
 *   R8:     bf16(f32(table[tier(idx)]) * f32(absmax[min(i / group, nb - 1)]))
 *   B:      tables[row][k / group][code]
 *   NESTED: fp16(f32(coarse[c]) + f32(refine[c][r]))  (or coarse[c], tier 1)
 * Replaces vllm_lut/quantizer.py:449-477 (decompress_blocklut),
 * vllm_lut/quant_method.py:281-308 (_decompress_one / _batch_decompress). */
BLUT_API int blut_dequant(const blut_mat_desc* desc, const blut_canon* src, void* out, void* stream);

/* Reference-shaped BlockLUT decompress: out[i] = bf16(cb[idx[i]] * absmax[i / block_size]).
 * Replaces launch_blocklut_decompress (vllm_lut/cuda/lut_decompress_kernel.cu:125-154)
 * and lut_moe_launch_blocklut_recover (csrc/kernels/tensor_recover.hpp:31-38),
 * without their device synchronisation. */
BLUT_API int blut_blocklut_decompress(void* out_bf16, const void* idx_u8, const void* absmax_bf16,
                             const void* codebook_bf16, int64_t n, int32_t block_size,
                             void* stream);

/* Batched per-expert decompress with per-expert absmax blocks.
 * Replaces launch_batch_blocklut_decompress (lut_decompress_kernel.cu:156-180),
 * which is limited to 1024 elements per expert; this one is not. */
BLUT_API int blut_batch_blocklut_decompress(void* out_bf16, const void* idx_u8, const void* absmax_bf16,
                                   const void* codebook_bf16, int64_t num_experts,
                                   int64_t elements_per_expert, int64_t blocks_per_expert,
                                   int32_t block_size, void* stream);

/* Plain LUT recover out[i] = lut[idx[i]] (no scale).
 * Replaces lut_moe_launch_lut_recover (csrc/kernels/tensor_recover.hpp:23-29). */
BLUT_API int blut_lut_recover(void* out_u16, const void* idx_u8, const void* lut_u16, int64_t n, void* stream);

/* ------------------------------------------ progressive bit-plane tiers -- */

/* Progressive bit-plane storage of n Format R indices (n % 4 == 0), as
 * runtime/model_offload.py:751-758 writes it: one buffer of n bytes holding
 *   low4  [n/2]  byte q: element 2q in bits 0-3, element 2q+1 in bits 4-7
 *   mid2  [n/4]  byte q: bits 4-5 of element 4q+j in bits 2j..2j+1
 *   high2 [n/4]  byte q: bits 6-7 of element 4q+j in bits 2j..2j+1
 * A tier reads a prefix of it (csrc/tensor_engine/tensor_engine.cpp:505-509):
 * tier 2 the low section, tier 1 low + mid, tier 0 everything. */

/* Bytes of the buffer that `tier` reads: n/2, 3n/4 or n; BLUT_ERR_INVALID
 * when n <= 0, n % 4 != 0 or tier is not 0, 1, 2. */
BLUT_API int64_t blut_bitplane_bytes(int64_t n, int32_t tier);

/* Write the bit-plane buffer planes [n] of idx [n] on the GPU.
 * Replaces the host packing of runtime/model_offload.py:751-758. */
BLUT_API int blut_bitplane_pack(void* planes_u8, const void* idx_u8, int64_t n, void* stream);

/* One pass from a tier's sections to bf16:
 *   out[i] = bf16(table[index(i)] * absmax[min(i / block_size, nb - 1)])
 * with index = low | mid << 4 | high << 6 over the sections the tier reads
 * (idx & 0x0F, idx & 0x3F, idx). Only the first blut_bitplane_bytes(n, tier)
 * bytes of planes are read, and only the first 16 / 64 / 256 entries of table
 * (the tier's table: mapped16, mapped64, full).
 * Replaces, for one tensor of a tier, lut_moe_launch_unpack_4bit
 * (csrc/kernels/tensor_recover.cu:166-192), the host 6-bit unpack
 * (csrc/tensor_engine/tensor_engine.cpp:535-547) and the
 * lut_moe_launch_blocklut_recover that follows them
 * (csrc/topology/model_topology.cpp:597-618). */
BLUT_API int blut_bitplane_recover(void* out_bf16, const void* planes_u8, const void* absmax_bf16,
                                   const void* table_bf16, int64_t n, int32_t tier, int32_t block_size,
                                   void* stream);

/* ------------------------------------------------------- tiled layout ---- */

/* Bytes of the tiled device layout of one matrix (16-row tiles x 128-column
 * chunks, codes and tables in MMA-fragment order, 256-byte aligned).  The
 * layout needs rows % 16 == 0 and cols % 128 == 0; returns < 0 otherwise. */
BLUT_API int64_t blut_tiled_bytes(const blut_mat_desc* desc);

/* Repack one matrix from the canonical layout into the tiled layout
 * (load time; the tiled buffer is what blut_moe_forward streams). */
BLUT_API int blut_pack_tiled(const blut_mat_desc* desc, const blut_canon* src, void* tiled, void* stream);

/* Dense [rows][cols] matrix rebuilt from the tiled layout through the same
 * fragment lookups the MoE kernels use (bf16 for FMT_R8, else fp16); equal
 * bit for bit to blut_dequant of the canonical tensors.  Diagnostic entry
 * point with no counterpart in the reference; lut_table is FMT_R8's table. */
BLUT_API int blut_dequant_tiled(const blut_mat_desc* desc, const void* tiled, const void* lut_table, void* out,
                                void* stream);

/* --------------------------------------------------- single-matrix matmul -- */

/* y = W x for one matrix in the tiled layout: x [m][cols] and y [m][rows]
 * in desc->dtype (fp32 when y_f32 != 0), 1 <= m <= 2^20, cols % 128 == 0,
 * desc->layout without BLUT_LAYOUT_PAIRED.  Runs on the tcgen05 matmul for
 * BLUT_LAYOUT_TC matrices and on the mma.sync matmul otherwise, fp32
 * accumulation; lut_table is FMT_R8's table (NULL otherwise).  Three launches
 * on `stream`, no allocation, no synchronisation; the workspace (256-byte
 * aligned, blut_matmul_workspace_size bytes) holds the status word that
 * blut_moe_check_status reads.  Replaces the reference's single-matrix LUT
 * GEMV lut_gemv (vllm_lut/cuda_lut_gemv.py:153-169) and fused_lut_gemv
 * (vllm_lut/fused_kernel.py:13-46), for every format and token count. */
BLUT_API size_t blut_matmul_workspace_size(const blut_mat_desc* desc, int64_t m);
BLUT_API int blut_matmul(const blut_mat_desc* desc, const void* w_tiled, const void* lut_table, const void* x,
                         int64_t m, void* y, int32_t y_f32, void* workspace, size_t workspace_bytes,
                         void* stream);
/* Kernel launches one blut_matmul call makes (< 0 for invalid arguments). */
BLUT_API int blut_matmul_launch_count(const blut_mat_desc* desc, int64_t m);

/* ---------------------------------------------------------------- encode -- */

/* Format B / NestedLUT encoder: per (row, block) 1-D Lloyd k-means (10
 * iterations, uniform-grid initialisation, float32 means), fp16 sorted
 * tables, nearest-entry codes; bit-identical to the CPU restatement.
 * w: f32 [rows][cols]; writes the canonical layout (codes, tables[, codes2,
 * tables2]).  New format: the reference's per-block Lloyd is
 * vllm_lut/quantizer.py:120-178, its assignment quantizer.py:292-296. */
BLUT_API int blut_encode(const blut_mat_desc* desc, const float* w, void* codes, void* tables,
                void* codes2, void* tables2, void* stream);

/* Reference BlockLUT encoder on bf16 input (block absmax, bf16 normalisation,
 * first-index argmin over the 256-entry table).  Bit-exact with
 * LUTQuantizer.quantize (vllm_lut/quantizer.py:243-306), the encoder of
 * convert_checkpoint.py's quantize_weight.  block_size: 32 .. 256, a
 * multiple of 32. */
BLUT_API int blut_encode_r(const void* w_bf16, int64_t n, const void* codebook_bf16, int32_t block_size,
                  void* idx_u8, void* absmax_bf16, void* stream);

/* The other reference BlockLUT encoder, fast_encode.encode_lut
 * (vllm_lut/fast_encode.py:22-102,172-180, used by convert_model.py): absmax
 * floored at 1e-10 in fp32, the normalised value w / absmax kept in fp32,
 * nearest entry of an fp32 codebook (first index on ties); absmax stored
 * rounded to bf16.  Near codebook midpoints its indices can differ from
 * blut_encode_r's.  The reference kernel builds with fast math; this one
 * divides exactly, which is what the reference's own check of that kernel
 * compares against (fast_encode.py:205-221). */
BLUT_API int blut_encode_lut_f32(const void* w_bf16, int64_t n, const float* codebook_f32, int32_t block_size,
                        void* idx_u8, void* absmax_bf16, void* stream);

/* ------------------------------------------------------------------ GEMV -- */

/* Fused Format-R LUT-dequant GEMV on the canonical layout (one token):
 *   y[r] = sum_c x[c] * cb[idx[r, c]] * absmax[min((r*K + c) / 128, nb - 1)]
 * fp32 accumulation, bf16 in/out.  Replaces lut_gemv
 * (vllm_lut/cuda_lut_gemv.py:23-81,153-169) without its per-call device
 * synchronisation. */
BLUT_API int blut_lut_gemv(const void* x_bf16, const void* idx_u8, const void* codebook_bf16,
                  const void* absmax_bf16, void* y_bf16, int64_t m, int64_t k, int64_t num_blocks,
                  void* stream);

/* ---------------------------------------------------------------- router -- */

/* Fused router: logits = x W_r^T (fp32 accumulation), softmax (fp32), top-k
 * (descending, lowest expert index on ties), optional renormalisation, and,
 * when has_shared_gate, sigmoid(x . W_r[num_experts]) for the shared expert.
 * x [T][hidden], w_router [num_experts (+1)][hidden] in `dtype`; logits is a
 * caller buffer of T * (num_experts + has_shared_gate) floats that receives
 * the router logits.  Replaces vllm_lut/moe_layer.py:358-376 (_routing) and
 * customized/qwen.py:44-54,99. */
BLUT_API int blut_router(const void* x, const void* w_router, int32_t num_tokens, int32_t hidden,
                int32_t num_experts, int32_t top_k, int32_t renorm, int32_t has_shared_gate,
                int32_t dtype, int32_t* topk_ids, float* topk_weights, float* shared_gate,
                float* logits, void* stream);

/* ------------------------------------------------------------------- MoE -- */

typedef struct {
  int32_t num_tokens;  /* T                                                     */
  int32_t hidden;      /* H                                                     */
  int32_t inter;       /* I (per routed expert)                                 */
  int32_t num_experts; /* E                                                     */
  int32_t top_k;       /* k, at most 32; at most E when the library routes
                          (router_w), any with the caller's topk_ids       */
  int32_t dtype;       /* activation / output dtype: BLUT_F16 or BLUT_BF16      */
  blut_mat_desc w13;   /* per expert [2I, H]: rows 0..I-1 gate, I..2I-1 up      */
  blut_mat_desc w2;    /* per expert [H, I]                                     */
  const void* w13_tiled;  /* E matrices in the tiled layout, stride below       */
  const void* w2_tiled;
  int64_t w13_stride;     /* bytes between experts (>= blut_tiled_bytes(&w13))  */
  int64_t w2_stride;
  const void* lut_table;  /* FMT_R8: bf16 [256] tier table; NULL otherwise      */
  const void* x;          /* [T][H]                                             */
  const int32_t* topk_ids;  /* [T][k]; NULL: route with router_w.  An id of -1
                               marks an empty slot (skipped; expert parallelism
                               uses it for experts owned by other ranks); other
                               ids outside [0, E) are skipped and reported by
                               blut_moe_check_status                           */
  const float* topk_weights;/* [T][k]                                           */
  const void* router_w;     /* [E (+1 with shared gate)][H], used when topk_ids==NULL */
  int32_t renorm;           /* renormalise the top-k weights (router only)     */
  int32_t shared_inter;     /* I_s of the shared expert; 0 = none              */
  int32_t shared_gate_mode; /* 0: shared output added unscaled; 1: scaled by
                               sigmoid(x . g_s), g_s = shared_gate_w or router row E */
  int32_t reserved;
  blut_mat_desc s13;        /* shared expert [2 I_s, H]                         */
  blut_mat_desc s2;         /* shared expert [H, I_s]                           */
  const void* s13_tiled;
  const void* s2_tiled;
  const void* shared_gate_w;/* [H] or NULL (then router row E when routing)   */
  void* out;                /* [T][H]                                           */
  void* const* prof_events; /* NULL, or 4 cudaEvent_t recorded on the stream
                               before/after the routed gate/up launch and
                               before/after the routed down launch (timing);
                               on the single-token path those launches also
                               carry the shared expert                        */
  int32_t out_f32;          /* 1: out is float32 [T][H] (unrounded partial sums,
                               used by expert parallelism); 0: out is `dtype` */
  int32_t expected_slots;   /* 0: every slot of topk_ids may name a local
                               expert.  > 0: how many of the T*k slots the
                               caller expects to be non-empty (expert
                               parallelism: the received rows' slots owned by
                               this rank, about T*k*E_local/E_global).  Only
                               the choice of token grouping and K split uses
                               it; results never depend on it. */
} blut_moe_args;

/* Workspace bytes blut_moe_forward needs for these arguments (0 on error). */
BLUT_API size_t blut_moe_workspace_size(const blut_moe_args* args);

/* One MoE layer of routed LUT experts (+ optional shared expert):
 *   out[t] = sum_j w[t,j] * W2_e(silu(W1_e x_t) * W3_e x_t)  (+ g_t * shared(x_t))
 * with e = topk_ids[t, j]; every active (token, expert) pair of the layer runs
 * in one launch per stage (router, plan, gate/up+SiLU*up, down, combine).
 * Replaces LUTFusedMoEMethod.apply (vllm_lut/quant_method.py:230-279) and
 * fused_lut_moe (vllm_lut/fast_moe.py:30-80).  Any T*k up to 2^22 slots
 * (decode and prefill).  Work is ordered after earlier work on `stream` and
 * the call returns with all of it ordered before later work on `stream`;
 * the shared expert's passes run on a library-owned side stream (one per
 * device and host thread, made by the first call that is not inside a stream
 * capture) forked from and joined back into `stream` with events, so the
 * call can be captured into a CUDA graph. */
BLUT_API int blut_moe_forward(const blut_moe_args* args, void* workspace, size_t workspace_bytes,
                     void* stream);

/* blut_moe_forward without a caller workspace, for callers that cannot
 * allocate device memory when they call (a plugin that a host framework hands
 * only its input and output pointers, a serving loop that must not call
 * cudaMalloc).  No counterpart in the reference.  The scratch is one
 * library-owned device array of 16 MiB per GPU, held on each GPU from the
 * library's first use there (from load time with eager module loading)
 * until the process exits; layers whose blut_moe_workspace_size exceeds
 * 16 MiB are rejected with BLUT_ERR_WORKSPACE before anything is launched.
 * The first call on a device looks the array's device address up (make it
 * before any stream capture).  Nothing is allocated and nothing
 * synchronised.  All calls on a GPU share the array, so calls that can
 * overlap on that GPU (different streams without ordering between them) race
 * and must be serialised by the caller.  The device status of the last call
 * (a bounded wait that timed out, an expert id out of range) is read with
 * blut_moe_check_status(NULL, stream). */
BLUT_API int blut_moe_forward_noalloc(const blut_moe_args* args, void* stream);

/* Read (and clear) the device-side status word of a workspace last used by
 * blut_moe_forward on `stream` (workspace NULL: the current device's
 * blut_moe_forward_noalloc scratch): synchronises the stream, returns
 * BLUT_OK, BLUT_ERR_TIMEOUT when a kernel's bounded wait gave up, or
 * BLUT_ERR_INVALID when a caller-supplied expert id was out of range.
 * Diagnostic only. */
BLUT_API int blut_moe_check_status(void* workspace, void* stream);

/* Number of this library's kernel launches one blut_moe_forward issues for
 * these arguments (used to report launch counts). */
BLUT_API int blut_moe_launch_count(const blut_moe_args* args);

/* Diagnostic, no counterpart in the reference: sets the limit, in
 * nanoseconds, of every bounded device-side wait in the tcgen05 kernels
 * launched after this call (0 restores the default of 2 s).  A wait that
 * runs out aborts its kernel cleanly and the next blut_moe_check_status
 * returns BLUT_ERR_TIMEOUT; tests use a tiny limit to exercise that path.
 * Process-wide; not for use while other threads launch. */
BLUT_API int blut_debug_set_wait_limit(uint64_t ns);

/* ------------------------------------- expert-parallel exchange (EP) ----
 * Replaces the dispatch / combine all_to_all of the reference's only
 * expert-parallel code (models/deepseek/modeling_deepseek.py:604-660: count
 * the rows per rank, exchange the counts, send each token row only to the
 * ranks owning one of its experts, return the outputs).  One process per
 * GPU; each rank owns a contiguous range of every layer's experts.  The rows
 * move by direct stores to and loads from the other GPUs' memory (NVLink),
 * with no host synchronisation, so a layer can be captured in a CUDA graph.
 *
 * Setup (once, not on the hot path; these are the entry points that
 * allocate or synchronise): every rank allocates a window of
 * blut_ep_window_bytes with blut_ep_alloc (zeroed), shares the
 * BLUT_EP_HANDLE_BYTES handle from blut_ep_ipc_handle with the other ranks
 * (out of band, e.g. torch.distributed.all_gather_object), and maps theirs
 * with blut_ep_ipc_open.  One window serves every layer of the model.
 *
 * Per layer, on every rank (with or without rows for a peer):
 *   blut_ep_dispatch  rows to their owners; returns with this rank's window
 *                     holding every source's rows (blut_ep_views: x, ids, w)
 *   blut_moe_forward  on the window's world*capacity rows with the window's
 *                     ids and weights (-1 ids are empty slots), out_f32 = 1,
 *                     out = the window's `ret` region
 *   blut_ep_combine   out[t] = sum over owners of their rows for token t
 *                     (+ shared_out[t]), one rounding
 * Waits are bounded (blut_debug_set_wait_limit); a wait that gives up makes
 * blut_ep_check_status return BLUT_ERR_TIMEOUT. */
#define BLUT_EP_MAX_RANKS 8
#define BLUT_EP_HANDLE_BYTES 64

typedef struct {
  int32_t world;    /* ranks in the exchange, 1 .. BLUT_EP_MAX_RANKS            */
  int32_t rank;     /* this rank                                               */
  int32_t capacity; /* most tokens a rank sends per layer (its largest batch)  */
  int32_t hidden;   /* row length, a multiple of 8                             */
  int32_t top_k;    /* experts per token, 1 .. 64                              */
  int32_t dtype;    /* BLUT_F16 / BLUT_BF16 of the rows                        */
  void* windows[BLUT_EP_MAX_RANKS]; /* every rank's window as mapped in this
                                       process (windows[rank]: the own one)    */
} blut_ep_desc;

/* Window bytes for these sizes, 0 if a size is out of range. */
BLUT_API size_t blut_ep_window_bytes(int world, int capacity, int hidden, int top_k);
/* cudaMalloc + zero fill (synchronises the device). */
BLUT_API int blut_ep_alloc(size_t bytes, void** ptr);
BLUT_API int blut_ep_free(void* ptr);
/* The window's IPC handle (BLUT_EP_HANDLE_BYTES bytes), and mapping /
 * unmapping another process's window by its handle. */
BLUT_API int blut_ep_ipc_handle(const void* window, void* handle);
BLUT_API int blut_ep_ipc_open(const void* handle, void** ptr);
BLUT_API int blut_ep_ipc_close(void* ptr);
/* Device pointers into the own window: received rows x [world*capacity,
 * hidden] (dtype), their local expert ids and weights [world*capacity,
 * top_k], and the expert outputs region ret [world*capacity, hidden] (fp32)
 * that blut_moe_forward writes.  Any of them may be NULL. */
BLUT_API int blut_ep_views(const blut_ep_desc* d, void** x, int32_t** ids, float** w, float** ret);
/* Sends this rank's num_tokens rows (x [T, hidden], global expert ids and
 * weights [T, top_k]) to the ranks owning their experts: owner[e] = rank of
 * expert e, local[e] = its index on that rank (device int32 [num_experts]). */
BLUT_API int blut_ep_dispatch(const blut_ep_desc* d, const void* x, const int32_t* topk_ids,
                              const float* topk_weights, int num_tokens, const int32_t* owner,
                              const int32_t* local, int num_experts, void* stream);
/* out [T, hidden] (dtype, or fp32 with out_f32) = the sum of the owners'
 * output rows for each of this rank's tokens, plus shared_out [T, hidden]
 * fp32 when not NULL. */
BLUT_API int blut_ep_combine(const blut_ep_desc* d, int num_tokens, const float* shared_out, void* out,
                             int out_f32, void* stream);
/* Synchronises the stream, returns (and clears) BLUT_ERR_TIMEOUT if a wait of
 * this rank's exchanges gave up. */
BLUT_API int blut_ep_check_status(const blut_ep_desc* d, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* BLUT_H_ */
