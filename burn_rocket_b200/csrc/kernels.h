// kernels.h — internal launch interface between the C ABI (abi.cu) and the
// kernel translation units. Not part of the public ABI.
#pragma once

#include <cstdint>
#include <cuda.h>
#include <cuda_runtime.h>

#include "../../include/rocket_b200.h"

// Internal-only output type: raw int32 accumulators of the int8 GEMM.
#define RB_DTYPE_I32 3

namespace rb {

struct GemmLaunch {
  int M, N, K;
  const int8_t* w_codes;  // Q8_0 codes [w_rows, K] (all experts of a grouped weight)
  const void* w_scales;   // Q8_0 f16 scales [K/32, w_pitch]
  int64_t w_pitch;        // Q8_0 scale row pitch
  int64_t w_rows;         // Q8_0 weight rows in memory
  const float* s_row;     // W8A8 per-row activation scale [M]
  const float* s_col;     // W8A8 per-channel weight scale [N]
  void* out;
  int ldo;
  int out_dtype;
  float out_scale;        // W8A8: 0 = unrounded output
  const int* tile_expert; // grouped GEMM table (one expert id per 128 rows), or nullptr
  int gated;              // gate/up interleaved in 32-row blocks: out = silu(gate) * up, N/2 f16 columns
  int act;                // RB_ACT_*: element-wise activation before the f16 output rounding
  uint32_t* err;
  int num_sms;
  // Launch with programmatic stream serialization: the previous kernel of the
  // stream (a cast or quantiser producing A) lets this GEMM start early; the
  // GEMM waits for it before reading anything it wrote.
  int pdl;
};

// Tile plan of one matmul. Single CTA: a (128*mh) x bn output tile per CTA.
// Pair: a 256 x bn tile per (2,1,1) cluster of CTAs running cta_group::2 UMMA,
// each CTA staging 128 rows of A and bn/2 rows of the weight.
struct GemmPlan {
  int bn;
  int mh;
  bool pair;
  int weight_rows() const { return pair ? bn / 2 : bn; }  // weight map box height
  int a_rows() const { return pair ? 128 : 128 * mh; }     // activation map box height
};
// pair96: also consider 96-column Q8_0 CTA-pair tiles (f32 output only).
GemmPlan gemm_plan(bool i8, int M, int N, int K, int num_sms, bool pair96 = false);
// Restricts gemm_plan to single-CTA or (preferably) pair tiles; returns the old policy.
int set_gemm_policy(int policy);
int gemm_policy();
int set_attention_split(int policy);
// selftest.cu: one bounded wait on an mbarrier nothing arrives on.
int launch_wait_timeout_probe(uint32_t* err, int64_t limit_ns, uint32_t* waited_us, cudaStream_t st);  // RB_ATTN_SPLIT_*; returns the previous one
// Q8_0: tmA = f16 activations [M, K] (box 64 x a_rows(), 128-B swizzle);
// tmCodes = codes [N, K] (box 64 x weight_rows()); tmScales = f16 scales
// [K/32, N] (box weight_rows() x 2); tmC = output map (box 32 rows x 128 B,
// 128-B swizzle) or nullptr for direct stores.
int launch_q8_gemm(const GemmLaunch& L, const GemmPlan& plan, const CUtensorMap& tmA,
                   const CUtensorMap& tmCodes, const CUtensorMap& tmScales, const CUtensorMap* tmC,
                   cudaStream_t stream);
// W8A8: tmA = s8 activation codes [M, K] (box 128 x 128), tmB = s8 weight
// codes [N, K] (box 128 x weight_rows()), both 128-B swizzled.
int launch_w8a8_gemm(const GemmLaunch& L, const GemmPlan& plan, const CUtensorMap& tmA,
                     const CUtensorMap& tmB, const CUtensorMap* tmC, cudaStream_t stream);
// f16 weights (the reference's fp16-resident pack): tmB = f16 weight [N, K]
// (box 64 x weight_rows(), 128-B swizzle); same tile plans as W8A8.
int launch_f16_gemm(const GemmLaunch& L, const GemmPlan& plan, const CUtensorMap& tmA,
                    const CUtensorMap& tmB, const CUtensorMap* tmC, cudaStream_t stream);
int launch_q8_dequant(const int8_t* codes, const void* scales, int N, int K, int pitch, void* out,
                      bool f16_out, cudaStream_t stream);

// Mixture-of-experts routing / dispatch / combine (moe.cu). Workspace offsets
// in int32 words.
struct MoeLayout {
  int64_t max_rows, max_tiles;
  int64_t counts, seg_start, cursor, tile_expert, row_of_slot, token_of_row, words;
};
MoeLayout moe_layout(int64_t tokens, int top_k, int experts);
int launch_moe_route(const float* logits, int64_t tokens, int experts, int top_k, int norm, int32_t* ids,
                     float* wts, cudaStream_t st);
int launch_moe_dispatch(const int32_t* ids, int64_t tokens, int top_k, int experts, const void* x, int64_t hidden,
                        int32_t* ws, void* x_perm, uint32_t* err, cudaStream_t st);
int launch_moe_combine(float* x, const void* y, int64_t hidden, const int32_t* ids, const float* wts,
                       const int32_t* ws, int64_t tokens, int top_k, int experts, cudaStream_t st);

int launch_ep_build_send(const int32_t* ids, int64_t tokens, int top_k, int experts, int ranks, const void* x,
                         int64_t hidden, int32_t* dest_counts, int32_t* dest_cursor, int32_t* send_meta,
                         int32_t* slot_pos, void* send_rows, uint32_t* err, cudaStream_t st);
int launch_gather_rows(const void* in, const int32_t* idx, int64_t n, int64_t hidden, void* out, cudaStream_t st);
int launch_ep_build_send_fixed(const int32_t* ids, int64_t tokens, int top_k, int experts, int ranks, int cap,
                               const void* x, int64_t hidden, int32_t* dest_counts, int32_t* dest_cursor,
                               int32_t* send_meta, int32_t* slot_pos, void* send_rows, uint32_t* err,
                               cudaStream_t st);
int launch_moe_combine_rows(float* x, const void* y, int64_t hidden, const int32_t* ids, const float* wts,
                            const int32_t* row_of_slot, int64_t tokens, int top_k, cudaStream_t st);

// Elementwise / codec kernels (quant.cu).
int launch_quantize_groups(const void* x, int x_dtype, int64_t m, int64_t k, int group, int8_t* codes,
                           float* scales, cudaStream_t st);
// Group-wise int8 GEMM with in-kernel group promotion (gemm_group.cu): y =
// sum over groups g of f32(a_s[m,g] * b_st[g,n]) * f32(int32 partial of group g).
int launch_i8g_gemm(int M, int N, int K, int G, const float* a_s, const float* b_st, int ldb, void* out,
                    int out_dtype, const CUtensorMap& tmA, const CUtensorMap& tmB, const CUtensorMap* tmC,
                    uint32_t* err, int num_sms, cudaStream_t stream);
int launch_cast(const void* x, int x_dtype, void* y, int y_dtype, int64_t count,
                cudaStream_t stream);
int launch_quantize_rows_i8(const void* x, int x_dtype, int64_t m, int64_t k, float in_scale,
                            int8_t* codes, float* row_scale, cudaStream_t stream);
// Q8_0 planes: codes [n, k]; scales [k/32, pitch] with pitch = round_up(n, 8)
// so every scale row starts on a 16-byte boundary (TMA).
int launch_q8_0_encode(const float* w, int64_t n, int64_t k, int64_t pitch, int8_t* codes,
                       uint16_t* scales, cudaStream_t stream);
int launch_w8a8_weight_quant(const float* w, int64_t n, int64_t k, int8_t* codes, float* scale,
                             cudaStream_t stream);
int launch_q8_0_unpack_blocks(const uint8_t* blocks, int64_t n, int64_t k, int64_t pitch,
                              int8_t* codes, uint16_t* scales, cudaStream_t stream);

// Attention (attention.cu).
// Query tiles are 128 rows, key/value tiles kAttnKeyTile rows (the TMA box
// height of the K and V maps).
constexpr int kAttnKeyTile = 128;
// Attention split-mode workspace bounds: partial-result records for up to
// kAttnMaxCtas CTAs (head width <= 128) and arrival counters for up to
// kAttnMaxUnits work units (query-slot pairs x KV heads x sequences).
constexpr int kAttnMaxCtas = 160;
constexpr int kAttnMaxUnits = 1 << 18;
constexpr size_t kAttnRecBytes = static_cast<size_t>(kAttnMaxCtas) * 4 * (128 * 128 + 2 * 128) * sizeof(float);
constexpr size_t kAttnCntBytes = static_cast<size_t>(kAttnMaxUnits) * 2 * sizeof(int);

struct AttnLaunch {
  const void* q;
  const void* k;
  const void* v;
  void* out;
  int dtype;  // RB_DTYPE_F16 or RB_DTYPE_BF16
  int batch;     // sequences laid back to back (>= 1)
  int n_q, n_kv;  // per sequence
  int n_head, n_kv_heads, head_dim;  // head_dim: staged width (64, 80 or 128)
  int d_out;                          // output columns per head (real head_dim)
  int head_maps;  // 1: the maps are [rows, heads, d_out] views (coordinates: column, head, row)
  int ldq, ldk, ldv, ldo;  // row strides in elements
  float scale, softcap;
  int mask_mode;
  int64_t window, q_start, kv_start;
  uint32_t* err;
  int num_sms;
  float* ws_rec;  // split-mode workspace (kAttnRecBytes), or null: one CTA per unit
  int* ws_cnt;    // kAttnCntBytes, zeroed once; counters reset themselves
};
// tm[0..2]: Q, K, V maps of the 64-column atoms (128-B swizzle); tm[3..5]: the
// 16-column tail maps (32-B swizzle) used when head_dim == 80 (72-wide heads
// staged as 80 through [rows, heads, 72] maps, head_maps = 1).
int launch_attention(const CUtensorMap* tm, const AttnLaunch& L, cudaStream_t stream);

// Glue (glue.cu).
int launch_rms_norm(const void* x, int xdt, const float* w, float eps, void* y, int ydt, int64_t rows,
                    int d, cudaStream_t st);
int launch_gated(int act, const void* a, const void* b, int dt, int64_t lda, int64_t ldb, void* out,
                 int odt, int64_t ldo, int64_t rows, int64_t cols, cudaStream_t st);
int launch_silu_mul_halves_f16(const void* gu, int64_t rows, int64_t n, void* out, cudaStream_t st);
int launch_rope(const void* x, int dt, const float* cos_t, const float* sin_t, void* y, int64_t rows,
                int heads, int d, int seq, cudaStream_t st);
int launch_embed_gather(const int32_t* ids, const void* table, int64_t vocab, int d, float* x,
                        int64_t rows, uint32_t* err, cudaStream_t st);
int launch_add_rms_norm(float* x, const void* delta, const float* w, float eps, void* h, int64_t rows,
                        int d, cudaStream_t st);
int launch_qk_norm_rope(void* qkv, int64_t ld, int64_t tokens, int hq, int hk, const float* wq,
                        const float* wk, float eps, const float* cos_t, const float* sin_t, int seq,
                        cudaStream_t st);
// dst[r, h, 0:d] = src[r, h*d : h*d+d], dst[r, h, d:dp] = 0 (2-byte elements;
// d and dp multiples of 8).
int launch_add_layer_norm_quant(float* x, const void* delta, const float* g, const float* b, float eps,
                                int8_t* codes, float* row_scale, int64_t rows, int d, cudaStream_t st);
int launch_add_layer_norm(float* x, const void* delta, const float* g, const float* b, float eps,
                          void* h, int64_t rows, int d, cudaStream_t st);
int launch_gelu_f16(void* y, int64_t count, cudaStream_t st);
int launch_last_token_l2(const float* x, int d, int seq, int batch, const float* w, float eps,
                         float* out, cudaStream_t st);

// Tensor-map helper (abi.cu): 2D row-major [rows, cols] tile map with a
// 128-byte swizzle; box = {box_cols, box_rows}.
int make_tmap_2d(CUtensorMap* map, const void* base, int elem_bytes, uint64_t rows,
                 uint64_t cols, uint64_t row_stride_elems, uint32_t box_cols, uint32_t box_rows,
                 int swizzle_bytes);  // 0 (none), 32, 64 or 128
// Index of an N tile in the per-weight tensor-map caches ({256,128,96,64}).
int bn_index(int bn);

// Engine accessors for entry points in other translation units (abi.cu).
int report_error(int rc, const char* msg);  // records rb_last_error, returns rc
void count_launches(int n);
bool make_output_map(CUtensorMap* map, void* y, int y_dtype, int64_t m, int64_t n);
struct W8A8View {
  const int8_t* codes;     // [n, k]
  const float* w_scale;    // [n]
  int64_t n, k;
  float in_scale, out_scale;
  int act;                  // RB_ACT_* fused into the epilogue
  CUtensorMap tm_codes[4];  // box heights 256 / 128 / 96 / 64 (bn_index)
  uint32_t* err;
  int num_sms;
  int device;
};
// Copies out what a W8A8 matmul needs of packed weight `id` (engine lock held
// for the copy only; weights are never freed).
int w8a8_view(int64_t id, W8A8View* v);

}  // namespace rb
