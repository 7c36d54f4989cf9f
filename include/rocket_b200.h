/*
 * rocket_b200.h — C ABI of librocket_b200.so, the B200 (sm_100a) replacement
 * for the operations burn-rocket offloads through its Burn backend extension
 * (crates/burn-rocket/src/ext.rs:57-164, trait RocketOps).
 *
 * Conventions
 *   - Every entry point returns RB_OK (0) or a negative status code; the codes
 *     are burn-rocket's (crates/burn-rocket/src/lib.rs:116-146) extended with
 *     rocket-npu's RANGE/IO (crates/rocket-npu/src/error.rs:28-55). Pack entry
 *     points return a positive weight id or a negative status code.
 *   - Tensor arguments are DEVICE pointers unless the name ends in _host.
 *     Device entry points are asynchronous on the given stream (a cudaStream_t
 *     passed as void*, NULL = legacy default stream); host entry points copy
 *     in and out themselves and return after the result is on the host.
 *   - Layouts follow burn-rocket's boundary: weights [N, K] row-major
 *     (ext.rs:758-779), activations [M, K] row-major, attention tensors
 *     token-major [S, heads * head_dim] (ext.rs:1680-1701).
 *   - One engine per process and device (rb_init). Calls are serialised by an
 *     internal mutex, as the reference serialises through its global ENGINE
 *     mutex (ext.rs:537-556). Resident weights live until process exit
 *     ("pack-and-drop", ext.rs:39-50).
 */
#ifndef ROCKET_B200_H
#define ROCKET_B200_H

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define RB_API __attribute__((visibility("default")))
#else
#define RB_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

/* Status codes (lib.rs:116-146 and rocket-npu error.rs:28-55). */
#define RB_OK 0
#define RB_E_SHAPE (-1)       /* unsupported shape / bad argument */
#define RB_E_TILING (-2)      /* shape not tileable (caller may fall back) */
#define RB_E_NOMEM (-3)       /* allocation failed */
#define RB_E_DEVICE (-4)      /* CUDA runtime / device failure */
#define RB_E_UNSUPPORTED (-5) /* feature not implemented */
#define RB_E_RANGE (-6)       /* value left the output type's range */
#define RB_E_IO (-7)          /* argument / state failure outside the above */

/* Element types of activation / output buffers. */
#define RB_DTYPE_F32 0
#define RB_DTYPE_F16 1
#define RB_DTYPE_BF16 2

/* Attention mask modes: ext.rs:1643-1667 (enum MaskMode). */
#define RB_MASK_NONE 0          /* full bidirectional, n_q == n_kv            */
#define RB_MASK_NONE_BLOCK 1    /* bidirectional over a query chunk           */
#define RB_MASK_CAUSAL 2        /* j <= t                                     */
#define RB_MASK_WINDOW 3        /* |t - j| <= window                          */
#define RB_MASK_CAUSAL_WINDOW 4 /* t - window < j <= t                        */
#define RB_MASK_WINDOW_BLOCK 5  /* |(q0+i) - (k0+j)| <= window                */
#define RB_MASK_CAUSAL_BLOCK 6  /* k0+j <= q0+i (and q0+i-window < k0+j if w>=0) */

/* Weight kinds held by the registry. */
#define RB_WEIGHT_Q8_0 1 /* int8 codes + f16 scale per 32-wide K block           */
#define RB_WEIGHT_W8A8 2 /* per-output-channel int8 codes + f32 scale (QAT form) */
#define RB_WEIGHT_I8G 3  /* group-wise int8 codes + f32 scale per (row, K group)  */
#define RB_WEIGHT_F16 4  /* f16 values [N, K] (the reference's fp16-resident pack) */

/* Replaces burn_rocket::init(threads) (ext.rs:561-580): binds the calling
 * process to CUDA device `device_ordinal` and creates the engine. Later calls
 * are no-ops returning RB_OK. */
RB_API int rb_init(int device_ordinal);

/* Copies the last error message of this thread into buf (NUL-terminated).
 * Returns the message length. The reference logs its failures on stderr
 * before panicking with OpFailure (ext.rs:344-352). */
RB_API int rb_last_error(char* buf, size_t len);

/* Synchronises the engine's device and reports kernel-side failures recorded
 * in the device error word (a bounded wait that timed out, a shape guard):
 * RB_OK, or RB_E_DEVICE with the detail in rb_last_error. Clears the word. */
RB_API int rb_check_device_errors(void);

/* ---- packing (weights become resident; the caller's buffer can be freed) */

/* GGUF Q8_0 blocks (34 bytes: f16 scale + 32 int8 codes, util/gguf.rs:197-215)
 * of an [n, k] weight in HOST memory, blocks running along K. Replaces
 * rocket_pack for Q8_0 checkpoints (ext.rs:586-597, 829-872). */
RB_API int64_t rb_pack_q8_0(const void* blocks_host, int64_t n, int64_t k);

/* f32 [n_i, k] weights in HOST memory, quantised to Q8_0 with the reference
 * encoder (q8_bench.rs:199-219) and concatenated along N. num_parts = 1, 2, 3
 * replace rocket_pack / rocket_pack2 / rocket_pack3 (ext.rs:59-64, 829-934). */
RB_API int64_t rb_pack_f32_q8_0(const float* const* parts_host, const int64_t* n_parts,
                         int num_parts, int64_t k);

/* rb_pack_f32_q8_0 with the f32 parts in DEVICE memory (same encoder). */
RB_API int64_t rb_pack_f32_q8_0_device(const float* const* parts_dev, const int64_t* n_parts,
                                       int num_parts, int64_t k);

/* Per-output-channel int8 weight of a QAT checkpoint: codes [n, k] and
 * w_scale [n] in HOST memory. in_scale == 0 selects the dynamic per-row
 * activation scale max|x|/127; out_scale == 0 leaves the output unrounded.
 * Replaces burn_rocket::pack_qat (ext.rs:1382-1425). */
RB_API int64_t rb_pack_w8a8(const int8_t* codes_host, const float* w_scale_host, int64_t n, int64_t k,
                     float in_scale, float out_scale);

/* Per-output-channel int8 weight from an f32 [n, k] DEVICE weight: codes
 * clamp(round_ties_even(w / s), -127, 127) with s = max(max|w_row|/127, 1e-12)
 * per row, packed like rb_pack_w8a8 (for float checkpoints such as the
 * SigLIP-style tower's f16 weights; the reference takes pre-quantised QAT
 * codes only). */
RB_API int64_t rb_pack_f32_w8a8_device(const float* w_dev, int64_t n, int64_t k, float in_scale,
                                       float out_scale);

/* W8A8 matmul on activations already quantised per row (int8 codes [m, k],
 * f32 scales [m], e.g. from rb_quantize_rows_i8 or rb_add_layer_norm_quant):
 * the same product and epilogue as rb_matmul without the quantiser pass.
 * codes must be 16-byte aligned with k % 16 == 0. */
RB_API int rb_matmul_w8a8_codes(int64_t id, const int8_t* codes, const float* row_scale, int64_t m, int64_t k,
                                void* y, int y_dtype, void* stream);
/* rb_add_layer_norm with the W8A8 dynamic per-row quantiser fused in: writes
 * int8 codes [rows, d] and f32 row scales [rows] of the f16-rounded normalised
 * rows, bit-identical to rb_add_layer_norm then rb_quantize_rows_i8
 * (ext.rs:1236-1238, 1263-1279), and no f16 rows. d in {768, 1024, 1152}. */
RB_API int rb_add_layer_norm_quant(float* x, const void* delta_f16, const float* g, const float* b, float eps,
                                   int8_t* codes, float* row_scale, int64_t rows, int64_t d, void* stream);

/* Element-wise activation fused into the matmul epilogue of weight `id`
 * (no counterpart in the reference's trait; the GEMM-side form of its
 * rocket_gelu glue, host.rs:15-18): later rb_matmul calls on this weight write
 * act(x W^T) and need an f16 output (W8A8: without an output grid).
 * RB_ACT_NONE restores the plain product. Returns RB_OK or RB_E_SHAPE. */
#define RB_ACT_NONE 0
#define RB_ACT_GELU_TANH 1
RB_API int rb_set_weight_activation(int64_t id, int act);

/* Gated (SwiGLU) Q8_0 weight from device-resident f32 gate and up weights,
 * each [n_inter, k] (n_inter a multiple of 64): rows are stored interleaved in
 * blocks of 32 (gate block b, then up block b), and rb_matmul /
 * rb_matmul_grouped on it write the fused f16 output silu(x gate^T) * (x up^T)
 * of width n_inter (per expert for grouped weights, whose experts' gate and
 * up blocks are stacked in order) — the gate|up matmul and silu_mul of a
 * SwiGLU MLP in one kernel (host.rs:31-38). rb_weight_info reports n_inter. */
RB_API int64_t rb_pack_f32_q8_0_gated_device(const float* gate_dev, const float* up_dev, int64_t n_inter, int64_t k);

/* fp16-resident weight (rocket_pack / pack2 / pack3, ext.rs:829-934): host parts
 * [n_parts[i], k] of dtype src_dtype (RB_DTYPE_F32 / F16 / BF16) concatenated
 * along N and rounded to f16 (RNE); rb_matmul is then f16 x f16 with f32
 * accumulation. K % 8 == 0. */
RB_API int64_t rb_pack_f16(const void* const* parts_host, const int64_t* n_parts, int num_parts, int64_t k,
                           int src_dtype);

/* Group-wise int8 weight from a host f32 [n, k] weight (rocket_pack_i8,
 * ext.rs:939-1029): per row and per `group`-wide K block, scale = max(max|w|/127,
 * 1e-12) and code = clamp(round_half_away(w / scale), -127, 127)
 * (host.rs:77-90). group must be a positive multiple of 32 dividing K.
 * rb_matmul with such an id quantises the activation rows the same way and
 * returns sum over groups g (in order) of f32(a_s[m,g]*b_s[n,g]) * f32(int32
 * partial of group g) (matmul_i8 / matmul_gw, ext.rs:1505-1554,
 * matmul/int8.rs:641-672). */
RB_API int64_t rb_pack_i8(const float* w_host, int64_t n, int64_t k, int64_t group);
/* Device group-wise row quantiser: codes int8 [m, k], scales f32 [m, k/group]. */
RB_API int rb_quantize_row_groups(const void* x, int x_dtype, int64_t m, int64_t k, int64_t group,
                                  int8_t* codes, float* scales, void* stream);

/* Weight geometry of a packed id: kind (RB_WEIGHT_*), n, k. */
RB_API int rb_weight_info(int64_t id, int* kind, int64_t* n, int64_t* k);

/* ---- matmul */

/* y[m, n] = x[m, k] · W[n, k]^T with resident weight `id`. x and y are device
 * buffers of x_dtype / y_dtype (RB_DTYPE_*). Replaces rocket_matmul /
 * matmul_impl (ext.rs:85, 1208-1232): Q8_0 weights run the tcgen05 f16 GEMM
 * (activations rounded to f16 like f32_to_f16_par, ext.rs:2144-2156); W8A8
 * weights quantise each activation row to int8 (ext.rs:1263-1279) and run the
 * tcgen05 int8 GEMM with the f32 epilogue of ext.rs:1350-1363. */
RB_API int rb_matmul(int64_t id, const void* x, int x_dtype, int64_t m, int64_t k, void* y,
              int y_dtype, void* stream);

/* Same as rb_matmul with HOST x (x_dtype) and HOST y (y_dtype): the
 * host<->device copies happen inside the call, as in the reference whose
 * Burn tensors live in host memory. */
RB_API int rb_matmul_host(int64_t id, const void* x_host, int x_dtype, int64_t m, int64_t k,
                   void* y_host, int y_dtype);

/* rb_matmul for a W8A8 weight that allocates nothing. No counterpart in the
 * reference: it exists for callers that cannot allocate device memory in the
 * middle of their work, such as code running while a CUDA graph is being
 * captured, code under a fixed device-memory budget or custom allocator, or
 * latency-critical paths that cannot take a synchronising cudaMalloc. The
 * int8 activation codes and row scales that rb_matmul stages in growable
 * engine scratch go instead to one file-scope device array of 32 MiB per GPU
 * (held until process exit); calls needing more than round_up(m*k, 256) +
 * 4*m <= 32 MiB are rejected with RB_E_SHAPE. The first call on a device
 * resolves that array's address, so make it before any stream capture. All
 * calls share the array: calls whose work overlaps on the GPU race and must
 * be serialised by the caller. Results equal rb_matmul's bit for bit. */
RB_API int rb_matmul_w8a8_noalloc(int64_t id, const void* x, int x_dtype, int64_t m, int64_t k,
                                  void* y, int y_dtype, void* stream);

/* ---- attention */

/* Masked grouped-query attention (ext.rs:1669-1858, attention_impl):
 * out = softmax(scale·QK^T (softcapped when softcap != 0) + mask) · V per head,
 * head h reading KV head h / (n_head / n_kv_heads). q/out are [n_q, n_head*d],
 * k/v are [n_kv, n_kv_heads*d], all of `dtype`. mask_mode is RB_MASK_*;
 * window < 0 means "no window" for the windowed modes; q_start / kv_start are
 * the absolute offsets of the block modes (clamped at 0 like ext.rs:736-741).
 * Scores follow fa_score (attn/oneshot.rs:193-199): masked keys score -30000,
 * so a fully masked row averages the values of the keys it iterates. */
RB_API int rb_attention(const void* q, const void* k, const void* v, void* out, int dtype, int64_t n_q,
                 int64_t n_kv, int n_head, int n_kv_heads, int head_dim, float scale,
                 float softcap, int mask_mode, int64_t window, int64_t q_start, int64_t kv_start,
                 void* stream);

/* rb_attention with HOST q/k/v/out buffers (copies inside the call). */
RB_API int rb_attention_host(const void* q, const void* k, const void* v, void* out, int dtype,
                      int64_t n_q, int64_t n_kv, int n_head, int n_kv_heads, int head_dim,
                      float scale, float softcap, int mask_mode, int64_t window, int64_t q_start,
                      int64_t kv_start);

/* Batched, strided form of rb_attention: `batch` sequences lie back to back
 * (sequence b owns query rows [b*n_q, (b+1)*n_q) and key rows
 * [b*n_kv, (b+1)*n_kv)); ldq/ldk/ldv/ldo are row strides in elements, so q, k
 * and v can be column slices of one fused q|k|v projection (the NPU route's
 * split of the fused matmul output, src/qwen3_embedding/model.rs:355-368).
 * f16/bf16 only when strided. */
RB_API int rb_attention_batched(const void* q, int64_t ldq, const void* k, int64_t ldk, const void* v,
                                int64_t ldv, void* out, int64_t ldo, int dtype, int64_t batch,
                                int64_t n_q, int64_t n_kv, int n_head, int n_kv_heads, int head_dim,
                                float scale, float softcap, int mask_mode, int64_t window,
                                int64_t q_start, int64_t kv_start, void* stream);

/* head_dim 72 (the SigLIP-style config) is supported by every attention entry:
 * heads are read in place and staged as 80 columns (the UMMA K granularity,
 * the 8 columns past each head read as zeros) and the output keeps 72
 * columns. */

/* ---- glue ops of the RocketOps surface (ext.rs:70-83, 1054-1152; formulas
 * host.rs:15-72). Device buffers, any float dtype, asynchronous on `stream`. */

/* rocket_rms_norm / rocket_rms_norm_noscale: y = x * (mean(x^2) + eps)^-0.5 * w
 * over rows of length d; w == NULL is the scale-free form. */
RB_API int rb_rms_norm(const void* x, int x_dtype, const float* w, float eps, void* y, int y_dtype,
                       int64_t rows, int64_t d, void* stream);
/* rocket_silu_mul: out = gate * sigmoid(gate) * up (host.rs:31-38). */
RB_API int rb_silu_mul(const void* gate, const void* up, int dtype, void* out, int64_t count,
                       void* stream);
/* rocket_gelu_mul: out = gelu_tanh(gate) * up (host.rs:15-27). */
RB_API int rb_gelu_mul(const void* gate, const void* up, int dtype, void* out, int64_t count,
                       void* stream);
/* rocket_rope: x [batch, seq, heads, head_dim], cos/sin f32 [seq, head_dim/2];
 * rotate-half (host.rs:61-72). In place when y == x. */
RB_API int rb_rope(const void* x, int dtype, const float* cos, const float* sin, void* y,
                   int64_t batch, int64_t seq, int heads, int head_dim, void* stream);

/* ---- fused steps of the embedding-model forward (src/qwen3_embedding/model.rs) */

/* x[t, :] = f32(table[ids[t], :]) for an f16 table [vocab, d]; an id outside
 * the vocabulary reads row 0 and flags the device error word. */
RB_API int rb_embed_gather(const int32_t* ids, int64_t tokens, const void* table_f16, int64_t vocab,
                           int64_t d, float* x, void* stream);
/* x += delta (f16, NULL = none); h = rms_norm(x, w, eps) as f16. d in {1024, 1152, 2048}. */
RB_API int rb_add_rms_norm(float* x, const void* delta_f16, const float* w, float eps, void* h_f16,
                           int64_t rows, int64_t d, void* stream);
/* x += delta (f16, NULL = none); h = layer_norm(x) * g + b as f16 (biased
 * variance, eps inside the sqrt). d in {768, 1024, 1152}. */
RB_API int rb_add_layer_norm(float* x, const void* delta_f16, const float* g, const float* b, float eps,
                             void* h_f16, int64_t rows, int64_t d, void* stream);
/* In place: y = gelu_tanh(y) for f16 y (host.rs:15-18); count % 8 == 0. */
RB_API int rb_gelu(void* y_f16, int64_t count, void* stream);
/* In place on a fused q|k|v f16 buffer [tokens, ld]: per-head RMSNorm of the
 * q heads (q_norm_w) and k heads (k_norm_w), then RoPE at position t % seq
 * (model.rs:369-376). head_dim 128. */
RB_API int rb_qk_norm_rope(void* qkv_f16, int64_t ld, int64_t tokens, int n_q_heads, int n_kv_heads,
                           int head_dim, const float* q_norm_w, const float* k_norm_w, float eps,
                           const float* cos, const float* sin, int64_t seq, void* stream);
/* out[r, :] = silu(gu[r, :n]) * gu[r, n:2n] for a fused gate|up f16 output
 * (model.rs:593-606). */
RB_API int rb_silu_mul_halves(const void* gu_f16, int64_t rows, int64_t n, void* out_f16, void* stream);
/* out[b, :] = l2_normalise(rms_norm(x[b*seq + seq-1, :], w, eps)): the final
 * norm of each sequence's last token (model.rs:230-235), L2-normalised. */
RB_API int rb_last_token_l2(const float* x, int64_t batch, int64_t seq, int64_t d, const float* w,
                            float eps, float* out, void* stream);

/* ---- codec and quantiser surfaces (parity / debugging) */

/* Dequantise a packed Q8_0 weight into a device buffer: f32 (exact d·q, the
 * GGUF decode of util/gguf.rs:197-215) or f16 (RNE(d·q), the values the GEMM
 * stages in shared memory). */
RB_API int rb_q8_0_dequant(int64_t id, void* out, int out_dtype, void* stream);

/* Per-row dynamic int8 quantisation of an [m, k] device activation
 * (ext.rs:1263-1279): scale = max(max|x|/127, 1e-12), code =
 * clamp(round_ties_even(x · (1/scale)), -128, 127). */
RB_API int rb_quantize_rows_i8(const void* x, int x_dtype, int64_t m, int64_t k, int8_t* codes,
                        float* row_scale, void* stream);

/* Raw int32 accumulators acc[m, n] = codes[m, k] · W[n, k]^T of a W8A8 weight
 * (the exact integer product the reference checks under ROCKET_QAT_CHECK,
 * ext.rs:1309-1334). */
RB_API int rb_matmul_i8_acc(int64_t id, const int8_t* codes, int64_t m, int32_t* acc, void* stream);

/* ---- mixture of experts (the Clef MoE layer around its expert GEMMs:
 * route src/clef/model.rs:462-489, Buckets::build / combine
 * src/clef/engine.rs:284-340; device-side, so a layer stays graph-capturable). */
/* Workspace bytes and permuted-row capacity for `tokens` x top_k routed slots
 * over `experts` (segments are 256-row aligned: one CTA-pair tile of the
 * grouped GEMM never spans two experts). */
RB_API int64_t rb_moe_workspace_bytes(int64_t tokens, int top_k, int experts);
RB_API int64_t rb_moe_max_rows(int64_t tokens, int top_k, int experts);
/* int32-word offset, inside the workspace, of the slot -> permuted-row map
 * [tokens * top_k] that rb_moe_dispatch writes. */
RB_API int64_t rb_moe_slot_rows_offset(int64_t tokens, int top_k, int experts);
/* f32 logits [tokens, experts] -> ids int32 [tokens, top_k] (descending
 * probability, ties to the lower id) and weights f32 (renormalised over the
 * selected experts when normalize != 0). experts <= 256, top_k <= 32. */
RB_API int rb_moe_route(const float* logits, int64_t tokens, int experts, int top_k, int normalize,
                        int32_t* ids, float* weights, void* stream);
/* Buckets the routed slots per expert in `workspace` and gathers each slot's
 * f16 token row x[tokens, hidden] into x_perm[rb_moe_max_rows(), hidden]
 * (256-row-aligned expert segments, padding rows zeroed). An id of -1 means
 * "no expert" (the padding rows of a fixed-capacity exchange): the slot gets
 * no row and its slot -> row entry is -1. */
RB_API int rb_moe_dispatch(const int32_t* ids, int64_t tokens, int top_k, int experts, const void* x_f16,
                           int64_t hidden, void* workspace, void* x_perm_f16, void* stream);
/* y_perm[r, :] = x_perm[r, :] · W_e^T for the expert e owning row r, where the
 * Q8_0 weight `id` stacks the experts' [N, K] blocks (experts * N rows). Output
 * f16 or f32 [max_rows, N]. */
RB_API int rb_matmul_grouped(int64_t id, int experts, const void* x_perm_f16, int64_t max_rows,
                             const void* workspace, int64_t tokens, int top_k, void* y, int y_dtype,
                             void* stream);
/* x[t, :] (f32, in place) += sum over the token's slots in ascending expert id
 * of weight * y_perm[row of slot, :] (f16). */
RB_API int rb_moe_combine(float* x, const void* y_perm_f16, int64_t hidden, const int32_t* ids,
                          const float* weights, const void* workspace, int64_t tokens, int top_k, int experts,
                          void* stream);

/* ---- expert parallelism (no counterpart in the reference: its experts run
 * on one board). Experts are split over `ranks` in consecutive blocks of
 * experts/ranks ids. rb_ep_build_send groups the routed slots by destination
 * rank: dest_counts[ranks] (rows per destination), send_rows[tokens*top_k,
 * hidden] f16 (the token rows in destination order), send_meta[tokens*top_k]
 * (expert id local to the destination) and slot_pos[tokens*top_k] (send
 * position of each slot). dest_cursor[ranks] is scratch. */
RB_API int rb_ep_build_send(const int32_t* ids, int64_t tokens, int top_k, int experts, int ranks,
                            const void* x_f16, int64_t hidden, int32_t* dest_counts, int32_t* dest_cursor,
                            int32_t* send_meta, int32_t* slot_pos, void* send_rows_f16, void* stream);
/* rb_ep_build_send with a fixed capacity per destination, so the exchange
 * needs no counts on the host (equal all-to-all splits of `capacity` rows; a
 * layer stays graph-capturable): destination q owns send positions
 * [q*capacity, (q+1)*capacity) of send_rows [ranks*capacity, hidden] and
 * send_meta [ranks*capacity]; unused positions hold send_meta = -1 (no expert:
 * rb_moe_dispatch skips such rows, rb_gather_rows skips index -1). A slot past
 * its destination's capacity is not sent (slot_pos = -1, rb_moe_combine_rows
 * skips it) and sets the exchange-overflow bit that rb_check_device_errors
 * reports. dest_counts[ranks] still receives the true rows per destination. */
RB_API int rb_ep_build_send_capacity(const int32_t* ids, int64_t tokens, int top_k, int experts, int ranks,
                                     int64_t capacity, const void* x_f16, int64_t hidden, int32_t* dest_counts,
                                     int32_t* dest_cursor, int32_t* send_meta, int32_t* slot_pos,
                                     void* send_rows_f16, void* stream);
/* out[i, :] = in[idx[i], :] for f16 rows (rows with idx[i] < 0 are left as they are). */
RB_API int rb_gather_rows(const void* in_f16, const int32_t* idx, int64_t n, int64_t hidden, void* out_f16,
                          void* stream);
/* rb_moe_combine with an explicit slot -> row map (e.g. slot_pos after the
 * outputs came back from the expert ranks). */
RB_API int rb_moe_combine_rows(float* x, const void* y_f16, int64_t hidden, const int32_t* ids,
                               const float* weights, const int32_t* row_of_slot, int64_t tokens, int top_k,
                               void* stream);

/* ---- statistics (MemStats, lib.rs:44-96) */
RB_API int rb_mem_stats(int64_t* weights_bytes, int64_t* scratch_bytes, int64_t* num_weights);

/* Number of rocket-b200 kernel launches issued since the last reset. */
RB_API int64_t rb_launch_count(int reset);

/* GEMM tile policy for later matmul calls (process-wide; no counterpart in the
 * reference): RB_TILES_AUTO picks single-CTA or CTA-pair tiles by a cost model,
 * RB_TILES_SINGLE uses only single-CTA tiles, RB_TILES_PAIR prefers CTA-pair
 * (256-row, cta_group::2) tiles. Results are bit-identical across policies for
 * W8A8 and identical up to f32 summation order for Q8_0. Returns the previous
 * policy, or RB_E_SHAPE for an unknown one. */
#define RB_TILES_AUTO 0
#define RB_TILES_SINGLE 1
#define RB_TILES_PAIR 2
RB_API int rb_set_tile_policy(int policy);

/* Attention work split for later attention calls (process-wide; no
 * counterpart in the reference): RB_ATTN_SPLIT_AUTO compares, per call, a
 * greedy one-CTA-per-unit schedule (unit = a KV head's pair of 128-row query
 * slots) against one CTA per SM over equal shares of all key tiles, with units
 * cut at share boundaries and merged by their last finishing part;
 * RB_ATTN_SPLIT_NEVER / RB_ATTN_SPLIT_ALWAYS force one of them. Results agree
 * within f32 summation order. Returns the previous policy, or RB_E_SHAPE. */
/* Failure-path self-test (no counterpart in the reference): one CTA waits,
 * with the bounded mbarrier wait every pipeline uses, on a barrier nothing
 * arrives on, for limit_ns (1 ns .. 1 s). The wait runs out, the kernel
 * flags the engine's wait-timeout error bit and returns; this call then
 * reads and clears the error word like rb_check_device_errors and returns its
 * result (RB_E_DEVICE, last error naming "wait-timeout"). *waited_us receives
 * how long the wait lasted. No GPU fault is involved and the context stays
 * usable. */
RB_API int rb_selftest_wait_timeout(int64_t limit_ns, int64_t* waited_us);

#define RB_ATTN_SPLIT_AUTO 0
#define RB_ATTN_SPLIT_NEVER 1
#define RB_ATTN_SPLIT_ALWAYS 2
RB_API int rb_set_attention_split(int policy);

#ifdef __cplusplus
}
#endif

#endif /* ROCKET_B200_H */
