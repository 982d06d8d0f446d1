/*
 * C ABI of libluce_megakernel_b200.so -- the sm_100a implementation of the Qwen3.5-0.8B
 * hybrid decode / prefill hot path.  Plain pointers and sizes only; every pointer is a
 * CUDA device pointer unless stated otherwise.
 *
 * The launch_* entry points keep the names and argument lists of the C entry points the
 * reference's PyTorch extension binds (reference: megakernel/torch_bindings.cpp:56-71,
 * 144-145, 354-368), so the reference's binding file links against this library unchanged.
 * They return an int status (the reference returns void; a caller that ignores the value
 * is unaffected): 0 = enqueued, otherwise one of the MK_ERR_* codes below.
 *
 * Threading: calls are asynchronous with respect to the host and are ordered on `stream`.
 * The library keeps one small workspace per device (allocated on the first call on that
 * device) and is not re-entrant for concurrent calls on the same device.
 */
#ifndef LUCE_MEGAKERNEL_B200_H
#define LUCE_MEGAKERNEL_B200_H

#include <cuda_runtime_api.h>

#ifdef __cplusplus
extern "C" {
#endif

#define MK_OK 0
#define MK_ERR_BAD_ARG 1        /* null pointer, misaligned pointer, size out of range */
#define MK_ERR_CUDA 2           /* a CUDA runtime call failed; see mk_last_error_string() */
#define MK_ERR_DEVICE_TIMEOUT 3 /* a previous launch gave up on a bounded device-side wait */

/* Layer pointer table entry (reference: megakernel/torch_bindings.cpp:30-34,
 * megakernel/kernel.cu:104-111).  24 entries; attention layers use 11 pointers, DeltaNet
 * layers 14, in the order megakernel/model.py:95-133 packs them. */
typedef struct {
    int layer_type; /* 0 = Gated DeltaNet, 1 = full attention */
    int _pad[3];
    void *ptrs[14];
} MkLayerWeights;

/* One greedy decode step.  Replaces launch_decode (reference: megakernel/kernel.cu:952-1010,
 * declared at megakernel/torch_bindings.cpp:56-71).  Scratch arguments the new kernel does not
 * need (g_activations, g_residual, barrier_*, block_max_*, lm_sync_counter) are accepted and
 * left untouched. */
int launch_decode(
    int input_token_id, int *output_token_id,
    const void *embed_weight, const MkLayerWeights *layer_weights,
    const void *final_norm_weight, const void *lm_head_weight,
    void *fa_k_cache, void *fa_v_cache,
    void *dn_states, void *conv_bufs,
    void *hidden_buffer, void *g_activations, void *g_residual,
    void *g_qkv_scratch, void *g_kv_scratch, void *g_attn_out,
    void *g_mlp_inter, void *g_z_scratch, void *g_beta_scratch,
    void *g_alpha_scratch, void *g_normalized,
    unsigned int *barrier_counter, unsigned int *barrier_generation,
    float *block_max_vals, int *block_max_idxs,
    unsigned int *lm_sync_counter,
    float *seen_token_mask,
    float repetition_penalty,
    int position, int max_seq_len, cudaStream_t stream);

/* NVFP4 decode step and multi-step decode with device token feedback.  Replace launch_decode_nvfp4
 * and launch_decode_many_nvfp4 (reference: megakernel/kernel_gb10_nvfp4.cu:2068-2257, declared at
 * megakernel/torch_bindings.cpp:74-106) with the same argument lists.  layer_weights is the 24 x
 * 208-byte table {int type; int group_size; int pad[2]; void *ptrs[24]} of the reference's NVFP4
 * driver (megakernel/model_nvfp4.py:274-311, 456-473): quantised matrices as (packed e2m1, fp16
 * scales per 32) pairs, norms / conv / beta / alpha in bf16; the LM head is the packed 16-block
 * E4M3 format of launch_quantize_nvfp4_lm_out.  input_token_ptr / token_buffer are device
 * pointers.  group_size must be 32.  The lm_hidden_* / lm_logits_f16 and the other scratch
 * arguments are accepted and ignored. */
int launch_decode_nvfp4(
    const int *input_token_ptr, int *output_token_id,
    const void *embed_weight, const void *layer_weights, const void *final_norm_weight,
    const void *lm_head_weight_packed, const void *lm_head_scales,
    void *lm_hidden_bf16, void *lm_hidden_packed, void *lm_hidden_scales, void *lm_logits_f16,
    void *fa_k_cache, void *fa_v_cache, void *dn_states, void *conv_bufs,
    void *hidden_buffer, void *g_activations, void *g_residual,
    void *g_qkv_scratch, void *g_kv_scratch, void *g_attn_out,
    void *g_mlp_inter, void *g_z_scratch, void *g_beta_scratch,
    void *g_alpha_scratch, void *g_normalized,
    unsigned int *barrier_counter, unsigned int *barrier_generation,
    float *block_max_vals, int *block_max_idxs, unsigned int *lm_sync_counter,
    int position, int max_seq_len, int group_size, cudaStream_t stream);
int launch_decode_many_nvfp4(
    int *token_buffer, int *output_tokens, int steps,
    const void *embed_weight, const void *layer_weights, const void *final_norm_weight,
    const void *lm_head_weight_packed, const void *lm_head_scales,
    void *lm_hidden_bf16, void *lm_hidden_packed, void *lm_hidden_scales, void *lm_logits_f16,
    void *fa_k_cache, void *fa_v_cache, void *dn_states, void *conv_bufs,
    void *hidden_buffer, void *g_activations, void *g_residual,
    void *g_qkv_scratch, void *g_kv_scratch, void *g_attn_out,
    void *g_mlp_inter, void *g_z_scratch, void *g_beta_scratch,
    void *g_alpha_scratch, void *g_normalized,
    unsigned int *barrier_counter, unsigned int *barrier_generation,
    float *block_max_vals, int *block_max_idxs, unsigned int *lm_sync_counter,
    int position, int max_seq_len, int group_size, cudaStream_t stream);

/* Resident-block ceiling and decode grid override
 * (reference: megakernel/kernel.cu:1012-1020, megakernel/torch_bindings.cpp:144-145).
 * The kernel runs one CTA per SM; overrides are clamped to [129, ceiling]. */
void set_decode_blocks_override(int blocks);
int query_max_safe_decode_blocks(void);

/* `steps` greedy decode steps with the token fed back on the device (no host sync between
 * steps); output_tokens[i] receives step i's token, token_buffer[0] holds the running token
 * and must contain the first input token on entry.  bf16 counterpart of
 * launch_decode_many_nvfp4 (reference: megakernel/kernel_gb10_nvfp4.cu:2192-2257), same
 * argument meaning as launch_decode otherwise. */
int mk_decode_many_bf16(
    int *token_buffer, int *output_tokens, int steps,
    const void *embed_weight, const MkLayerWeights *layer_weights,
    const void *final_norm_weight, const void *lm_head_weight,
    void *fa_k_cache, void *fa_v_cache,
    void *dn_states, void *conv_bufs,
    void *hidden_buffer,
    void *g_qkv_scratch, void *g_kv_scratch, void *g_attn_out,
    void *g_mlp_inter, void *g_z_scratch, void *g_beta_scratch,
    void *g_alpha_scratch, void *g_normalized,
    float *seen_token_mask, float repetition_penalty,
    int position, int max_seq_len, cudaStream_t stream);

/* NVFP4 weight quantisers, bit-exact to the reference's kernels.
 * launch_quantize_nvfp4_out: layer-weight format (reference: megakernel/kernel_gb10_nvfp4.cu:1778-1817,
 *   declared at megakernel/torch_bindings.cpp:108-110): weight bf16 [rows, cols] -> packed uint8
 *   [rows, cols/2] (low nibble = even element) + fp16 scales [rows, cols/group_size].
 * launch_quantize_nvfp4_lm_out: LM-head / tensor-core format (reference:
 *   megakernel/kernel_gb10_nvfp4.cu:1373-1437, megakernel/torch_bindings.cpp:112-114): 16-element blocks,
 *   E4M3 scales in 128-row x 4-column tiles of 512 bytes; rows % 128 == 0, cols % 64 == 0,
 *   scales_out has (rows/128)*(cols/64)*512 bytes. */
int launch_quantize_nvfp4_out(const void *weight, int rows, int cols, int group_size,
                              void *packed_out, void *scales_out, cudaStream_t stream);
int launch_quantize_nvfp4_lm_out(const void *weight, int rows, int cols,
                                 void *packed_out, void *scales_out, cudaStream_t stream);
const char *mk_quantize_error(void);
/* Arithmetic of the two quantisers above.  1 (default): that of the reference's binary -- its extension is built
 * with --use_fast_math (megakernel/setup.py:49-59), so amax / 6 and 1 / scale are an approximate divide and an
 * approximate reciprocal; packed codes and scales then equal what the reference extension writes.  0: every divide and
 * multiply correctly rounded (the arithmetic of a plain-C restatement); about one packed byte in 1700 differs from
 * mode 1 on N(0, 0.02) weights, always by one code step at a threshold. */
void mk_set_quantize_arithmetic(int reference_binary);

/* NVFP4 weights dequantised in registers.  format 0 = layer-weight format (fp16 scales per 32),
 * format 1 = LM-head format (E4M3 scales per 16, tiled); value = e2m1(code) * scale
 * (reference: megakernel/kernel_gb10_nvfp4.cu:80-83, 528-552, 682-856, 1439-1530).
 * mk_matvec_nvfp4: y[rows] = dequant(W)[rows, cols] . x[cols], f32 in and out (the streaming
 *   row product of the reference's matvec_nvfp4 / lm_head_kernel_nvfp4).
 * mk_dequantize_nvfp4: out[rows, cols] f32 = dequantised weights, bit-exact to the reference's LUT * scale. */
int mk_matvec_nvfp4(int format, const void *packed, const void *scales, const float *x, float *y,
                    int rows, int cols, int group_size, cudaStream_t stream);
int mk_dequantize_nvfp4(int format, const void *packed, const void *scales, float *out,
                        int rows, int cols, int group_size, cudaStream_t stream);
const char *mk_nvfp4_error(void);

/* The NVFP4 format with an fp32 per-tensor scale: e2m1 values in 16-element blocks, E4M3 block scales in the tiling
 * of the LM-head format, and s_t = amax(tensor) / (6 * 448) (1 for an all-zero tensor); block scale =
 * E4M3(max((amax(block) / 6) / s_t, 2^-28)), code = e2m1_rne(x / (block * s_t)), value = e2m1(code) * (block * s_t).
 * The reference's 16-block quantiser has no tensor scale (megakernel/kernel_gb10_nvfp4.cu:1373-1437, alpha = 1 at
 * :451); this is an additional format next to its two.  rows % 128 == 0, cols % 64 == 0;
 * packed_out uint8 [rows][cols / 2], scales_out uint8 [(rows / 128) * (cols / 64) * 512], tensor_scale device float[1].
 * Dequantised f32 values are bit-exact to the CPU restatement; out_is_bf16 = 1 rounds them to bf16. */
int mk_quantize_nvfp4_tensor_scale(const void *weight, int rows, int cols, void *packed_out, void *scales_out,
                                   float *tensor_scale_out, cudaStream_t stream);
int mk_dequantize_nvfp4_tensor_scale(const void *packed, const void *scales, const float *tensor_scale, void *out,
                                     int out_is_bf16, int rows, int cols, cudaStream_t stream);

/* Decode on the NVFP4 format with a per-tensor scale (e2m1 values in 16-element blocks, E4M3 block scales, one fp32
 * scale per matrix; every linear layer and the LM head, produced by mk_quantize_nvfp4_tensor_scale): `steps` greedy
 * steps in one launch, the running token read from and written back to token_buffer[0] (device), step s's token to
 * output_tokens[s].  No counterpart in the reference, whose NVFP4 decode (megakernel/kernel_gb10_nvfp4.cu:2006-2257)
 * reads 32-element groups with fp16 scales and no tensor scale; same kernel schedule as launch_decode_nvfp4.
 * layer_weights: num_layers entries of 224 bytes {int type; int pad[3]; void *ptrs[26]}; a quantised matrix takes
 * three slots (packed codes [rows][K/2]; block scales as plain rows [rows][K/16], see mk_nvfp4_scales_to_rows; device
 * pointer to its fp32 tensor scale), everything else one bf16 slot:
 *   DeltaNet : in_norm, qkv(3), z(3), w_beta, w_alpha, conv_w, A_log, dt_bias, norm_w, out(3), post_norm, gate(3),
 *              up(3), down(3)
 *   attention: in_norm, q(3), k(3), v(3), q_norm, k_norm, o(3), post_norm, gate(3), up(3), down(3)
 * The kernel multiplies exact f16 products code x block scale on the tensor cores, accumulates in f32 and applies the
 * tensor scale to each finished row product.
 * mk_nvfp4_scales_to_rows converts block scales from the 128 x 4 tiles the quantisers write to plain rows. */
int mk_decode_nvfp4_ts(
    int *token_buffer, int *output_tokens, int steps,
    const void *embed_weight, const void *layer_weights, const void *final_norm_weight,
    const void *lm_head_packed, const void *lm_head_scales_rows, const float *lm_head_tensor_scale,
    void *fa_k_cache, void *fa_v_cache, void *dn_states, void *conv_bufs,
    void *hidden_buffer, void *g_normalized, int position, int max_seq_len, cudaStream_t stream);
int mk_nvfp4_scales_to_rows(const void *tiled_scales, int rows, int cols, void *rows_out, cudaStream_t stream);

/* The decode of mk_decode_nvfp4_ts on the block-scaled 5th-generation tensor cores: tcgen05.mma kind::mxf4nvf4 reads
 * the e2m1 codes from shared memory and the E4M3 block scales from tensor memory, accumulators live in tensor memory.
 * Same quantised values and tensor scales as mk_decode_nvfp4_ts, same 224-byte table, except that the FIRST slot of
 * each phase's matrix group (DeltaNet: qkv, out, gate, down; attention: q, o, gate, down) points at an array of 148
 * chunk images, one per CTA of the decode grid, holding that CTA's rows of the phase (qkv|z, q|k|v, out, gate|up,
 * down) in the operand layout of the MMA, and lm_head_images at 148 x lm_image_chunks images of 56 LM-head rows
 * (the down projection has two images per CTA, one per half of K):
 *   codes : K/256 tiles of RP x 128 bytes (RP = 56, 40, 8, 56, 8; 56 for the LM head); tile t, local row i = codes
 *           k = 256 t .. 256 t + 255 of that row, its eight 16-byte pieces stored at piece j ^ (i % 8);
 *   scales: one unit of 32 lanes x 16 bytes (one tcgen05.cp) per MMA step of 64 k: unit ks, lane l, byte 4 g + b =
 *           the scale of block b of row l + 32 g in that step; bytes of absent rows are zero;
 *   CTA c owns rows [n c / 148, n (c + 1) / 148) of the phase's n rows; gate row o and up row o of an output sit at
 *   local rows o - first and 28 + o - first; image sizes 36864, 28672, 24576, 36864, 2 x 21504 and 36864 bytes.
 * (luce_megakernel_b200/nvfp4_images.py builds them from the quantiser's output.)  The activation vector of every
 * projection is the other operand: it is scaled to a fixed range and expanded on the fly into act_terms (1..8) NVFP4
 * residual terms, term n + 1 encoding six times what term n left over, one MMA column per term; 8 terms reproduce
 * the f32 vector to about 1e-6 of each block's largest value, 4 terms to better than bf16.  Needs a device that
 * co-schedules 148 CTAs.  No counterpart in the reference (its NVFP4 decode dequantises through a LUT and multiplies
 * on mma.sync, megakernel/kernel_gb10_nvfp4.cu:528-552). */
int mk_decode_nvfp4_mma(
    int *token_buffer, int *output_tokens, int steps,
    const void *embed_weight, const void *layer_weights, const void *final_norm_weight,
    const void *lm_head_images, int lm_image_chunks, const float *lm_head_tensor_scale,
    void *fa_k_cache, void *fa_v_cache, void *dn_states, void *conv_bufs,
    void *hidden_buffer, void *g_normalized, int position, int max_seq_len, int act_terms, cudaStream_t stream);

/* Prefill of a prompt of seq_len tokens from position 0: fills the KV caches for positions
 * 0..seq_len-1, advances the DeltaNet and conv state from their current content (callers zero
 * them first), writes the first generated token to output_token, the last row's final-normed
 * vector to final_normed (bf16 [1024]) and its pre-norm hidden to hidden_bf16_out (bf16 [1024]).
 * Replaces launch_prefill_bf16 (reference: megakernel/prefill.cu:1559-1793, declared at
 * megakernel/torch_bindings.cpp:354-368) with the same argument list; the scratch buffers of that
 * signature are accepted and ignored (the library keeps its own workspace, grown on demand:
 * about 45 KB per prompt token).  token_ids is a device pointer.  fused_fa_qkv_base is
 * [n_fa, 5120, 1024] (q|k|v rows) and fused_gate_up_base [num_layers, 7168, 1024] (gate|up rows),
 * as the reference driver packs them (megakernel/model.py:245-260).
 * mk_prefill_bf16 is the same call without the unused scratch arguments and with explicit depth
 * and vocabulary. */
int launch_prefill_bf16(
    const int *token_ids, int seq_len, int *output_token,
    const void *embed_weight, const MkLayerWeights *layers,
    const void *final_norm_w, const void *lm_head_w,
    void *fa_k_cache, void *fa_v_cache, void *dn_states, void *conv_bufs,
    void *hidden, void *residual, void *normalized,
    void *proj_buf, void *proj_buf2, void *attn_buf, void *mlp_buf,
    void *dn_out_buf, void *beta_buf, void *alpha_buf, void *dn_pre_qkv,
    void *dn_u_scratch, void *dn_w_scratch, void *dn_cs_scratch,
    const void *fused_fa_qkv_base, const void *fused_gate_up_base,
    void *final_normed, void *hidden_bf16_out,
    void *lm_bmv, void *lm_bmi,
    int max_seq_len, cudaStream_t stream);
int mk_prefill_bf16(
    const int *token_ids, int seq_len, int *output_token,
    const void *embed_weight, const MkLayerWeights *layers, const void *final_norm_w, const void *lm_head_w,
    void *fa_k_cache, void *fa_v_cache, void *dn_states, void *conv_bufs,
    const void *fused_fa_qkv_base, const void *fused_gate_up_base,   /* either may be null: per-matrix GEMMs */
    void *final_normed, void *hidden_bf16_out,
    int max_seq_len, int num_layers, int vocab, cudaStream_t stream);
const char *mk_prefill_error(void);
/* The prefill entry points and the batched decode step share one library workspace per device (about 45 KB per
 * prompt token).  It only ever grows: a call that needs more tokens than it holds synchronises the device, frees
 * every buffer and allocates larger ones.  Consequences for callers:
 *   - growing is refused (MK_ERR_CUDA) while `stream` is being captured into a CUDA graph: call
 *     mk_prefill_reserve(max_tokens) once, before capturing, with the longest prompt the graphs will see;
 *   - a graph captured before a growth holds device pointers into the freed buffers and must be captured again:
 *     mk_prefill_workspace_generation() changes whenever the workspace was reallocated;
 *   - a prefill and a batched step on one device use the same buffers: keep them on one stream or serialise them. */
int mk_prefill_reserve(int max_tokens);
int mk_prefill_workspace_tokens(void);              /* prompt tokens the workspace holds at present */
unsigned int mk_prefill_workspace_generation(void);

/* Batched decode: `batch` (1..16) independent sequences advance by one token each and share every weight pass.
 * The reference has no batched op (all of megakernel/torch_bindings.cpp:569-675 are batch 1); these calls keep the
 * reference's per-sequence layouts and put a leading batch dimension on them:
 *   tokens, positions, output_tokens: device int32 [batch] (positions[b] = index the new token of sequence b is
 *   written at = tokens of b already in its cache; every sequence has its own length, all < max_seq_len),
 *   fa_k_cache / fa_v_cache bf16 [batch][n_fa][2][max_seq_len][256], dn_states f32 [batch][n_dn][16][128][128],
 *   conv_bufs f32 [batch][n_dn][6144][4]  (slice b is exactly what mk_prefill_bf16 / decode take for one sequence),
 *   final_normed / hidden_bf16_out: bf16 [batch][1024] or null.
 * mk_decode_batch runs one step and leaves tokens / positions untouched; mk_decode_batch_many runs `steps` steps
 * with the chosen tokens fed back on the device: tokens and positions are updated in place and tokens_log
 * [steps][batch] receives every step's tokens.  Enqueue only (no synchronisation once the pointer table is cached):
 * capturable into a CUDA graph.  Rounding points are those of the prompt path. */
int mk_decode_batch(
    const int *tokens, const int *positions, int *output_tokens, int batch,
    const void *embed_weight, const MkLayerWeights *layers, const void *final_norm_w, const void *lm_head_w,
    void *fa_k_cache, void *fa_v_cache, void *dn_states, void *conv_bufs,
    const void *fused_fa_qkv_base, const void *fused_gate_up_base, void *final_normed, void *hidden_bf16_out,
    int max_seq_len, int num_layers, int vocab, cudaStream_t stream);
/* LM head of the batched step: 1 (default) = tensor cores with the f32 activations as two bf16 terms, 0 = f32 FMAs. */
void mk_decode_batch_set_lm_head(int tensor_cores);
/* Projections back into the residual stream (out / o / down): 1 or 2 (default) = straight-line kernel, 8 rows per CTA,
 * all weights requested before the dependency wait, activations staged by bulk async copies; 0 = 16 rows per CTA with K
 * split over 4 CTAs. */
void mk_decode_batch_set_residual_kernel(int mode);
int mk_decode_batch_many(
    int steps, int *tokens, int *positions, int *tokens_log, int batch,
    const void *embed_weight, const MkLayerWeights *layers, const void *final_norm_w, const void *lm_head_w,
    void *fa_k_cache, void *fa_v_cache, void *dn_states, void *conv_bufs,
    const void *fused_fa_qkv_base, const void *fused_gate_up_base,
    int max_seq_len, int num_layers, int vocab, cudaStream_t stream);

/* The batched step on the NVFP4 format with a per-tensor scale (see mk_decode_nvfp4_ts for the format and the 224-byte
 * table): `steps` steps for `batch` sequences.  steps == 1 with output_tokens set: one step, tokens / positions
 * untouched (mk_decode_batch's behaviour); otherwise the chosen tokens are fed back on the device, tokens / positions
 * are updated in place and tokens_log [steps][batch] receives every step's tokens (mk_decode_batch_many's).  State
 * tensors as for mk_decode_batch.  Same kernel sequence as the bf16 step; the projections and the LM head read 4-bit
 * weights (0.5625 bytes per weight).  No counterpart in the reference. */
int mk_decode_batch_nvfp4_ts(
    int steps, int *tokens, int *positions, int *output_tokens, int *tokens_log, int batch,
    const void *embed_weight, const void *layers, const void *final_norm_w,
    const void *lm_head_packed, const void *lm_head_scales_rows, const float *lm_head_tensor_scale,
    void *fa_k_cache, void *fa_v_cache, void *dn_states, void *conv_bufs, void *final_normed, void *hidden_bf16_out,
    int max_seq_len, int num_layers, int vocab, cudaStream_t stream);

/* The reference's other prefill entry points, with their argument lists: launch_prefill_bf16_mega (bf16, per-matrix
 * weights from the 128-byte table only; reference: megakernel/prefill_megakernel.cu:1031-1045),
 * launch_prefill_bf16_nvfp4_lm (bf16 layers, NVFP4 LM head; megakernel/prefill_bw.cu:1486-1503) and
 * launch_prefill_megakernel_nvfp4 (NVFP4 layer weights from the 208-byte table, NVFP4 LM head;
 * megakernel/kernel_gb10_nvfp4.cu:2127-2145).  All run the same kernels as launch_prefill_bf16; NVFP4 layer
 * matrices are dequantised to bf16 scratch one layer ahead of their GEMMs (that rounding to bf16 is the one
 * place where the prefill is less exact than the NVFP4 decode kernel).  Scratch arguments are accepted and
 * ignored.  The first two carry no max_seq_len: the cache stride comes from mk_set_prefill_max_seq_len
 * (default 2048).  The mk_* forms take the model dimensions explicitly. */
void mk_set_prefill_max_seq_len(int max_seq_len);
int launch_prefill_bf16_mega(
    const int *token_ids, int seq_len, int *output_token,
    const void *embed_weight, const MkLayerWeights *layers, const void *final_norm_w, const void *lm_head_w,
    void *fa_k_cache, void *fa_v_cache, void *dn_states, void *conv_bufs,
    void *hidden, void *residual, void *normalized, void *proj_buf, void *proj_buf2, void *attn_buf, void *mlp_buf,
    void *dn_out_buf, void *beta_buf, void *alpha_buf, void *final_normed, void *hidden_bf16_out,
    void *lm_bmv, void *lm_bmi, cudaStream_t stream);
int launch_prefill_bf16_nvfp4_lm(
    const int *token_ids, int seq_len, int *output_token,
    const void *embed_weight, const MkLayerWeights *layers, const void *fused_layers,
    const void *final_norm_w, const void *lm_head_w, const void *lm_head_weight_packed, const void *lm_head_scales,
    void *fa_k_cache, void *fa_v_cache, void *dn_states, void *conv_bufs,
    void *hidden, void *residual, void *normalized,
    void *proj_buf, void *proj_buf2, void *proj_buf_half, void *proj_act_packed, void *proj_act_scales,
    void *attn_buf, void *mlp_buf, void *dn_out_buf, void *beta_buf, void *alpha_buf,
    void *final_normed, void *hidden_bf16_out, void *lm_bmv, void *lm_bmi,
    void *lm_hidden_bf16, void *lm_hidden_packed, void *lm_hidden_scales, void *lm_logits_f16, cudaStream_t stream);
int launch_prefill_megakernel_nvfp4(
    const int *token_ids, int seq_len, int *output_token_id,
    const void *embed_weight, const void *layer_weights, const void *final_norm_weight,
    const void *lm_head_weight_packed, const void *lm_head_scales,
    void *lm_hidden_bf16, void *lm_hidden_packed, void *lm_hidden_scales, void *lm_logits_f16,
    void *fa_k_cache, void *fa_v_cache, void *dn_states, void *conv_bufs,
    void *hidden_buffer, void *g_activations, void *g_residual,
    void *g_qkv_scratch, void *g_kv_scratch, void *g_attn_out,
    void *g_mlp_inter, void *g_z_scratch, void *g_beta_scratch, void *g_alpha_scratch, void *g_normalized,
    unsigned int *barrier_counter, unsigned int *barrier_generation,
    float *block_max_vals, int *block_max_idxs, unsigned int *lm_sync_counter,
    int max_seq_len, int group_size, cudaStream_t stream);
int mk_prefill_bf16_nvfp4_lm(
    const int *token_ids, int seq_len, int *output_token,
    const void *embed_weight, const MkLayerWeights *layers, const void *final_norm_w,
    const void *lm_head_weight_packed, const void *lm_head_scales,
    void *fa_k_cache, void *fa_v_cache, void *dn_states, void *conv_bufs,
    void *final_normed, void *hidden_bf16_out,
    int max_seq_len, int num_layers, int vocab, cudaStream_t stream);
int mk_prefill_nvfp4(
    const int *token_ids, int seq_len, int *output_token,
    const void *embed_weight, const void *layers, const void *final_norm_w,
    const void *lm_head_weight_packed, const void *lm_head_scales,
    void *fa_k_cache, void *fa_v_cache, void *dn_states, void *conv_bufs,
    void *final_normed, void *hidden_bf16_out,
    int max_seq_len, int group_size, int num_layers, int vocab, cudaStream_t stream);
/* Which form of the gated delta rule the prefill uses: 1 (default) = chunks of 64 tokens on the tensor cores
 * (reference: the chunked kernels megakernel/prefill.cu:355-680), 0 = token-serial recurrence
 * (reference: megakernel/prefill.cu:114-221).  Both give the same result up to rounding. */
void mk_prefill_set_scan_mode(int chunked);
/* Dense prefill attention kernel: 1 = tcgen05 / TMEM kernel, 0 = mma.sync kernel (the block-sparse mode always
 * uses the mma.sync kernel).  Both compute softmax(q k^T / 16) v * sigmoid(gate). */
void mk_prefill_set_attention_impl(int tcgen05);
/* Elementwise steps folded into the projection kernels of the bf16 prefill: 1 = both (default), 0 = kernels of their
 * own, 2 = SwiGLU only, 3 = RMSNorm only.
 *   SwiGLU of the MLP (reference: megakernel/prefill.cu:1239-1247) inside the epilogue of the gate|up product, the
 *   [S, 7168] intermediate never reaching memory (fused gate|up matrix only);
 *   the RMSNorm after the out / o / down projections (megakernel/prefill.cu:72-88) inside the kernel that adds the
 *   K parts of those products (prompts short enough for the products to be split along K);
 *   with the SwiGLU setting, the qkv and the z projection of a DeltaNet layer also run as one launch over both weight
 *   matrices (the tiles of the two products, side by side).
 * Both settings give the same bits: the folded forms round where the separate kernels read rounded values. */
void mk_prefill_set_fused_swiglu(int on);
/* Status word of the prefill kernels on the current device (synchronises the device): 0 = every bounded wait
 * inside the kernels completed; 1 / 2 / 3 = a wait ran out in a GEMM / the chunk scan / the attention kernel
 * (the affected prefill's results are invalid). */
int mk_prefill_status(void);
/* The prefill keeps a host copy of each layer pointer table it has seen (keyed by device and table address), as
 * the reference does (megakernel/prefill.cu:1578-1584).  Call this after rewriting a table in place. */
void mk_prefill_forget_tables(void);

/* Block-sparse attention for long prompts (off by default: dense causal attention).  Attention runs over
 * 128 x 128 blocks; per query head and query block the kept key blocks are the first `sink` blocks, the `window`
 * most recent ones (the diagonal included) and the ceil(top_frac * causal blocks) best by
 * mean-pooled q . mean-pooled k (ties to the lower index).  Structure after the reference's selection
 * (reference: dflash/src/flashprefill_select.cpp:27-84, dflash/src/flashprefill_kernels.cu:57-90,130-219);
 * the benchmark's rule is sink 1, window 4, top_frac 0.10. */
int mk_prefill_set_block_sparse(int enable, double top_frac, int window, int sink);
/* The two building blocks on their own.  qkv: bf16 [S][5120] = 8 x [q | gate] | k | v with q normalised and
 * rotated; k_cache / v_cache: bf16 [2][max_seq_len][256]; mask: uint32 [8][B][ceil(B/32)], B = ceil(S/128), one bit per
 * key block (null in mk_attention_prefill = dense); out: bf16 [S][2048] = softmax(q k^T / 16) v * sigmoid(gate);
 * scratch: mk_block_select_scratch_bytes(S) bytes of device memory. */
int mk_block_select(const void *qkv, const void *k_cache, int seq_len, int max_seq_len, double top_frac, int window,
                    int sink, unsigned int *mask_out, void *scratch, cudaStream_t stream);
size_t mk_block_select_scratch_bytes(int seq_len);
/* The same scores under the reference's own keep rule (dflash/src/flashprefill_select.cpp:27-84, block_select_host):
 * per query head and query block m the kept causal key blocks n <= m are n < sink, m - n < window, every block when
 * m >= blocks - last_n_full, and score(m, n) >= alpha * max over n <= m of score(m, n) (one f32 multiply, compared
 * with >=).  scores_out (optional, device): f32 [8][blocks][blocks], entries n <= m written -- the scores the rule
 * saw, so that a caller can replay the decision.  mk_prefill_set_block_sparse_threshold selects this rule for
 * the prefill ops (mk_prefill_set_block_sparse switches back to the ranking rule). */
int mk_block_select_threshold(const void *qkv, const void *k_cache, int seq_len, int max_seq_len, float alpha,
                              int window, int sink, int last_n_full, unsigned int *mask_out, float *scores_out,
                              void *scratch, cudaStream_t stream);
int mk_prefill_set_block_sparse_threshold(int enable, float alpha, int window, int sink, int last_n_full);
int mk_attention_prefill(const void *qkv, const void *k_cache, const void *v_cache, void *out, int seq_len,
                         int max_seq_len, const unsigned int *mask, cudaStream_t stream);

/* The prefill projection GEMM on its own: C[M,N] = A[M,K] . W[N,K]^T (+ residual[M,N]), bf16 row-major,
 * f32 accumulation (tcgen05 / TMEM / TMA).  Replaces the cublasGemmEx call of the reference prefill
 * (reference: megakernel/prefill.cu:1526-1534).  N % 128 == 0, K % 64 == 0, 16-byte aligned pointers. */
int mk_gemm_bf16_tn(const void *A, const void *W, void *C, const void *residual, int M, int N, int K,
                    cudaStream_t stream);

/* Prefill with NVFP4 weights and NVFP4 activations: the input of every projection (normed hidden state, DeltaNet /
 * attention output, SwiGLU output) is quantised per 16 values along K with E4M3 block scales (the arithmetic of
 * launch_quantize_nvfp4_lm_out, no tensor scale) and multiplied with the tensor-scale NVFP4 weights by
 * mk_gemm_nvfp4_tn's kernel; no bf16 copy of a weight matrix is made.  The reference's NVFP4 prefill dequantises
 * every matrix to bf16 scratch and calls cuBLAS (megakernel/kernel_gb10_nvfp4.cu:2127-2145); its Blackwell prefill
 * keeps bf16 weights (megakernel/prefill_bw.cu:1036-1171).  layer_weights: the 224-byte entries of mk_decode_nvfp4_ts
 * with each matrix's scale slot pointing at the quantiser's 128 x 4 scale tiles instead of plain rows; beta / alpha
 * projections, norms and the convolution stay bf16.  Outputs and state as mk_prefill_bf16.  vocab % 128 == 0. */
int mk_prefill_nvfp4_mma(
    const int *token_ids, int seq_len, int *output_token,
    const void *embed_weight, const void *layer_weights, const void *final_norm_weight,
    const void *lm_head_packed, const void *lm_head_scales_tiled,
    void *fa_k_cache, void *fa_v_cache, void *dn_states, void *conv_bufs,
    void *final_normed, void *hidden_bf16_out,
    int max_seq_len, int num_layers, int vocab, cudaStream_t stream);

/* Prompt compression for speculative prefill, with this model as its own drafter (the reference's pflash drafter scores
 * a long prompt with a small model and keeps the chunks the last tokens attend to: dflash/src/qwen3_drafter.cpp:86-183,
 * tail attention in dflash/src/qwen3_0p6b_graph.cpp:430-496).
 * mk_prefill_set_tail_scoring(n, buf): later prefill calls of more than n tokens also fill buf [n][seq_len] (device
 *   f32) with running_max[t][j] = max over attention layers and query heads of softmax_j(q_t . k_j / 16), t = the last n
 *   prompt positions, keys j <= position of t (0 beyond); n = 0 or buf = NULL switches it off.  Works with the dense
 *   and the block-sparse prefill (mk_prefill_set_block_sparse), which is how a long prompt is scored cheaply.
 * mk_drafter_select (host arrays): mean over the n rows, average-pool smoothing over pool_kernel positions, mean per
 *   chunk of chunk_size positions, the max(1, int(n_chunks * keep_ratio)) best chunks (equal means: lower chunk first);
 *   writes the kept token positions in ascending order, returns their count (-1: bad argument). */
void mk_prefill_set_tail_scoring(int n_lookahead, float *running_max);
int mk_drafter_select(const float *running_max, int n_lookahead, int seq_len, float keep_ratio, int chunk_size,
                      int pool_kernel, int *kept_positions_out);

/* NVFP4 x NVFP4 product on the block-scaled tensor-core path (tcgen05.mma kind::mxf4nvf4, E4M3 scales per 16 values
 * read from tensor memory): C[M,N] = a_tensor_scale[0] * w_tensor_scale[0] * (A[M,K] . W[N,K]^T) (+ residual), C and
 * residual bf16 row-major.  Both operands in the format mk_quantize_nvfp4_tensor_scale writes (packed e2m1 rows, 128 x 4
 * scale tiles, device fp32 tensor scale); an operand with M % 128 != 0 is quantised from a zero-padded copy, so that
 * its scale array covers whole 128-row blocks.  No counterpart in the reference, which dequantises NVFP4 weights to
 * bf16 for cuBLAS in prefill (megakernel/kernel_gb10_nvfp4.cu:2127-2145) and multiplies them on mma.sync in decode
 * (megakernel/kernel_gb10_nvfp4.cu:528-552).  N % 128 == 0, K % 256 == 0, 16-byte aligned pointers.
 * mk_gemm_nvfp4_status: 0, or 1 after a bounded wait inside the kernel ran out (synchronises the device). */
int mk_gemm_nvfp4_tn(const void *a_packed, const void *a_scales, const float *a_tensor_scale, const void *w_packed,
                     const void *w_scales, const float *w_tensor_scale, void *C, const void *residual, int M, int N, int K,
                     cudaStream_t stream);
int mk_gemm_nvfp4_status(void);

/* launch_decode for a host loop that needs every token at once (the reference's Decoder.step(),
 * megakernel/model.py:278-293, reads the token back with .item() after each launch): the kernel also writes the token
 * and a ticket into mapped pinned memory and this call returns when the ticket has arrived, without a device-to-host
 * copy or a stream synchronisation.  Arguments as launch_decode (minus the scratch the kernel never used);
 * *next_token_out is host memory; output_token_id (device) is written as well. */
int mk_decode_step_host(
    int input_token_id, int *output_token_id, int *next_token_out,
    const void *embed_weight, const MkLayerWeights *layer_weights,
    const void *final_norm_weight, const void *lm_head_weight,
    void *fa_k_cache, void *fa_v_cache, void *dn_states, void *conv_bufs,
    void *hidden_buffer,
    void *g_qkv_scratch, void *g_kv_scratch, void *g_attn_out,
    void *g_mlp_inter, void *g_z_scratch, void *g_beta_scratch,
    void *g_alpha_scratch, void *g_normalized,
    float *seen_token_mask, float repetition_penalty,
    int position, int max_seq_len, cudaStream_t stream);

/* Model depth and vocabulary the entry points assume (defaults 24 and 248320, the
 * compile-time constants of the reference: megakernel/kernel.cu:20,22).  Reduced values let
 * the parity tests run the same kernels on a small model.  num_layers in [1,24]; the layer
 * types are read from the pointer table. */
int mk_set_model_dims(int num_layers, int vocab);
void mk_get_model_dims(int *num_layers, int *vocab);

/* Status of the last device-side failure on the current device (0 = none) and a text for the
 * last error returned on this thread.  mk_clear_error() re-arms the library after a timeout. */
int mk_device_status(void);
/* The whole status word: bits 0-7 the code mk_device_status() returns, 8-11 the phase of the kernel's schedule in
 * which the first wait gave up (0 DeltaNet in-proj, 1 recurrence, 2 out-proj, 3 attention qkv-proj, 4 attention, 5 o-proj,
 * 6 gate/up, 7 down, 8 LM head), 12-22 the layer, 23 set when it was the weight-streaming warp, 24-31 the step of the launch. */
unsigned int mk_device_status_detail(void);
const char *mk_last_error_string(void);
void mk_clear_error(void);

/* mk_decode_many_bf16 / launch_decode_many_nvfp4 run all their steps in ONE persistent launch
 *   (the argmax of a step reaches the next step's embedding gather through the library workspace); a positive
 *   value cuts a call into launches of at most that many steps (1 = one launch per token, as the reference's
 *   launch_decode_many_nvfp4 does, megakernel/kernel_gb10_nvfp4.cu:2192-2257).  For measurements; default 0. */
void mk_set_decode_steps_per_launch(int steps);

/* Limits of the decode kernel's device-side waits.  The reference's grid barrier spins without a limit
 * (megakernel/kernel.cu:128-137); here every wait is bounded and a launch that gives up drains, writes -1 as its
 * token and leaves a status (ST codes: 1 = a poll of an exchanged activation ran out, 2 = a ring barrier, 3 =
 * misaligned source) that the next call reports as MK_ERR_DEVICE_TIMEOUT until mk_clear_error().
 * poll_cycles: SM clocks a poll may take; mbar_tries: attempts on a ring barrier; 0 restores the default
 * (about 2 s each).
 * mk_selftest_bounded_wait launches two small CTAs that run the kernel's poll on a word nobody writes, so that
 * the wait runs out after the configured limit and the whole failure path (status word, error return, re-arm)
 * can be exercised without a launch that hangs: set a short limit first (1e6 cycles is about 0.5 ms). */
void mk_set_wait_limits(unsigned long long poll_cycles, unsigned int mbar_tries);
int mk_selftest_bounded_wait(cudaStream_t stream);

/* Sampling at the LM-head boundary.  The reference decodes greedily; its hook here is the repetition penalty on the
 * logits before the argmax (megakernel/kernel.cu:793-795).
 * mk_set_logits_buffer: every decode entry point of this library also stores the step's logits (f32 [vocab], after the
 *   penalty; the last step's for a multi-step call) into `logits` while it takes the argmax; NULL switches it off.
 * mk_sample_top_k: draws a token from softmax(logits / temperature) restricted to the top_k largest logits (ties to
 *   the lower index; top_k <= 0 keeps everything; temperature <= 0 or top_k == 1 is the argmax) as
 *   argmax_i( logit_i / temperature - log(-log(u_i)) ) with u_i a hash of (seed, counter, i): exact categorical
 *   sampling, reproducible from (seed, counter).  token_out: device int32[1], e.g. the token buffer the next
 *   launch_decode_nvfp4 / mk_decode_many_bf16 call reads its input from. */
void mk_set_logits_buffer(float *logits);
int mk_sample_top_k(const float *logits, int n, float temperature, int top_k, unsigned long long seed,
                    unsigned long long counter, int *token_out, cudaStream_t stream);
/* The same with a nucleus cut after top_k, in the order of the sampler chain of the reference's speculative-decoding
 * driver (top_k -> softmax(logit / temperature) -> top_p -> draw; dflash/test/test_dflash.cpp:127-188): of the set
 * top_k keeps, in descending logit order, the shortest prefix whose probability mass reaches top_p stays (the
 * element that crosses it included; logits equal to it all stay); top_p <= 0 or >= 1 cuts nothing.  The draw is
 * the Gumbel-max rule above over what is left (the reference draws by inverse CDF from a Mersenne twister: the
 * two agree in distribution, not draw for draw). */
int mk_sample_top_k_top_p(const float *logits, int n, float temperature, int top_k, float top_p,
                          unsigned long long seed, unsigned long long counter, int *token_out, cudaStream_t stream);
const char *mk_sample_error(void);

/* Optional per-phase timeline: `buf` is a device buffer of
 * query_max_safe_decode_blocks() * slots_per_cta uint64; thread 0 of every CTA appends the global
 * timer at four points of each phase (barrier entry, barrier exit, activations staged, rows done)
 * and stops at slots_per_cta entries.  Pass NULL to switch it off. */
void mk_set_trace_buffer(unsigned long long *buf, int slots_per_cta);

/* One greedy decode step that allocates nothing.  No counterpart in the reference.
 *
 * For hosts that cannot let a library allocate device memory: a server that gave all free HBM
 * to its own pool at start-up (a later cudaMalloc fails), or a latency-critical loop that cannot
 * take the device-wide synchronisation of cudaMalloc / cudaFree.  Same kernel and same results
 * as launch_decode(), but the activation exchange buffers, argmax partials and attention partials
 * live in a static __device__ array inside the library (about 300 KB on every GPU that loads it, held
 * until the process exits) instead of a workspace allocated on first use; the call makes no
 * cudaMalloc / cudaFree / cudaHostAlloc and no allocating library call.  The caller passes all
 * inputs, outputs and the activation scratch vectors, as for launch_decode(); the model depth
 * and vocabulary are arguments here instead of mk_set_model_dims() state.
 *
 * Limits: the array is sized for grids of at most MK_STATIC_SCRATCH_MAX_CTAS CTAs (one per SM)
 * and num_layers <= 24; anything beyond is refused with MK_ERR_BAD_ARG and a message from
 * mk_decode_bf16_static_scratch_error().
 * First call on a device: resolves the array's device address (cudaGetSymbolAddress) and sizes
 * the grid, with that device current; make that call before any stream capture.
 * Sharing: every call on a device uses the same array and finds the previous call's contents
 * there; the entry point clears the control words it needs at zero on `stream` before the
 * launch.  Two calls that overlap on the GPU (different streams) race on the array: serialise
 * them.  Pointer alignment: 16 bytes for weights, caches, states and the vector scratch, as for launch_decode().
 * Failure: if a bounded device-side wait runs out, the launch drains and writes -1 to *output_token_id; the
 * cause stays in the array until the next call clears it and can be fetched, again without an allocation, with
 * mk_decode_bf16_static_scratch_status(): it queues a 4-byte copy of that word (0 = normal completion) to
 * status_out (device or pinned host memory) on `stream`. */
#define MK_STATIC_SCRATCH_MAX_CTAS 256
int mk_decode_bf16_static_scratch(
    int input_token_id, int *output_token_id,
    const void *embed_weight, const MkLayerWeights *layer_weights,
    const void *final_norm_weight, const void *lm_head_weight,
    void *fa_k_cache, void *fa_v_cache,
    void *dn_states, void *conv_bufs,
    void *hidden_buffer,
    void *g_qkv_scratch, void *g_kv_scratch, void *g_attn_out,
    void *g_mlp_inter, void *g_z_scratch, void *g_beta_scratch,
    void *g_alpha_scratch, void *g_normalized,
    float *seen_token_mask, float repetition_penalty,
    int position, int max_seq_len, int num_layers, int vocab, cudaStream_t stream);
int mk_decode_bf16_static_scratch_status(unsigned int *status_out, cudaStream_t stream);
const char *mk_decode_bf16_static_scratch_error(void);

#ifdef __cplusplus
}
#endif
#endif /* LUCE_MEGAKERNEL_B200_H */
