// PyTorch op surface over the C ABI.  Registers, in the namespace the reference's Python
// drivers call (torch.ops.qwen35_megakernel_bf16_C), ops with the reference's schemas
// (reference: megakernel/torch_bindings.cpp:568-601), so megakernel/model.py-style callers run
// unchanged.  Every op validates its tensors, forwards raw device pointers and the current
// CUDA stream to libluce_megakernel_b200.so and turns a non-zero status into an exception.
#include <Python.h>
#include <c10/cuda/CUDAStream.h>
#include <torch/all.h>
#include <torch/library.h>

#include "../../include/luce_megakernel_b200.h"

namespace {

using torch::Tensor;

void need(const Tensor& t, const char* name, c10::ScalarType dt, int64_t min_numel) {
    TORCH_CHECK(t.defined(), name, " is undefined");
    TORCH_CHECK(t.is_cuda(), name, " must be a CUDA tensor");
    TORCH_CHECK(t.is_contiguous(), name, " must be contiguous");
    TORCH_CHECK(t.scalar_type() == dt, name, " has dtype ", t.scalar_type(), ", expected ", dt);
    TORCH_CHECK(t.numel() >= min_numel, name, " has ", t.numel(), " elements, needs at least ", min_numel);
}

void check_status(int rc, const char* op) {
    TORCH_CHECK(rc == MK_OK, "qwen35_megakernel_bf16_C::", op, " failed (", rc, "): ", mk_last_error_string());
}

cudaStream_t current_stream(const Tensor& t) { return c10::cuda::getCurrentCUDAStream(t.get_device()).stream(); }

struct DeviceGuard {
    int prev = -1;
    explicit DeviceGuard(const Tensor& t) {
        cudaGetDevice(&prev);
        if (prev != t.get_device()) cudaSetDevice(t.get_device());
    }
    ~DeviceGuard() {
        int cur = -1;
        cudaGetDevice(&cur);
        if (cur != prev && prev >= 0) cudaSetDevice(prev);
    }
};

void decode(Tensor output_token, int64_t input_token_id, Tensor embed_weight, Tensor layer_weights_packed,
            Tensor final_norm_weight, Tensor lm_head_weight, Tensor fa_k_cache, Tensor fa_v_cache, Tensor dn_states,
            Tensor conv_bufs, Tensor hidden_buffer, Tensor activations, Tensor residual, Tensor qkv_scratch,
            Tensor kv_scratch, Tensor attn_out, Tensor mlp_inter, Tensor z_scratch, Tensor beta_scratch,
            Tensor alpha_scratch, Tensor normalized, Tensor barrier_counter, Tensor barrier_generation,
            Tensor block_max_vals, Tensor block_max_idxs, Tensor lm_sync_counter, Tensor seen_token_mask,
            double repetition_penalty, int64_t position, int64_t max_seq_len) {
    const auto bf16 = torch::kBFloat16;
    const auto f32 = torch::kFloat32;
    need(output_token, "output_token", torch::kInt32, 1);
    need(embed_weight, "embed_weight", bf16, 1024);
    need(layer_weights_packed, "layer_weights_packed", torch::kUInt8, 128);
    need(final_norm_weight, "final_norm_weight", bf16, 1024);
    need(lm_head_weight, "lm_head_weight", bf16, 1024);
    need(fa_k_cache, "fa_k_cache", bf16, 2 * max_seq_len * 256);
    need(fa_v_cache, "fa_v_cache", bf16, 2 * max_seq_len * 256);
    need(dn_states, "dn_states", f32, 16 * 128 * 128);
    need(conv_bufs, "conv_bufs", f32, 6144 * 4);
    need(hidden_buffer, "hidden_buffer", bf16, 1024);
    need(qkv_scratch, "qkv_scratch", f32, 6144);
    need(kv_scratch, "kv_scratch", f32, 1024);
    need(attn_out, "attn_out", f32, 2048);
    need(mlp_inter, "mlp_inter", f32, 3584);
    need(z_scratch, "z_scratch", f32, 2048);
    need(beta_scratch, "beta_scratch", f32, 16);
    need(alpha_scratch, "alpha_scratch", f32, 16);
    need(normalized, "normalized", f32, 1024);
    if (repetition_penalty > 1.0) need(seen_token_mask, "seen_token_mask", f32, embed_weight.size(0));
    TORCH_CHECK(embed_weight.dim() == 2 && embed_weight.size(1) == 1024, "embed_weight must be [vocab, 1024]");
    TORCH_CHECK(layer_weights_packed.numel() % 128 == 0, "layer_weights_packed must hold 128-byte entries");
    DeviceGuard guard(embed_weight);
    check_status(mk_set_model_dims((int)(layer_weights_packed.numel() / 128), (int)embed_weight.size(0)), "decode");
    const int rc = launch_decode(
        (int)input_token_id, (int*)output_token.data_ptr(), embed_weight.data_ptr(),
        (const MkLayerWeights*)layer_weights_packed.data_ptr(), final_norm_weight.data_ptr(),
        lm_head_weight.data_ptr(), fa_k_cache.data_ptr(), fa_v_cache.data_ptr(), dn_states.data_ptr(),
        conv_bufs.data_ptr(), hidden_buffer.data_ptr(), activations.defined() ? activations.data_ptr() : nullptr,
        residual.defined() ? residual.data_ptr() : nullptr, qkv_scratch.data_ptr(), kv_scratch.data_ptr(),
        attn_out.data_ptr(), mlp_inter.data_ptr(), z_scratch.data_ptr(), beta_scratch.data_ptr(),
        alpha_scratch.data_ptr(), normalized.data_ptr(), nullptr, nullptr, nullptr, nullptr, nullptr,
        seen_token_mask.defined() ? (float*)seen_token_mask.data_ptr() : nullptr, (float)repetition_penalty,
        (int)position, (int)max_seq_len, current_stream(embed_weight));
    check_status(rc, "decode");
    (void)barrier_counter; (void)barrier_generation; (void)block_max_vals; (void)block_max_idxs; (void)lm_sync_counter;
}

void prefill_bf16(Tensor output_token, Tensor token_ids, Tensor embed_weight, Tensor layer_weights_packed,
                  Tensor final_norm_weight, Tensor lm_head_weight, Tensor fa_k_cache, Tensor fa_v_cache,
                  Tensor dn_states, Tensor conv_bufs, Tensor hidden, Tensor residual, Tensor normalized,
                  Tensor proj_buf, Tensor proj_buf2, Tensor attn_buf, Tensor mlp_buf, Tensor dn_out_buf,
                  Tensor beta_buf, Tensor alpha_buf, Tensor dn_pre_qkv, Tensor dn_u_scratch, Tensor dn_w_scratch,
                  Tensor dn_cs_scratch, Tensor fused_fa_qkv, Tensor fused_gate_up, Tensor final_normed,
                  Tensor hidden_bf16_out, Tensor lm_bmv, Tensor lm_bmi, int64_t max_seq_len) {
    const auto bf16 = torch::kBFloat16;
    const auto f32 = torch::kFloat32;
    need(output_token, "output_token", torch::kInt32, 1);
    need(token_ids, "token_ids", torch::kInt32, 1);
    TORCH_CHECK(token_ids.dim() == 1, "token_ids must be 1-D");
    need(embed_weight, "embed_weight", bf16, 1024);
    need(layer_weights_packed, "layer_weights_packed", torch::kUInt8, 128);
    need(final_norm_weight, "final_norm_weight", bf16, 1024);
    need(lm_head_weight, "lm_head_weight", bf16, 1024);
    need(fa_k_cache, "fa_k_cache", bf16, 2 * max_seq_len * 256);
    need(fa_v_cache, "fa_v_cache", bf16, 2 * max_seq_len * 256);
    need(dn_states, "dn_states", f32, 16 * 128 * 128);
    need(conv_bufs, "conv_bufs", f32, 6144 * 4);
    need(fused_fa_qkv, "fused_fa_qkv", bf16, 5120 * 1024);
    need(fused_gate_up, "fused_gate_up", bf16, 7168 * 1024);
    need(final_normed, "final_normed", bf16, 1024);
    need(hidden_bf16_out, "hidden_bf16_out", bf16, 1024);
    TORCH_CHECK(token_ids.size(0) <= max_seq_len, "prompt longer than max_seq_len");
    DeviceGuard guard(embed_weight);
    check_status(mk_set_model_dims((int)(layer_weights_packed.numel() / 128), (int)embed_weight.size(0)), "prefill_bf16");
    const int rc = launch_prefill_bf16(
        (const int*)token_ids.data_ptr(), (int)token_ids.size(0), (int*)output_token.data_ptr(), embed_weight.data_ptr(),
        (const MkLayerWeights*)layer_weights_packed.data_ptr(), final_norm_weight.data_ptr(), lm_head_weight.data_ptr(),
        fa_k_cache.data_ptr(), fa_v_cache.data_ptr(), dn_states.data_ptr(), conv_bufs.data_ptr(), nullptr, nullptr,
        nullptr, nullptr, nullptr, nullptr, nullptr, nullptr, nullptr, nullptr, nullptr, nullptr, nullptr, nullptr,
        fused_fa_qkv.data_ptr(), fused_gate_up.data_ptr(), final_normed.data_ptr(), hidden_bf16_out.data_ptr(), nullptr,
        nullptr, (int)max_seq_len, current_stream(embed_weight));
    TORCH_CHECK(rc == MK_OK, "qwen35_megakernel_bf16_C::prefill_bf16 failed (", rc, "): ", mk_prefill_error());
    (void)hidden; (void)residual; (void)normalized; (void)proj_buf; (void)proj_buf2; (void)attn_buf; (void)mlp_buf;
    (void)dn_out_buf; (void)beta_buf; (void)alpha_buf; (void)dn_pre_qkv; (void)dn_u_scratch; (void)dn_w_scratch;
    (void)dn_cs_scratch; (void)lm_bmv; (void)lm_bmi;
}

// NVFP4 decode ops (reference: megakernel/torch_bindings.cpp:182-270): the token is seeded into
// device memory on the current stream, then the C ABI is called with the reference's argument list.
static void seed_token(const Tensor& buf, int token_id) {
    const cudaError_t e = cudaMemcpyAsync(buf.data_ptr(), &token_id, sizeof(int), cudaMemcpyHostToDevice,
                                          current_stream(buf));
    TORCH_CHECK(e == cudaSuccess, "cudaMemcpyAsync(token) failed: ", cudaGetErrorString(e));
}

#define MK_NVFP4_TENSOR_ARGS                                                                                       \
    Tensor embed_weight, Tensor layer_weights_packed, Tensor final_norm_weight, Tensor lm_head_weight_packed,      \
    Tensor lm_head_scales, Tensor lm_hidden_bf16, Tensor lm_hidden_packed, Tensor lm_hidden_scales,                \
    Tensor lm_logits_f16, Tensor fa_k_cache, Tensor fa_v_cache, Tensor dn_states, Tensor conv_bufs,                \
    Tensor hidden_buffer, Tensor activations, Tensor residual, Tensor qkv_scratch, Tensor kv_scratch,              \
    Tensor attn_out, Tensor mlp_inter, Tensor z_scratch, Tensor beta_scratch, Tensor alpha_scratch,                \
    Tensor normalized, Tensor barrier_counter, Tensor barrier_generation, Tensor block_max_vals,                   \
    Tensor block_max_idxs, Tensor lm_sync_counter, int64_t position, int64_t max_seq_len, int64_t group_size

static void check_nvfp4_common(const Tensor& embed_weight, const Tensor& layer_weights_packed, const Tensor& final_norm_weight,
                               const Tensor& lm_packed, const Tensor& lm_scales, const Tensor& fa_k_cache,
                               const Tensor& fa_v_cache, const Tensor& dn_states, const Tensor& conv_bufs,
                               const Tensor& hidden_buffer, const Tensor& normalized, int64_t max_seq_len, const char* op) {
    need(embed_weight, "embed_weight", torch::kBFloat16, 1024);
    need(layer_weights_packed, "layer_weights_packed", torch::kUInt8, 208);
    TORCH_CHECK(layer_weights_packed.numel() % 208 == 0, "layer_weights_packed must hold 208-byte entries");
    need(final_norm_weight, "final_norm_weight", torch::kBFloat16, 1024);
    need(lm_packed, "lm_head_weight_packed", torch::kUInt8, 512);
    need(lm_scales, "lm_head_scales", torch::kUInt8, 512);
    need(fa_k_cache, "fa_k_cache", torch::kBFloat16, 2 * max_seq_len * 256);
    need(fa_v_cache, "fa_v_cache", torch::kBFloat16, 2 * max_seq_len * 256);
    need(dn_states, "dn_states", torch::kFloat32, 16 * 128 * 128);
    need(conv_bufs, "conv_bufs", torch::kFloat32, 6144 * 4);
    need(hidden_buffer, "hidden_buffer", torch::kBFloat16, 1024);
    need(normalized, "normalized", torch::kFloat32, 1024);
    check_status(mk_set_model_dims((int)(layer_weights_packed.numel() / 208), (int)embed_weight.size(0)), op);
}

void decode_nvfp4(Tensor output_token, int64_t input_token_id, MK_NVFP4_TENSOR_ARGS) {
    need(output_token, "output_token", torch::kInt32, 1);
    DeviceGuard guard(embed_weight);
    check_nvfp4_common(embed_weight, layer_weights_packed, final_norm_weight, lm_head_weight_packed, lm_head_scales,
                       fa_k_cache, fa_v_cache, dn_states, conv_bufs, hidden_buffer, normalized, max_seq_len, "decode_nvfp4");
    seed_token(output_token, (int)input_token_id);
    const int rc = launch_decode_nvfp4(
        (const int*)output_token.data_ptr(), (int*)output_token.data_ptr(), embed_weight.data_ptr(),
        layer_weights_packed.data_ptr(), final_norm_weight.data_ptr(), lm_head_weight_packed.data_ptr(),
        lm_head_scales.data_ptr(), nullptr, nullptr, nullptr, nullptr, fa_k_cache.data_ptr(), fa_v_cache.data_ptr(),
        dn_states.data_ptr(), conv_bufs.data_ptr(), hidden_buffer.data_ptr(), nullptr, nullptr, nullptr, nullptr, nullptr,
        nullptr, nullptr, nullptr, nullptr, normalized.data_ptr(), nullptr, nullptr, nullptr, nullptr, nullptr,
        (int)position, (int)max_seq_len, (int)group_size, current_stream(embed_weight));
    check_status(rc, "decode_nvfp4");
}

void decode_many_nvfp4(Tensor output_tokens, Tensor token_buffer, int64_t input_token_id, MK_NVFP4_TENSOR_ARGS) {
    need(output_tokens, "output_tokens", torch::kInt32, 0);
    TORCH_CHECK(output_tokens.dim() == 1, "output_tokens must be 1D");
    need(token_buffer, "token_buffer", torch::kInt32, 1);
    TORCH_CHECK(token_buffer.numel() == 1, "token_buffer must contain exactly one int32 token");
    DeviceGuard guard(embed_weight);
    check_nvfp4_common(embed_weight, layer_weights_packed, final_norm_weight, lm_head_weight_packed, lm_head_scales,
                       fa_k_cache, fa_v_cache, dn_states, conv_bufs, hidden_buffer, normalized, max_seq_len,
                       "decode_many_nvfp4");
    seed_token(token_buffer, (int)input_token_id);
    const int rc = launch_decode_many_nvfp4(
        (int*)token_buffer.data_ptr(), (int*)output_tokens.data_ptr(), (int)output_tokens.numel(), embed_weight.data_ptr(),
        layer_weights_packed.data_ptr(), final_norm_weight.data_ptr(), lm_head_weight_packed.data_ptr(),
        lm_head_scales.data_ptr(), nullptr, nullptr, nullptr, nullptr, fa_k_cache.data_ptr(), fa_v_cache.data_ptr(),
        dn_states.data_ptr(), conv_bufs.data_ptr(), hidden_buffer.data_ptr(), nullptr, nullptr, nullptr, nullptr, nullptr,
        nullptr, nullptr, nullptr, nullptr, normalized.data_ptr(), nullptr, nullptr, nullptr, nullptr, nullptr,
        (int)position, (int)max_seq_len, (int)group_size, current_stream(embed_weight));
    check_status(rc, "decode_many_nvfp4");
}

// The reference's other prefill ops (reference: megakernel/torch_bindings.cpp:409-565, schemas :632-670).
void prefill_bf16_mega(Tensor output_token, Tensor token_ids, Tensor embed_weight, Tensor layer_weights_packed,
                       Tensor final_norm_weight, Tensor lm_head_weight, Tensor fa_k_cache, Tensor fa_v_cache,
                       Tensor dn_states, Tensor conv_bufs, Tensor hidden, Tensor residual, Tensor normalized,
                       Tensor proj_buf, Tensor proj_buf2, Tensor attn_buf, Tensor mlp_buf, Tensor dn_out_buf,
                       Tensor beta_buf, Tensor alpha_buf, Tensor final_normed, Tensor hidden_bf16_out, Tensor lm_bmv,
                       Tensor lm_bmi) {
    need(output_token, "output_token", torch::kInt32, 1);
    need(token_ids, "token_ids", torch::kInt32, 1);
    TORCH_CHECK(token_ids.dim() == 1, "token_ids must be 1-D");
    need(embed_weight, "embed_weight", torch::kBFloat16, 1024);
    need(layer_weights_packed, "layer_weights_packed", torch::kUInt8, 128);
    need(lm_head_weight, "lm_head_weight", torch::kBFloat16, 1024);
    TORCH_CHECK(fa_k_cache.dim() == 4 && fa_k_cache.size(3) == 256, "fa_k_cache must be [layers, 2, max_seq_len, 256]");
    const int64_t max_seq_len = fa_k_cache.size(2);
    need(fa_k_cache, "fa_k_cache", torch::kBFloat16, 2 * max_seq_len * 256);
    need(fa_v_cache, "fa_v_cache", torch::kBFloat16, 2 * max_seq_len * 256);
    need(dn_states, "dn_states", torch::kFloat32, 16 * 128 * 128);
    need(conv_bufs, "conv_bufs", torch::kFloat32, 6144 * 4);
    need(final_normed, "final_normed", torch::kBFloat16, 1024);
    need(hidden_bf16_out, "hidden_bf16_out", torch::kBFloat16, 1024);
    TORCH_CHECK(token_ids.size(0) <= max_seq_len, "prompt longer than the cache");
    DeviceGuard guard(embed_weight);
    check_status(mk_set_model_dims((int)(layer_weights_packed.numel() / 128), (int)embed_weight.size(0)), "prefill_bf16_mega");
    mk_set_prefill_max_seq_len((int)max_seq_len);
    const int rc = launch_prefill_bf16_mega(
        (const int*)token_ids.data_ptr(), (int)token_ids.size(0), (int*)output_token.data_ptr(), embed_weight.data_ptr(),
        (const MkLayerWeights*)layer_weights_packed.data_ptr(), final_norm_weight.data_ptr(), lm_head_weight.data_ptr(),
        fa_k_cache.data_ptr(), fa_v_cache.data_ptr(), dn_states.data_ptr(), conv_bufs.data_ptr(), nullptr, nullptr, nullptr,
        nullptr, nullptr, nullptr, nullptr, nullptr, nullptr, nullptr, final_normed.data_ptr(), hidden_bf16_out.data_ptr(),
        nullptr, nullptr, current_stream(embed_weight));
    TORCH_CHECK(rc == MK_OK, "qwen35_megakernel_bf16_C::prefill_bf16_mega failed (", rc, "): ", mk_prefill_error());
    (void)hidden; (void)residual; (void)normalized; (void)proj_buf; (void)proj_buf2; (void)attn_buf; (void)mlp_buf;
    (void)dn_out_buf; (void)beta_buf; (void)alpha_buf; (void)lm_bmv; (void)lm_bmi;
}

// Batched decode step: no counterpart in the reference (megakernel/torch_bindings.cpp:569-675 are all batch 1).
// State tensors are the reference's with a leading batch dimension; tokens, positions, output_tokens: int32 [batch].
void decode_batch(Tensor output_tokens, Tensor tokens, Tensor positions, Tensor embed_weight, Tensor layer_weights_packed,
                  Tensor final_norm_weight, Tensor lm_head_weight, Tensor fa_k_cache, Tensor fa_v_cache, Tensor dn_states,
                  Tensor conv_bufs, Tensor fused_fa_qkv, Tensor fused_gate_up, Tensor final_normed, Tensor hidden_bf16_out) {
    need(tokens, "tokens", torch::kInt32, 1);
    const int64_t batch = tokens.numel();
    TORCH_CHECK(batch >= 1 && batch <= 16, "batch must be in [1, 16]");
    need(output_tokens, "output_tokens", torch::kInt32, batch);
    need(positions, "positions", torch::kInt32, batch);
    need(embed_weight, "embed_weight", torch::kBFloat16, 1024);
    need(layer_weights_packed, "layer_weights_packed", torch::kUInt8, 128);
    need(lm_head_weight, "lm_head_weight", torch::kBFloat16, 1024);
    TORCH_CHECK(fa_k_cache.dim() == 5 && fa_k_cache.size(0) == batch && fa_k_cache.size(4) == 256,
                "fa_k_cache must be [batch, layers, 2, max_seq_len, 256]");
    const int64_t max_seq_len = fa_k_cache.size(3);
    need(fa_k_cache, "fa_k_cache", torch::kBFloat16, batch * 2 * max_seq_len * 256);
    need(fa_v_cache, "fa_v_cache", torch::kBFloat16, batch * 2 * max_seq_len * 256);
    TORCH_CHECK(fa_v_cache.numel() == fa_k_cache.numel(), "fa_v_cache must have the shape of fa_k_cache");
    TORCH_CHECK(dn_states.dim() == 5 && dn_states.size(0) == batch, "dn_states must be [batch, layers, 16, 128, 128]");
    TORCH_CHECK(conv_bufs.dim() == 4 && conv_bufs.size(0) == batch, "conv_bufs must be [batch, layers, 6144, 4]");
    need(dn_states, "dn_states", torch::kFloat32, batch * 16 * 128 * 128);
    need(conv_bufs, "conv_bufs", torch::kFloat32, batch * 6144 * 4);
    need(fused_fa_qkv, "fused_fa_qkv", torch::kBFloat16, 5120 * 1024);
    need(fused_gate_up, "fused_gate_up", torch::kBFloat16, 7168 * 1024);
    need(final_normed, "final_normed", torch::kBFloat16, batch * 1024);
    need(hidden_bf16_out, "hidden_bf16_out", torch::kBFloat16, batch * 1024);
    DeviceGuard guard(embed_weight);
    const int num_layers = (int)(layer_weights_packed.numel() / 128);
    const int rc = mk_decode_batch(
        (const int*)tokens.data_ptr(), (const int*)positions.data_ptr(), (int*)output_tokens.data_ptr(), (int)batch,
        embed_weight.data_ptr(), (const MkLayerWeights*)layer_weights_packed.data_ptr(), final_norm_weight.data_ptr(),
        lm_head_weight.data_ptr(), fa_k_cache.data_ptr(), fa_v_cache.data_ptr(), dn_states.data_ptr(), conv_bufs.data_ptr(),
        fused_fa_qkv.data_ptr(), fused_gate_up.data_ptr(), final_normed.data_ptr(), hidden_bf16_out.data_ptr(), (int)max_seq_len,
        num_layers, (int)embed_weight.size(0), current_stream(embed_weight));
    TORCH_CHECK(rc == MK_OK, "qwen35_megakernel_bf16_C::decode_batch failed (", rc, "): ", mk_prefill_error());
}

void prefill_megakernel_nvfp4(Tensor output_token, Tensor token_ids, Tensor embed_weight, Tensor layer_weights_packed,
                              Tensor final_norm_weight, Tensor lm_head_weight_packed, Tensor lm_head_scales,
                              Tensor lm_hidden_bf16, Tensor lm_hidden_packed, Tensor lm_hidden_scales, Tensor lm_logits_f16,
                              Tensor fa_k_cache, Tensor fa_v_cache, Tensor dn_states, Tensor conv_bufs, Tensor hidden_buffer,
                              Tensor activations, Tensor residual, Tensor qkv_scratch, Tensor kv_scratch, Tensor attn_out,
                              Tensor mlp_inter, Tensor z_scratch, Tensor beta_scratch, Tensor alpha_scratch, Tensor normalized,
                              Tensor barrier_counter, Tensor barrier_generation, Tensor block_max_vals, Tensor block_max_idxs,
                              Tensor lm_sync_counter, int64_t max_seq_len, int64_t group_size) {
    need(output_token, "output_token", torch::kInt32, 1);
    need(token_ids, "token_ids", torch::kInt32, 1);
    TORCH_CHECK(token_ids.dim() == 1, "token_ids must be 1-D");
    TORCH_CHECK(token_ids.size(0) <= max_seq_len, "prompt longer than max_seq_len");
    DeviceGuard guard(embed_weight);
    check_nvfp4_common(embed_weight, layer_weights_packed, final_norm_weight, lm_head_weight_packed, lm_head_scales, fa_k_cache,
                       fa_v_cache, dn_states, conv_bufs, hidden_buffer, normalized, max_seq_len, "prefill_megakernel_nvfp4");
    const int rc = launch_prefill_megakernel_nvfp4(
        (const int*)token_ids.data_ptr(), (int)token_ids.size(0), (int*)output_token.data_ptr(), embed_weight.data_ptr(),
        layer_weights_packed.data_ptr(), final_norm_weight.data_ptr(), lm_head_weight_packed.data_ptr(), lm_head_scales.data_ptr(),
        nullptr, nullptr, nullptr, nullptr, fa_k_cache.data_ptr(), fa_v_cache.data_ptr(), dn_states.data_ptr(),
        conv_bufs.data_ptr(), hidden_buffer.data_ptr(), nullptr, nullptr, nullptr, nullptr, nullptr, nullptr, nullptr, nullptr,
        nullptr, nullptr, nullptr, nullptr, nullptr, nullptr, nullptr, (int)max_seq_len, (int)group_size,
        current_stream(embed_weight));
    TORCH_CHECK(rc == MK_OK, "qwen35_megakernel_bf16_C::prefill_megakernel_nvfp4 failed (", rc, "): ", mk_prefill_error());
    (void)lm_hidden_bf16; (void)lm_hidden_packed; (void)lm_hidden_scales; (void)lm_logits_f16; (void)activations; (void)residual;
    (void)qkv_scratch; (void)kv_scratch; (void)attn_out; (void)mlp_inter; (void)z_scratch; (void)beta_scratch;
    (void)alpha_scratch; (void)barrier_counter; (void)barrier_generation; (void)block_max_vals; (void)block_max_idxs;
    (void)lm_sync_counter;
}

void prefill_bf16_nvfp4_lm(Tensor output_token, Tensor token_ids, Tensor embed_weight, Tensor layer_weights_packed,
                           Tensor prefill_fused_weights_packed, Tensor final_norm_weight, Tensor lm_head_weight,
                           Tensor lm_head_weight_packed, Tensor lm_head_scales, Tensor fa_k_cache, Tensor fa_v_cache,
                           Tensor dn_states, Tensor conv_bufs, Tensor hidden, Tensor residual, Tensor normalized,
                           Tensor proj_buf, Tensor proj_buf2, Tensor proj_buf_half, Tensor proj_act_packed,
                           Tensor proj_act_scales, Tensor attn_buf, Tensor mlp_buf, Tensor dn_out_buf, Tensor beta_buf,
                           Tensor alpha_buf, Tensor final_normed, Tensor hidden_bf16_out, Tensor lm_bmv, Tensor lm_bmi,
                           Tensor lm_hidden_bf16, Tensor lm_hidden_packed, Tensor lm_hidden_scales, Tensor lm_logits_f16) {
    need(output_token, "output_token", torch::kInt32, 1);
    need(token_ids, "token_ids", torch::kInt32, 1);
    TORCH_CHECK(token_ids.dim() == 1, "token_ids must be 1-D");
    need(embed_weight, "embed_weight", torch::kBFloat16, 1024);
    need(layer_weights_packed, "layer_weights_packed", torch::kUInt8, 128);
    need(lm_head_weight_packed, "lm_head_weight_packed", torch::kUInt8, 512);
    need(lm_head_scales, "lm_head_scales", torch::kUInt8, 512);
    TORCH_CHECK(fa_k_cache.dim() == 4 && fa_k_cache.size(3) == 256, "fa_k_cache must be [layers, 2, max_seq_len, 256]");
    const int64_t max_seq_len = fa_k_cache.size(2);
    need(fa_k_cache, "fa_k_cache", torch::kBFloat16, 2 * max_seq_len * 256);
    need(fa_v_cache, "fa_v_cache", torch::kBFloat16, 2 * max_seq_len * 256);
    need(dn_states, "dn_states", torch::kFloat32, 16 * 128 * 128);
    need(conv_bufs, "conv_bufs", torch::kFloat32, 6144 * 4);
    need(final_normed, "final_normed", torch::kBFloat16, 1024);
    need(hidden_bf16_out, "hidden_bf16_out", torch::kBFloat16, 1024);
    TORCH_CHECK(token_ids.size(0) <= max_seq_len, "prompt longer than the cache");
    DeviceGuard guard(embed_weight);
    check_status(mk_set_model_dims((int)(layer_weights_packed.numel() / 128), (int)embed_weight.size(0)), "prefill_bf16_nvfp4_lm");
    mk_set_prefill_max_seq_len((int)max_seq_len);
    const int rc = launch_prefill_bf16_nvfp4_lm(
        (const int*)token_ids.data_ptr(), (int)token_ids.size(0), (int*)output_token.data_ptr(), embed_weight.data_ptr(),
        (const MkLayerWeights*)layer_weights_packed.data_ptr(), nullptr, final_norm_weight.data_ptr(), nullptr,
        lm_head_weight_packed.data_ptr(), lm_head_scales.data_ptr(), fa_k_cache.data_ptr(), fa_v_cache.data_ptr(),
        dn_states.data_ptr(), conv_bufs.data_ptr(), nullptr, nullptr, nullptr, nullptr, nullptr, nullptr, nullptr, nullptr, nullptr,
        nullptr, nullptr, nullptr, nullptr, final_normed.data_ptr(), hidden_bf16_out.data_ptr(), nullptr, nullptr, nullptr, nullptr,
        nullptr, nullptr, current_stream(embed_weight));
    TORCH_CHECK(rc == MK_OK, "qwen35_megakernel_bf16_C::prefill_bf16_nvfp4_lm failed (", rc, "): ", mk_prefill_error());
    (void)prefill_fused_weights_packed; (void)lm_head_weight; (void)hidden; (void)residual; (void)normalized; (void)proj_buf;
    (void)proj_buf2; (void)proj_buf_half; (void)proj_act_packed; (void)proj_act_scales; (void)attn_buf; (void)mlp_buf;
    (void)dn_out_buf; (void)beta_buf; (void)alpha_buf; (void)lm_bmv; (void)lm_bmi; (void)lm_hidden_bf16; (void)lm_hidden_packed;
    (void)lm_hidden_scales; (void)lm_logits_f16;
}

// NVFP4 quantisers (reference: megakernel/torch_bindings.cpp:272-337): same checks, same outputs.
void quantize_nvfp4_out(Tensor packed_out, Tensor scales_out, Tensor weight, int64_t group_size) {
    TORCH_CHECK(weight.is_cuda() && weight.is_contiguous() && weight.dim() == 2, "weight must be a contiguous 2-D CUDA tensor");
    TORCH_CHECK(weight.scalar_type() == torch::kBFloat16, "weight must be bfloat16");
    TORCH_CHECK(group_size > 0 && (group_size % 2) == 0, "group_size must be a positive even integer");
    const int rows = (int)weight.size(0), cols = (int)weight.size(1);
    TORCH_CHECK((cols % 2) == 0 && (cols % group_size) == 0, "in_dim must be divisible by 2 and by group_size");
    need(packed_out, "packed_out", torch::kUInt8, (int64_t)rows * (cols / 2));
    need(scales_out, "scales_out", torch::kFloat16, (int64_t)rows * (cols / group_size));
    TORCH_CHECK(packed_out.numel() == (int64_t)rows * (cols / 2), "packed_out has the wrong size");
    TORCH_CHECK(scales_out.numel() == (int64_t)rows * (cols / group_size), "scales_out has the wrong size");
    DeviceGuard guard(weight);
    const int rc = launch_quantize_nvfp4_out(weight.data_ptr(), rows, cols, (int)group_size, packed_out.data_ptr(),
                                             scales_out.data_ptr(), current_stream(weight));
    TORCH_CHECK(rc == MK_OK, "quantize_nvfp4_out failed: ", mk_quantize_error());
}

void quantize_nvfp4_lm_out(Tensor packed_out, Tensor scales_out, Tensor weight) {
    TORCH_CHECK(weight.is_cuda() && weight.is_contiguous() && weight.dim() == 2, "weight must be a contiguous 2-D CUDA tensor");
    TORCH_CHECK(weight.scalar_type() == torch::kBFloat16, "weight must be bfloat16");
    const int rows = (int)weight.size(0), cols = (int)weight.size(1);
    TORCH_CHECK((rows % 128) == 0, "out_dim must be divisible by 128");
    TORCH_CHECK((cols % 64) == 0, "in_dim must be divisible by 64");
    need(packed_out, "packed_out", torch::kUInt8, (int64_t)rows * (cols / 2));
    need(scales_out, "scales_out", torch::kUInt8, (int64_t)(rows / 128) * (cols / 64) * 512);
    TORCH_CHECK(scales_out.numel() == (int64_t)(rows / 128) * (cols / 64) * 512, "scales_out has the wrong size");
    DeviceGuard guard(weight);
    const int rc = launch_quantize_nvfp4_lm_out(weight.data_ptr(), rows, cols, packed_out.data_ptr(), scales_out.data_ptr(),
                                                current_stream(weight));
    TORCH_CHECK(rc == MK_OK, "quantize_nvfp4_lm_out failed: ", mk_quantize_error());
}

// 16-block / E4M3 / fp32 per-tensor scale: an additional format, the reference's 16-block quantiser has no tensor
// scale (megakernel/kernel_gb10_nvfp4.cu:1373-1437).  Argument order follows quantize_nvfp4_lm_out.
void quantize_nvfp4_tensor_scale_out(Tensor packed_out, Tensor scales_out, Tensor tensor_scale_out, Tensor weight) {
    TORCH_CHECK(weight.is_cuda() && weight.is_contiguous() && weight.dim() == 2, "weight must be a contiguous 2-D CUDA tensor");
    TORCH_CHECK(weight.scalar_type() == torch::kBFloat16, "weight must be bfloat16");
    const int rows = (int)weight.size(0), cols = (int)weight.size(1);
    TORCH_CHECK((rows % 128) == 0, "out_dim must be divisible by 128");
    TORCH_CHECK((cols % 64) == 0, "in_dim must be divisible by 64");
    need(packed_out, "packed_out", torch::kUInt8, (int64_t)rows * (cols / 2));
    need(scales_out, "scales_out", torch::kUInt8, (int64_t)(rows / 128) * (cols / 64) * 512);
    need(tensor_scale_out, "tensor_scale_out", torch::kFloat32, 1);
    DeviceGuard guard(weight);
    const int rc = mk_quantize_nvfp4_tensor_scale(weight.data_ptr(), rows, cols, packed_out.data_ptr(), scales_out.data_ptr(),
                                                  (float*)tensor_scale_out.data_ptr(), current_stream(weight));
    TORCH_CHECK(rc == MK_OK, "quantize_nvfp4_tensor_scale_out failed: ", mk_quantize_error());
}

int64_t max_safe_decode_blocks() { return query_max_safe_decode_blocks(); }

void set_decode_blocks(int64_t blocks) {
    TORCH_CHECK(blocks >= 0, "blocks must be non-negative");
    set_decode_blocks_override((int)blocks);
}

}  // namespace

TORCH_LIBRARY(qwen35_megakernel_bf16_C, ops) {
    ops.def("decode(Tensor output_token, int input_token_id, "
            "Tensor embed_weight, Tensor layer_weights_packed, "
            "Tensor final_norm_weight, Tensor lm_head_weight, "
            "Tensor fa_k_cache, Tensor fa_v_cache, Tensor dn_states, Tensor conv_bufs, "
            "Tensor hidden_buffer, Tensor activations, Tensor residual, "
            "Tensor qkv_scratch, Tensor kv_scratch, Tensor attn_out, "
            "Tensor mlp_inter, Tensor z_scratch, Tensor beta_scratch, "
            "Tensor alpha_scratch, Tensor normalized, "
            "Tensor barrier_counter, Tensor barrier_generation, "
            "Tensor block_max_vals, Tensor block_max_idxs, Tensor lm_sync_counter, "
            "Tensor seen_token_mask, float repetition_penalty, "
            "int position, int max_seq_len) -> ()");
    ops.impl("decode", torch::kCUDA, &decode);

    ops.def("prefill_bf16(Tensor output_token, Tensor token_ids, "
            "Tensor embed_weight, Tensor layer_weights_packed, "
            "Tensor final_norm_weight, Tensor lm_head_weight, "
            "Tensor fa_k_cache, Tensor fa_v_cache, Tensor dn_states, Tensor conv_bufs, "
            "Tensor hidden, Tensor residual, Tensor normalized, "
            "Tensor proj_buf, Tensor proj_buf2, Tensor attn_buf, Tensor mlp_buf, "
            "Tensor dn_out_buf, Tensor beta_buf, Tensor alpha_buf, "
            "Tensor dn_pre_qkv, "
            "Tensor dn_u_scratch, Tensor dn_w_scratch, Tensor dn_cs_scratch, "
            "Tensor fused_fa_qkv, Tensor fused_gate_up, "
            "Tensor final_normed, Tensor hidden_bf16_out, "
            "Tensor lm_bmv, Tensor lm_bmi, int max_seq_len) -> ()");
    ops.impl("prefill_bf16", torch::kCUDA, &prefill_bf16);

    ops.def("max_safe_decode_blocks() -> int");
    ops.impl("max_safe_decode_blocks", &max_safe_decode_blocks);

    ops.def("set_decode_blocks(int blocks) -> ()");
    ops.impl("set_decode_blocks", &set_decode_blocks);

    ops.def("decode_nvfp4(Tensor output_token, int input_token_id, "
            "Tensor embed_weight, Tensor layer_weights_packed, "
            "Tensor final_norm_weight, Tensor lm_head_weight_packed, Tensor lm_head_scales, "
            "Tensor lm_hidden_bf16, Tensor lm_hidden_packed, Tensor lm_hidden_scales, Tensor lm_logits_f16, "
            "Tensor fa_k_cache, Tensor fa_v_cache, Tensor dn_states, Tensor conv_bufs, "
            "Tensor hidden_buffer, Tensor activations, Tensor residual, "
            "Tensor qkv_scratch, Tensor kv_scratch, Tensor attn_out, "
            "Tensor mlp_inter, Tensor z_scratch, Tensor beta_scratch, "
            "Tensor alpha_scratch, Tensor normalized, "
            "Tensor barrier_counter, Tensor barrier_generation, "
            "Tensor block_max_vals, Tensor block_max_idxs, Tensor lm_sync_counter, "
            "int position, int max_seq_len, int group_size) -> ()");
    ops.impl("decode_nvfp4", torch::kCUDA, &decode_nvfp4);

    ops.def("decode_many_nvfp4(Tensor output_tokens, Tensor token_buffer, int input_token_id, "
            "Tensor embed_weight, Tensor layer_weights_packed, "
            "Tensor final_norm_weight, Tensor lm_head_weight_packed, Tensor lm_head_scales, "
            "Tensor lm_hidden_bf16, Tensor lm_hidden_packed, Tensor lm_hidden_scales, Tensor lm_logits_f16, "
            "Tensor fa_k_cache, Tensor fa_v_cache, Tensor dn_states, Tensor conv_bufs, "
            "Tensor hidden_buffer, Tensor activations, Tensor residual, "
            "Tensor qkv_scratch, Tensor kv_scratch, Tensor attn_out, "
            "Tensor mlp_inter, Tensor z_scratch, Tensor beta_scratch, "
            "Tensor alpha_scratch, Tensor normalized, "
            "Tensor barrier_counter, Tensor barrier_generation, "
            "Tensor block_max_vals, Tensor block_max_idxs, Tensor lm_sync_counter, "
            "int position, int max_seq_len, int group_size) -> ()");
    ops.impl("decode_many_nvfp4", torch::kCUDA, &decode_many_nvfp4);

    ops.def("prefill_bf16_mega(Tensor output_token, Tensor token_ids, "
            "Tensor embed_weight, Tensor layer_weights_packed, "
            "Tensor final_norm_weight, Tensor lm_head_weight, "
            "Tensor fa_k_cache, Tensor fa_v_cache, Tensor dn_states, Tensor conv_bufs, "
            "Tensor hidden, Tensor residual, Tensor normalized, "
            "Tensor proj_buf, Tensor proj_buf2, Tensor attn_buf, Tensor mlp_buf, "
            "Tensor dn_out_buf, Tensor beta_buf, Tensor alpha_buf, "
            "Tensor final_normed, Tensor hidden_bf16_out, "
            "Tensor lm_bmv, Tensor lm_bmi) -> ()");
    ops.impl("prefill_bf16_mega", torch::kCUDA, &prefill_bf16_mega);

    ops.def("decode_batch(Tensor output_tokens, Tensor tokens, Tensor positions, "
            "Tensor embed_weight, Tensor layer_weights_packed, "
            "Tensor final_norm_weight, Tensor lm_head_weight, "
            "Tensor fa_k_cache, Tensor fa_v_cache, Tensor dn_states, Tensor conv_bufs, "
            "Tensor fused_fa_qkv, Tensor fused_gate_up, "
            "Tensor final_normed, Tensor hidden_bf16_out) -> ()");
    ops.impl("decode_batch", torch::kCUDA, &decode_batch);

    ops.def("prefill_megakernel_nvfp4(Tensor output_token, Tensor token_ids, "
            "Tensor embed_weight, Tensor layer_weights_packed, "
            "Tensor final_norm_weight, Tensor lm_head_weight_packed, Tensor lm_head_scales, "
            "Tensor lm_hidden_bf16, Tensor lm_hidden_packed, Tensor lm_hidden_scales, Tensor lm_logits_f16, "
            "Tensor fa_k_cache, Tensor fa_v_cache, Tensor dn_states, Tensor conv_bufs, "
            "Tensor hidden_buffer, Tensor activations, Tensor residual, "
            "Tensor qkv_scratch, Tensor kv_scratch, Tensor attn_out, "
            "Tensor mlp_inter, Tensor z_scratch, Tensor beta_scratch, "
            "Tensor alpha_scratch, Tensor normalized, "
            "Tensor barrier_counter, Tensor barrier_generation, "
            "Tensor block_max_vals, Tensor block_max_idxs, Tensor lm_sync_counter, "
            "int max_seq_len, int group_size) -> ()");
    ops.impl("prefill_megakernel_nvfp4", torch::kCUDA, &prefill_megakernel_nvfp4);

    ops.def("prefill_bf16_nvfp4_lm(Tensor output_token, Tensor token_ids, "
            "Tensor embed_weight, Tensor layer_weights_packed, Tensor prefill_fused_weights_packed, "
            "Tensor final_norm_weight, Tensor lm_head_weight, "
            "Tensor lm_head_weight_packed, Tensor lm_head_scales, "
            "Tensor fa_k_cache, Tensor fa_v_cache, Tensor dn_states, Tensor conv_bufs, "
            "Tensor hidden, Tensor residual, Tensor normalized, "
            "Tensor proj_buf, Tensor proj_buf2, Tensor proj_buf_half, Tensor proj_act_packed, Tensor proj_act_scales, "
            "Tensor attn_buf, Tensor mlp_buf, "
            "Tensor dn_out_buf, Tensor beta_buf, Tensor alpha_buf, "
            "Tensor final_normed, Tensor hidden_bf16_out, "
            "Tensor lm_bmv, Tensor lm_bmi, "
            "Tensor lm_hidden_bf16, Tensor lm_hidden_packed, Tensor lm_hidden_scales, Tensor lm_logits_f16) -> ()");
    ops.impl("prefill_bf16_nvfp4_lm", torch::kCUDA, &prefill_bf16_nvfp4_lm);

    ops.def("quantize_nvfp4_out(Tensor packed_out, Tensor scales_out, Tensor weight, int group_size) -> ()");
    ops.impl("quantize_nvfp4_out", torch::kCUDA, &quantize_nvfp4_out);

    ops.def("quantize_nvfp4_lm_out(Tensor packed_out, Tensor scales_out, Tensor weight) -> ()");
    ops.impl("quantize_nvfp4_lm_out", torch::kCUDA, &quantize_nvfp4_lm_out);

    ops.def("quantize_nvfp4_tensor_scale_out(Tensor packed_out, Tensor scales_out, Tensor tensor_scale_out, Tensor weight) -> ()");
    ops.impl("quantize_nvfp4_tensor_scale_out", torch::kCUDA, &quantize_nvfp4_tensor_scale_out);
}

// Importable as a Python module of the same name, like the reference extension
// (reference: megakernel/torch_bindings.cpp:23-28,679).
PyMODINIT_FUNC PyInit_qwen35_megakernel_bf16_C(void) {
    static struct PyModuleDef module = {PyModuleDef_HEAD_INIT, "qwen35_megakernel_bf16_C", nullptr, 0, nullptr};
    return PyModule_Create(&module);
}
