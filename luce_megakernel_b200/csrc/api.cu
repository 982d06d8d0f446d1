// C ABI: argument validation, per-device workspace, launch bookkeeping.
#include <stdio.h>
#include <string.h>

#include "../../include/luce_megakernel_b200.h"
#include "mk_common.cuh"
#include "mk_decode.h"
#include "mk_prefill.h"

namespace {

constexpr int MAX_DEVICES = 64;

struct DeviceState {
    mk::DecodeWorkspace* ws = nullptr;
    uint32_t* host_status = nullptr;      // mapped pinned block: word 0 = status the kernels write on failure,
                                          // words 4, 5 = {token, ticket} of mk_decode_step_host
    uint32_t* host_status_dev = nullptr;  // its device alias
    uint32_t ticket = 0;                  // last ticket handed to a launch
    int max_grid = 0;
};

DeviceState g_dev[MAX_DEVICES];
int g_blocks_override = 0;
int g_num_layers = mk::MAX_LAYERS;
int g_vocab = mk::DEFAULT_VOCAB;
float* g_logits = nullptr;
unsigned long long* g_trace = nullptr;
int g_trace_slots = 0;
unsigned long long g_poll_limit = mk::DEFAULT_POLL_LIMIT_CYCLES;
uint32_t g_mbar_tries = mk::DEFAULT_MBAR_LIMIT_TRIES;
int g_steps_per_launch = 0;     // 0 = a multi-step call is one launch
thread_local char g_err[256] = "";

int set_err(int code, const char* what, cudaError_t e = cudaSuccess) {
    if (e != cudaSuccess) snprintf(g_err, sizeof(g_err), "%s: %s", what, cudaGetErrorString(e));
    else snprintf(g_err, sizeof(g_err), "%s", what);
    return code;
}

// Workspace of the current device; allocated and zeroed on first use (synchronous, once).
int device_state(DeviceState** out) {
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return set_err(MK_ERR_CUDA, "cudaGetDevice", e);
    if (dev < 0 || dev >= MAX_DEVICES) return set_err(MK_ERR_BAD_ARG, "device index out of range");
    DeviceState& d = g_dev[dev];
    if (!d.ws) {
        e = cudaMalloc(&d.ws, sizeof(mk::DecodeWorkspace));
        if (e != cudaSuccess) return set_err(MK_ERR_CUDA, "cudaMalloc(workspace)", e);
        e = cudaMemset(d.ws, 0, sizeof(mk::DecodeWorkspace));
        if (e != cudaSuccess) return set_err(MK_ERR_CUDA, "cudaMemset(workspace)", e);
        e = cudaHostAlloc(&d.host_status, 16 * sizeof(uint32_t), cudaHostAllocMapped);
        if (e != cudaSuccess) return set_err(MK_ERR_CUDA, "cudaHostAlloc(status)", e);
        memset(d.host_status, 0, 16 * sizeof(uint32_t));
        e = cudaHostGetDevicePointer(&d.host_status_dev, d.host_status, 0);
        if (e != cudaSuccess) return set_err(MK_ERR_CUDA, "cudaHostGetDevicePointer", e);
        d.max_grid = mk::decode_max_grid();
        if (d.max_grid < mk::MIN_GRID) return set_err(MK_ERR_CUDA, "decode kernel needs at least 129 co-resident CTAs (one per SM)");
    }
    *out = &d;
    return MK_OK;
}

bool misaligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) != 0; }

int decode_grid(const DeviceState& d) {
    int g = d.max_grid;
    if (g_blocks_override > 0 && g_blocks_override < g) g = g_blocks_override;
    if (g < mk::MIN_GRID) g = mk::MIN_GRID;    // smaller grids would not fit a phase into the ring bookkeeping
    return g;
}

int check_device_status(DeviceState& d, cudaStream_t stream) {
    const uint32_t st = *reinterpret_cast<volatile uint32_t*>(d.host_status);
    if (st == 0) return MK_OK;
    snprintf(g_err, sizeof(g_err),
             "a previous launch gave up on a bounded device-side wait (status %u, %s warp, layer %u, phase %u, step %u); "
             "call mk_clear_error()", st & 0xffu, (st & 0x800000u) ? "weight-streaming" : "consumer", (st >> 12) & 0x7ffu,
             (st >> 8) & 0xfu, st >> 24);
    (void)stream;
    return MK_ERR_DEVICE_TIMEOUT;
}

struct DecodeCall {
    const void *embed, *final_norm, *lm_head;
    const MkLayerWeights* layers;
    void *k_cache, *v_cache, *dn_states, *conv_bufs, *hidden;
    void *qkv, *kv, *attn_out, *mlp_inter, *z, *beta, *alpha, *normalized;
    float* seen;
    float penalty;
    int position, max_seq_len;
};

int validate(const DecodeCall& a) {
    const void* req[] = {a.embed, a.final_norm, a.lm_head, a.layers, a.k_cache, a.v_cache, a.dn_states, a.conv_bufs,
                         a.hidden, a.qkv, a.kv, a.attn_out, a.mlp_inter, a.z, a.beta, a.alpha, a.normalized};
    for (const void* p : req)
        if (!p) return set_err(MK_ERR_BAD_ARG, "null pointer argument");
    const void* al[] = {a.embed, a.final_norm, a.lm_head, a.layers, a.k_cache, a.v_cache, a.dn_states, a.conv_bufs,
                        a.hidden, a.qkv, a.kv, a.attn_out, a.mlp_inter, a.z, a.normalized};
    for (const void* p : al)
        if (misaligned16(p)) return set_err(MK_ERR_BAD_ARG, "pointer argument is not 16-byte aligned");
    if (a.max_seq_len <= 0) return set_err(MK_ERR_BAD_ARG, "max_seq_len must be positive");
    if (a.position < 0 || a.position >= a.max_seq_len) return set_err(MK_ERR_BAD_ARG, "position out of range");
    if (!(a.penalty >= 1.0f) && a.penalty != 0.0f) return set_err(MK_ERR_BAD_ARG, "repetition_penalty must be >= 1");
    return MK_OK;
}

mk::DecodeParams make_params(const DecodeCall& a, DeviceState& d) {
    mk::DecodeParams p;
    memset(&p, 0, sizeof(p));
    p.embed = a.embed; p.layers = a.layers;
    p.final_norm = a.final_norm; p.lm_head = a.lm_head;
    p.k_cache = a.k_cache; p.v_cache = a.v_cache;
    p.dn_states = (float*)a.dn_states; p.conv_bufs = (float*)a.conv_bufs;
    p.hidden = a.hidden;
    p.qkv = (float*)a.qkv; p.kv = (float*)a.kv; p.attn_out = (float*)a.attn_out; p.mlp_inter = (float*)a.mlp_inter;
    p.z = (float*)a.z; p.beta = (float*)a.beta; p.alpha = (float*)a.alpha; p.normalized = (float*)a.normalized;
    p.seen_mask = a.seen; p.rep_penalty = a.penalty;
    p.position = a.position; p.max_seq_len = a.max_seq_len;
    p.num_layers = g_num_layers; p.vocab = g_vocab;
    p.ws = d.ws; p.host_status = d.host_status_dev; p.trace = g_trace; p.trace_slots = g_trace_slots;
    p.poll_limit_cycles = g_poll_limit; p.mbar_limit_tries = g_mbar_tries;
    p.steps = 1; p.logits_out = g_logits;
    return p;
}

}  // namespace

extern "C" {

int launch_decode(
    int input_token_id, int* output_token_id,
    const void* embed_weight, const MkLayerWeights* layer_weights,
    const void* final_norm_weight, const void* lm_head_weight,
    void* fa_k_cache, void* fa_v_cache, void* dn_states, void* conv_bufs,
    void* hidden_buffer, void* g_activations, void* g_residual,
    void* g_qkv_scratch, void* g_kv_scratch, void* g_attn_out,
    void* g_mlp_inter, void* g_z_scratch, void* g_beta_scratch,
    void* g_alpha_scratch, void* g_normalized,
    unsigned int* barrier_counter, unsigned int* barrier_generation,
    float* block_max_vals, int* block_max_idxs, unsigned int* lm_sync_counter,
    float* seen_token_mask, float repetition_penalty,
    int position, int max_seq_len, cudaStream_t stream) {
    (void)g_activations; (void)g_residual; (void)barrier_counter; (void)barrier_generation;
    (void)block_max_vals; (void)block_max_idxs; (void)lm_sync_counter;
    DecodeCall a{embed_weight, final_norm_weight, lm_head_weight, layer_weights,
                 fa_k_cache, fa_v_cache, dn_states, conv_bufs, hidden_buffer,
                 g_qkv_scratch, g_kv_scratch, g_attn_out, g_mlp_inter, g_z_scratch, g_beta_scratch, g_alpha_scratch,
                 g_normalized, seen_token_mask, repetition_penalty, position, max_seq_len};
    if (!output_token_id) return set_err(MK_ERR_BAD_ARG, "null output_token_id");
    if (input_token_id < 0 || input_token_id >= g_vocab) return set_err(MK_ERR_BAD_ARG, "input_token_id out of range");
    int rc = validate(a);
    if (rc) return rc;
    DeviceState* d = nullptr;
    if ((rc = device_state(&d))) return rc;
    if ((rc = check_device_status(*d, stream))) return rc;
    mk::DecodeParams p = make_params(a, *d);
    p.token_ptr = nullptr; p.token_val = input_token_id; p.out_token = output_token_id;
    mk::fill_rope(p);
    cudaError_t e = mk::launch_decode_kernel(p, decode_grid(*d), stream);
    if (e != cudaSuccess) return set_err(MK_ERR_CUDA, "decode launch", e);
    return MK_OK;
}

// launch_decode for a host loop that needs the token at once: the kernel also writes the token and a ticket into
// mapped pinned memory, and this call spins on the ticket instead of paying a device-to-host copy and a stream
// synchronisation.  Same arguments as launch_decode; *next_token_out receives the token (host memory).
int mk_decode_step_host(
    int input_token_id, int* output_token_id, int* next_token_out,
    const void* embed_weight, const MkLayerWeights* layer_weights,
    const void* final_norm_weight, const void* lm_head_weight,
    void* fa_k_cache, void* fa_v_cache, void* dn_states, void* conv_bufs,
    void* hidden_buffer,
    void* g_qkv_scratch, void* g_kv_scratch, void* g_attn_out,
    void* g_mlp_inter, void* g_z_scratch, void* g_beta_scratch,
    void* g_alpha_scratch, void* g_normalized,
    float* seen_token_mask, float repetition_penalty,
    int position, int max_seq_len, cudaStream_t stream) {
    DecodeCall a{embed_weight, final_norm_weight, lm_head_weight, layer_weights,
                 fa_k_cache, fa_v_cache, dn_states, conv_bufs, hidden_buffer,
                 g_qkv_scratch, g_kv_scratch, g_attn_out, g_mlp_inter, g_z_scratch, g_beta_scratch, g_alpha_scratch,
                 g_normalized, seen_token_mask, repetition_penalty, position, max_seq_len};
    if (!output_token_id || !next_token_out) return set_err(MK_ERR_BAD_ARG, "null output pointer");
    if (input_token_id < 0 || input_token_id >= g_vocab) return set_err(MK_ERR_BAD_ARG, "input_token_id out of range");
    int rc = validate(a);
    if (rc) return rc;
    DeviceState* d = nullptr;
    if ((rc = device_state(&d))) return rc;
    if ((rc = check_device_status(*d, stream))) return rc;
    mk::DecodeParams p = make_params(a, *d);
    p.token_ptr = nullptr; p.token_val = input_token_id; p.out_token = output_token_id;
    const uint32_t ticket = ++d->ticket ? d->ticket : ++d->ticket;      // never 0
    p.host_token = reinterpret_cast<int*>(d->host_status_dev + 4);
    p.host_ticket = ticket;
    mk::fill_rope(p);
    cudaError_t e = mk::launch_decode_kernel(p, decode_grid(*d), stream);
    if (e != cudaSuccess) return set_err(MK_ERR_CUDA, "decode launch", e);
    volatile uint32_t* hv = d->host_status;
    unsigned n = 0;
    while (hv[5] != ticket) {
        if ((++n & 0xfffu) == 0) {          // every few thousand looks: has the stream finished or failed without a ticket?
            e = cudaStreamQuery(stream);
            if (e == cudaSuccess) { if (hv[5] == ticket) break; return set_err(MK_ERR_CUDA, "decode finished without publishing its token"); }
            if (e != cudaErrorNotReady) return set_err(MK_ERR_CUDA, "decode step", e);
        }
    }
    *next_token_out = (int)hv[4];
    if (hv[0] != 0) return check_device_status(*d, stream);
    return MK_OK;
}

int mk_decode_many_bf16(
    int* token_buffer, int* output_tokens, int steps,
    const void* embed_weight, const MkLayerWeights* layer_weights,
    const void* final_norm_weight, const void* lm_head_weight,
    void* fa_k_cache, void* fa_v_cache, void* dn_states, void* conv_bufs,
    void* hidden_buffer,
    void* g_qkv_scratch, void* g_kv_scratch, void* g_attn_out,
    void* g_mlp_inter, void* g_z_scratch, void* g_beta_scratch,
    void* g_alpha_scratch, void* g_normalized,
    float* seen_token_mask, float repetition_penalty,
    int position, int max_seq_len, cudaStream_t stream) {
    DecodeCall a{embed_weight, final_norm_weight, lm_head_weight, layer_weights,
                 fa_k_cache, fa_v_cache, dn_states, conv_bufs, hidden_buffer,
                 g_qkv_scratch, g_kv_scratch, g_attn_out, g_mlp_inter, g_z_scratch, g_beta_scratch, g_alpha_scratch,
                 g_normalized, seen_token_mask, repetition_penalty, position, max_seq_len};
    if (!token_buffer || !output_tokens) return set_err(MK_ERR_BAD_ARG, "null token buffer");
    if (steps < 0) return set_err(MK_ERR_BAD_ARG, "steps must be non-negative");
    if (steps == 0) return MK_OK;
    int rc = validate(a);
    if (rc) return rc;
    if (position + steps > max_seq_len) return set_err(MK_ERR_BAD_ARG, "position + steps exceeds max_seq_len");
    DeviceState* d = nullptr;
    if ((rc = device_state(&d))) return rc;
    if ((rc = check_device_status(*d, stream))) return rc;
    mk::DecodeParams p = make_params(a, *d);
    const int grid = decode_grid(*d);
    mk::fill_rope(p);
    // one launch runs all the steps (the token travels from the argmax of one step to the embedding of the next
    // through the workspace); mk_set_decode_steps_per_launch() can cut it into shorter launches
    const int per = (g_steps_per_launch > 0) ? g_steps_per_launch : steps;
    for (int s = 0; s < steps; s += per) {
        p.token_ptr = token_buffer; p.token_val = 0;
        p.out_token = output_tokens + s; p.token_feedback = token_buffer;
        p.position = position + s;
        p.steps = (steps - s < per) ? steps - s : per;
        cudaError_t e = mk::launch_decode_kernel(p, grid, stream);
        if (e != cudaSuccess) return set_err(MK_ERR_CUDA, "decode launch", e);
    }
    return MK_OK;
}

// NVFP4 decode step: same kernel schedule with packed e2m1 layer weights (fp16 scales per 32) and
// the LM head in the 16-block E4M3 format; the token is read from device memory.
static int decode_nvfp4_common(const int* token_in, int* token_out, int* token_feedback, const void* embed_weight,
                               const void* layer_weights, const void* final_norm_weight, const void* lm_packed,
                               const void* lm_scales, void* fa_k_cache, void* fa_v_cache, void* dn_states, void* conv_bufs,
                               void* hidden_buffer, void* g_normalized, int position, int max_seq_len, int group_size,
                               int steps, cudaStream_t stream) {
    if (!token_in || !token_out || !embed_weight || !layer_weights || !final_norm_weight || !lm_packed || !lm_scales ||
        !fa_k_cache || !fa_v_cache || !dn_states || !conv_bufs || !hidden_buffer || !g_normalized)
        return set_err(MK_ERR_BAD_ARG, "null pointer argument");
    if (group_size != 32) return set_err(MK_ERR_BAD_ARG, "the NVFP4 decode kernel is built for group_size 32");
    if (g_vocab % 128) return set_err(MK_ERR_BAD_ARG, "the NVFP4 LM-head format needs a vocabulary divisible by 128");
    if (max_seq_len <= 0 || position < 0 || position >= max_seq_len) return set_err(MK_ERR_BAD_ARG, "position out of range");
    if (steps < 1 || position + steps > max_seq_len) return set_err(MK_ERR_BAD_ARG, "position + steps exceeds max_seq_len");
    const void* al[] = {embed_weight, layer_weights, final_norm_weight, lm_packed, fa_k_cache, fa_v_cache, dn_states,
                        conv_bufs, hidden_buffer, g_normalized};
    for (const void* q : al)
        if (misaligned16(q)) return set_err(MK_ERR_BAD_ARG, "pointer argument is not 16-byte aligned");
    DeviceState* d = nullptr;
    int rc = device_state(&d);
    if (rc) return rc;
    if ((rc = check_device_status(*d, stream))) return rc;
    mk::DecodeParams p;
    memset(&p, 0, sizeof(p));
    p.embed = embed_weight; p.layers = layer_weights; p.final_norm = final_norm_weight;
    p.lm_head = lm_packed; p.lm_scales = lm_scales; p.wfmt = 1;
    p.k_cache = fa_k_cache; p.v_cache = fa_v_cache; p.dn_states = (float*)dn_states; p.conv_bufs = (float*)conv_bufs;
    p.hidden = hidden_buffer; p.normalized = (float*)g_normalized;
    p.seen_mask = nullptr; p.rep_penalty = 1.0f;
    p.token_ptr = token_in; p.token_val = 0; p.out_token = token_out; p.token_feedback = token_feedback;
    p.position = position; p.max_seq_len = max_seq_len; p.num_layers = g_num_layers; p.vocab = g_vocab;
    p.ws = d->ws; p.host_status = d->host_status_dev; p.trace = nullptr; p.trace_slots = 0;
    p.poll_limit_cycles = g_poll_limit; p.mbar_limit_tries = g_mbar_tries;
    p.steps = steps; p.logits_out = g_logits;
    mk::fill_rope(p);
    cudaError_t e = mk::launch_decode_kernel(p, decode_grid(*d), stream);
    if (e != cudaSuccess) return set_err(MK_ERR_CUDA, "decode launch", e);
    return MK_OK;
}

int launch_decode_nvfp4(
    const int* input_token_ptr, int* output_token_id,
    const void* embed_weight, const void* layer_weights, const void* final_norm_weight,
    const void* lm_head_weight_packed, const void* lm_head_scales,
    void* lm_hidden_bf16, void* lm_hidden_packed, void* lm_hidden_scales, void* lm_logits_f16,
    void* fa_k_cache, void* fa_v_cache, void* dn_states, void* conv_bufs,
    void* hidden_buffer, void* g_activations, void* g_residual,
    void* g_qkv_scratch, void* g_kv_scratch, void* g_attn_out,
    void* g_mlp_inter, void* g_z_scratch, void* g_beta_scratch,
    void* g_alpha_scratch, void* g_normalized,
    unsigned int* barrier_counter, unsigned int* barrier_generation,
    float* block_max_vals, int* block_max_idxs, unsigned int* lm_sync_counter,
    int position, int max_seq_len, int group_size, cudaStream_t stream) {
    (void)lm_hidden_bf16; (void)lm_hidden_packed; (void)lm_hidden_scales; (void)lm_logits_f16; (void)g_activations;
    (void)g_residual; (void)g_qkv_scratch; (void)g_kv_scratch; (void)g_attn_out; (void)g_mlp_inter; (void)g_z_scratch;
    (void)g_beta_scratch; (void)g_alpha_scratch; (void)barrier_counter; (void)barrier_generation; (void)block_max_vals;
    (void)block_max_idxs; (void)lm_sync_counter;
    return decode_nvfp4_common(input_token_ptr, output_token_id, nullptr, embed_weight, layer_weights, final_norm_weight,
                               lm_head_weight_packed, lm_head_scales, fa_k_cache, fa_v_cache, dn_states, conv_bufs,
                               hidden_buffer, g_normalized, position, max_seq_len, group_size, 1, stream);
}

int launch_decode_many_nvfp4(
    int* token_buffer, int* output_tokens, int steps,
    const void* embed_weight, const void* layer_weights, const void* final_norm_weight,
    const void* lm_head_weight_packed, const void* lm_head_scales,
    void* lm_hidden_bf16, void* lm_hidden_packed, void* lm_hidden_scales, void* lm_logits_f16,
    void* fa_k_cache, void* fa_v_cache, void* dn_states, void* conv_bufs,
    void* hidden_buffer, void* g_activations, void* g_residual,
    void* g_qkv_scratch, void* g_kv_scratch, void* g_attn_out,
    void* g_mlp_inter, void* g_z_scratch, void* g_beta_scratch,
    void* g_alpha_scratch, void* g_normalized,
    unsigned int* barrier_counter, unsigned int* barrier_generation,
    float* block_max_vals, int* block_max_idxs, unsigned int* lm_sync_counter,
    int position, int max_seq_len, int group_size, cudaStream_t stream) {
    (void)lm_hidden_bf16; (void)lm_hidden_packed; (void)lm_hidden_scales; (void)lm_logits_f16; (void)g_activations;
    (void)g_residual; (void)g_qkv_scratch; (void)g_kv_scratch; (void)g_attn_out; (void)g_mlp_inter; (void)g_z_scratch;
    (void)g_beta_scratch; (void)g_alpha_scratch; (void)barrier_counter; (void)barrier_generation; (void)block_max_vals;
    (void)block_max_idxs; (void)lm_sync_counter;
    if (!output_tokens) return set_err(MK_ERR_BAD_ARG, "null output_tokens");
    if (steps < 0) return set_err(MK_ERR_BAD_ARG, "steps must be non-negative");
    if (position + steps > max_seq_len) return set_err(MK_ERR_BAD_ARG, "position + steps exceeds max_seq_len");
    if (steps == 0) return MK_OK;
    // one launch: step s writes output_tokens[s] and the running token back into token_buffer
    return decode_nvfp4_common(token_buffer, output_tokens, token_buffer, embed_weight, layer_weights,
                               final_norm_weight, lm_head_weight_packed, lm_head_scales, fa_k_cache, fa_v_cache,
                               dn_states, conv_bufs, hidden_buffer, g_normalized, position, max_seq_len,
                               group_size, steps, stream);
}

// Decode on the NVFP4 format with a per-tensor scale (16-element blocks, E4M3 block scales in plain rows, fp32 scale
// per matrix): `steps` greedy steps in one launch, token in / out through device memory.
int mk_decode_nvfp4_ts(
    int* token_buffer, int* output_tokens, int steps,
    const void* embed_weight, const void* layer_weights, const void* final_norm_weight,
    const void* lm_head_packed, const void* lm_head_scales_rows, const float* lm_head_tensor_scale,
    void* fa_k_cache, void* fa_v_cache, void* dn_states, void* conv_bufs,
    void* hidden_buffer, void* g_normalized, int position, int max_seq_len, cudaStream_t stream) {
    if (!token_buffer || !output_tokens || !embed_weight || !layer_weights || !final_norm_weight || !lm_head_packed ||
        !lm_head_scales_rows || !lm_head_tensor_scale || !fa_k_cache || !fa_v_cache || !dn_states || !conv_bufs ||
        !hidden_buffer || !g_normalized)
        return set_err(MK_ERR_BAD_ARG, "null pointer argument");
    if (steps < 0) return set_err(MK_ERR_BAD_ARG, "steps must be non-negative");
    if (steps == 0) return MK_OK;
    if (max_seq_len <= 0 || position < 0 || position + steps > max_seq_len)
        return set_err(MK_ERR_BAD_ARG, "position + steps exceeds max_seq_len");
    const void* al[] = {embed_weight, layer_weights, final_norm_weight, lm_head_packed, lm_head_scales_rows, fa_k_cache,
                        fa_v_cache, dn_states, conv_bufs, hidden_buffer, g_normalized};
    for (const void* q : al)
        if (misaligned16(q)) return set_err(MK_ERR_BAD_ARG, "pointer argument is not 16-byte aligned");
    DeviceState* d = nullptr;
    int rc = device_state(&d);
    if (rc) return rc;
    if ((rc = check_device_status(*d, stream))) return rc;
    mk::DecodeParams p;
    memset(&p, 0, sizeof(p));
    p.embed = embed_weight; p.layers = layer_weights; p.final_norm = final_norm_weight;
    p.lm_head = lm_head_packed; p.lm_scales = lm_head_scales_rows; p.lm_tensor_scale = lm_head_tensor_scale; p.wfmt = 2;
    p.k_cache = fa_k_cache; p.v_cache = fa_v_cache; p.dn_states = (float*)dn_states; p.conv_bufs = (float*)conv_bufs;
    p.hidden = hidden_buffer; p.normalized = (float*)g_normalized;
    p.seen_mask = nullptr; p.rep_penalty = 1.0f;
    p.token_ptr = token_buffer; p.token_val = 0; p.out_token = output_tokens; p.token_feedback = token_buffer;
    p.position = position; p.max_seq_len = max_seq_len; p.num_layers = g_num_layers; p.vocab = g_vocab;
    p.ws = d->ws; p.host_status = d->host_status_dev; p.trace = g_trace; p.trace_slots = g_trace_slots;
    p.poll_limit_cycles = g_poll_limit; p.mbar_limit_tries = g_mbar_tries;
    p.steps = steps; p.logits_out = g_logits;
    mk::fill_rope(p);
    cudaError_t e = mk::launch_decode_kernel(p, decode_grid(*d), stream);
    if (e != cudaSuccess) return set_err(MK_ERR_CUDA, "decode launch", e);
    return MK_OK;
}

// The same decode on the block-scaled tensor cores (tcgen05.mma kind::mxf4nvf4): the table's matrix slots and
// lm_head_images point at per-CTA chunk images (see the header), the activation is expanded into act_terms NVFP4
// residual terms.
int mk_decode_nvfp4_mma(
    int* token_buffer, int* output_tokens, int steps,
    const void* embed_weight, const void* layer_weights, const void* final_norm_weight,
    const void* lm_head_images, int lm_image_chunks, const float* lm_head_tensor_scale,
    void* fa_k_cache, void* fa_v_cache, void* dn_states, void* conv_bufs,
    void* hidden_buffer, void* g_normalized, int position, int max_seq_len, int act_terms, cudaStream_t stream) {
    if (!token_buffer || !output_tokens || !embed_weight || !layer_weights || !final_norm_weight || !lm_head_images ||
        !lm_head_tensor_scale || !fa_k_cache || !fa_v_cache || !dn_states || !conv_bufs || !hidden_buffer || !g_normalized)
        return set_err(MK_ERR_BAD_ARG, "null pointer argument");
    if (steps < 0) return set_err(MK_ERR_BAD_ARG, "steps must be non-negative");
    if (steps == 0) return MK_OK;
    if (max_seq_len <= 0 || position < 0 || position + steps > max_seq_len)
        return set_err(MK_ERR_BAD_ARG, "position + steps exceeds max_seq_len");
    if (act_terms < 1 || act_terms > 8) return set_err(MK_ERR_BAD_ARG, "act_terms must be in [1, 8]");
    const int ctas = mk::decode_image_ctas();
    if (lm_image_chunks < 1 || (long long)lm_image_chunks * 56 * ctas < (long long)g_vocab)
        return set_err(MK_ERR_BAD_ARG, "lm_image_chunks does not cover the vocabulary");
    const void* al[] = {embed_weight, layer_weights, final_norm_weight, lm_head_images, fa_k_cache,
                        fa_v_cache, dn_states, conv_bufs, hidden_buffer, g_normalized};
    for (const void* q : al)
        if (misaligned16(q)) return set_err(MK_ERR_BAD_ARG, "pointer argument is not 16-byte aligned");
    DeviceState* d = nullptr;
    int rc = device_state(&d);
    if (rc) return rc;
    if ((rc = check_device_status(*d, stream))) return rc;
    if (d->max_grid < ctas) return set_err(MK_ERR_BAD_ARG, "the device cannot co-schedule the 148 CTAs the chunk images are cut for");
    mk::DecodeParams p;
    memset(&p, 0, sizeof(p));
    p.embed = embed_weight; p.layers = layer_weights; p.final_norm = final_norm_weight;
    p.lm_head = lm_head_images; p.lm_image_chunks = lm_image_chunks; p.lm_tensor_scale = lm_head_tensor_scale; p.wfmt = 3;
    p.act_terms = act_terms;
    p.k_cache = fa_k_cache; p.v_cache = fa_v_cache; p.dn_states = (float*)dn_states; p.conv_bufs = (float*)conv_bufs;
    p.hidden = hidden_buffer; p.normalized = (float*)g_normalized;
    p.seen_mask = nullptr; p.rep_penalty = 1.0f;
    p.token_ptr = token_buffer; p.token_val = 0; p.out_token = output_tokens; p.token_feedback = token_buffer;
    p.position = position; p.max_seq_len = max_seq_len; p.num_layers = g_num_layers; p.vocab = g_vocab;
    p.ws = d->ws; p.host_status = d->host_status_dev; p.trace = g_trace; p.trace_slots = g_trace_slots;
    p.poll_limit_cycles = g_poll_limit; p.mbar_limit_tries = g_mbar_tries;
    p.steps = steps; p.logits_out = g_logits;
    mk::fill_rope(p);
    cudaError_t e = mk::launch_decode_kernel(p, ctas, stream);
    if (e != cudaSuccess) return set_err(MK_ERR_CUDA, "decode launch", e);
    return MK_OK;
}

void set_decode_blocks_override(int blocks) { g_blocks_override = blocks < 0 ? 0 : blocks; }

int query_max_safe_decode_blocks(void) {
    DeviceState* d = nullptr;
    if (device_state(&d)) return 1;
    return d->max_grid;
}

int mk_set_model_dims(int num_layers, int vocab) {
    if (num_layers < 1 || num_layers > mk::MAX_LAYERS) return set_err(MK_ERR_BAD_ARG, "num_layers must be in [1,24]");
    if (vocab < 1) return set_err(MK_ERR_BAD_ARG, "vocab must be positive");
    g_num_layers = num_layers;
    g_vocab = vocab;
    return MK_OK;
}

void mk_get_model_dims(int* num_layers, int* vocab) {
    if (num_layers) *num_layers = g_num_layers;
    if (vocab) *vocab = g_vocab;
}

int mk_device_status(void) {
    DeviceState* d = nullptr;
    if (device_state(&d)) return -1;
    return (int)(*reinterpret_cast<volatile uint32_t*>(d->host_status) & 0xffu);
}

unsigned int mk_device_status_detail(void) {
    DeviceState* d = nullptr;
    if (device_state(&d)) return 0xffffffffu;
    return *reinterpret_cast<volatile uint32_t*>(d->host_status);
}

const char* mk_last_error_string(void) { return g_err; }

void mk_clear_error(void) {
    DeviceState* d = nullptr;
    if (device_state(&d)) return;
    cudaDeviceSynchronize();
    cudaMemset(d->ws, 0, sizeof(mk::DecodeWorkspace));
    *d->host_status = 0;
    g_err[0] = 0;
}

static int* g_nvfp4_gemm_err = nullptr;

int mk_gemm_bf16_tn(const void* A, const void* W, void* C, const void* residual, int M, int N, int K,
                    cudaStream_t stream) {
    if (!A || !W || !C) return set_err(MK_ERR_BAD_ARG, "null pointer argument");
    static int* err_flag = nullptr;
    if (!err_flag) {
        cudaError_t e0 = cudaMalloc(&err_flag, sizeof(int));
        if (e0 != cudaSuccess) return set_err(MK_ERR_CUDA, "cudaMalloc(gemm status)", e0);
        cudaMemset(err_flag, 0, sizeof(int));
    }
    cudaError_t e = mk::gemm_bf16_tn(A, W, C, residual, M, N, K, K, N, err_flag, nullptr, 0, stream);
    if (e == cudaErrorInvalidValue) return set_err(MK_ERR_BAD_ARG, "gemm shape or alignment not supported (N % 128, K % 64, 16-byte pointers)");
    if (e != cudaSuccess) return set_err(MK_ERR_CUDA, "gemm launch", e);
    return MK_OK;
}

int mk_gemm_nvfp4_tn(const void* a_packed, const void* a_scales, const float* a_tensor_scale, const void* w_packed,
                     const void* w_scales, const float* w_tensor_scale, void* C, const void* residual, int M, int N, int K,
                     cudaStream_t stream) {
    if (!a_packed || !a_scales || !a_tensor_scale || !w_packed || !w_scales || !w_tensor_scale || !C)
        return set_err(MK_ERR_BAD_ARG, "null pointer argument");
    static int* err_flag = nullptr;
    if (!err_flag) {
        cudaError_t e0 = cudaMalloc(&err_flag, sizeof(int));
        if (e0 != cudaSuccess) return set_err(MK_ERR_CUDA, "cudaMalloc(gemm status)", e0);
        cudaMemset(err_flag, 0, sizeof(int));
    }
    cudaError_t e = mk::gemm_nvfp4_tn(a_packed, a_scales, a_tensor_scale, w_packed, w_scales, w_tensor_scale, C, residual, M, N, K,
                                      N, err_flag, stream);
    if (e == cudaErrorInvalidValue)
        return set_err(MK_ERR_BAD_ARG, "nvfp4 gemm shape or alignment not supported (N % 128, K % 256, 16-byte pointers)");
    if (e != cudaSuccess) return set_err(MK_ERR_CUDA, "nvfp4 gemm launch", e);
    g_nvfp4_gemm_err = err_flag;
    return MK_OK;
}

int mk_gemm_nvfp4_status(void) {
    if (!g_nvfp4_gemm_err) return 0;
    int v = 0;
    if (cudaMemcpy(&v, g_nvfp4_gemm_err, sizeof(int), cudaMemcpyDeviceToHost) != cudaSuccess) return -1;
    return v;
}

void mk_set_decode_steps_per_launch(int steps) { g_steps_per_launch = steps > 0 ? steps : 0; }

void mk_set_wait_limits(unsigned long long poll_cycles, unsigned int mbar_tries) {
    g_poll_limit = poll_cycles ? poll_cycles : mk::DEFAULT_POLL_LIMIT_CYCLES;
    g_mbar_tries = mbar_tries ? mbar_tries : mk::DEFAULT_MBAR_LIMIT_TRIES;
}

int mk_selftest_bounded_wait(cudaStream_t stream) {
    DeviceState* d = nullptr;
    int rc = device_state(&d);
    if (rc) return rc;
    mk::DecodeParams p;
    memset(&p, 0, sizeof(p));
    p.ws = d->ws; p.host_status = d->host_status_dev;
    p.poll_limit_cycles = g_poll_limit; p.mbar_limit_tries = g_mbar_tries;
    cudaError_t e = mk::launch_wait_selftest(p, stream);
    if (e != cudaSuccess) return set_err(MK_ERR_CUDA, "wait self-test launch", e);
    return MK_OK;
}

void mk_set_logits_buffer(float* logits) { g_logits = logits; }

void mk_set_trace_buffer(unsigned long long* buf, int slots_per_cta) {
    g_trace = (buf && slots_per_cta > 0) ? buf : nullptr;
    g_trace_slots = g_trace ? slots_per_cta : 0;
}

}  // extern "C"
