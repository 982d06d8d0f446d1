// Decode step for callers that must not allocate device memory.
//
// Some hosts of this library cannot let it call cudaMalloc: an inference server that hands all
// free HBM to its own pool at start-up (a later cudaMalloc from a library then fails), or a
// latency-critical decode loop that cannot accept the device-wide synchronisation cudaMalloc and
// cudaFree imply.  launch_decode() keeps its activation exchange buffers, argmax partials and
// attention partials in a workspace it allocates on first use; the entry point below runs the same kernel
// with that scratch placed in a file-scope __device__ array instead, so it allocates nothing:
// no cudaMalloc / cudaFree / cudaHostAlloc and no allocating library call.
//
// The array costs sizeof(DecodeWorkspace) (about 300 KB) on every GPU that loads the library,
// until the process exits, and is sized for grids of at most MK_STATIC_SCRATCH_MAX_CTAS CTAs.
#include <stdio.h>
#include <string.h>

#include "../../include/luce_megakernel_b200.h"
#include "mk_common.cuh"
#include "mk_decode.h"

static_assert(MK_STATIC_SCRATCH_MAX_CTAS == mk::MAX_GRID, "header and kernel disagree on the static scratch size");

// The scratch itself.  In host code this name is only a handle for cudaGetSymbolAddress: it is
// not a device address and must never be passed to a kernel as it stands.
static __device__ __align__(256) unsigned char g_decode_static_scratch[sizeof(mk::DecodeWorkspace)];

namespace {

constexpr int MAX_DEVICES = 64;

struct StaticSetup {
    bool done = false;
    mk::DecodeWorkspace* scratch = nullptr;   // device address of g_decode_static_scratch on this device
    int grid = 0;
};
StaticSetup g_static[MAX_DEVICES];
thread_local char g_static_err[256] = "";

int fail_with(int code, const char* what, cudaError_t e = cudaSuccess) {
    if (e != cudaSuccess) snprintf(g_static_err, sizeof(g_static_err), "%s: %s", what, cudaGetErrorString(e));
    else snprintf(g_static_err, sizeof(g_static_err), "%s", what);
    return code;
}

}  // namespace

extern "C" const char* mk_decode_bf16_static_scratch_error(void) { return g_static_err; }

extern "C" int mk_decode_bf16_static_scratch(
    int input_token_id, int* output_token_id,
    const void* embed_weight, const MkLayerWeights* layer_weights,
    const void* final_norm_weight, const void* lm_head_weight,
    void* fa_k_cache, void* fa_v_cache, void* dn_states, void* conv_bufs,
    void* hidden_buffer,
    void* g_qkv_scratch, void* g_kv_scratch, void* g_attn_out,
    void* g_mlp_inter, void* g_z_scratch, void* g_beta_scratch,
    void* g_alpha_scratch, void* g_normalized,
    float* seen_token_mask, float repetition_penalty,
    int position, int max_seq_len, int num_layers, int vocab, cudaStream_t stream) {
    const void* req[] = {output_token_id, embed_weight, layer_weights, final_norm_weight, lm_head_weight,
                         fa_k_cache, fa_v_cache, dn_states, conv_bufs, hidden_buffer, g_qkv_scratch, g_kv_scratch,
                         g_attn_out, g_mlp_inter, g_z_scratch, g_beta_scratch, g_alpha_scratch, g_normalized};
    for (const void* p : req)
        if (!p) return fail_with(MK_ERR_BAD_ARG, "null pointer argument");
    // the kernel streams weight and cache rows with 16-byte bulk copies and vector loads: same rule as launch_decode()
    const void* al16[] = {embed_weight, layer_weights, final_norm_weight, lm_head_weight, fa_k_cache, fa_v_cache,
                          dn_states, conv_bufs, hidden_buffer, g_qkv_scratch, g_kv_scratch, g_attn_out, g_mlp_inter,
                          g_z_scratch, g_normalized};
    for (const void* p : al16)
        if (reinterpret_cast<uintptr_t>(p) & 15u) return fail_with(MK_ERR_BAD_ARG, "pointer argument is not 16-byte aligned");
    const void* al4[] = {output_token_id, g_beta_scratch, g_alpha_scratch, seen_token_mask};
    for (const void* p : al4)
        if (reinterpret_cast<uintptr_t>(p) & 3u) return fail_with(MK_ERR_BAD_ARG, "pointer argument is not 4-byte aligned");
    if (num_layers < 1 || num_layers > mk::MAX_LAYERS)
        return fail_with(MK_ERR_BAD_ARG, "num_layers beyond the maximum of 24 the static scratch variant is built for");
    if (vocab < 1) return fail_with(MK_ERR_BAD_ARG, "vocab must be positive");
    if (input_token_id < 0 || input_token_id >= vocab) return fail_with(MK_ERR_BAD_ARG, "input_token_id out of range");
    if (max_seq_len <= 0 || position < 0 || position >= max_seq_len)
        return fail_with(MK_ERR_BAD_ARG, "position out of range");
    if (!(repetition_penalty >= 1.0f) && repetition_penalty != 0.0f)
        return fail_with(MK_ERR_BAD_ARG, "repetition_penalty must be >= 1");

    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return fail_with(MK_ERR_CUDA, "cudaGetDevice", e);
    if (dev < 0 || dev >= MAX_DEVICES) return fail_with(MK_ERR_BAD_ARG, "device index out of range");
    StaticSetup& s = g_static[dev];
    if (!s.done) {
        // One-time set-up for this device (it must be the current device): resolve the device
        // address of the scratch array and size the grid.  Do this before any stream capture.
        void* addr = nullptr;
        e = cudaGetSymbolAddress(&addr, g_decode_static_scratch);
        if (e != cudaSuccess) return fail_with(MK_ERR_CUDA, "cudaGetSymbolAddress(static scratch)", e);
        int sms = 0;
        e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
        if (e != cudaSuccess) return fail_with(MK_ERR_CUDA, "cudaDeviceGetAttribute", e);
        const int grid = mk::decode_max_grid();
        if (grid < mk::MIN_GRID) return fail_with(MK_ERR_CUDA, "decode kernel needs at least 129 co-resident CTAs (one per SM)");
        if (sms > MK_STATIC_SCRATCH_MAX_CTAS) {
            snprintf(g_static_err, sizeof(g_static_err),
                     "this device runs %d CTAs; the static scratch holds partial results for at most %d", sms,
                     MK_STATIC_SCRATCH_MAX_CTAS);
            return MK_ERR_BAD_ARG;
        }
        s.scratch = static_cast<mk::DecodeWorkspace*>(addr);
        s.grid = grid;
        s.done = true;
    }

    // Every call shares the array and finds the previous call's contents in it.  Only the
    // control words (argmax arrival count and abort flag: the first 64 bytes) have to start at
    // zero; the launch counter that follows them must persist, and every exchanged value and
    // partial result is written before it is read.
    e = cudaMemsetAsync(s.scratch, 0, 64, stream);
    if (e != cudaSuccess) return fail_with(MK_ERR_CUDA, "cudaMemsetAsync(static scratch)", e);

    mk::DecodeParams p;
    memset(&p, 0, sizeof(p));
    p.embed = embed_weight; p.layers = layer_weights;
    p.final_norm = final_norm_weight; p.lm_head = lm_head_weight;
    p.k_cache = fa_k_cache; p.v_cache = fa_v_cache;
    p.dn_states = (float*)dn_states; p.conv_bufs = (float*)conv_bufs; p.hidden = hidden_buffer;
    p.qkv = (float*)g_qkv_scratch; p.kv = (float*)g_kv_scratch; p.attn_out = (float*)g_attn_out;
    p.mlp_inter = (float*)g_mlp_inter; p.z = (float*)g_z_scratch; p.beta = (float*)g_beta_scratch;
    p.alpha = (float*)g_alpha_scratch; p.normalized = (float*)g_normalized;
    p.seen_mask = seen_token_mask; p.rep_penalty = repetition_penalty;
    p.token_ptr = nullptr; p.token_val = input_token_id; p.out_token = output_token_id;
    p.position = position; p.max_seq_len = max_seq_len; p.num_layers = num_layers; p.vocab = vocab;
    p.ws = s.scratch;
    p.host_status = nullptr;   // the mapped status word of launch_decode would be an allocation
    p.trace = nullptr; p.trace_slots = 0;
    p.poll_limit_cycles = mk::DEFAULT_POLL_LIMIT_CYCLES; p.mbar_limit_tries = mk::DEFAULT_MBAR_LIMIT_TRIES;
    p.steps = 1;
    mk::fill_rope(p);
    e = mk::launch_decode_kernel(p, s.grid, stream);
    if (e != cudaSuccess) return fail_with(MK_ERR_CUDA, "decode launch", e);
    return MK_OK;
}

// Status of the last call on the current device, without an allocation: copies the array's "a wait ran out"
// word (0 = the launch completed normally) to `status_out` on `stream`.  Queue it after the decode call and
// before the next one, which clears the word.
extern "C" int mk_decode_bf16_static_scratch_status(unsigned int* status_out, cudaStream_t stream) {
    if (!status_out) return fail_with(MK_ERR_BAD_ARG, "null status_out");
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return fail_with(MK_ERR_CUDA, "cudaGetDevice", e);
    if (dev < 0 || dev >= MAX_DEVICES || !g_static[dev].done)
        return fail_with(MK_ERR_BAD_ARG, "no static-scratch decode call has run on this device yet");
    e = cudaMemcpyAsync(status_out, &g_static[dev].scratch->abort_flag, sizeof(unsigned int), cudaMemcpyDefault, stream);
    if (e != cudaSuccess) return fail_with(MK_ERR_CUDA, "cudaMemcpyAsync(static scratch status)", e);
    return MK_OK;
}
