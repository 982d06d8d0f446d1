// Host-visible parameter block and launcher declarations for the bf16 decode megakernel.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

namespace mk {

struct LayerWeights;

constexpr int ATT_MAX_CHUNKS = 16;     // KV chunks per KV head in one decode step
constexpr int ATT_CHUNK_POS = 64;      // target positions per chunk
constexpr int ATT_PART_STRIDE = 260;   // floats per (head, chunk) partial: m, l, 2 pad, o[256]
constexpr int MAX_GRID = 256;

// Library-owned scratch in global memory, zero on entry to every launch.
struct DecodeWorkspace {
    uint32_t bar;        // grid-barrier arrivals of the current launch
    uint32_t lm_count;   // CTAs that have published their argmax partial
    uint32_t abort_flag; // set by the first CTA whose bounded wait ran out
    uint32_t pad[29];
    float argmax_val[MAX_GRID];
    int argmax_idx[MAX_GRID];
    float attn_part[8 * ATT_MAX_CHUNKS * ATT_PART_STRIDE];
};

struct DecodeParams {
    const void* embed;            // bf16 [vocab, 1024]
    const LayerWeights* layers;   // device pointer table
    const void* final_norm;       // bf16 [1024]
    const void* lm_head;          // bf16 [vocab, 1024]
    void* k_cache;                // bf16 [n_fa, 2, max_seq, 256]
    void* v_cache;
    float* dn_states;             // f32 [n_dn, 16, 128(value), 128(key)]
    float* conv_bufs;             // f32 [n_dn, 6144, 4]
    void* hidden;                 // bf16 [1024] residual stream between phases
    float* qkv;                   // f32 [6144]: DeltaNet q|k|v after conv, or attention per-head [q|gate] (4096)
    float* kv;                    // f32 [1024]
    float* attn_out;              // f32 [2048]
    float* mlp_inter;             // f32 [3584]
    float* z;                     // f32 [2048]
    float* beta;                  // f32 [16]
    float* alpha;                 // f32 [16]
    float* normalized;            // f32 [1024] final-normed hidden (output)
    float* seen_mask;             // f32 [vocab] or null
    float rep_penalty;
    const int* token_ptr;         // device token (feedback mode) or null
    int token_val;                // host token when token_ptr is null
    int* out_token;               // int32 [1]
    int* token_feedback;          // optional: also receives the new token
    int* out_tokens_slot;         // optional: also receives the new token
    int position;
    int max_seq_len;
    int num_layers;
    int vocab;
    DecodeWorkspace* ws;
    uint32_t* host_status;        // mapped pinned word, written only on failure
    unsigned long long* trace;    // optional [grid][trace_slots] globaltimer stamps
    int trace_slots;              // entries per CTA in `trace`
};

// Launches the persistent decode kernel (cooperative launch, `grid` CTAs of 544 threads).
cudaError_t launch_decode_kernel(const DecodeParams& p, int grid, cudaStream_t stream);
// Largest grid that is guaranteed co-resident on the current device.
int decode_max_grid();
size_t decode_smem_bytes();

}  // namespace mk
