// Host-visible parameter block and launcher declarations for the bf16 decode megakernel.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace mk {

struct LayerWeights;

constexpr int ATT_MAX_CHUNKS = 16;     // KV chunks per KV head in one decode step
constexpr int ATT_CHUNK_POS = 64;      // target positions per chunk
constexpr int ATT_PART_STRIDE = 260;   // floats per (head, chunk) partial: m, l, 2 pad, o[256]
constexpr int MAX_GRID = 256;
// Smallest grid the kernel accepts: every phase must fit its rows of one CTA into four ring
// chunks (8224 in-projection rows / 129 CTAs = 64 rows = 4 chunks of 16).
constexpr int MIN_GRID = 129;

// Library-owned scratch in global memory.  Activation vectors travel between CTAs as 64-bit
// words {f32 value, epoch}: a reader spins on the word itself until the epoch matches, so no
// grid barrier and no separate flag are needed.  The epoch is unique per launch and layer
// (derived from `seq`, which the last CTA of every launch increments), so nothing has to be
// cleared between launches; only `lm_count` and `abort_flag` must be zero on entry.
struct DecodeWorkspace {
    uint32_t lm_count;    // CTAs that have published their argmax partial
    uint32_t abort_flag;  // set by the first CTA whose bounded wait ran out
    uint32_t pad0[14];
    uint32_t seq;         // decode steps completed on this workspace
    uint32_t pad1a;
    unsigned long long next_token;   // {token, epoch}: a step's argmax, handed to the next step of the same launch
    uint32_t pad1[12];
    float argmax_val[MAX_GRID];
    int argmax_idx[MAX_GRID];
    uint32_t att_ready[32];                 // per attention unit: epoch once its partials are written
    unsigned long long x_hidden[2][1024];   // residual stream after out-proj [0] / after down-proj [1]
    unsigned long long x_dnin[8224];        // DeltaNet: q|k|v after conv+SiLU, z, beta, decay
    unsigned long long x_o[2048];           // DeltaNet recurrence output
    unsigned long long x_mlp[3584];         // SwiGLU output
    unsigned long long x_fain[5120];        // attention: per head [q|gate], k, v
    float attn_part[8 * ATT_MAX_CHUNKS * ATT_PART_STRIDE];
};

struct DecodeParams {
    // Tensor maps over the K and the V cache, seen as [n_fa * 2 * max_seq rows][256] bf16: a K/V tile of the attention
    // phase travels as 64-element x 32-row boxes with the 128-byte swizzle (four per ring chunk) instead of one bulk
    // copy per row.  Filled by launch_decode_kernel.
    alignas(64) CUtensorMap map_k;
    alignas(64) CUtensorMap map_v;
    const void* embed;            // bf16 [vocab, 1024]
    const void* layers;           // device pointer table: LayerWeights[] (bf16) or LayerWeightsNVFP4[] (wfmt 1)
    const void* final_norm;       // bf16 [1024]
    const void* lm_head;          // bf16 [vocab, 1024], or packed e2m1 [vocab, 512] when wfmt is 1
    const void* lm_scales;        // wfmt 1: E4M3 block scales of the LM head (128 x 4 tiles); wfmt 2: row-major [vocab][64]
    const float* lm_tensor_scale; // wfmt 2: fp32 scale of the LM-head matrix
    int wfmt;                     // 0 = bf16 weights, 1 = NVFP4 (layer format A, LM head format B), 2 = NVFP4 with
                                  // 16-element blocks, E4M3 block scales (row-major) and an fp32 scale per matrix,
                                  // 3 = the values of 2 as per-CTA chunk images for the block-scaled tcgen05 path
    void* k_cache;                // bf16 [n_fa, 2, max_seq, 256]
    void* v_cache;
    float* dn_states;             // f32 [n_dn, 16, 128(value), 128(key)]
    float* conv_bufs;             // f32 [n_dn, 6144, 4]
    void* hidden;                 // bf16 [1024]: receives the last layer's output
    float* qkv;                   // caller scratch of the reference signature (unused by the kernel)
    float* kv;
    float* attn_out;
    float* mlp_inter;
    float* z;
    float* beta;
    float* alpha;
    float* normalized;            // f32 [1024] final-normed hidden (output)
    float* seen_mask;             // f32 [vocab] or null
    float* logits_out;            // optional f32 [vocab]: receives every logit of the (last) step, after the penalty
    float rep_penalty;
    const int* token_ptr;         // device token (feedback mode) or null
    int token_val;                // host token when token_ptr is null
    int* out_token;               // int32 [steps]: out_token[s] receives the token chosen by step s
    int* token_feedback;          // optional: also receives every new token (the last one remains)
    int position;                 // position of the first step's token; step s decodes at position + s
    int steps;                    // greedy steps in this launch (>= 1), the argmax fed back on the device
    float rope_inv_freq[32];      // theta^(-2i/64), filled by fill_rope(); the angles are formed on the device
    int max_seq_len;
    int num_layers;
    int n_fa_layers;              // attention layers the caches hold (0 = num_layers / 4, the reference model's pattern)
    int vocab;
    DecodeWorkspace* ws;
    uint32_t* host_status;        // mapped pinned word, written only on failure
    unsigned long long* trace;    // optional [grid][trace_slots] globaltimer stamps
    int trace_slots;              // entries per CTA in `trace`
    unsigned long long poll_limit_cycles;   // SM clocks a poll of a flagged word may take before the CTA gives up
    uint32_t mbar_limit_tries;              // try_wait attempts on a ring barrier before the CTA gives up
    int* host_token;              // optional mapped pinned {token, ticket}: the last step's token for a host that spins
    uint32_t host_ticket;         // value written to host_token[1] after the token (system-scope fence in between)
    int lm_image_chunks;          // wfmt 3: 64-row chunk images per CTA in the LM-head image array
    int act_terms;                // wfmt 3: NVFP4 residual terms the activation vector is expanded into (1..8)
};

// Defaults of the two wait limits: about 2 s of SM clock each.
constexpr unsigned long long DEFAULT_POLL_LIMIT_CYCLES = 4000000000ull;
constexpr uint32_t DEFAULT_MBAR_LIMIT_TRIES = 1u << 22;

// Fills rope_inv_freq (position-independent).
void fill_rope(DecodeParams& p);
// Launches the persistent decode kernel (cooperative launch, `grid` CTAs of 544 threads).
cudaError_t launch_decode_kernel(const DecodeParams& p, int grid, cudaStream_t stream);
// Largest grid that is guaranteed co-resident on the current device.
int decode_max_grid();
size_t decode_smem_bytes();
// Grid size the chunk images of the tcgen05 NVFP4 variant (wfmt 3) are cut for.
int decode_image_ctas();
// Two CTAs run the kernel's own poll of a flagged word on a word nobody writes, with p.poll_limit_cycles as the
// limit: the wait runs out, the CTAs record ST_GRID_TIMEOUT through the kernel's failure path and return.  Exists
// so that the failure path can be exercised without a hung launch; p needs ws, host_status and the limit only.
cudaError_t launch_wait_selftest(const DecodeParams& p, cudaStream_t stream);

}  // namespace mk
