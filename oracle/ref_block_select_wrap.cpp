// TEST INFRASTRUCTURE ONLY.  C entry point for the reference's host-side block selection
// (dflash/src/flashprefill_select.cpp:27-84, dflash27b::flashprefill::block_select_host): build_oracle.py compiles
// this file together with that source file, where it lies in the reference checkout, into
// oracle/_ref/libref_block_select.so.  Nothing of the reference is restated here.
#include <cstdint>

namespace dflash27b {
namespace flashprefill {
void block_select_host(const float* score, int B, int M, int N, int H, int attention_sink, int window, int last_n_full,
                       float alpha, int32_t* idx_out, int32_t* cnt_out);
}
}  // namespace dflash27b

// score [B][M][N][H] f32; idx_out [B][M][N][H] (kept key blocks in ascending order, then -1); cnt_out [B][M][H]
extern "C" void ref_block_select_host(const float* score, int B, int M, int N, int H, int attention_sink, int window,
                                      int last_n_full, float alpha, int32_t* idx_out, int32_t* cnt_out) {
    dflash27b::flashprefill::block_select_host(score, B, M, N, H, attention_sink, window, last_n_full, alpha, idx_out, cnt_out);
}
