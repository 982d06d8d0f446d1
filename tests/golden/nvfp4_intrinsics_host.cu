// Host-side run of the CUDA conversion intrinsics the reference quantisers call
// (reference: megakernel/kernel_gb10_nvfp4.cu:1406-1421): __nv_cvt_float_to_fp8 (E4M3, SATFINITE),
// __nv_cvt_fp8_to_halfraw and __nv_cvt_float2_to_fp4x2 (E2M1, round-to-nearest).  These are
// __host__ __device__ functions of the CUDA headers, so their results can be recorded on a
// machine without a GPU.  Output: a binary table read by make_nvfp4_golden.py.
#include <cstdio>
#include <cstdint>
#include <cstring>
#include <cuda_fp16.h>
#include <cuda_fp8.h>
#include <cuda_fp4.h>

int main(int argc, char** argv) {
    FILE* f = fopen(argv[1], "wb");
    // 1. every E4M3 code decoded to float
    for (int c = 0; c < 256; ++c) {
        __half_raw h = __nv_cvt_fp8_to_halfraw((__nv_fp8_storage_t)c, __NV_E4M3);
        float v = __half2float(*reinterpret_cast<__half*>(&h));
        fwrite(&v, 4, 1, f);
    }
    // 2. float -> E4M3 for a dense sweep of bit patterns (positive floats, stride through exponent range)
    uint32_t n = 0;
    long pos_n = ftell(f);
    fwrite(&n, 4, 1, f);
    for (uint32_t bits = 0x30000000u; bits < 0x44800000u; bits += 0x00003fffu) {   // 2^-31 .. 1024
        float x; memcpy(&x, &bits, 4);
        uint8_t c = (uint8_t)__nv_cvt_float_to_fp8(x, __NV_SATFINITE, __NV_E4M3);
        fwrite(&bits, 4, 1, f); fwrite(&c, 1, 1, f); ++n;
    }
    long end = ftell(f); fseek(f, pos_n, SEEK_SET); fwrite(&n, 4, 1, f); fseek(f, end, SEEK_SET);
    // 3. float2 -> fp4x2 for a sweep including every tie point, both signs
    uint32_t m = 0;
    long pos_m = ftell(f);
    fwrite(&m, 4, 1, f);
    for (int i = -1400; i <= 1400; ++i) {
        float a = i * 0.005f, b = -a * 0.5f + 0.125f;
        float2 v = make_float2(a, b);
        uint8_t p = (uint8_t)__nv_cvt_float2_to_fp4x2(v, __NV_E2M1, cudaRoundNearest);
        fwrite(&a, 4, 1, f); fwrite(&b, 4, 1, f); fwrite(&p, 1, 1, f); ++m;
    }
    end = ftell(f); fseek(f, pos_m, SEEK_SET); fwrite(&m, 4, 1, f); fseek(f, end, SEEK_SET);
    fclose(f);
    return 0;
}
