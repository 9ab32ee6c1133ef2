/*
 * ref_shim.cpp -- C entry points over the reference's own CPU kernels, for timing them as the
 * reference CPU baseline (test / benchmark infrastructure only; the product never loads this).
 *
 * The kernels are compiled from the reference's sources where they lie, by ref_build.py:
 *   cpu::gemm_avx2_f32        src/cpu_backend/gemm_avx2.cpp:6-25
 *   cpu::dequantize_q4_0_f32  src/cpu_backend/dequantize_cpu.cpp:6-49
 * with the reference's compiler flags (CMakeLists.txt:16: -mavx2 -mfma -mf16c -O3
 * -ffast-math).  Both are numerically invalid as a matrix product / a GGUF Q4_0 decode (the
 * "GEMM" multiplies lane-wise and reads every eighth row of B; the decoder reads 20-byte
 * blocks of an fp32 scale and 16 nibble bytes, and the pair b[0], b[1] per 32 outputs), so
 * only their speed is used.  The declarations repeat the reference headers' signatures.
 */
#include <cstddef>
#include <cstdint>

namespace cpu {
void gemm_avx2_f32(const float* A, const float* B, float* C, uint32_t M, uint32_t N, uint32_t K);
void dequantize_q4_0_f32(const void* src, float* dst, size_t n);
}  // namespace cpu

extern "C" {
__attribute__((visibility("default"))) void ref_gemm_avx2_f32(const float* A, const float* B, float* C, uint32_t M,
                                                              uint32_t N, uint32_t K) {
  cpu::gemm_avx2_f32(A, B, C, M, N, K);
}
/* src must hold n / 32 + 1 blocks of 20 bytes: the decoder reads one block past its range */
__attribute__((visibility("default"))) void ref_dequantize_q4_0_f32(const void* src, float* dst, size_t n) {
  cpu::dequantize_q4_0_f32(src, dst, n);
}
}
