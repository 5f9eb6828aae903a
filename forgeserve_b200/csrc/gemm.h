// Internal declarations of the projection GEMMs (see gemm_tc.cu, gemm_simt.cu).
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

namespace fs {

enum Epilogue : int { EPI_STORE = 0, EPI_RESIDUAL = 1, EPI_SWIGLU = 2 };
constexpr int EPI_FLAG_SYSTEM_FENCE = 0x100;   // ORed into the epilogue: C may be another GPU's memory

namespace tcg {
int set_persistent_sms(int n);
int set_pair_mode(int on);
bool supported(const void* A, int64_t lda, const void* B, int64_t ldb, int64_t K);
int gemm_tc(const void* A, int64_t lda, const void* B, int64_t ldb, void* C, int64_t ldc, const void* R,
            int64_t ldr, int64_t M, int64_t N, int64_t K, int64_t n_out, int epi, bool sys_fence,
            cudaStream_t stream);
}  // namespace tcg

int gemm_simt(int dtype, const void* A, int64_t lda, const void* B, int64_t ldb, void* C, int64_t ldc,
              const void* R, int64_t ldr, int64_t M, int64_t N, int64_t K, int64_t n_out, int epi,
              cudaStream_t stream);

}  // namespace fs
