// CUDA-core GEMM with the same epilogues as gemm_tc.cu, for the fp32 parity mode (true fp32 arithmetic,
// no TF32) and for bf16 shapes the TMA path cannot take (row strides that are not a multiple of 16 bytes).
//
//   C[M, n_out] = epilogue( A[M, K] @ B[N, K]^T ), fp32 accumulation.
//
// 64x64 output tile per 256-thread block, 4x4 outputs per thread, K staged through shared memory in steps of
// 16. For EPI_SWIGLU, B = [W_gate; W_up]: output column j reads gate row j and up row n_out + j of B and
// keeps two accumulators.
#include "common.cuh"
#include "gemm.h"

namespace fs {
namespace {

constexpr int TM = 64, TN = 64, TK = 16, THREADS = 256;

template <typename T, int EPI>
__global__ void __launch_bounds__(THREADS)
    gemm_simt_kernel(const T* __restrict__ A, int64_t lda, const T* __restrict__ B, int64_t ldb, T* C,
                     int64_t ldc, const T* R, int64_t ldr, int M, int N, int K, int n_out) {
  constexpr int NB = EPI == EPI_SWIGLU ? 2 : 1;
  __shared__ float As[TK][TM + 4];
  __shared__ float Bs[NB][TK][TN + 4];

  const int tx = threadIdx.x % 16, ty = threadIdx.x / 16;  // 16 x 16 threads, 4 x 4 outputs each
  const int m0 = blockIdx.y * TM, n0 = blockIdx.x * TN;
  float acc[NB][4][4] = {};

  for (int k0 = 0; k0 < K; k0 += TK) {
    // A tile: 64 rows x 16 k  (1024 values, 4 per thread)
    for (int i = threadIdx.x; i < TM * TK; i += THREADS) {
      const int r = i / TK, c = i % TK;
      const int gm = m0 + r, gk = k0 + c;
      As[c][r] = (gm < M && gk < K) ? to_f(A[static_cast<int64_t>(gm) * lda + gk]) : 0.f;
    }
    for (int i = threadIdx.x; i < TN * TK; i += THREADS) {
      const int r = i / TK, c = i % TK;
      const int gj = n0 + r, gk = k0 + c;
#pragma unroll
      for (int b = 0; b < NB; ++b) {
        float v = 0.f;
        if (gk < K) {
          if (EPI == EPI_SWIGLU) {
            if (gj < n_out) v = to_f(B[(static_cast<int64_t>(gj) + b * n_out) * ldb + gk]);
          } else if (gj < N) {
            v = to_f(B[static_cast<int64_t>(gj) * ldb + gk]);
          }
        }
        Bs[b][c][r] = v;
      }
    }
    __syncthreads();
#pragma unroll
    for (int kk = 0; kk < TK; ++kk) {
      float a[4], bv[NB][4];
#pragma unroll
      for (int i = 0; i < 4; ++i) a[i] = As[kk][ty * 4 + i];
#pragma unroll
      for (int b = 0; b < NB; ++b)
#pragma unroll
        for (int j = 0; j < 4; ++j) bv[b][j] = Bs[b][kk][tx * 4 + j];
#pragma unroll
      for (int b = 0; b < NB; ++b)
#pragma unroll
        for (int i = 0; i < 4; ++i)
#pragma unroll
          for (int j = 0; j < 4; ++j) acc[b][i][j] = fmaf(a[i], bv[b][j], acc[b][i][j]);
    }
    __syncthreads();
  }

#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int gm = m0 + ty * 4 + i;
    if (gm >= M) continue;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int gj = n0 + tx * 4 + j;
      if (gj >= n_out) continue;
      float v = rnd<T>(acc[0][i][j]);
      if constexpr (EPI == EPI_SWIGLU) {
        const float u = rnd<T>(acc[1][i][j]);
        v = rnd<T>(v / (1.0f + expf(-v))) * u;
      } else if constexpr (EPI == EPI_RESIDUAL) {
        v += to_f(R[static_cast<int64_t>(gm) * ldr + gj]);
      }
      C[static_cast<int64_t>(gm) * ldc + gj] = from_f<T>(v);
    }
  }
}

template <typename T>
int launch(const void* A, int64_t lda, const void* B, int64_t ldb, void* C, int64_t ldc, const void* R, int64_t ldr,
           int64_t M, int64_t N, int64_t K, int64_t n_out, int epi, cudaStream_t st) {
  dim3 grid(static_cast<unsigned>((n_out + TN - 1) / TN), static_cast<unsigned>((M + TM - 1) / TM));
  if (grid.y > 65535) return fail("gemm_simt: M too large");
  auto a = static_cast<const T*>(A);
  auto b = static_cast<const T*>(B);
  auto c = static_cast<T*>(C);
  auto r = static_cast<const T*>(R);
  const int m = static_cast<int>(M), n = static_cast<int>(N), k = static_cast<int>(K), no = static_cast<int>(n_out);
  switch (epi) {
    case EPI_STORE: gemm_simt_kernel<T, EPI_STORE><<<grid, THREADS, 0, st>>>(a, lda, b, ldb, c, ldc, r, ldr, m, n, k, no); break;
    case EPI_RESIDUAL: gemm_simt_kernel<T, EPI_RESIDUAL><<<grid, THREADS, 0, st>>>(a, lda, b, ldb, c, ldc, r, ldr, m, n, k, no); break;
    case EPI_SWIGLU: gemm_simt_kernel<T, EPI_SWIGLU><<<grid, THREADS, 0, st>>>(a, lda, b, ldb, c, ldc, r, ldr, m, n, k, no); break;
    default: return fail("gemm: unknown epilogue");
  }
  return check_launch("gemm_simt_kernel");
}

}  // namespace

int gemm_simt(int dtype, const void* A, int64_t lda, const void* B, int64_t ldb, void* C, int64_t ldc,
              const void* R, int64_t ldr, int64_t M, int64_t N, int64_t K, int64_t n_out, int epi,
              cudaStream_t stream) {
  if (M <= 0 || n_out <= 0) return 0;
  if (M > INT32_MAX / 2 || N > INT32_MAX / 2 || K > INT32_MAX / 2) return fail("gemm: dimension too large");
  if (dtype == F32) return launch<float>(A, lda, B, ldb, C, ldc, R, ldr, M, N, K, n_out, epi, stream);
  if (dtype == BF16) return launch<__nv_bfloat16>(A, lda, B, ldb, C, ldc, R, ldr, M, N, K, n_out, epi, stream);
  return fail("gemm: unsupported dtype");
}

}  // namespace fs
