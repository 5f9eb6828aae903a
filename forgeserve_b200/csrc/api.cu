// The C ABI (include/forgeserve_b200.h): argument checks, dispatch, error strings, launch counting.
#include <cudaTypedefs.h>

#include <atomic>
#include <cstdlib>
#include <cstring>
#include <string>

#include "../../include/forgeserve_b200.h"
#include "common.cuh"
#include "gemm.h"
#include "kernels.h"

namespace fs {

static thread_local std::string t_last_error;
static std::atomic<int64_t> g_launches{0};

void set_last_error(const std::string& msg) { t_last_error = msg; }
int fail(const std::string& msg) {
  set_last_error(msg);
  return -1;
}
bool pdl_enabled() {
  static const bool on = [] {
    const char* v = std::getenv("FORGESERVE_PDL");
    return !(v && v[0] == '0');
  }();
  return on;
}

int check_launch(const char* what) {
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return fail(std::string(what) + ": " + cudaGetErrorString(e));
  g_launches.fetch_add(1, std::memory_order_relaxed);
  return 0;
}

static KVCache to_internal(const fs_kv_cache* c) {
  KVCache k;
  k.k = c->k;
  k.v = c->v;
  k.table = c->table;
  k.table_stride = c->table_stride;
  k.table_cols = c->table_cols;
  k.block_size = c->block_size;
  k.block_stride = c->block_stride;
  k.head_stride = c->head_stride;
  k.num_blocks = c->num_blocks;
  return k;
}

static int check_kv(const fs_kv_cache* c) {
  if (!c) return fail("kv cache descriptor is NULL");
  if (!c->k || !c->v || !c->table) return fail("kv cache: NULL pointer");
  if (c->block_size <= 0 || c->num_blocks <= 0 || c->table_cols <= 0) return fail("kv cache: empty cache");
  return 0;
}

static bool dtype_ok(int dtype) { return dtype == F32 || dtype == BF16; }

static unsigned* g_error_words[64] = {nullptr};

int static_decode_error_bits(int clear, unsigned* bits);  // attention_decode.cu

unsigned* error_word() {
  unsigned** words = g_error_words;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) {
    fail("error_word: no current CUDA device");
    return nullptr;
  }
  if (!words[dev]) {
    unsigned* p = nullptr;
    if (cudaMalloc(&p, sizeof(unsigned)) != cudaSuccess || cudaMemset(p, 0, sizeof(unsigned)) != cudaSuccess) {
      fail("error_word: cudaMalloc failed");
      return nullptr;
    }
    words[dev] = p;
  }
  return words[dev];
}

// Wait self-test: one warp. Lane 0 sets up an mbarrier that needs two arrivals and arrives once, then every lane
// waits on its first phase with the bounded wait of the tensor-core kernels (mbar_wait) and a short limit. Nothing
// else ever arrives, so the wait must run out, flag ERR_WAIT_TIMEOUT and return; the kernel then exits normally.
// out[0] = nanoseconds lane 0 waited, out[1] = 1 if its wait completed (it never should).
__global__ void wait_selftest_kernel(uint64_t limit_ns, unsigned* err, unsigned long long* out) {
  __shared__ __align__(8) uint64_t bar;
  if (threadIdx.x == 0) {
    mbar_init(&bar, 2);
    fence_barrier_init();
  }
  __syncthreads();
  if (threadIdx.x == 0) mbar_arrive(&bar);
  const uint64_t t0 = globaltimer_ns();
  const bool done = mbar_wait(&bar, 0, err, limit_ns);
  const uint64_t t1 = globaltimer_ns();
  if (threadIdx.x == 0) {
    out[0] = t1 - t0;
    out[1] = done ? 1ull : 0ull;
  }
}

}  // namespace fs

using namespace fs;

extern "C" {

int fs_wait_selftest(int64_t limit_ns, unsigned long long* out, void* stream) {
  if (!out) return fail("fs_wait_selftest: NULL output");
  if (limit_ns < 1000 || limit_ns > static_cast<int64_t>(kWaitLimitNs))
    return fail("fs_wait_selftest: limit_ns must lie in [1000, " + std::to_string(kWaitLimitNs) + "]");
  unsigned* err = error_word();
  if (!err) return -1;
  wait_selftest_kernel<<<1, 32, 0, static_cast<cudaStream_t>(stream)>>>(static_cast<uint64_t>(limit_ns), err, out);
  return check_launch("wait_selftest_kernel");
}

int fs_version(void) { return 100; }

const char* fs_last_error(void) { return t_last_error.c_str(); }

int fs_device_error(int clear, unsigned* out_bits) {
  unsigned bits = 0;
  unsigned* word = error_word();
  if (!word) return -1;
  cudaError_t e = cudaDeviceSynchronize();
  if (e != cudaSuccess) return fail(std::string("fs_device_error: ") + cudaGetErrorString(e));
  e = cudaMemcpy(&bits, word, sizeof(bits), cudaMemcpyDeviceToHost);
  if (e != cudaSuccess) return fail(std::string("fs_device_error: ") + cudaGetErrorString(e));
  if (clear) {
    e = cudaMemset(word, 0, sizeof(unsigned));
    if (e != cudaSuccess) return fail(std::string("fs_device_error: ") + cudaGetErrorString(e));
  }
  unsigned static_bits = 0;
  if (static_decode_error_bits(clear, &static_bits)) return -1;
  bits |= static_bits;
  if (out_bits) *out_bits = bits;
  return 0;
}

int64_t fs_launch_count(void) { return g_launches.load(std::memory_order_relaxed); }

int fs_set_persistent_sms(int n) { return tcg::set_persistent_sms(n); }

int fs_set_gemm_pair_mode(int on) { return tcg::set_pair_mode(on); }

// ------------------------------------------------------------------------------------------ inter-process
static PFN_cuMemGetAddressRange_v3020 address_range_fn() {
  static PFN_cuMemGetAddressRange_v3020 fn = nullptr;
  if (!fn) {
    cudaDriverEntryPointQueryResult q;
    void* ptr = nullptr;
    if (cudaGetDriverEntryPoint("cuMemGetAddressRange", &ptr, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuMemGetAddressRange_v3020>(ptr);
  }
  return fn;
}

int fs_ipc_handle(const void* ptr, void* handle, int64_t* offset) {
  if (!ptr || !handle || !offset) return fail("fs_ipc_handle: NULL pointer");
  auto range = address_range_fn();
  if (!range) return fail("fs_ipc_handle: cuMemGetAddressRange is unavailable from the CUDA driver");
  CUdeviceptr base = 0;
  size_t size = 0;
  if (range(&base, &size, reinterpret_cast<CUdeviceptr>(ptr)) != CUDA_SUCCESS)
    return fail("fs_ipc_handle: the pointer is not inside a device allocation");
  cudaIpcMemHandle_t h;
  const cudaError_t e = cudaIpcGetMemHandle(&h, reinterpret_cast<void*>(base));
  if (e != cudaSuccess) return fail(std::string("fs_ipc_handle: cudaIpcGetMemHandle: ") + cudaGetErrorString(e));
  static_assert(sizeof(h) == FS_IPC_HANDLE_BYTES, "CUDA IPC handle size");
  std::memcpy(handle, &h, sizeof(h));
  *offset = static_cast<int64_t>(reinterpret_cast<CUdeviceptr>(ptr) - base);
  return 0;
}

int fs_ipc_open(const void* handle, void** base) {
  if (!handle || !base) return fail("fs_ipc_open: NULL pointer");
  cudaIpcMemHandle_t h;
  std::memcpy(&h, handle, sizeof(h));
  const cudaError_t e = cudaIpcOpenMemHandle(base, h, cudaIpcMemLazyEnablePeerAccess);
  if (e != cudaSuccess) return fail(std::string("fs_ipc_open: cudaIpcOpenMemHandle: ") + cudaGetErrorString(e));
  return 0;
}

int fs_copy_2d(void* dst, int64_t dpitch, const void* src, int64_t spitch, int64_t width, int64_t height,
               void* stream) {
  if (width <= 0 || height <= 0) return 0;
  if (!dst || !src) return fail("fs_copy_2d: NULL pointer");
  if (dpitch < width || spitch < width) return fail("fs_copy_2d: pitch smaller than the row width");
  const cudaError_t e = cudaMemcpy2DAsync(dst, static_cast<size_t>(dpitch), src, static_cast<size_t>(spitch),
                                          static_cast<size_t>(width), static_cast<size_t>(height), cudaMemcpyDefault,
                                          static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return fail(std::string("fs_copy_2d: cudaMemcpy2DAsync: ") + cudaGetErrorString(e));
  return 0;
}

int fs_ipc_close(void* base) {
  if (!base) return fail("fs_ipc_close: NULL pointer");
  const cudaError_t e = cudaIpcCloseMemHandle(base);
  if (e != cudaSuccess) return fail(std::string("fs_ipc_close: cudaIpcCloseMemHandle: ") + cudaGetErrorString(e));
  return 0;
}

int fs_rmsnorm(const void* x, int64_t x_stride, const void* w, void* y, int64_t y_stride, int64_t rows, int64_t dim,
               float eps, int dtype, void* stream) {
  if (!x || !w || !y) return rows <= 0 ? 0 : fail("fs_rmsnorm: NULL pointer");
  if (x_stride < dim || y_stride < dim) return fail("fs_rmsnorm: row stride smaller than dim");
  return rmsnorm(dtype, x, x_stride, w, y, y_stride, rows, dim, eps, static_cast<cudaStream_t>(stream));
}

static int gemm_common(bool allow_tc, const void* A, int64_t lda, const void* B, int64_t ldb, void* C, int64_t ldc,
                       const void* R, int64_t ldr, int64_t M, int64_t N, int64_t K, int64_t n_out, int epi, int dtype,
                       void* stream) {
  if (M <= 0 || n_out <= 0) return 0;
  const bool sys_fence = (epi & EPI_FLAG_SYSTEM_FENCE) != 0;
  epi &= ~EPI_FLAG_SYSTEM_FENCE;
  if (!A || !B || !C) return fail("fs_gemm: NULL pointer");
  if (!dtype_ok(dtype)) return fail("fs_gemm: unsupported dtype");
  if (K <= 0 || N <= 0) return fail("fs_gemm: K and N must be positive");
  if (lda < K || ldb < K) return fail("fs_gemm: row stride smaller than K");
  if (epi == EPI_RESIDUAL && !R) return fail("fs_gemm: residual epilogue needs R");
  if (epi == EPI_SWIGLU) {
    if (N != 2 * n_out) return fail("fs_gemm: swiglu weight [W_gate; W_up] must have 2 * n_out rows");
  } else if (epi == EPI_STORE || epi == EPI_RESIDUAL) {
    if (n_out != N) return fail("fs_gemm: n_out must equal N");
  } else {
    return fail("fs_gemm: unknown epilogue");
  }
  if (ldc < n_out || (epi == EPI_RESIDUAL && ldr < n_out)) return fail("fs_gemm: output row stride too small");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (allow_tc && dtype == BF16 && tcg::supported(A, lda, B, ldb, K))
    return tcg::gemm_tc(A, lda, B, ldb, C, ldc, R, ldr, M, N, K, n_out, epi, sys_fence, st);
  if (sys_fence) return fail("fs_gemm: FS_EPI_SYSTEM_FENCE needs the tensor-core kernel (bf16, aligned operands)");
  return gemm_simt(dtype, A, lda, B, ldb, C, ldc, R, ldr, M, N, K, n_out, epi, st);
}

int fs_gemm(const void* A, int64_t lda, const void* B, int64_t ldb, void* C, int64_t ldc, const void* R, int64_t ldr,
            int64_t M, int64_t N, int64_t K, int64_t n_out, int epilogue, int dtype, void* stream) {
  return gemm_common(true, A, lda, B, ldb, C, ldc, R, ldr, M, N, K, n_out, epilogue, dtype, stream);
}

int fs_gemm_simt(const void* A, int64_t lda, const void* B, int64_t ldb, void* C, int64_t ldc, const void* R,
                 int64_t ldr, int64_t M, int64_t N, int64_t K, int64_t n_out, int epilogue, int dtype, void* stream) {
  return gemm_common(false, A, lda, B, ldb, C, ldc, R, ldr, M, N, K, n_out, epilogue, dtype, stream);
}

int fs_rope_kv_write(void* qkv, int64_t ld, const float* cos_t, const float* sin_t, int64_t rope_rows,
                     const int64_t* positions, const fs_kv_cache* kv, int64_t B, int64_t T, int64_t nh, int64_t nkv,
                     int64_t hd, int64_t slot_base, int slot_from_pos, int apply_rope, int dtype, void* stream) {
  if (B * T <= 0) return 0;
  if (check_kv(kv)) return -1;
  if (!qkv || !positions || (apply_rope && (!cos_t || !sin_t))) return fail("fs_rope_kv_write: NULL pointer");
  if (ld < (nh + 2 * nkv) * hd) return fail("fs_rope_kv_write: qkv row stride too small");
  return rope_kv_write(dtype, qkv, ld, cos_t, sin_t, rope_rows, positions, to_internal(kv), B, T, nh, nkv, hd, slot_base,
                       slot_from_pos, apply_rope, static_cast<cudaStream_t>(stream));
}

int fs_kv_store(const void* k, const void* v, const int64_t* positions, const fs_kv_cache* kv, int64_t B, int64_t T,
                int64_t nkv, int64_t hd, int dtype, void* stream) {
  if (B * T <= 0) return 0;
  if (check_kv(kv)) return -1;
  if (!k || !v || !positions) return fail("fs_kv_store: NULL pointer");
  return kv_store(dtype, k, v, positions, to_internal(kv), B, T, nkv, hd, static_cast<cudaStream_t>(stream));
}

int fs_paged_gather(const void* pool, const int64_t* table, int64_t B, int64_t nb, int64_t num_blocks, int64_t nkv,
                    int64_t block_size, int64_t hd, void* out, int dtype, void* stream) {
  if (B * nb <= 0) return 0;
  if (!pool || !table || !out) return fail("fs_paged_gather: NULL pointer");
  return paged_gather(dtype, pool, table, B, nb, num_blocks, nkv, block_size, hd, out, static_cast<cudaStream_t>(stream));
}

static int attention_common(int impl, const void* q, int64_t ldq, const fs_kv_cache* kv, int64_t n_slots,
                            const int64_t* positions, void* out, int64_t ldo, int64_t B, int64_t T, int64_t nh,
                            int64_t nkv, int64_t hd, float scale, int dtype, void* stream) {
  if (B * T <= 0) return 0;
  if (check_kv(kv)) return -1;
  if (!q || !positions || !out) return fail("fs_attention: NULL pointer");
  if (n_slots <= 0) return fail("fs_attention: the cache view has no slots");
  if (ldq < nh * hd || ldo < nh * hd) return fail("fs_attention: row stride too small");
  if (impl < 0 || impl > 3) return fail("fs_attention: unknown kernel selector");
  return attention(dtype, q, ldq, to_internal(kv), n_slots, positions, out, ldo, B, T, nh, nkv, hd, scale, impl,
                   static_cast<cudaStream_t>(stream));
}

int fs_attention(const void* q, int64_t ldq, const fs_kv_cache* kv, int64_t n_slots, const int64_t* positions,
                 void* out, int64_t ldo, int64_t B, int64_t T, int64_t nh, int64_t nkv, int64_t hd, float scale,
                 int dtype, void* stream) {
  return attention_common(0, q, ldq, kv, n_slots, positions, out, ldo, B, T, nh, nkv, hd, scale, dtype, stream);
}

int fs_attention_impl(const void* q, int64_t ldq, const fs_kv_cache* kv, int64_t n_slots, const int64_t* positions,
                      void* out, int64_t ldo, int64_t B, int64_t T, int64_t nh, int64_t nkv, int64_t hd, float scale,
                      int impl, int dtype, void* stream) {
  return attention_common(impl, q, ldq, kv, n_slots, positions, out, ldo, B, T, nh, nkv, hd, scale, dtype, stream);
}

static int decode_sms() {
  static int n[64] = {0};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64) dev = 0;
  if (!n[dev]) cudaDeviceGetAttribute(&n[dev], cudaDevAttrMultiProcessorCount, dev);
  return n[dev] > 0 ? n[dev] : 148;
}

int64_t fs_attention_decode_workspace(int64_t B, int64_t nh, int64_t nkv, int64_t hd, int64_t n_slots) {
  if (B <= 0 || nh <= 0 || nkv <= 0 || hd <= 0 || n_slots <= 0) return 0;
  return decode::workspace_bytes(B, nh, hd, decode::choose_splits(B, nkv, n_slots, decode_sms()));
}

int fs_attention_decode(const void* q, int64_t ldq, const fs_kv_cache* kv, int64_t n_slots, const int64_t* positions,
                        void* out, int64_t ldo, int64_t B, int64_t nh, int64_t nkv, int64_t hd, float scale,
                        void* workspace, int64_t workspace_bytes, int dtype, void* stream) {
  if (B <= 0) return 0;
  if (check_kv(kv)) return -1;
  if (!q || !positions || !out) return fail("fs_attention_decode: NULL pointer");
  if (n_slots <= 0) return fail("fs_attention_decode: the cache view has no slots");
  if (!dtype_ok(dtype)) return fail("fs_attention_decode: unsupported dtype");
  if (ldq < nh * hd || ldo < nh * hd) return fail("fs_attention_decode: row stride too small");
  const KVCache c = to_internal(kv);
  if (!decode::supported(dtype, hd, nh, nkv, q, ldq, c))
    return fail("fs_attention_decode: needs head_dim 64 or 128, n_heads / n_kv_heads <= 8 and 16-byte aligned rows");
  const int splits = decode::choose_splits(B, nkv, n_slots, decode_sms());
  const int64_t need = decode::workspace_bytes(B, nh, hd, splits);
  if (need > 0 && (!workspace || workspace_bytes < need))
    return fail("fs_attention_decode: workspace of " + std::to_string(need) + " bytes needed");
  unsigned* err = error_word();
  if (!err) return -1;
  return decode::launch(dtype, q, ldq, c, n_slots, positions, out, ldo, B, nh, nkv, hd, scale, splits,
                        static_cast<float*>(workspace), err, static_cast<cudaStream_t>(stream));
}

int fs_embed(const int64_t* ids, int64_t n, const void* table, int64_t vocab, int64_t dim, void* out, int dtype,
             void* stream) {
  if (n <= 0) return 0;
  if (!ids || !table || !out) return fail("fs_embed: NULL pointer");
  return embed(dtype, ids, n, table, vocab, dim, out, static_cast<cudaStream_t>(stream));
}

int fs_argmax(const void* x, int64_t rows, int64_t n, int64_t row_stride, int64_t* out, int dtype, void* stream) {
  if (rows <= 0) return 0;
  if (!x || !out) return fail("fs_argmax: NULL pointer");
  if (row_stride < n) return fail("fs_argmax: row stride smaller than n");
  return argmax(dtype, x, rows, n, row_stride, out, static_cast<cudaStream_t>(stream));
}

}  // extern "C"
