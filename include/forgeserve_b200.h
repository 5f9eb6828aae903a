/* forgeserve_b200 — C ABI of the B200 (sm_100a) kernels behind the pipeline-parallel forward path.
 *
 * The reference (omkarbhad/forgeserve) is pure PyTorch: each entry point below replaces the ATen calls of
 * one step of a decoder stage, cited as file:line of the reference project. All pointers are device
 * pointers unless stated; `stream` is a cudaStream_t passed as void*. Every entry point only enqueues work
 * on `stream` and returns 0 on success, or a negative status with a message readable through
 * fs_last_error() (thread-local). Kernels never trap: bad token ids, cache slots or positions found on the
 * device, and waits that run out of time, set bits of a device error word read by fs_device_error().
 *
 * dtype: FS_F32 (true fp32 arithmetic, the 1e-4 parity mode) or FS_BF16 (tensor-core mode).
 * Matrices are row-major with an explicit row stride in elements.
 */
#ifndef FORGESERVE_B200_H
#define FORGESERVE_B200_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

enum { FS_F32 = 0, FS_BF16 = 1 };
enum { FS_EPI_STORE = 0, FS_EPI_RESIDUAL = 1, FS_EPI_SWIGLU = 2 };
/* ORed into fs_gemm's epilogue: C may be another GPU's memory (mapped with fs_ipc_open); every CTA of the
 * tensor-core kernel ends with a system-scope fence, so the stores are performed before the kernel completes. */
enum { FS_EPI_SYSTEM_FENCE = 0x100 };
enum { FS_IPC_HANDLE_BYTES = 64 };
enum { FS_ERR_WAIT_TIMEOUT = 1, FS_ERR_BAD_TOKEN = 2, FS_ERR_BAD_SLOT = 4, FS_ERR_BAD_POSITION = 8 };

/* Library version (major*10000 + minor*100 + patch). */
int fs_version(void);

/* Message of the last failed call on this host thread ("" if none). */
const char* fs_last_error(void);

/* Reads (and, if clear != 0, resets) the device error word of the current device. Synchronises the device. */
int fs_device_error(int clear, unsigned* out_bits);

/* Self-test of the bounded device waits: launches one warp that waits, through the same bounded mbarrier wait as
 * the tensor-core kernels, on a barrier that never completes, with a time limit of limit_ns (1000 ns .. 2 s; the
 * kernels use 2 s). The wait gives up, sets FS_ERR_WAIT_TIMEOUT in the device error word and the kernel returns, so
 * the context stays usable. out: two device uint64 words, the nanoseconds waited and 1 if the wait completed.
 * Stands in, on the device, for the reference's host-side timeout on a stuck rank (forgeserve/tensor_parallel.py
 * :76-87, a RuntimeError instead of a hang). */
int fs_wait_selftest(int64_t limit_ns, unsigned long long* out, void* stream);

/* Number of kernel launches made by this library in this process (all devices). */
int64_t fs_launch_count(void);

/* Caps the number of SMs the persistent tensor-core GEMM spreads over on the current device (0 = all).
 * A pipeline stage that overlaps NCCL send/recv with compute leaves a few SMs to the NCCL kernels this way, so
 * that no GEMM CTA waits behind a resident communication kernel. No counterpart in the reference (CPU/gloo). */
int fs_set_persistent_sms(int n);

/* on != 0 (default): bf16 GEMMs with M > 128 run on CTA pairs (tcgen05 cta_group::2, 256 x 256 tiles); 0: always on
 * single CTAs (128 x 256 tiles). Process-wide. For comparing the two kernels. No counterpart in the reference. */
int fs_set_gemm_pair_mode(int on);

/* Inter-process mapping of a device buffer, so that pipeline stages (one process per GPU) can write their vocab
 * slice of the output head straight into the last stage's logits tensor over NVLink. No counterpart in the
 * reference (its stages are CPU processes that exchange tensors through gloo; pipeline.py:112-118 computes the
 * whole head on the last stage).
 * fs_ipc_handle: the CUDA IPC handle (FS_IPC_HANDLE_BYTES bytes, written to `handle`) of the device allocation
 *   that holds `ptr`, and ptr's byte offset inside that allocation.
 * fs_ipc_open: maps another process's allocation into this one (peer access enabled); *base is the allocation's
 *   start as seen from the current device. A process maps a given allocation once; fs_ipc_close unmaps it. */
int fs_ipc_handle(const void* ptr, void* handle, int64_t* offset);
int fs_ipc_open(const void* handle, void** base);
int fs_ipc_close(void* base);

/* Copies `height` rows of `width` bytes from src (rows spitch bytes apart) to dst (rows dpitch bytes apart) on
 * `stream`, by the copy engine (no SM takes part). Either side may be another GPU's memory mapped with
 * fs_ipc_open: a stage moves its slice of the split head's logits into the last stage's output this way.
 * No counterpart in the reference. */
int fs_copy_2d(void* dst, int64_t dpitch, const void* src, int64_t spitch, int64_t width, int64_t height,
               void* stream);

/* RMSNorm over rows: y = T(T(x * rsqrt(mean(x^2) + eps)) * w), fp32 statistics.
 * Replaces RMSNorm.forward, forgeserve/model.py:29-31. y may alias x. */
int fs_rmsnorm(const void* x, int64_t x_stride, const void* w, void* y, int64_t y_stride, int64_t rows, int64_t dim,
               float eps, int dtype, void* stream);

/* Projection GEMM: C[M, n_out] = epi(A[M, K] @ B[N, K]^T), B in nn.Linear (out, in) layout.
 *   FS_EPI_STORE:    n_out = N.
 *   FS_EPI_RESIDUAL: C = R + C (R may alias C), the residual adds of Block.forward (model.py:105-106).
 *   FS_EPI_SWIGLU:   C = silu(gate) * up, SwiGLU.forward (model.py:93); B = [W_gate; W_up], N = 2 * n_out.
 * Replaces nn.Linear calls at model.py:64-66, :77, :93 and pipeline.py:112 (lm_head).
 * bf16 runs on the tcgen05/TMEM tensor-core kernel when A/B are 16-byte aligned with row strides a multiple of
 * 8 elements; fp32 (and other bf16 layouts) run on CUDA cores with fp32 accumulation. */
int fs_gemm(const void* A, int64_t lda, const void* B, int64_t ldb, void* C, int64_t ldc, const void* R, int64_t ldr,
            int64_t M, int64_t N, int64_t K, int64_t n_out, int epilogue, int dtype, void* stream);

/* Same as fs_gemm but never uses the tensor-core kernel (CUDA-core path), for cross-checking. */
int fs_gemm_simt(const void* A, int64_t lda, const void* B, int64_t ldb, void* C, int64_t ldc, const void* R,
                 int64_t ldr, int64_t M, int64_t N, int64_t K, int64_t n_out, int epilogue, int dtype, void* stream);

/* KV cache of one layer. Slot s of batch row r, KV head g is at
 *   base + table[r*table_stride + s/block_size]*block_stride + g*head_stride + (s % block_size)*head_dim.
 * Paged pool (num_blocks, n_kv, block_size, hd) (forgeserve/paged.py:48-50): table = block table.
 * Contiguous per-row cache (B, n_kv, capacity, hd) (forgeserve/kv.py:10-24): block_size = capacity,
 * table = [0, 1, ..., B-1]. */
typedef struct {
  void* k;
  void* v;
  const int64_t* table;
  int64_t table_stride;
  int64_t table_cols;
  int64_t block_size;
  int64_t block_stride;
  int64_t head_stride;
  int64_t num_blocks;
} fs_kv_cache;

/* RoPE on the fused q/k/v projection output + store of the new keys/values into the cache.
 * qkv: (B*T, ld) rows [q: nh*hd | k: nkv*hd | v: nkv*hd]; q is rotated in place. cos/sin: fp32 (rope_rows, hd/2)
 * tables (model.py:34-37), rotation as model.py:40-45. Slot of token (r, j): slot_base + j if slot_from_pos == 0
 * (contiguous cache, ContiguousKV.update kv.py:21-24), positions[r, j] otherwise (PagedLayerView.update
 * paged.py:74-78). apply_rope = 0 stores k unrotated (used by tests). */
int fs_rope_kv_write(void* qkv, int64_t ld, const float* cos_t, const float* sin_t, int64_t rope_rows,
                     const int64_t* positions, const fs_kv_cache* kv, int64_t B, int64_t T, int64_t nh, int64_t nkv,
                     int64_t hd, int64_t slot_base, int slot_from_pos, int apply_rope, int dtype, void* stream);

/* Store k, v of shape (B, nkv, T, hd) at slots positions[r, j] (write half of PagedLayerView.update,
 * paged.py:72-78). */
int fs_kv_store(const void* k, const void* v, const int64_t* positions, const fs_kv_cache* kv, int64_t B, int64_t T,
                int64_t nkv, int64_t hd, int dtype, void* stream);

/* out (B, nkv, nb*bs, hd) = pool[table] permuted (read half of PagedLayerView.update, paged.py:80-81). */
int fs_paged_gather(const void* pool, const int64_t* table, int64_t B, int64_t nb, int64_t num_blocks, int64_t nkv,
                    int64_t block_size, int64_t hd, void* out, int dtype, void* stream);

/* GQA attention of B*T new queries over the cache: key slot s visible iff s <= positions[r, j] and s < n_slots
 * (model.py:69-76: cache update, repeat_interleave, mask, scaled_dot_product_attention with scale 1/sqrt(hd)).
 * q rows (B*T, ldq) hold nh heads; out rows (B*T, ldo). bf16 with hd 64/128 runs on tensor cores: the
 * tcgen05/TMEM kernel for T >= 64 (cache block_size a multiple of 16), the mma.sync kernel for shorter query blocks. */
int fs_attention(const void* q, int64_t ldq, const fs_kv_cache* kv, int64_t n_slots, const int64_t* positions,
                 void* out, int64_t ldo, int64_t B, int64_t T, int64_t nh, int64_t nkv, int64_t hd, float scale,
                 int dtype, void* stream);

/* fs_attention with an explicit kernel: FS_ATTN_AUTO, FS_ATTN_CUDA_CORE (fp32/bf16, any even hd <= 256),
 * FS_ATTN_MMA_SYNC (bf16, hd 64/128) or FS_ATTN_TCGEN05 (bf16, hd 64/128, block_size % 16 == 0); a kernel that
 * cannot take the layout returns an error. For cross-checking the kernels against each other. */
enum { FS_ATTN_AUTO = 0, FS_ATTN_CUDA_CORE = 1, FS_ATTN_MMA_SYNC = 2, FS_ATTN_TCGEN05 = 3 };
int fs_attention_impl(const void* q, int64_t ldq, const fs_kv_cache* kv, int64_t n_slots, const int64_t* positions,
                      void* out, int64_t ldo, int64_t B, int64_t T, int64_t nh, int64_t nkv, int64_t hd, float scale,
                      int impl, int dtype, void* stream);

/* Decode attention: one new query per batch row (positions[r] its position), split over the keys ("flash decoding")
 * so that every K/V row is read once for all query heads of its KV head. Same semantics as fs_attention with T = 1
 * (model.py:69-76 on the decode step of the Engine, engine.py:125). head_dim 64 or 128, n_heads / n_kv_heads <= 8.
 * workspace: device memory of at least fs_attention_decode_workspace(...) bytes (0 bytes when one split suffices),
 * owned by the caller, not read before being written; calls that overlap on the GPU need separate workspaces. */
int64_t fs_attention_decode_workspace(int64_t B, int64_t nh, int64_t nkv, int64_t hd, int64_t n_slots);
int fs_attention_decode(const void* q, int64_t ldq, const fs_kv_cache* kv, int64_t n_slots, const int64_t* positions,
                        void* out, int64_t ldo, int64_t B, int64_t nh, int64_t nkv, int64_t hd, float scale,
                        void* workspace, int64_t workspace_bytes, int dtype, void* stream);

/* fs_attention_decode for callers that cannot allocate device memory where they run a decode step (a host that
 * owns all device memory through its own pool, a plugin that is only handed device pointers, a loop that cannot
 * take the synchronisation of a cudaMalloc mid-step): the split partials go to a fixed 4 MiB scratch array that is
 * part of the library image (held on every GPU that loads it until exit) instead of a caller workspace.
 * Allocates nothing. The first call on a device looks up that array's address and, under CUDA's default lazy
 * module loading, loads the kernels and reserves the array: make one real call at start-up, before a host pool
 * takes the device's free memory and before any stream capture on the device. Calls needing more scratch than
 * 4 MiB (fs_attention_decode_workspace: B * n_heads * splits * (head_dim + 2) * 4 bytes, a split per 512 cache
 * slots; e.g. 64 rows of 32 x 128 heads fit up to 1536 slots) are refused with an error. All calls share the
 * array, so calls that overlap on the GPU race and must not be issued. Device-side errors go to a file-scope
 * word that fs_device_error reads with the library's own.
 * No counterpart in the reference (it has no kernels or device memory). */
int fs_attention_decode_static(const void* q, int64_t ldq, const fs_kv_cache* kv, int64_t n_slots,
                               const int64_t* positions, void* out, int64_t ldo, int64_t B, int64_t nh, int64_t nkv,
                               int64_t hd, float scale, int dtype, void* stream);

/* Token embedding gather out[i] = table[ids[i]] (nn.Embedding at pipeline.py:106 / model.py:134-135). */
int fs_embed(const int64_t* ids, int64_t n, const void* table, int64_t vocab, int64_t dim, void* out, int dtype,
             void* stream);

/* Greedy sampling: out[i] = argmax(x[i, :n]) with the lowest index on ties (sampling.py:18-19,
 * pipeline.py:133). */
int fs_argmax(const void* x, int64_t rows, int64_t n, int64_t row_stride, int64_t* out, int dtype, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* FORGESERVE_B200_H */
