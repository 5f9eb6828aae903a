// Internal declarations shared by the kernel files and the C-ABI layer (api.cu).
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

namespace fs {

// One layer's K/V cache as the kernels address it (see elementwise.cu for the addressing formula).
struct KVCache {
  void* k;
  void* v;
  const int64_t* table;   // (B, table_cols) block numbers, row stride table_stride
  int64_t table_stride;
  int64_t table_cols;
  int64_t block_size;     // slots per block
  int64_t block_stride;   // elements between consecutive blocks
  int64_t head_stride;    // elements between consecutive KV heads inside a block
  int64_t num_blocks;     // blocks in the cache (bounds check for table entries)
};

int rmsnorm(int dtype, const void* x, int64_t xs, const void* w, void* y, int64_t ys, int64_t rows, int64_t dim,
            float eps, cudaStream_t st);
int rope_kv_write(int dtype, void* qkv, int64_t ld, const float* cos_t, const float* sin_t, int64_t rope_rows,
                  const int64_t* positions, const KVCache& kv, int64_t B, int64_t T_new, int64_t nh, int64_t nkv,
                  int64_t hd, int64_t slot_base, int slot_from_pos, int apply_rope, cudaStream_t st);
int kv_store(int dtype, const void* k, const void* v, const int64_t* positions, const KVCache& kv, int64_t B,
             int64_t T_new, int64_t nkv, int64_t hd, cudaStream_t st);
int paged_gather(int dtype, const void* pool, const int64_t* table, int64_t B, int64_t nb, int64_t num_blocks,
                 int64_t nkv, int64_t bs, int64_t hd, void* out, cudaStream_t st);
int embed(int dtype, const int64_t* ids, int64_t n, const void* table, int64_t vocab, int64_t dim, void* out,
          cudaStream_t st);
int argmax(int dtype, const void* x, int64_t rows, int64_t n, int64_t row_stride, int64_t* out, cudaStream_t st);

// Attention of B*T new queries against the cache (GQA, mask: key slot s visible iff s <= position and
// s < n_slots). q: row (b*T + t) holds nh heads of hd at stride ldq; out likewise at stride ldo.
// impl: 0 = automatic, 1 = CUDA-core kernel, 2 = mma.sync kernel, 3 = tcgen05 kernel.
int attention(int dtype, const void* q, int64_t ldq, const KVCache& kv, int64_t n_slots, const int64_t* positions,
              void* out, int64_t ldo, int64_t B, int64_t T, int64_t nh, int64_t nkv, int64_t hd, float scale,
              int impl, cudaStream_t st);

namespace attn_tc {
bool supported(const void* q, int64_t ldq, const KVCache& kv, int64_t hd, int64_t T);
int launch(const void* q, int64_t ldq, const KVCache& kv, int64_t n_slots, const int64_t* positions, void* out,
           int64_t ldo, int64_t B, int64_t T, int64_t nh, int64_t nkv, int64_t hd, float scale, cudaStream_t st);
}  // namespace attn_tc

namespace decode {
int choose_splits(int64_t B, int64_t nkv, int64_t n_slots, int sms);
int64_t workspace_bytes(int64_t B, int64_t nh, int64_t hd, int splits);
bool supported(int dtype, int64_t hd, int64_t nh, int64_t nkv, const void* q, int64_t ldq, const KVCache& kv);
int launch(int dtype, const void* q, int64_t ldq, const KVCache& kv, int64_t n_slots, const int64_t* positions,
           void* out, int64_t ldo, int64_t B, int64_t nh, int64_t nkv, int64_t hd, float scale, int splits, float* ws,
           unsigned* err, cudaStream_t st);
}  // namespace decode

}  // namespace fs
