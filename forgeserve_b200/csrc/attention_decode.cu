// Decode attention (one new query per batch row) over a paged or contiguous KV cache: split-KV "flash decoding".
//
// Same semantics as attention.cu (forgeserve/model.py:69-76): query head h reads KV head h / rep, key slot s is
// visible iff s <= position and s < n_slots, scale 1/sqrt(hd). This is the step the reference's Engine runs for
// every running request (forgeserve/engine.py:125, paged gather at forgeserve/paged.py:80-81). It is HBM-bound,
// so each CTA reads every K/V row of its key range exactly once, for all `rep` query heads of its KV head:
//
//   attn_decode_kernel   grid (splits, n_kv, B), 128 threads. Per 64-key chunk: K and V rows fetched with
//                        cp.async through the block table into row-padded shared memory (conflict-free 16-byte
//                        reads); scores of the rep heads (fp32 FMA); online softmax statistics per head (one warp
//                        per head, kept in shared memory); P V accumulated per output dimension. With one split the
//                        normalised output is written directly; otherwise the split's unnormalised O and its
//                        (max, sum) go to the workspace.
//   attn_combine_kernel  grid (B, nh): merges the splits (log-sum-exp weights) into the output.
//
// Workspace (fp32): O partials [B][nh][splits][hd], then (max, sum) pairs [B][nh][splits][2].
#include <string>

#include "../../include/forgeserve_b200.h"
#include "common.cuh"
#include "kernels.h"

namespace fs {
namespace decode {

constexpr int THREADS = 128, CHUNK = 64, MAX_REP = 8, MAX_SPLITS = 64;

__device__ __forceinline__ int64_t key_row_offset(const KVCache& kv, int r, int64_t s, int g, int hd, bool& ok) {
  const int64_t bi = s / kv.block_size;
  int64_t blk = -1;
  if (bi < kv.table_cols) blk = kv.table[static_cast<int64_t>(r) * kv.table_stride + bi];
  ok = blk >= 0 && blk < kv.num_blocks;
  return ok ? blk * kv.block_stride + static_cast<int64_t>(g) * kv.head_stride + (s % kv.block_size) * hd : 0;
}

__device__ __forceinline__ void cp_async16(uint32_t dst, const void* src, bool valid) {
  const int n = valid ? 16 : 0;   // 0 source bytes: zero fill
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst), "l"(src), "r"(n) : "memory");
}
__device__ __forceinline__ void cp_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
__device__ __forceinline__ void cp_wait_all() { asm volatile("cp.async.wait_group 0;" ::: "memory"); }

template <typename T, int HD>
struct Smem {
  static constexpr int ROW = HD * static_cast<int>(sizeof(T)) + 16;   // padded row (bytes)
  static constexpr int K_OFF = 0, V_OFF = CHUNK * ROW;
  static constexpr int Q_OFF = 2 * CHUNK * ROW;                       // fp32 [MAX_REP][HD]
  static constexpr int P_OFF = Q_OFF + MAX_REP * HD * 4;              // fp32 [MAX_REP][CHUNK]
  static constexpr int STAT_OFF = P_OFF + MAX_REP * CHUNK * 4;        // fp32 m[MAX_REP], l[MAX_REP], corr[MAX_REP]
  static constexpr int BYTES = STAT_OFF + 3 * MAX_REP * 4;
};

template <typename T, int HD>
__global__ void __launch_bounds__(THREADS)
    attn_decode_kernel(const T* __restrict__ q, int64_t ldq, KVCache kv, int64_t n_slots,
                       const int64_t* __restrict__ positions, T* __restrict__ out, int64_t ldo, int nh, int rep,
                       int splits, float scale, float* __restrict__ ws, unsigned* err) {
  using S = Smem<T, HD>;
  constexpr int VEC = 16 / static_cast<int>(sizeof(T));   // elements per 16-byte chunk
  constexpr int CPR = HD / VEC;                           // chunks per row
  extern __shared__ __align__(16) uint8_t smem[];
  float* qs = reinterpret_cast<float*>(smem + S::Q_OFF);
  float* ps = reinterpret_cast<float*>(smem + S::P_OFF);
  float* m_s = reinterpret_cast<float*>(smem + S::STAT_OFF);
  float* l_s = m_s + MAX_REP;
  float* c_s = l_s + MAX_REP;

  const int split = blockIdx.x, g = blockIdx.y, r = blockIdx.z;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  int64_t pos = positions[r];
  if (pos < 0) pos = 0;
  const int64_t n_vis = pos + 1 < n_slots ? pos + 1 : n_slots;
  const int64_t per = ((n_vis + splits - 1) / splits + CHUNK - 1) / CHUNK * CHUNK;
  const int64_t k_begin = static_cast<int64_t>(split) * per;
  const int64_t k_end = k_begin + per < n_vis ? k_begin + per : n_vis;

  for (int i = tid; i < rep * HD; i += THREADS)
    qs[i] = to_f(q[static_cast<int64_t>(r) * ldq + static_cast<int64_t>(g * rep + i / HD) * HD + i % HD]);
  if (tid < MAX_REP) {
    m_s[tid] = -INFINITY;
    l_s[tid] = 0.f;
    c_s[tid] = 1.f;
  }
  float acc[MAX_REP];
#pragma unroll
  for (int h = 0; h < MAX_REP; ++h) acc[h] = 0.f;
  const T* kbase = static_cast<const T*>(kv.k);
  const T* vbase = static_cast<const T*>(kv.v);
  const int d = tid;   // this thread's output dimension (threads >= HD accumulate nothing)

  for (int64_t c0 = k_begin; c0 < k_end; c0 += CHUNK) {
    const int n = static_cast<int>(k_end - c0 < CHUNK ? k_end - c0 : CHUNK);
    __syncthreads();   // the previous chunk is fully consumed (and q / statistics are initialised)
    for (int i = tid; i < CHUNK * CPR; i += THREADS) {
      const int row = i / CPR, ch = i % CPR;
      bool ok = false;
      int64_t off = 0;
      if (row < n) {
        off = key_row_offset(kv, r, c0 + row, g, HD, ok);
        if (!ok) flag_error(err, ERR_BAD_SLOT);
      }
      cp_async16(smem_u32(smem + S::K_OFF + row * S::ROW + ch * 16), kbase + off + ch * VEC, ok);
      cp_async16(smem_u32(smem + S::V_OFF + row * S::ROW + ch * 16), vbase + off + ch * VEC, ok);
    }
    cp_commit();
    cp_wait_all();
    __syncthreads();
    {   // scores: thread -> key tid % CHUNK, heads tid / CHUNK + 2 i
      const int kk = tid % CHUNK;
      const uint8_t* krow = smem + S::K_OFF + kk * S::ROW;
      for (int h = tid / CHUNK; h < rep; h += THREADS / CHUNK) {
        const float* qh = qs + h * HD;
        float dot = 0.f;
#pragma unroll 4
        for (int ch = 0; ch < CPR; ++ch) {
          const uint4 u = *reinterpret_cast<const uint4*>(krow + ch * 16);
          const T* e = reinterpret_cast<const T*>(&u);
#pragma unroll
          for (int j = 0; j < VEC; ++j) dot = fmaf(qh[ch * VEC + j], to_f(e[j]), dot);
        }
        ps[h * CHUNK + kk] = kk < n ? dot * scale : -INFINITY;
      }
    }
    __syncthreads();
    for (int h = warp; h < rep; h += THREADS / 32) {   // softmax statistics: warp w owns heads w, w + 4
      const float s0 = ps[h * CHUNK + lane], s1 = ps[h * CHUNK + lane + 32];
      float mx = fmaxf(s0, s1);
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
      const float m_old = m_s[h];
      const float m_new = fmaxf(m_old, mx);            // finite: every chunk holds at least one visible key
      const float p0 = expf(s0 - m_new), p1 = expf(s1 - m_new);
      float sum = p0 + p1;
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
      ps[h * CHUNK + lane] = p0;
      ps[h * CHUNK + lane + 32] = p1;
      __syncwarp();
      if (lane == 0) {
        const float c = expf(m_old - m_new);           // 0 on the first chunk (m_old = -inf)
        c_s[h] = c;
        m_s[h] = m_new;
        l_s[h] = l_s[h] * c + sum;
      }
    }
    __syncthreads();
    if (d < HD) {   // P V for this thread's output dimension (heads unrolled so acc stays in registers)
#pragma unroll
      for (int h = 0; h < MAX_REP; ++h) {
        if (h < rep) {
          const float* ph = ps + h * CHUNK;
          float a = acc[h] * c_s[h];
          for (int k = 0; k < n; ++k)
            a = fmaf(ph[k], to_f(reinterpret_cast<const T*>(smem + S::V_OFF + k * S::ROW)[d]), a);
          acc[h] = a;
        }
      }
    }
  }
  __syncthreads();
  if (d < HD) {
#pragma unroll
    for (int h = 0; h < MAX_REP; ++h) {
      if (h >= rep) break;
      const int hh = g * rep + h;
      if (splits == 1) {
        const float l = l_s[h];
        out[static_cast<int64_t>(r) * ldo + static_cast<int64_t>(hh) * HD + d] = from_f<T>(l > 0.f ? acc[h] / l : 0.f);
      } else {
        const int64_t slot = (static_cast<int64_t>(r) * nh + hh) * splits + split;
        ws[slot * HD + d] = acc[h];
      }
    }
  }
  if (splits > 1 && tid < rep) {
    const int64_t slot = (static_cast<int64_t>(r) * nh + g * rep + tid) * splits + split;
    float* ml = ws + static_cast<int64_t>(gridDim.z) * nh * splits * HD;
    ml[2 * slot] = m_s[tid];       // -inf for an empty split
    ml[2 * slot + 1] = l_s[tid];
  }
}

template <typename T, int HD>
__global__ void __launch_bounds__(THREADS)
    attn_combine_kernel(const float* __restrict__ ws, int B, int nh, int splits, T* __restrict__ out, int64_t ldo) {
  const int r = blockIdx.x, h = blockIdx.y, d = threadIdx.x;
  const int64_t base = (static_cast<int64_t>(r) * nh + h) * splits;
  const float* ml = ws + static_cast<int64_t>(B) * nh * splits * HD;
  float M = -INFINITY;
  for (int s = 0; s < splits; ++s) M = fmaxf(M, ml[2 * (base + s)]);
  float L = 0.f, o = 0.f;
  for (int s = 0; s < splits; ++s) {
    const float m = ml[2 * (base + s)];
    const float w = m == -INFINITY ? 0.f : expf(m - M);
    L += w * ml[2 * (base + s) + 1];
    if (d < HD) o += w * ws[(base + s) * HD + d];
  }
  if (d < HD) out[static_cast<int64_t>(r) * ldo + static_cast<int64_t>(h) * HD + d] = from_f<T>(L > 0.f ? o / L : 0.f);
}

template <typename T, int HD>
int launch_t(const void* q, int64_t ldq, const KVCache& kv, int64_t n_slots, const int64_t* positions, void* out,
             int64_t ldo, int64_t B, int64_t nh, int64_t nkv, float scale, int splits, float* ws, cudaStream_t st) {
  using S = Smem<T, HD>;
  static bool attr[64] = {false};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev >= 0 && dev < 64 && !attr[dev]) {
    if (cudaFuncSetAttribute(attn_decode_kernel<T, HD>, cudaFuncAttributeMaxDynamicSharedMemorySize, S::BYTES) !=
        cudaSuccess)
      return check_launch("attn_decode set smem");
    attr[dev] = true;
  }
  unsigned* err = error_word();
  if (!err) return -1;
  dim3 grid(static_cast<unsigned>(splits), static_cast<unsigned>(nkv), static_cast<unsigned>(B));
  attn_decode_kernel<T, HD><<<grid, THREADS, S::BYTES, st>>>(
      static_cast<const T*>(q), ldq, kv, n_slots, positions, static_cast<T*>(out), ldo, static_cast<int>(nh),
      static_cast<int>(nh / nkv), splits, scale, ws, err);
  if (check_launch("attn_decode_kernel")) return -1;
  if (splits > 1) {
    attn_combine_kernel<T, HD><<<dim3(static_cast<unsigned>(B), static_cast<unsigned>(nh)), THREADS, 0, st>>>(
        ws, static_cast<int>(B), static_cast<int>(nh), splits, static_cast<T*>(out), ldo);
    return check_launch("attn_combine_kernel");
  }
  return 0;
}

int choose_splits(int64_t B, int64_t nkv, int64_t n_slots, int sm_target) {
  const int64_t base = B * nkv;
  int64_t s = (sm_target + base - 1) / base;             // enough CTAs to fill the GPU
  const int64_t by_len = (n_slots + 4 * CHUNK - 1) / (4 * CHUNK);   // at least 256 keys per split
  if (s > by_len) s = by_len;
  if (s > MAX_SPLITS) s = MAX_SPLITS;
  return s < 1 ? 1 : static_cast<int>(s);
}

int64_t workspace_bytes(int64_t B, int64_t nh, int64_t hd, int splits) {
  return splits <= 1 ? 0 : B * nh * splits * (hd + 2) * static_cast<int64_t>(sizeof(float));
}

bool supported(int dtype, int64_t hd, int64_t nh, int64_t nkv, const void* q, int64_t ldq, const KVCache& kv) {
  if (hd != 64 && hd != 128) return false;
  if (nkv <= 0 || nh % nkv || nh / nkv > MAX_REP) return false;
  const int64_t vec = dtype == F32 ? 4 : 8;
  if (ldq % vec || kv.block_stride % vec || kv.head_stride % vec) return false;
  return ((reinterpret_cast<uintptr_t>(q) | reinterpret_cast<uintptr_t>(kv.k) | reinterpret_cast<uintptr_t>(kv.v)) &
          15) == 0;
}

int launch(int dtype, const void* q, int64_t ldq, const KVCache& kv, int64_t n_slots, const int64_t* positions,
           void* out, int64_t ldo, int64_t B, int64_t nh, int64_t nkv, int64_t hd, float scale, int splits, float* ws,
           cudaStream_t st) {
  if (B > 65535 || nkv > 65535) return fail("attention_decode: grid too large");
  if (splits > 1 && !ws) return fail("attention_decode: a workspace is needed for more than one split");
  if (dtype == BF16 && hd == 128)
    return launch_t<__nv_bfloat16, 128>(q, ldq, kv, n_slots, positions, out, ldo, B, nh, nkv, scale, splits, ws, st);
  if (dtype == BF16 && hd == 64)
    return launch_t<__nv_bfloat16, 64>(q, ldq, kv, n_slots, positions, out, ldo, B, nh, nkv, scale, splits, ws, st);
  if (dtype == F32 && hd == 128)
    return launch_t<float, 128>(q, ldq, kv, n_slots, positions, out, ldo, B, nh, nkv, scale, splits, ws, st);
  if (dtype == F32 && hd == 64)
    return launch_t<float, 64>(q, ldq, kv, n_slots, positions, out, ldo, B, nh, nkv, scale, splits, ws, st);
  return fail("attention_decode: head_dim must be 64 or 128 and dtype fp32 or bf16");
}

}  // namespace decode
}  // namespace fs

// =============================================================================================================
// Decode attention without any device allocation.
//
// Some callers cannot allocate device memory at the point where they run a decode step: a host framework that
// has reserved all of the GPU's memory in its own pool up front (and fails any other cudaMalloc), a plugin that
// is only handed device pointers by its host, or a serving loop that cannot afford the device-wide
// synchronisation a cudaMalloc / cudaFree may cause in the middle of a step. fs_attention_decode needs a
// workspace for its per-split partial results; this entry point uses a fixed scratch area that is part of the
// library image instead: a file-scope __device__ array of kStaticScratchBytes (4 MiB), which every GPU that
// loads the library holds until the process exits.
//
// * Set-up: the first call on a device resolves the array's device address with cudaGetSymbolAddress (and sets
//   the kernels' shared-memory attribute) with that device current; make that first call before any stream
//   capture on that device.
// * Limit: calls whose split partials need more than kStaticScratchBytes are refused with an error naming the
//   size (fs_attention_decode_workspace() gives the size a call needs).
// * Sharing: every call uses the same array and leaves its contents behind; each call writes every partial it
//   reads, so nothing needs clearing, but calls that overlap on the GPU (different streams, no ordering) race on
//   the array and must not be issued.
// * It allocates nothing: no cudaMalloc, cudaFree or allocating library routine. Device-side input errors (a block
//   table entry outside the pool) are recorded in the library's error word only if that word already exists on
//   the device (any other entry point creates it); the kernel never reads outside the cache either way.
// =============================================================================================================
namespace fs {
namespace decode {

constexpr int64_t kStaticScratchBytes = int64_t(4) << 20;
static __device__ __align__(256) unsigned char g_static_scratch[kStaticScratchBytes];

struct StaticScratch {
  float* ptr = nullptr;
  bool ready = false;
};

static int static_scratch(float** out) {
  static StaticScratch per_dev[64];
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return fail("no current CUDA device");
  StaticScratch& s = per_dev[dev];
  if (!s.ready) {
    void* p = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&p, g_static_scratch);
    if (e != cudaSuccess) return fail(std::string("cudaGetSymbolAddress(decode scratch): ") + cudaGetErrorString(e));
    using S128 = Smem<float, 128>;
    using S64 = Smem<float, 64>;
    if (cudaFuncSetAttribute(attn_decode_kernel<float, 128>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             S128::BYTES) != cudaSuccess ||
        cudaFuncSetAttribute(attn_decode_kernel<float, 64>, cudaFuncAttributeMaxDynamicSharedMemorySize, S64::BYTES) !=
            cudaSuccess ||
        cudaFuncSetAttribute(attn_decode_kernel<__nv_bfloat16, 128>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             Smem<__nv_bfloat16, 128>::BYTES) != cudaSuccess ||
        cudaFuncSetAttribute(attn_decode_kernel<__nv_bfloat16, 64>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             Smem<__nv_bfloat16, 64>::BYTES) != cudaSuccess)
      return check_launch("decode scratch set-up");
    s.ptr = static_cast<float*>(p);
    s.ready = true;
  }
  *out = s.ptr;
  return 0;
}

template <typename T, int HD>
static int launch_static_t(const void* q, int64_t ldq, const KVCache& kv, int64_t n_slots, const int64_t* positions,
                           void* out, int64_t ldo, int64_t B, int64_t nh, int64_t nkv, float scale, int splits,
                           float* ws, unsigned* err, cudaStream_t st) {
  using S = Smem<T, HD>;
  dim3 grid(static_cast<unsigned>(splits), static_cast<unsigned>(nkv), static_cast<unsigned>(B));
  attn_decode_kernel<T, HD><<<grid, THREADS, S::BYTES, st>>>(
      static_cast<const T*>(q), ldq, kv, n_slots, positions, static_cast<T*>(out), ldo, static_cast<int>(nh),
      static_cast<int>(nh / nkv), splits, scale, ws, err);
  if (check_launch("attn_decode_kernel")) return -1;
  if (splits > 1) {
    attn_combine_kernel<T, HD><<<dim3(static_cast<unsigned>(B), static_cast<unsigned>(nh)), THREADS, 0, st>>>(
        ws, static_cast<int>(B), static_cast<int>(nh), splits, static_cast<T*>(out), ldo);
    return check_launch("attn_combine_kernel");
  }
  return 0;
}

}  // namespace decode
unsigned* error_word_if_present();
}  // namespace fs

extern "C" int fs_attention_decode_static(const void* q, int64_t ldq, const fs_kv_cache* kvd, int64_t n_slots,
                                          const int64_t* positions, void* out, int64_t ldo, int64_t B, int64_t nh,
                                          int64_t nkv, int64_t hd, float scale, int dtype, void* stream) {
  using namespace fs;
  using namespace fs::decode;
  if (B <= 0) return 0;
  if (!kvd || !kvd->k || !kvd->v || !kvd->table) return fail("fs_attention_decode_static: NULL cache pointer");
  if (kvd->block_size <= 0 || kvd->num_blocks <= 0 || kvd->table_cols <= 0)
    return fail("fs_attention_decode_static: empty cache");
  KVCache cache;
  cache.k = kvd->k;
  cache.v = kvd->v;
  cache.table = kvd->table;
  cache.table_stride = kvd->table_stride;
  cache.table_cols = kvd->table_cols;
  cache.block_size = kvd->block_size;
  cache.block_stride = kvd->block_stride;
  cache.head_stride = kvd->head_stride;
  cache.num_blocks = kvd->num_blocks;
  const KVCache* kv = &cache;
  if (!q || !positions || !out) return fail("fs_attention_decode_static: NULL pointer");
  if (n_slots <= 0) return fail("fs_attention_decode_static: the cache view has no slots");
  if (dtype != F32 && dtype != BF16) return fail("fs_attention_decode_static: unsupported dtype");
  if (ldq < nh * hd || ldo < nh * hd) return fail("fs_attention_decode_static: row stride too small");
  if (B > 65535 || nkv > 65535) return fail("fs_attention_decode_static: grid too large");
  if (!supported(dtype, hd, nh, nkv, q, ldq, *kv))
    return fail("fs_attention_decode_static: needs head_dim 64 or 128, n_heads / n_kv_heads <= 8, aligned rows");
  int sms = 0, dev = 0;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const int splits = choose_splits(B, nkv, n_slots, 2 * (sms > 0 ? sms : 148));
  const int64_t need = workspace_bytes(B, nh, hd, splits);
  if (need > kStaticScratchBytes)
    return fail("fs_attention_decode_static: this call needs " + std::to_string(need) +
                " bytes of scratch, more than the fixed " + std::to_string(kStaticScratchBytes) +
                " bytes; use fs_attention_decode with a caller-owned workspace");
  float* ws = nullptr;
  if (static_scratch(&ws)) return -1;
  unsigned* err = error_word_if_present();
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (dtype == BF16 && hd == 128)
    return launch_static_t<__nv_bfloat16, 128>(q, ldq, *kv, n_slots, positions, out, ldo, B, nh, nkv, scale, splits, ws, err, st);
  if (dtype == BF16)
    return launch_static_t<__nv_bfloat16, 64>(q, ldq, *kv, n_slots, positions, out, ldo, B, nh, nkv, scale, splits, ws, err, st);
  if (hd == 128)
    return launch_static_t<float, 128>(q, ldq, *kv, n_slots, positions, out, ldo, B, nh, nkv, scale, splits, ws, err, st);
  return launch_static_t<float, 64>(q, ldq, *kv, n_slots, positions, out, ldo, B, nh, nkv, scale, splits, ws, err, st);
}
