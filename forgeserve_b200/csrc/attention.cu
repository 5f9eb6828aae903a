// Grouped-query attention against a KV cache addressed through a block table (forgeserve/model.py:69-76
// with forgeserve/kv.py:21-24 or forgeserve/paged.py:71-82).
//
// Semantics kept from the reference: query head h reads KV head h / (nh / nkv) (repeat_interleave,
// model.py:70-71); key slot s is visible to a query at position p iff s <= p (model.py:75), and only the
// n_slots slots of the view exist; scores are scaled by 1/sqrt(hd) (SDPA default). The reference materialises
// the gathered, head-repeated K/V (paged.py:80-81, model.py:70-71); here every kernel reads each key row once
// through the block table instead.
//
// Kernels:
//   attn_generic_kernel  CUDA cores, fp32 or bf16, any even hd <= 256, online softmax over chunks of keys.
//                        Used for the fp32 parity mode and for shapes the tensor-core kernel does not cover.
//   attn_fa_kernel<HD>   bf16, hd in {64, 128}: 64 queries x 64 keys tiles, QK^T and PV on the legacy mma.sync
//                        tensor-core path (m16n8k16, fp32 accumulate), K/V rows fetched with cp.async through the
//                        block table into double-buffered, XOR-swizzled shared memory. Used for short query blocks
//                        (decode steps of several tokens) and block sizes the tcgen05 kernel cannot take.
//   attention_tc.cu      the tcgen05/TMEM/TMA kernel used for prefill (T >= 64).
#include "common.cuh"
#include "kernels.h"

namespace fs {
namespace {

__device__ __forceinline__ int64_t key_offset(const KVCache& kv, int r, int64_t s, int g, int hd, bool& ok) {
  const int64_t bi = s / kv.block_size;
  int64_t blk = -1;
  if (bi < kv.table_cols) blk = kv.table[static_cast<int64_t>(r) * kv.table_stride + bi];
  ok = blk >= 0 && blk < kv.num_blocks;
  return ok ? blk * kv.block_stride + static_cast<int64_t>(g) * kv.head_stride + (s % kv.block_size) * hd : 0;
}

// ======================================================================================= generic kernel
constexpr int GEN_THREADS = 128, GEN_CHUNK = 512;

__device__ __forceinline__ float block_reduce(float v, float* red, bool is_max) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float w = __shfl_xor_sync(0xffffffffu, v, o);
    v = is_max ? fmaxf(v, w) : v + w;
  }
  __syncthreads();
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = v;
  __syncthreads();
  float r = red[0];
#pragma unroll
  for (int i = 1; i < GEN_THREADS / 32; ++i) r = is_max ? fmaxf(r, red[i]) : r + red[i];
  return r;
}

template <typename T>
__global__ void __launch_bounds__(GEN_THREADS)
    attn_generic_kernel(const T* __restrict__ q, int64_t ldq, KVCache kv, int64_t n_slots,
                        const int64_t* __restrict__ positions, T* __restrict__ out, int64_t ldo, int T_new, int nh,
                        int nkv, int hd, float scale, unsigned* err) {
  __shared__ float sq[256];
  __shared__ float sc[GEN_CHUNK];
  __shared__ float red[GEN_THREADS / 32];
  const int64_t tok = blockIdx.x;
  const int h = blockIdx.y;
  const int r = static_cast<int>(tok / T_new);
  const int g = h / (nh / nkv);
  const T* qr = q + tok * ldq + static_cast<int64_t>(h) * hd;
  for (int d = threadIdx.x; d < hd; d += GEN_THREADS) sq[d] = to_f(qr[d]);
  const int64_t pos = positions[tok];
  int64_t n_vis = pos + 1 < n_slots ? pos + 1 : n_slots;
  if (n_vis < 1) n_vis = 1;  // positions are >= 0 for every real query; keep the softmax finite regardless
  __syncthreads();

  const T* kbase = static_cast<const T*>(kv.k);
  const T* vbase = static_cast<const T*>(kv.v);
  float m = -INFINITY, l = 0.f, acc0 = 0.f, acc1 = 0.f;
  const int d0 = threadIdx.x, d1 = threadIdx.x + GEN_THREADS;
  for (int64_t c0 = 0; c0 < n_vis; c0 += GEN_CHUNK) {
    const int n = static_cast<int>(n_vis - c0 < GEN_CHUNK ? n_vis - c0 : GEN_CHUNK);
    float cmax = -INFINITY;
    for (int i = threadIdx.x; i < n; i += GEN_THREADS) {
      bool ok;
      const int64_t off = key_offset(kv, r, c0 + i, g, hd, ok);
      float dot = 0.f;
      if (ok) {
        const T* kr = kbase + off;
        for (int d = 0; d < hd; ++d) dot = fmaf(sq[d], to_f(kr[d]), dot);
      } else {
        flag_error(err, ERR_BAD_SLOT);
      }
      const float s = dot * scale;
      sc[i] = s;
      cmax = fmaxf(cmax, s);
    }
    cmax = block_reduce(cmax, red, true);
    const float m_new = fmaxf(m, cmax);
    const float corr = expf(m - m_new);
    float lsum = 0.f;
    __syncthreads();
    for (int i = threadIdx.x; i < n; i += GEN_THREADS) {
      const float p = expf(sc[i] - m_new);
      sc[i] = p;
      lsum += p;
    }
    lsum = block_reduce(lsum, red, false);
    l = l * corr + lsum;
    acc0 *= corr;
    acc1 *= corr;
    // sc[] complete (block_reduce synchronised)
    for (int i = 0; i < n; ++i) {
      bool ok;
      const int64_t off = key_offset(kv, r, c0 + i, g, hd, ok);
      if (!ok) continue;
      const float p = sc[i];
      const T* vr = vbase + off;
      if (d0 < hd) acc0 = fmaf(p, to_f(vr[d0]), acc0);
      if (d1 < hd) acc1 = fmaf(p, to_f(vr[d1]), acc1);
    }
    m = m_new;
    __syncthreads();
  }
  T* orow = out + tok * ldo + static_cast<int64_t>(h) * hd;
  const float inv = 1.f / l;
  if (d0 < hd) orow[d0] = from_f<T>(acc0 * inv);
  if (d1 < hd) orow[d1] = from_f<T>(acc1 * inv);
}

// ================================================================================== tensor-core kernel
constexpr int FA_BM = 64, FA_BN = 64, FA_THREADS = 128;

__device__ __forceinline__ void cp_async16(uint32_t dst, const void* src, bool valid) {
  const int n = valid ? 16 : 0;  // 0 source bytes = zero fill
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst), "l"(src), "r"(n) : "memory");
}
__device__ __forceinline__ void cp_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}
__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}
__device__ __forceinline__ void mma_bf16(float (&c)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}
__device__ __forceinline__ uint32_t pack2(float lo, float hi) {
  __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&v);
}

// Swizzled shared-memory tile of rows x HD bf16: 16-byte chunk c of row r lives at chunk (c ^ (r & 7)).
template <int HD>
__device__ __forceinline__ uint32_t swz(uint32_t base, int row, int chunk) {
  return base + static_cast<uint32_t>((row * (HD / 8) + (chunk ^ (row & 7))) * 16);
}

template <int HD>
__global__ void __launch_bounds__(FA_THREADS)
    attn_fa_kernel(const __nv_bfloat16* __restrict__ q, int64_t ldq, KVCache kv, int64_t n_slots,
                   const int64_t* __restrict__ positions, __nv_bfloat16* __restrict__ out, int64_t ldo, int T_new,
                   int nh, int nkv, float scale_log2, unsigned* err) {
  constexpr int CH = HD / 8;         // 16-byte chunks per row
  constexpr int KSTEPS = HD / 16;    // k-steps of QK^T
  constexpr int NT_S = FA_BN / 8;    // n-blocks of S per warp (8 keys each)
  constexpr int NT_O = HD / 8;       // n-blocks of O per warp
  extern __shared__ __align__(128) uint8_t smem[];
  const uint32_t sQ = smem_u32(smem);
  const uint32_t sK0 = sQ + FA_BM * HD * 2;
  const uint32_t sV0 = sK0 + 2 * FA_BN * HD * 2;
  constexpr uint32_t KV_TILE = FA_BN * HD * 2;

  const int qb = blockIdx.x, h = blockIdx.y, r = blockIdx.z;
  const int g = h / (nh / nkv);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int j0 = qb * FA_BM;
  const int64_t tok0 = static_cast<int64_t>(r) * T_new;

  // ---- block-wide key range: keys 0 .. min(n_slots, max position + 1) - 1
  __shared__ int64_t s_maxpos[FA_THREADS / 32];
  int64_t my = -1;
  if (tid < FA_BM && j0 + tid < T_new) my = positions[tok0 + j0 + tid];
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const int64_t w = __shfl_xor_sync(0xffffffffu, my, o);
    my = w > my ? w : my;
  }
  if (lane == 0) s_maxpos[warp] = my;

  // ---- Q tile -> shared (rows beyond T are zero)
  for (int i = tid; i < FA_BM * CH; i += FA_THREADS) {
    const int row = i / CH, ch = i % CH;
    const bool valid = j0 + row < T_new;
    const __nv_bfloat16* src = q + (tok0 + (valid ? j0 + row : 0)) * ldq + static_cast<int64_t>(h) * HD + ch * 8;
    cp_async16(swz<HD>(sQ, row, ch), src, valid);
  }
  cp_commit();
  __syncthreads();
  int64_t maxpos = s_maxpos[0];
#pragma unroll
  for (int i = 1; i < FA_THREADS / 32; ++i) maxpos = s_maxpos[i] > maxpos ? s_maxpos[i] : maxpos;
  int64_t n_keys = maxpos + 1 < n_slots ? maxpos + 1 : n_slots;
  if (n_keys < 1) n_keys = 1;
  const int n_tiles = static_cast<int>((n_keys + FA_BN - 1) / FA_BN);

  const __nv_bfloat16* kbase = static_cast<const __nv_bfloat16*>(kv.k);
  const __nv_bfloat16* vbase = static_cast<const __nv_bfloat16*>(kv.v);
  auto load_kv = [&](int kt, int buf) {
    // each thread: chunk (tid % CH) of rows (tid / CH) + i * (FA_THREADS / CH)
    const int ch = tid % CH;
    constexpr int ROWS_PER_PASS = FA_THREADS / CH;
#pragma unroll
    for (int i = 0; i < FA_BN / ROWS_PER_PASS; ++i) {
      const int row = tid / CH + i * ROWS_PER_PASS;
      const int64_t s = static_cast<int64_t>(kt) * FA_BN + row;
      bool ok = false;
      int64_t off = 0;
      if (s < n_keys) {
        off = key_offset(kv, r, s, g, HD, ok);
        if (!ok) flag_error(err, ERR_BAD_SLOT);
      }
      cp_async16(swz<HD>(sK0 + buf * KV_TILE, row, ch), kbase + off + ch * 8, ok);
      cp_async16(swz<HD>(sV0 + buf * KV_TILE, row, ch), vbase + off + ch * 8, ok);
    }
  };
  load_kv(0, 0);
  cp_commit();

  // ---- per-thread rows: g8 = lane / 4 and g8 + 8 of this warp's 16 rows
  const int g8 = lane >> 2, t4 = lane & 3;
  const int row_a = warp * 16 + g8, row_b = row_a + 8;
  int64_t pos_a = (j0 + row_a < T_new) ? positions[tok0 + j0 + row_a] : 0;
  int64_t pos_b = (j0 + row_b < T_new) ? positions[tok0 + j0 + row_b] : 0;
  if (pos_a < 0) pos_a = 0;
  if (pos_b < 0) pos_b = 0;
  const int64_t warp_max = pos_a > pos_b ? pos_a : pos_b;  // reduced across the warp below
  int64_t wmax = warp_max;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const int64_t w = __shfl_xor_sync(0xffffffffu, wmax, o);
    wmax = w > wmax ? w : wmax;
  }

  // ---- Q fragments (registers for the whole loop)
  cp_wait<1>();
  __syncthreads();
  uint32_t qf[KSTEPS][4];
#pragma unroll
  for (int ks = 0; ks < KSTEPS; ++ks) {
    const int row = warp * 16 + (lane & 15);
    const int ch = ks * 2 + (lane >> 4);
    ldsm_x4(swz<HD>(sQ, row, ch), qf[ks][0], qf[ks][1], qf[ks][2], qf[ks][3]);
  }

  float o_acc[NT_O][4];
#pragma unroll
  for (int i = 0; i < NT_O; ++i) o_acc[i][0] = o_acc[i][1] = o_acc[i][2] = o_acc[i][3] = 0.f;
  float m_a = -INFINITY, m_b = -INFINITY, l_a = 0.f, l_b = 0.f;

  for (int kt = 0; kt < n_tiles; ++kt) {
    const int buf = kt & 1;
    if (kt + 1 < n_tiles) load_kv(kt + 1, buf ^ 1);
    cp_commit();
    cp_wait<1>();
    __syncthreads();
    const int64_t key0 = static_cast<int64_t>(kt) * FA_BN;
    if (key0 <= wmax) {  // some row of this warp sees keys of this tile
      const uint32_t sK = sK0 + buf * KV_TILE, sV = sV0 + buf * KV_TILE;
      float s_acc[NT_S][4];
#pragma unroll
      for (int i = 0; i < NT_S; ++i) s_acc[i][0] = s_acc[i][1] = s_acc[i][2] = s_acc[i][3] = 0.f;
#pragma unroll
      for (int ks = 0; ks < KSTEPS; ++ks) {
#pragma unroll
        for (int nb = 0; nb < NT_S; nb += 2) {
          // matrices: (keys nb*8..+7, k lo), (keys nb*8.., k hi), (keys nb*8+8.., k lo), (keys nb*8+8.., k hi)
          const int key = nb * 8 + (lane & 7) + ((lane >> 4) << 3);
          const int ch = ks * 2 + ((lane >> 3) & 1);
          uint32_t b0, b1, b2, b3;
          ldsm_x4(swz<HD>(sK, key, ch), b0, b1, b2, b3);
          mma_bf16(s_acc[nb], qf[ks], b0, b1);
          mma_bf16(s_acc[nb + 1], qf[ks], b2, b3);
        }
      }
      // mask + online softmax (log2 domain)
      float mx_a = -INFINITY, mx_b = -INFINITY;
#pragma unroll
      for (int nb = 0; nb < NT_S; ++nb) {
#pragma unroll
        for (int e = 0; e < 2; ++e) {
          const int64_t key = key0 + nb * 8 + t4 * 2 + e;
          const bool vis_a = key <= pos_a && key < n_slots;
          const bool vis_b = key <= pos_b && key < n_slots;
          s_acc[nb][e] = vis_a ? s_acc[nb][e] * scale_log2 : -INFINITY;
          s_acc[nb][2 + e] = vis_b ? s_acc[nb][2 + e] * scale_log2 : -INFINITY;
          mx_a = fmaxf(mx_a, s_acc[nb][e]);
          mx_b = fmaxf(mx_b, s_acc[nb][2 + e]);
        }
      }
#pragma unroll
      for (int o = 1; o <= 2; o <<= 1) {
        mx_a = fmaxf(mx_a, __shfl_xor_sync(0xffffffffu, mx_a, o));
        mx_b = fmaxf(mx_b, __shfl_xor_sync(0xffffffffu, mx_b, o));
      }
      const float mn_a = fmaxf(m_a, mx_a), mn_b = fmaxf(m_b, mx_b);
      // rows with nothing visible so far keep m = -inf; use 0 as the subtrahend so exp2 stays finite
      const float sub_a = mn_a == -INFINITY ? 0.f : mn_a, sub_b = mn_b == -INFINITY ? 0.f : mn_b;
      const float corr_a = exp2f(m_a - sub_a), corr_b = exp2f(m_b - sub_b);
      m_a = mn_a;
      m_b = mn_b;
      float rs_a = 0.f, rs_b = 0.f;
      uint32_t pf[NT_S / 2][4];
#pragma unroll
      for (int nb = 0; nb < NT_S; ++nb) {
        const float p0 = exp2f(s_acc[nb][0] - sub_a), p1 = exp2f(s_acc[nb][1] - sub_a);
        const float p2 = exp2f(s_acc[nb][2] - sub_b), p3 = exp2f(s_acc[nb][3] - sub_b);
        rs_a += p0 + p1;
        rs_b += p2 + p3;
        // S accumulator layout -> A fragment of P (16 x 16 per pair of n-blocks)
        const int kk = nb >> 1, hi = nb & 1;
        pf[kk][hi * 2 + 0] = pack2(p0, p1);
        pf[kk][hi * 2 + 1] = pack2(p2, p3);
      }
      l_a = l_a * corr_a + rs_a;  // partial (this thread's columns); reduced across the quad at the end
      l_b = l_b * corr_b + rs_b;
#pragma unroll
      for (int i = 0; i < NT_O; ++i) {
        o_acc[i][0] *= corr_a;
        o_acc[i][1] *= corr_a;
        o_acc[i][2] *= corr_b;
        o_acc[i][3] *= corr_b;
      }
      // O += P V
#pragma unroll
      for (int kk = 0; kk < NT_S / 2; ++kk) {
#pragma unroll
        for (int nb = 0; nb < NT_O; nb += 2) {
          // matrices (keys kk*16..+7, hd nb*8..), (keys kk*16+8.., hd nb*8..), (keys kk*16.., hd nb*8+8..), (+8, +8)
          const int key = kk * 16 + (lane & 7) + (((lane >> 3) & 1) << 3);
          const int ch = nb + (lane >> 4);
          uint32_t b0, b1, b2, b3;
          ldsm_x4_t(swz<HD>(sV, key, ch), b0, b1, b2, b3);
          // pf[kk] is {a0 (row g, keys 0-7), a1 (row g+8, keys 0-7), a2 (row g, keys 8-15), a3 (row g+8, 8-15)}
          const uint32_t a[4] = {pf[kk][0], pf[kk][1], pf[kk][2], pf[kk][3]};
          mma_bf16(o_acc[nb], a, b0, b1);
          mma_bf16(o_acc[nb + 1], a, b2, b3);
        }
      }
    }
    __syncthreads();  // the buffer is overwritten by the next iteration's prefetch
  }
  cp_wait<0>();

#pragma unroll
  for (int o = 1; o <= 2; o <<= 1) {
    l_a += __shfl_xor_sync(0xffffffffu, l_a, o);
    l_b += __shfl_xor_sync(0xffffffffu, l_b, o);
  }
  const float inv_a = l_a > 0.f ? 1.f / l_a : 0.f, inv_b = l_b > 0.f ? 1.f / l_b : 0.f;
  const bool ok_a = j0 + row_a < T_new, ok_b = j0 + row_b < T_new;
  __nv_bfloat16* oa = out + (tok0 + j0 + row_a) * ldo + static_cast<int64_t>(h) * HD;
  __nv_bfloat16* ob = out + (tok0 + j0 + row_b) * ldo + static_cast<int64_t>(h) * HD;
#pragma unroll
  for (int nb = 0; nb < NT_O; ++nb) {
    const int col = nb * 8 + t4 * 2;
    if (ok_a) *reinterpret_cast<uint32_t*>(oa + col) = pack2(o_acc[nb][0] * inv_a, o_acc[nb][1] * inv_a);
    if (ok_b) *reinterpret_cast<uint32_t*>(ob + col) = pack2(o_acc[nb][2] * inv_b, o_acc[nb][3] * inv_b);
  }
}

template <int HD>
int launch_fa(const void* q, int64_t ldq, const KVCache& kv, int64_t n_slots, const int64_t* positions, void* out,
              int64_t ldo, int64_t B, int64_t T, int64_t nh, int64_t nkv, float scale, cudaStream_t st) {
  constexpr int SMEM = (FA_BM + 4 * FA_BN) * HD * 2;
  static bool attr[64] = {false};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev >= 0 && dev < 64 && !attr[dev]) {
    if (cudaFuncSetAttribute(attn_fa_kernel<HD>, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM) != cudaSuccess)
      return check_launch("attn_fa set smem");
    attr[dev] = true;
  }
  dim3 grid(static_cast<unsigned>((T + FA_BM - 1) / FA_BM), static_cast<unsigned>(nh), static_cast<unsigned>(B));
  attn_fa_kernel<HD><<<grid, FA_THREADS, SMEM, st>>>(
      static_cast<const __nv_bfloat16*>(q), ldq, kv, n_slots, positions, static_cast<__nv_bfloat16*>(out), ldo,
      static_cast<int>(T), static_cast<int>(nh), static_cast<int>(nkv), scale * 1.4426950408889634f, error_word());
  return check_launch("attn_fa_kernel");
}

}  // namespace

int attention(int dtype, const void* q, int64_t ldq, const KVCache& kv, int64_t n_slots, const int64_t* positions,
              void* out, int64_t ldo, int64_t B, int64_t T, int64_t nh, int64_t nkv, int64_t hd, float scale,
              int impl, cudaStream_t st) {
  if (B <= 0 || T <= 0 || nh <= 0) return 0;
  if (nkv <= 0 || nh % nkv) return fail("attention: n_heads must be a multiple of n_kv_heads");
  if (hd <= 0 || hd > 256 || hd % 2) return fail("attention: head_dim must be even and <= 256");
  if (B * T > INT32_MAX || B > 65535 || nh > 65535) return fail("attention: too many queries");
  const bool aligned = ((reinterpret_cast<uintptr_t>(q) | reinterpret_cast<uintptr_t>(out) |
                         reinterpret_cast<uintptr_t>(kv.k) | reinterpret_cast<uintptr_t>(kv.v)) & 15) == 0 &&
                       ldq % 8 == 0 && ldo % 8 == 0 && kv.block_stride % 8 == 0 && kv.head_stride % 8 == 0;
  const bool tc_ok = dtype == BF16 && attn_tc::supported(q, ldq, kv, hd, T);
  const bool fa_ok = dtype == BF16 && aligned && (hd == 64 || hd == 128);
  if (impl == 3 && !tc_ok) return fail("attention: the tcgen05 kernel does not support this layout");
  if (impl == 2 && !fa_ok) return fail("attention: the mma.sync kernel does not support this layout");
  if (impl == 3 || (impl == 0 && tc_ok && T >= 64))
    return attn_tc::launch(q, ldq, kv, n_slots, positions, out, ldo, B, T, nh, nkv, hd, scale, st);
  if (impl == 2 || (impl == 0 && fa_ok && T >= 16)) {
    if (hd == 128) return launch_fa<128>(q, ldq, kv, n_slots, positions, out, ldo, B, T, nh, nkv, scale, st);
    return launch_fa<64>(q, ldq, kv, n_slots, positions, out, ldo, B, T, nh, nkv, scale, st);
  }
  dim3 grid(static_cast<unsigned>(B * T), static_cast<unsigned>(nh));
  if (dtype == F32)
    attn_generic_kernel<float><<<grid, GEN_THREADS, 0, st>>>(static_cast<const float*>(q), ldq, kv, n_slots, positions,
                                                              static_cast<float*>(out), ldo, static_cast<int>(T),
                                                              static_cast<int>(nh), static_cast<int>(nkv),
                                                              static_cast<int>(hd), scale, error_word());
  else if (dtype == BF16)
    attn_generic_kernel<__nv_bfloat16><<<grid, GEN_THREADS, 0, st>>>(
        static_cast<const __nv_bfloat16*>(q), ldq, kv, n_slots, positions, static_cast<__nv_bfloat16*>(out), ldo,
        static_cast<int>(T), static_cast<int>(nh), static_cast<int>(nkv), static_cast<int>(hd), scale, error_word());
  else
    return fail("attention: unsupported dtype");
  return check_launch("attn_generic_kernel");
}

}  // namespace fs
