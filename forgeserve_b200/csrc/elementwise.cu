// HBM-bound kernels of a decoder stage: RMSNorm, RoPE fused with the KV-cache slot store, the paged
// gather that backs the KV "view" protocol, the token embedding and greedy argmax.
//
// KV-cache addressing (shared with attention.cu). Slot s of batch row r, KV head g lives at
//     base + table[r * table_stride + s / block_size] * block_stride + g * head_stride + (s % block_size) * hd
// which covers both cache layouts of the reference:
//   * paged pool (num_blocks, n_kv, block_size, hd)     forgeserve/paged.py:48-50; table = block table
//   * contiguous per-row cache (B, n_kv, capacity, hd)  forgeserve/kv.py:10-24; block_size = capacity,
//     table[r] = r (one "block" per row)
#include "common.cuh"
#include "kernels.h"

namespace fs {

namespace {

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// --------------------------------------------------------------------------------------------- RMSNorm
// y = T( T(x * rsqrt(mean(x^2) + eps)) * w ), mean in fp32   (forgeserve/model.py:29-31)
template <typename T, int THREADS>
__global__ void __launch_bounds__(THREADS)
    rmsnorm_kernel(const T* __restrict__ x, int64_t xs, const T* __restrict__ w, T* __restrict__ y, int64_t ys,
                   int dim, float eps) {
  pdl_trigger();
  pdl_wait();   // launched with PDL: everything below reads or writes other kernels' data
  const int64_t row = blockIdx.x;
  const T* xr = x + row * xs;
  T* yr = y + row * ys;
  __shared__ float red[THREADS / 32];
  float ss = 0.f;
  constexpr int VEC = 16 / sizeof(T);
  const bool vec = (dim % VEC == 0) && ((reinterpret_cast<uintptr_t>(xr) & 15) == 0) &&
                   ((reinterpret_cast<uintptr_t>(yr) & 15) == 0) && ((reinterpret_cast<uintptr_t>(w) & 15) == 0);
  if (vec) {
    for (int i = threadIdx.x * VEC; i < dim; i += THREADS * VEC) {
      const uint4 u = *reinterpret_cast<const uint4*>(xr + i);
      const T* e = reinterpret_cast<const T*>(&u);
#pragma unroll
      for (int j = 0; j < VEC; ++j) {
        const float f = to_f(e[j]);
        ss += f * f;
      }
    }
  } else {
    for (int i = threadIdx.x; i < dim; i += THREADS) {
      const float f = to_f(xr[i]);
      ss += f * f;
    }
  }
  ss = warp_sum(ss);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
  __syncthreads();
  if (threadIdx.x < 32) {
    float v = threadIdx.x < THREADS / 32 ? red[threadIdx.x] : 0.f;
    v = warp_sum(v);
    if (threadIdx.x == 0) red[0] = v;
  }
  __syncthreads();
  const float r = rsqrtf(red[0] / static_cast<float>(dim) + eps);
  if (vec) {
    for (int i = threadIdx.x * VEC; i < dim; i += THREADS * VEC) {
      const uint4 u = *reinterpret_cast<const uint4*>(xr + i);
      const uint4 wu = *reinterpret_cast<const uint4*>(w + i);
      const T* e = reinterpret_cast<const T*>(&u);
      const T* we = reinterpret_cast<const T*>(&wu);
      uint4 o;
      T* oe = reinterpret_cast<T*>(&o);
#pragma unroll
      for (int j = 0; j < VEC; ++j) oe[j] = from_f<T>(rnd<T>(to_f(e[j]) * r) * to_f(we[j]));
      *reinterpret_cast<uint4*>(yr + i) = o;
    }
  } else {
    for (int i = threadIdx.x; i < dim; i += THREADS) yr[i] = from_f<T>(rnd<T>(to_f(xr[i]) * r) * to_f(w[i]));
  }
}

// ------------------------------------------------------------------------------- RoPE + KV slot store
// One block per new token. qkv row layout: [q: nh*hd | k: nkv*hd | v: nkv*hd] (the fused q/k/v projection).
// q is rotated in place; rotated k and raw v are stored into the cache slot of the token.
// Rotation (forgeserve/model.py:40-45): half split, c = T(cos[pos]), s = T(sin[pos]),
//   out1 = T(T(x1*c) - T(x2*s)), out2 = T(T(x2*c) + T(x1*s)).
// Slot of token j of row r: slot_base + j (contiguous cache, appended after the cached prefix) or
// positions[r, j] (paged cache, written at its absolute position; forgeserve/paged.py:74-78).
template <typename T>
__global__ void rope_kv_kernel(T* __restrict__ qkv, int64_t ld, const float* __restrict__ cos_t,
                               const float* __restrict__ sin_t, int rope_rows, const int64_t* __restrict__ positions,
                               KVCache kv, int T_new, int nh, int nkv, int hd, int64_t slot_base, int slot_from_pos,
                               int apply_rope, unsigned* err) {
  pdl_trigger();
  pdl_wait();   // launched with PDL: everything below reads or writes other kernels' data
  const int64_t tok = blockIdx.x;
  const int r = static_cast<int>(tok / T_new), j = static_cast<int>(tok % T_new);
  const int64_t pos = positions[tok];
  const int half = hd / 2;
  T* row = qkv + tok * ld;
  const bool pos_ok = pos >= 0 && pos < rope_rows;
  if (apply_rope && !pos_ok) {
    if (threadIdx.x == 0) flag_error(err, ERR_BAD_POSITION);
    return;
  }
  const int64_t slot = slot_from_pos ? pos : slot_base + j;
  const int64_t blk_idx = slot / kv.block_size;
  bool slot_ok = slot >= 0 && blk_idx < kv.table_cols;
  int64_t blk = slot_ok ? kv.table[static_cast<int64_t>(r) * kv.table_stride + blk_idx] : -1;
  slot_ok = slot_ok && blk >= 0 && blk < kv.num_blocks;
  if (!slot_ok && threadIdx.x == 0) flag_error(err, ERR_BAD_SLOT);
  const int64_t slot_off = slot_ok ? blk * kv.block_stride + (slot % kv.block_size) * hd : 0;

  const float* cr = cos_t + pos * half;
  const float* sr = sin_t + pos * half;
  // rotate q (nh heads) and k (nkv heads): (nh + nkv) * half pairs
  const int pairs = (nh + nkv) * half;
  for (int i = threadIdx.x; i < pairs; i += blockDim.x) {
    const int h = i / half, d = i % half;
    T* base = row + h * hd;
    float o1 = to_f(base[d]), o2 = to_f(base[d + half]);
    if (apply_rope) {
      const float c = rnd<T>(cr[d]), s = rnd<T>(sr[d]);
      const float x1 = o1, x2 = o2;
      o1 = rnd<T>(rnd<T>(x1 * c) - rnd<T>(x2 * s));
      o2 = rnd<T>(rnd<T>(x2 * c) + rnd<T>(x1 * s));
    }
    if (h < nh) {
      base[d] = from_f<T>(o1);
      base[d + half] = from_f<T>(o2);
    } else if (slot_ok) {
      T* dst = static_cast<T*>(kv.k) + slot_off + static_cast<int64_t>(h - nh) * kv.head_stride;
      dst[d] = from_f<T>(o1);
      dst[d + half] = from_f<T>(o2);
    }
  }
  if (slot_ok) {
    const T* vsrc = row + (nh + nkv) * hd;
    for (int i = threadIdx.x; i < nkv * hd; i += blockDim.x) {
      const int g = i / hd, d = i % hd;
      static_cast<T*>(kv.v)[slot_off + static_cast<int64_t>(g) * kv.head_stride + d] = vsrc[i];
    }
  }
}

// Vectorised bf16 variant for head_dim % 16 == 0: each work item moves 8 elements (16 bytes) of x1 and the
// matching 8 of x2 (rotation) or 8 values of v (copy); same arithmetic and rounding as rope_kv_kernel.
__global__ void __launch_bounds__(128)
    rope_kv_vec_kernel(__nv_bfloat16* __restrict__ qkv, int64_t ld, const float* __restrict__ cos_t,
                       const float* __restrict__ sin_t, int rope_rows, const int64_t* __restrict__ positions,
                       KVCache kv, int T_new, int nh, int nkv, int hd, int64_t slot_base, int slot_from_pos,
                       unsigned* err) {
  pdl_trigger();
  pdl_wait();   // launched with PDL: everything below reads or writes other kernels' data
  using bf = __nv_bfloat16;
  const int64_t tok = blockIdx.x;
  const int r = static_cast<int>(tok / T_new), j = static_cast<int>(tok % T_new);
  const int64_t pos = positions[tok];
  if (pos < 0 || pos >= rope_rows) {
    if (threadIdx.x == 0) flag_error(err, ERR_BAD_POSITION);
    return;
  }
  const int half = hd / 2, cph = half / 8;   // 8-element chunks per half head
  bf* row = qkv + tok * ld;
  const int64_t slot = slot_from_pos ? pos : slot_base + j;
  const int64_t blk_idx = slot / kv.block_size;
  bool slot_ok = slot >= 0 && blk_idx < kv.table_cols;
  const int64_t blk = slot_ok ? kv.table[static_cast<int64_t>(r) * kv.table_stride + blk_idx] : -1;
  slot_ok = slot_ok && blk >= 0 && blk < kv.num_blocks;
  if (!slot_ok && threadIdx.x == 0) flag_error(err, ERR_BAD_SLOT);
  const int64_t slot_off = slot_ok ? blk * kv.block_stride + (slot % kv.block_size) * hd : 0;
  const float* cr = cos_t + pos * half;
  const float* sr = sin_t + pos * half;
  const int rot = (nh + nkv) * cph, vchunks = nkv * hd / 8;
  for (int i = threadIdx.x; i < rot + vchunks; i += blockDim.x) {
    if (i < rot) {
      const int h = i / cph, d0 = (i % cph) * 8;
      bf* base = row + h * hd;
      const uint4 u1 = *reinterpret_cast<const uint4*>(base + d0);
      const uint4 u2 = *reinterpret_cast<const uint4*>(base + half + d0);
      const float4 c0 = *reinterpret_cast<const float4*>(cr + d0), c1 = *reinterpret_cast<const float4*>(cr + d0 + 4);
      const float4 s0 = *reinterpret_cast<const float4*>(sr + d0), s1 = *reinterpret_cast<const float4*>(sr + d0 + 4);
      const float cc[8] = {c0.x, c0.y, c0.z, c0.w, c1.x, c1.y, c1.z, c1.w};
      const float ss[8] = {s0.x, s0.y, s0.z, s0.w, s1.x, s1.y, s1.z, s1.w};
      const bf* e1 = reinterpret_cast<const bf*>(&u1);
      const bf* e2 = reinterpret_cast<const bf*>(&u2);
      uint4 o1, o2;
      bf* f1 = reinterpret_cast<bf*>(&o1);
      bf* f2 = reinterpret_cast<bf*>(&o2);
#pragma unroll
      for (int k = 0; k < 8; ++k) {
        const float c = rnd<bf>(cc[k]), sn = rnd<bf>(ss[k]);
        const float x1 = to_f(e1[k]), x2 = to_f(e2[k]);
        f1[k] = from_f<bf>(rnd<bf>(x1 * c) - rnd<bf>(x2 * sn));
        f2[k] = from_f<bf>(rnd<bf>(x2 * c) + rnd<bf>(x1 * sn));
      }
      if (h < nh) {
        *reinterpret_cast<uint4*>(base + d0) = o1;
        *reinterpret_cast<uint4*>(base + half + d0) = o2;
      } else if (slot_ok) {
        bf* dst = static_cast<bf*>(kv.k) + slot_off + static_cast<int64_t>(h - nh) * kv.head_stride;
        *reinterpret_cast<uint4*>(dst + d0) = o1;
        *reinterpret_cast<uint4*>(dst + half + d0) = o2;
      }
    } else if (slot_ok) {
      const int c = i - rot;
      const int g = (c * 8) / hd, d0 = (c * 8) % hd;
      const uint4 val = *reinterpret_cast<const uint4*>(row + (nh + nkv) * hd + c * 8);
      *reinterpret_cast<uint4*>(static_cast<bf*>(kv.v) + slot_off + static_cast<int64_t>(g) * kv.head_stride + d0) = val;
    }
  }
}

// ------------------------------------------------------------------- KV store from (B, h, T, d) tensors
// The write half of PagedLayerView.update (forgeserve/paged.py:72-78): new k/v of shape (B, nkv, T, hd),
// token (r, j) goes to slot positions[r, j].
template <typename T>
__global__ void kv_store_kernel(const T* __restrict__ k, const T* __restrict__ v, const int64_t* __restrict__ positions,
                                KVCache kv, int T_new, int nkv, int hd, unsigned* err) {
  pdl_trigger();
  pdl_wait();   // launched with PDL: everything below reads or writes other kernels' data
  const int64_t tok = blockIdx.x;
  const int r = static_cast<int>(tok / T_new), j = static_cast<int>(tok % T_new);
  const int64_t slot = positions[tok];
  const int64_t blk_idx = slot / kv.block_size;
  bool ok = slot >= 0 && blk_idx < kv.table_cols;
  const int64_t blk = ok ? kv.table[static_cast<int64_t>(r) * kv.table_stride + blk_idx] : -1;
  ok = ok && blk >= 0 && blk < kv.num_blocks;
  if (!ok) {
    if (threadIdx.x == 0) flag_error(err, ERR_BAD_SLOT);
    return;
  }
  const int64_t off = blk * kv.block_stride + (slot % kv.block_size) * hd;
  for (int i = threadIdx.x; i < nkv * hd; i += blockDim.x) {
    const int g = i / hd, d = i % hd;
    const int64_t src = ((static_cast<int64_t>(r) * nkv + g) * T_new + j) * hd + d;
    static_cast<T*>(kv.k)[off + g * kv.head_stride + d] = k[src];
    static_cast<T*>(kv.v)[off + g * kv.head_stride + d] = v[src];
  }
}

// --------------------------------------------------------------------------------------- paged gather
// Read half of PagedLayerView.update (forgeserve/paged.py:80-81): out[b, g, t*bs + s, :] = pool[table[b, t], g, s, :]
template <typename T>
__global__ void paged_gather_kernel(const T* __restrict__ pool, const int64_t* __restrict__ table, int64_t nb,
                                    int64_t num_blocks, int nkv, int bs, int hd, T* __restrict__ out, unsigned* err) {
  pdl_trigger();
  pdl_wait();   // launched with PDL: everything below reads or writes other kernels' data
  // grid: (B * nb * nkv); each block copies one (row, table entry, head) = bs * hd values
  const int64_t id = blockIdx.x;
  const int g = static_cast<int>(id % nkv);
  const int64_t t = (id / nkv) % nb;
  const int64_t b = id / (nkv * nb);
  const int64_t blk = table[b * nb + t];
  const bool ok = blk >= 0 && blk < num_blocks;
  if (!ok && threadIdx.x == 0) flag_error(err, ERR_BAD_SLOT);
  const T* src = pool + (blk * nkv + g) * static_cast<int64_t>(bs) * hd;
  T* dst = out + ((b * nkv + g) * nb + t) * static_cast<int64_t>(bs) * hd;
  for (int i = threadIdx.x; i < bs * hd; i += blockDim.x) dst[i] = ok ? src[i] : from_f<T>(0.f);
}

// ------------------------------------------------------------------------------------------ embedding
// out[i, :] = table[ids[i], :]   (nn.Embedding; forgeserve/pipeline.py:106, model.py:134-135)
template <typename T>
__global__ void embed_kernel(const int64_t* __restrict__ ids, const T* __restrict__ table, int64_t vocab, int dim,
                             T* __restrict__ out, unsigned* err) {
  pdl_trigger();
  pdl_wait();   // launched with PDL: everything below reads or writes other kernels' data
  const int64_t i = blockIdx.x;
  const int64_t id = ids[i];
  T* dst = out + i * dim;
  if (id < 0 || id >= vocab) {
    if (threadIdx.x == 0) flag_error(err, ERR_BAD_TOKEN);
    for (int c = threadIdx.x; c < dim; c += blockDim.x) dst[c] = from_f<T>(0.f);
    return;
  }
  const T* src = table + id * dim;
  constexpr int VEC = 16 / sizeof(T);
  if (dim % VEC == 0 && (reinterpret_cast<uintptr_t>(src) & 15) == 0 && (reinterpret_cast<uintptr_t>(dst) & 15) == 0) {
    for (int c = threadIdx.x * VEC; c < dim; c += blockDim.x * VEC)
      *reinterpret_cast<uint4*>(dst + c) = *reinterpret_cast<const uint4*>(src + c);
  } else {
    for (int c = threadIdx.x; c < dim; c += blockDim.x) dst[c] = src[c];
  }
}

// --------------------------------------------------------------------------------------------- argmax
// Greedy sampling (forgeserve/sampling.py:18-19): index of the first maximum; NaN counts as the maximum,
// as in torch.argmax.
__device__ __forceinline__ bool better(float a, int64_t ia, float b, int64_t ib) {
  const bool na = a != a, nb = b != b;
  if (na != nb) return na;
  if (!na && a != b) return a > b;
  return ia < ib;
}

template <typename T>
__global__ void argmax_kernel(const T* __restrict__ x, int64_t row_stride, int64_t n, int64_t* __restrict__ out) {
  pdl_trigger();
  pdl_wait();   // launched with PDL: everything below reads or writes other kernels' data
  const T* xr = x + static_cast<int64_t>(blockIdx.x) * row_stride;
  float best = -INFINITY;
  int64_t bi = INT64_MAX;
  for (int64_t i = threadIdx.x; i < n; i += blockDim.x) {
    const float v = to_f(xr[i]);
    if (bi == INT64_MAX || better(v, i, best, bi)) best = v, bi = i;
  }
  __shared__ float sv[32];
  __shared__ int64_t si[32];
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float ov = __shfl_xor_sync(0xffffffffu, best, o);
    const int64_t oi = __shfl_xor_sync(0xffffffffu, bi, o);
    if (oi != INT64_MAX && (bi == INT64_MAX || better(ov, oi, best, bi))) best = ov, bi = oi;
  }
  if ((threadIdx.x & 31) == 0) sv[threadIdx.x >> 5] = best, si[threadIdx.x >> 5] = bi;
  __syncthreads();
  if (threadIdx.x < 32) {
    const int nw = blockDim.x / 32;
    best = threadIdx.x < nw ? sv[threadIdx.x] : -INFINITY;
    bi = threadIdx.x < nw ? si[threadIdx.x] : INT64_MAX;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float ov = __shfl_xor_sync(0xffffffffu, best, o);
      const int64_t oi = __shfl_xor_sync(0xffffffffu, bi, o);
      if (oi != INT64_MAX && (bi == INT64_MAX || better(ov, oi, best, bi))) best = ov, bi = oi;
    }
    if (threadIdx.x == 0) out[blockIdx.x] = bi == INT64_MAX ? 0 : bi;
  }
}

// bf16 rows of dim = 256 * VPL: one warp per row (8 rows per CTA, or 1 for a few rows, so that a decode step's 64
// rows spread over 64 SMs; the per-row arithmetic is the same either way), lanes reading consecutive 16-byte vectors.
// Pass 1 accumulates the sum of squares (a shuffle reduction, no block barrier); pass 2 reads the row again (now
// in L1/L2) with w and writes y. Few registers, so every warp slot of an SM can hold a row in flight. Same
// rounding points as rmsnorm_kernel.
template <int VPL>
__global__ void __launch_bounds__(256)
    rmsnorm_warp_kernel(const __nv_bfloat16* __restrict__ x, int64_t xs, const __nv_bfloat16* __restrict__ w,
                        __nv_bfloat16* __restrict__ y, int64_t ys, int64_t rows, float eps) {
  pdl_trigger();
  pdl_wait();   // launched with PDL: everything below reads or writes other kernels' data
  using bf = __nv_bfloat16;
  const int64_t row = static_cast<int64_t>(blockIdx.x) * (blockDim.x >> 5) + (threadIdx.x >> 5);
  if (row >= rows) return;
  const int lane = threadIdx.x & 31;
  const uint4* xr = reinterpret_cast<const uint4*>(x + row * xs);
  float ss = 0.f;
#pragma unroll 4
  for (int i = 0; i < VPL; ++i) {
    const uint4 u = xr[i * 32 + lane];
    const bf* e = reinterpret_cast<const bf*>(&u);
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const float f = __bfloat162float(e[j]);
      ss = fmaf(f, f, ss);
    }
  }
  ss = warp_sum(ss);
  const float r = rsqrtf(ss / static_cast<float>(VPL * 256) + eps);
  const uint4* wr = reinterpret_cast<const uint4*>(w);
  uint4* yr = reinterpret_cast<uint4*>(y + row * ys);
#pragma unroll 4
  for (int i = 0; i < VPL; ++i) {
    const uint4 u = xr[i * 32 + lane];
    const uint4 wu = wr[i * 32 + lane];
    const bf* e = reinterpret_cast<const bf*>(&u);
    const bf* we = reinterpret_cast<const bf*>(&wu);
    uint4 o;
    bf* oe = reinterpret_cast<bf*>(&o);
#pragma unroll
    for (int j = 0; j < 8; ++j) oe[j] = from_f<bf>(rnd<bf>(__bfloat162float(e[j]) * r) * __bfloat162float(we[j]));
    yr[i * 32 + lane] = o;
  }
}

template <int VPL>
static void launch_rmsnorm_warp(const void* x, int64_t xs, const void* w, void* y, int64_t ys, int64_t rows, float eps,
                                cudaStream_t st) {
  const int per_cta = rows >= 2048 ? 8 : 1;   // rows (warps) per CTA
  launch_pdl_async(rmsnorm_warp_kernel<VPL>, static_cast<unsigned>((rows + per_cta - 1) / per_cta), 32 * per_cta, 0, st,
      static_cast<const __nv_bfloat16*>(x), xs, static_cast<const __nv_bfloat16*>(w), static_cast<__nv_bfloat16*>(y),
      ys, rows, eps);
}

}  // namespace

// ================================================================================================ host

int rmsnorm(int dtype, const void* x, int64_t xs, const void* w, void* y, int64_t ys, int64_t rows, int64_t dim,
            float eps, cudaStream_t st) {
  if (rows <= 0) return 0;
  if (dim <= 0 || dim > (1 << 24)) return fail("rmsnorm: bad dim");
  if (rows > INT32_MAX) return fail("rmsnorm: too many rows");
  constexpr int TH = 256;
  const bool aligned = ((reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(y) |
                         reinterpret_cast<uintptr_t>(w)) & 15) == 0 && xs % 8 == 0 && ys % 8 == 0;
  if (dtype == BF16 && aligned && dim % 256 == 0) {
    switch (dim / 256) {
      case 1: launch_rmsnorm_warp<1>(x, xs, w, y, ys, rows, eps, st); return check_launch("rmsnorm_warp_kernel");
      case 2: launch_rmsnorm_warp<2>(x, xs, w, y, ys, rows, eps, st); return check_launch("rmsnorm_warp_kernel");
      case 4: launch_rmsnorm_warp<4>(x, xs, w, y, ys, rows, eps, st); return check_launch("rmsnorm_warp_kernel");
      case 8: launch_rmsnorm_warp<8>(x, xs, w, y, ys, rows, eps, st); return check_launch("rmsnorm_warp_kernel");
      case 16: launch_rmsnorm_warp<16>(x, xs, w, y, ys, rows, eps, st); return check_launch("rmsnorm_warp_kernel");
      case 32: launch_rmsnorm_warp<32>(x, xs, w, y, ys, rows, eps, st); return check_launch("rmsnorm_warp_kernel");
      default: break;
    }
  }
  if (dtype == F32)
    launch_pdl_async(rmsnorm_kernel<float, TH>, static_cast<unsigned>(rows), TH, 0, st,
        static_cast<const float*>(x), xs, static_cast<const float*>(w), static_cast<float*>(y), ys, static_cast<int>(dim), eps);
  else if (dtype == BF16)
    launch_pdl_async(rmsnorm_kernel<__nv_bfloat16, TH>, static_cast<unsigned>(rows), TH, 0, st,
        static_cast<const __nv_bfloat16*>(x), xs, static_cast<const __nv_bfloat16*>(w), static_cast<__nv_bfloat16*>(y), ys,
        static_cast<int>(dim), eps);
  else
    return fail("rmsnorm: unsupported dtype");
  return check_launch("rmsnorm_kernel");
}

int rope_kv_write(int dtype, void* qkv, int64_t ld, const float* cos_t, const float* sin_t, int64_t rope_rows,
                  const int64_t* positions, const KVCache& kv, int64_t B, int64_t T_new, int64_t nh, int64_t nkv,
                  int64_t hd, int64_t slot_base, int slot_from_pos, int apply_rope, cudaStream_t st) {
  const int64_t tokens = B * T_new;
  if (tokens <= 0) return 0;
  if (hd % 2) return fail("rope: head_dim must be even");
  if (tokens > INT32_MAX) return fail("rope: too many tokens");
  const int th = 128;
  const bool vec = dtype == BF16 && apply_rope && hd % 16 == 0 && ld % 8 == 0 && kv.block_stride % 8 == 0 &&
                   kv.head_stride % 8 == 0 &&
                   ((reinterpret_cast<uintptr_t>(qkv) | reinterpret_cast<uintptr_t>(kv.k) |
                     reinterpret_cast<uintptr_t>(kv.v)) & 15) == 0;
  if (vec) {
    launch_pdl_async(rope_kv_vec_kernel, static_cast<unsigned>(tokens), 128, 0, st,
        static_cast<__nv_bfloat16*>(qkv), ld, cos_t, sin_t, static_cast<int>(rope_rows), positions, kv,
        static_cast<int>(T_new), static_cast<int>(nh), static_cast<int>(nkv), static_cast<int>(hd), slot_base,
        slot_from_pos, error_word());
    return check_launch("rope_kv_vec_kernel");
  }
  if (dtype == F32)
    launch_pdl_async(rope_kv_kernel<float>, static_cast<unsigned>(tokens), th, 0, st,
        static_cast<float*>(qkv), ld, cos_t, sin_t, static_cast<int>(rope_rows), positions, kv, static_cast<int>(T_new),
        static_cast<int>(nh), static_cast<int>(nkv), static_cast<int>(hd), slot_base, slot_from_pos, apply_rope, error_word());
  else if (dtype == BF16)
    launch_pdl_async(rope_kv_kernel<__nv_bfloat16>, static_cast<unsigned>(tokens), th, 0, st,
        static_cast<__nv_bfloat16*>(qkv), ld, cos_t, sin_t, static_cast<int>(rope_rows), positions, kv,
        static_cast<int>(T_new), static_cast<int>(nh), static_cast<int>(nkv), static_cast<int>(hd), slot_base,
        slot_from_pos, apply_rope, error_word());
  else
    return fail("rope: unsupported dtype");
  return check_launch("rope_kv_kernel");
}

int kv_store(int dtype, const void* k, const void* v, const int64_t* positions, const KVCache& kv, int64_t B,
             int64_t T_new, int64_t nkv, int64_t hd, cudaStream_t st) {
  const int64_t tokens = B * T_new;
  if (tokens <= 0) return 0;
  if (tokens > INT32_MAX) return fail("kv_store: too many tokens");
  if (dtype == F32)
    launch_pdl_async(kv_store_kernel<float>, static_cast<unsigned>(tokens), 128, 0, st,
        static_cast<const float*>(k), static_cast<const float*>(v), positions, kv, static_cast<int>(T_new),
        static_cast<int>(nkv), static_cast<int>(hd), error_word());
  else if (dtype == BF16)
    launch_pdl_async(kv_store_kernel<__nv_bfloat16>, static_cast<unsigned>(tokens), 128, 0, st,
        static_cast<const __nv_bfloat16*>(k), static_cast<const __nv_bfloat16*>(v), positions, kv,
        static_cast<int>(T_new), static_cast<int>(nkv), static_cast<int>(hd), error_word());
  else
    return fail("kv_store: unsupported dtype");
  return check_launch("kv_store_kernel");
}

int paged_gather(int dtype, const void* pool, const int64_t* table, int64_t B, int64_t nb, int64_t num_blocks,
                 int64_t nkv, int64_t bs, int64_t hd, void* out, cudaStream_t st) {
  const int64_t n = B * nb * nkv;
  if (n <= 0) return 0;
  if (n > INT32_MAX) return fail("paged_gather: too large");
  if (dtype == F32)
    launch_pdl_async(paged_gather_kernel<float>, static_cast<unsigned>(n), 128, 0, st,
        static_cast<const float*>(pool), table, nb, num_blocks, static_cast<int>(nkv), static_cast<int>(bs),
        static_cast<int>(hd), static_cast<float*>(out), error_word());
  else if (dtype == BF16)
    launch_pdl_async(paged_gather_kernel<__nv_bfloat16>, static_cast<unsigned>(n), 128, 0, st,
        static_cast<const __nv_bfloat16*>(pool), table, nb, num_blocks, static_cast<int>(nkv), static_cast<int>(bs),
        static_cast<int>(hd), static_cast<__nv_bfloat16*>(out), error_word());
  else
    return fail("paged_gather: unsupported dtype");
  return check_launch("paged_gather_kernel");
}

int embed(int dtype, const int64_t* ids, int64_t n, const void* table, int64_t vocab, int64_t dim, void* out,
          cudaStream_t st) {
  if (n <= 0) return 0;
  if (n > INT32_MAX) return fail("embed: too many ids");
  if (dtype == F32)
    launch_pdl_async(embed_kernel<float>, static_cast<unsigned>(n), 128, 0, st, ids, static_cast<const float*>(table), vocab,
                                                                   static_cast<int>(dim), static_cast<float*>(out), error_word());
  else if (dtype == BF16)
    launch_pdl_async(embed_kernel<__nv_bfloat16>, static_cast<unsigned>(n), 128, 0, st,
        ids, static_cast<const __nv_bfloat16*>(table), vocab, static_cast<int>(dim), static_cast<__nv_bfloat16*>(out),
        error_word());
  else
    return fail("embed: unsupported dtype");
  return check_launch("embed_kernel");
}

int argmax(int dtype, const void* x, int64_t rows, int64_t n, int64_t row_stride, int64_t* out, cudaStream_t st) {
  if (rows <= 0) return 0;
  if (n <= 0) return fail("argmax: empty rows");
  if (rows > INT32_MAX) return fail("argmax: too many rows");
  if (dtype == F32)
    launch_pdl_async(argmax_kernel<float>, static_cast<unsigned>(rows), 1024, 0, st, static_cast<const float*>(x), row_stride, n, out);
  else if (dtype == BF16)
    launch_pdl_async(argmax_kernel<__nv_bfloat16>, static_cast<unsigned>(rows), 1024, 0, st, static_cast<const __nv_bfloat16*>(x),
                                                                               row_stride, n, out);
  else
    return fail("argmax: unsupported dtype");
  return check_launch("argmax_kernel");
}

}  // namespace fs
