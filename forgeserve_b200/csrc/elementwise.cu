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

// Two fp32 values rounded to bf16 (nearest even) by one packing conversion: lo in bits 0-15, hi in bits 16-31.
__device__ __forceinline__ uint32_t pack2_bf16(float lo, float hi) {
  const __nv_bfloat162 h = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<const uint32_t*>(&h);
}
// a and b rounded to bf16 precision (nearest even) and returned as fp32: the same values as rnd<bf16> of each, with
// one conversion instruction for the two.
__device__ __forceinline__ void rnd2_bf16(float& a, float& b) {
  const uint32_t u = pack2_bf16(a, b);
  a = __uint_as_float(u << 16);
  b = __uint_as_float(u & 0xffff0000u);
}
// The two bf16 values of a packed word as fp32 (exact).
__device__ __forceinline__ float bf16_lo(uint32_t u) { return __uint_as_float(u << 16); }
__device__ __forceinline__ float bf16_hi(uint32_t u) { return __uint_as_float(u & 0xffff0000u); }

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

// Vectorised bf16 variant for head_dim % 16 == 0 with hd / 16 dividing the block size (the host checks both): each
// work item moves 8 elements (16 bytes) of x1 and the matching 8 of x2 (rotation) or 8 values of v (copy); same
// arithmetic and rounding as rope_kv_kernel. Thread t always handles the 8-element chunk t % (hd / 16) of a half
// head, so its cos / sin values are loaded once; the loads of up to four heads and of the token's v chunk are
// issued together, before the position is checked, so that their latencies overlap.
__global__ void __launch_bounds__(128)
    rope_kv_vec_kernel(__nv_bfloat16* __restrict__ qkv, int64_t ld, const float* __restrict__ cos_t,
                       const float* __restrict__ sin_t, int rope_rows, const int64_t* __restrict__ positions,
                       KVCache kv, int T_new, int nh, int nkv, int hd, int64_t slot_base, int slot_from_pos,
                       unsigned* err) {
  pdl_trigger();
  pdl_wait();   // launched with PDL: everything below reads or writes other kernels' data
  using bf = __nv_bfloat16;
  constexpr int G = 4;   // heads per thread whose loads are in flight together
  const int64_t tok = blockIdx.x;
  const int r = static_cast<int>(tok / T_new), j = static_cast<int>(tok % T_new);
  const int64_t pos = positions[tok];
  const int half = hd / 2, cph = half / 8;   // 8-element chunks per half head
  const int d0 = (threadIdx.x % cph) * 8, hstep = blockDim.x / cph, heads = nh + nkv;
  const int vchunks = nkv * hd / 8;
  bf* row = qkv + tok * ld;
  uint4 a[G], b[G];
  auto load_group = [&](int h0) {
#pragma unroll
    for (int k = 0; k < G; ++k) {
      const int h = h0 + k * hstep;
      if (h < heads) {
        a[k] = *reinterpret_cast<const uint4*>(row + h * hd + d0);
        b[k] = *reinterpret_cast<const uint4*>(row + h * hd + half + d0);
      }
    }
  };
  const int h_first = threadIdx.x / cph;
  load_group(h_first);
  uint4 vval = make_uint4(0, 0, 0, 0);
  if (static_cast<int>(threadIdx.x) < vchunks) vval = *reinterpret_cast<const uint4*>(row + heads * hd + threadIdx.x * 8);

  if (pos < 0 || pos >= rope_rows) {
    if (threadIdx.x == 0) flag_error(err, ERR_BAD_POSITION);
    return;
  }
  const int64_t slot = slot_from_pos ? pos : slot_base + j;
  const int64_t blk_idx = slot / kv.block_size;
  bool slot_ok = slot >= 0 && blk_idx < kv.table_cols;
  const int64_t blk = slot_ok ? kv.table[static_cast<int64_t>(r) * kv.table_stride + blk_idx] : -1;
  slot_ok = slot_ok && blk >= 0 && blk < kv.num_blocks;
  if (!slot_ok && threadIdx.x == 0) flag_error(err, ERR_BAD_SLOT);
  const int64_t slot_off = slot_ok ? blk * kv.block_stride + (slot % kv.block_size) * hd : 0;
  float cc[8], ss[8];
  {
    const float4 c0 = *reinterpret_cast<const float4*>(cos_t + pos * half + d0);
    const float4 c1 = *reinterpret_cast<const float4*>(cos_t + pos * half + d0 + 4);
    const float4 s0 = *reinterpret_cast<const float4*>(sin_t + pos * half + d0);
    const float4 s1 = *reinterpret_cast<const float4*>(sin_t + pos * half + d0 + 4);
    const float cv[8] = {c0.x, c0.y, c0.z, c0.w, c1.x, c1.y, c1.z, c1.w};
    const float sv[8] = {s0.x, s0.y, s0.z, s0.w, s1.x, s1.y, s1.z, s1.w};
#pragma unroll
    for (int k = 0; k < 8; ++k) cc[k] = rnd<bf>(cv[k]), ss[k] = rnd<bf>(sv[k]);
  }
  for (int h0 = h_first; h0 < heads; h0 += G * hstep) {
    if (h0 != h_first) load_group(h0);
#pragma unroll
    for (int k = 0; k < G; ++k) {
      const int h = h0 + k * hstep;
      if (h >= heads) break;
      // out1 = T(T(x1 c) - T(x2 s)), out2 = T(T(x2 c) + T(x1 s)); the roundings go two to a conversion
      const uint32_t w1[4] = {a[k].x, a[k].y, a[k].z, a[k].w}, w2[4] = {b[k].x, b[k].y, b[k].z, b[k].w};
      uint32_t r1[4], r2[4];
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        float o1[2], o2[2];
#pragma unroll
        for (int t = 0; t < 2; ++t) {
          const int e = 2 * q + t;
          const float x1 = t ? bf16_hi(w1[q]) : bf16_lo(w1[q]), x2 = t ? bf16_hi(w2[q]) : bf16_lo(w2[q]);
          float p1 = x1 * cc[e], p2 = x2 * ss[e], p3 = x2 * cc[e], p4 = x1 * ss[e];
          rnd2_bf16(p1, p2);
          rnd2_bf16(p3, p4);
          o1[t] = p1 - p2;
          o2[t] = p3 + p4;
        }
        r1[q] = pack2_bf16(o1[0], o1[1]);
        r2[q] = pack2_bf16(o2[0], o2[1]);
      }
      const uint4 o1 = make_uint4(r1[0], r1[1], r1[2], r1[3]), o2 = make_uint4(r2[0], r2[1], r2[2], r2[3]);
      if (h < nh) {
        *reinterpret_cast<uint4*>(row + h * hd + d0) = o1;
        *reinterpret_cast<uint4*>(row + h * hd + half + d0) = o2;
      } else if (slot_ok) {
        bf* dst = static_cast<bf*>(kv.k) + slot_off + static_cast<int64_t>(h - nh) * kv.head_stride;
        *reinterpret_cast<uint4*>(dst + d0) = o1;
        *reinterpret_cast<uint4*>(dst + half + d0) = o2;
      }
    }
  }
  if (slot_ok) {
    for (int c = threadIdx.x; c < vchunks; c += blockDim.x) {
      const uint4 val = c == static_cast<int>(threadIdx.x) ? vval
                                                           : *reinterpret_cast<const uint4*>(row + heads * hd + c * 8);
      const int g = (c * 8) / hd, dv = (c * 8) % hd;
      *reinterpret_cast<uint4*>(static_cast<bf*>(kv.v) + slot_off + static_cast<int64_t>(g) * kv.head_stride + dv) =
          val;
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
// Up to 4096 columns the row stays in registers: all of it is requested at once, the sum of squares is taken (a
// shuffle reduction, no block barrier), and y is written from the registers, so x is read from memory once. Wider
// rows take two passes (the second from cache). Three CTAs per SM (24 rows in flight; 80 registers, a few bytes
// spilled at 4096 columns) measured 30.8 us against 36.9 us at two CTAs per SM (86 registers) on 8192 x 4096.
// Same rounding points as rmsnorm_kernel.
template <int VPL>
__global__ void __launch_bounds__(256, 3)
    rmsnorm_warp_kernel(const __nv_bfloat16* __restrict__ x, int64_t xs, const __nv_bfloat16* __restrict__ w,
                        __nv_bfloat16* __restrict__ y, int64_t ys, int64_t rows, float eps) {
  pdl_trigger();
  pdl_wait();   // launched with PDL: everything below reads or writes other kernels' data
  using bf = __nv_bfloat16;
  const int64_t row = static_cast<int64_t>(blockIdx.x) * (blockDim.x >> 5) + (threadIdx.x >> 5);
  if (row >= rows) return;
  const int lane = threadIdx.x & 31;
  const uint4* xr = reinterpret_cast<const uint4*>(x + row * xs);
  const uint4* wr = reinterpret_cast<const uint4*>(w);
  uint4* yr = reinterpret_cast<uint4*>(y + row * ys);
  auto scale_store = [&](int i, const uint4& u, float r) {
    const uint4 wu = wr[i * 32 + lane];
    const bf* e = reinterpret_cast<const bf*>(&u);
    const bf* we = reinterpret_cast<const bf*>(&wu);
    uint4 o;
    bf* oe = reinterpret_cast<bf*>(&o);
#pragma unroll
    for (int j = 0; j < 8; ++j) oe[j] = from_f<bf>(rnd<bf>(__bfloat162float(e[j]) * r) * __bfloat162float(we[j]));
    yr[i * 32 + lane] = o;
  };
  float ss = 0.f;
  if constexpr (VPL <= 16) {
    // The row stays in registers (VPL x 16 bytes per lane): x is read from memory once, all of it in flight at once.
    uint4 u[VPL];
#pragma unroll
    for (int i = 0; i < VPL; ++i) u[i] = xr[i * 32 + lane];
#pragma unroll
    for (int i = 0; i < VPL; ++i) {
      const uint32_t wv[4] = {u[i].x, u[i].y, u[i].z, u[i].w};
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float lo = bf16_lo(wv[j]), hi = bf16_hi(wv[j]);
        ss = fmaf(lo, lo, ss);
        ss = fmaf(hi, hi, ss);
      }
    }
    ss = warp_sum(ss);
    const float r = rsqrtf(ss / static_cast<float>(VPL * 256) + eps);
#pragma unroll
    for (int i = 0; i < VPL; ++i) scale_store(i, u[i], r);
  } else {
    // Wider rows: two passes over the row (the second from cache).
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
#pragma unroll 4
    for (int i = 0; i < VPL; ++i) scale_store(i, xr[i * 32 + lane], r);
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
  if (hd <= 0 || nh <= 0 || nkv <= 0) return fail("rope: head_dim and the head counts must be positive");
  if (hd % 2) return fail("rope: head_dim must be even");
  if (tokens > INT32_MAX) return fail("rope: too many tokens");
  const int th = 128;
  const bool vec = dtype == BF16 && apply_rope && hd % 16 == 0 && 128 % (hd / 16) == 0 && ld % 8 == 0 &&
                   kv.block_stride % 8 == 0 &&
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
