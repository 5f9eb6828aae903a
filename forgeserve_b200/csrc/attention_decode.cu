// Decode attention (one new query per batch row) over a paged or contiguous KV cache: split-KV "flash decoding".
//
// Same semantics as attention.cu (forgeserve/model.py:69-76): query head h reads KV head h / rep, key slot s is
// visible iff s <= position and s < n_slots, scale 1/sqrt(hd). This is the step the reference's Engine runs for
// every running request (forgeserve/engine.py:125, paged gather at forgeserve/paged.py:80-81). It is HBM-bound:
// every K/V row of the visible context is read once, for all `rep` query heads of its KV head, and the kernels
// are built to keep enough bytes in flight to stream at HBM speed.
//
//   attn_decode_tc_kernel  (bf16, block size a multiple of 16) grid (splits, n_kv, B), 4 warps. A split's keys go
//                          in 16-key tiles (one paged block at block size 16) to the warps in turn; each warp owns
//                          a 3-stage ring of TMA tile loads (128-byte swizzle, K and V of one tile = 8 KB at hd
//                          128) and keeps its own online-softmax state, so the main loop has no block barrier.
//                          Scores S^T = K Q^T and the output O^T = V^T P^T are mma.sync m16n8k16 products with the
//                          <= 8 query heads of the KV head as the N = 8 side (keys / head dims are the M side);
//                          P^T reaches the B-operand layout through movmatrix. The warps' partial results are
//                          merged through shared memory at the end.
//   attn_decode_kernel     CUDA-core fallback (fp32, or layouts the tile loads cannot address): grid as above,
//                          128 threads, 64-key chunks fetched with cp.async into row-padded shared memory.
//   attn_combine_kernel    grid (B, nh): merges the splits (log-sum-exp weights) into the output.
//
// Splits: a split covers a fixed number of key slots (chosen from the batch size, n_slots and the SM count so
// that there are several CTAs per SM), so CTAs carry similar work whatever the spread of context lengths; splits
// past a row's context end at once. Workspace (fp32): O partials [B][nh][splits][hd], then (max, sum) pairs
// [B][nh][splits][2] (natural-log domain).
#include <string>

#include "../../include/forgeserve_b200.h"
#include "common.cuh"
#include "kernels.h"

namespace fs {
namespace decode {

constexpr int THREADS = 128, CHUNK = 64, MAX_REP = 8, MAX_SPLITS = 64, SPLIT_KEYS = 512;

// Key slots per split: SPLIT_KEYS, wider (a multiple of CHUNK) only when n_slots exceeds MAX_SPLITS of them.
// Split s covers slots [s * per, (s + 1) * per); a split at or past a row's last visible key is empty.
__host__ __device__ __forceinline__ int64_t split_keys(int64_t n_slots, int splits) {
  return splits * static_cast<int64_t>(SPLIT_KEYS) >= n_slots
             ? SPLIT_KEYS
             : ((n_slots + splits - 1) / splits + CHUNK - 1) / CHUNK * CHUNK;
}

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
  pdl_trigger();
  pdl_wait();   // launched with PDL: everything below reads or writes other kernels' data
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
  const int64_t per = split_keys(n_slots, splits);
  const int64_t k_begin = static_cast<int64_t>(split) * per;
  const int64_t k_end = k_begin + per < n_vis ? k_begin + per : n_vis;
  if (k_begin >= n_vis) return;   // empty split: nothing to write (the combine does not read it)

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
        if (m_s[h] != -INFINITY) ws[slot * HD + d] = acc[h];   // an empty split is skipped by the combine
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
    attn_combine_kernel(const float* __restrict__ ws, int B, int nh, int splits, const int64_t* __restrict__ positions,
                        int64_t n_slots, T* __restrict__ out, int64_t ldo) {
  pdl_trigger();
  pdl_wait();   // launched with PDL: everything below reads or writes other kernels' data
  const int r = blockIdx.x, h = blockIdx.y, d = threadIdx.x;
  const int64_t base = (static_cast<int64_t>(r) * nh + h) * splits;
  const float* ml = ws + static_cast<int64_t>(B) * nh * splits * HD;
  int64_t pos = positions[r];
  if (pos < 0) pos = 0;
  const int64_t n_vis = pos + 1 < n_slots ? pos + 1 : n_slots;
  const int64_t per = split_keys(n_slots, splits);
  const int used = static_cast<int>((n_vis + per - 1) / per < splits ? (n_vis + per - 1) / per : splits);
  float M = -INFINITY;
  for (int s = 0; s < used; ++s) M = fmaxf(M, ml[2 * (base + s)]);
  float L = 0.f, o = 0.f;
  for (int s = 0; s < used; ++s) {
    const float m = ml[2 * (base + s)];
    if (m == -INFINITY) continue;   // no visible key in this split (its O partial is not written)
    const float w = expf(m - M);
    L += w * ml[2 * (base + s) + 1];
    if (d < HD) o += w * ws[(base + s) * HD + d];
  }
  if (d < HD) out[static_cast<int64_t>(r) * ldo + static_cast<int64_t>(h) * HD + d] = from_f<T>(L > 0.f ? o / L : 0.f);
}

// ------------------------------------------------------------------------------ tensor-core tile kernel
namespace tcd {

constexpr int TILE = 16, WARPS = 4, THREADS_TC = 32 * WARPS, STAGES = 3, BOX_BYTES = TILE * 128;

template <int HD>
struct Geo {
  static constexpr int NB = HD / 64;                       // 128-byte column boxes per K (or V) row
  static constexpr int KV_BYTES = NB * BOX_BYTES;          // K (or V) of one 16-key tile
  static constexpr int STAGE_BYTES = 2 * KV_BYTES;
  static constexpr int RING_BYTES = WARPS * STAGES * STAGE_BYTES;
  static constexpr int BAR_OFF = RING_BYTES;
  static constexpr int STAT_OFF = BAR_OFF + WARPS * STAGES * 8;   // m and l: [WARPS][8] floats each
  static constexpr int SMEM = STAT_OFF + 2 * WARPS * 8 * 4 + 1024;  // + slack for the 1024-byte alignment
  static_assert(WARPS * 8 * HD * 4 <= RING_BYTES, "the warp-merge area must fit in the rings");
};

struct Params {
  const __nv_bfloat16* q;
  int64_t ldq;
  const int64_t* table;
  int64_t table_stride, table_cols, block_size, rows_per_block, rows_per_head, num_blocks, kv_rows;
  int64_t n_slots;
  const int64_t* positions;
  __nv_bfloat16* out;
  int64_t ldo;
  int nh, rep, splits, per;
  float scale_log2;
  float* ws;
  unsigned* err;
};

__device__ __forceinline__ void ldsm_x4(uint32_t (&r)[4], uint32_t addr) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(addr));
}
__device__ __forceinline__ void ldsm_x4_trans(uint32_t (&r)[4], uint32_t addr) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(addr));
}
// c (16 x 8, fp32) += a (16 x 16, bf16, row-major) * b (16 x 8, bf16, column-major)
__device__ __forceinline__ void mma16816(float (&c)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}
__device__ __forceinline__ uint32_t movmatrix_trans(uint32_t x) {
  uint32_t y;
  asm volatile("movmatrix.sync.aligned.m8n8.trans.b16 %0, %1;" : "=r"(y) : "r"(x));
  return y;
}
__device__ __forceinline__ uint32_t pack_bf16(float lo, float hi) {
  uint32_t d;
  asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(d) : "f"(hi), "f"(lo));
  return d;
}
__device__ __forceinline__ void st_shared_zero16(uint32_t addr) {
  asm volatile("st.shared.v4.u32 [%0], {%1, %1, %1, %1};" ::"r"(addr), "r"(0u) : "memory");
}
// Orders this thread's earlier shared-memory accesses before later async-proxy (TMA) writes to the same bytes.
__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// Byte address of 16-byte chunk `chunk` (8 bf16 of the row) of tile row `row` in a 128-byte-swizzled box pair.
__device__ __forceinline__ uint32_t tile_addr(uint32_t base, int row, int chunk) {
  return base + static_cast<uint32_t>((chunk >> 3) * BOX_BYTES + row * 128 + (((chunk & 7) ^ (row & 7)) << 4));
}

template <int HD>
__global__ void __launch_bounds__(THREADS_TC)
    attn_decode_tc_kernel(const __grid_constant__ CUtensorMap tmK, const __grid_constant__ CUtensorMap tmV, Params p) {
  pdl_trigger();
  pdl_wait();   // launched with PDL: everything below reads or writes other kernels' data
  using G = Geo<HD>;
  extern __shared__ uint8_t smem_raw[];
  __shared__ int abort_flag;
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + G::BAR_OFF);
  float* sm_m = reinterpret_cast<float*>(smem + G::STAT_OFF);
  float* sm_l = sm_m + WARPS * 8;

  const int split = blockIdx.x, g = blockIdx.y, r = blockIdx.z;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  int64_t pos = p.positions[r];
  if (pos < 0) pos = 0;
  const int64_t n_vis = pos + 1 < p.n_slots ? pos + 1 : p.n_slots;
  const int64_t k_begin = static_cast<int64_t>(split) * p.per;
  const int64_t k_end = k_begin + p.per < n_vis ? k_begin + p.per : n_vis;
  if (k_begin >= n_vis) return;   // empty split: the whole CTA leaves before any set-up (the combine skips it)
  const int n_tiles = static_cast<int>((k_end - k_begin + TILE - 1) / TILE);
  const int my_n = n_tiles > warp ? (n_tiles - warp + WARPS - 1) / WARPS : 0;   // tiles warp, warp+4, ...

  if (threadIdx.x == 0) {
    for (int i = 0; i < WARPS * STAGES; ++i) mbar_init(&full[i], 1);
    abort_flag = 0;
    fence_barrier_init();
    prefetch_tmap(&tmK);
    prefetch_tmap(&tmV);
  }
  __syncthreads();

  uint8_t* ring = smem + warp * STAGES * G::STAGE_BYTES;
  uint64_t* wfull = full + warp * STAGES;
  // Every cached key and value is read once per step: evict-first in L2, so that the split partials written
  // meanwhile are still there for the combine.
  const uint64_t kv_policy = l2_policy_evict_first();
  // Cache block of the warp's j-th tile (keys k0 .. k0+15, all in one block); -1 past the table.
  auto tile_block = [&](int j) -> int64_t {
    const int64_t k0 = k_begin + static_cast<int64_t>(warp + WARPS * j) * TILE;
    const int64_t bi = k0 / p.block_size;
    return bi < p.table_cols ? p.table[static_cast<int64_t>(r) * p.table_stride + bi] : -1;
  };
  // Lane l holds the block of tile base + l of this warp, loaded 32 tiles at a time by the whole warp, so that a
  // TMA issue does not wait on a table load of its own.
  int64_t lane_blk = lane < my_n ? tile_block(lane) : -1;
  // Lane 0 of the warp fetches the warp's j-th tile (block blk) into stage j % STAGES.
  auto issue = [&](int j, int64_t blk) {
    const int64_t k0 = k_begin + static_cast<int64_t>(warp + WARPS * j) * TILE;
    int64_t row;
    if (blk < 0 || blk >= p.num_blocks) {
      flag_error(p.err, ERR_BAD_SLOT);
      row = p.kv_rows;   // a box wholly outside the tensor: TMA fills it with zeros
    } else {
      row = blk * p.rows_per_block + static_cast<int64_t>(g) * p.rows_per_head + k0 % p.block_size;
    }
    uint8_t* st = ring + (j % STAGES) * G::STAGE_BYTES;
    uint64_t* bar = &wfull[j % STAGES];
    mbar_arrive_expect_tx(bar, G::STAGE_BYTES);
#pragma unroll
    for (int b = 0; b < G::NB; ++b) {
      tma_load_2d_hint(st + b * BOX_BYTES, &tmK, bar, 64 * b, static_cast<int>(row), kv_policy);
      tma_load_2d_hint(st + G::KV_BYTES + b * BOX_BYTES, &tmV, bar, 64 * b, static_cast<int>(row), kv_policy);
    }
  };

  // Q^T as the B operand: head lane/4, dims 16 ks + 2 (lane % 4) + {0, 1} (and + 8); heads >= rep are zero.
  uint32_t qf[HD / 16][2];
  {
    const int hq = lane >> 2;
    const bool ok = hq < p.rep;
    const __nv_bfloat16* qrow = p.q + static_cast<int64_t>(r) * p.ldq +
                                static_cast<int64_t>(g * p.rep + (ok ? hq : 0)) * HD + 2 * (lane & 3);
#pragma unroll
    for (int ks = 0; ks < HD / 16; ++ks) {
      qf[ks][0] = ok ? *reinterpret_cast<const uint32_t*>(qrow + ks * 16) : 0u;
      qf[ks][1] = ok ? *reinterpret_cast<const uint32_t*>(qrow + ks * 16 + 8) : 0u;
    }
  }
  // This lane's score / output columns are heads h0 = 2 (lane % 4) and h0 + 1 (log2-domain softmax state).
  float m0 = -INFINITY, m1 = -INFINITY, l0 = 0.f, l1 = 0.f;
  float acc[HD / 16][4];
#pragma unroll
  for (int mt = 0; mt < HD / 16; ++mt) acc[mt][0] = acc[mt][1] = acc[mt][2] = acc[mt][3] = 0.f;

  for (int j = 0; j < STAGES; ++j) {
    const int64_t b = __shfl_sync(0xffffffffu, lane_blk, j);
    if (lane == 0 && j < my_n) issue(j, b);
  }
  int j = 0;
  bool timed_out = false;
  for (; j < my_n; ++j) {
    const int s = j % STAGES;
    const bool ok = mbar_wait(&wfull[s], static_cast<uint32_t>((j / STAGES) & 1), p.err);
    if (!__all_sync(0xffffffffu, ok)) {
      timed_out = true;
      break;
    }
    const uint32_t kb = smem_u32(ring + s * G::STAGE_BYTES), vb = kb + G::KV_BYTES;
    const int64_t k0 = k_begin + static_cast<int64_t>(warp + WARPS * j) * TILE;
    const int n = static_cast<int>(k_end - k0 < TILE ? k_end - k0 : TILE);   // >= 1 visible key

    // S^T (16 keys x 8 heads) = K (16 x HD) Q^T (HD x 8)
    float c[4] = {0.f, 0.f, 0.f, 0.f};
    {
      const int mi = lane >> 3, key = ((mi & 1) << 3) | (lane & 7);
#pragma unroll
      for (int ks = 0; ks < HD / 16; ++ks) {
        uint32_t a[4];
        ldsm_x4(a, tile_addr(kb, key, ks * 2 + (mi >> 1)));
        mma16816(c, a, qf[ks][0], qf[ks][1]);
      }
    }
    const int kA = lane >> 2, kB = kA + 8;   // keys of c[0..1] and c[2..3]
    const float s0 = kA < n ? c[0] * p.scale_log2 : -INFINITY, s1 = kA < n ? c[1] * p.scale_log2 : -INFINITY;
    const float s2 = kB < n ? c[2] * p.scale_log2 : -INFINITY, s3 = kB < n ? c[3] * p.scale_log2 : -INFINITY;
    float t0 = fmaxf(s0, s2), t1 = fmaxf(s1, s3);
#pragma unroll
    for (int o = 4; o < 32; o <<= 1) {
      t0 = fmaxf(t0, __shfl_xor_sync(0xffffffffu, t0, o));
      t1 = fmaxf(t1, __shfl_xor_sync(0xffffffffu, t1, o));
    }
    const float mn0 = fmaxf(m0, t0), mn1 = fmaxf(m1, t1);           // finite: the tile has a visible key
    const float cr0 = exp2f(m0 - mn0), cr1 = exp2f(m1 - mn1);         // 0 on the warp's first tile
    const float p0 = exp2f(s0 - mn0), p1 = exp2f(s1 - mn1), p2 = exp2f(s2 - mn0), p3 = exp2f(s3 - mn1);
    l0 = l0 * cr0 + p0 + p2;   // per-lane partial sums; the lanes of one head are added up at the end
    l1 = l1 * cr1 + p1 + p3;
    m0 = mn0;
    m1 = mn1;
#pragma unroll
    for (int mt = 0; mt < HD / 16; ++mt) {
      acc[mt][0] *= cr0;
      acc[mt][1] *= cr1;
      acc[mt][2] *= cr0;
      acc[mt][3] *= cr1;
    }
    // P^T (16 keys x 8 heads) as the B operand: transpose the two 8 x 8 halves of P held in C layout
    const uint32_t pb0 = movmatrix_trans(pack_bf16(p0, p1)), pb1 = movmatrix_trans(pack_bf16(p2, p3));
    if (n < TILE) {   // V rows past the last key hold stale cache contents (possibly non-finite): zero them
      for (int i = lane; i < (TILE - n) * G::NB * 8; i += 32) {
        const int row = n + i / (G::NB * 8), rest = i % (G::NB * 8);
        st_shared_zero16(vb + static_cast<uint32_t>((rest >> 3) * BOX_BYTES + row * 128 + (rest & 7) * 16));
      }
      __syncwarp();
    }
    // O^T (HD x 8 heads) += V^T (HD x 16 keys) P^T (16 keys x 8 heads)
    {
      const int mi = lane >> 3, key = ((mi >> 1) << 3) | (lane & 7);
#pragma unroll
      for (int mt = 0; mt < HD / 16; ++mt) {
        uint32_t a[4];
        ldsm_x4_trans(a, tile_addr(vb, key, mt * 2 + (mi & 1)));
        mma16816(acc[mt], a, pb0, pb1);
      }
    }
    __syncwarp();   // every lane's reads of this stage are done before it is refilled
    {
      const int jn = j + STAGES;   // the tile that goes into the stage just freed
      if ((jn & 31) == 0 && jn < my_n) lane_blk = jn + lane < my_n ? tile_block(jn + lane) : -1;   // next 32
      const int64_t b = __shfl_sync(0xffffffffu, lane_blk, jn & 31);
      if (lane == 0 && jn < my_n) {
        fence_proxy_async_smem();
        issue(jn, b);
      }
    }
  }
  if (timed_out) {   // let the copies still in flight land (bounded) before the CTA gives its shared memory back
    const int issued = my_n < j + STAGES ? my_n : j + STAGES;
    for (int t = j; t < issued; ++t) mbar_wait(&wfull[t % STAGES], static_cast<uint32_t>((t / STAGES) & 1), p.err);
    if (lane == 0) abort_flag = 1;
  }
#pragma unroll
  for (int o = 4; o < 32; o <<= 1) {
    l0 += __shfl_xor_sync(0xffffffffu, l0, o);
    l1 += __shfl_xor_sync(0xffffffffu, l1, o);
  }
  __syncthreads();   // all warps are done with their rings: reuse them for the merge
  if (abort_flag) return;
  float* osm = reinterpret_cast<float*>(smem);   // [WARPS][8 heads][HD]
  const int h0 = 2 * (lane & 3);
  if (lane < 4) {
    sm_m[warp * 8 + h0] = m0;
    sm_m[warp * 8 + h0 + 1] = m1;
    sm_l[warp * 8 + h0] = l0;
    sm_l[warp * 8 + h0 + 1] = l1;
  }
#pragma unroll
  for (int mt = 0; mt < HD / 16; ++mt) {
    const int d = mt * 16 + (lane >> 2);
    float* o0 = osm + (warp * 8 + h0) * HD;
    o0[d] = acc[mt][0];
    o0[HD + d] = acc[mt][1];
    o0[d + 8] = acc[mt][2];
    o0[HD + d + 8] = acc[mt][3];
  }
  __syncthreads();
  for (int i = threadIdx.x; i < p.rep * HD; i += THREADS_TC) {
    const int h = i / HD, d = i % HD;
    float M = -INFINITY;
#pragma unroll
    for (int w = 0; w < WARPS; ++w) M = fmaxf(M, sm_m[w * 8 + h]);
    float L = 0.f, o = 0.f;
#pragma unroll
    for (int w = 0; w < WARPS; ++w) {
      const float mw = sm_m[w * 8 + h];
      const float f = mw == -INFINITY ? 0.f : exp2f(mw - M);
      L += f * sm_l[w * 8 + h];
      o += f * osm[(w * 8 + h) * HD + d];
    }
    const int hh = g * p.rep + h;
    if (p.splits == 1) {
      p.out[static_cast<int64_t>(r) * p.ldo + static_cast<int64_t>(hh) * HD + d] =
          __float2bfloat16_rn(L > 0.f ? o / L : 0.f);
    } else {
      const int64_t slot = (static_cast<int64_t>(r) * p.nh + hh) * p.splits + split;
      if (M != -INFINITY) p.ws[slot * HD + d] = o;   // an empty split is skipped by the combine
      if (d == 0) {
        float* ml = p.ws + static_cast<int64_t>(gridDim.z) * p.nh * p.splits * HD;
        ml[2 * slot] = M == -INFINITY ? -INFINITY : M * 0.6931471805599453f;   // log2 -> natural-log domain
        ml[2 * slot + 1] = L;
      }
    }
  }
}

// The tile loads address the cache as one 2-D tensor of hd-wide rows (row = block * rows_per_block +
// kv_head * rows_per_head + slot) in 16-row boxes, so a 16-key tile must sit inside one block.
bool supported(const KVCache& kv, int64_t hd) {
  if (kv.block_size % TILE != 0) return false;
  if (kv.block_stride % hd != 0 || kv.head_stride % hd != 0 || kv.head_stride / hd < kv.block_size) return false;
  const int64_t rows = kv.num_blocks * (kv.block_stride / hd);
  return rows < (int64_t(1) << 31) - 2 * TILE;
}

template <int HD>
int launch_t(const void* q, int64_t ldq, const KVCache& kv, int64_t n_slots, const int64_t* positions, void* out,
             int64_t ldo, int64_t B, int64_t nh, int64_t nkv, float scale, int splits, float* ws, unsigned* err,
             cudaStream_t st) {
  using G = Geo<HD>;
  const int64_t kv_rows = kv.num_blocks * (kv.block_stride / HD);
  CUtensorMap mk, mv;
  if (make_bf16_map(&mk, kv.k, HD, kv_rows, HD, TILE) || make_bf16_map(&mv, kv.v, HD, kv_rows, HD, TILE)) return -1;
  Params p;
  p.q = static_cast<const __nv_bfloat16*>(q);
  p.ldq = ldq;
  p.table = kv.table;
  p.table_stride = kv.table_stride;
  p.table_cols = kv.table_cols;
  p.block_size = kv.block_size;
  p.rows_per_block = kv.block_stride / HD;
  p.rows_per_head = kv.head_stride / HD;
  p.num_blocks = kv.num_blocks;
  p.kv_rows = kv_rows;
  p.n_slots = n_slots;
  p.positions = positions;
  p.out = static_cast<__nv_bfloat16*>(out);
  p.ldo = ldo;
  p.nh = static_cast<int>(nh);
  p.rep = static_cast<int>(nh / nkv);
  p.splits = splits;
  p.per = static_cast<int>(split_keys(n_slots, splits));
  p.scale_log2 = scale * 1.4426950408889634f;
  p.ws = ws;
  p.err = err;
  static bool attr[64] = {false};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev >= 0 && dev < 64 && !attr[dev]) {
    if (cudaFuncSetAttribute(attn_decode_tc_kernel<HD>, cudaFuncAttributeMaxDynamicSharedMemorySize, G::SMEM) !=
        cudaSuccess)
      return check_launch("attn_decode_tc set smem");
    attr[dev] = true;
  }
  dim3 grid(static_cast<unsigned>(splits), static_cast<unsigned>(nkv), static_cast<unsigned>(B));
  launch_pdl_async(attn_decode_tc_kernel<HD>, grid, THREADS_TC, G::SMEM, st, mk, mv, p);
  return check_launch("attn_decode_tc_kernel");
}

}  // namespace tcd

template <typename T, int HD>
int launch_t(const void* q, int64_t ldq, const KVCache& kv, int64_t n_slots, const int64_t* positions, void* out,
             int64_t ldo, int64_t B, int64_t nh, int64_t nkv, float scale, int splits, float* ws, unsigned* err,
             cudaStream_t st) {
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
  dim3 grid(static_cast<unsigned>(splits), static_cast<unsigned>(nkv), static_cast<unsigned>(B));
  launch_pdl_async(attn_decode_kernel<T, HD>, grid, THREADS, S::BYTES, st,
      static_cast<const T*>(q), ldq, kv, n_slots, positions, static_cast<T*>(out), ldo, static_cast<int>(nh),
      static_cast<int>(nh / nkv), splits, scale, ws, err);
  return check_launch("attn_decode_kernel");
}

template <typename T, int HD>
int combine_t(float* ws, int64_t B, int64_t nh, int splits, const int64_t* positions, int64_t n_slots, void* out,
              int64_t ldo, cudaStream_t st) {
  launch_pdl_async(attn_combine_kernel<T, HD>, dim3(static_cast<unsigned>(B), static_cast<unsigned>(nh)), THREADS, 0, st,
      ws, static_cast<int>(B), static_cast<int>(nh), splits, positions, n_slots, static_cast<T*>(out), ldo);
  return check_launch("attn_combine_kernel");
}

int choose_splits(int64_t B, int64_t nkv, int64_t n_slots, int sms) {
  // A split covers a fixed number of key slots (SPLIT_KEYS), more only past MAX_SPLITS: the partition of a row's
  // keys, and so the order of the sums, is the same whatever the batch size and the width of the block table
  // (splits past a row's context end at once and add exact zeros), so a step gives the same result in a CUDA
  // graph (tables padded to the longest possible row), eagerly, or split into micro-batches.
  (void)B;
  (void)nkv;
  (void)sms;
  int64_t s = (n_slots + SPLIT_KEYS - 1) / SPLIT_KEYS;
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
           unsigned* err, cudaStream_t st) {
  if (B > 65535 || nkv > 65535) return fail("attention_decode: grid too large");
  if (splits > 1 && !ws) return fail("attention_decode: a workspace is needed for more than one split");
  if (hd != 64 && hd != 128) return fail("attention_decode: head_dim must be 64 or 128");
  int rc;
  if (dtype == BF16 && tcd::supported(kv, hd)) {
    rc = hd == 128 ? tcd::launch_t<128>(q, ldq, kv, n_slots, positions, out, ldo, B, nh, nkv, scale, splits, ws, err, st)
                   : tcd::launch_t<64>(q, ldq, kv, n_slots, positions, out, ldo, B, nh, nkv, scale, splits, ws, err, st);
  } else if (dtype == BF16) {
    rc = hd == 128
             ? launch_t<__nv_bfloat16, 128>(q, ldq, kv, n_slots, positions, out, ldo, B, nh, nkv, scale, splits, ws, err, st)
             : launch_t<__nv_bfloat16, 64>(q, ldq, kv, n_slots, positions, out, ldo, B, nh, nkv, scale, splits, ws, err, st);
  } else if (dtype == F32) {
    rc = hd == 128 ? launch_t<float, 128>(q, ldq, kv, n_slots, positions, out, ldo, B, nh, nkv, scale, splits, ws, err, st)
                   : launch_t<float, 64>(q, ldq, kv, n_slots, positions, out, ldo, B, nh, nkv, scale, splits, ws, err, st);
  } else {
    return fail("attention_decode: dtype must be fp32 or bf16");
  }
  if (rc || splits == 1) return rc;
  if (dtype == BF16)
    return hd == 128 ? combine_t<__nv_bfloat16, 128>(ws, B, nh, splits, positions, n_slots, out, ldo, st)
                     : combine_t<__nv_bfloat16, 64>(ws, B, nh, splits, positions, n_slots, out, ldo, st);
  return hd == 128 ? combine_t<float, 128>(ws, B, nh, splits, positions, n_slots, out, ldo, st)
                   : combine_t<float, 64>(ws, B, nh, splits, positions, n_slots, out, ldo, st);
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
// loads this module holds until the process exits.
//
// * Set-up and loading: the first call on a device resolves the array's device address (and that of a device
//   error word beside it) with cudaGetSymbolAddress, with that device current, and launches the kernels for the
//   first time. Under CUDA's lazy module loading (the default since CUDA 12) that first call is also what loads
//   this module onto the device, which reserves the 4 MiB array and the kernels' code. So make one real call at
//   start-up, before a host pool takes the device's free memory and before any stream capture on that device;
//   after it, calls need no further device memory.
// * Limit: calls whose split partials need more than kStaticScratchBytes are refused with an error naming the
//   size (fs_attention_decode_workspace() gives the size a call needs: B * n_heads * splits * (head_dim + 2) * 4
//   bytes). Example: at 32 query heads of head_dim 128, 64 rows fit up to 1536 cache slots (3 splits of 512).
// * Sharing: every call uses the same array and leaves its contents behind; each call writes every partial it
//   reads, so nothing needs clearing, but calls that overlap on the GPU (different streams, no ordering) race on
//   the array and must not be issued.
// * Errors: bad block-table entries and waits that run out of time are recorded in the file-scope word
//   g_static_error (never in allocated memory); fs_device_error() reports and clears it together with the
//   library's allocated error word.
// * It allocates nothing: no cudaMalloc, cudaFree or allocating library routine.
// =============================================================================================================
namespace fs {
namespace decode {

constexpr int64_t kStaticScratchBytes = int64_t(4) << 20;
static __device__ __align__(256) unsigned char g_static_scratch[kStaticScratchBytes];
static __device__ unsigned g_static_error;

struct StaticScratch {
  float* ptr = nullptr;
  unsigned* err = nullptr;
  bool ready = false;
};
static StaticScratch g_static_per_dev[64];

static int static_scratch(float** out, unsigned** err) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return fail("no current CUDA device");
  StaticScratch& s = g_static_per_dev[dev];
  if (!s.ready) {
    void* p = nullptr;
    void* e_word = nullptr;
    cudaError_t e = cudaGetSymbolAddress(&p, g_static_scratch);
    if (e != cudaSuccess) return fail(std::string("cudaGetSymbolAddress(decode scratch): ") + cudaGetErrorString(e));
    e = cudaGetSymbolAddress(&e_word, g_static_error);
    if (e != cudaSuccess) return fail(std::string("cudaGetSymbolAddress(decode error word): ") + cudaGetErrorString(e));
    s.ptr = static_cast<float*>(p);
    s.err = static_cast<unsigned*>(e_word);
    s.ready = true;
  }
  *out = s.ptr;
  *err = s.err;
  return 0;
}

}  // namespace decode

// Bits of the static entry point's error word on the current device (0 if it never ran there); clears them if
// asked. Called by fs_device_error after a device synchronisation; copies only, no allocation.
int static_decode_error_bits(int clear, unsigned* bits) {
  *bits = 0;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 0;
  const decode::StaticScratch& s = decode::g_static_per_dev[dev];
  if (!s.ready) return 0;
  cudaError_t e = cudaMemcpy(bits, s.err, sizeof(unsigned), cudaMemcpyDeviceToHost);
  if (e != cudaSuccess) return fail(std::string("static decode error word: ") + cudaGetErrorString(e));
  if (clear) {
    e = cudaMemset(s.err, 0, sizeof(unsigned));
    if (e != cudaSuccess) return fail(std::string("static decode error word: ") + cudaGetErrorString(e));
  }
  return 0;
}

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
  const int splits = choose_splits(B, nkv, n_slots, sms);
  const int64_t need = workspace_bytes(B, nh, hd, splits);
  if (need > kStaticScratchBytes)
    return fail("fs_attention_decode_static: this call needs " + std::to_string(need) +
                " bytes of scratch, more than the fixed " + std::to_string(kStaticScratchBytes) +
                " bytes; use fs_attention_decode with a caller-owned workspace");
  float* ws = nullptr;
  unsigned* err = nullptr;
  if (static_scratch(&ws, &err)) return -1;
  return launch(dtype, q, ldq, *kv, n_slots, positions, out, ldo, B, nh, nkv, hd, scale, splits, ws, err,
                static_cast<cudaStream_t>(stream));
}
