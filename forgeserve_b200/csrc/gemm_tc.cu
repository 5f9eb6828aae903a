// Dense bf16 projection GEMM on the 5th-generation tensor cores (tcgen05 + TMEM), sm_100a.
//
//   C[M, n_out] = epilogue( A[M, K] @ B[N, K]^T )          A = activations, B = nn.Linear weight (out, in)
//
// This is the kernel behind every projection of a decoder layer (forgeserve/model.py:64-66 q/k/v,
// :77 o, :93 gate/up/down) and the output head (forgeserve/pipeline.py:112 lm_head). Epilogues fuse
// what follows each projection in the reference module:
//   EPI_STORE     C = bf16(acc)
//   EPI_RESIDUAL  C = bf16(R + bf16(acc))                    Block.forward residual add (model.py:105-106)
//   EPI_SWIGLU    C = bf16(bf16(silu(bf16(g))) * bf16(u))    SwiGLU (model.py:93); B = [W_gate; W_up]
//                 (2 * n_out rows): an output tile of 128 columns j0.. reads gate rows j0.. and up rows n_out+j0..
//
// Design (one CTA per SM, persistent over output tiles):
//   warp 0      TMA producer: A tile 128x64 and two B half-tiles 128x64 per k-block (rows n0.. and n1..:
//               n1 = n0 + 128 for plain tiles, the matching up rows for SwiGLU), 128-byte swizzle, 4-stage ring
//   warp 1      MMA issuer: one thread issues tcgen05.mma (M=128, N=256, K=16) into a TMEM accumulator
//   warp 2      TMEM allocator (2 accumulators x 256 fp32 columns = all 512 columns)
//   warps 4-7   epilogue: tcgen05.ld 32 lanes x 32 columns, fused epilogue, vector stores to global memory
// The two TMEM accumulators let the epilogue of one tile overlap the main loop of the next.
// No TMA multicast is used anywhere (the kernel also runs in multi-GPU jobs).
#include <cstdlib>
#include <map>
#include <mutex>
#include <utility>

#include <cudaTypedefs.h>

#include "common.cuh"
#include "gemm.h"

namespace fs {
namespace tcg {

// A stage of the 1-SM kernel holds KP1 64-wide K panels of A and B (one k-block = 64 * KP1 of K).
#ifndef FS_GEMM_KPANELS
#define FS_GEMM_KPANELS 1
#endif
#ifndef FS_GEMM_STAGES
#define FS_GEMM_STAGES (4 / FS_GEMM_KPANELS)
#endif
constexpr int KP1 = FS_GEMM_KPANELS;
constexpr int BM = 128, BN = 256, BK = 64, STAGES = FS_GEMM_STAGES;
constexpr int A_BYTES = BM * BK * 2;  // 16 KiB
constexpr int B_BYTES = BN * BK * 2;  // 32 KiB (two 128-row halves)
constexpr int BH_BYTES = B_BYTES / 2;
constexpr int STAGE_BYTES = KP1 * (A_BYTES + B_BYTES);
constexpr int NUM_ACC = 2;
constexpr int TMEM_COLS = NUM_ACC * BN;  // 512
constexpr int THREADS = 256;
constexpr int BAR_BYTES = 256;
constexpr int SMEM_BYTES = STAGES * STAGE_BYTES + 1024 + BAR_BYTES;
constexpr int THIN_STAGES = 5;   // stages of the M <= 64 form (64-row A boxes)
constexpr int THIN_SMEM_BYTES = THIN_STAGES * KP1 * (A_BYTES / 2 + B_BYTES) + 1024 + BAR_BYTES;
static_assert(THIN_SMEM_BYTES <= 227 * 1024, "thin GEMM stages must fit in shared memory");
constexpr uint32_t IDESC = idesc_bf16_f32(BM, BN);

struct Params {
  __nv_bfloat16* C;
  const __nv_bfloat16* R;
  int64_t ldc, ldr;
  int M, n_out;
  int num_m_blocks, num_tiles, k_blocks;
  int sys_fence;   // C may be another GPU's memory: end every epilogue thread with a system-scope fence
  unsigned* sched; // 1-SM kernel: [next tile, CTAs finished], zero at launch; the last CTA to finish re-zeroes it
  // Split K (1-SM kernel, one m-block): work unit u = (tile u / k_split, K chunk c = u % k_split), chunk c covering
  // k-blocks [c * k_blocks / k_split, (c + 1) * k_blocks / k_split) (sizes differ by one at most); each unit stores
  // its fp32 partial of the B rows it covers to ws[(chunk * M + row) * ldw + B row], and splitk_reduce_kernel
  // applies the epilogue to the sums. k_split = 1: whole K, fused epilogue.
  int k_split;
  float* ws;
  int64_t ldw;
  unsigned* err;
  int b_once;   // 1-SM kernel, one m-block: every weight byte is read once, under the L2 evict-first policy
};

constexpr int TQ = 4;   // tile-queue entries (claimed tiles handed from the producer to the MMA and epilogue warps)

// Tile order. Tiles are numbered so that the CTAs working at one time share operands in L2: M fastest inside
// groups of GROUP_M m-blocks, groups in N order (GROUP_M = 0: M fastest over the whole matrix).
#ifndef FS_GEMM_GROUP_M
#define FS_GEMM_GROUP_M 8
#endif
constexpr int GROUP_M = FS_GEMM_GROUP_M;

__device__ __forceinline__ void tile_coords(int tile, int num_m, int num_n, int& m_blk, int& n_blk) {
  if (GROUP_M <= 0 || num_m <= GROUP_M) {
    m_blk = tile % num_m;
    n_blk = tile / num_m;
    return;
  }
  const int per_group = GROUP_M * num_n;
  const int first = (tile / per_group) * GROUP_M;
  const int gm = num_m - first < GROUP_M ? num_m - first : GROUP_M;
  const int local = tile - (tile / per_group) * per_group;
  m_blk = first + local % gm;
  n_blk = local / gm;
}

__device__ __forceinline__ float bf16_lo(uint32_t v) { return __uint_as_float(v << 16); }
__device__ __forceinline__ float bf16_hi(uint32_t v) { return __uint_as_float(v & 0xFFFF0000u); }
__device__ __forceinline__ uint32_t pack_bf16(float lo, float hi) {
  __nv_bfloat162 h = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&h);
}
__device__ __forceinline__ float silu_f(float x) { return x / (1.0f + expf(-x)); }

// Store 32 consecutive outputs of one row (values already final fp32, rounded to bf16 here).
__device__ __forceinline__ void store_row32(__nv_bfloat16* crow, int col0, int n_out, bool vec_ok,
                                            const float (&v)[32]) {
  if (vec_ok && col0 + 32 <= n_out) {
    uint4* dst = reinterpret_cast<uint4*>(crow + col0);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      uint4 w;
      w.x = pack_bf16(v[8 * i + 0], v[8 * i + 1]);
      w.y = pack_bf16(v[8 * i + 2], v[8 * i + 3]);
      w.z = pack_bf16(v[8 * i + 4], v[8 * i + 5]);
      w.w = pack_bf16(v[8 * i + 6], v[8 * i + 7]);
      dst[i] = w;
    }
  } else {
#pragma unroll
    for (int i = 0; i < 32; ++i)
      if (col0 + i < n_out) crow[col0 + i] = __float2bfloat16_rn(v[i]);
  }
}

__device__ __forceinline__ bool warp_wait(uint64_t* bar, uint32_t parity, unsigned* err) {
  // Every lane waits (bounded); the warp proceeds only if all lanes saw the phase complete, so that the
  // following .sync.aligned tcgen05 instructions are executed by the whole warp or by none of it.
  bool ok = mbar_wait(bar, parity, err);
  return __all_sync(0xffffffffu, ok);
}

// One accumulator (128 rows x 256 fp32 columns in TMEM, lanes 32q..32q+31 read by this warp) -> global memory,
// with the fused epilogue. `row` is this thread's output row.
template <int EPI>
__device__ __forceinline__ void epilogue_tile(const Params& p, uint32_t tmem_base, int acc, int q, int lane, int row,
                                              int n_blk, bool vec_ok) {
  const bool row_ok = row < p.M;
  __nv_bfloat16* crow = p.C + static_cast<int64_t>(row) * p.ldc;
  const uint32_t taddr = tmem_base + (static_cast<uint32_t>(q * 32) << 16) + static_cast<uint32_t>(acc * BN);
  if constexpr (EPI == EPI_SWIGLU) {
#pragma unroll 1
    for (int c = 0; c < BN / 64; ++c) {
      uint32_t g[32], u[32];
      tmem_ld_32x32b_x32(taddr + c * 32, g);
      tmem_ld_32x32b_x32(taddr + BN / 2 + c * 32, u);
      tc_wait_ld();
      tmem_regs_ready(g);
      tmem_regs_ready(u);
      float v[32];
#pragma unroll
      for (int i = 0; i < 32; ++i) {
        const float gb = rnd<__nv_bfloat16>(__uint_as_float(g[i]));
        const float ub = rnd<__nv_bfloat16>(__uint_as_float(u[i]));
        v[i] = rnd<__nv_bfloat16>(silu_f(gb)) * ub;
      }
      if (row_ok) store_row32(crow, n_blk * (BN / 2) + c * 32, p.n_out, vec_ok, v);
    }
  } else {
#pragma unroll 1
    for (int c = 0; c < BN / 32; ++c) {
      uint32_t r[32];
      tmem_ld_32x32b_x32(taddr + c * 32, r);
      tc_wait_ld();
      tmem_regs_ready(r);
      const int col0 = n_blk * BN + c * 32;
      float v[32];
#pragma unroll
      for (int i = 0; i < 32; ++i) v[i] = rnd<__nv_bfloat16>(__uint_as_float(r[i]));
      if constexpr (EPI == EPI_RESIDUAL) {
        if (row_ok) {
          const __nv_bfloat16* rrow = p.R + static_cast<int64_t>(row) * p.ldr;
          if (vec_ok && col0 + 32 <= p.n_out) {
            const uint4* src = reinterpret_cast<const uint4*>(rrow + col0);
#pragma unroll
            for (int i = 0; i < 4; ++i) {
              const uint4 w = src[i];
              v[8 * i + 0] += bf16_lo(w.x), v[8 * i + 1] += bf16_hi(w.x);
              v[8 * i + 2] += bf16_lo(w.y), v[8 * i + 3] += bf16_hi(w.y);
              v[8 * i + 4] += bf16_lo(w.z), v[8 * i + 5] += bf16_hi(w.z);
              v[8 * i + 6] += bf16_lo(w.w), v[8 * i + 7] += bf16_hi(w.w);
            }
          } else {
#pragma unroll
            for (int i = 0; i < 32; ++i)
              if (col0 + i < p.n_out) v[i] += __bfloat162float(rrow[col0 + i]);
          }
        }
      }
      if (row_ok) store_row32(crow, col0, p.n_out, vec_ok, v);
    }
  }
}

// Split-K epilogue: this unit's fp32 partial sums (no rounding) to the workspace, by B row.
template <int EPI>
__device__ __forceinline__ void epilogue_partial(const Params& p, uint32_t tmem_base, int acc, int q, int lane, int row,
                                                 int n_blk, int chunk) {
  const uint32_t taddr = tmem_base + (static_cast<uint32_t>(q * 32) << 16) + static_cast<uint32_t>(acc * BN);
  float* wrow = p.ws + (static_cast<int64_t>(chunk) * p.M + row) * p.ldw;
  const int n_b = EPI == EPI_SWIGLU ? 2 * p.n_out : p.n_out;   // B rows
  const bool row_ok = row < p.M;
#pragma unroll 1
  for (int c = 0; c < BN / 32; ++c) {
    uint32_t r[32];
    __syncwarp();   // the whole warp takes part in the collective TMEM load
    tmem_ld_32x32b_x32(taddr + c * 32, r);
    tc_wait_ld();
    tmem_regs_ready(r);
    int brow0, lim;   // first B row of these 32 accumulator columns, and the end of their half (or of B)
    if constexpr (EPI == EPI_SWIGLU) {
      const int half_col = (c * 32) % (BN / 2);
      brow0 = (c * 32 < BN / 2 ? 0 : p.n_out) + n_blk * (BN / 2) + half_col;
      lim = (c * 32 < BN / 2 ? 0 : p.n_out) + p.n_out;
    } else {
      brow0 = n_blk * BN + c * 32;
      lim = n_b;
    }
    if (!row_ok) {
    } else if (brow0 + 32 <= lim && ((p.ldw | brow0) & 3) == 0) {
      float4* dst = reinterpret_cast<float4*>(wrow + brow0);
#pragma unroll
      for (int i = 0; i < 8; ++i)
        dst[i] = make_float4(__uint_as_float(r[4 * i]), __uint_as_float(r[4 * i + 1]), __uint_as_float(r[4 * i + 2]),
                             __uint_as_float(r[4 * i + 3]));
    } else {
#pragma unroll
      for (int i = 0; i < 32; ++i)
        if (brow0 + i < lim) wrow[brow0 + i] = __uint_as_float(r[i]);
    }
  }
}

// Sums the split-K partials and applies the epilogue with the fused kernel's rounding points.
template <int EPI>
__global__ void __launch_bounds__(256)
    splitk_reduce_kernel(const float* __restrict__ ws, int64_t ldw, int k_split, int M, int n_out,
                         __nv_bfloat16* __restrict__ C, int64_t ldc, const __nv_bfloat16* __restrict__ R, int64_t ldr) {
  pdl_trigger();
  pdl_wait();
  const int64_t total = static_cast<int64_t>(M) * n_out;
  const int64_t plane = static_cast<int64_t>(M) * ldw;
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < total;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int row = static_cast<int>(i / n_out), j = static_cast<int>(i % n_out);
    const float* w = ws + static_cast<int64_t>(row) * ldw;
    float a = 0.f, b = 0.f;
    for (int k = 0; k < k_split; ++k) {
      a += w[k * plane + j];
      if constexpr (EPI == EPI_SWIGLU) b += w[k * plane + n_out + j];
    }
    float v;
    if constexpr (EPI == EPI_SWIGLU) {
      v = rnd<__nv_bfloat16>(silu_f(rnd<__nv_bfloat16>(a))) * rnd<__nv_bfloat16>(b);
    } else {
      v = rnd<__nv_bfloat16>(a);
      if constexpr (EPI == EPI_RESIDUAL) v += __bfloat162float(R[static_cast<int64_t>(row) * ldr + j]);
    }
    C[static_cast<int64_t>(row) * ldc + j] = __float2bfloat16_rn(v);
  }
}

// The same sums and epilogue, four consecutive outputs of one row per thread: grid (column groups, rows), float4
// loads of the partials, each output summed over the chunks in the same order as above (the same bits). Needs
// n_out % 4 == 0 and 8-byte aligned rows of C (and R); the workspace rows are 16-byte aligned (ldw % 4 == 0). C may
// be R (an in-place residual): every thread reads its own four residuals before it stores them.
template <int EPI>
__global__ void __launch_bounds__(256)
    splitk_reduce_vec_kernel(const float* __restrict__ ws, int64_t ldw, int k_split, int M, int n_out,
                             __nv_bfloat16* C, int64_t ldc, const __nv_bfloat16* R, int64_t ldr) {
  pdl_trigger();
  pdl_wait();
  const int row = blockIdx.y;
  const int j = (blockIdx.x * 256 + threadIdx.x) * 4;
  if (j >= n_out) return;
  const int64_t plane = static_cast<int64_t>(M) * ldw;
  const float* w = ws + static_cast<int64_t>(row) * ldw + j;
  float a[4] = {0.f, 0.f, 0.f, 0.f}, b[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll 4
  for (int k = 0; k < k_split; ++k) {
    const float4 x = *reinterpret_cast<const float4*>(w + k * plane);
    a[0] += x.x;
    a[1] += x.y;
    a[2] += x.z;
    a[3] += x.w;
    if constexpr (EPI == EPI_SWIGLU) {
      const float4 y = *reinterpret_cast<const float4*>(w + k * plane + n_out);
      b[0] += y.x;
      b[1] += y.y;
      b[2] += y.z;
      b[3] += y.w;
    }
  }
  float v[4];
  if constexpr (EPI == EPI_RESIDUAL) {
    const uint2 rr = *reinterpret_cast<const uint2*>(R + static_cast<int64_t>(row) * ldr + j);
    v[0] = rnd<__nv_bfloat16>(a[0]) + bf16_lo(rr.x);
    v[1] = rnd<__nv_bfloat16>(a[1]) + bf16_hi(rr.x);
    v[2] = rnd<__nv_bfloat16>(a[2]) + bf16_lo(rr.y);
    v[3] = rnd<__nv_bfloat16>(a[3]) + bf16_hi(rr.y);
  } else {
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      if constexpr (EPI == EPI_SWIGLU)
        v[i] = rnd<__nv_bfloat16>(silu_f(rnd<__nv_bfloat16>(a[i]))) * rnd<__nv_bfloat16>(b[i]);
      else
        v[i] = rnd<__nv_bfloat16>(a[i]);
    }
  }
  uint2 out;
  out.x = pack_bf16(v[0], v[1]);
  out.y = pack_bf16(v[2], v[3]);
  *reinterpret_cast<uint2*>(C + static_cast<int64_t>(row) * ldc + j) = out;
}

template <int EPI, bool THIN>
__global__ void __launch_bounds__(THREADS, 1)
    gemm_tc_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB, Params p) {
  // THIN (M <= 64: decode steps): the A box is the 64 live rows (8 KB; the MMA's rows 64-127 read whatever follows
  // and land in accumulator rows that are never stored), which leaves room for a fifth stage of weights in flight.
  constexpr int NST = THIN ? THIN_STAGES : STAGES;
  constexpr int ABYTES = THIN ? A_BYTES / 2 : A_BYTES;
  constexpr int SBYTES = KP1 * (ABYTES + B_BYTES);
  static_assert((2 * NST + 2 * NUM_ACC + 1) * 8 + 8 <= 128, "stage barriers, TMEM slot and abort flag fill 128 bytes");
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* tiles = smem;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + NST * SBYTES);
  uint64_t* full = bars;
  uint64_t* empty = bars + NST;
  uint64_t* tfull = bars + 2 * NST;
  uint64_t* tempty = bars + 2 * NST + NUM_ACC;
  uint64_t* mma_done = bars + 2 * NST + 2 * NUM_ACC;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(mma_done + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  uint64_t* tq_full = reinterpret_cast<uint64_t*>(smem + NST * SBYTES + 128);
  uint64_t* tq_empty = tq_full + TQ;
  volatile int* tq = reinterpret_cast<volatile int*>(tq_empty + TQ);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int s = 0; s < NST; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int a = 0; a < NUM_ACC; ++a) {
      mbar_init(&tfull[a], 1);
      mbar_init(&tempty[a], 128);
    }
    for (int i = 0; i < TQ; ++i) {
      mbar_init(&tq_full[i], 1);
      mbar_init(&tq_empty[i], 1 + 4);   // the MMA thread and one lane of each epilogue warp
    }
    mbar_init(mma_done, 1);
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 0 && lane == 0) {
    prefetch_tmap(&tmA);
    prefetch_tmap(&tmB);
  }
  if (warp == 2) {
    tmem_alloc(tmem_slot, TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  pdl_trigger();   // TMEM is held: the next kernel on the stream may start its own set-up

  // The first unit of every CTA is its own index, so that (launched with PDL) its weight loads can start while the
  // kernel before it still runs; everything else waits for that kernel (pdl_wait). Later units are claimed at run
  // time from a counter shared by the grid, in increasing order (M fastest), so a CTA slowed down by other work on
  // its SM (a resident NCCL kernel) takes fewer units instead of holding the whole GEMM back. The producer claims;
  // the tile queue hands each unit (or -1: none left) to the MMA thread and the epilogue warps.
  if (warp == 0) {
    // ------------------------------------------------------------------ TMA producer
    if (lane == 0) {
      int s = 0;
      uint32_t ph = 0;
      bool issued[NST];
      uint32_t last_ph[NST];
#pragma unroll
      for (int i = 0; i < NST; ++i) issued[i] = false, last_ph[i] = 0;
      const int total = p.num_tiles * p.k_split;
      const int first = static_cast<int>(blockIdx.x) < total ? static_cast<int>(blockIdx.x) : -1;
      auto unit_coords = [&](int unit, int& kb0, int& kb1, int& m_blk, int& b_row0, int& b_row1) {
        const int tile = unit / p.k_split, chunk = unit % p.k_split;
        kb0 = chunk * p.k_blocks / p.k_split;
        kb1 = (chunk + 1) * p.k_blocks / p.k_split;
        int n_blk;
        tile_coords(tile, p.num_m_blocks, p.num_tiles / p.num_m_blocks, m_blk, n_blk);
        b_row0 = EPI == EPI_SWIGLU ? n_blk * (BN / 2) : n_blk * BN;
        b_row1 = EPI == EPI_SWIGLU ? p.n_out + n_blk * (BN / 2) : n_blk * BN + BN / 2;
      };
      const uint64_t b_policy = p.b_once ? l2_policy_evict_first() : 0;
      auto load_b = [&](void* dst, uint64_t* bar, int kx, int row) {
        if (p.b_once)
          tma_load_2d_hint(dst, &tmB, bar, kx, row, b_policy);
        else
          tma_load_2d(dst, &tmB, bar, kx, row);
      };
      // Weights of the first unit's first k-blocks (the ring is fresh: stage i, phase 0), before the wait.
      int pre = 0;
      if (first >= 0) {
        int kb0, kb1, m_blk, b_row0, b_row1;
        unit_coords(first, kb0, kb1, m_blk, b_row0, b_row1);
        for (int kb = kb0; kb < kb1 && pre < NST; ++kb, ++pre) {
          mbar_arrive_expect_tx(&full[pre], SBYTES);
#pragma unroll
          for (int pk = 0; pk < KP1; ++pk) {
            const int kx = (kb * KP1 + pk) * BK;
            uint8_t* st = tiles + pre * SBYTES;
            load_b(st + KP1 * ABYTES + pk * B_BYTES, &full[pre], kx, b_row0);
            load_b(st + KP1 * ABYTES + pk * B_BYTES + BH_BYTES, &full[pre], kx, b_row1);
          }
          issued[pre] = true;
        }
      }
      pdl_wait();
      if (pre > 0) {   // ... and then the activations of those k-blocks, so that no stage is ever left half-issued
        int kb0, kb1, m_blk, b_row0, b_row1;
        unit_coords(first, kb0, kb1, m_blk, b_row0, b_row1);
        for (int j = 0; j < pre; ++j)
#pragma unroll
          for (int pk = 0; pk < KP1; ++pk)
            tma_load_2d(tiles + j * SBYTES + pk * ABYTES, &tmA, &full[j], ((kb0 + j) * KP1 + pk) * BK,
                        m_blk * BM);
      }
      bool ok = true;
      for (int i = 0; ok; ++i) {
        const int slot = i & (TQ - 1);
        if (!mbar_wait(&tq_empty[slot], static_cast<uint32_t>((i / TQ) & 1) ^ 1u, p.err) || *abort_flag) {
          ok = false;
          break;
        }
        int unit = first;
        if (i > 0) {
          unit = static_cast<int>(gridDim.x + atomicAdd(p.sched, 1u));
          if (unit >= total) unit = -1;
        }
        tq[slot] = unit;
        mbar_arrive(&tq_full[slot]);
        if (unit < 0) break;
        int kb0, kb1, m_blk, b_row0, b_row1;
        unit_coords(unit, kb0, kb1, m_blk, b_row0, b_row1);
        for (int kb = kb0; kb < kb1; ++kb) {
          if (!(i == 0 && kb - kb0 < pre)) {   // (the first `pre` k-blocks of the first unit are issued already)
            if (!mbar_wait(&empty[s], ph ^ 1u, p.err) || *abort_flag) {
              ok = false;
              break;
            }
            mbar_arrive_expect_tx(&full[s], SBYTES);
#pragma unroll
            for (int pk = 0; pk < KP1; ++pk) {
              const int kx = (kb * KP1 + pk) * BK;
              uint8_t* st = tiles + s * SBYTES;
              tma_load_2d(st + pk * ABYTES, &tmA, &full[s], kx, m_blk * BM);
              load_b(st + KP1 * ABYTES + pk * B_BYTES, &full[s], kx, b_row0);
              load_b(st + KP1 * ABYTES + pk * B_BYTES + BH_BYTES, &full[s], kx, b_row1);
            }
          }
          issued[s] = true;
          last_ph[s] = ph;
          if (++s == NST) s = 0, ph ^= 1u;
        }
      }
      if (!ok) {
        *abort_flag = 1;
        // Let every copy this thread started land before the CTA can exit (bounded).
        for (int i = 0; i < NST; ++i)
          if (issued[i]) mbar_wait(&full[i], last_ph[i], p.err);
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      int s = 0, acc = 0;
      uint32_t ph = 0, acc_ph = 0;
      bool ok = true;
      for (int i = 0; ok; ++i) {
        const int slot = i & (TQ - 1);
        if (!mbar_wait(&tq_full[slot], static_cast<uint32_t>((i / TQ) & 1), p.err) || *abort_flag) {
          ok = false;
          break;
        }
        const int unit = tq[slot];
        mbar_arrive(&tq_empty[slot]);
        if (unit < 0) break;
        const int chunk = unit % p.k_split;
        const int kb0 = chunk * p.k_blocks / p.k_split, kb1 = (chunk + 1) * p.k_blocks / p.k_split;
        if (!mbar_wait(&tempty[acc], acc_ph ^ 1u, p.err) || *abort_flag) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + static_cast<uint32_t>(acc * BN);
        for (int kb = kb0; kb < kb1; ++kb) {
          if (!mbar_wait(&full[s], ph, p.err) || *abort_flag) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a_addr = smem_u32(tiles + s * SBYTES);
#pragma unroll
          for (int pk = 0; pk < KP1; ++pk) {
            const uint64_t adesc = sw128_kmajor_desc(a_addr + pk * ABYTES);
            const uint64_t bdesc = sw128_kmajor_desc(a_addr + KP1 * ABYTES + pk * B_BYTES);
#pragma unroll
            for (int k = 0; k < BK / 16; ++k) {
              // +32 bytes along K inside the 128-byte swizzle row = +2 in the descriptor's address field
              tc_mma_f16(d_tmem, adesc + 2u * k, bdesc + 2u * k, IDESC, (kb != kb0 || pk != 0 || k != 0) ? 1u : 0u);
            }
          }
          tc_commit(&empty[s]);  // the smem stage is free once these MMAs have read it
          if (++s == NST) s = 0, ph ^= 1u;
        }
        if (!ok) break;
        tc_commit(&tfull[acc]);  // accumulator complete
        if (++acc == NUM_ACC) acc = 0, acc_ph ^= 1u;
      }
      if (!ok) *abort_flag = 1;
      tc_commit(mma_done);  // arrives once every MMA issued above has completed
    }
  } else if (warp >= 4) {
    // ------------------------------------------------------------------ epilogue (TMEM -> global)
    const int q = warp - 4;  // this warp may read TMEM lanes 32q .. 32q+31
    const bool vec_ok = ((p.ldc & 7) == 0) && ((reinterpret_cast<uintptr_t>(p.C) & 15) == 0) &&
                        (EPI != EPI_RESIDUAL || (((p.ldr & 7) == 0) && ((reinterpret_cast<uintptr_t>(p.R) & 15) == 0)));
    pdl_wait();   // C, R and the split-K workspace belong to the kernels before this one until they complete
    int acc = 0;
    uint32_t acc_ph = 0;
    for (int i = 0;; ++i) {
      const int slot = i & (TQ - 1);
      if (!warp_wait(&tq_full[slot], static_cast<uint32_t>((i / TQ) & 1), p.err)) break;
      const int unit = tq[slot];
      __syncwarp();
      if (lane == 0) mbar_arrive(&tq_empty[slot]);
      if (unit < 0) break;
      if (!warp_wait(&tfull[acc], acc_ph, p.err)) break;
      tc_fence_after();
      int m_blk, n_blk;
      tile_coords(unit / p.k_split, p.num_m_blocks, p.num_tiles / p.num_m_blocks, m_blk, n_blk);
      if (THIN && q >= 2) {
        // accumulator lanes 64-127 hold rows that do not exist
      } else if (p.k_split > 1) {
        epilogue_partial<EPI>(p, tmem_base, acc, q, lane, m_blk * BM + q * 32 + lane, n_blk, unit % p.k_split);
      } else {
        epilogue_tile<EPI>(p, tmem_base, acc, q, lane, m_blk * BM + q * 32 + lane, n_blk, vec_ok);
      }
      tc_fence_before();
      mbar_arrive(&tempty[acc]);
      if (++acc == NUM_ACC) acc = 0, acc_ph ^= 1u;
    }
  }

  if (p.sys_fence) __threadfence_system();   // peer stores performed before the kernel completes
  __syncthreads();
  if (warp == 2) {
    // All MMAs must have completed before the accumulators are released (they have, unless a wait ran out).
    mbar_wait(mma_done, 0, p.err);
    tc_fence_after();
    tmem_dealloc(tmem_base, TMEM_COLS);
  }
  if (threadIdx.x == 0) {
    // Every CTA has finished claiming once all have counted themselves out; the last one re-zeroes the counter
    // for the next launch on this stream (on every path, the ones that gave up included).
    __threadfence();
    if (atomicAdd(p.sched + 1, 1u) == gridDim.x - 1) {
      atomicExch(p.sched, 0u);
      atomicExch(p.sched + 1, 0u);
    }
  }
}

// ============================================================================ 2-SM (cta_group::2) variant
// A CTA pair (cluster of 2) computes a 256 x 256 tile with tcgen05.mma.cta_group::2 (M 256, N 256): each CTA stages
// its own 128 rows of A and its own 128-row half of B (32 KB per k-block instead of 48 KB), so shared-memory
// traffic per FLOP drops by a third against the 1-SM kernel, and 6 stages fit. The leader CTA (rank 0) issues
// the MMAs; every copy completes on the leader's barrier; the leader signals both CTAs' barriers; both CTAs'
// epilogues read their own TMEM (their 128 rows) and report to the leader's accumulator-free barrier.
// A stage of the pair kernel holds KP 64-wide K panels of A and B (one k-block = 64 * KP of K); the ring keeps
// ~192 KB of stages either way.
#ifndef FS_GEMM_PAIR_KPANELS
#define FS_GEMM_PAIR_KPANELS 2
#endif
#ifndef FS_GEMM_PAIR_STAGES
#define FS_GEMM_PAIR_STAGES (6 / FS_GEMM_PAIR_KPANELS)
#endif
constexpr int KP = FS_GEMM_PAIR_KPANELS;
constexpr int STAGES2 = FS_GEMM_PAIR_STAGES;
constexpr int STAGE2_BYTES = KP * (A_BYTES + BH_BYTES);  // 32 KiB per CTA per 64 of K
constexpr int SMEM2_BYTES = STAGES2 * STAGE2_BYTES + 1024 + BAR_BYTES;
constexpr uint32_t IDESC2 = idesc_bf16_f32(2 * BM, BN);

__device__ __forceinline__ uint32_t cluster_ctarank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
// Address of the same shared-memory offset in CTA `cta` of the cluster.
__device__ __forceinline__ uint32_t map_to_cta(uint32_t smem_addr, uint32_t cta) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(smem_addr), "r"(cta));
  return r;
}
__device__ __forceinline__ void cluster_sync_all() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
__device__ __forceinline__ void mbar_arrive_remote(uint32_t cluster_addr) {
  asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(cluster_addr) : "memory");
}
__device__ __forceinline__ void st_cluster_u32(uint32_t cluster_addr, uint32_t v) {
  asm volatile("st.shared::cluster.u32 [%0], %1;" ::"r"(cluster_addr), "r"(v) : "memory");
}
__device__ __forceinline__ bool mbar_try_wait_cluster(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}
// Bounded wait whose acquire covers writes the other CTA of the pair made before its release-arrive.
__device__ __forceinline__ bool mbar_wait_cluster(uint64_t* bar, uint32_t parity, unsigned* err) {
  if (mbar_try_wait_cluster(bar, parity)) return true;
  const uint64_t t0 = globaltimer_ns();
  uint32_t spins = 0;
  while (true) {
    if (mbar_try_wait_cluster(bar, parity)) return true;
    if ((++spins & 255u) == 0 && globaltimer_ns() - t0 > kWaitLimitNs) {
      flag_error(err, ERR_WAIT_TIMEOUT);
      return false;
    }
  }
}
// 2-D TMA load into this CTA's shared memory whose completion is counted on a barrier of either CTA of the pair.
__device__ __forceinline__ void tma_load_2d_pair(void* smem_dst, const CUtensorMap* map, uint32_t bar_cluster_addr,
                                                 int x, int y) {
  asm volatile(
      "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4}], "
      "[%2];" ::"r"(smem_u32(smem_dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(bar_cluster_addr), "r"(x), "r"(y)
      : "memory");
}
__device__ __forceinline__ void tc_mma_f16_pair(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                                uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}
// Arrive on a barrier (of either CTA of the pair) once every pair MMA issued so far by this thread has completed.
__device__ __forceinline__ void tc_commit_pair(uint32_t bar_cluster_addr) {
  asm volatile("tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar_cluster_addr)
               : "memory");
}
__device__ __forceinline__ void tmem_alloc_pair(uint32_t* smem_slot, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(smem_slot)),
               "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void tmem_relinquish_pair() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc_pair(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}

template <int EPI>
__global__ void __launch_bounds__(THREADS, 1)
    gemm_tc2_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB, Params p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* tiles = smem;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + STAGES2 * STAGE2_BYTES);
  uint64_t* full = bars;                          // leader's: both CTAs' copies complete here
  uint64_t* empty = bars + STAGES2;               // each CTA's own: the leader's MMAs released the stage
  uint64_t* tfull = bars + 2 * STAGES2;           // each CTA's own: accumulator ready
  uint64_t* tempty = bars + 2 * STAGES2 + NUM_ACC;  // leader's: both epilogues released the accumulator
  uint64_t* mma_done = bars + 2 * STAGES2 + 2 * NUM_ACC;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(mma_done + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  uint64_t* tq_full = reinterpret_cast<uint64_t*>(smem + STAGES2 * STAGE2_BYTES + 128);   // each CTA's own
  uint64_t* tq_empty = tq_full + TQ;                                                     // the leader's is used
  volatile int* tq = reinterpret_cast<volatile int*>(tq_empty + TQ);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t cta = cluster_ctarank();

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES2; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int a = 0; a < NUM_ACC; ++a) {
      mbar_init(&tfull[a], 1);
      mbar_init(&tempty[a], 2 * 128);
    }
    for (int i = 0; i < TQ; ++i) {
      mbar_init(&tq_full[i], 1);
      mbar_init(&tq_empty[i], 2 + 1 + 2 * 4);   // both producers, the MMA thread, both CTAs' epilogue warps
    }
    mbar_init(mma_done, 1);
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 2) {
    tmem_alloc_pair(tmem_slot, TMEM_COLS);
    tmem_relinquish_pair();
  }
  tc_fence_before();
  __syncthreads();
  cluster_sync_all();   // both CTAs' barriers exist before any copy or arrive reaches them
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  const int num_m_pairs = (p.num_m_blocks + 1) >> 1;
  // Tile queue: the leader's producer claims a tile from the grid's counter and publishes it in both CTAs' queue
  // slot (the peer's by a store to its shared memory and a release-arrive on its barrier); every consumer of the
  // slot (both producers, the MMA thread, both CTAs' epilogue warps) releases it on the leader's tq_empty.
  const uint32_t leader_tq_empty = map_to_cta(smem_u32(tq_empty), 0);
  auto release_slot = [&](int slot) {
    if (cta == 0) mbar_arrive(&tq_empty[slot]);
    else mbar_arrive_remote(leader_tq_empty + 8u * static_cast<uint32_t>(slot));
  };

  if (warp == 0) {
    // -------------------------------------------------------------------------------- TMA producer (both CTAs)
    if (lane == 0) {
      int s = 0;
      uint32_t ph = 0;
      bool ok = true;
      for (int i = 0; ok; ++i) {
        const int slot = i & (TQ - 1);
        const uint32_t qph = static_cast<uint32_t>((i / TQ) & 1);
        if (cta == 0) {
          if (!mbar_wait_cluster(&tq_empty[slot], qph ^ 1u, p.err) || *abort_flag) {
            ok = false;
            break;
          }
          int claim = static_cast<int>(atomicAdd(p.sched, 1u));
          if (claim >= p.num_tiles) claim = -1;
          tq[slot] = claim;
          st_cluster_u32(map_to_cta(smem_u32(const_cast<int*>(&tq[slot])), 1), static_cast<uint32_t>(claim));
          mbar_arrive(&tq_full[slot]);
          mbar_arrive_remote(map_to_cta(smem_u32(&tq_full[slot]), 1));
        }
        if (!mbar_wait_cluster(&tq_full[slot], qph, p.err) || *abort_flag) {
          ok = false;
          break;
        }
        const int tile = tq[slot];
        release_slot(slot);
        if (tile < 0) break;
        int m_pair, n_blk;
        tile_coords(tile, num_m_pairs, p.num_tiles / num_m_pairs, m_pair, n_blk);
        const int a_row = m_pair * 2 * BM + static_cast<int>(cta) * BM;
        const int b_row = EPI == EPI_SWIGLU ? (cta == 0 ? n_blk * (BN / 2) : p.n_out + n_blk * (BN / 2))
                                            : n_blk * BN + static_cast<int>(cta) * (BN / 2);
        for (int kb = 0; kb < p.k_blocks; ++kb) {
          if (!mbar_wait(&empty[s], ph ^ 1u, p.err) || *abort_flag) {
            ok = false;
            break;
          }
          const uint32_t leader_full = map_to_cta(smem_u32(&full[s]), 0);
          if (cta == 0) mbar_arrive_expect_tx(&full[s], 2 * STAGE2_BYTES);
#pragma unroll
          for (int pk = 0; pk < KP; ++pk) {
            tma_load_2d_pair(tiles + s * STAGE2_BYTES + pk * A_BYTES, &tmA, leader_full, (kb * KP + pk) * BK, a_row);
            tma_load_2d_pair(tiles + s * STAGE2_BYTES + KP * A_BYTES + pk * BH_BYTES, &tmB, leader_full,
                             (kb * KP + pk) * BK, b_row);
          }
          if (++s == STAGES2) s = 0, ph ^= 1u;
        }
      }
      if (!ok) *abort_flag = 1;
    }
  } else if (warp == 1) {
    // -------------------------------------------------------------------------------- MMA issuer (leader only)
    if (lane == 0 && cta == 0) {
      int s = 0, acc = 0;
      uint32_t ph = 0, acc_ph = 0;
      bool ok = true;
      for (int i = 0; ok; ++i) {
        const int slot = i & (TQ - 1);
        if (!mbar_wait_cluster(&tq_full[slot], static_cast<uint32_t>((i / TQ) & 1), p.err) || *abort_flag) {
          ok = false;
          break;
        }
        const int tile = tq[slot];
        release_slot(slot);
        if (tile < 0) break;
        if (!mbar_wait(&tempty[acc], acc_ph ^ 1u, p.err) || *abort_flag) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + static_cast<uint32_t>(acc * BN);
        for (int kb = 0; kb < p.k_blocks; ++kb) {
          if (!mbar_wait(&full[s], ph, p.err) || *abort_flag) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a_addr = smem_u32(tiles + s * STAGE2_BYTES);
#pragma unroll
          for (int pk = 0; pk < KP; ++pk) {
            const uint64_t adesc = sw128_kmajor_desc(a_addr + pk * A_BYTES);
            const uint64_t bdesc = sw128_kmajor_desc(a_addr + KP * A_BYTES + pk * BH_BYTES);
#pragma unroll
            for (int k = 0; k < BK / 16; ++k)
              tc_mma_f16_pair(d_tmem, adesc + 2u * k, bdesc + 2u * k, IDESC2, (kb | pk | k) != 0);
          }
          const uint32_t e = smem_u32(&empty[s]);
          tc_commit_pair(map_to_cta(e, 0));
          tc_commit_pair(map_to_cta(e, 1));
          if (++s == STAGES2) s = 0, ph ^= 1u;
        }
        if (!ok) break;
        const uint32_t f = smem_u32(&tfull[acc]);
        tc_commit_pair(map_to_cta(f, 0));
        tc_commit_pair(map_to_cta(f, 1));
        if (++acc == NUM_ACC) acc = 0, acc_ph ^= 1u;
      }
      if (!ok) *abort_flag = 1;
      const uint32_t d = smem_u32(mma_done);
      tc_commit_pair(map_to_cta(d, 0));
      tc_commit_pair(map_to_cta(d, 1));
    }
  } else if (warp >= 4) {
    // -------------------------------------------------------------------------------- epilogue (both CTAs)
    const int q = warp - 4;
    const bool vec_ok = ((p.ldc & 7) == 0) && ((reinterpret_cast<uintptr_t>(p.C) & 15) == 0) &&
                        (EPI != EPI_RESIDUAL || (((p.ldr & 7) == 0) && ((reinterpret_cast<uintptr_t>(p.R) & 15) == 0)));
    int acc = 0;
    uint32_t acc_ph = 0;
    for (int i = 0;; ++i) {
      const int slot = i & (TQ - 1);
      if (!__all_sync(0xffffffffu, mbar_wait_cluster(&tq_full[slot], static_cast<uint32_t>((i / TQ) & 1), p.err)))
        break;
      const int tile = tq[slot];
      __syncwarp();
      if (lane == 0) release_slot(slot);
      if (tile < 0) break;
      if (!warp_wait(&tfull[acc], acc_ph, p.err)) break;
      tc_fence_after();
      int m_pair, n_blk;
      tile_coords(tile, num_m_pairs, p.num_tiles / num_m_pairs, m_pair, n_blk);
      const int row = m_pair * 2 * BM + static_cast<int>(cta) * BM + q * 32 + lane;
      epilogue_tile<EPI>(p, tmem_base, acc, q, lane, row, n_blk, vec_ok);
      tc_fence_before();
      const uint32_t te = smem_u32(&tempty[acc]);
      if (cta == 0) mbar_arrive(&tempty[acc]);
      else mbar_arrive_remote(map_to_cta(te, 0));
      if (++acc == NUM_ACC) acc = 0, acc_ph ^= 1u;
    }
  }

  if (p.sys_fence) __threadfence_system();   // peer stores performed before the kernel completes
  __syncthreads();
  if (warp == 2) {
    mbar_wait(mma_done, 0, p.err);   // every pair MMA has completed (this CTA's TMEM included)
    tc_fence_after();
    tmem_dealloc_pair(tmem_base, TMEM_COLS);
  }
  cluster_sync_all();   // neither CTA leaves while the other may still signal its barriers
  if (threadIdx.x == 0) {
    // every CTA has finished claiming once all have counted themselves out; the last one re-zeroes the counter
    __threadfence();
    if (atomicAdd(p.sched + 1, 1u) == gridDim.x - 1) {
      atomicExch(p.sched, 0u);
      atomicExch(p.sched + 1, 0u);
    }
  }
}

// ------------------------------------------------------------------------------------------------ host
static PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  if (!fn) {
    cudaDriverEntryPointQueryResult q;
    void* ptr = nullptr;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(ptr);
  }
  return fn;
}

// K-major bf16 matrix [rows, K] with row stride ld (elements) -> tensor map with box (box_rows x 64).
static int make_kmajor_map(CUtensorMap* map, const void* ptr, int64_t rows, int64_t K, int64_t ld, int box_rows) {
  auto fn = encode_fn();
  if (!fn) return fail("cuTensorMapEncodeTiled is unavailable from the CUDA driver");
  cuuint64_t dims[2] = {static_cast<cuuint64_t>(K), static_cast<cuuint64_t>(rows)};
  cuuint64_t strides[1] = {static_cast<cuuint64_t>(ld) * 2};
  cuuint32_t box[2] = {static_cast<cuuint32_t>(BK), static_cast<cuuint32_t>(box_rows)};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(ptr), dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail("cuTensorMapEncodeTiled failed with CUresult " + std::to_string(int(r)));
  return 0;
}

static int g_sm_budget[64] = {0};   // persistent-grid cap per device (0 = every SM)

static int sm_count() {
  static int n[64] = {0};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64) dev = 0;
  if (!n[dev]) cudaDeviceGetAttribute(&n[dev], cudaDevAttrMultiProcessorCount, dev);
  const int all = n[dev] > 0 ? n[dev] : 148;
  return g_sm_budget[dev] > 0 && g_sm_budget[dev] < all ? g_sm_budget[dev] : all;
}

int set_persistent_sms(int n) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return fail("no current CUDA device");
  if (n < 0) return fail("persistent SM budget must be >= 0");
  g_sm_budget[dev] = n;
  return 0;
}

bool supported(const void* A, int64_t lda, const void* B, int64_t ldb, int64_t K) {
  // TMA: base 16-byte aligned, row strides a multiple of 16 bytes.
  return ((reinterpret_cast<uintptr_t>(A) & 15) == 0) && ((reinterpret_cast<uintptr_t>(B) & 15) == 0) &&
         (lda % 8 == 0) && (ldb % 8 == 0) && K >= 8 && K % 8 == 0;
}

template <int EPI, bool THIN>
static int launch_t(const CUtensorMap& ma, const CUtensorMap& mb, const Params& p, int grid, cudaStream_t st) {
  static bool attr_set[64] = {false};
  constexpr int smem = THIN ? THIN_SMEM_BYTES : SMEM_BYTES;
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev >= 0 && dev < 64 && !attr_set[dev]) {
    if (cudaFuncSetAttribute(gemm_tc_kernel<EPI, THIN>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem) !=
        cudaSuccess)
      return check_launch("gemm_tc set smem");
    attr_set[dev] = true;
  }
  return launch_pdl("gemm_tc_kernel", gemm_tc_kernel<EPI, THIN>, dim3(grid), dim3(THREADS), smem, st, ma, mb, p);
}

template <int EPI>
static int launch_pair_t(const CUtensorMap& ma, const CUtensorMap& mb, const Params& p, int grid, cudaStream_t st) {
  static bool attr_set[64] = {false};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev >= 0 && dev < 64 && !attr_set[dev]) {
    if (cudaFuncSetAttribute(gemm_tc2_kernel<EPI>, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM2_BYTES) !=
        cudaSuccess)
      return check_launch("gemm_tc2 set smem");
    attr_set[dev] = true;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(static_cast<unsigned>(grid));
  cfg.blockDim = dim3(THREADS);
  cfg.dynamicSmemBytes = SMEM2_BYTES;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  const cudaError_t e = cudaLaunchKernelEx(&cfg, gemm_tc2_kernel<EPI>, ma, mb, p);
  if (e != cudaSuccess) return fail(std::string("gemm_tc2_kernel launch: ") + cudaGetErrorString(e));
  return check_launch("gemm_tc2_kernel");
}

// Tile counters of the 1-SM kernel, one pair per (device, stream): launches on one stream run one after another,
// and each leaves its counter at zero for the next.
static unsigned* sched_counter(cudaStream_t st) {
  static std::mutex mu;
  static std::map<std::pair<int, cudaStream_t>, unsigned*> counters;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) {
    fail("gemm: no current CUDA device");
    return nullptr;
  }
  std::lock_guard<std::mutex> lock(mu);
  const auto key = std::make_pair(dev, st);
  const auto it = counters.find(key);
  if (it != counters.end()) return it->second;
  unsigned* c = nullptr;
  if (cudaMalloc(&c, 2 * sizeof(unsigned)) != cudaSuccess ||
      cudaMemsetAsync(c, 0, 2 * sizeof(unsigned), st) != cudaSuccess) {
    fail("gemm: cannot set up the tile counter");
    return nullptr;
  }
  counters[key] = c;
  return c;
}

// Split-K partial sums, one growing buffer per (device, stream). An outgrown buffer is kept (not freed): a CUDA
// graph captured on that stream may still address it.
static float* splitk_workspace(cudaStream_t st, int64_t bytes) {
  static std::mutex mu;
  static std::map<std::pair<int, cudaStream_t>, std::pair<float*, int64_t>> bufs;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) {
    fail("gemm: no current CUDA device");
    return nullptr;
  }
  std::lock_guard<std::mutex> lock(mu);
  auto& b = bufs[std::make_pair(dev, st)];
  if (b.second < bytes) {
    b = {nullptr, 0};
    const int64_t want = (bytes + (int64_t(1) << 20) - 1) >> 20 << 20;
    if (cudaMalloc(&b.first, static_cast<size_t>(want)) != cudaSuccess) {
      b = {nullptr, 0};
      fail("gemm: cannot allocate the split-K workspace");
      return nullptr;
    }
    b.second = want;
  }
  return b.first;
}

template <int EPI>
static int launch_reduce_t(const Params& p, int64_t M, int64_t n_out, cudaStream_t st) {
  const bool vec = n_out % 4 == 0 && p.ldc % 4 == 0 && (reinterpret_cast<uintptr_t>(p.C) & 7) == 0 &&
                   (EPI != EPI_RESIDUAL || (p.ldr % 4 == 0 && (reinterpret_cast<uintptr_t>(p.R) & 7) == 0));
  if (vec && M <= 65535) {
    const dim3 grid(static_cast<unsigned>((n_out / 4 + 255) / 256), static_cast<unsigned>(M));
    return launch_pdl("splitk_reduce_vec_kernel", splitk_reduce_vec_kernel<EPI>, grid, dim3(256), 0, st,
                      static_cast<const float*>(p.ws), p.ldw, p.k_split, static_cast<int>(M), static_cast<int>(n_out),
                      p.C, p.ldc, static_cast<const __nv_bfloat16*>(p.R), p.ldr);
  }
  const int64_t total = M * n_out;
  int64_t blocks = (total + 255) / 256;
  if (blocks > 4 * sm_count()) blocks = 4 * sm_count();
  return launch_pdl("splitk_reduce_kernel", splitk_reduce_kernel<EPI>, dim3(static_cast<unsigned>(blocks)), dim3(256), 0,
                    st, static_cast<const float*>(p.ws), p.ldw, p.k_split, static_cast<int>(M),
                    static_cast<int>(n_out), p.C, p.ldc, static_cast<const __nv_bfloat16*>(p.R), p.ldr);
}

// K split of a GEMM with one m-block (M <= 128 rows: decode steps). Such a GEMM streams the weights once and is
// HBM-bound, and one CTA streams well below its share of HBM bandwidth (a 4-stage ring of 48 KB), so the split keeps
// every persistent CTA streaming: the smallest split whose units fill the waves of `sms` CTAs to at least 90 %
// (units / (waves x sms)), else the one that fills them best. FORGESERVE_DECODE_SPLIT=wave instead takes the smallest
// split that keeps 60 % of the CTAs busy in one wave (fewer fp32 partials; for comparisons). Chunks keep at least
// KB_MIN k-blocks (64 of K each). The split depends on the weight shape and the SM budget only, not on M: rows get
// the same sums whatever the batch (eager, graph-captured or micro-batched decode steps).
static bool split_one_wave() {
  static const bool w = [] {
    const char* v = std::getenv("FORGESERVE_DECODE_SPLIT");
    return v && std::string(v) == "wave";
  }();
  return w;
}

// M <= 64 runs the thin form of the 1-SM kernel (64-row A boxes, five stages) unless FORGESERVE_GEMM_THIN=0. Rows
// get the same sums either way: each output row is the same K-ordered MMA chain over the same weights.
// With one m-block every weight byte is read once: those loads carry the L2 evict-first policy (unless
// FORGESERVE_GEMM_L2HINT=0), so that the split-K partials written meanwhile stay in L2 for the reduce.
static bool l2_hint_enabled() {
  static const bool t = [] {
    const char* v = std::getenv("FORGESERVE_GEMM_L2HINT");
    return !(v && std::string(v) == "0");
  }();
  return t;
}

static bool thin_enabled() {
  static const bool t = [] {
    const char* v = std::getenv("FORGESERVE_GEMM_THIN");
    return !(v && std::string(v) == "0");
  }();
  return t;
}

int choose_k_split(int tiles, int k_blocks, int sms) {
  constexpr int KB_MIN = 6;
  if (sms <= 0 || tiles >= sms || k_blocks < 2 * KB_MIN) return 1;
  int best = 1;
  if (split_one_wave()) {
    for (int split = 1; split <= k_blocks / KB_MIN; ++split) {
      const int units = tiles * split;
      if (units > sms) break;
      best = split;
      if (units >= 0.6 * sms) break;
    }
    return best;
  }
  double best_fill = 0.0;
  for (int split = 1; split <= k_blocks / KB_MIN; ++split) {
    const int units = tiles * split;
    const int waves = (units + sms - 1) / sms;
    const double fill = static_cast<double>(units) / (static_cast<double>(waves) * sms);
    if (fill >= 0.9) return split;
    if (fill > best_fill + 1e-9) best = split, best_fill = fill;
  }
  return best;
}

static int g_pair_mode = 1;   // 1: use the 2-SM kernel for M > 128; 0: always the 1-SM kernel

int set_pair_mode(int on) {
  g_pair_mode = on ? 1 : 0;
  return 0;
}

int gemm_tc(const void* A, int64_t lda, const void* B, int64_t ldb, void* C, int64_t ldc, const void* R,
            int64_t ldr, int64_t M, int64_t N, int64_t K, int64_t n_out, int epi, bool sys_fence, cudaStream_t stream) {
  if (M <= 0 || N <= 0 || n_out <= 0) return 0;
  if (M > INT32_MAX / 2 || N > INT32_MAX / 2 || K > INT32_MAX / 2) return fail("gemm: dimension too large");
  const bool thin = M <= BM / 2 && thin_enabled();
  CUtensorMap ma, mb;
  if (make_kmajor_map(&ma, A, M, K, lda, thin ? BM / 2 : BM)) return -1;
  if (make_kmajor_map(&mb, B, N, K, ldb, BN / 2)) return -1;
  Params p;
  p.C = static_cast<__nv_bfloat16*>(C);
  p.R = static_cast<const __nv_bfloat16*>(R);
  p.ldc = ldc;
  p.ldr = ldr;
  p.M = static_cast<int>(M);
  p.n_out = static_cast<int>(n_out);
  p.num_m_blocks = static_cast<int>((M + BM - 1) / BM);
  const int n_tile = epi == EPI_SWIGLU ? BN / 2 : BN;  // output columns per tile
  const int num_n_blocks = static_cast<int>((n_out + n_tile - 1) / n_tile);
  p.num_tiles = p.num_m_blocks * num_n_blocks;
  p.k_blocks = static_cast<int>((K + BK * KP1 - 1) / (BK * KP1));   // k-blocks of the 1-SM kernel
  p.sys_fence = sys_fence ? 1 : 0;
  p.sched = nullptr;
  p.k_split = 1;
  p.ws = nullptr;
  p.ldw = 0;
  p.err = error_word();
  if (!p.err) return -1;
  p.b_once = 0;
  if (g_pair_mode && M > BM) {
    p.k_blocks = static_cast<int>((K + BK * KP - 1) / (BK * KP));   // k-blocks of 64 * KP
    p.sched = sched_counter(stream);
    if (!p.sched) return -1;
    const int num_m_pairs = (p.num_m_blocks + 1) / 2;
    p.num_tiles = num_m_pairs * num_n_blocks;
    const int pairs = p.num_tiles < sm_count() / 2 ? p.num_tiles : sm_count() / 2;
    switch (epi) {
      case EPI_STORE: return launch_pair_t<EPI_STORE>(ma, mb, p, 2 * pairs, stream);
      case EPI_RESIDUAL: return launch_pair_t<EPI_RESIDUAL>(ma, mb, p, 2 * pairs, stream);
      case EPI_SWIGLU: return launch_pair_t<EPI_SWIGLU>(ma, mb, p, 2 * pairs, stream);
      default: return fail("gemm: unknown epilogue");
    }
  }
  p.sched = sched_counter(stream);
  if (!p.sched) return -1;
  p.b_once = p.num_m_blocks == 1 && l2_hint_enabled() ? 1 : 0;
  const int sms = sm_count();
  // Few rows (a decode step): with one m-block there are few tiles, and the GEMM streams the weights; the time is
  // set by how evenly the SMs share them. Split K so that the units fill whole waves of the persistent grid.
  const int split = p.num_m_blocks == 1 && !sys_fence ? choose_k_split(p.num_tiles, p.k_blocks, sms) : 1;
  if (split >= 2) {
    const int64_t n_b = epi == EPI_SWIGLU ? 2 * n_out : n_out;
    p.ldw = (n_b + 3) / 4 * 4;
    p.ws = splitk_workspace(stream, static_cast<int64_t>(split) * M * p.ldw * static_cast<int64_t>(sizeof(float)));
    if (!p.ws) return -1;
    p.k_split = split;
  }
  const int units = p.num_tiles * p.k_split;
  const int grid = units < sms ? units : sms;
  int rc;
  switch (epi * 2 + (thin ? 1 : 0)) {
    case EPI_STORE * 2: rc = launch_t<EPI_STORE, false>(ma, mb, p, grid, stream); break;
    case EPI_RESIDUAL * 2: rc = launch_t<EPI_RESIDUAL, false>(ma, mb, p, grid, stream); break;
    case EPI_SWIGLU * 2: rc = launch_t<EPI_SWIGLU, false>(ma, mb, p, grid, stream); break;
    case EPI_STORE * 2 + 1: rc = launch_t<EPI_STORE, true>(ma, mb, p, grid, stream); break;
    case EPI_RESIDUAL * 2 + 1: rc = launch_t<EPI_RESIDUAL, true>(ma, mb, p, grid, stream); break;
    case EPI_SWIGLU * 2 + 1: rc = launch_t<EPI_SWIGLU, true>(ma, mb, p, grid, stream); break;
    default: return fail("gemm: unknown epilogue");
  }
  if (rc || p.k_split == 1) return rc;
  switch (epi) {
    case EPI_STORE: return launch_reduce_t<EPI_STORE>(p, M, n_out, stream);
    case EPI_RESIDUAL: return launch_reduce_t<EPI_RESIDUAL>(p, M, n_out, stream);
    default: return launch_reduce_t<EPI_SWIGLU>(p, M, n_out, stream);
  }
}

}  // namespace tcg
}  // namespace fs
