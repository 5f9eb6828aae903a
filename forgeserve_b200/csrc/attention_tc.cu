// Prefill attention on the 5th-generation tensor cores (tcgen05 + TMEM + TMA), bf16, head_dim 64 or 128.
//
// Same semantics as attention.cu (forgeserve/model.py:69-76): GQA (query head h reads KV head h / rep), key slot s
// visible to a query at position p iff s <= p and s < n_slots, scale 1/sqrt(hd), output bf16.
//
// One CTA computes 128 queries of one head against the keys 0 .. min(n_slots, max position + 1) - 1, 64 keys per
// step; two CTAs share an SM (256 TMEM columns and ~97 KB of shared memory each), so one CTA's MMAs run during the
// other's softmax:
//   warp 4      TMA producer: the Q tile once; per step the K and V tiles, fetched in 16-key boxes through the
//               block table (a paged pool's blocks or a contiguous cache's one block per row), 2-stage rings
//   warp 5      MMA issuer (one thread): S_j = Q K_j^T into one of two TMEM buffers; O += P_{j-1} V_{j-1} with
//               P read from TMEM and V from shared memory (MN-major operand); S_j's buffer is released by the
//               commit that follows P_j V_j
//   warps 0-3   softmax, one thread per query row: S row from TMEM, causal mask, running max in the log2
//               domain, P = exp2(S - m) packed to bf16 over the first half of S_j's columns; O rescaled in TMEM
//               only when the running max grows by more than 2^8 (otherwise the stale max is kept, bounding P by
//               2^8); final O / l to global
// TMEM: S_0 [0,64) S_1 [64,128), P_j over the first half of S_j, O [128, 128+hd). Every wait is bounded (common.cuh).
// No TMA multicast (the kernel also runs in multi-GPU jobs).
#include <cudaTypedefs.h>

#include "common.cuh"
#include "kernels.h"

namespace fs {
namespace attn_tc {

constexpr int BM = 128, BN = 64, CHUNK = 16, K_STAGES = 2, V_STAGES = 2, THREADS = 192;
// TMEM: S_0 [0, 64), S_1 [64, 128); P_j (bf16 pairs, 32 columns) is written over the first half of S_j's own
// columns; O [128, 128 + hd). 256 columns, ~97 KB of shared memory: two CTAs share an SM.
constexpr int S_COL = 0, O_COL = 2 * BN, TMEM_COLS = 256;
constexpr float RESCALE_THRESHOLD = 8.0f;   // log2 units

template <int HD>
struct Geo {
  static constexpr int HALVES = HD / 64;                 // 64-column (128-byte) swizzle panels
  static constexpr int Q_PANEL = BM * 128;               // bytes of one 64-column panel of Q
  static constexpr int KV_PANEL = BN * 128;
  static constexpr int Q_BYTES = Q_PANEL * HALVES;
  static constexpr int KV_BYTES = KV_PANEL * HALVES;     // one K (or V) tile
  static constexpr int K_OFF = Q_BYTES;
  static constexpr int V_OFF = Q_BYTES + K_STAGES * KV_BYTES;
  static constexpr int BAR_OFF = V_OFF + V_STAGES * KV_BYTES;
  static constexpr int SMEM = BAR_OFF + 256 + 1024;      // + barriers + alignment slack
  static constexpr uint32_t IDESC_S = idesc_bf16_f32(BM, BN);
  static constexpr uint32_t IDESC_O = idesc_bf16_f32(BM, HD) | (1u << 16);  // B (= V) is MN-major
};

struct Params {
  const int64_t* positions;
  const int64_t* table;
  int64_t table_stride;
  int64_t n_slots;
  int64_t block_size;
  int64_t rows_per_block;   // block_stride / hd
  int64_t rows_per_head;    // head_stride / hd
  int64_t num_blocks;
  __nv_bfloat16* out;
  int64_t ldo;
  int T, nh, rep, n_qb;
  float scale_log2;
  unsigned* err;
};

__device__ __forceinline__ void mma_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc, uint32_t idesc,
                                       uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d_tmem),
      "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

__device__ __forceinline__ void tmem_st_32x32b_x16(uint32_t taddr, const uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], "
      "{%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]), "r"(r[9]),
      "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15])
      : "memory");
}
__device__ __forceinline__ void tmem_st_32x32b_x32(uint32_t taddr, const uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], "
      "{%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,"
      "%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]), "r"(r[9]),
      "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15]), "r"(r[16]), "r"(r[17]), "r"(r[18]),
      "r"(r[19]), "r"(r[20]), "r"(r[21]), "r"(r[22]), "r"(r[23]), "r"(r[24]), "r"(r[25]), "r"(r[26]), "r"(r[27]),
      "r"(r[28]), "r"(r[29]), "r"(r[30]), "r"(r[31])
      : "memory");
}
// 32 lanes x 64 columns of 32-bit TMEM -> 64 registers per thread (thread i reads lane base + i).
__device__ __forceinline__ void tmem_ld_32x32b_x64(uint32_t taddr, uint32_t (&r)[64]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x64.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32,%33,%34,%35,%36,%37,%38,%39,%40,%41,%42,%43,%44,%45,%46,%47,%48,%49,%50,%51,%52,%53,%54,%55,%56,%57,%58,%59,%60,%61,%62,%63}, [%64];"
      : "=r"(r[0]),"=r"(r[1]),"=r"(r[2]),"=r"(r[3]),"=r"(r[4]),"=r"(r[5]),"=r"(r[6]),"=r"(r[7]),"=r"(r[8]),"=r"(r[9]),"=r"(r[10]),"=r"(r[11]),"=r"(r[12]),"=r"(r[13]),"=r"(r[14]),"=r"(r[15]),"=r"(r[16]),"=r"(r[17]),"=r"(r[18]),"=r"(r[19]),"=r"(r[20]),"=r"(r[21]),"=r"(r[22]),"=r"(r[23]),"=r"(r[24]),"=r"(r[25]),"=r"(r[26]),"=r"(r[27]),"=r"(r[28]),"=r"(r[29]),"=r"(r[30]),"=r"(r[31]),"=r"(r[32]),"=r"(r[33]),"=r"(r[34]),"=r"(r[35]),"=r"(r[36]),"=r"(r[37]),"=r"(r[38]),"=r"(r[39]),"=r"(r[40]),"=r"(r[41]),"=r"(r[42]),"=r"(r[43]),"=r"(r[44]),"=r"(r[45]),"=r"(r[46]),"=r"(r[47]),"=r"(r[48]),"=r"(r[49]),"=r"(r[50]),"=r"(r[51]),"=r"(r[52]),"=r"(r[53]),"=r"(r[54]),"=r"(r[55]),"=r"(r[56]),"=r"(r[57]),"=r"(r[58]),"=r"(r[59]),"=r"(r[60]),"=r"(r[61]),"=r"(r[62]),"=r"(r[63])
      : "r"(taddr));
}
__device__ __forceinline__ void tc_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }
__device__ __forceinline__ void fence_async_smem() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

// MN-major operand with 128-byte swizzle: 64-element MN panels `panel_bytes` apart (leading byte offset), 8-row
// K groups 1024 bytes apart (stride byte offset).
__device__ __forceinline__ uint64_t sw128_mnmajor_desc(uint32_t smem_addr, uint32_t panel_bytes) {
  uint64_t d = 0;
  d |= static_cast<uint64_t>((smem_addr >> 4) & 0x3FFFu);
  d |= static_cast<uint64_t>((panel_bytes >> 4) & 0x3FFFu) << 16;
  d |= static_cast<uint64_t>(1024u >> 4) << 32;
  d |= static_cast<uint64_t>(1u) << 46;
  d |= static_cast<uint64_t>(2u) << 61;
  return d;
}

// 2^x by the MUFU instruction (ex2.approx, flushes subnormal results to zero); x <= 8 here.
__device__ __forceinline__ float exp2_approx(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

__device__ __forceinline__ uint32_t pack_bf16x2(float lo, float hi) {
  __nv_bfloat162 h = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&h);
}

template <int HD>
__global__ void __launch_bounds__(THREADS, 2)
    attn_tc_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                   const __grid_constant__ CUtensorMap tmV, const __grid_constant__ CUtensorMap tmK128,
                   const __grid_constant__ CUtensorMap tmV128, Params p) {
  using G = Geo<HD>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + G::BAR_OFF);
  uint64_t* q_full = bars + 0;
  uint64_t* k_full = bars + 1;       // [K_STAGES]
  uint64_t* k_empty = bars + 4;      // [K_STAGES]
  uint64_t* v_full = bars + 7;       // [V_STAGES]
  uint64_t* v_empty = bars + 9;      // [V_STAGES]
  uint64_t* s_full = bars + 11;      // [2]
  uint64_t* s_empty = bars + 13;     // [2]
  uint64_t* p_full = bars + 15;
  uint64_t* pv_done = bars + 16;
  uint64_t* o_full = bars + 17;
  uint64_t* mma_done = bars + 18;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 19);
  int* s_ntiles = reinterpret_cast<int*>(bars + 20);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(bars + 21);
  __shared__ int64_t s_maxpos[4];

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int qb = p.n_qb - 1 - static_cast<int>(blockIdx.x);   // heaviest (latest) query blocks first
  const int h = blockIdx.y, r = blockIdx.z;
  const int g = h / p.rep;
  const int j0 = qb * BM;
  const int64_t tok0 = static_cast<int64_t>(r) * p.T;
  const int valid_rows = p.T - j0 < BM ? p.T - j0 : BM;

  // ---- setup: barriers, TMEM, the key range of this CTA (max position of its rows)
  int64_t my_pos = 0;
  if (warp < 4) {
    const int row = warp * 32 + lane;
    my_pos = row < valid_rows ? p.positions[tok0 + j0 + row] : 0;
    if (my_pos < 0) my_pos = 0;
    int64_t m = my_pos;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const int64_t w = __shfl_xor_sync(0xffffffffu, m, o);
      m = w > m ? w : m;
    }
    if (lane == 0) s_maxpos[warp] = m;
  }
  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    for (int s = 0; s < K_STAGES; ++s) {
      mbar_init(&k_full[s], 1);
      mbar_init(&k_empty[s], 1);
    }
    for (int s = 0; s < V_STAGES; ++s) {
      mbar_init(&v_full[s], 1);
      mbar_init(&v_empty[s], 1);
    }
    for (int s = 0; s < 2; ++s) {
      mbar_init(&s_full[s], 1);
      mbar_init(&s_empty[s], 1);   // released by the commit after P_j V_j, which reads P_j from S_j's columns
    }
    mbar_init(p_full, BM);
    mbar_init(pv_done, 1);
    mbar_init(o_full, 1);
    mbar_init(mma_done, 1);
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 4) {
    tmem_alloc(tmem_slot, TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (threadIdx.x == 0) {
    int64_t mp = s_maxpos[0];
    for (int i = 1; i < 4; ++i) mp = s_maxpos[i] > mp ? s_maxpos[i] : mp;
    int64_t n_keys = mp + 1 < p.n_slots ? mp + 1 : p.n_slots;
    if (n_keys < 1) n_keys = 1;
    s_ntiles[0] = static_cast<int>((n_keys + BN - 1) / BN);
    s_ntiles[1] = static_cast<int>(n_keys);
  }
  __syncthreads();
  const uint32_t tmem = *tmem_slot;
  const int n_tiles = s_ntiles[0];
  const int n_keys = s_ntiles[1];

  if (warp == 4) {
    // ------------------------------------------------------------------------------------------ producer
    if (lane == 0) {
      prefetch_tmap(&tmQ);
      prefetch_tmap(&tmK);
      prefetch_tmap(&tmV);
      prefetch_tmap(&tmK128);
      prefetch_tmap(&tmV128);
      mbar_arrive_expect_tx(q_full, G::Q_BYTES);
      for (int hf = 0; hf < G::HALVES; ++hf)
        tma_load_2d(smem + hf * G::Q_PANEL, &tmQ, q_full, h * HD + 64 * hf, static_cast<int>(tok0 + j0));
      for (int j = 0; j < n_tiles; ++j) {
        const int ks = j % K_STAGES, vs = j % V_STAGES;
        const int key0 = j * BN;
        const int rem = n_keys - key0;
        const int nch = rem >= BN ? BN / CHUNK : (rem + CHUNK - 1) / CHUNK;
        // Block numbers of the tile's 16-key chunks, all loaded before any copy is issued (the copies are
        // compiler barriers: a lookup placed between them would be one full memory round trip each).
        const bool one_block = (key0 % p.block_size) + BN <= p.block_size;
        int64_t blk[BN / CHUNK];
#pragma unroll
        for (int c = 0; c < BN / CHUNK; ++c) {
          const int64_t s0 = key0 + c * CHUNK;
          blk[c] = (c < nch && (c == 0 || !one_block)) ? p.table[static_cast<int64_t>(r) * p.table_stride + s0 / p.block_size]
                                                      : 0;
        }
#pragma unroll
        for (int c = 0; c < BN / CHUNK; ++c)
          if (blk[c] < 0 || blk[c] >= p.num_blocks) {
            if (c < nch) flag_error(p.err, ERR_BAD_SLOT);
            blk[c] = 0;
          }
        const uint32_t bytes = one_block ? BN * 128 * G::HALVES : nch * CHUNK * 128 * G::HALVES;
        for (int which = 0; which < 2; ++which) {   // K then V, each into its own ring
          uint64_t* full = which == 0 ? &k_full[ks] : &v_full[vs];
          uint64_t* empty = which == 0 ? &k_empty[ks] : &v_empty[vs];
          const int nst = which == 0 ? K_STAGES : V_STAGES;
          if (!mbar_wait(empty, ((j / nst) & 1) ^ 1, p.err) || *abort_flag) {
            *abort_flag = 1;
            break;
          }
          uint8_t* dst = smem + (which == 0 ? G::K_OFF + ks * G::KV_BYTES : G::V_OFF + vs * G::KV_BYTES);
          const CUtensorMap* map16 = which == 0 ? &tmK : &tmV;
          const CUtensorMap* map128 = which == 0 ? &tmK128 : &tmV128;
          mbar_arrive_expect_tx(full, bytes);
          if (one_block) {
            // the whole tile lies in one block (a contiguous cache): one 128-row box per panel
            const int row = static_cast<int>(blk[0] * p.rows_per_block + g * p.rows_per_head + key0 % p.block_size);
            for (int hf = 0; hf < G::HALVES; ++hf) tma_load_2d(dst + hf * G::KV_PANEL, map128, full, 64 * hf, row);
          } else {
            for (int c = 0; c < nch; ++c) {
              const int64_t s0 = key0 + c * CHUNK;
              const int row = static_cast<int>(blk[c] * p.rows_per_block + g * p.rows_per_head + s0 % p.block_size);
              for (int hf = 0; hf < G::HALVES; ++hf)
                tma_load_2d(dst + hf * G::KV_PANEL + c * CHUNK * 128, map16, full, 64 * hf, row);
            }
          }
        }
        if (*abort_flag) break;
      }
    }
  } else if (warp == 5) {
    // ------------------------------------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      const uint32_t q_addr = smem_u32(smem);
      bool ok = mbar_wait(q_full, 0, p.err);
      // S_j = Q K_j^T into TMEM buffer j & 1; frees K stage j once the MMAs have read it
      auto issue_s = [&](int j) -> bool {
        const int ks = j % K_STAGES;
        if (!mbar_wait(&k_full[ks], (j / K_STAGES) & 1, p.err) ||
            !mbar_wait(&s_empty[j & 1], ((j >> 1) & 1) ^ 1, p.err) || *abort_flag)
          return false;
        tc_fence_after();
        const uint32_t k_addr = smem_u32(smem + G::K_OFF + ks * G::KV_BYTES);
#pragma unroll
        for (int kk = 0; kk < HD / 16; ++kk) {
          const int hf = kk / 4, kq = kk % 4;
          const uint64_t adesc = sw128_kmajor_desc(q_addr + hf * G::Q_PANEL) + 2u * kq;
          const uint64_t bdesc = sw128_kmajor_desc(k_addr + hf * G::KV_PANEL) + 2u * kq;
          tc_mma_f16(tmem + S_COL + (j & 1) * BN, adesc, bdesc, G::IDESC_S, kk != 0);
        }
        tc_commit(&s_full[j & 1]);
        tc_commit(&k_empty[ks]);
        return true;
      };
      // O += P_j V_j (P from TMEM); frees V stage j
      auto issue_pv = [&](int j) -> bool {
        const int vs = j % V_STAGES;
        if (!mbar_wait(&v_full[vs], (j / V_STAGES) & 1, p.err) || !mbar_wait(p_full, j & 1, p.err) || *abort_flag)
          return false;
        tc_fence_after();
        const uint32_t v_addr = smem_u32(smem + G::V_OFF + vs * G::KV_BYTES);
#pragma unroll
        for (int kk = 0; kk < BN / 16; ++kk) {
          const uint64_t bdesc = sw128_mnmajor_desc(v_addr + kk * 2048u, G::KV_PANEL);
          mma_ts(tmem + O_COL, tmem + S_COL + (j & 1) * BN + kk * 8, bdesc, G::IDESC_O, (j | kk) != 0);
        }
        tc_commit(pv_done);
        tc_commit(&v_empty[vs]);
        tc_commit(&s_empty[j & 1]);   // S_j's columns (P_j) are free once P_j V_j has completed
        return true;
      };
      if (ok) ok = issue_s(0);
      for (int j = 0; j < n_tiles && ok; ++j) {
        if (j + 1 < n_tiles) ok = issue_s(j + 1);   // the next scores overlap this tile's softmax
        if (ok) ok = issue_pv(j);
      }
      if (ok) tc_commit(o_full);
      if (!ok) *abort_flag = 1;
      tc_commit(mma_done);
    }
  } else {
    // ------------------------------------------------------------------------------------------ softmax
    // One thread per query row. S_j is read from TMEM twice, 32 columns at a time (pass 1: row max; pass 2:
    // P = exp2(S * scale - m), stored to P buffer j & 1 chunk by chunk), so the loops stay rolled and short and
    // the max and the sum run in four independent chains each.
    const int row = warp * 32 + lane;
    const uint32_t lane_base = static_cast<uint32_t>(warp * 32) << 16;
    const int64_t last_vis = my_pos < p.n_slots - 1 ? my_pos : p.n_slots - 1;
    float m_ref = -INFINITY, l = 0.f;
    bool ok = true;
    for (int j = 0; j < n_tiles; ++j) {
      const int sb = j & 1;
      ok = __all_sync(0xffffffffu, mbar_wait(&s_full[sb], (j >> 1) & 1, p.err));
      if (!ok) break;
      tc_fence_after();
      const int64_t key0 = static_cast<int64_t>(j) * BN;
      const bool whole = key0 + BN - 1 <= last_vis;   // every key of the tile is visible to this row
      const uint32_t s_addr = tmem + lane_base + S_COL + sb * BN;
      static_assert(BN == 64, "the softmax holds one 64-column S row in registers");
      uint32_t t[BN];   // the row's scores: one TMEM load serves both passes
      tmem_ld_32x32b_x64(s_addr, t);
      tc_wait_ld();
      tmem_regs_ready(t);
      if (!whole) {
#pragma unroll
        for (int i = 0; i < BN; ++i)
          if (key0 + i > last_vis) t[i] = __float_as_uint(-INFINITY);
      }
      float m4[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
#pragma unroll
      for (int i = 0; i < BN; ++i) m4[i & 3] = fmaxf(m4[i & 3], __uint_as_float(t[i]));
      const float mx = fmaxf(fmaxf(m4[0], m4[1]), fmaxf(m4[2], m4[3])) * p.scale_log2;   // log2 domain
      const float m_new = fmaxf(m_ref, mx);
      // Whether a row moves its reference max is decided per row, but the TMEM accesses that rescale O are
      // .sync.aligned warp instructions: the warp takes the rescale path if any of its rows needs it, and rows that
      // do not need it multiply by 1.
      const bool need = m_ref == -INFINITY || m_new > m_ref + RESCALE_THRESHOLD;
      const float corr = (need && m_ref != -INFINITY) ? exp2_approx(m_ref - m_new) : 1.f;
      if (need) m_ref = m_new;
      const float sub = m_ref == -INFINITY ? 0.f : m_ref;
      // P (bf16 pairs, 32 columns) over the first half of S_j's columns: the whole row is in registers already
      float s4[4] = {0.f, 0.f, 0.f, 0.f};
      uint32_t pk[BN / 2];
#pragma unroll
      for (int i = 0; i < BN / 2; ++i) {
        const float p0 = exp2_approx(fmaf(__uint_as_float(t[2 * i]), p.scale_log2, -sub));
        const float p1 = exp2_approx(fmaf(__uint_as_float(t[2 * i + 1]), p.scale_log2, -sub));
        s4[i & 3] += p0 + p1;
        pk[i] = pack_bf16x2(p0, p1);
      }
      tmem_st_32x32b_x32(s_addr, pk);
      tc_wait_st();
      l = l * corr + ((s4[0] + s4[1]) + (s4[2] + s4[3]));
      if (j >= 1) {
        // P V_{j-1} has completed (waited for in order, tile by tile, so the barrier's phase is never ambiguous)
        // before O is rescaled and before P V_j may start.
        ok = __all_sync(0xffffffffu, mbar_wait(pv_done, (j - 1) & 1, p.err));
        if (!ok) break;
        tc_fence_after();
        if (__any_sync(0xffffffffu, corr != 1.f)) {
#pragma unroll 1
          for (int c = 0; c < HD / 32; ++c) {
            uint32_t t[32];
            const uint32_t addr = tmem + lane_base + O_COL + c * 32;
            tmem_ld_32x32b_x32(addr, t);
            tc_wait_ld();
            tmem_regs_ready(t);
#pragma unroll
            for (int i = 0; i < 32; ++i) t[i] = __float_as_uint(__uint_as_float(t[i]) * corr);
            tmem_st_32x32b_x32(addr, t);
          }
          tc_wait_st();
        }
      }
      if (key0 + BN > n_keys) {                    // the tile with the last key: same for every row
        // V rows past the last key hold stale data; P is 0 there but 0 * NaN is not, so zero them. V_j is waited
        // for first (softmax j follows S_j, which only waited for K_j).
        ok = __all_sync(0xffffffffu, mbar_wait(&v_full[j % V_STAGES], (j / V_STAGES) & 1, p.err));
        if (!ok) break;
        if (row < BN && key0 + row >= n_keys) {
          uint4* vrow = reinterpret_cast<uint4*>(smem + G::V_OFF + (j % V_STAGES) * G::KV_BYTES + row * 128);
#pragma unroll
          for (int hf = 0; hf < G::HALVES; ++hf)
#pragma unroll
            for (int i = 0; i < 8; ++i) vrow[hf * (G::KV_PANEL / 16) + i] = make_uint4(0, 0, 0, 0);
          fence_async_smem();
        }
      }
      tc_fence_before();
      mbar_arrive(p_full);
    }
    if (ok && n_tiles > 0) ok = __all_sync(0xffffffffu, mbar_wait(o_full, 0, p.err));
    if (ok) {
      tc_fence_after();
      const float inv = l > 0.f ? 1.f / l : 0.f;
      __nv_bfloat16* orow = p.out + (tok0 + j0 + row) * p.ldo + static_cast<int64_t>(h) * HD;
#pragma unroll 1
      for (int c = 0; c < HD / 32; ++c) {
        uint32_t t[32];
        tmem_ld_32x32b_x32(tmem + lane_base + O_COL + c * 32, t);
        tc_wait_ld();
        tmem_regs_ready(t);
        if (row < valid_rows) {
          uint4* dst = reinterpret_cast<uint4*>(orow + c * 32);
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            uint4 w;
            w.x = pack_bf16x2(__uint_as_float(t[8 * i + 0]) * inv, __uint_as_float(t[8 * i + 1]) * inv);
            w.y = pack_bf16x2(__uint_as_float(t[8 * i + 2]) * inv, __uint_as_float(t[8 * i + 3]) * inv);
            w.z = pack_bf16x2(__uint_as_float(t[8 * i + 4]) * inv, __uint_as_float(t[8 * i + 5]) * inv);
            w.w = pack_bf16x2(__uint_as_float(t[8 * i + 6]) * inv, __uint_as_float(t[8 * i + 7]) * inv);
            dst[i] = w;
          }
        }
      }
    } else {
      *abort_flag = 1;
    }
  }

  __syncthreads();
  if (warp == 4) {
    mbar_wait(mma_done, 0, p.err);   // every MMA has completed before TMEM is released
    tc_fence_after();
    tmem_dealloc(tmem, TMEM_COLS);
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

static int make_map(CUtensorMap* map, const void* ptr, int64_t cols, int64_t rows, int64_t ld, int box_rows) {
  auto fn = encode_fn();
  if (!fn) return fail("cuTensorMapEncodeTiled is unavailable from the CUDA driver");
  cuuint64_t dims[2] = {static_cast<cuuint64_t>(cols), static_cast<cuuint64_t>(rows)};
  cuuint64_t strides[1] = {static_cast<cuuint64_t>(ld) * 2};
  cuuint32_t box[2] = {64, static_cast<cuuint32_t>(box_rows)};
  cuuint32_t estr[2] = {1, 1};
  CUresult res = fn(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(ptr), dims, strides, box, estr,
                    CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                    CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (res != CUDA_SUCCESS) return fail("cuTensorMapEncodeTiled failed with CUresult " + std::to_string(int(res)));
  return 0;
}

bool supported(const void* q, int64_t ldq, const KVCache& kv, int64_t hd, int64_t T) {
  if (hd != 64 && hd != 128) return false;
  if (T < 1 || kv.block_size % CHUNK != 0) return false;
  if (kv.block_stride % hd != 0 || kv.head_stride % hd != 0 || kv.head_stride / hd < kv.block_size) return false;
  if (ldq % 8 != 0) return false;
  const uintptr_t a = reinterpret_cast<uintptr_t>(q) | reinterpret_cast<uintptr_t>(kv.k) | reinterpret_cast<uintptr_t>(kv.v);
  if (a & 15) return false;
  const int64_t rows = kv.num_blocks * (kv.block_stride / hd);
  return rows < (int64_t(1) << 31);
}

template <int HD>
static int launch_t(const void* q, int64_t ldq, const KVCache& kv, int64_t n_slots, const int64_t* positions, void* out,
                    int64_t ldo, int64_t B, int64_t T, int64_t nh, int64_t nkv, float scale, cudaStream_t st) {
  using G = Geo<HD>;
  CUtensorMap mq, mk, mv;
  const int64_t q_rows = B * T;
  if (make_map(&mq, q, ldq, q_rows, ldq, BM)) return -1;
  const int64_t kv_rows = kv.num_blocks * (kv.block_stride / HD);
  CUtensorMap mk128, mv128;
  if (make_map(&mk, kv.k, HD, kv_rows, HD, CHUNK)) return -1;
  if (make_map(&mv, kv.v, HD, kv_rows, HD, CHUNK)) return -1;
  if (make_map(&mk128, kv.k, HD, kv_rows, HD, BN)) return -1;
  if (make_map(&mv128, kv.v, HD, kv_rows, HD, BN)) return -1;
  Params p;
  p.positions = positions;
  p.table = kv.table;
  p.table_stride = kv.table_stride;
  p.n_slots = n_slots;
  p.block_size = kv.block_size;
  p.rows_per_block = kv.block_stride / HD;
  p.rows_per_head = kv.head_stride / HD;
  p.num_blocks = kv.num_blocks;
  p.out = static_cast<__nv_bfloat16*>(out);
  p.ldo = ldo;
  p.T = static_cast<int>(T);
  p.nh = static_cast<int>(nh);
  p.rep = static_cast<int>(nh / nkv);
  p.n_qb = static_cast<int>((T + BM - 1) / BM);
  p.scale_log2 = scale * 1.4426950408889634f;
  p.err = error_word();
  if (!p.err) return -1;
  static bool attr[64] = {false};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev >= 0 && dev < 64 && !attr[dev]) {
    if (cudaFuncSetAttribute(attn_tc_kernel<HD>, cudaFuncAttributeMaxDynamicSharedMemorySize, G::SMEM) != cudaSuccess)
      return check_launch("attn_tc set smem");
    attr[dev] = true;
  }
  dim3 grid(static_cast<unsigned>(p.n_qb), static_cast<unsigned>(nh), static_cast<unsigned>(B));
  attn_tc_kernel<HD><<<grid, THREADS, G::SMEM, st>>>(mq, mk, mv, mk128, mv128, p);
  return check_launch("attn_tc_kernel");
}

int launch(const void* q, int64_t ldq, const KVCache& kv, int64_t n_slots, const int64_t* positions, void* out,
           int64_t ldo, int64_t B, int64_t T, int64_t nh, int64_t nkv, int64_t hd, float scale, cudaStream_t st) {
  if (B > 65535 || nh > 65535) return fail("attention: grid too large");
  if (hd == 128) return launch_t<128>(q, ldq, kv, n_slots, positions, out, ldo, B, T, nh, nkv, scale, st);
  if (hd == 64) return launch_t<64>(q, ldq, kv, n_slots, positions, out, ldo, B, T, nh, nkv, scale, st);
  return fail("attention (tcgen05): head_dim must be 64 or 128");
}

}  // namespace attn_tc

int make_bf16_map(CUtensorMap* map, const void* ptr, int64_t cols, int64_t rows, int64_t ld, int box_rows) {
  return attn_tc::make_map(map, ptr, cols, rows, ld, box_rows);
}

}  // namespace fs
