// Shared helpers for the forgeserve_b200 kernels (sm_100a only).
//
// * dtype handling: every kernel is templated on the activation type (float or __nv_bfloat16); arithmetic is
//   done in fp32 and rounded back to the activation type at exactly the points where the reference PyTorch
//   module rounds (forgeserve/model.py:29-31 RMSNorm, :40-45 RoPE, :92-93 SwiGLU, :104-106 residual adds).
// * error reporting: host entry points return an int status and leave a message in a thread-local buffer
//   (fs_last_error). Device code never traps; a kernel that meets bad input or a wait that runs out of time
//   ORs a code into the per-device error word, which the host reads with fs_device_error().
// * PTX wrappers for mbarrier, TMA (cp.async.bulk.tensor, never with .multicast::cluster) and tcgen05.
#pragma once

#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <cstdio>
#include <string>
#include <utility>

namespace fs {

enum DType : int { F32 = 0, BF16 = 1 };

// Device error bits (ORed into g_device_error).
enum DeviceError : unsigned {
  ERR_WAIT_TIMEOUT = 1u,      // an mbarrier wait exceeded its time limit; the kernel abandoned its work
  ERR_BAD_TOKEN = 2u,         // an embedding id outside [0, vocab)
  ERR_BAD_SLOT = 4u,          // a KV slot or block-table entry outside the cache
  ERR_BAD_POSITION = 8u,      // a position outside the RoPE table
};

// Per-device error word (allocated once per device on first use; never freed).
unsigned* error_word();

void set_last_error(const std::string& msg);
int fail(const std::string& msg);                     // set_last_error + return -1
int check_launch(const char* what);                   // cudaGetLastError -> status

// Programmatic dependent launch (PDL). A kernel launched with launch_pdl() may start while the kernel before it on
// the stream is still running: it must call pdl_wait() before its first access to any memory another kernel
// writes (every read or write of activations, caches, counters, workspaces; only weights may be read before), and
// it calls pdl_trigger() to let the kernel after it start early in turn. Launched without PDL, both are no-ops.
// A kernel that allocates TMEM triggers only after its allocation, so that a dependent never holds TMEM that a
// kernel it waits for still needs.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

bool pdl_enabled();   // FORGESERVE_PDL=0 turns programmatic launches off (for comparisons)

// Launches `kernel` on `st`, with programmatic stream serialization when pdl_enabled(); the kernel must follow the
// pdl_wait() rule above.
template <typename... KArgs, typename... Args>
int launch_pdl(const char* what, void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st,
               Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl_enabled() ? 1 : 0;
  const cudaError_t e = cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
  if (e != cudaSuccess) return fail(std::string(what) + " launch: " + cudaGetErrorString(e));
  return check_launch(what);
}

// The same launch where the caller checks it afterwards with check_launch() (a failed launch leaves its error for
// cudaGetLastError, as a <<<>>> launch does).
template <typename... KArgs, typename... Args>
void launch_pdl_async(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st, Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl_enabled() ? 1 : 0;
  (void)cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
}


template <typename T> struct TypeOf;
template <> struct TypeOf<float> { static constexpr int value = F32; };
template <> struct TypeOf<__nv_bfloat16> { static constexpr int value = BF16; };

__device__ __forceinline__ float to_f(float x) { return x; }
__device__ __forceinline__ float to_f(__nv_bfloat16 x) { return __bfloat162float(x); }
template <typename T> __device__ __forceinline__ T from_f(float x);
template <> __device__ __forceinline__ float from_f<float>(float x) { return x; }
template <> __device__ __forceinline__ __nv_bfloat16 from_f<__nv_bfloat16>(float x) { return __float2bfloat16_rn(x); }
// Round x to the activation type and back (identity for fp32).
template <typename T> __device__ __forceinline__ float rnd(float x) { return to_f(from_f<T>(x)); }

__device__ __forceinline__ void flag_error(unsigned* err, unsigned code) {
  if (err) atomicOr(err, code);
}

// 2-D bf16 tensor map with 128-byte swizzle and boxes of 64 columns x box_rows rows, over a row-major matrix of
// `rows` rows of `cols` elements at a stride of `ld` elements (defined in attention_tc.cu).
int make_bf16_map(CUtensorMap* map, const void* ptr, int64_t cols, int64_t rows, int64_t ld, int box_rows);

// ---------------------------------------------------------------------------------------------------------
// mbarrier / TMA / tcgen05 PTX wrappers
// ---------------------------------------------------------------------------------------------------------
__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count));
}

__device__ __forceinline__ void fence_barrier_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
               : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

__device__ __forceinline__ uint64_t globaltimer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
  return t;
}

// Wait time limit for every spin in this library: far above any legitimate wait (a whole GEMM tile is
// well under a millisecond), far below anything that would look like a hung GPU.
constexpr uint64_t kWaitLimitNs = 2000000000ull;  // 2 s

// Bounded wait on an mbarrier phase. Returns false (and flags ERR_WAIT_TIMEOUT) if the phase did not
// complete within limit_ns (kWaitLimitNs unless a caller passes a shorter limit, as the wait self-test does);
// callers then abandon their work and fall through to the kernel's clean-up.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, unsigned* err,
                                          uint64_t limit_ns = kWaitLimitNs) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = globaltimer_ns();
  uint32_t spins = 0;
  while (true) {
    if (mbar_try_wait(bar, parity)) return true;
    if ((++spins & 255u) == 0 && globaltimer_ns() - t0 > limit_ns) {
      flag_error(err, ERR_WAIT_TIMEOUT);
      return false;
    }
  }
}

// 2-D tiled TMA load (no multicast) into shared memory, completing on `bar` with byte accounting.
__device__ __forceinline__ void tma_load_2d(void* smem_dst, const CUtensorMap* map, uint64_t* bar, int x,
                                            int y) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4}], "
      "[%2];" ::"r"(smem_u32(smem_dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(x), "r"(y)
      : "memory");
}

// L2 policy for data read exactly once (a decode step's weights): its lines are the first evicted, so that what is
// read again soon (split-K partials, activations) stays in L2.
__device__ __forceinline__ uint64_t l2_policy_evict_first() {
  uint64_t pol;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(pol));
  return pol;
}

// tma_load_2d with an L2 cache policy from createpolicy.
__device__ __forceinline__ void tma_load_2d_hint(void* smem_dst, const CUtensorMap* map, uint64_t* bar, int x, int y,
                                                 uint64_t policy) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1, {%3, "
      "%4}], [%2], %5;" ::"r"(smem_u32(smem_dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(x), "r"(y), "l"(policy)
      : "memory");
}

__device__ __forceinline__ void prefetch_tmap(const CUtensorMap* map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}

// --- tcgen05 (5th generation tensor cores, tensor memory) ---
__device__ __forceinline__ void tmem_alloc(uint32_t* smem_slot, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(smem_slot)),
               "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void tmem_relinquish() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}
__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}
// D[tmem] (+)= A[smem] * B[smem]^T, kind::f16 (bf16 inputs, fp32 accumulate), issued by one thread.
__device__ __forceinline__ void tc_mma_f16(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                           uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}
// Arrive on `bar` once every tcgen05.mma issued so far by this thread has completed.
__device__ __forceinline__ void tc_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                   smem_u32(bar))
               : "memory");
}
__device__ __forceinline__ void tc_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }
// tcgen05.ld writes its registers asynchronously; they are valid after tcgen05.wait::ld. The compiler only sees
// the ld as their producer, so after the wait, pass them through an empty volatile asm: every later use then
// depends on an instruction that cannot move above the wait.
template <int N>
__device__ __forceinline__ void tmem_regs_ready(uint32_t (&r)[N]) {
#pragma unroll
  for (int i = 0; i < N; ++i) asm volatile("" : "+r"(r[i]));
}

// 32 lanes x 32 columns of 32-bit TMEM -> 32 registers per thread (thread i reads lane base+i).
__device__ __forceinline__ void tmem_ld_32x32b_x32(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
        "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]),
        "=r"(r[23]), "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]),
        "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
}

// Shared-memory matrix descriptor for tcgen05.mma, K-major operand staged by TMA with 128-byte swizzle:
// rows of 64 bf16 (128 B), 8-row swizzle atoms 1024 B apart (stride byte offset), version 1 (sm_100),
// layout type 2 = SWIZZLE_128B. The leading byte offset is unused for swizzled K-major layouts.
__device__ __forceinline__ uint64_t sw128_kmajor_desc(uint32_t smem_addr) {
  uint64_t d = 0;
  d |= static_cast<uint64_t>((smem_addr >> 4) & 0x3FFFu);        // start address  [0,14)
  d |= static_cast<uint64_t>(1u) << 16;                           // leading byte offset (unused) [16,30)
  d |= static_cast<uint64_t>(1024u >> 4) << 32;                   // stride byte offset [32,46)
  d |= static_cast<uint64_t>(1u) << 46;                           // version [46,48)
  d |= static_cast<uint64_t>(2u) << 61;                           // SWIZZLE_128B [61,64)
  return d;
}

// Instruction descriptor, kind::f16: fp32 accumulator, bf16 A and B, both K-major, shape M x N.
__host__ __device__ constexpr uint32_t idesc_bf16_f32(int M, int N) {
  return (1u << 4)                                   // D format F32
         | (1u << 7)                                 // A format BF16
         | (1u << 10)                                // B format BF16
         | (static_cast<uint32_t>(N >> 3) << 17)     // N / 8
         | (static_cast<uint32_t>(M >> 4) << 24);    // M / 16
}

}  // namespace fs
