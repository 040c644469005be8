// Shared device helpers for the sm_100a kernels: vector types, reductions, and thin inline-PTX
// wrappers for mbarriers, TMA (cp.async.bulk.tensor) and the 5th-generation tensor core
// (tcgen05: TMEM alloc / mma / commit / ld). Every spin-wait is bounded: on timeout it records
// an error code in `minisgl_error_word` and returns false so the caller can unwind.
#pragma once
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>
#include <stdlib.h>

#include <atomic>
#include <mutex>
#include <utility>

#define MSGL_DEVICE __device__ __forceinline__

namespace msgl {

// Error codes written to the device error word (read by the host after a step).
enum : int {
  kErrNone = 0,
  kErrMbarTimeout = 1,
  kErrPeerTimeout = 2,
  kErrBounds = 3,
};

// Device error word, one copy per translation unit (no relocatable device code). Each .cu file
// exposes a read-and-clear accessor through MSGL_ERROR_ACCESSOR; msgl_get_error polls them all.
static __device__ int minisgl_error_word = 0;
static __device__ int minisgl_error_info = 0;

MSGL_DEVICE void report_error(int code, int info) {
  if (atomicCAS(&minisgl_error_word, 0, code) == 0) minisgl_error_info = info;
}

// Index checks of the bounds-check build (compiled with -DMINISGL_BOUNDS_CHECK=1, loaded when
// MINISGL_BOUNDS_CHECK=1): a failed check records kErrBounds with the site below as its info and
// evaluates to false, and the caller skips the access instead of faulting (no trap, no device
// assert). In the release build the macro is the constant true and the checks compile away.
enum : int {
  kBcEmbeddingId = 1,   // token id outside the vocabulary (unmasked embedding)
  kBcKvSlot = 2,        // KV-cache slot outside [0, num_slots) in a cache store
  kBcRopePos = 3,       // position outside the cos/sin table
  kBcAttnRow = 4,       // page-table row or kv length outside the page table
  kBcAttnSlot = 5,      // page-table entry outside [0, num_slots) in an attention read
  kBcMoePerm = 6,       // MoE gather index outside the token rows
  kBcMoeInv = 7,        // MoE combine index outside the expert-output rows
};
#if defined(MINISGL_BOUNDS_CHECK) && MINISGL_BOUNDS_CHECK
#define MSGL_IN_BOUNDS(cond, site) ((cond) ? true : (::msgl::report_error(::msgl::kErrBounds, (site)), false))
#else
#define MSGL_IN_BOUNDS(cond, site) true
#endif

// ------------------------------------------------------------------------------------------
// scalar / vector helpers
struct alignas(16) bf16x8 {
  __nv_bfloat162 v[4];
};

MSGL_DEVICE float warp_sum(float x) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) x += __shfl_xor_sync(0xffffffffu, x, o);
  return x;
}

MSGL_DEVICE float warp_max(float x) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) x = fmaxf(x, __shfl_xor_sync(0xffffffffu, x, o));
  return x;
}

// Block-wide sum; `red` must hold >= 32 floats. All threads get the result.
MSGL_DEVICE float block_sum(float x, float* red) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int nwarps = (blockDim.x + 31) >> 5;
  x = warp_sum(x);
  __syncthreads();
  if (lane == 0) red[warp] = x;
  __syncthreads();
  float y = lane < nwarps ? red[lane] : 0.f;
  return warp_sum(y);
}

MSGL_DEVICE uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

MSGL_DEVICE bool elect_one() {
  uint32_t pred = 0;
  asm volatile(
      "{\n\t.reg .pred P;\n\t"
      "elect.sync _|P, 0xffffffff;\n\t"
      "selp.b32 %0, 1, 0, P;\n\t}"
      : "=r"(pred));
  return pred != 0;
}

// ------------------------------------------------------------------------------------------
// mbarrier
MSGL_DEVICE void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count));
}

MSGL_DEVICE void fence_barrier_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

MSGL_DEVICE void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

MSGL_DEVICE void mbar_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)),
               "r"(bytes)
               : "memory");
}

MSGL_DEVICE bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred P;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 P, [%1], %2;\n\t"
      "selp.b32 %0, 1, 0, P;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// Non-blocking probe: has the phase with this parity completed?
MSGL_DEVICE bool mbar_test(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred P;\n\t"
      "mbarrier.test_wait.parity.shared::cta.b64 P, [%1], %2;\n\t"
      "selp.b32 %0, 1, 0, P;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

MSGL_DEVICE uint64_t globaltimer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
  return t;
}

// Upper bound of any single intra-kernel wait. Nothing legitimate waits this long; on expiry
// the kernel records kErrMbarTimeout and unwinds instead of hanging the GPU.
constexpr uint64_t kWaitTimeoutNs = 4000000000ull;

MSGL_DEVICE bool mbar_wait(uint64_t* bar, uint32_t parity, int where = 0) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = globaltimer_ns();
  while (!mbar_try_wait(bar, parity)) {
    if (globaltimer_ns() - t0 > kWaitTimeoutNs) {
      report_error(kErrMbarTimeout, where);
      return false;
    }
  }
  return true;
}

// ------------------------------------------------------------------------------------------
// TMA (tiled bulk tensor copies, no multicast)
MSGL_DEVICE void tma_load_2d(void* smem_dst, const CUtensorMap* map, uint64_t* bar, int x, int y) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4}], [%2];" ::"r"(smem_u32(smem_dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(x), "r"(y)
      : "memory");
}

MSGL_DEVICE void tma_load_3d(void* smem_dst, const CUtensorMap* map, uint64_t* bar, int x, int y, int z) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4, %5}], [%2];" ::"r"(smem_u32(smem_dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(x), "r"(y), "r"(z)
      : "memory");
}

// smem -> global tiled store (bulk group); bounds outside the tensor are clipped by hardware
MSGL_DEVICE void tma_store_2d(const CUtensorMap* map, const void* smem_src, int x, int y) {
  asm volatile(
      "cp.async.bulk.tensor.2d.global.shared::cta.bulk_group [%0, {%2, %3}], [%1];" ::"l"(
          reinterpret_cast<uint64_t>(map)),
      "r"(smem_u32(smem_src)), "r"(x), "r"(y)
      : "memory");
}
MSGL_DEVICE void bulk_commit() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }
template <int N>
MSGL_DEVICE void bulk_wait_read() { asm volatile("cp.async.bulk.wait_group.read %0;" ::"n"(N) : "memory"); }
template <int N>
MSGL_DEVICE void bulk_wait() { asm volatile("cp.async.bulk.wait_group %0;" ::"n"(N) : "memory"); }
MSGL_DEVICE void fence_async_smem() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

MSGL_DEVICE void red_add_v4(float* addr, float a, float b, float c, float d) {
  asm volatile("red.global.add.v4.f32 [%0], {%1, %2, %3, %4};" ::"l"(addr), "f"(a), "f"(b), "f"(c), "f"(d)
               : "memory");
}

// ---- 2-SM (cta_group::2) tensor-core helpers: a CTA pair shares one MMA of M = 256
MSGL_DEVICE void tmem_alloc_2sm(uint32_t* dst_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(dst_smem)),
               "r"(ncols));
}
MSGL_DEVICE void tmem_relinquish_2sm() { asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;"); }
MSGL_DEVICE void tmem_dealloc_2sm(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols));
}
MSGL_DEVICE void tc_mma_f16_2sm(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate));
}
// arrive (once all prior MMAs of this thread complete) on the barrier at this smem offset in every
// CTA of `cta_mask`
MSGL_DEVICE void tc_commit_2sm_mc(uint64_t* bar, uint16_t cta_mask) {
  asm volatile(
      "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64 [%0], %1;" ::"r"(
          smem_u32(bar)),
      "h"(cta_mask)
      : "memory");
}
// TMA tile load into this CTA's smem whose completion is counted on `bar_cluster_addr` (the pair
// leader's barrier, a shared::cluster address). No multicast.
MSGL_DEVICE void tma_load_2d_2sm(void* smem_dst, const CUtensorMap* map, uint32_t bar_cluster_addr, int x, int y) {
  asm volatile(
      "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4}], [%2];" ::"r"(smem_u32(smem_dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(bar_cluster_addr), "r"(x), "r"(y)
      : "memory");
}
MSGL_DEVICE void tma_load_3d_2sm(void* smem_dst, const CUtensorMap* map, uint32_t bar_cluster_addr, int x, int y,
                                 int z) {
  asm volatile(
      "cp.async.bulk.tensor.3d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4, %5}], [%2];" ::"r"(smem_u32(smem_dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(bar_cluster_addr), "r"(x), "r"(y), "r"(z)
      : "memory");
}
MSGL_DEVICE void mbar_arrive_cluster(uint32_t bar_cluster_addr) {
  asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(bar_cluster_addr) : "memory");
}

// ---- thread-block clusters / distributed shared memory
MSGL_DEVICE uint32_t cluster_ctarank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %cluster_ctarank;" : "=r"(r));
  return r;
}
MSGL_DEVICE void cluster_sync() {
  // non-.aligned form: warps whose lanes took different roles may arrive divergently
  asm volatile("barrier.cluster.arrive.release;\n\tbarrier.cluster.wait.acquire;" ::: "memory");
}
// address of the same smem variable in CTA `rank` of this cluster
MSGL_DEVICE uint32_t dsmem_addr(uint32_t local_smem_addr, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(local_smem_addr), "r"(rank));
  return r;
}
// fire-and-forget 16-byte store into another cluster CTA's smem; completion is counted (in bytes)
// on that CTA's mbarrier
MSGL_DEVICE void st_async_v4(uint32_t remote_addr, float a, float b, float c, float d, uint32_t remote_bar) {
  asm volatile("st.async.shared::cluster.mbarrier::complete_tx::bytes.v4.f32 [%0], {%1, %2, %3, %4}, [%5];" ::"r"(
                   remote_addr),
               "f"(a), "f"(b), "f"(c), "f"(d), "r"(remote_bar)
               : "memory");
}

// Bulk copy of `bytes` (multiple of 16, both addresses 16-byte aligned) from this CTA's smem
// into another cluster CTA's smem; completion is counted in bytes on that CTA's mbarrier.
MSGL_DEVICE void bulk_push_dsmem(uint32_t remote_dst, const void* src, uint32_t bytes, uint32_t remote_bar) {
  asm volatile("cp.async.bulk.shared::cluster.shared::cta.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];"
               ::"r"(remote_dst), "r"(smem_u32(src)), "r"(bytes), "r"(remote_bar)
               : "memory");
}

// Untiled bulk copy global -> this CTA's shared memory, completing on a local mbarrier (no
// multicast). Both addresses 16-byte aligned, bytes a multiple of 16.
MSGL_DEVICE void bulk_load(void* smem_dst, const void* gsrc, uint32_t bytes, uint64_t* bar) {
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];"
               ::"r"(smem_u32(smem_dst)), "l"(gsrc), "r"(bytes), "r"(smem_u32(bar))
               : "memory");
}

MSGL_DEVICE float4 ld_dsmem_v4(uint32_t addr) {
  float4 v;
  asm volatile("ld.shared::cluster.v4.f32 {%0, %1, %2, %3}, [%4];"
               : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w) : "r"(addr) : "memory");
  return v;
}

MSGL_DEVICE void prefetch_tmap(const CUtensorMap* map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}

// ------------------------------------------------------------------------------------------
// tcgen05 / TMEM
MSGL_DEVICE void tmem_alloc(uint32_t* dst_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                   smem_u32(dst_smem)),
               "r"(ncols));
}

MSGL_DEVICE void tmem_relinquish() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
}

MSGL_DEVICE void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols));
}

MSGL_DEVICE void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
MSGL_DEVICE void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// D[tmem] (+)= A[smem desc] * B[smem desc]^T, bf16/fp16 inputs, fp32 accumulate.
MSGL_DEVICE void tc_mma_f16(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                            uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate));
}

// A operand read from tensor memory (M rows = TMEM lanes, K along the columns, two 16-bit elements
// per 32-bit column, the lower K index in the low half), B from shared memory.
MSGL_DEVICE void tc_mma_f16_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc, uint32_t idesc,
                               uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d_tmem),
      "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate));
}

// Arrive on an mbarrier once all previously issued tcgen05.mma of this thread complete.
MSGL_DEVICE void tc_commit(uint64_t* bar) {
  asm volatile(
      "tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
          smem_u32(bar))
      : "memory");
}

MSGL_DEVICE void tc_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

// 32 lanes x 32 consecutive 32-bit columns; thread i of the warp gets lane (base + i).
MSGL_DEVICE void tmem_ld_32x32b_x32(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
        "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]),
        "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]),
        "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
}

MSGL_DEVICE void tmem_ld_32x32b_x16(uint32_t taddr, uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
        "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
}

// Shared-memory matrix descriptor for a K-major operand tile stored with the 128-byte swizzle
// (rows of 64 bf16 = 128 B, 8-row / 1024 B swizzle atoms stacked along M/N).
//   bits  0-13 start address >> 4      bits 16-29 leading byte offset >> 4 (unused: 1)
//   bits 32-45 stride byte offset >> 4 (1024 B between 8-row groups)
//   bits 46-47 version = 1 (sm_100)     bits 61-63 layout = 2 (SWIZZLE_128B)
MSGL_DEVICE uint64_t smem_desc_sw128(uint32_t saddr) {
  uint64_t d = 0;
  d |= (uint64_t)((saddr >> 4) & 0x3FFF);
  d |= (uint64_t)1 << 16;
  d |= (uint64_t)(1024 >> 4) << 32;
  d |= (uint64_t)1 << 46;
  d |= (uint64_t)2 << 61;
  return d;
}

// Descriptor for an MN-major operand tile with the 128-byte swizzle: each 128-byte row holds 64
// consecutive MN elements of one K index; 8-row (K) groups are 1024 B apart (stride byte offset)
// and consecutive 64-element MN groups `lbo_bytes` apart (leading byte offset).
MSGL_DEVICE uint64_t smem_desc_sw128_mn(uint32_t saddr, uint32_t lbo_bytes) {
  uint64_t d = 0;
  d |= (uint64_t)((saddr >> 4) & 0x3FFF);
  d |= (uint64_t)((lbo_bytes >> 4) & 0x3FFF) << 16;
  d |= (uint64_t)(1024 >> 4) << 32;
  d |= (uint64_t)1 << 46;
  d |= (uint64_t)2 << 61;
  return d;
}

// 32 lanes x 32 consecutive 32-bit columns from registers (thread i writes lane base + i).
MSGL_DEVICE void tmem_st_32x32b_x32(uint32_t taddr, const uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], "
      "{%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,"
      "%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};"
      ::"r"(taddr), "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]),
        "r"(r[8]), "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15]),
        "r"(r[16]), "r"(r[17]), "r"(r[18]), "r"(r[19]), "r"(r[20]), "r"(r[21]), "r"(r[22]), "r"(r[23]),
        "r"(r[24]), "r"(r[25]), "r"(r[26]), "r"(r[27]), "r"(r[28]), "r"(r[29]), "r"(r[30]), "r"(r[31])
      : "memory");
}
MSGL_DEVICE void tc_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

// Instruction descriptor for kind::f16 with bf16 A/B, fp32 D, both K-major.
__host__ __device__ constexpr uint32_t idesc_bf16_f32(int M, int N) {
  return (1u << 4)                       // D format: f32
         | (1u << 7)                     // A format: bf16
         | (1u << 10)                    // B format: bf16
         | ((uint32_t)(N >> 3) << 17)    // N >> 3
         | ((uint32_t)(M >> 4) << 24);   // M >> 4
}
// bit 16 of the kind::f16 instruction descriptor: B operand MN-major
constexpr uint32_t kIdescBMajorMN = 1u << 16;

// ------------------------------------------------------------------------------------------
// Programmatic dependent launch: a kernel launched with the PDL attribute may start while its
// predecessor in the stream is still running. It must call pdl_wait() before touching any global
// memory the predecessor (or anything earlier) reads or writes; work on static data (weights) may
// run before. pdl_launch() lets the successor start being scheduled.
MSGL_DEVICE void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
MSGL_DEVICE void pdl_launch() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

// ------------------------------------------------------------------------------------------
// cross-GPU signalling (NVLink / NVSwitch peer and multicast memory)
MSGL_DEVICE uint32_t ld_acquire_sys(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
// atomic add on the same offset of every GPU bound to the multicast object (release, system scope)
MSGL_DEVICE void mm_red_release_add(void* mc_addr, uint32_t v) {
  asm volatile("multimem.red.release.sys.global.add.u32 [%0], %1;" ::"l"(mc_addr), "r"(v) : "memory");
}
// orders this thread's async-proxy (TMA) global writes, completed by bulk_wait, with its later
// generic-proxy operations
MSGL_DEVICE void fence_proxy_async_global() { asm volatile("fence.proxy.async.global;" ::: "memory"); }

// Rank-wide arrival on a multicast counter, one call per CTA (one thread, after a CTA barrier that
// follows the CTA's writes): CTAs take tickets from a local counter; the last of `ctas` resets it
// for the next use and adds 1 to the counter on every GPU with release semantics at system scope,
// so a rank that sees the counter reach its target also sees every write of every CTA of every
// arrived rank (the fences make the ticket chain cumulative, as in a threadfence reduction).
MSGL_DEVICE void rank_arrive(uint32_t* ticket, uint32_t ctas, void* counter_mc) {
  __threadfence();
  const uint32_t old = atomicAdd(ticket, 1u);
  if (old == ctas - 1) {
    atomicExch(ticket, 0u);
    __threadfence();  // acquire side of the ticket chain; the red's release covers system scope
    mm_red_release_add(counter_mc, 1u);
  }
}

// ------------------------------------------------------------------------------------------
// named barriers among a subset of warps
MSGL_DEVICE void named_bar_sync(int id, int nthreads) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(nthreads) : "memory");
}

MSGL_DEVICE float bf16_lo(uint32_t v) { return __uint_as_float(v << 16); }
MSGL_DEVICE float bf16_hi(uint32_t v) { return __uint_as_float(v & 0xffff0000u); }

MSGL_DEVICE uint32_t pack_bf16(float a, float b) {
  __nv_bfloat162 t = __floats2bfloat162_rn(a, b);
  return *reinterpret_cast<uint32_t*>(&t);
}

}  // namespace msgl

// Launch with programmatic stream serialization (and an optional cluster shape).
// MINISGL_PDL=0 in the environment turns the attribute off (plain stream ordering).
inline bool msgl_pdl_enabled() {
  static int v = -1;
  if (v < 0) {
    const char* e = getenv("MINISGL_PDL");
    v = (e != nullptr && e[0] == '0') ? 0 : 1;
  }
  return v == 1;
}

template <typename... KArgs, typename... Args>
inline cudaError_t msgl_launch(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t s,
                               int cluster_x, Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[2];
  int n = 0;
  if (msgl_pdl_enabled()) {
    attr[n].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[n].val.programmaticStreamSerializationAllowed = 1;
    ++n;
  }
  if (cluster_x > 1) {
    attr[n].id = cudaLaunchAttributeClusterDimension;
    attr[n].val.clusterDim.x = cluster_x;
    attr[n].val.clusterDim.y = 1;
    attr[n].val.clusterDim.z = 1;
    ++n;
  }
  cfg.attrs = attr;
  cfg.numAttrs = n;
  return cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
}

// cudaFuncSetAttribute(MaxDynamicSharedMemorySize) for one kernel, done once per (kernel, device):
// the attribute belongs to the device's context, so a process that launches on several GPUs sets it
// on each. Thread-safe; returns the CUDA error of the attribute call (cudaSuccess once it is set).
// carveout >= 0 also sets the preferred shared-memory carveout (percent of the unified L1 /
// shared storage), e.g. 100 for kernels that rely on two large CTAs fitting on one SM.
template <auto Kernel>
inline cudaError_t msgl_set_smem(int bytes, int carveout = -1) {
  static std::mutex mu;
  static std::atomic<uint64_t> done{0};  // bit d: set on device d (devices 0..63)
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  const uint64_t bit = dev < 64 ? (1ull << dev) : 0;
  if (bit != 0 && (done.load(std::memory_order_acquire) & bit)) return cudaSuccess;
  std::lock_guard<std::mutex> g(mu);
  if (bit != 0 && (done.load(std::memory_order_relaxed) & bit)) return cudaSuccess;
  e = cudaFuncSetAttribute(reinterpret_cast<const void*>(Kernel), cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
  if (e == cudaSuccess && carveout >= 0)
    e = cudaFuncSetAttribute(reinterpret_cast<const void*>(Kernel), cudaFuncAttributePreferredSharedMemoryCarveout,
                             carveout);
  if (e == cudaSuccess) done.fetch_or(bit, std::memory_order_release);
  return e;
}

#define MSGL_ERROR_ACCESSOR(fn)                                                   \
  extern "C" int fn(int* info) {                                                  \
    int code = 0, inf = 0;                                                        \
    cudaMemcpyFromSymbol(&code, msgl::minisgl_error_word, sizeof(int));           \
    cudaMemcpyFromSymbol(&inf, msgl::minisgl_error_info, sizeof(int));            \
    if (code != 0) {                                                              \
      const int zero = 0;                                                         \
      cudaMemcpyToSymbol(msgl::minisgl_error_word, &zero, sizeof(int));           \
    }                                                                             \
    if (info) *info = inf;                                                        \
    return code;                                                                  \
  }
