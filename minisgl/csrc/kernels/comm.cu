// Collectives over CUDA IPC peer memory (NVLink / NVSwitch), this engine's own:
//
//   * every rank owns one symmetric buffer: [flags | data parity 0 | data parity 1];
//   * per-CTA device counters (advanced by the kernel itself, so CUDA-graph replays stay in sync)
//     give each barrier a fresh epoch and each call a data parity;
//   * CTA b of every rank owns the same slice b: it stages its slice locally, publishes e into
//     flags[b][rank] of every peer (st.release.sys), waits until flags[b][src] >= e for all src
//     (ld.acquire.sys, bounded by %globaltimer), then reads the peers' slices over NVLink.
//
// One-shot all-reduce (each rank sums all peers' copies of its slice) suits small messages; the
// two-shot form (reduce-scatter then all-gather through peer memory) moves 2(n-1)/n of the data
// per rank for large ones; all-gather copies every peer's slice. Waits never exceed a time limit: on expiry the kernel
// records kErrPeerTimeout and returns, leaving the context usable. No multicast is used.
#include <algorithm>
#include <cstdio>
#include <cstdlib>

#include "api.h"
#include "common.cuh"

using namespace msgl;

namespace {

constexpr int kMaxRanks = 8;
constexpr int kMaxBlocks = 256;
constexpr int kFlagLine = 128;                          // flags[b][0..kMaxRanks) share one line per CTA
constexpr int kFlagBytes = kMaxBlocks * kFlagLine;      // flags[b][src]

struct PeerBufs {
  uint8_t* base[kMaxRanks];  // symmetric buffer of every rank (own included)
};

__device__ __forceinline__ void st_release_sys(uint32_t* p, uint32_t v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

// Publish epoch to all ranks for block b, then wait for every rank's epoch. Returns false on timeout.
__device__ bool block_barrier(const PeerBufs& bufs, int rank, int world, int b, uint32_t epoch,
                              uint64_t timeout_ns) {
  __syncthreads();
  bool ok = true;
  if (threadIdx.x < world) {
    __threadfence_system();
    uint32_t* remote = reinterpret_cast<uint32_t*>(bufs.base[threadIdx.x] + b * kFlagLine) + rank;
    st_release_sys(remote, epoch);
    const uint32_t* mine = reinterpret_cast<const uint32_t*>(bufs.base[rank] + b * kFlagLine) + threadIdx.x;
    const uint64_t t0 = globaltimer_ns();
    while ((int)(ld_acquire_sys(mine) - epoch) < 0) {
      if (globaltimer_ns() - t0 > timeout_ns) {
        report_error(kErrPeerTimeout, b * kMaxRanks + threadIdx.x);
        ok = false;
        break;
      }
    }
  }
  return __syncthreads_and(ok) != 0;
}

__device__ __forceinline__ void add_bf16x8(float (&acc)[8], const uint4& u) {
  acc[0] += bf16_lo(u.x); acc[1] += bf16_hi(u.x); acc[2] += bf16_lo(u.y); acc[3] += bf16_hi(u.y);
  acc[4] += bf16_lo(u.z); acc[5] += bf16_hi(u.z); acc[6] += bf16_lo(u.w); acc[7] += bf16_hi(u.w);
}

// Every collective launches exactly kGrid CTAs, and CTA b always owns "sub-slice b" of every
// part of the message, so per-CTA state stays in lockstep across calls and ranks:
//   state[b] = {epoch (one per barrier), calls (one per collective; parity of the data buffer)}.
constexpr int kGrid = 64;
constexpr int kThreadsC = 512;

struct Slice {
  int64_t lo, hi;
};

// sub-slice b of part q when a message of n16 vectors is cut into `parts` parts
__device__ __forceinline__ Slice sub_slice(int64_t n16, int parts, int q, int b) {
  const int64_t part = (n16 + parts - 1) / parts;
  const int64_t p0 = q * part, p1 = min(n16, p0 + part);
  const int64_t sub = (part + kGrid - 1) / kGrid;
  const int64_t lo = min(p1, p0 + b * sub), hi = min(p1, lo + sub);
  return {lo, hi};
}

__device__ __forceinline__ void sum_peers(uint4* __restrict__ dst, const PeerBufs& bufs, size_t data_off, int rank,
                                          int world, int64_t lo, int64_t hi) {
  for (int64_t i = lo + threadIdx.x; i < hi; i += blockDim.x) {
    uint4 v[kMaxRanks];
#pragma unroll
    for (int r = 0; r < kMaxRanks; ++r)
      if (r < world) v[r] = reinterpret_cast<const uint4*>(bufs.base[(rank + r) % world] + data_off)[i];
    float acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
#pragma unroll
    for (int r = 0; r < kMaxRanks; ++r)
      if (r < world) add_bf16x8(acc, v[r]);
    uint4 o;
    o.x = pack_bf16(acc[0], acc[1]); o.y = pack_bf16(acc[2], acc[3]);
    o.z = pack_bf16(acc[4], acc[5]); o.w = pack_bf16(acc[6], acc[7]);
    dst[i] = o;
  }
}

// mode 0: one-shot all-reduce (bf16 sum); 1: two-shot all-reduce (reduce-scatter + all-gather
// through the peers' buffers); 2: all-gather (out[r * n16 + i] = in_r[i]).
__global__ void __launch_bounds__(kThreadsC) peer_collective_kernel(PeerBufs bufs, int rank, int world, int mode,
                                                                    uint4* __restrict__ out,
                                                                    const uint4* __restrict__ in, int64_t n16,
                                                                    int64_t cap16, uint32_t* __restrict__ state,
                                                                    uint64_t timeout_ns) {
  const int b = blockIdx.x;
  pdl_wait();
  pdl_launch();
  __shared__ uint32_t s_epoch, s_calls;
  if (threadIdx.x == 0) {
    s_epoch = state[2 * b];
    s_calls = state[2 * b + 1] + 1;
  }
  __syncthreads();
  uint32_t epoch = s_epoch;
  const uint32_t calls = s_calls;
  const size_t data_off = kFlagBytes + (size_t)(calls & 1) * cap16 * 16;
  uint4* mine = reinterpret_cast<uint4*>(bufs.base[rank] + data_off);
  const int parts = mode == 1 ? world : 1;
  // stage: this CTA's sub-slice of every part
  for (int q = 0; q < parts; ++q) {
    const Slice sl = sub_slice(n16, parts, q, b);
    for (int64_t i = sl.lo + threadIdx.x; i < sl.hi; i += blockDim.x) mine[i] = in[i];
  }
  bool ok = block_barrier(bufs, rank, world, b, ++epoch, timeout_ns);
  if (ok) {
    if (mode == 0) {
      const Slice sl = sub_slice(n16, 1, 0, b);
      sum_peers(out, bufs, data_off, rank, world, sl.lo, sl.hi);
    } else if (mode == 2) {
      const Slice sl = sub_slice(n16, 1, 0, b);
      for (int r = 0; r < world; ++r) {
        const uint4* src = reinterpret_cast<const uint4*>(bufs.base[r] + data_off);
        for (int64_t i = sl.lo + threadIdx.x; i < sl.hi; i += blockDim.x) out[r * n16 + i] = src[i];
      }
    } else {
      // reduce my part in place (peers only read the other parts of my buffer in this phase)
      const Slice mine_sl = sub_slice(n16, world, rank, b);
      sum_peers(mine, bufs, data_off, rank, world, mine_sl.lo, mine_sl.hi);
      ok = block_barrier(bufs, rank, world, b, ++epoch, timeout_ns);
      if (ok) {
        for (int q = 0; q < world; ++q) {
          const Slice sl = sub_slice(n16, world, q, b);
          const uint4* src = reinterpret_cast<const uint4*>(bufs.base[q] + data_off);
          for (int64_t i = sl.lo + threadIdx.x; i < sl.hi; i += blockDim.x) out[i] = src[i];
        }
      }
    }
  } else if (mode == 1) {
    ++epoch;  // keep the epoch sequence aligned with the ranks that did not time out
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    state[2 * b] = epoch;
    state[2 * b + 1] = calls;
  }
}

}  // namespace

extern "C" {

int msgl_peer_flag_bytes() { return kFlagBytes; }

void* msgl_peer_alloc(int64_t bytes) {
  void* p = nullptr;
  if (cudaMalloc(&p, bytes) != cudaSuccess) return nullptr;
  cudaMemset(p, 0, bytes);
  return p;
}

void msgl_peer_free(void* p) { cudaFree(p); }

int msgl_ipc_handle(void* p, void* out64) {
  cudaIpcMemHandle_t h;
  const cudaError_t e = cudaIpcGetMemHandle(&h, p);
  if (e != cudaSuccess) return (int)e;
  memcpy(out64, &h, sizeof(h));
  return 0;
}

void* msgl_ipc_open(const void* in64) {
  cudaIpcMemHandle_t h;
  memcpy(&h, in64, sizeof(h));
  void* p = nullptr;
  if (cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess) != cudaSuccess) return nullptr;
  return p;
}

void msgl_ipc_close(void* p) { cudaIpcCloseMemHandle(p); }

int msgl_peer_grid() { return kGrid; }

void msgl_peer_collective(void* const* bases, int rank, int world, int mode, void* out, const void* in,
                          int64_t bytes, int64_t cap_bytes, uint32_t* state, int64_t timeout_ns, cudaStream_t s) {
  PeerBufs bufs;
  for (int r = 0; r < kMaxRanks; ++r) bufs.base[r] = r < world ? reinterpret_cast<uint8_t*>(bases[r]) : nullptr;
  msgl_launch(peer_collective_kernel, dim3(kGrid), dim3(kThreadsC), 0, s, 1, bufs, rank, world, mode,
              reinterpret_cast<uint4*>(out), reinterpret_cast<const uint4*>(in), bytes / 16, cap_bytes / 16, state,
              (uint64_t)timeout_ns);
}

}  // extern "C"




// =================================================================================================
// NVLink SHARP (NVLS) all-reduce fused with residual add + RMSNorm (the collective that follows
// every row-parallel GEMM of a tensor-parallel decoder, and the vocab-parallel embedding).
//
// Every rank's symmetric buffer is bound to one NVLink multicast object: a multimem store or
// reduction on the multicast address reaches the same offset on every GPU through the switch, and
// multimem.ld_reduce returns the sum of all GPUs' copies (fp32 accumulation in the switch).
// Buffer: [flags: kNvlsGrid x 128 B | LL parity 0 | LL parity 1 | staging | gather], `cap` bytes
// per data region. Per-CTA state words in device memory advance inside the kernel, so CUDA-graph
// replays stay in lockstep across ranks.
//
// Small messages (world x T x H x 4 bytes below a limit): "LL" form, no barrier. Every rank stores
// its rows with multimem.st as 8-byte {bf16x2 data, epoch} words into its own slot on every GPU; a
// reader spins on its local copy until every word carries the epoch (an aligned 8-byte store lands
// whole), so data and synchronisation arrive together in one NVLink trip. Each rank then sums all
// slots for every row itself. Parity reuse is safe: a CTA writes parity p again only in the call
// after next, which it starts after seeing every peer's data of the next call, which each peer
// sends after finishing its reads of parity p.
//
// Larger messages: reduce-scatter + norm + all-gather ("RS" form), the shape of the fused
// row-parallel path:
//   1. the rank's partial sum [T, H] lands in its staging region: written there by the producing
//      GEMM's epilogue (mode 3: that GEMM's last CTA also signals arrival), by the previous kernel
//      (mode 2), or copied in here (mode 1); arrival = one multimem.red on counter 1 per rank;
//   2. once every rank arrived, rank r owns rows i with i % world == r: it reads their sum with
//      multimem.ld_reduce, adds its residual rows, normalises, keeps the new residual rows (the
//      residual stream stays sharded by row between the fused norms, which are its only readers),
//      and multimem-stores the normalised rows into the gather region of every GPU;
//   3. arrival on counter 2 after those stores; CTA 0 waits for every rank's, so the kernel ends
//      only when the gather region (the returned activations) holds every row on this GPU.
// Each GPU sends/receives T x H x 2 bytes per phase instead of every rank reducing every row
// (world x the switch traffic). Staging and gather need no parity: a rank writes its staging for
// call c+1 only after call c's second barrier (every rank done reading it), and every rank's
// gather stores of call c+1 follow the first barrier of c+1, which follows every rank's reads of
// call c's gathered rows (by the GEMM that consumes them, earlier in its stream).
// All waits are bounded by %globaltimer: on expiry the kernel records kErrPeerTimeout and returns.
namespace {

constexpr int kNvlsGrid = 128;
constexpr int kNvlsThreads = 256;
constexpr int kNvlsFlagStride = 128;  // one counter per 128-byte line
constexpr int kNvlsFlagBytes = kNvlsGrid * kNvlsFlagStride;
constexpr int kNvlsMaxVec = 8;  // 16-byte vectors per thread per row: H <= 8 * 8 * 256 = 16384
// state words: LL call count per CTA [0, kNvlsGrid); the RS call count; two local arrival tickets
// (each on its own 128-byte line)
constexpr int kStateRS = 4 * kNvlsGrid;
constexpr int kTicket1 = 4 * kNvlsGrid + 32;
constexpr int kTicket2 = 4 * kNvlsGrid + 64;
constexpr int kNvlsStateWords = 4 * kNvlsGrid + 96;

enum NvlsMode : int { kModeLL = 0, kModeStage = 1, kModePrestaged = 2, kModeGemmArrived = 3 };

struct NvlsParams {
  uint8_t* uc;        // this rank's symmetric buffer
  uint8_t* mc;        // multicast address of the same buffer
  int rank, world;
  const uint4* x;     // [T, H] partial (bf16); unused in modes 2 and 3 (already in staging)
  uint4* residual;    // [T, H] bf16, updated in place (residual += sum); RS: this rank's rows only
  const uint4* w;     // [H] bf16 norm weight
  uint4* out;         // [T, H] bf16 normalised (LL); RS writes the gather region instead
  int T, H;
  float eps;
  int64_t cap;
  uint32_t* state;    // kNvlsStateWords
  uint64_t timeout_ns;
  int first;          // 1: residual is not read (it becomes the sum)
  int mode;
  uint64_t* trace;    // optional [kNvlsGrid][8] %globaltimer stamps of the RS phases (profiling)
};

__device__ __forceinline__ uint4 mm_ld_reduce_bf16x8(const uint8_t* mc_addr) {
  uint4 r;
  asm volatile("multimem.ld_reduce.relaxed.sys.global.add.acc::f32.v4.bf16x2 {%0, %1, %2, %3}, [%4];"
               : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
               : "l"(mc_addr)
               : "memory");
  return r;
}
__device__ __forceinline__ void mm_st_bf16x8(uint8_t* mc_addr, const uint4& v) {
  asm volatile("multimem.st.relaxed.sys.global.v4.bf16x2 [%0], {%1, %2, %3, %4};" ::"l"(mc_addr), "r"(v.x),
               "r"(v.y), "r"(v.z), "r"(v.w)
               : "memory");
}
__device__ __forceinline__ void mm_st_b64(uint8_t* mc_addr, uint64_t v) {
  asm volatile("multimem.st.relaxed.sys.global.b64 [%0], %1;" ::"l"(mc_addr), "l"(v) : "memory");
}
__device__ __forceinline__ void ld_relaxed_v2_u64(const uint8_t* p, uint64_t& a, uint64_t& b) {
  asm volatile("ld.relaxed.sys.global.v2.u64 {%0, %1}, [%2];" : "=l"(a), "=l"(b) : "l"(p) : "memory");
}

__device__ __forceinline__ void unpack8(const uint4& u, float (&f)[8]) {
  f[0] = bf16_lo(u.x); f[1] = bf16_hi(u.x); f[2] = bf16_lo(u.y); f[3] = bf16_hi(u.y);
  f[4] = bf16_lo(u.z); f[5] = bf16_hi(u.z); f[6] = bf16_lo(u.w); f[7] = bf16_hi(u.w);
}
__device__ __forceinline__ uint4 pack8(const float (&f)[8]) {
  return make_uint4(pack_bf16(f[0], f[1]), pack_bf16(f[2], f[3]), pack_bf16(f[4], f[5]), pack_bf16(f[6], f[7]));
}

// spin (one thread) until the counter reaches `target` (wrap-safe); false on timeout
__device__ __forceinline__ bool wait_counter(const uint8_t* counter, uint32_t target, uint64_t timeout_ns, int site) {
  const uint32_t* c = reinterpret_cast<const uint32_t*>(counter);
  if ((int)(ld_acquire_sys(c) - target) >= 0) return true;
  const uint64_t t0 = globaltimer_ns();
  while ((int)(ld_acquire_sys(c) - target) < 0) {
    if (globaltimer_ns() - t0 > timeout_ns) {
      report_error(kErrPeerTimeout, site);
      return false;
    }
  }
  return true;
}

// LL form: sum over every rank's slot of one 8-element group (4 words {bf16x2, epoch}); spins on
// the local copy until all words carry `epoch`. Returns false on timeout.
__device__ __forceinline__ bool ll_gather8(const uint8_t* base, int64_t slot_bytes, int world, int64_t goff,
                                           uint32_t epoch, uint64_t timeout_ns, float (&f)[8]) {
#pragma unroll
  for (int j = 0; j < 8; ++j) f[j] = 0.f;
  uint64_t t0 = 0;
  for (int r = 0; r < world; ++r) {
    const uint8_t* src = base + r * slot_bytes + goff;
    uint64_t w0, w1, w2, w3;
    while (true) {
      ld_relaxed_v2_u64(src, w0, w1);
      ld_relaxed_v2_u64(src + 16, w2, w3);
      if ((uint32_t)(w0 >> 32) == epoch && (uint32_t)(w1 >> 32) == epoch && (uint32_t)(w2 >> 32) == epoch &&
          (uint32_t)(w3 >> 32) == epoch)
        break;
      const uint64_t now = globaltimer_ns();
      if (t0 == 0) t0 = now;
      else if (now - t0 > timeout_ns) return false;
    }
    const uint32_t d[4] = {(uint32_t)w0, (uint32_t)w1, (uint32_t)w2, (uint32_t)w3};
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      f[2 * j] += bf16_lo(d[j]);
      f[2 * j + 1] += bf16_hi(d[j]);
    }
  }
  // the all-reduce result is bf16, as with ld_reduce
#pragma unroll
  for (int j = 0; j < 8; j += 2) {
    const uint32_t q = pack_bf16(f[j], f[j + 1]);
    f[j] = bf16_lo(q);
    f[j + 1] = bf16_hi(q);
  }
  return true;
}

// Sum (already in vals) + residual -> residual (bf16); RMS-normalise the stored residual; returns
// the normalised 16-byte vectors in vals. Block-wide: every thread calls it for the same row.
__device__ __forceinline__ void add_residual_norm(const NvlsParams& p, int row, float (&vals)[kNvlsMaxVec][8],
                                                  float* s_red) {
  const int tid = threadIdx.x, nv = p.H / 8;
  float ss = 0.f;
#pragma unroll
  for (int k = 0; k < kNvlsMaxVec; ++k) {
    const int v = tid + k * kNvlsThreads;
    if (v < nv) {
      const int64_t idx = (int64_t)row * nv + v;
      if (!p.first) {
        float r[8];
        unpack8(p.residual[idx], r);
#pragma unroll
        for (int j = 0; j < 8; ++j) vals[k][j] += r[j];
      }
      const uint4 packed = pack8(vals[k]);
      p.residual[idx] = packed;
      unpack8(packed, vals[k]);  // normalise the stored (bf16) residual
#pragma unroll
      for (int j = 0; j < 8; ++j) ss += vals[k][j] * vals[k][j];
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
  if ((tid & 31) == 0) s_red[tid >> 5] = ss;
  __syncthreads();
  float tot = 0.f;
#pragma unroll
  for (int i = 0; i < kNvlsThreads / 32; ++i) tot += s_red[i];
  __syncthreads();  // s_red reuse by the next row
  const float rstd = rsqrtf(tot / (float)p.H + p.eps);
#pragma unroll
  for (int k = 0; k < kNvlsMaxVec; ++k) {
    const int v = tid + k * kNvlsThreads;
    if (v < nv) {
      float wf[8];
      unpack8(p.w[v], wf);
#pragma unroll
      for (int j = 0; j < 8; ++j) vals[k][j] = vals[k][j] * rstd * wf[j];
    }
  }
}

// RS rows: groups of kRsGroup threads per row, kRsGroups per CTA; H <= kRsMaxVec x 8 x kRsGroup
constexpr int kRsGroup = 128;
constexpr int kRsGroups = kNvlsThreads / kRsGroup;
constexpr int kRsMaxVec = 8;

// add_residual_norm for one 128-thread group (rank-local rows of the RS form): the sum of squares
// goes through the group's own slice of s_red and named barrier 1 + g.
__device__ __forceinline__ void group_residual_norm(const NvlsParams& p, int row, int g, int gt,
                                                    float (&vals)[kRsMaxVec][8], float* s_red) {
  const int nv = p.H / 8;
  float ss = 0.f;
#pragma unroll
  for (int k = 0; k < kRsMaxVec; ++k) {
    const int v = gt + k * kRsGroup;
    if (v < nv) {
      const int64_t idx = (int64_t)row * nv + v;
      if (!p.first) {
        float r[8];
        unpack8(p.residual[idx], r);
#pragma unroll
        for (int j = 0; j < 8; ++j) vals[k][j] += r[j];
      }
      const uint4 packed = pack8(vals[k]);
      p.residual[idx] = packed;
      unpack8(packed, vals[k]);  // normalise the stored (bf16) residual
#pragma unroll
      for (int j = 0; j < 8; ++j) ss += vals[k][j] * vals[k][j];
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
  if ((gt & 31) == 0) s_red[gt >> 5] = ss;
  named_bar_sync(1 + g, kRsGroup);
  float tot = 0.f;
#pragma unroll
  for (int i = 0; i < kRsGroup / 32; ++i) tot += s_red[i];
  named_bar_sync(1 + g, kRsGroup);  // s_red reuse by the group's next row
  const float rstd = rsqrtf(tot / (float)p.H + p.eps);
#pragma unroll
  for (int k = 0; k < kRsMaxVec; ++k) {
    const int v = gt + k * kRsGroup;
    if (v < nv) {
      float wf[8];
      unpack8(p.w[v], wf);
#pragma unroll
      for (int j = 0; j < 8; ++j) vals[k][j] = vals[k][j] * rstd * wf[j];
    }
  }
}

__global__ void __launch_bounds__(kNvlsThreads) nvls_ar_rmsnorm_kernel(NvlsParams p) {
  const int b = blockIdx.x, tid = threadIdx.x;
  const int nv = p.H / 8;
  __shared__ float s_red[kNvlsThreads / 32];
  __shared__ uint32_t s_calls;
  pdl_launch();
  if (p.mode == kModeLL) {
    pdl_wait();
    if (tid == 0) s_calls = p.state[b] + 1;
    __syncthreads();
    const uint32_t calls = s_calls;
    const size_t off = kNvlsFlagBytes + (size_t)(calls & 1) * p.cap;
    const int64_t slot_bytes = (int64_t)p.T * p.H * 4;  // 8 bytes per bf16 pair
    // 1. send: my rows into my slot on every GPU, each bf16 pair tagged with the epoch
    uint8_t* my_slot = p.mc + off + p.rank * slot_bytes;
    const uint64_t tag = (uint64_t)calls << 32;
    for (int row = b; row < p.T; row += kNvlsGrid)
      for (int v = tid; v < nv; v += kNvlsThreads) {
        const uint4 u = p.x[(int64_t)row * nv + v];
        uint8_t* dst = my_slot + ((int64_t)row * nv + v) * 32;
        mm_st_b64(dst, tag | u.x);
        mm_st_b64(dst + 8, tag | u.y);
        mm_st_b64(dst + 16, tag | u.z);
        mm_st_b64(dst + 24, tag | u.w);
      }
    // 2. every rank's slot, summed, + residual, normalised
    const uint8_t* ldata = p.uc + off;
    for (int row = b; row < p.T; row += kNvlsGrid) {
      float vals[kNvlsMaxVec][8];
      bool good = true;
#pragma unroll
      for (int k = 0; k < kNvlsMaxVec; ++k) {
        const int v = tid + k * kNvlsThreads;
        if (v < nv) good &= ll_gather8(ldata, slot_bytes, p.world, ((int64_t)row * nv + v) * 32, calls,
                                       p.timeout_ns, vals[k]);
      }
      if (!good) report_error(kErrPeerTimeout, 2000 + b);
      add_residual_norm(p, row, vals, s_red);
#pragma unroll
      for (int k = 0; k < kNvlsMaxVec; ++k) {
        const int v = tid + k * kNvlsThreads;
        if (v < nv) p.out[(int64_t)row * nv + v] = pack8(vals[k]);
      }
    }
    if (tid == 0) p.state[b] = calls;
    return;
  }

  // ---------------------------------------------------------------------------- RS form
  // Wait for the producer in every mode: the per-CTA call counters (and tickets) were last written
  // by the previous call of this kernel, which completed before the producer did (every kernel of
  // the chain waits for its predecessor before it ends), but not necessarily before this grid
  // started (programmatic launch lets several grids of the chain be resident at once). In mode 3
  // the producer GEMM already published its tiles to every rank before finishing.
  pdl_wait();
  uint64_t* tr = (p.trace != nullptr && tid == 0) ? p.trace + b * 8 : nullptr;
  if (tr) tr[0] = globaltimer_ns();
  if (tid == 0) s_calls = p.state[kStateRS] + 1;
  __syncthreads();
  const uint32_t rs = s_calls;
  const uint32_t target = rs * (uint32_t)p.world;  // each rank adds 1 per call to each counter
  uint8_t* stage_uc = p.uc + kNvlsFlagBytes + 2 * p.cap;
  const uint8_t* stage_mc = p.mc + kNvlsFlagBytes + 2 * p.cap;
  uint8_t* gather_mc = p.mc + kNvlsFlagBytes + 3 * p.cap;
  uint8_t* cnt1_mc = p.mc;
  uint8_t* cnt2_mc = p.mc + kNvlsFlagStride;
  if (p.mode != kModeGemmArrived) {
    // stage (or just publish) this rank's partial sum
    if (p.mode == kModeStage) {
      const int64_t n16 = (int64_t)p.T * nv;
      uint4* dst = reinterpret_cast<uint4*>(stage_uc);
      for (int64_t i = (int64_t)b * kNvlsThreads + tid; i < n16; i += (int64_t)gridDim.x * kNvlsThreads)
        dst[i] = p.x[i];
    }
    __syncthreads();
    if (tid == 0) rank_arrive(p.state + kTicket1, gridDim.x, cnt1_mc);
  }
  if (tr) tr[1] = globaltimer_ns();
  // 1. every rank's partial is staged
  bool ok = true;
  if (tid == 0) ok = wait_counter(p.uc, target, p.timeout_ns, 3000 + b);
  ok = __syncthreads_and(ok) != 0;
  if (tr) tr[2] = globaltimer_ns();
  if (ok) {
    // 2. reduce-scatter by row, residual + norm, all-gather of the normalised rows. Each CTA is two
    // 128-thread groups working on different rows (reductions through a group-local named barrier),
    // so twice as many rows are in flight as CTAs: the phase costs about one multimem round trip.
    const int g = tid / kRsGroup, gt = tid % kRsGroup;
    for (int j = b * kRsGroups + g;; j += gridDim.x * kRsGroups) {
      const int i = j * p.world + p.rank;
      if (i >= p.T) break;
      float vals[kRsMaxVec][8];
#pragma unroll
      for (int k = 0; k < kRsMaxVec; ++k) {
        const int v = gt + k * kRsGroup;
        if (v < nv) unpack8(mm_ld_reduce_bf16x8(stage_mc + ((int64_t)i * nv + v) * 16), vals[k]);
      }
      group_residual_norm(p, i, g, gt, vals, s_red + g * (kRsGroup / 32));
#pragma unroll
      for (int k = 0; k < kRsMaxVec; ++k) {
        const int v = gt + k * kRsGroup;
        if (v < nv) mm_st_bf16x8(gather_mc + ((int64_t)i * nv + v) * 16, pack8(vals[k]));
      }
    }
  }
  // 3. this CTA's gather stores are issued; the rank's last CTA publishes them
  __syncthreads();
  if (tid == 0) {
    if (tr) tr[3] = globaltimer_ns();
    rank_arrive(p.state + kTicket2, gridDim.x, cnt2_mc);
    if (tr) tr[4] = globaltimer_ns();
    if (b == 0) {
      if (wait_counter(p.uc + kNvlsFlagStride, target, p.timeout_ns, 4000))
        fence_proxy_async_global();  // gathered rows are read next by TMA loads
      // every CTA of this call read the count before its arrival, and the second barrier passed
      // only after all of them arrived
      p.state[kStateRS] = rs;
    }
    if (tr) tr[5] = globaltimer_ns();
  }
}

}  // namespace

extern "C" int msgl_nvls_grid() { return kNvlsGrid; }
extern "C" int msgl_nvls_flag_bytes() { return kNvlsFlagBytes; }
extern "C" int msgl_nvls_state_words() { return kNvlsStateWords; }
extern "C" int64_t msgl_nvls_ticket_offset() { return (int64_t)kTicket1 * 4; }

extern "C" int msgl_nvls_allreduce_rmsnorm(void* uc, void* mc, int rank, int world, const void* x, void* residual,
                                           const void* w, void* out, int T, int H, float eps, int64_t cap_bytes,
                                           uint32_t* state, int64_t timeout_ns, int first, int mode, uint64_t* trace,
                                           cudaStream_t s) {
  if (H % 8 != 0 || H > 8 * kNvlsMaxVec * kNvlsThreads || (int64_t)T * H * 2 > cap_bytes) return 3;
  if (mode < kModeLL || mode > kModeGemmArrived || world < 1 || rank < 0 || rank >= world) return 3;
  if (mode == kModeLL && (int64_t)world * T * H * 4 > cap_bytes) return 3;
  if (mode != kModeLL && H > kRsMaxVec * 8 * kRsGroup) return 3;
  NvlsParams p;
  p.uc = reinterpret_cast<uint8_t*>(uc);
  p.mc = reinterpret_cast<uint8_t*>(mc);
  p.rank = rank;
  p.world = world;
  p.x = reinterpret_cast<const uint4*>(x);
  p.residual = reinterpret_cast<uint4*>(residual);
  p.w = reinterpret_cast<const uint4*>(w);
  p.out = reinterpret_cast<uint4*>(out);
  p.T = T;
  p.H = H;
  p.eps = eps;
  p.cap = cap_bytes;
  p.state = state;
  p.timeout_ns = (uint64_t)timeout_ns;
  p.first = first;
  p.mode = mode;
  p.trace = trace;
  // RS: one 128-thread group per row of this rank's share (rows i % world == rank), two per CTA
  const int rows_local = (T + world - 1) / world;
  const int grid = mode == kModeLL ? kNvlsGrid
                                   : std::max(1, std::min(kNvlsGrid, (rows_local + kRsGroups - 1) / kRsGroups));
  return msgl_launch(nvls_ar_rmsnorm_kernel, dim3(grid), dim3(kNvlsThreads), 0, s, 1, p) == cudaSuccess ? 0 : 4;
}

MSGL_ERROR_ACCESSOR(msgl_err_comm)
