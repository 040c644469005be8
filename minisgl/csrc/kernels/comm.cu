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
#include <cstdio>

#include "api.h"
#include "common.cuh"

using namespace msgl;

namespace {

constexpr int kMaxRanks = 8;
constexpr int kMaxBlocks = 256;
constexpr int kFlagBytes = kMaxBlocks * kMaxRanks * 4;  // flags[b][src]

struct PeerBufs {
  uint8_t* base[kMaxRanks];  // symmetric buffer of every rank (own included)
};

__device__ __forceinline__ void st_release_sys(uint32_t* p, uint32_t v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// Publish epoch to all ranks for block b, then wait for every rank's epoch. Returns false on timeout.
__device__ bool block_barrier(const PeerBufs& bufs, int rank, int world, int b, uint32_t epoch,
                              uint64_t timeout_ns) {
  __syncthreads();
  bool ok = true;
  if (threadIdx.x < world) {
    __threadfence_system();
    uint32_t* remote = reinterpret_cast<uint32_t*>(bufs.base[threadIdx.x]) + b * kMaxRanks + rank;
    st_release_sys(remote, epoch);
    const uint32_t* mine = reinterpret_cast<const uint32_t*>(bufs.base[rank]) + b * kMaxRanks + threadIdx.x;
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

MSGL_ERROR_ACCESSOR(msgl_err_comm)
