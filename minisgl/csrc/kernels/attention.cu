// Paged-KV attention for prefill (ragged, causal, prefix/chunk aware) and decode (split-KV),
// with grouped-query packing, optional sliding window and per-head attention sinks.
//
// Layout: q [T, nq, hd] bf16; k_cache / v_cache [slots, nkv, hd] bf16; page_table[row, pos] is the
// KV slot of position `pos` of the request in that row (token granular, so any page size works).
// The queries of request b are the last q_len(b) positions of its kv_len(b)-long sequence.
//
// Both kernels pack the G = nq/nkv query heads that share a KV head into the rows of one tile:
// row r <-> (token r / G, head r % G), so every K/V tile fetched from HBM serves the whole group.
// K/V tiles of 64 keys are gathered through the page table with cp.async (double buffered, zero
// fill past the end) into 128-byte-swizzled shared memory; QK^T and PV run on mma.sync bf16 with
// an fp32 online softmax in the log2 domain.
#include <algorithm>
#include <cfloat>

#include "api.h"
#include "common.cuh"

#include <atomic>
#include <cstring>
#include <mutex>

using namespace msgl;

namespace {

constexpr int KC = 64;        // keys per chunk
constexpr int kWarps = 4;
constexpr float kLog2e = 1.4426950408889634f;

struct AttnParams {
  __nv_bfloat16* o;
  const __nv_bfloat16* q;
  const __nv_bfloat16* k;
  const __nv_bfloat16* v;
  const int32_t* page_table;
  int64_t pt_stride;
  const int32_t* rows;
  const int32_t* cu_q;
  const int32_t* kv_lens;
  int nq, nkv, group;
  int64_t cache_stride;
  int64_t num_slots;  // cache rows (index checks of the bounds-check build)
  float scale_log2;
  int window;
  const float* sinks;
  int num_splits;
  float* ws;  // decode partials: o [bs*nq*splits*hd] then (m,l) pairs
};

__device__ __forceinline__ void cp_async16(uint32_t dst, const void* src, bool valid) {
  const int n = valid ? 16 : 0;
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst), "l"(src), "r"(n) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() { asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory"); }

__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3) : "r"(addr));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3) : "r"(addr));
}

__device__ __forceinline__ void mma_bf16(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

// byte offset of (row, 16B chunk) inside a swizzled [rows][HD] bf16 tile
template <int HD>
__device__ __forceinline__ uint32_t swz(int row, int chunk) {
  constexpr int CH = HD / 8;
  return (uint32_t)(row * CH + (chunk ^ (row & 7))) * 16u;
}

// Gather keys [k0, k0 + KC) of one request / kv head into swizzled smem; positions >= kend are
// zero-filled.
template <int HD>
__device__ __forceinline__ void load_kv_chunk(uint32_t sk, uint32_t sv, const AttnParams& p, int row,
                                              int kvh, int k0, int kend) {
  constexpr int CH = HD / 8;
  const int32_t* pt = p.page_table + (int64_t)row * p.pt_stride;
#pragma unroll
  for (int i = 0; i < KC * CH / (kWarps * 32); ++i) {
    const int c = threadIdx.x + i * kWarps * 32;
    const int key = c / CH, part = c % CH;
    const int pos = k0 + key;
    bool valid = pos < kend;
    int64_t slot = valid ? pt[pos] : 0;
    if (valid && !MSGL_IN_BOUNDS(slot >= 0 && slot < p.num_slots, kBcAttnSlot)) valid = false, slot = 0;
    const int64_t off = slot * p.cache_stride + (int64_t)kvh * HD + part * 8;
    cp_async16(sk + swz<HD>(key, part), p.k + off, valid);
    cp_async16(sv + swz<HD>(key, part), p.v + off, valid);
  }
}

// S[16 x 8*NT] = Q(16 x HD) K^T for keys [key0, key0 + 8*NT) of the smem tile
template <int HD, int NT>
__device__ __forceinline__ void qk(float (&s)[NT][4], const uint32_t (&qf)[HD / 16][4], uint32_t sk, int key0) {
  const int lane = threadIdx.x & 31;
#pragma unroll
  for (int n = 0; n < NT; ++n) s[n][0] = s[n][1] = s[n][2] = s[n][3] = 0.f;
#pragma unroll
  for (int kk = 0; kk < HD / 16; ++kk) {
#pragma unroll
    for (int n = 0; n < NT; n += 2) {
      const int idx = lane >> 3;
      const int key = key0 + n * 8 + (idx >> 1) * 8 + (lane & 7);
      const int chunk = kk * 2 + (idx & 1);
      uint32_t b0, b1, b2, b3;
      ldsm_x4(sk + swz<HD>(key, chunk), b0, b1, b2, b3);
      mma_bf16(s[n], qf[kk], b0, b1);
      if (n + 1 < NT) mma_bf16(s[n + 1], qf[kk], b2, b3);
    }
  }
}

// O[16 x HD] += P(16 x 16*KS) V for keys [key0, key0 + 16*KS)
template <int HD, int KS>
__device__ __forceinline__ void pv(float (&o)[HD / 8][4], const uint32_t (&pf)[KS][4], uint32_t sv, int key0) {
  const int lane = threadIdx.x & 31;
#pragma unroll
  for (int ks = 0; ks < KS; ++ks) {
#pragma unroll
    for (int n = 0; n < HD / 8; n += 2) {
      const int idx = lane >> 3;
      const int key = key0 + ks * 16 + (idx & 1) * 8 + (lane & 7);
      const int chunk = n + (idx >> 1);
      uint32_t b0, b1, b2, b3;
      ldsm_x4_t(sv + swz<HD>(key, chunk), b0, b1, b2, b3);
      mma_bf16(o[n], pf[ks], b0, b1);
      mma_bf16(o[n + 1], pf[ks], b2, b3);
    }
  }
}

// Online softmax update for this thread's two rows (lane/4 and lane/4 + 8) over the S tile.
// Scores are already in the log2 domain; masked entries are -inf.
template <int NT>
__device__ __forceinline__ void softmax_update(float (&s)[NT][4], float (&m)[2], float (&l)[2],
                                               float (&scale_o)[2]) {
#pragma unroll
  for (int h = 0; h < 2; ++h) {
    float mx = m[h];
#pragma unroll
    for (int n = 0; n < NT; ++n) mx = fmaxf(mx, fmaxf(s[n][2 * h], s[n][2 * h + 1]));
    mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
    mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
    const float base = mx == -FLT_MAX || mx == -INFINITY ? 0.f : mx;
    scale_o[h] = exp2f(m[h] - base);
    float sum = 0.f;
#pragma unroll
    for (int n = 0; n < NT; ++n) {
      s[n][2 * h] = exp2f(s[n][2 * h] - base);
      s[n][2 * h + 1] = exp2f(s[n][2 * h + 1] - base);
      sum += s[n][2 * h] + s[n][2 * h + 1];
    }
    sum += __shfl_xor_sync(0xffffffffu, sum, 1);
    sum += __shfl_xor_sync(0xffffffffu, sum, 2);
    l[h] = l[h] * scale_o[h] + sum;
    m[h] = mx;
  }
}

template <int NT>
__device__ __forceinline__ void pack_p(uint32_t (&pf)[NT / 2][4], const float (&s)[NT][4]) {
#pragma unroll
  for (int k = 0; k < NT / 2; ++k) {
    pf[k][0] = pack_bf16(s[2 * k][0], s[2 * k][1]);
    pf[k][1] = pack_bf16(s[2 * k][2], s[2 * k][3]);
    pf[k][2] = pack_bf16(s[2 * k + 1][0], s[2 * k + 1][1]);
    pf[k][3] = pack_bf16(s[2 * k + 1][2], s[2 * k + 1][3]);
  }
}

// ================================================================================ prefill
// grid (row blocks of 64 packed rows, requests, kv heads), 4 warps x 16 rows.
template <int HD>
__global__ void __launch_bounds__(kWarps * 32) prefill_kernel(AttnParams p) {
  extern __shared__ __align__(128) uint8_t smem[];
  pdl_wait();
  pdl_launch();
  const int qb = blockIdx.x, b = blockIdx.y, kvh = blockIdx.z;
  const int G = p.group;
  const int q0 = p.cu_q[b], n = p.cu_q[b + 1] - q0;
  const int total_rows = n * G;
  if (qb * 64 >= total_rows) return;
  const int L = p.kv_lens[b], row = p.rows[b];
  if (!MSGL_IN_BOUNDS(row >= 0 && L >= n && L <= p.pt_stride, kBcAttnRow)) return;  // CTA-uniform
  const int qpos0 = L - n;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  const uint32_t sq = smem_u32(smem);
  const uint32_t sk0 = sq + 64 * HD * 2;
  const uint32_t sv0 = sk0 + 2 * KC * HD * 2;

  // stage Q rows of this block
  constexpr int CH = HD / 8;
  for (int c = threadIdx.x; c < 64 * CH; c += kWarps * 32) {
    const int r = c / CH, part = c % CH;
    const int gr = qb * 64 + r;
    const bool valid = gr < total_rows;
    const int t = valid ? gr / G : 0, g = valid ? gr % G : 0;
    const __nv_bfloat16* src = p.q + ((int64_t)(q0 + t) * p.nq + kvh * G + g) * HD + part * 8;
    cp_async16(sq + swz<HD>(r, part), src, valid);
  }
  cp_async_commit();

  const int last_row = min(total_rows - 1, qb * 64 + 63);
  const int kend = qpos0 + last_row / G + 1;  // exclusive
  int kbeg = 0;
  if (p.window > 0) kbeg = max(0, qpos0 + (qb * 64) / G - p.window + 1);
  kbeg = kbeg / KC * KC;
  const int nchunks = (kend - kbeg + KC - 1) / KC;

  load_kv_chunk<HD>(sk0, sv0, p, row, kvh, kbeg, kend);
  cp_async_commit();

  cp_async_wait<1>();
  __syncthreads();
  uint32_t qf[HD / 16][4];
#pragma unroll
  for (int kk = 0; kk < HD / 16; ++kk) {
    const int r = warp * 16 + (lane & 15), chunk = kk * 2 + (lane >> 4);
    ldsm_x4(sq + swz<HD>(r, chunk), qf[kk][0], qf[kk][1], qf[kk][2], qf[kk][3]);
  }

  // per-thread rows and their query positions
  int qpos[2];
#pragma unroll
  for (int h = 0; h < 2; ++h) {
    const int gr = qb * 64 + warp * 16 + (lane >> 2) + 8 * h;
    qpos[h] = gr < total_rows ? qpos0 + gr / G : -1;
  }
  float m[2] = {-INFINITY, -INFINITY}, l[2] = {0.f, 0.f};
  float o[HD / 8][4];
#pragma unroll
  for (int i = 0; i < HD / 8; ++i) o[i][0] = o[i][1] = o[i][2] = o[i][3] = 0.f;

  for (int ci = 0; ci < nchunks; ++ci) {
    const int buf = ci & 1;
    if (ci + 1 < nchunks) {
      load_kv_chunk<HD>(sk0 + (buf ^ 1) * KC * HD * 2, sv0 + (buf ^ 1) * KC * HD * 2, p, row, kvh,
                        kbeg + (ci + 1) * KC, kend);
    }
    cp_async_commit();
    cp_async_wait<1>();
    __syncthreads();
    const uint32_t sk = sk0 + buf * KC * HD * 2, sv = sv0 + buf * KC * HD * 2;
    const int k0 = kbeg + ci * KC;
    float s[8][4];
    qk<HD, 8>(s, qf, sk, 0);
#pragma unroll
    for (int nt = 0; nt < 8; ++nt) {
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int h = e >> 1;
        const int kp = k0 + nt * 8 + 2 * (lane & 3) + (e & 1);
        bool ok = kp <= qpos[h] && kp < kend;
        if (p.window > 0) ok = ok && kp > qpos[h] - p.window;
        s[nt][e] = ok ? s[nt][e] * p.scale_log2 : -INFINITY;
      }
    }
    float so[2];
    softmax_update<8>(s, m, l, so);
#pragma unroll
    for (int i = 0; i < HD / 8; ++i) {
      o[i][0] *= so[0]; o[i][1] *= so[0]; o[i][2] *= so[1]; o[i][3] *= so[1];
    }
    uint32_t pf[4][4];
    pack_p<8>(pf, s);
    pv<HD, 4>(o, pf, sv, 0);
    __syncthreads();
  }
  cp_async_wait<0>();

  // finalize (+ sinks) and store
#pragma unroll
  for (int h = 0; h < 2; ++h) {
    const int gr = qb * 64 + warp * 16 + (lane >> 2) + 8 * h;
    if (gr >= total_rows) continue;
    const int t = gr / G, g = gr % G, head = kvh * G + g;
    float mm = m[h], ll = l[h], f = 1.f;
    if (p.sinks != nullptr) {
      const float sk = p.sinks[head] * kLog2e;
      const float mn = fmaxf(mm, sk);
      f = exp2f(mm - mn);
      ll = ll * f + exp2f(sk - mn);
    }
    const float inv = ll > 0.f ? f / ll : 0.f;
    __nv_bfloat16* dst = p.o + ((int64_t)(q0 + t) * p.nq + head) * HD;
#pragma unroll
    for (int i = 0; i < HD / 8; ++i) {
      const int col = i * 8 + 2 * (lane & 3);
      *reinterpret_cast<uint32_t*>(dst + col) = pack_bf16(o[i][2 * h] * inv, o[i][2 * h + 1] * inv);
    }
  }
}

// ================================================================================ decode
// grid (requests, kv heads, splits). The G query heads of the group are the 16 MMA rows
// (padded); the 4 warps take 16-key quarters of each 64-key chunk and merge at the end.
// The KV slots of the CTA's key range are fetched into smem once up front (segments of kSlots),
// so the cp.async ring (kDecStages deep) never waits on a dependent page-table load.
constexpr int kDecStages = 3;
constexpr int kSlots = 2048;

template <int HD>
__device__ __forceinline__ void load_kv_chunk_slots(uint32_t sk, uint32_t sv, const AttnParams& p,
                                                    const int32_t* slots, int kvh, int k0, int kend, int seg0) {
  constexpr int CH = HD / 8;
#pragma unroll
  for (int i = 0; i < KC * CH / (kWarps * 32); ++i) {
    const int c = threadIdx.x + i * kWarps * 32;
    const int key = c / CH, part = c % CH;
    const int pos = k0 + key;
    const bool valid = pos < kend;
    const int64_t slot = valid ? slots[pos - seg0] : 0;
    const int64_t off = slot * p.cache_stride + (int64_t)kvh * HD + part * 8;
    cp_async16(sk + swz<HD>(key, part), p.k + off, valid);
    cp_async16(sv + swz<HD>(key, part), p.v + off, valid);
  }
}

template <int HD>
__global__ void __launch_bounds__(kWarps * 32) decode_kernel(AttnParams p) {
  extern __shared__ __align__(128) uint8_t smem[];
  pdl_wait();
  pdl_launch();
  // KV heads vary fastest across the grid: the heads of one request share every 2 KB token row
  // of the cache, so fetching them together keeps DRAM rows open.
  const int kvh = blockIdx.x, b = blockIdx.y, split = blockIdx.z;
  const int G = p.group;
  const int L = p.kv_lens[b], row = p.rows[b];
  if (!MSGL_IN_BOUNDS(row >= 0 && L >= 0 && L <= p.pt_stride, kBcAttnRow)) return;  // CTA-uniform
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  constexpr int CH = HD / 8;
  constexpr int kStageBytes = 2 * KC * HD * 2;

  int lo = 0;
  if (p.window > 0) lo = max(0, L - p.window);
  const int nchunk_total = (L - lo + KC - 1) / KC;
  const int per = (nchunk_total + p.num_splits - 1) / p.num_splits;
  const int kbeg = lo + split * per * KC;
  const int kend = min(L, kbeg + per * KC);

  const uint32_t sq = smem_u32(smem);
  int32_t* slots = reinterpret_cast<int32_t*>(smem + 16 * HD * 2);
  const uint32_t ring = smem_u32(smem + 16 * HD * 2 + kSlots * 4);
  // merge scratch aliases the ring, which is idle once the key loop has drained
  float* red = reinterpret_cast<float*>(smem + 16 * HD * 2 + kSlots * 4);

  for (int c = threadIdx.x; c < 16 * CH; c += kWarps * 32) {
    const int r = c / CH, part = c % CH;
    const bool valid = r < G;
    const __nv_bfloat16* src = p.q + ((int64_t)b * p.nq + kvh * G + (valid ? r : 0)) * HD + part * 8;
    cp_async16(sq + swz<HD>(r, part), src, valid);
  }
  cp_async_commit();

  float m[2] = {-INFINITY, -INFINITY}, l[2] = {0.f, 0.f};
  float o[HD / 8][4];
#pragma unroll
  for (int i = 0; i < HD / 8; ++i) o[i][0] = o[i][1] = o[i][2] = o[i][3] = 0.f;
  uint32_t qf[HD / 16][4];
  bool have_q = false;
  const int32_t* pt = p.page_table + (int64_t)row * p.pt_stride;

  for (int seg0 = kbeg; seg0 < kend; seg0 += kSlots) {
    const int seg1 = min(kend, seg0 + kSlots);
    __syncthreads();  // previous segment's readers are done with `slots`
    for (int i = threadIdx.x; i < seg1 - seg0; i += kWarps * 32) {
      int sl = pt[seg0 + i];
      if (!MSGL_IN_BOUNDS(sl >= 0 && sl < p.num_slots, kBcAttnSlot)) sl = 0;
      slots[i] = sl;
    }
    __syncthreads();
    const int nchunks = (seg1 - seg0 + KC - 1) / KC;
#pragma unroll
    for (int s = 0; s < kDecStages - 1; ++s) {
      if (s < nchunks)
        load_kv_chunk_slots<HD>(ring + s * kStageBytes, ring + s * kStageBytes + KC * HD * 2, p, slots, kvh,
                                seg0 + s * KC, seg1, seg0);
      cp_async_commit();
    }
    for (int ci = 0; ci < nchunks; ++ci) {
      cp_async_wait<kDecStages - 2>();
      __syncthreads();
      if (!have_q) {
#pragma unroll
        for (int kk = 0; kk < HD / 16; ++kk) {
          const int r = lane & 15, chunk = kk * 2 + (lane >> 4);
          ldsm_x4(sq + swz<HD>(r, chunk), qf[kk][0], qf[kk][1], qf[kk][2], qf[kk][3]);
        }
        have_q = true;
      }
      {
        const int nx = ci + kDecStages - 1;
        const int st = nx % kDecStages;
        if (nx < nchunks)
          load_kv_chunk_slots<HD>(ring + st * kStageBytes, ring + st * kStageBytes + KC * HD * 2, p, slots, kvh,
                                  seg0 + nx * KC, seg1, seg0);
        cp_async_commit();
      }
      const int st = ci % kDecStages;
      const uint32_t sk = ring + st * kStageBytes, sv = sk + KC * HD * 2;
      const int k0 = seg0 + ci * KC + warp * 16;
      float s[2][4];
      qk<HD, 2>(s, qf, sk, warp * 16);
#pragma unroll
      for (int nt = 0; nt < 2; ++nt)
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const int kp = k0 + nt * 8 + 2 * (lane & 3) + (e & 1);
          s[nt][e] = kp < seg1 ? s[nt][e] * p.scale_log2 : -INFINITY;
        }
      float so[2];
      softmax_update<2>(s, m, l, so);
#pragma unroll
      for (int i = 0; i < HD / 8; ++i) {
        o[i][0] *= so[0]; o[i][1] *= so[0]; o[i][2] *= so[1]; o[i][3] *= so[1];
      }
      uint32_t pf[1][4];
      pack_p<2>(pf, s);
      pv<HD, 1>(o, pf, sv, warp * 16);
    }
    cp_async_wait<0>();
  }
  cp_async_wait<0>();
  __syncthreads();

  // merge the 4 warps: rows (lane/4) and (lane/4 + 8); only rows < G matter.
  float* rm = red;
  float* rl = red + kWarps * 16;
  float* ro = red + 2 * kWarps * 16;
#pragma unroll
  for (int h = 0; h < 2; ++h) {
    const int r = (lane >> 2) + 8 * h;
    if ((lane & 3) == 0) {
      rm[warp * 16 + r] = m[h];
      rl[warp * 16 + r] = l[h];
    }
#pragma unroll
    for (int i = 0; i < HD / 8; ++i) {
      const int col = i * 8 + 2 * (lane & 3);
      ro[(warp * 16 + r) * HD + col] = o[i][2 * h];
      ro[(warp * 16 + r) * HD + col + 1] = o[i][2 * h + 1];
    }
  }
  __syncthreads();
  for (int idx = threadIdx.x; idx < G * HD; idx += kWarps * 32) {
    const int r = idx / HD, col = idx % HD;
    float mx = -INFINITY;
#pragma unroll
    for (int w = 0; w < kWarps; ++w) mx = fmaxf(mx, rm[w * 16 + r]);
    const float base = mx == -INFINITY ? 0.f : mx;
    float ll = 0.f, acc = 0.f;
#pragma unroll
    for (int w = 0; w < kWarps; ++w) {
      const float f = exp2f(rm[w * 16 + r] - base);
      ll += rl[w * 16 + r] * f;
      acc += ro[(w * 16 + r) * HD + col] * f;
    }
    const int head = kvh * G + r;
    if (p.num_splits == 1) {
      float f = 1.f;
      if (p.sinks != nullptr) {
        const float sk = p.sinks[head] * kLog2e;
        const float mn = fmaxf(mx, sk);
        f = exp2f(base - mn);
        ll = ll * f + exp2f(sk - mn);
      }
      const float v = ll > 0.f ? acc * f / ll : 0.f;
      p.o[((int64_t)b * p.nq + head) * HD + col] = __float2bfloat16(v);
    } else {
      const int64_t slot = ((int64_t)b * p.nq + head) * p.num_splits + split;
      p.ws[slot * HD + col] = acc;
      if (col == 0) {
        float* ml = p.ws + (int64_t)gridDim.y * p.nq * p.num_splits * HD;
        ml[slot * 2] = mx;
        ml[slot * 2 + 1] = ll;
      }
    }
  }
}

// merge split partials: one warp per (request, head)
template <int HD>
__global__ void decode_combine_kernel(AttnParams p, int bs) {
  pdl_wait();
  pdl_launch();
  const int gw = blockIdx.x * (blockDim.x / 32) + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (gw >= bs * p.nq) return;
  const int head = gw % p.nq;
  const float* ml = p.ws + (int64_t)bs * p.nq * p.num_splits * HD;
  float mx = -INFINITY;
  for (int s = 0; s < p.num_splits; ++s) mx = fmaxf(mx, ml[((int64_t)gw * p.num_splits + s) * 2]);
  float sink = -INFINITY;
  if (p.sinks != nullptr) sink = p.sinks[head] * kLog2e;
  const float mn = fmaxf(mx, sink);
  const float base = mn == -INFINITY ? 0.f : mn;
  float ll = p.sinks != nullptr ? exp2f(sink - base) : 0.f;
  float acc[HD / 32];
#pragma unroll
  for (int i = 0; i < HD / 32; ++i) acc[i] = 0.f;
  for (int s = 0; s < p.num_splits; ++s) {
    const int64_t slot = (int64_t)gw * p.num_splits + s;
    const float f = exp2f(ml[slot * 2] - base);
    ll += ml[slot * 2 + 1] * f;
#pragma unroll
    for (int i = 0; i < HD / 32; ++i) acc[i] += p.ws[slot * HD + lane + 32 * i] * f;
  }
  const float inv = ll > 0.f ? 1.f / ll : 0.f;
#pragma unroll
  for (int i = 0; i < HD / 32; ++i)
    p.o[(int64_t)gw * HD + lane + 32 * i] = __float2bfloat16(acc[i] * inv);
}

template <int HD>
int prefill_smem() { return 64 * HD * 2 + 4 * KC * HD * 2; }
template <int HD>
int decode_smem() {
  static_assert((2 * kWarps * 16 + kWarps * 16 * HD) * 4 <= kDecStages * 2 * KC * HD * 2,
                "merge scratch must fit the K/V ring");
  return 16 * HD * 2 + kSlots * 4 + kDecStages * 2 * KC * HD * 2;
}

template <int HD>
void run_prefill(const AttnParams& p, int num_reqs, int max_q_len, cudaStream_t s) {
  msgl_set_smem<prefill_kernel<HD>>(prefill_smem<HD>());
  const dim3 grid((max_q_len * p.group + 63) / 64, num_reqs, p.nkv);
  msgl_launch(prefill_kernel<HD>, grid, dim3(kWarps * 32), prefill_smem<HD>(), s, 1, p);
}

// Returns the first CUDA error of the attribute call or the launches (cudaSuccess if all went out).
template <int HD>
cudaError_t run_decode(const AttnParams& p, int bs, cudaStream_t s) {
  cudaError_t e = msgl_set_smem<decode_kernel<HD>>(decode_smem<HD>());
  if (e != cudaSuccess) return e;
  const dim3 grid(p.nkv, bs, p.num_splits);
  e = msgl_launch(decode_kernel<HD>, grid, dim3(kWarps * 32), decode_smem<HD>(), s, 1, p);
  if (e == cudaSuccess && p.num_splits > 1) {
    const int warps = bs * p.nq;
    e = msgl_launch(decode_combine_kernel<HD>, dim3((warps + 7) / 8), dim3(256), 0, s, 1, p, bs);
  }
  return e;
}

AttnParams make_params(void* o, const void* q, const void* k, const void* v, const int32_t* pt,
                       int64_t pt_stride, const int32_t* rows, const int32_t* cu_q, const int32_t* kv_lens,
                       int nq, int nkv, int64_t cache_stride, float sm_scale, int window,
                       const float* sinks, int64_t num_slots = INT64_MAX) {
  AttnParams p;
  p.o = reinterpret_cast<__nv_bfloat16*>(o);
  p.q = reinterpret_cast<const __nv_bfloat16*>(q);
  p.k = reinterpret_cast<const __nv_bfloat16*>(k);
  p.v = reinterpret_cast<const __nv_bfloat16*>(v);
  p.page_table = pt;
  p.pt_stride = pt_stride;
  p.rows = rows;
  p.cu_q = cu_q;
  p.kv_lens = kv_lens;
  p.nq = nq;
  p.nkv = nkv;
  p.group = nq / nkv;
  p.cache_stride = cache_stride;
  p.num_slots = num_slots;
  p.scale_log2 = sm_scale * kLog2e;
  p.window = window;
  p.sinks = sinks;
  p.num_splits = 1;
  p.ws = nullptr;
  return p;
}

}  // namespace

extern "C" void msgl_attention_prefill(void* o, const void* q, const void* k_cache, const void* v_cache,
                                       const int32_t* page_table, int64_t pt_stride, const int32_t* rows,
                                       const int32_t* cu_q, const int32_t* kv_lens, int num_reqs,
                                       int total_q, int max_q_len, int nq, int nkv, int hd,
                                       int64_t cache_stride, int64_t num_slots, float sm_scale, int window,
                                       const float* sinks, cudaStream_t s) {
  if (num_reqs == 0 || total_q == 0) return;
  AttnParams p = make_params(o, q, k_cache, v_cache, page_table, pt_stride, rows, cu_q, kv_lens, nq,
                             nkv, cache_stride, sm_scale, window, sinks, num_slots);
  if (hd == 64) run_prefill<64>(p, num_reqs, max_q_len, s);
  else run_prefill<128>(p, num_reqs, max_q_len, s);
}

extern "C" void msgl_attention_decode(void* o, const void* q, const void* k_cache, const void* v_cache,
                                      const int32_t* page_table, int64_t pt_stride, const int32_t* rows,
                                      const int32_t* kv_lens, int bs, int nq, int nkv, int hd,
                                      int64_t cache_stride, int64_t num_slots, float sm_scale, int window,
                                      const float* sinks, int num_splits, void* workspace,
                                      cudaStream_t s) {
  if (bs == 0) return;
  AttnParams p = make_params(o, q, k_cache, v_cache, page_table, pt_stride, rows, nullptr, kv_lens,
                             nq, nkv, cache_stride, sm_scale, window, sinks, num_slots);
  p.num_splits = num_splits < 1 ? 1 : num_splits;
  p.ws = reinterpret_cast<float*>(workspace);
  if (hd == 64) run_decode<64>(p, bs, s);
  else run_decode<128>(p, bs, s);
}

MSGL_ERROR_ACCESSOR(msgl_err_attention)

// ================================================================================ decode (paged)
// Persistent decode attention over a host-built work list, for page sizes of 16, 32 or 64 tokens.
//
// Work: each request's keys are cut into chunks of whole 64-key blocks; an entry is one chunk
// (request b, blocks [blk0, blk1), chunk j of nchunks, partial slot base), and an item is an
// (entry, kv head) pair. The host sorts entries longest first; CTA c of P takes items in snake
// order (c, 2P-1-c, 2P+c, ...), which balances variable context lengths without atomics.
//
// Warp roles (192 threads, one CTA per SM):
//   warp 5     scheduler: resolves items ahead of use (work entry, length, page-table row and the
//              first slot of every page of the chunk) into a ring of kPdDesc smem descriptors, so
//              the dependent global loads never stall the data path.
//   warp 0     TMA producer: per item the query tile (16 rows, G valid), then per page one 3-D box
//              (64 head dims x 1 head x page) per column half of K and of V from the
//              [slots, kv heads, head dim] cache into a 128-byte-swizzled ring of kPdStages
//              64-key stages.
//   warps 1-4  each take 16 keys of every block (mma.sync m16n8k16 with the G query heads as MMA
//              rows, online softmax in the log2 domain) and merge at the end of the item.
// A single-chunk request writes its output directly; otherwise each chunk writes an fp32 partial,
// and the last chunk of the (request, head) to arrive (gpu-scope acq_rel counter) combines them.
namespace {

constexpr int kPdStages = 5;
constexpr int kPdConsumers = 4;
constexpr int kPdDesc = 4;          // descriptor ring depth (items resolved ahead)
constexpr int kPdMaxGroups = 256;   // pages per item (64 blocks of 16-token pages)
constexpr int kPdMaxChunks = 128;   // chunks per request (combine scratch)
constexpr int kPdThreads = 32 * (2 + kPdConsumers);

struct PagedDecodeParams {
  __nv_bfloat16* o;
  const int32_t* page_table;
  int64_t pt_stride;
  int64_t num_slots;
  const int32_t* rows;
  const int32_t* kv_lens;
  const int4* work;       // per entry two int4: {b, blk0, blk1, j}, {nchunks, slot0, -, -}
  const int32_t* n_work;  // number of entries (device scalar)
  float* ws;              // partial o [slot][nkv][G][HD], then (m, l) [slot][nkv][G][2]
  int ws_slots;
  int32_t* counters;      // [bs][nkv] arrivals; every launch leaves them at zero
  const float* sinks;
  int nq, nkv, group, page;
  float scale_log2;
  int window;
};

// one resolved item
struct PdDesc {
  int b, kvh, first, blk1, j, nchunks, slot0, L, lo, valid, pad[6];
  int slots[kPdMaxGroups];  // first cache slot of each page of blocks [first, blk1)
};

template <int HD>
struct PdCfg {
  static constexpr int kHalfTile = 64 * 128;            // 64 rows x 64 head dims (bf16)
  static constexpr int kTile = 64 * HD * 2;             // one 64-key K or V block
  static constexpr int kStage = 2 * kTile;
  static constexpr int kQ = 16 * HD * 2;                // 16 query rows (G <= 16, padded)
  // merge scratch (4 warps' m, l, o rows), reused by the combine ([chunks][16] m and weights + [16])
  static constexpr int kMerge = std::max((kPdConsumers * 16 * HD + 2 * kPdConsumers * 16) * 4,
                                         (2 * kPdMaxChunks * 16 + 16) * 4);
  static constexpr int kSmem = 1024 + kPdStages * kStage + 2 * kQ + kMerge + kPdDesc * (int)sizeof(PdDesc) + 256;
};

// byte offset of (row, 16-byte chunk c) in a [rows][HD] bf16 tile stored as HD/64 column halves
// of [rows][128 B] with the TMA 128-byte swizzle (chunk XOR row % 8)
__device__ __forceinline__ uint32_t swz_tma(int row, int c, int rows) {
  return (uint32_t)((c >> 3) * rows * 128 + row * 128 + (((c & 7) ^ (row & 7)) << 4));
}

template <int HD>
__device__ __forceinline__ void qk_tma(float (&s)[2][4], const uint32_t (&qf)[HD / 16][4], uint32_t sk, int key0) {
  const int lane = threadIdx.x & 31;
#pragma unroll
  for (int n = 0; n < 2; ++n) s[n][0] = s[n][1] = s[n][2] = s[n][3] = 0.f;
#pragma unroll
  for (int kk = 0; kk < HD / 16; ++kk) {
    const int idx = lane >> 3;
    const int key = key0 + (idx >> 1) * 8 + (lane & 7);
    const int chunk = kk * 2 + (idx & 1);
    uint32_t b0, b1, b2, b3;
    ldsm_x4(sk + swz_tma(key, chunk, 64), b0, b1, b2, b3);
    mma_bf16(s[0], qf[kk], b0, b1);
    mma_bf16(s[1], qf[kk], b2, b3);
  }
}

template <int HD>
__device__ __forceinline__ void pv_tma(float (&o)[HD / 8][4], const uint32_t (&pf)[4], uint32_t sv, int key0) {
  const int lane = threadIdx.x & 31;
#pragma unroll
  for (int n = 0; n < HD / 8; n += 2) {
    const int idx = lane >> 3;
    const int key = key0 + (idx & 1) * 8 + (lane & 7);
    const int chunk = n + (idx >> 1);
    uint32_t b0, b1, b2, b3;
    ldsm_x4_t(sv + swz_tma(key, chunk, 64), b0, b1, b2, b3);
    mma_bf16(o[n], pf, b0, b1);
    mma_bf16(o[n + 1], pf, b2, b3);
  }
}

__device__ __forceinline__ void pd_consumer_sync() { asm volatile("bar.sync 1, %0;" ::"n"(kPdConsumers * 32) : "memory"); }

// item r of this CTA in snake order; false when the CTA has no more work
__device__ __forceinline__ bool pd_item(const PagedDecodeParams& p, int n_items, int r, int& e, int& kvh) {
  const int P = gridDim.x, c = blockIdx.x;
  const int idx = r * P + ((r & 1) ? (P - 1 - c) : c);
  if (idx >= n_items) return false;
  e = idx / p.nkv;
  kvh = idx - e * p.nkv;
  return true;
}

template <int HD>
__global__ void __launch_bounds__(kPdThreads, 1)
paged_decode_kernel(const __grid_constant__ CUtensorMap tk, const __grid_constant__ CUtensorMap tv,
                    const __grid_constant__ CUtensorMap tq, PagedDecodeParams p) {
  using C = PdCfg<HD>;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* ring = smem;
  uint8_t* sq = ring + kPdStages * C::kStage;
  float* red = reinterpret_cast<float*>(sq + 2 * C::kQ);
  PdDesc* desc = reinterpret_cast<PdDesc*>(reinterpret_cast<uint8_t*>(red) + C::kMerge);
  uint64_t* bars = reinterpret_cast<uint64_t*>(desc + kPdDesc);
  uint64_t* full = bars;
  uint64_t* empty = bars + kPdStages;
  uint64_t* qfull = bars + 2 * kPdStages;
  uint64_t* qempty = qfull + 2;
  uint64_t* dfull = qempty + 2;
  uint64_t* dempty = dfull + kPdDesc;
  int* flag = reinterpret_cast<int*>(dempty + kPdDesc);
  volatile int* abort_flag = flag + 1;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    for (int i = 0; i < kPdStages; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], kPdConsumers);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&qfull[i], 1);
      mbar_init(&qempty[i], kPdConsumers);
    }
    for (int i = 0; i < kPdDesc; ++i) {
      mbar_init(&dfull[i], 1);
      mbar_init(&dempty[i], 1 + kPdConsumers);  // producer + consumer warps
    }
    *abort_flag = 0;
    fence_barrier_init();
    prefetch_tmap(&tk);
    prefetch_tmap(&tv);
    prefetch_tmap(&tq);
  }
  __syncthreads();
  pdl_wait();
  pdl_launch();
  const int n_items = *p.n_work * p.nkv;
  const int G = p.group;

  if (warp == 5) {
    // ------------------------------------------------------------------ scheduler
    const int g = p.page, gpb = 64 / g;
    int e, kvh;
    for (int r = 0;; ++r) {
      const bool valid = pd_item(p, n_items, r, e, kvh);
      const int d = r % kPdDesc;
      if (lane == 0 && !mbar_wait(&dempty[d], ((r / kPdDesc) & 1) ^ 1, 430)) break;
      __syncwarp();
      PdDesc& D = desc[d];
      if (valid) {
        const int4 w0 = p.work[2 * e];
        const int4 w1 = p.work[2 * e + 1];
        const int b = w0.x;
        const int L = p.kv_lens[b];
        const int lo = p.window > 0 ? max(0, L - p.window) : 0;
        const int first = max(w0.y, lo / 64), blk1 = w0.z;
        const int32_t* pt = p.page_table + (int64_t)p.rows[b] * p.pt_stride;
        int ngroups = min(kPdMaxGroups, max(0, blk1 - first) * gpb);
        if (!MSGL_IN_BOUNDS(p.rows[b] >= 0 && L >= 0 && L <= p.pt_stride, kBcAttnRow)) ngroups = 0;  // warp-uniform
        for (int gi = lane; gi < ngroups; gi += 32) {
          const int pos = first * 64 + gi * g;
          int sl = pos < L ? pt[pos] : 0;
          if (!MSGL_IN_BOUNDS(sl >= 0 && sl < p.num_slots, kBcAttnSlot)) sl = 0;
          D.slots[gi] = sl;
        }
        if (lane == 0) {
          D.b = b; D.kvh = kvh; D.first = first; D.blk1 = first + ngroups / gpb; D.j = w0.w;
          D.nchunks = w1.x; D.slot0 = w1.y; D.L = L; D.lo = lo; D.valid = 1;
        }
      } else if (lane == 0) {
        D.valid = 0;
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&dfull[d]);  // release: the descriptor writes above
      if (!valid) break;
    }
  } else if (warp == 0) {
    // ------------------------------------------------------------------ TMA producer
    const int g = p.page, gpb = 64 / g;
    int stage = 0;
    uint32_t phase = 0;
    if (lane == 0) {
      for (int r = 0;; ++r) {
        const int d = r % kPdDesc;
        if (!mbar_wait(&dfull[d], (r / kPdDesc) & 1, 440)) break;
        const PdDesc& D = desc[d];
        if (!D.valid) break;
        const int qb = r & 1;
        bool ok = mbar_wait(&qempty[qb], ((r >> 1) & 1) ^ 1, 441);
        if (ok) {
          mbar_expect_tx(&qfull[qb], C::kQ);
#pragma unroll
          for (int h = 0; h < HD / 64; ++h)
            tma_load_2d(sq + qb * C::kQ + h * 16 * 128, &tq, &qfull[qb], h * 64, D.b * p.nq + D.kvh * G);
        }
        const int ngroups = (D.blk1 - D.first) * gpb;
        for (int gi = 0; ok && gi < ngroups; ++gi) {
          const int sub = gi % gpb;
          if (sub == 0) {
            if (!mbar_wait(&empty[stage], phase ^ 1, 442)) { ok = false; break; }
            mbar_expect_tx(&full[stage], C::kStage);
          }
          const int s0 = D.slots[gi];
          uint8_t* kt = ring + stage * C::kStage;
#pragma unroll
          for (int h = 0; h < HD / 64; ++h) {
            tma_load_3d(kt + h * C::kHalfTile + sub * g * 128, &tk, &full[stage], h * 64, D.kvh, s0);
            tma_load_3d(kt + C::kTile + h * C::kHalfTile + sub * g * 128, &tv, &full[stage], h * 64, D.kvh, s0);
          }
          if (sub == gpb - 1 && ++stage == kPdStages) { stage = 0; phase ^= 1; }
        }
        mbar_arrive(&dempty[d]);
        if (!ok) break;
      }
    }
  } else {
    // ------------------------------------------------------------------ consumers
    const int cw = warp - 1;
    const int ctid = threadIdx.x - 32;
    float* rm = red;
    float* rl = red + kPdConsumers * 16;
    float* ro = red + 2 * kPdConsumers * 16;
    int stage = 0;
    uint32_t phase = 0;
    // A warp whose wait times out (error recorded) raises abort_flag, skips the rest of the item
    // and still reaches the item's first consumer barrier, after which all consumer warps leave
    // together; so the named barriers never wait for a warp that has gone.
    bool dead = false;
    for (int r = 0;; ++r) {
      const int d = r % kPdDesc;
      if (!dead && !mbar_wait(&dfull[d], (r / kPdDesc) & 1, 450)) { dead = true; *abort_flag = 1; }
      const PdDesc& D = desc[d];
      if (!dead && !D.valid) break;  // end of work: every consumer warp reads the same descriptor
      const int b = D.b, kvh = D.kvh, first = D.first, blk1 = D.blk1, j = D.j, nchunks = D.nchunks;
      const int slot0 = D.slot0, L = D.L, lo = D.lo;

      const int qb = r & 1;
      if (!dead && !mbar_wait(&qfull[qb], (r >> 1) & 1, 451)) { dead = true; *abort_flag = 1; }
      uint32_t qf[HD / 16][4];
      const uint32_t qbase = smem_u32(sq + qb * C::kQ);
#pragma unroll
      for (int kk = 0; kk < HD / 16; ++kk)
        ldsm_x4(qbase + swz_tma(lane & 15, kk * 2 + (lane >> 4), 16), qf[kk][0], qf[kk][1], qf[kk][2], qf[kk][3]);
      __syncwarp();
      if (lane == 0) mbar_arrive(&qempty[qb]);

      float m[2] = {-INFINITY, -INFINITY}, l[2] = {0.f, 0.f};
      float o[HD / 8][4];
#pragma unroll
      for (int i = 0; i < HD / 8; ++i) o[i][0] = o[i][1] = o[i][2] = o[i][3] = 0.f;
      for (int blk = first; blk < blk1 && !dead; ++blk) {
        if (!mbar_wait(&full[stage], phase, 452)) { dead = true; *abort_flag = 1; break; }
        const uint32_t sk = smem_u32(ring + stage * C::kStage), sv = sk + C::kTile;
        float s[2][4];
        qk_tma<HD>(s, qf, sk, cw * 16);
        const int k0 = blk * 64 + cw * 16;
#pragma unroll
        for (int nt = 0; nt < 2; ++nt)
#pragma unroll
          for (int x = 0; x < 4; ++x) {
            const int kp = k0 + nt * 8 + 2 * (lane & 3) + (x & 1);
            s[nt][x] = (kp >= lo && kp < L) ? s[nt][x] * p.scale_log2 : -INFINITY;
          }
        float so[2];
        softmax_update<2>(s, m, l, so);
#pragma unroll
        for (int i = 0; i < HD / 8; ++i) {
          o[i][0] *= so[0]; o[i][1] *= so[0]; o[i][2] *= so[1]; o[i][3] *= so[1];
        }
        uint32_t pf[1][4];
        pack_p<2>(pf, s);
        pv_tma<HD>(o, pf[0], sv, cw * 16);
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[stage]);
        if (++stage == kPdStages) { stage = 0; phase ^= 1; }
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&dempty[d]);  // descriptor fields are in registers now

      // merge the 4 warps' rows (lane/4 and lane/4 + 8)
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        const int rr = (lane >> 2) + 8 * h;
        if ((lane & 3) == 0) {
          rm[cw * 16 + rr] = m[h];
          rl[cw * 16 + rr] = l[h];
        }
#pragma unroll
        for (int i = 0; i < HD / 8; ++i) {
          const int col = i * 8 + 2 * (lane & 3);
          *reinterpret_cast<float2*>(&ro[(cw * 16 + rr) * HD + col]) = make_float2(o[i][2 * h], o[i][2 * h + 1]);
        }
      }
      pd_consumer_sync();
      if (*abort_flag) break;
      const int64_t pslot = ((int64_t)(slot0 + j) * p.nkv + kvh) * G;  // partial row base
      float* ws_o = p.ws;
      float* ws_ml = p.ws + (int64_t)p.ws_slots * p.nkv * G * HD;
      for (int idx = ctid; idx < G * HD; idx += kPdConsumers * 32) {
        const int rr = idx / HD, col = idx - rr * HD;
        float mx = -INFINITY;
#pragma unroll
        for (int w = 0; w < kPdConsumers; ++w) mx = fmaxf(mx, rm[w * 16 + rr]);
        const float base = mx == -INFINITY ? 0.f : mx;
        float ll = 0.f, acc = 0.f;
#pragma unroll
        for (int w = 0; w < kPdConsumers; ++w) {
          const float f = exp2f(rm[w * 16 + rr] - base);
          ll += rl[w * 16 + rr] * f;
          acc += ro[(w * 16 + rr) * HD + col] * f;
        }
        const int head = kvh * G + rr;
        if (nchunks == 1) {
          float f = 1.f;
          if (p.sinks != nullptr) {
            const float skv = p.sinks[head] * kLog2e;
            const float mn = fmaxf(mx, skv);
            f = exp2f(base - mn);
            ll = ll * f + exp2f(skv - mn);
          }
          p.o[((int64_t)b * p.nq + head) * HD + col] = __float2bfloat16(ll > 0.f ? acc * f / ll : 0.f);
        } else {
          ws_o[(pslot + rr) * HD + col] = acc;
          if (col == 0) {
            ws_ml[(pslot + rr) * 2] = mx;
            ws_ml[(pslot + rr) * 2 + 1] = ll;
          }
        }
      }
      if (nchunks > 1) {
        // Publish: the barrier orders every consumer thread's partial stores before thread 0's
        // release (cumulative) add; the last arriver's acquire plus the next barrier orders the
        // other chunks' partials before this CTA's combine loads.
        pd_consumer_sync();
        if (ctid == 0) {
          int32_t* cnt = p.counters + (int64_t)b * p.nkv + kvh;
          int old;
          asm volatile("atom.add.acq_rel.gpu.s32 %0, [%1], 1;" : "=r"(old) : "l"(cnt) : "memory");
          const int last = old == nchunks - 1;
          if (last) *cnt = 0;
          *flag = last;
        }
        pd_consumer_sync();
        if (*flag) {
          // combine every chunk's partial of (b, kvh): (m, l) of all chunks into smem in one round
          // of loads, per-row weights, then each thread sums 4 columns over the chunks
          float* cm = red;                                  // [nchunks][G]
          float* cwt = red + kPdMaxChunks * 16;             // [nchunks][G] weights
          float* cinv = red + 2 * kPdMaxChunks * 16;        // [G]
          const int nc = min(nchunks, kPdMaxChunks);
          for (int i = ctid; i < nc * G; i += kPdConsumers * 32) {
            const int c = i / G, rr = i - c * G;
            const int64_t rowi = ((int64_t)(slot0 + c) * p.nkv + kvh) * G + rr;
            const float2 ml = __ldcg(reinterpret_cast<const float2*>(ws_ml) + rowi);
            cm[i] = ml.x;
            cwt[i] = ml.y;
          }
          pd_consumer_sync();
          for (int rr = ctid; rr < G; rr += kPdConsumers * 32) {
            float mx = p.sinks != nullptr ? p.sinks[kvh * G + rr] * kLog2e : -INFINITY;
            const float sink = mx;
            for (int c = 0; c < nc; ++c) mx = fmaxf(mx, cm[c * G + rr]);
            const float base = mx == -INFINITY ? 0.f : mx;
            float ll = p.sinks != nullptr ? exp2f(sink - base) : 0.f;
            for (int c = 0; c < nc; ++c) {
              const float f = exp2f(cm[c * G + rr] - base);
              ll += cwt[c * G + rr] * f;
              cwt[c * G + rr] = f;
            }
            cinv[rr] = ll > 0.f ? 1.f / ll : 0.f;
          }
          pd_consumer_sync();
          for (int i = ctid; i < G * HD / 4; i += kPdConsumers * 32) {
            const int rr = i / (HD / 4), c4 = i - rr * (HD / 4);
            float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll 4
            for (int c = 0; c < nc; ++c) {
              const int64_t rowi = ((int64_t)(slot0 + c) * p.nkv + kvh) * G + rr;
              const float4 v = __ldcg(reinterpret_cast<const float4*>(ws_o + rowi * HD) + c4);
              const float f = cwt[c * G + rr];
              acc.x += v.x * f; acc.y += v.y * f; acc.z += v.z * f; acc.w += v.w * f;
            }
            const float inv = cinv[rr];
            __nv_bfloat16* dst = p.o + ((int64_t)b * p.nq + kvh * G + rr) * HD + c4 * 4;
            *reinterpret_cast<uint2*>(dst) = make_uint2(pack_bf16(acc.x * inv, acc.y * inv), pack_bf16(acc.z * inv, acc.w * inv));
          }
        }
      }
      pd_consumer_sync();  // merge scratch and flag are reused by the next item
    }
  }
}

typedef CUresult (*PdEncodeFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                               const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                               CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

PdEncodeFn pd_encode_fn() {
  static PdEncodeFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PdEncodeFn>(ptr);
  });
  return fn;
}

bool pd_encode(CUtensorMap* m, const void* base, int rank, const cuuint64_t* dims, const cuuint64_t* strides,
               const cuuint32_t* box) {
  memset(m, 0, sizeof(*m));
  PdEncodeFn fn = pd_encode_fn();
  if (fn == nullptr) return false;
  const cuuint32_t estr[3] = {1, 1, 1};
  return fn(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, rank, const_cast<void*>(base), dims, strides, box, estr,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

template <int HD>
int run_paged_decode(const PagedDecodeParams& p, const void* q, int q_rows, const void* k, const void* v,
                     int64_t num_slots, int64_t cache_stride, cudaStream_t s) {
  using C = PdCfg<HD>;
  msgl_set_smem<paged_decode_kernel<HD>>(C::kSmem);
  CUtensorMap tk, tv, tq;
  const cuuint64_t kdims[3] = {(cuuint64_t)HD, (cuuint64_t)p.nkv, (cuuint64_t)num_slots};
  const cuuint64_t kstr[2] = {(cuuint64_t)HD * 2, (cuuint64_t)cache_stride * 2};
  const cuuint32_t kbox[3] = {64, 1, (cuuint32_t)p.page};
  const cuuint64_t qdims[2] = {(cuuint64_t)HD, (cuuint64_t)q_rows};
  const cuuint64_t qstr[1] = {(cuuint64_t)HD * 2};
  const cuuint32_t qbox[2] = {64, 16};
  if (!pd_encode(&tk, k, 3, kdims, kstr, kbox) || !pd_encode(&tv, v, 3, kdims, kstr, kbox) ||
      !pd_encode(&tq, q, 2, qdims, qstr, qbox))
    return 2;
  int sms = 0, dev = 0;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  msgl_launch(paged_decode_kernel<HD>, dim3(sms), dim3(kPdThreads), C::kSmem, s, 1, tk, tv, tq, p);
  return 0;
}

}  // namespace

// ================================================================================ prefill (tcgen05)
// Ragged causal prefill attention on the 5th-generation tensor core, for head_dim 128 and page
// sizes of 16 / 32 / 64 tokens. The work items are (query tile, kv head) pairs: a tile is TT = 128 /
// G tokens of one request, whose TT x G packed (token, head) rows are the MMA M = 128 rows (G =
// query heads per kv head), so every K/V tile fetched serves the whole group. The kernel is
// persistent with two CTAs per SM (~113 KB of shared memory and 256 TMEM columns each); a CTA
// takes work items one at a time from a device counter (largest tile of each request first) and
// its roles run through them as independent streams, so the loads of the next tile overlap the
// softmax and epilogue of the current one and the two CTAs of an SM fill each other's gaps.
//
//   warp 0     producer: looks each tile up (a prefix scan of the requests' tile counts), publishes
//              it in a 4-entry tile ring, and streams TMA loads: the tile's Q (3-D box 64 dims x G
//              heads x TT tokens, per 64-dim half) once the previous tile's last QK^T is done, then
//              per 64-key block the K pages and the V pages (3-D boxes over [slots, kv heads, head
//              dim]) into a 2-stage K ring and a 3-stage V ring (V waits on the later consumer).
//              Whichever load can go goes first (a new tile's Q, then K, then V, then the next
//              tile), so a V load waiting for a PV never holds back K; an idle pass sleeps briefly
//              so the polling leaves issue slots to the softmax.
//   warp 1     MMA issuer, out of order between two streams: S_i = Q K_i^T into TMEM buffer i % 2
//              (i counts key blocks across tiles) once K_i has landed and that buffer's previous PV
//              is done; O += P_i V_i once the softmax has written P_i and V_i has landed (a tile's
//              first PV also waits until the softmax has read the previous tile's O). P is read
//              straight from TMEM (the A operand), V from shared memory as an MN-major operand.
//   warps 2-5  softmax, one thread per row (TMEM lane): read the S row, mask (causal / length /
//              window) only on blocks that cross the row's limits, online max and sum in the log2
//              domain, and write P as packed bf16 over the first 32 columns of its own S buffer. O
//              is rescaled in TMEM only when a row's max grows by more than 2^8 (lazy rescaling: P
//              then stays <= 256). Epilogue: O is read out of TMEM (and released), then O / l (with
//              the sink term) stored as bf16.
// TMEM: S / P buffers at columns 0 and 64, O at 128 (256 allocated).
namespace {

constexpr int kFmKB = 64;  // keys per block
constexpr int kFmThreads = 192;
constexpr int kFmKStages = 2, kFmVStages = 3;
constexpr int kFmRing = 4;  // tile-info ring entries

struct FmhaParams {
  __nv_bfloat16* o;
  const int32_t* page_table;
  int64_t pt_stride;
  int64_t num_slots;
  const int32_t* rows;
  const int32_t* cu_q;
  const int32_t* kv_lens;
  const float* sinks;
  int nq, nkv, group, tt, page;
  float scale_log2;
  int window;
  int num_reqs;
  uint32_t* trace;  // optional per-CTA phase stamps of its first tile (profiling)
  int trace_ctas;
  uint32_t epoch;   // launch number (picks the work counter slot); 0: static round-robin
};

// Work distribution: CTAs take work items from a per-device counter with atomicAdd. Launch e uses
// counter slot e % kFmSlots; the last CTA to finish zeroes that slot and the next one, so a replay
// of the same launch and the next launch both start from zero (even after a launch that did not
// finish). Launches of this kernel on one device must be stream-ordered: each fetches only after
// the programmatic-launch wait, i.e. after the previous launch has completed.
constexpr int kFmSlots = 64;
__device__ int g_fmha_work[kFmSlots];
__device__ int g_fmha_exit[kFmSlots];

// trace slots (SM clock cycles since the CTA started, for the CTA's third tile): 1 tile published,
// 2 key blocks, 3 Q issued, 4 first QK^T issued, 5 dynamic smem base mod 1024; per key block i < 8: 8 + i K loads issued, 16 + i V loads
// issued, 24 + i S_i issued, 32 + i PV_i issued; first softmax warp: 40 + 4i S_i landed, 41 + 4i
// row max taken, 42 + 4i exponentials done, 43 + 4i P_i handed over; 80 last PV done, 81 O stored,
// 82 CTA done; 6 SM id, 7 / 83 %globaltimer / 32 at start / end, 84 tiles taken, 85 TMEM
// allocated, 86 past the programmatic-launch wait, 87 first work item fetched, 88 softmax starts
// the traced tile, 89 MMA takes it, 90-93 its first QK^T inputs ready (Q, K, S buffer, PV lag).
constexpr int kFmTrace = 96;

// One work item, as published in the tile ring (nb < 0: no more work).
struct FmTile {
  int b, q0, t0, t1, L, qpos0, blk0, nb, kvh, row, pad0, pad1;
};

struct FmSmem {
  static constexpr int kQHalf = 128 * 128;       // one 64-dim half of the 128-row Q tile
  static constexpr int kHalf = kFmKB * 128;      // one 64-dim half of a 64-key K / V tile
  static constexpr int kT = 2 * kHalf;           // one K or V stage
  static constexpr int kOffK = 2 * kQHalf;
  static constexpr int kOffV = kOffK + kFmKStages * kT;
  static constexpr int kTiles = kOffV + kFmVStages * kT;  // 1024-aligned operand tiles
  // tile ring + barriers: in front of the tiles when the alignment gap has room, else behind them
  static constexpr int kRingBytes = kFmRing * (int)sizeof(FmTile);
  static constexpr int kMeta = kRingBytes + 256;
  // the dynamic smem base is 16-byte aligned, so the gap to the next 1 KB boundary is 0..1008
  static constexpr int kBytes = kTiles + (1008 > 2 * kMeta - 16 ? 1008 : 2 * kMeta - 16);
};
static_assert(2 * (FmSmem::kBytes + 1024) <= 228 * 1024, "prefill attention must fit two CTAs per SM");

// 2^x on the MUFU unit (flushes results below 2^-126 to zero; 2^-inf = 0)
__device__ __forceinline__ float fm_exp2_mufu(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// 2^x on the FMA / ALU pipes, to take part of the softmax's exponentials off the MUFU unit: range
// reduction x = n + f (n = floor(x), f in [0, 1)), 2^f from a cubic through 2^0 = 1 whose other
// three coefficients are a least-squares fit of 2^f on [0, 1) (computed offline with numpy; max
// relative error 1.3e-4, below the bf16 rounding of P), and 2^n added to the exponent field.
// Inputs below -126 (masked keys: -inf) give 2^-126, negligible next to a row sum >= 1.
__device__ __forceinline__ float fm_exp2_poly(float x) {
  x = fmaxf(x, -126.f);
  const float n = floorf(x);
  const float f = x - n;
  const float q = fmaf(fmaf(fmaf(0.07737474f, f, 0.22694686f), f, 0.69542833f), f, 1.f);
  return __int_as_float(__float_as_int(q) + (__float2int_rz(n) << 23));
}

// Page-table batch: lane j holds the first KV slot of page (32 * batch + j) of the tile's key range.
__device__ __forceinline__ int fm_page_slots(const FmhaParams& p, const FmTile& T, int batch, int lane) {
  const int g = p.page;
  const int ngroups = T.nb * (kFmKB / g);
  int slot = 0;
  const int gi = batch * 32 + lane;
  if (gi < ngroups) {
    const int pos = T.blk0 * kFmKB + gi * g;
    slot = pos < T.L ? p.page_table[(int64_t)T.row * p.pt_stride + pos] : 0;
    if (!MSGL_IN_BOUNDS(slot >= 0 && slot < p.num_slots, kBcAttnSlot)) slot = 0;
  }
  return slot;
}

// TMA loads of one 64-key block's pages (K or V) into a stage: pages of `g` keys, two 64-dim halves
// each. Lane (first + sub) of the warp holds the first KV slot of page `sub` of the block.
__device__ __forceinline__ void fm_load_pages(uint8_t* stage, const CUtensorMap* map, uint64_t* bar, int kvh,
                                              int slot, int first, int gpb, int g, int lane) {
  for (int sub = 0; sub < gpb; ++sub) {
    const int s0 = __shfl_sync(0xffffffffu, slot, first + sub);
    if (lane == 0) {
      for (int h = 0; h < 2; ++h) tma_load_3d(stage + h * FmSmem::kHalf + sub * g * 128, map, bar, h * 64, kvh, s0);
    }
  }
}

// Warp-wide: the tile of work item w (= tile * nkv + kv head). Tiles are numbered request by
// request, ceil(q_len / TT) per request, the last tile of a request (the most key blocks) first.
// The scan state (first request of the current 32-request window, tiles before it) only moves
// forward, as a CTA's work items increase. Returns false past the last tile; T.nb = 0 marks a
// malformed request (skipped).
__device__ __forceinline__ bool fm_lookup(const FmhaParams& p, int w, int& scan_base, int& scan_before, FmTile& T,
                                          int lane) {
  const int tile = w / p.nkv;
  const int TT = p.tt;
  int b = -1, qb = 0;
  while (scan_base < p.num_reqs) {
    const int j = scan_base + lane;
    int c = 0;
    if (j < p.num_reqs) c = max(0, (p.cu_q[j + 1] - p.cu_q[j] + TT - 1) / TT);
    int incl = c;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int v = __shfl_up_sync(0xffffffffu, incl, o);
      if (lane >= o) incl += v;
    }
    const int tot = __shfl_sync(0xffffffffu, incl, 31);
    if (tile < scan_before + tot) {  // warp-uniform
      const int first = __ffs(__ballot_sync(0xffffffffu, tile < scan_before + incl)) - 1;
      const int excl = __shfl_sync(0xffffffffu, incl - c, first);
      const int cnt = __shfl_sync(0xffffffffu, c, first);
      b = scan_base + first;
      qb = cnt - 1 - (tile - scan_before - excl);
      break;
    }
    scan_base += 32;
    scan_before += tot;
  }
  if (b < 0) return false;
  T.b = b;
  T.kvh = w - tile * p.nkv;
  T.q0 = p.cu_q[b];
  const int n = p.cu_q[b + 1] - T.q0;
  T.t0 = qb * TT;
  T.t1 = min(n, T.t0 + TT);
  T.L = p.kv_lens[b];
  T.row = p.rows[b];
  T.nb = 0;
  if (T.t0 < n && MSGL_IN_BOUNDS(T.row >= 0 && T.L >= n && T.L <= p.pt_stride, kBcAttnRow)) {
    T.qpos0 = T.L - n;
    const int kend = T.qpos0 + T.t1;  // exclusive
    const int kbeg = p.window > 0 ? max(0, T.qpos0 + T.t0 - p.window + 1) : 0;
    T.blk0 = kbeg / kFmKB;
    T.nb = (kend + kFmKB - 1) / kFmKB - T.blk0;
  }
  return true;
}

__global__ void __launch_bounds__(kFmThreads, 2)
fmha_prefill_kernel(const __grid_constant__ CUtensorMap tq, const __grid_constant__ CUtensorMap tk,
                    const __grid_constant__ CUtensorMap tv, FmhaParams p) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  const uint32_t gap = (1024u - (smem_u32(smem_raw) & 1023u)) & 1023u;
  uint8_t* smem = smem_raw + gap;
  uint8_t* meta = gap >= (uint32_t)FmSmem::kMeta ? smem_raw : smem + FmSmem::kTiles;
  uint8_t* sQ = smem;
  uint8_t* sK = smem + FmSmem::kOffK;
  uint8_t* sV = smem + FmSmem::kOffV;
  FmTile* ring = reinterpret_cast<FmTile*>(meta);
  uint64_t* bars = reinterpret_cast<uint64_t*>(meta + FmSmem::kRingBytes);
  uint64_t* qfull = bars;                     // Q of a tile landed (one phase per tile)
  uint64_t* qempty = bars + 1;                // last QK^T of a tile done: Q buffer free
  uint64_t* ofree = bars + 2;                 // the softmax has read a tile's O (4 warps)
  uint64_t* kfull = bars + 3;                 // [kFmKStages]
  uint64_t* kempty = kfull + kFmKStages;      // [kFmKStages]
  uint64_t* vfull = kempty + kFmKStages;      // [kFmVStages]
  uint64_t* vempty = vfull + kFmVStages;      // [kFmVStages]
  uint64_t* sfull = vempty + kFmVStages;      // [2] S_i landed in buffer i % 2
  uint64_t* pfull = sfull + 2;                // [2] P_i written over buffer i % 2 (4 warps)
  uint64_t* pvdone = pfull + 2;               // [2] PV_i done: buffer i % 2 free, O updated
  uint64_t* tfull = pvdone + 2;               // [kFmRing] tile entry published
  uint64_t* tempty = tfull + kFmRing;         // [kFmRing] entry released (MMA, 4 softmax, V stream)
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(tempty + kFmRing);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int G = p.group, TT = p.tt;
  const long long c_start = clock64();
  uint32_t* tr = (p.trace != nullptr && (int)blockIdx.x < p.trace_ctas)
                     ? p.trace + (size_t)blockIdx.x * kFmTrace : nullptr;
  constexpr int TS = 2;  // the traced tile of each CTA (its third: past the start-up transient)
#define FM_STAMP(cond, slot)                                                   \
  do {                                                                         \
    if (tr != nullptr && (cond)) tr[slot] = (uint32_t)(clock64() - c_start);   \
  } while (0)

  if (warp == 1) {
    if (lane == 0) {
      mbar_init(qfull, 1);
      mbar_init(qempty, 1);
      mbar_init(ofree, 4);
      for (int i = 0; i < kFmKStages; ++i) {
        mbar_init(&kfull[i], 1);
        mbar_init(&kempty[i], 1);
      }
      for (int i = 0; i < kFmVStages; ++i) {
        mbar_init(&vfull[i], 1);
        mbar_init(&vempty[i], 1);
      }
      for (int i = 0; i < 2; ++i) {
        mbar_init(&sfull[i], 1);
        mbar_init(&pfull[i], 4);
        mbar_init(&pvdone[i], 1);
      }
      for (int i = 0; i < kFmRing; ++i) {
        mbar_init(&tfull[i], 1);
        mbar_init(&tempty[i], 6);
      }
      fence_barrier_init();
    }
    __syncwarp();
    tmem_alloc(tmem_slot, 256);
    tmem_relinquish();
    FM_STAMP(lane == 0, 85);
  } else if (warp == 0 && lane == 0) {
    prefetch_tmap(&tq);
    prefetch_tmap(&tk);
    prefetch_tmap(&tv);
    if (tr != nullptr) {
      tr[5] = smem_u32(smem_raw) & 1023u;  // alignment of the dynamic smem base
      uint32_t sm;
      asm volatile("mov.u32 %0, %%smid;" : "=r"(sm));
      tr[6] = sm;
      tr[7] = (uint32_t)(globaltimer_ns() >> 5);  // start, 32 ns units
    }
  }
  pdl_wait();
  FM_STAMP(threadIdx.x == 0, 86);
  pdl_launch();
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    // ------------------------------------------------------------------ producer (tiles, Q, K, V)
    const int g = p.page, gpb = kFmKB / g, bpb = 32 / gpb;  // pages per block, blocks per batch
    int scan_base = 0, scan_before = 0, next_static = blockIdx.x;
    int k_seq = 0;          // tiles published (the current K tile is k_seq - 1)
    bool k_have = false, k_done = false, q_issued = false;
    int ik = 0, gk = 0, batch_k = -1, slot_k = 0;
    FmTile KT;
    int v_seq = 0;          // ring entry the V stream reads next
    bool v_have = false, v_done = false;
    int iv = 0, gv = 0, batch_v = -1, slot_v = 0;
    FmTile VT;
    uint32_t spins = 0;
    uint64_t t_wait = 0;
    while (!(k_done && v_done)) {
      int act = 0;  // 1 K block, 2 V block, 3 Q, 4 publish the next tile, 5 V stream takes a tile
      if (lane == 0) {
        if (k_have && !q_issued && (k_seq == 1 || mbar_test(qempty, (k_seq - 2) & 1)))
          act = 3;
        else if (k_have && ik < KT.nb && mbar_test(&kempty[gk % kFmKStages], ((gk / kFmKStages) & 1) ^ 1))
          act = 1;
        else if (v_have && iv < VT.nb && mbar_test(&vempty[gv % kFmVStages], ((gv / kFmVStages) & 1) ^ 1))
          act = 2;
        else if (!k_done && (!k_have || (ik == KT.nb && q_issued)) &&
                 mbar_test(&tempty[k_seq % kFmRing], ((k_seq / kFmRing) & 1) ^ 1))
          act = 4;
        else if (!v_done && !v_have && mbar_test(&tfull[v_seq % kFmRing], (v_seq / kFmRing) & 1))
          act = 5;
        else if ((++spins & 63) == 0) {
          const uint64_t now = globaltimer_ns();
          if (t_wait == 0) t_wait = now;
          else if (now - t_wait > kWaitTimeoutNs) {
            report_error(kErrMbarTimeout, 500);
            act = -1;
          }
        }
        if (act > 0) t_wait = 0;
      }
      act = __shfl_sync(0xffffffffu, act, 0);
      if (act < 0) break;
      if (act == 0) __nanosleep(64);  // idle: leave the issue slots to the softmax warps
      if (act == 1) {
        if (ik / bpb != batch_k) {
          batch_k = ik / bpb;
          slot_k = fm_page_slots(p, KT, batch_k, lane);
        }
        const int st = gk % kFmKStages;
        if (lane == 0) {
          mbar_expect_tx(&kfull[st], FmSmem::kT);
          FM_STAMP(k_seq == TS + 1 && ik < 8, 8 + ik);
        }
        fm_load_pages(sK + st * FmSmem::kT, &tk, &kfull[st], KT.kvh, slot_k, (ik % bpb) * gpb, gpb, g, lane);
        ++ik;
        ++gk;
      } else if (act == 2) {
        if (iv / bpb != batch_v) {
          batch_v = iv / bpb;
          slot_v = fm_page_slots(p, VT, batch_v, lane);
        }
        const int st = gv % kFmVStages;
        if (lane == 0) {
          mbar_expect_tx(&vfull[st], FmSmem::kT);
          FM_STAMP(v_seq == TS && iv < 8, 16 + iv);
        }
        fm_load_pages(sV + st * FmSmem::kT, &tv, &vfull[st], VT.kvh, slot_v, (iv % bpb) * gpb, gpb, g, lane);
        ++iv;
        ++gv;
        if (iv == VT.nb) {  // every V load of the tile issued: release the entry
          if (lane == 0) mbar_arrive(&tempty[v_seq % kFmRing]);
          v_have = false;
          ++v_seq;
        }
      } else if (act == 3) {
        if (lane == 0) {
          mbar_expect_tx(qfull, 2 * TT * G * 128);
          for (int h = 0; h < 2; ++h)
            tma_load_3d(sQ + h * FmSmem::kQHalf, &tq, qfull, h * 64, KT.kvh * G, KT.q0 + KT.t0);
          FM_STAMP(k_seq == TS + 1, 3);
        }
        q_issued = true;
      } else if (act == 4) {
        // next work item with key blocks (malformed requests are skipped), or the end marker
        bool more = false;
        while (true) {
          int w = next_static;
          next_static += gridDim.x;
          if (p.epoch != 0) {
            if (lane == 0) w = atomicAdd(&g_fmha_work[p.epoch % kFmSlots], 1);
            w = __shfl_sync(0xffffffffu, w, 0);
            if (tr != nullptr && lane == 0 && tr[87] == 0) tr[87] = (uint32_t)(clock64() - c_start) | 1u;
          }
          more = fm_lookup(p, w, scan_base, scan_before, KT, lane);
          if (!more || KT.nb > 0) break;
        }
        if (!more) KT.nb = -1;
        if (tr != nullptr && lane == 0 && more) tr[84] += 1;  // tiles taken
        if (lane == 0) {
          ring[k_seq % kFmRing] = KT;
          mbar_arrive(&tfull[k_seq % kFmRing]);  // release: the entry is visible to its readers
          FM_STAMP(k_seq == TS, 1);
          if (tr != nullptr && k_seq == TS) tr[2] = (uint32_t)max(KT.nb, 0);
        }
        __syncwarp();  // the entry is read back by this warp's V stream
        ++k_seq;
        if (more) {
          k_have = true;
          q_issued = false;
          ik = 0;
          batch_k = -1;
        } else {
          k_have = false;
          k_done = true;
        }
      } else if (act == 5) {
        VT = ring[v_seq % kFmRing];
        if (VT.nb < 0) {
          v_done = true;
        } else {
          v_have = true;
          iv = 0;
          batch_v = -1;
        }
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      constexpr uint32_t idesc_s = idesc_bf16_f32(128, kFmKB);
      constexpr uint32_t idesc_o = idesc_bf16_f32(128, 128) | kIdescBMajorMN;
      const uint32_t q_base = smem_u32(sQ);
      int s_seq = 0, s_nb = 0, is = 0, gs = 0;  // S stream: ring entry, its key blocks, block, global block
      bool s_have = false, s_done = false;
      int p_seq = 0, p_nb = 0, ip = 0, gp = 0;  // PV stream
      bool p_have = false, p_done = false;
      uint32_t spins = 0;
      uint64_t t_wait = 0;
      while (!(s_done && p_done)) {
        bool progress = false;
        if (!s_have && !s_done && mbar_test(&tfull[s_seq % kFmRing], (s_seq / kFmRing) & 1)) {
          s_nb = ring[s_seq % kFmRing].nb;
          if (s_nb < 0) s_done = true;
          else { s_have = true; is = 0; }
          FM_STAMP(s_seq == TS, 89);
          progress = true;
        }
        if (tr != nullptr && s_have && is == 0 && s_seq == TS) {  // which input of the tile's first S is late
          if (tr[90] == 0 && mbar_test(qfull, s_seq & 1)) FM_STAMP(true, 90);
          if (tr[91] == 0 && mbar_test(&kfull[gs % kFmKStages], (gs / kFmKStages) & 1)) FM_STAMP(true, 91);
          if (tr[92] == 0 && (gs < 2 || mbar_test(&pvdone[gs & 1], ((gs - 2) >> 1) & 1))) FM_STAMP(true, 92);
          if (tr[93] == 0 && gs - gp < 2) FM_STAMP(true, 93);
        }
        // S_gs: Q and K landed, buffer gs % 2 free (PV_{gs-2} done), at most two S ahead of PV
        if (s_have && gs - gp < 2 && (is > 0 || mbar_test(qfull, s_seq & 1)) &&
            mbar_test(&kfull[gs % kFmKStages], (gs / kFmKStages) & 1) &&
            (gs < 2 || mbar_test(&pvdone[gs & 1], ((gs - 2) >> 1) & 1))) {
          tc_fence_after();
          if (is == 0) FM_STAMP(s_seq == TS, 4);
          const uint32_t k_base = smem_u32(sK + (gs % kFmKStages) * FmSmem::kT);
#pragma unroll
          for (int k = 0; k < 128 / 16; ++k) {  // head dim, 16 per MMA
            tc_mma_f16(tmem + (gs & 1) * kFmKB, smem_desc_sw128(q_base + (k >> 2) * FmSmem::kQHalf + (k & 3) * 32),
                       smem_desc_sw128(k_base + (k >> 2) * FmSmem::kHalf + (k & 3) * 32), idesc_s, k > 0 ? 1u : 0u);
          }
          tc_commit(&kempty[gs % kFmKStages]);
          tc_commit(&sfull[gs & 1]);
          FM_STAMP(s_seq == TS && is < 8, 24 + is);
          ++gs;
          if (++is == s_nb) {  // the tile's last QK^T: its Q buffer is free once this completes
            tc_commit(qempty);
            s_have = false;
            ++s_seq;
          }
          progress = true;
        }
        if (!p_have && !p_done && p_seq < s_seq + (s_have ? 1 : 0) + (s_done ? 1 : 0)) {
          // the PV stream follows the S stream through the ring (the entry is still held)
          p_nb = ring[p_seq % kFmRing].nb;
          if (p_nb < 0) p_done = true;
          else { p_have = true; ip = 0; }
          progress = true;
        }
        // PV_gp: P written, V landed, and for a tile's first block the previous tile's O read out
        if (p_have && gp < gs && mbar_test(&pfull[gp & 1], (gp >> 1) & 1) &&
            mbar_test(&vfull[gp % kFmVStages], (gp / kFmVStages) & 1) &&
            (ip > 0 || mbar_test(ofree, (p_seq & 1) ^ 1))) {
          tc_fence_after();
          const uint32_t a_tmem = tmem + (gp & 1) * kFmKB;  // P: 64 keys packed in 32 columns
          const uint32_t v_base = smem_u32(sV + (gp % kFmVStages) * FmSmem::kT);
#pragma unroll
          for (int k = 0; k < kFmKB / 16; ++k) {  // 16 keys per MMA
            tc_mma_f16_ts(tmem + 128, a_tmem + k * 8, smem_desc_sw128_mn(v_base + k * 16 * 128, FmSmem::kHalf),
                          idesc_o, (ip > 0 || k > 0) ? 1u : 0u);
          }
          tc_commit(&vempty[gp % kFmVStages]);
          tc_commit(&pvdone[gp & 1]);
          FM_STAMP(p_seq == TS && ip < 8, 32 + ip);
          ++gp;
          if (++ip == p_nb) {  // done with the tile's entry
            mbar_arrive(&tempty[p_seq % kFmRing]);
            p_have = false;
            ++p_seq;
          }
          progress = true;
        }
        if (progress) {
          spins = 0;
          t_wait = 0;
        } else {
          __nanosleep(32);  // idle: leave the issue slots to the softmax warps
          if ((++spins & 63) == 0) {
            const uint64_t now = globaltimer_ns();
            if (t_wait == 0) t_wait = now;
            else if (now - t_wait > kWaitTimeoutNs) {
              report_error(kErrMbarTimeout, 510);
              break;
            }
          }
        }
      }
    }
  } else {
    // ------------------------------------------------------------------ softmax + epilogue
    const int quad = warp & 3;
    const int r = quad * 32 + lane;  // accumulator row == TMEM lane
    const int t = r / G, gh = r - t * G;
    const uint32_t lane_base = tmem + ((uint32_t)(quad * 32) << 16);
    const float sl2 = p.scale_log2;
    const bool stamp = warp == 2 && lane == 0;
    int gsm = 0;  // global key block
    bool dead = false;
    for (int seq = 0;; ++seq) {
      if (!dead && !mbar_wait(&tfull[seq % kFmRing], (seq / kFmRing) & 1, 519)) dead = true;
      if (dead) break;
      const FmTile T = ring[seq % kFmRing];
      if (T.nb < 0) break;
      FM_STAMP(stamp && seq == TS, 88);
      const bool row_ok = r < TT * G && T.t0 + t < T.t1;
      const int qpos = T.qpos0 + T.t0 + t;
      const int kmax = min(qpos + 1, T.L);  // keys [kmin, kmax) are visible to this row
      const int kmin = p.window > 0 ? qpos - p.window + 1 : 0;
      const bool st0 = stamp && seq == TS;
      float m = -INFINITY, l = 0.f;
      for (int i = 0; i < T.nb; ++i, ++gsm) {
        const int sb = gsm & 1;
        if (!dead && !mbar_wait(&sfull[sb], (gsm >> 1) & 1, 520)) dead = true;
        if (st0 && i < 8) FM_STAMP(true, 40 + 4 * i);
        tc_fence_after();
        float s[kFmKB];
        {
          uint32_t u0[32], u1[32];
          tmem_ld_32x32b_x32(lane_base + sb * kFmKB, u0);
          tmem_ld_32x32b_x32(lane_base + sb * kFmKB + 32, u1);
          tc_wait_ld();
#pragma unroll
          for (int j = 0; j < 32; ++j) {
            s[j] = __uint_as_float(u0[j]);
            s[32 + j] = __uint_as_float(u1[j]);
          }
        }
        // visible key range of this row inside the block
        const int k0 = (T.blk0 + i) * kFmKB;
        const int lim = row_ok ? kmax - k0 : 0, lo = kmin - k0;
        if (!(lo <= 0 && lim >= kFmKB)) {
#pragma unroll
          for (int j = 0; j < kFmKB; ++j) s[j] = (j >= lo && j < lim) ? s[j] : -INFINITY;
        }
        float mx4[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
#pragma unroll
        for (int j = 0; j < kFmKB; ++j) mx4[j & 3] = fmaxf(mx4[j & 3], s[j]);
        float mx = fmaxf(fmaxf(mx4[0], mx4[1]), fmaxf(mx4[2], mx4[3]));
        if (st0 && i < 8) FM_STAMP(true, 41 + 4 * i);
        mx *= sl2;  // log2 domain (the scale is positive, so the max commutes with it)
        const bool grow = mx > m + 8.f;  // lazy rescale threshold
        float alpha = 1.f;
        if (grow) {
          alpha = m == -INFINITY ? 0.f : exp2f(m - mx);
          l *= alpha;
          m = mx;
        }
        if (i > 0 && __any_sync(0xffffffffu, grow)) {
          // O holds PV up to the previous block: wait for it, then rescale the row
          if (!dead && !mbar_wait(&pvdone[(gsm - 1) & 1], ((gsm - 1) >> 1) & 1, 521)) dead = true;
          tc_fence_after();
#pragma unroll
          for (int c = 0; c < 4; ++c) {
            uint32_t v[32];
            tmem_ld_32x32b_x32(lane_base + 128 + c * 32, v);
            tc_wait_ld();
#pragma unroll
            for (int j = 0; j < 32; ++j) v[j] = __float_as_uint(__uint_as_float(v[j]) * alpha);
            tmem_st_32x32b_x32(lane_base + 128 + c * 32, v);
          }
        }
        const float base = m == -INFINITY ? 0.f : m;
        float sum4[4] = {0.f, 0.f, 0.f, 0.f};
        uint32_t pk[32];
#pragma unroll
        for (int j = 0; j < kFmKB; j += 2) {
          // one pair in four on the FMA pipe (the MUFU unit is the softmax's bottleneck)
          const float x0 = fmaf(s[j], sl2, -base), x1 = fmaf(s[j + 1], sl2, -base);
          const bool poly = ((j >> 1) & 3) == 3;
          const float e0 = poly ? fm_exp2_poly(x0) : fm_exp2_mufu(x0);
          const float e1 = poly ? fm_exp2_poly(x1) : fm_exp2_mufu(x1);
          sum4[(j >> 1) & 3] += e0 + e1;
          pk[j >> 1] = pack_bf16(e0, e1);
        }
        l += (sum4[0] + sum4[1]) + (sum4[2] + sum4[3]);
        if (st0 && i < 8) FM_STAMP(true, 42 + 4 * i);
        // P over the first 32 columns of this block's S buffer (S is already in registers)
        tmem_st_32x32b_x32(lane_base + sb * kFmKB, pk);
        tc_wait_st();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&pfull[sb]);
        if (st0 && i < 8) FM_STAMP(true, 43 + 4 * i);
      }
      // epilogue: wait for the tile's last PV, read O out of TMEM and release it, normalise, store
      if (!dead && !mbar_wait(&pvdone[(gsm - 1) & 1], ((gsm - 1) >> 1) & 1, 522)) dead = true;
      FM_STAMP(st0, 80);
      tc_fence_after();
      uint32_t ov[128];
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        uint32_t v[32];
        tmem_ld_32x32b_x32(lane_base + 128 + c * 32, v);
        tc_wait_ld();
#pragma unroll
        for (int j = 0; j < 32; ++j) ov[c * 32 + j] = v[j];
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(ofree);
      float f = 1.f, ll = l;
      if (p.sinks != nullptr) {
        const float sk = p.sinks[T.kvh * G + gh] * kLog2e;
        const float mn = fmaxf(m, sk);
        f = exp2f(m - mn);
        ll = l * f + exp2f(sk - mn);
      }
      const float inv = ll > 0.f ? f / ll : 0.f;
      if (row_ok) {
        __nv_bfloat16* dst = p.o + ((int64_t)(T.q0 + T.t0 + t) * p.nq + T.kvh * G + gh) * 128;
#pragma unroll
        for (int j = 0; j < 128; j += 8)
          *reinterpret_cast<uint4*>(dst + j) = make_uint4(
              pack_bf16(__uint_as_float(ov[j]) * inv, __uint_as_float(ov[j + 1]) * inv),
              pack_bf16(__uint_as_float(ov[j + 2]) * inv, __uint_as_float(ov[j + 3]) * inv),
              pack_bf16(__uint_as_float(ov[j + 4]) * inv, __uint_as_float(ov[j + 5]) * inv),
              pack_bf16(__uint_as_float(ov[j + 6]) * inv, __uint_as_float(ov[j + 7]) * inv));
      }
      FM_STAMP(st0, 81);
      __syncwarp();
      if (lane == 0) mbar_arrive(&tempty[seq % kFmRing]);
    }
  }
  tc_fence_before();
  __syncthreads();
  FM_STAMP(threadIdx.x == 0, 82);
  if (tr != nullptr && threadIdx.x == 0) tr[83] = (uint32_t)(globaltimer_ns() >> 5);  // end, 32 ns units
  if (threadIdx.x == 0 && p.epoch != 0) {
    __threadfence();
    const int slot = p.epoch % kFmSlots, next = (slot + 1) % kFmSlots;
    if (atomicAdd(&g_fmha_exit[slot], 1) == (int)gridDim.x - 1) {  // last CTA out: reset
      atomicExch(&g_fmha_work[slot], 0);
      atomicExch(&g_fmha_exit[slot], 0);
      atomicExch(&g_fmha_work[next], 0);
      atomicExch(&g_fmha_exit[next], 0);
    }
  }
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, 256);
  }
#undef FM_STAMP
}

// Profiling hook: phase stamps of the next prefill launches (nullptr: off). Not for concurrent use.
static uint32_t* g_fmha_trace = nullptr;
static int g_fmha_trace_ctas = 0;

}  // namespace

extern "C" void msgl_attention_prefill_trace(uint32_t* buf, int ctas) {
  g_fmha_trace = buf;
  g_fmha_trace_ctas = buf != nullptr ? ctas : 0;
}

extern "C" int msgl_attention_prefill_fmha(void* o, const void* q, int64_t total_q, const void* k_cache,
                                           const void* v_cache, int64_t num_slots, int64_t cache_stride,
                                           const int32_t* page_table, int64_t pt_stride, const int32_t* rows,
                                           const int32_t* cu_q, const int32_t* kv_lens, int num_reqs, int max_q_len,
                                           int nq, int nkv, int hd, int page, float sm_scale, int window,
                                           const float* sinks, cudaStream_t s) {
  if (num_reqs == 0 || total_q == 0) return 0;
  if (hd != 128 || nq % nkv != 0 || nq / nkv > 128 || (page != 16 && page != 32 && page != 64)) return 3;
  FmhaParams p;
  p.o = reinterpret_cast<__nv_bfloat16*>(o);
  p.page_table = page_table;
  p.pt_stride = pt_stride;
  p.num_slots = num_slots;
  p.rows = rows;
  p.cu_q = cu_q;
  p.kv_lens = kv_lens;
  p.sinks = sinks;
  p.nq = nq;
  p.nkv = nkv;
  p.group = nq / nkv;
  p.tt = 128 / p.group;
  p.page = page;
  p.scale_log2 = sm_scale * kLog2e;
  p.window = window;
  msgl_set_smem<fmha_prefill_kernel>(FmSmem::kBytes, 100);  // two CTAs per SM need all of it
  CUtensorMap tq, tk, tv;
  const cuuint64_t qdims[3] = {(cuuint64_t)hd, (cuuint64_t)nq, (cuuint64_t)total_q};
  const cuuint64_t qstr[2] = {(cuuint64_t)hd * 2, (cuuint64_t)nq * hd * 2};
  const cuuint32_t qbox[3] = {64, (cuuint32_t)p.group, (cuuint32_t)p.tt};
  const cuuint64_t kdims[3] = {(cuuint64_t)hd, (cuuint64_t)nkv, (cuuint64_t)num_slots};
  const cuuint64_t kstr[2] = {(cuuint64_t)hd * 2, (cuuint64_t)cache_stride * 2};
  const cuuint32_t kbox[3] = {64, 1, (cuuint32_t)page};
  if (!pd_encode(&tq, q, 3, qdims, qstr, qbox) || !pd_encode(&tk, k_cache, 3, kdims, kstr, kbox) ||
      !pd_encode(&tv, v_cache, 3, kdims, kstr, kbox))
    return 2;
  p.num_reqs = num_reqs;
  // Work distribution: the device counter (default), or with MINISGL_FMHA_STATIC=1 the static
  // round-robin blockIdx.x + k * gridDim.x (kept for load-balance comparisons; 10-15 % slower on the
  // benchmark step because its slowest CTA ends well after the median one).
  static std::atomic<uint32_t> launches{0};
  static const bool static_rr = [] {
    const char* e = getenv("MINISGL_FMHA_STATIC");
    return e != nullptr && e[0] == '1';
  }();
  p.epoch = ++launches;
  if (p.epoch == 0) p.epoch = ++launches;
  if (static_rr) p.epoch = 0;
  p.trace = g_fmha_trace;
  p.trace_ctas = g_fmha_trace_ctas;
  (void)max_q_len;
  // persistent: two CTAs per SM, at most one per work item (upper bound of sum(ceil(q_len / tt))
  // over the requests, times the kv heads)
  const int64_t work = ((total_q + p.tt - 1) / p.tt + num_reqs) * nkv;
  if (work > INT32_MAX) return 3;
  int dev = 0, sms = 0;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const int grid = (int)std::min<int64_t>(work, 2 * (int64_t)sms);
  msgl_launch(fmha_prefill_kernel, dim3(grid), dim3(kFmThreads), FmSmem::kBytes, s, 1, tq, tk, tv, p);
  return 0;
}

extern "C" int msgl_attention_decode_paged(void* o, const void* q, int q_rows, const void* k_cache,
                                           const void* v_cache, int64_t num_slots, int64_t cache_stride,
                                           const int32_t* page_table, int64_t pt_stride, const int32_t* rows,
                                           const int32_t* kv_lens, const int32_t* work, const int32_t* n_work,
                                           float* ws, int ws_slots, int32_t* counters, int nq, int nkv, int hd,
                                           int page, float sm_scale, int window, const float* sinks,
                                           cudaStream_t s) {
  if (nq % nkv != 0 || nq / nkv > 16 || (hd != 64 && hd != 128) || (page != 16 && page != 32 && page != 64))
    return 3;
  PagedDecodeParams p;
  p.o = reinterpret_cast<__nv_bfloat16*>(o);
  p.page_table = page_table;
  p.pt_stride = pt_stride;
  p.num_slots = num_slots;
  p.rows = rows;
  p.kv_lens = kv_lens;
  p.work = reinterpret_cast<const int4*>(work);
  p.n_work = n_work;
  p.ws = ws;
  p.ws_slots = ws_slots;
  p.counters = counters;
  p.sinks = sinks;
  p.nq = nq;
  p.nkv = nkv;
  p.group = nq / nkv;
  p.page = page;
  p.scale_log2 = sm_scale * kLog2e;
  p.window = window;
  return hd == 64 ? run_paged_decode<64>(p, q, q_rows, k_cache, v_cache, num_slots, cache_stride, s)
                  : run_paged_decode<128>(p, q, q_rows, k_cache, v_cache, num_slots, cache_stride, s);
}

// =================================================================================================
// Allocation-free decode attention entry point (an addition of this engine: the reference has no
// counterpart to it).
//
// Some callers cannot allocate device memory at all: hosts that run our kernels from inside a
// fixed, pre-planned memory budget, plug-in environments whose callbacks may not call cudaMalloc,
// and code that launches while a CUDA graph it does not own is being captured. For them,
// msgl_attention_decode_noalloc takes only its inputs and outputs; the split-KV scratch that the
// regular entry point receives as a `workspace` argument lives instead in one file-scope device
// array of kNoAllocScratchBytes (every GPU that loads this library holds it until the process
// exits).
//
//   * Host code may not use the array's name as a device address. The first call on each device
//     looks its address up with cudaGetSymbolAddress (with that device current) and caches it;
//     make that first call before any stream capture.
//   * All calls share the array and it keeps the last call's contents. Calls that overlap on the
//     GPU (other streams, concurrently replayed graphs) race on it: the caller must serialize them.
//     Each call writes every scratch word before reading it, so nothing has to start at zero.
//   * The problem must fit: bs * nq * num_splits * (hd + 2) * 4 bytes <= kNoAllocScratchBytes when
//     num_splits > 1 (a single split uses no scratch). Larger requests are rejected before any launch.
//   * Nothing here calls cudaMalloc, cudaFree or an allocating library routine.
//   * `num_slots` is the number of KV-cache slots; the bounds-check build checks every page-table
//     entry the kernels read against it (the release build does not read it).
// Returns 0 on success, otherwise one of kNoAlloc* below. kNoAllocTooLarge, kNoAllocSetupFailed and
// kNoAllocBadArgs launch nothing; kNoAllocLaunch means a launch failed (the CUDA error of that launch,
// not an older sticky one, decides it).
// =================================================================================================
#include <mutex>

namespace {

constexpr size_t kNoAllocScratchBytes = 8u << 20;  // 8 MiB per GPU
static __device__ __align__(256) unsigned char g_noalloc_decode_scratch[kNoAllocScratchBytes];

enum : int { kNoAllocOk = 0, kNoAllocTooLarge = 1, kNoAllocSetupFailed = 2, kNoAllocBadArgs = 3, kNoAllocLaunch = 4 };

// device address of the scratch array for the current device (looked up once per device)
void* noalloc_scratch_for_current_device() {
  constexpr int kMaxDevices = 64;
  static std::mutex mu;
  static void* addr[kMaxDevices] = {};
  int dev = -1;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return nullptr;
  std::lock_guard<std::mutex> g(mu);
  if (addr[dev] == nullptr) {
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_noalloc_decode_scratch) != cudaSuccess || p == nullptr) return nullptr;
    addr[dev] = p;
  }
  return addr[dev];
}

}  // namespace

extern "C" __attribute__((visibility("default"))) int msgl_attention_decode_noalloc(
    void* o, const void* q, const void* k_cache, const void* v_cache, const int32_t* page_table, int64_t pt_stride,
    const int32_t* rows, const int32_t* kv_lens, int bs, int nq, int nkv, int hd, int64_t cache_stride,
    int64_t num_slots, float sm_scale, int window, const float* sinks, int num_splits, cudaStream_t s) {
  if (bs < 0 || nkv <= 0 || nq % nkv != 0 || nq / nkv > 16 || (hd != 64 && hd != 128) || num_slots <= 0)
    return kNoAllocBadArgs;
  if (bs == 0) return kNoAllocOk;
  const int splits = num_splits < 1 ? 1 : num_splits;
  const size_t need = splits > 1 ? (size_t)bs * nq * splits * (hd + 2) * 4 : 0;
  if (need > kNoAllocScratchBytes) return kNoAllocTooLarge;
  void* scratch = noalloc_scratch_for_current_device();
  if (scratch == nullptr) return kNoAllocSetupFailed;
  AttnParams p = make_params(o, q, k_cache, v_cache, page_table, pt_stride, rows, nullptr, kv_lens, nq, nkv,
                             cache_stride, sm_scale, window, sinks, num_slots);
  p.num_splits = splits;
  p.ws = reinterpret_cast<float*>(scratch);
  const cudaError_t e = hd == 64 ? run_decode<64>(p, bs, s) : run_decode<128>(p, bs, s);
  return e == cudaSuccess ? kNoAllocOk : kNoAllocLaunch;
}
