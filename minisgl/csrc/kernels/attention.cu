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
#include <cfloat>

#include "api.h"
#include "common.cuh"

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
    const bool valid = pos < kend;
    const int64_t slot = valid ? pt[pos] : 0;
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
    for (int i = threadIdx.x; i < seg1 - seg0; i += kWarps * 32) slots[i] = pt[seg0 + i];
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
  static bool set = false;
  if (!set) {
    cudaFuncSetAttribute(prefill_kernel<HD>, cudaFuncAttributeMaxDynamicSharedMemorySize, prefill_smem<HD>());
    set = true;
  }
  const dim3 grid((max_q_len * p.group + 63) / 64, num_reqs, p.nkv);
  msgl_launch(prefill_kernel<HD>, grid, dim3(kWarps * 32), prefill_smem<HD>(), s, 1, p);
}

template <int HD>
void run_decode(const AttnParams& p, int bs, cudaStream_t s) {
  static bool set = false;
  if (!set) {
    cudaFuncSetAttribute(decode_kernel<HD>, cudaFuncAttributeMaxDynamicSharedMemorySize, decode_smem<HD>());
    set = true;
  }
  const dim3 grid(p.nkv, bs, p.num_splits);
  msgl_launch(decode_kernel<HD>, grid, dim3(kWarps * 32), decode_smem<HD>(), s, 1, p);
  if (p.num_splits > 1) {
    const int warps = bs * p.nq;
    msgl_launch(decode_combine_kernel<HD>, dim3((warps + 7) / 8), dim3(256), 0, s, 1, p, bs);
  }
}

AttnParams make_params(void* o, const void* q, const void* k, const void* v, const int32_t* pt,
                       int64_t pt_stride, const int32_t* rows, const int32_t* cu_q, const int32_t* kv_lens,
                       int nq, int nkv, int64_t cache_stride, float sm_scale, int window,
                       const float* sinks) {
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
                                       int64_t cache_stride, float sm_scale, int window,
                                       const float* sinks, cudaStream_t s) {
  if (num_reqs == 0 || total_q == 0) return;
  AttnParams p = make_params(o, q, k_cache, v_cache, page_table, pt_stride, rows, cu_q, kv_lens, nq,
                             nkv, cache_stride, sm_scale, window, sinks);
  if (hd == 64) run_prefill<64>(p, num_reqs, max_q_len, s);
  else run_prefill<128>(p, num_reqs, max_q_len, s);
}

extern "C" void msgl_attention_decode(void* o, const void* q, const void* k_cache, const void* v_cache,
                                      const int32_t* page_table, int64_t pt_stride, const int32_t* rows,
                                      const int32_t* kv_lens, int bs, int nq, int nkv, int hd,
                                      int64_t cache_stride, float sm_scale, int window,
                                      const float* sinks, int num_splits, void* workspace,
                                      cudaStream_t s) {
  if (bs == 0) return;
  AttnParams p = make_params(o, q, k_cache, v_cache, page_table, pt_stride, rows, nullptr, kv_lens,
                             nq, nkv, cache_stride, sm_scale, window, sinks);
  p.num_splits = num_splits < 1 ? 1 : num_splits;
  p.ws = reinterpret_cast<float*>(workspace);
  if (hd == 64) run_decode<64>(p, bs, s);
  else run_decode<128>(p, bs, s);
}

MSGL_ERROR_ACCESSOR(msgl_err_attention)

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
// Returns 0 on success, otherwise one of kNoAlloc* below (nothing is launched on error).
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
    float sm_scale, int window, const float* sinks, int num_splits, cudaStream_t s) {
  if (bs < 0 || nkv <= 0 || nq % nkv != 0 || nq / nkv > 16 || (hd != 64 && hd != 128)) return kNoAllocBadArgs;
  if (bs == 0) return kNoAllocOk;
  const int splits = num_splits < 1 ? 1 : num_splits;
  const size_t need = splits > 1 ? (size_t)bs * nq * splits * (hd + 2) * 4 : 0;
  if (need > kNoAllocScratchBytes) return kNoAllocTooLarge;
  void* scratch = noalloc_scratch_for_current_device();
  if (scratch == nullptr) return kNoAllocSetupFailed;
  AttnParams p = make_params(o, q, k_cache, v_cache, page_table, pt_stride, rows, nullptr, kv_lens, nq, nkv,
                             cache_stride, sm_scale, window, sinks);
  p.num_splits = splits;
  p.ws = reinterpret_cast<float*>(scratch);
  if (hd == 64) run_decode<64>(p, bs, s);
  else run_decode<128>(p, bs, s);
  return cudaPeekAtLastError() == cudaSuccess ? kNoAllocOk : kNoAllocLaunch;
}
