// Temperature / top-k / top-p sampling, one CTA per row, no sort:
//   * top-k threshold  = exact k-th largest scaled logit by 4-pass radix select on the
//     order-preserving 32-bit key of each float. Counts go to per-warp histograms, and the lanes
//     of a warp that hit the same bin add once (match.any), so the few hot bins of the first digit
//     (sign and exponent) do not serialise the block on one shared-memory address;
//   * with 0 < k <= kCand the kept tokens (key >= threshold) are then compacted into shared memory
//     in one more pass, and the max, the top-p cut and the draw run on that list;
//   * top-p threshold  = exact nucleus cut by a mass-weighted radix select (walk bins from the
//     top accumulating exp(z - max) until the requested probability mass is reached);
//   * draw             = Gumbel-max: argmax over kept tokens of z - log(-log(u)), with u from a
//     counter-based hash of (seed, step, token id) (same hash as ops/reference.py).
// Greedy rows (temperature <= 0) take the plain argmax. Without top-k and top-p the draw is one
// pass over the row.
#include <cfloat>

#include "api.h"
#include "common.cuh"

using namespace msgl;

namespace {

constexpr int kThreads = 1024;
constexpr int kWarps = kThreads / 32;
constexpr int kCand = 4096;  // shared-memory candidate list of the top-k fast path

__device__ __forceinline__ uint32_t fkey(float f) {
  const uint32_t b = __float_as_uint(f);
  return (b & 0x80000000u) ? ~b : (b | 0x80000000u);
}

__device__ __forceinline__ float uniform01(uint32_t seed, uint32_t step, uint32_t idx) {
  uint32_t x = seed * 0x9E3779B1u + step * 0x85EBCA77u + idx * 0xC2B2AE3Du;
#pragma unroll
  for (int r = 0; r < 2; ++r) {
    x ^= x >> 16; x *= 0x85EBCA6Bu; x ^= x >> 13; x *= 0xC2B2AE35u; x ^= x >> 16;
  }
  return ((float)(x >> 8) + 0.5f) * (1.0f / 16777216.0f);
}

// Visit every element of a row as f(index, value, valid), in the same order on every lane of a warp
// (f may use warp-collective operations; valid is false on padding lanes). Four float4 loads per
// thread are in flight before any is used: with one scalar load per thread at a time the passes
// were bound by L2 latency, not bandwidth.
template <typename F>
__device__ __forceinline__ void for_row(const float* __restrict__ row, int vocab, F&& f) {
  constexpr int U = 4;
  const bool vec = (vocab % 4 == 0) && ((reinterpret_cast<uintptr_t>(row) & 15u) == 0);
  if (vec) {
    const float4* r4 = reinterpret_cast<const float4*>(row);
    const int n4 = vocab / 4;
    for (int base = 0; base < n4; base += kThreads * U) {
      float4 v[U];
#pragma unroll
      for (int u = 0; u < U; ++u) {
        const int j = base + u * kThreads + (int)threadIdx.x;
        v[u] = j < n4 ? __ldg(r4 + j) : make_float4(0.f, 0.f, 0.f, 0.f);
      }
#pragma unroll
      for (int u = 0; u < U; ++u) {
        const int j = base + u * kThreads + (int)threadIdx.x;
        const bool ok = j < n4;
        f(4 * j, v[u].x, ok);
        f(4 * j + 1, v[u].y, ok);
        f(4 * j + 2, v[u].z, ok);
        f(4 * j + 3, v[u].w, ok);
      }
    }
  } else {
    for (int base = 0; base < vocab; base += kThreads * U) {
      float v[U];
#pragma unroll
      for (int u = 0; u < U; ++u) {
        const int i = base + u * kThreads + (int)threadIdx.x;
        v[u] = i < vocab ? __ldg(row + i) : 0.f;
      }
#pragma unroll
      for (int u = 0; u < U; ++u) {
        const int i = base + u * kThreads + (int)threadIdx.x;
        f(i, v[u], i < vocab);
      }
    }
  }
}

struct Smem {
  union {
    uint32_t cnt[kWarps][256];
    float mass[kWarps][256];
  } h;  // per-warp histograms
  float cand_z[kCand];
  int cand_i[kCand];
  float bins_f[256];
  uint32_t bins_u[256];
  float red_f[32];
  int red_i[32];
  uint32_t sel_prefix;
  int sel_remaining;
  float sel_above;
  int cand_n;
};

__device__ float block_max(float v, Smem& sm) {
  v = warp_max(v);
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
  __syncthreads();
  if (lane == 0) sm.red_f[w] = v;
  __syncthreads();
  v = lane < kWarps ? sm.red_f[lane] : -FLT_MAX;
  return warp_max(v);
}

__device__ float block_sumf(float v, Smem& sm) {
  v = warp_sum(v);
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
  __syncthreads();
  if (lane == 0) sm.red_f[w] = v;
  __syncthreads();
  v = lane < kWarps ? sm.red_f[lane] : 0.f;
  return warp_sum(v);
}

// argmax of val with lowest-index ties across the block (*vout: the maximum)
__device__ int block_argmax(float v, int i, Smem& sm, float* vout) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float ov = __shfl_xor_sync(0xffffffffu, v, o);
    const int oi = __shfl_xor_sync(0xffffffffu, i, o);
    if (ov > v || (ov == v && oi < i)) { v = ov; i = oi; }
  }
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
  __syncthreads();
  if (lane == 0) { sm.red_f[w] = v; sm.red_i[w] = i; }
  __syncthreads();
  v = lane < kWarps ? sm.red_f[lane] : -FLT_MAX;
  i = lane < kWarps ? sm.red_i[lane] : 0x7fffffff;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float ov = __shfl_xor_sync(0xffffffffu, v, o);
    const int oi = __shfl_xor_sync(0xffffffffu, i, o);
    if (ov > v || (ov == v && oi < i)) { v = ov; i = oi; }
  }
  *vout = v;
  return i;
}

__device__ __forceinline__ void zero_hist(Smem& sm) {
  uint32_t* flat = &sm.h.cnt[0][0];
  for (int j = threadIdx.x; j < kWarps * 256; j += kThreads) flat[j] = 0u;
}

// Sum the per-warp histograms into bins_u / bins_f (threads 0..255), then clear them.
template <bool MASS>
__device__ __forceinline__ void fold_hist(Smem& sm) {
  __syncthreads();
  if (threadIdx.x < 256) {
    if constexpr (MASS) {
      float s = 0.f;
#pragma unroll 8
      for (int w = 0; w < kWarps; ++w) s += sm.h.mass[w][threadIdx.x];
      sm.bins_f[threadIdx.x] = s;
    } else {
      uint32_t s = 0;
#pragma unroll 8
      for (int w = 0; w < kWarps; ++w) s += sm.h.cnt[w][threadIdx.x];
      sm.bins_u[threadIdx.x] = s;
    }
  }
  __syncthreads();
  zero_hist(sm);
}

// Walk bins_u / bins_f from the top (bin 255) accumulating until `target` is reached; the bin
// where it is reached extends the prefix (bin 0 if never). Warp 0 scans, lane l owning bins
// 255 - 8l ... 248 - 8l. Writes sel_prefix and sel_remaining (counts) or sel_above (mass).
template <bool MASS>
__device__ __forceinline__ void select_bin(Smem& sm, int shift, uint32_t prefix, float target_f, int target_u,
                                           float above) {
  if (threadIdx.x < 32) {
    const int lane = threadIdx.x;
    float cf[8];
    uint32_t cu[8];
    float sf = 0.f;
    uint32_t su = 0;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const int b = 255 - 8 * lane - j;
      if constexpr (MASS) { cf[j] = sm.bins_f[b]; sf += cf[j]; }
      else { cu[j] = sm.bins_u[b]; su += cu[j]; }
    }
    float incf = sf;
    uint32_t incu = su;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const float tf = __shfl_up_sync(0xffffffffu, incf, o);
      const uint32_t tu = __shfl_up_sync(0xffffffffu, incu, o);
      if (lane >= o) { incf += tf; incu += tu; }
    }
    const bool reach = MASS ? (above + incf >= target_f) : (incu >= (uint32_t)target_u);
    const unsigned hit = __ballot_sync(0xffffffffu, reach);
    const int L = hit ? __ffs(hit) - 1 : 31;
    if (lane == L) {
      int j = 0;
      if constexpr (MASS) {
        float acc = above + (incf - sf);
        for (; j < 7; ++j) {
          if (acc + cf[j] >= target_f) break;
          acc += cf[j];
        }
        sm.sel_above = acc;
      } else {
        uint32_t acc = incu - su;
        for (; j < 7; ++j) {
          if (acc + cu[j] >= (uint32_t)target_u) break;
          acc += cu[j];
        }
        sm.sel_remaining = target_u - (int)acc;
      }
      sm.sel_prefix = prefix | ((uint32_t)(255 - 8 * L - j) << shift);
    }
  }
  __syncthreads();
}

// Column i of row r is token col_ids[r][i] when col_ids is given (a candidate list, ascending ids),
// else token id_offset + i (a vocabulary shard). The token id keys the Gumbel noise and is what
// out[r] receives; out_val[r] (optional) receives the winning Gumbel score (the maximum logit on
// greedy rows), which is what shards compare to combine their draws.
__global__ void __launch_bounds__(kThreads, 1) sample_kernel(int32_t* __restrict__ out, const float* __restrict__ logits,
                                                         int vocab, int64_t stride, const float* __restrict__ temperature,
                                                         const int32_t* __restrict__ top_k, const float* __restrict__ top_p,
                                                         const int64_t* __restrict__ seed, const int64_t* __restrict__ step,
                                                         const int32_t* __restrict__ col_ids, int id_offset,
                                                         float* __restrict__ out_val) {
  extern __shared__ __align__(16) uint8_t smem_raw[];
  Smem& sm = *reinterpret_cast<Smem*>(smem_raw);
  pdl_wait();
  pdl_launch();
  const int r = blockIdx.x;
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
  const float* row = logits + (size_t)r * stride;
  const int32_t* ids = col_ids != nullptr ? col_ids + (size_t)r * vocab : nullptr;
  auto token = [&](int i) -> int { return ids != nullptr ? ids[i] : id_offset + i; };
  auto emit = [&](int a, float v) {
    if (threadIdx.x == 0) {
      out[r] = token(a == 0x7fffffff ? 0 : a);
      if (out_val != nullptr) out_val[r] = a == 0x7fffffff ? -FLT_MAX : v;
    }
  };
  const float t = temperature[r];
  if (!(t > 0.f)) {
    float bv = -FLT_MAX;
    int bi = 0x7fffffff;
    for_row(row, vocab, [&](int i, float v, bool ok) {
      if (ok && (v > bv || (v == bv && i < bi))) { bv = v; bi = i; }
    });
    float mv;
    const int a = block_argmax(bv, bi, sm, &mv);
    emit(a, mv);
    return;
  }
  const float inv_t = 1.f / t;
  const int k = top_k[r];
  const float p = top_p[r];
  const uint32_t sd = (uint32_t)seed[r], st = (uint32_t)step[r];
  zero_hist(sm);
  // ---- top-k cut (key threshold; keep key >= kcut)
  uint32_t kcut = 0;
  if (k > 0 && k < vocab) {
    uint32_t prefix = 0, mask = 0;
    int remaining = k;
    __syncthreads();
    for (int shift = 24; shift >= 0; shift -= 8) {
      for_row(row, vocab, [&](int, float v, bool ok) {
        int bin = -1;
        if (ok) {
          const uint32_t key = fkey(v * inv_t);
          if ((key & mask) == prefix) bin = (int)((key >> shift) & 255u);
        }
        if (__any_sync(0xffffffffu, bin >= 0)) {  // later digits: most warps hold no matching key
          const unsigned m = __match_any_sync(0xffffffffu, bin);
          if (bin >= 0 && lane == __ffs(m) - 1) atomicAdd(&sm.h.cnt[w][bin], (uint32_t)__popc(m));
        }
      });
      fold_hist<false>(sm);
      select_bin<false>(sm, shift, prefix, 0.f, remaining, 0.f);
      prefix = sm.sel_prefix;
      remaining = sm.sel_remaining;
      mask |= 255u << shift;
    }
    kcut = prefix;
    if (k <= kCand) {
      // ---- compact the kept tokens into shared memory
      if (threadIdx.x == 0) sm.cand_n = 0;
      __syncthreads();
      for_row(row, vocab, [&](int i, float v, bool ok) {
        const float z = v * inv_t;
        const bool keep = ok && fkey(z) >= kcut;
        const unsigned bal = __ballot_sync(0xffffffffu, keep);
        if (bal) {  // warp-uniform
          int pos0 = 0;
          if (lane == 0) pos0 = atomicAdd(&sm.cand_n, __popc(bal));
          pos0 = __shfl_sync(0xffffffffu, pos0, 0);
          if (keep) {
            const int pos = pos0 + __popc(bal & ((1u << lane) - 1u));
            if (pos < kCand) { sm.cand_z[pos] = z; sm.cand_i[pos] = i; }
          }
        }
      });
      __syncthreads();
      const int n = sm.cand_n;
      if (n <= kCand) {
        float mx = -FLT_MAX;
        for (int j = threadIdx.x; j < n; j += kThreads) mx = fmaxf(mx, sm.cand_z[j]);
        mx = block_max(mx, sm);
        uint32_t pcut = kcut;
        if (p < 1.f) {
          float tot = 0.f;
          for (int j = threadIdx.x; j < n; j += kThreads) tot += __expf(sm.cand_z[j] - mx);
          tot = block_sumf(tot, sm);
          const float target = p * tot;
          uint32_t pre = 0, msk = 0;
          float above = 0.f;
          for (int shift = 24; shift >= 0; shift -= 8) {
            for (int j = threadIdx.x; j < n; j += kThreads) {
              const float z = sm.cand_z[j];
              const uint32_t key = fkey(z);
              if ((key & msk) == pre) atomicAdd(&sm.h.mass[w][(key >> shift) & 255u], __expf(z - mx));
            }
            fold_hist<true>(sm);
            select_bin<true>(sm, shift, pre, target, 0, above);
            pre = sm.sel_prefix;
            above = sm.sel_above;
            msk |= 255u << shift;
          }
          pcut = max(pre, kcut);
        }
        float bv = -FLT_MAX;
        int bi = 0x7fffffff;
        for (int j = threadIdx.x; j < n; j += kThreads) {
          const float z = sm.cand_z[j];
          if (fkey(z) < pcut) continue;
          const int i = sm.cand_i[j];
          const float g = z - logf(-logf(uniform01(sd, st, (uint32_t)token(i))));
          if (g > bv || (g == bv && i < bi)) { bv = g; bi = i; }
        }
        float mv;
        const int a = block_argmax(bv, bi, sm, &mv);
        emit(a, mv);
        return;
      }
      // more ties at the threshold than the list holds: continue over the whole row
    }
  }
  // ---- top-p over the whole row (no top-k, or the candidate list overflowed)
  uint32_t pcut = kcut;
  if (p < 1.f) {
    float mx = -FLT_MAX;
    for_row(row, vocab, [&](int, float v, bool ok) {
      const float z = v * inv_t;
      if (ok && fkey(z) >= kcut) mx = fmaxf(mx, z);
    });
    mx = block_max(mx, sm);
    float tot = 0.f;
    for_row(row, vocab, [&](int, float v, bool ok) {
      const float z = v * inv_t;
      if (ok && fkey(z) >= kcut) tot += __expf(z - mx);
    });
    tot = block_sumf(tot, sm);
    const float target = p * tot;
    uint32_t prefix = 0, mask = 0;
    float above = 0.f;
    for (int shift = 24; shift >= 0; shift -= 8) {
      for_row(row, vocab, [&](int, float v, bool ok) {
        const float z = v * inv_t;
        const uint32_t key = fkey(z);
        if (ok && key >= kcut && (key & mask) == prefix) atomicAdd(&sm.h.mass[w][(key >> shift) & 255u], __expf(z - mx));
      });
      fold_hist<true>(sm);
      select_bin<true>(sm, shift, prefix, target, 0, above);
      prefix = sm.sel_prefix;
      above = sm.sel_above;
      mask |= 255u << shift;
    }
    pcut = max(prefix, kcut);
  }
  // ---- Gumbel-max draw among kept tokens
  float bv = -FLT_MAX;
  int bi = 0x7fffffff;
  for_row(row, vocab, [&](int i, float v, bool ok) {
    const float z = v * inv_t;
    if (!ok || fkey(z) < pcut) return;
    const float g = z - logf(-logf(uniform01(sd, st, (uint32_t)token(i))));
    if (g > bv || (g == bv && i < bi)) { bv = g; bi = i; }
  });
  float mv;
  const int a = block_argmax(bv, bi, sm, &mv);
  emit(a, mv);
}

}  // namespace

extern "C" void msgl_sample(int32_t* out, const float* logits, int rows, int vocab, int64_t stride,
                            const float* temperature, const int32_t* top_k, const float* top_p,
                            const int64_t* seed, const int64_t* step, const int32_t* col_ids, int id_offset,
                            float* out_val, cudaStream_t s) {
  if (rows == 0) return;
  msgl_set_smem<sample_kernel>((int)sizeof(Smem));
  msgl_launch(sample_kernel, dim3(rows), dim3(kThreads), sizeof(Smem), s, 1, out, logits, vocab, stride, temperature,
              top_k, top_p, seed, step, col_ids, id_offset, out_val);
}

MSGL_ERROR_ACCESSOR(msgl_err_sampling)
