// Temperature / top-k / top-p sampling, one CTA per row, no sort:
//   * top-k threshold  = exact k-th largest scaled logit by 4-pass radix select on the
//     order-preserving 32-bit key of each float;
//   * top-p threshold  = exact nucleus cut by a mass-weighted radix select (walk bins from the
//     top accumulating exp(z - max) until the requested probability mass is reached);
//   * draw             = Gumbel-max: argmax over kept tokens of z - log(-log(u)), with u from a
//     counter-based hash of (seed, step, token id) (same hash as ops/reference.py).
// Greedy rows (temperature <= 0) take the plain argmax.
#include <cfloat>

#include "api.h"
#include "common.cuh"

using namespace msgl;

namespace {

constexpr int kThreads = 1024;

__device__ __forceinline__ uint32_t fkey(float f) {
  const uint32_t b = __float_as_uint(f);
  return (b & 0x80000000u) ? ~b : (b | 0x80000000u);
}
__device__ __forceinline__ float unkey(uint32_t k) {
  const uint32_t b = (k & 0x80000000u) ? (k & 0x7fffffffu) : ~k;
  return __uint_as_float(b);
}

__device__ __forceinline__ float uniform01(uint32_t seed, uint32_t step, uint32_t idx) {
  uint32_t x = seed * 0x9E3779B1u + step * 0x85EBCA77u + idx * 0xC2B2AE3Du;
#pragma unroll
  for (int r = 0; r < 2; ++r) {
    x ^= x >> 16; x *= 0x85EBCA6Bu; x ^= x >> 13; x *= 0xC2B2AE35u; x ^= x >> 16;
  }
  return ((float)(x >> 8) + 0.5f) * (1.0f / 16777216.0f);
}

struct Smem {
  float hist_mass[256];
  int hist_cnt[256];
  float red_f[32];
  int red_i[32];
  uint32_t sel_prefix;
  int sel_remaining;
  float sel_above;
};

__device__ float block_max(float v, Smem& sm) {
  v = warp_max(v);
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
  __syncthreads();
  if (lane == 0) sm.red_f[w] = v;
  __syncthreads();
  v = lane < (int)(blockDim.x >> 5) ? sm.red_f[lane] : -FLT_MAX;
  return warp_max(v);
}

__device__ float block_sumf(float v, Smem& sm) {
  v = warp_sum(v);
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
  __syncthreads();
  if (lane == 0) sm.red_f[w] = v;
  __syncthreads();
  v = lane < (int)(blockDim.x >> 5) ? sm.red_f[lane] : 0.f;
  return warp_sum(v);
}

// argmax of val with lowest-index ties across the block
__device__ int block_argmax(float v, int i, Smem& sm) {
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
  v = lane < (int)(blockDim.x >> 5) ? sm.red_f[lane] : -FLT_MAX;
  i = lane < (int)(blockDim.x >> 5) ? sm.red_i[lane] : 0x7fffffff;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float ov = __shfl_xor_sync(0xffffffffu, v, o);
    const int oi = __shfl_xor_sync(0xffffffffu, i, o);
    if (ov > v || (ov == v && oi < i)) { v = ov; i = oi; }
  }
  return i;
}

__global__ void __launch_bounds__(kThreads) sample_kernel(int32_t* __restrict__ out, const float* __restrict__ logits,
                                                         int vocab, int64_t stride, const float* __restrict__ temperature,
                                                         const int32_t* __restrict__ top_k, const float* __restrict__ top_p,
                                                         const int64_t* __restrict__ seed, const int64_t* __restrict__ step) {
  __shared__ Smem sm;
  pdl_wait();
  pdl_launch();
  const int r = blockIdx.x;
  const float* row = logits + (size_t)r * stride;
  const float t = temperature[r];
  if (!(t > 0.f)) {
    float bv = -FLT_MAX;
    int bi = 0x7fffffff;
    for (int i = threadIdx.x; i < vocab; i += blockDim.x) {
      const float v = row[i];
      if (v > bv) { bv = v; bi = i; }
    }
    const int a = block_argmax(bv, bi, sm);
    if (threadIdx.x == 0) out[r] = a == 0x7fffffff ? 0 : a;
    return;
  }
  const float inv_t = 1.f / t;
  // ---- top-k cut (key threshold; keep key >= kcut)
  uint32_t kcut = 0;
  const int k = top_k[r];
  if (k > 0 && k < vocab) {
    uint32_t prefix = 0, mask = 0;
    int remaining = k;
    for (int shift = 24; shift >= 0; shift -= 8) {
      for (int b = threadIdx.x; b < 256; b += blockDim.x) sm.hist_cnt[b] = 0;
      __syncthreads();
      for (int i = threadIdx.x; i < vocab; i += blockDim.x) {
        const uint32_t key = fkey(row[i] * inv_t);
        if ((key & mask) == prefix) atomicAdd(&sm.hist_cnt[(key >> shift) & 255], 1);
      }
      __syncthreads();
      if (threadIdx.x == 0) {
        int acc = 0, b = 255;
        for (; b > 0; --b) {
          if (acc + sm.hist_cnt[b] >= remaining) break;
          acc += sm.hist_cnt[b];
        }
        sm.sel_prefix = prefix | ((uint32_t)b << shift);
        sm.sel_remaining = remaining - acc;
      }
      __syncthreads();
      prefix = sm.sel_prefix;
      remaining = sm.sel_remaining;
      mask |= 255u << shift;
    }
    kcut = prefix;
  }
  // ---- max of kept scaled logits and the kept mass
  float mx = -FLT_MAX;
  for (int i = threadIdx.x; i < vocab; i += blockDim.x) {
    const float z = row[i] * inv_t;
    if (fkey(z) >= kcut) mx = fmaxf(mx, z);
  }
  mx = block_max(mx, sm);
  uint32_t pcut = kcut;
  const float p = top_p[r];
  if (p < 1.f) {
    float tot = 0.f;
    for (int i = threadIdx.x; i < vocab; i += blockDim.x) {
      const float z = row[i] * inv_t;
      if (fkey(z) >= kcut) tot += __expf(z - mx);
    }
    tot = block_sumf(tot, sm);
    const float target = p * tot;
    uint32_t prefix = 0, mask = 0;
    float above = 0.f;
    for (int shift = 24; shift >= 0; shift -= 8) {
      for (int b = threadIdx.x; b < 256; b += blockDim.x) sm.hist_mass[b] = 0.f;
      __syncthreads();
      for (int i = threadIdx.x; i < vocab; i += blockDim.x) {
        const float z = row[i] * inv_t;
        const uint32_t key = fkey(z);
        if (key >= kcut && (key & mask) == prefix) atomicAdd(&sm.hist_mass[(key >> shift) & 255], __expf(z - mx));
      }
      __syncthreads();
      if (threadIdx.x == 0) {
        float acc = above;
        int b = 255;
        for (; b > 0; --b) {
          if (acc + sm.hist_mass[b] >= target) break;
          acc += sm.hist_mass[b];
        }
        sm.sel_prefix = prefix | ((uint32_t)b << shift);
        sm.sel_above = acc;
      }
      __syncthreads();
      prefix = sm.sel_prefix;
      above = sm.sel_above;
      mask |= 255u << shift;
    }
    pcut = max(prefix, kcut);
  }
  // ---- Gumbel-max draw among kept tokens
  const uint32_t sd = (uint32_t)seed[r], st = (uint32_t)step[r];
  float bv = -FLT_MAX;
  int bi = 0x7fffffff;
  for (int i = threadIdx.x; i < vocab; i += blockDim.x) {
    const float z = row[i] * inv_t;
    if (fkey(z) < pcut) continue;
    const float u = uniform01(sd, st, (uint32_t)i);
    const float g = z - logf(-logf(u));
    if (g > bv) { bv = g; bi = i; }
  }
  const int a = block_argmax(bv, bi, sm);
  if (threadIdx.x == 0) out[r] = a == 0x7fffffff ? 0 : a;
}

}  // namespace

extern "C" void msgl_sample(int32_t* out, const float* logits, int rows, int vocab, int64_t stride,
                            const float* temperature, const int32_t* top_k, const float* top_p,
                            const int64_t* seed, const int64_t* step, cudaStream_t s) {
  if (rows == 0) return;
  msgl_launch(sample_kernel, dim3(rows), dim3(kThreads), 0, s, 1, out, logits, vocab, stride, temperature, top_k,
              top_p, seed, step);
}

MSGL_ERROR_ACCESSOR(msgl_err_sampling)
