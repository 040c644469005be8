// Memory-bound kernels: embedding gather, RMSNorm / fused add+RMSNorm, gated activations,
// KV-cache store, the fused QK-norm + RoPE + KV-store, and the row argmax.
// All use 16-byte vector accesses; rows are bf16.
#include <cfloat>

#include "api.h"
#include "common.cuh"

using namespace msgl;

namespace {

__device__ __forceinline__ void bf16x8_to_f32(const uint4& u, float (&f)[8]) {
  f[0] = bf16_lo(u.x); f[1] = bf16_hi(u.x); f[2] = bf16_lo(u.y); f[3] = bf16_hi(u.y);
  f[4] = bf16_lo(u.z); f[5] = bf16_hi(u.z); f[6] = bf16_lo(u.w); f[7] = bf16_hi(u.w);
}

__device__ __forceinline__ uint4 f32_to_bf16x8(const float (&f)[8]) {
  uint4 u;
  u.x = pack_bf16(f[0], f[1]); u.y = pack_bf16(f[2], f[3]);
  u.z = pack_bf16(f[4], f[5]); u.w = pack_bf16(f[6], f[7]);
  return u;
}

// ------------------------------------------------------------------------------ embedding
// One warp per output row; rows outside the owned vocab range are zero (TP shards).
__global__ void embedding_kernel(uint4* __restrict__ out, const uint4* __restrict__ w,
                                 const int32_t* __restrict__ ids, int n, int vec_per_row,
                                 int vocab_start, int vocab_len, int masked) {
  pdl_wait();
  pdl_launch();
  const int row = blockIdx.x * (blockDim.x / 32) + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (row >= n) return;
  int id = ids[row] - vocab_start;
  const bool valid = id >= 0 && id < vocab_len;
  uint4* dst = out + (size_t)row * vec_per_row;
  if (!valid && !masked) (void)MSGL_IN_BOUNDS(false, kBcEmbeddingId);
  if (masked && !valid) {
    for (int i = lane; i < vec_per_row; i += 32) dst[i] = make_uint4(0, 0, 0, 0);
    return;
  }
  if (!valid) id = 0;  // unmasked out-of-range ids are clamped instead of faulting
  const uint4* src = w + (size_t)id * vec_per_row;
  for (int i = lane; i < vec_per_row; i += 32) dst[i] = __ldg(src + i);
}

// ------------------------------------------------------------------------------ rmsnorm
// One CTA per row; each thread keeps up to VPT 8-element vectors in registers.
template <int VPT, bool ADD>
__global__ void rmsnorm_kernel(__nv_bfloat16* __restrict__ out, __nv_bfloat16* __restrict__ x,
                               __nv_bfloat16* __restrict__ residual, const __nv_bfloat16* __restrict__ w,
                               int dim, float eps) {
  pdl_wait();
  pdl_launch();
  __shared__ float red[32];
  const int row = blockIdx.x;
  const int nvec = dim / 8;
  uint4* xr = reinterpret_cast<uint4*>(x + (size_t)row * dim);
  uint4* rr = ADD ? reinterpret_cast<uint4*>(residual + (size_t)row * dim) : nullptr;
  float v[VPT][8];
  float ss = 0.f;
#pragma unroll
  for (int k = 0; k < VPT; ++k) {
    const int i = threadIdx.x + k * blockDim.x;
    if (i < nvec) {
      bf16x8_to_f32(xr[i], v[k]);
      if constexpr (ADD) {
        float r[8];
        bf16x8_to_f32(rr[i], r);
#pragma unroll
        for (int j = 0; j < 8; ++j) v[k][j] += r[j];
        // the residual stream is kept in bf16; normalize what is stored
        uint4 s = f32_to_bf16x8(v[k]);
        rr[i] = s;
        bf16x8_to_f32(s, v[k]);
      }
#pragma unroll
      for (int j = 0; j < 8; ++j) ss += v[k][j] * v[k][j];
    }
  }
  ss = block_sum(ss, red);
  const float inv = rsqrtf(ss / dim + eps);
  uint4* orow = reinterpret_cast<uint4*>(out + (size_t)row * dim);
  const uint4* wr = reinterpret_cast<const uint4*>(w);
#pragma unroll
  for (int k = 0; k < VPT; ++k) {
    const int i = threadIdx.x + k * blockDim.x;
    if (i < nvec) {
      float g[8];
      bf16x8_to_f32(__ldg(wr + i), g);
      float o[8];
#pragma unroll
      for (int j = 0; j < 8; ++j) o[j] = v[k][j] * inv * g[j];
      orow[i] = f32_to_bf16x8(o);
    }
  }
}

template <bool ADD>
void launch_rmsnorm(__nv_bfloat16* out, __nv_bfloat16* x, __nv_bfloat16* res, const __nv_bfloat16* w,
                    int rows, int dim, float eps, cudaStream_t s) {
  const int nvec = dim / 8;
  int threads = std::min(1024, ((nvec + 31) / 32) * 32);
  const int vpt = (nvec + threads - 1) / threads;
  if (vpt <= 1) msgl_launch(rmsnorm_kernel<1, ADD>, rows, threads, 0, s, 1, out, x, res, w, dim, eps);
  else if (vpt <= 2) msgl_launch(rmsnorm_kernel<2, ADD>, rows, threads, 0, s, 1, out, x, res, w, dim, eps);
  else msgl_launch(rmsnorm_kernel<4, ADD>, rows, threads, 0, s, 1, out, x, res, w, dim, eps);
}

// ------------------------------------------------------------------------------ act * mul
// x = [gate | up] halves (plain layout), out = act(gate) * up
__global__ void act_and_mul_kernel(uint4* __restrict__ out, const uint4* __restrict__ x, int rows,
                                   int inter_vec, int act) {
  pdl_wait();
  pdl_launch();
  const size_t total = (size_t)rows * inter_vec;
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < total; i += (size_t)gridDim.x * blockDim.x) {
    const size_t r = i / inter_vec, c = i % inter_vec;
    float g[8], u[8], o[8];
    bf16x8_to_f32(x[r * 2 * inter_vec + c], g);
    bf16x8_to_f32(x[r * 2 * inter_vec + inter_vec + c], u);
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      float a;
      if (act == 0) a = g[j] / (1.f + __expf(-g[j]));
      else a = 0.5f * g[j] * (1.f + tanhf(0.7978845608028654f * (g[j] + 0.044715f * g[j] * g[j] * g[j])));
      o[j] = a * u[j];
    }
    out[i] = f32_to_bf16x8(o);
  }
}

// ------------------------------------------------------------------------------ store kv
__global__ void store_kv_kernel(const uint4* __restrict__ k, const uint4* __restrict__ v,
                                uint4* __restrict__ kc, uint4* __restrict__ vc,
                                const int32_t* __restrict__ loc, int n, int vec_per_row,
                                int64_t k_stride_v, int64_t v_stride_v, int64_t c_stride_v,
                                int64_t num_slots) {
  pdl_wait();
  pdl_launch();
  const int row = blockIdx.x * (blockDim.x / 32) + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (row >= n) return;
  const int64_t slot = loc[row];
  if (!MSGL_IN_BOUNDS(slot >= 0 && slot < num_slots, kBcKvSlot)) return;
  for (int i = lane; i < vec_per_row; i += 32) {
    kc[slot * c_stride_v + i] = k[row * k_stride_v + i];
    vc[slot * c_stride_v + i] = v[row * v_stride_v + i];
  }
}

// ------------------------------------------------------------------------------ qk norm + rope + store
// One warp per (token, head) over the q, k and v heads of the merged qkv row. Lane l owns
// elements [l*E, l*E+E) of the first half and the same offsets of the second half (E = hd/64),
// so each neox-style rotation pair (i, i + hd/2) lives in one thread.
template <int E>
__global__ void qk_norm_rope_store_kernel(__nv_bfloat16* __restrict__ q_out,
                                          const __nv_bfloat16* __restrict__ qkv,
                                          const int32_t* __restrict__ positions,
                                          const float* __restrict__ cos_sin,
                                          const __nv_bfloat16* __restrict__ q_norm,
                                          const __nv_bfloat16* __restrict__ k_norm, float eps,
                                          __nv_bfloat16* __restrict__ k_cache,
                                          __nv_bfloat16* __restrict__ v_cache,
                                          const int32_t* __restrict__ out_loc, int n, int nq,
                                          int nkv, int64_t cache_stride, int64_t num_slots,
                                          int max_pos) {
  pdl_wait();
  pdl_launch();
  constexpr int HD = 64 * E;
  const int heads = nq + 2 * nkv;
  const int gw = blockIdx.x * (blockDim.x / 32) + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (gw >= n * heads) return;
  const int t = gw / heads, h = gw % heads;
  // (warp-uniform checks: one warp owns one (token, head))
  if (h >= nq && !MSGL_IN_BOUNDS(out_loc[t] >= 0 && out_loc[t] < num_slots, kBcKvSlot)) return;
  if (h < nq + nkv && !MSGL_IN_BOUNDS(positions[t] >= 0 && positions[t] < max_pos, kBcRopePos)) return;
  const __nv_bfloat16* src = qkv + (size_t)t * heads * HD + (size_t)h * HD;
  float a[E], b[E];
#pragma unroll
  for (int e = 0; e < E; ++e) {
    a[e] = __bfloat162float(src[lane * E + e]);
    b[e] = __bfloat162float(src[HD / 2 + lane * E + e]);
  }
  if (h >= nq + nkv) {  // v head: plain copy into the cache
    const int64_t slot = out_loc[t];
    __nv_bfloat16* dst = v_cache + slot * cache_stride + (size_t)(h - nq - nkv) * HD;
#pragma unroll
    for (int e = 0; e < E; ++e) {
      dst[lane * E + e] = __float2bfloat16(a[e]);
      dst[HD / 2 + lane * E + e] = __float2bfloat16(b[e]);
    }
    return;
  }
  const bool is_q = h < nq;
  const __nv_bfloat16* nw = is_q ? q_norm : k_norm;
  if (nw != nullptr) {
    float ss = 0.f;
#pragma unroll
    for (int e = 0; e < E; ++e) ss += a[e] * a[e] + b[e] * b[e];
    ss = warp_sum(ss);
    const float inv = rsqrtf(ss / HD + eps);
#pragma unroll
    for (int e = 0; e < E; ++e) {
      // match the reference rounding: normalized values are rounded to bf16 before RoPE
      a[e] = __bfloat162float(__float2bfloat16(a[e] * inv * __bfloat162float(nw[lane * E + e])));
      b[e] = __bfloat162float(__float2bfloat16(b[e] * inv * __bfloat162float(nw[HD / 2 + lane * E + e])));
    }
  }
  const int pos = positions[t];
  const float* cs = cos_sin + (size_t)pos * HD;
  __nv_bfloat16* dst;
  if (is_q) dst = q_out + ((size_t)t * nq + h) * HD;
  else dst = k_cache + (int64_t)out_loc[t] * cache_stride + (size_t)(h - nq) * HD;
#pragma unroll
  for (int e = 0; e < E; ++e) {
    const int i = lane * E + e;
    const float c = cs[i], s = cs[HD / 2 + i];
    dst[i] = __float2bfloat16(a[e] * c - b[e] * s);
    dst[HD / 2 + i] = __float2bfloat16(b[e] * c + a[e] * s);
  }
}

// ------------------------------------------------------------------------------ argmax
// One CTA per row; ties resolve to the lowest index (matches torch.argmax). 16-byte vector loads,
// four in flight per thread, so a row streams at HBM rate instead of one scalar per thread.
// Optionally writes the maximum value (for combining vocab shards across ranks).
template <typename T>
__global__ void argmax_kernel(int32_t* __restrict__ out, float* __restrict__ out_val, const T* __restrict__ logits,
                              int vocab, int64_t stride) {
  pdl_wait();
  pdl_launch();
  __shared__ float sv[32];
  __shared__ int si[32];
  const T* row = logits + (size_t)blockIdx.x * stride;
  float best = -FLT_MAX;
  int bi = 0x7fffffff;
  constexpr int VEC = 16 / (int)sizeof(T);
  constexpr int U = 4;
  const int nvec = (reinterpret_cast<uintptr_t>(row) % 16 == 0) ? vocab / VEC : 0;
  const uint4* rv = reinterpret_cast<const uint4*>(row);
  for (int base = threadIdx.x; base < nvec; base += blockDim.x * U) {
    uint4 u[U];
#pragma unroll
    for (int k = 0; k < U; ++k) {
      const int i = base + k * blockDim.x;
      if (i < nvec) u[k] = __ldg(rv + i);
    }
#pragma unroll
    for (int k = 0; k < U; ++k) {
      const int i = base + k * blockDim.x;
      if (i < nvec) {
        float f[VEC];
        if constexpr (sizeof(T) == 4) {
          f[0] = __uint_as_float(u[k].x); f[1] = __uint_as_float(u[k].y);
          f[2] = __uint_as_float(u[k].z); f[3] = __uint_as_float(u[k].w);
        } else {
          const uint32_t w[4] = {u[k].x, u[k].y, u[k].z, u[k].w};
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            f[2 * j] = __uint_as_float(w[j] << 16);
            f[2 * j + 1] = __uint_as_float(w[j] & 0xffff0000u);
          }
        }
#pragma unroll
        for (int j = 0; j < VEC; ++j)
          if (f[j] > best) { best = f[j]; bi = i * VEC + j; }
      }
    }
  }
  for (int i = nvec * VEC + threadIdx.x; i < vocab; i += blockDim.x) {
    float v;
    if constexpr (sizeof(T) == 4) v = row[i];
    else v = __bfloat162float(row[i]);
    if (v > best) { best = v; bi = i; }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float ov = __shfl_xor_sync(0xffffffffu, best, o);
    const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
    if (ov > best || (ov == best && oi < bi)) { best = ov; bi = oi; }
  }
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  if (lane == 0) { sv[warp] = best; si[warp] = bi; }
  __syncthreads();
  if (warp == 0) {
    const int nw = blockDim.x / 32;
    best = lane < nw ? sv[lane] : -FLT_MAX;
    bi = lane < nw ? si[lane] : 0x7fffffff;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float ov = __shfl_xor_sync(0xffffffffu, best, o);
      const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
      if (ov > best || (ov == best && oi < bi)) { best = ov; bi = oi; }
    }
    if (lane == 0) {
      out[blockIdx.x] = bi == 0x7fffffff ? 0 : bi;
      if (out_val != nullptr) out_val[blockIdx.x] = best;
    }
  }
}

}  // namespace

extern "C" void msgl_embedding(void* out, const void* weight, const int32_t* ids, int n, int dim,
                               int vocab_start, int vocab_len, int masked, cudaStream_t s) {
  if (n == 0) return;
  const int vec = dim / 8, wpb = 8;
  msgl_launch(embedding_kernel, (n + wpb - 1) / wpb, wpb * 32, 0, s, 1, reinterpret_cast<uint4*>(out),
              reinterpret_cast<const uint4*>(weight), ids, n, vec, vocab_start, vocab_len, masked);
}

extern "C" void msgl_rmsnorm(void* out, const void* x, const void* w, int rows, int dim, float eps,
                             cudaStream_t s) {
  if (rows == 0) return;
  launch_rmsnorm<false>(reinterpret_cast<__nv_bfloat16*>(out),
                        reinterpret_cast<__nv_bfloat16*>(const_cast<void*>(x)), nullptr,
                        reinterpret_cast<const __nv_bfloat16*>(w), rows, dim, eps, s);
}

extern "C" void msgl_fused_add_rmsnorm(void* x, void* residual, const void* w, int rows, int dim,
                                       float eps, cudaStream_t s) {
  if (rows == 0) return;
  auto xp = reinterpret_cast<__nv_bfloat16*>(x);
  launch_rmsnorm<true>(xp, xp, reinterpret_cast<__nv_bfloat16*>(residual),
                       reinterpret_cast<const __nv_bfloat16*>(w), rows, dim, eps, s);
}

extern "C" void msgl_act_and_mul(void* out, const void* x, int rows, int inter, int act, cudaStream_t s) {
  if (rows == 0) return;
  const size_t total = (size_t)rows * inter / 8;
  const int grid = (int)std::min<size_t>((total + 255) / 256, 148 * 16);
  msgl_launch(act_and_mul_kernel, grid, 256, 0, s, 1, reinterpret_cast<uint4*>(out),
              reinterpret_cast<const uint4*>(x), rows, inter / 8, act);
}

extern "C" void msgl_store_kv(const void* k, const void* v, void* k_cache, void* v_cache,
                              const int32_t* out_loc, int n, int row_elems, int64_t k_stride,
                              int64_t v_stride, int64_t cache_stride, int64_t num_slots, cudaStream_t s) {
  if (n == 0) return;
  const int wpb = 8;
  msgl_launch(store_kv_kernel, (n + wpb - 1) / wpb, wpb * 32, 0, s, 1, reinterpret_cast<const uint4*>(k),
              reinterpret_cast<const uint4*>(v), reinterpret_cast<uint4*>(k_cache),
              reinterpret_cast<uint4*>(v_cache), out_loc, n, row_elems / 8, k_stride / 8, v_stride / 8,
              cache_stride / 8, num_slots);
}

extern "C" void msgl_qk_norm_rope_store(void* q_out, const void* qkv, const int32_t* positions,
                                        const float* cos_sin, const void* q_norm, const void* k_norm,
                                        float eps, void* k_cache, void* v_cache,
                                        const int32_t* out_loc, int n, int nq, int nkv, int hd,
                                        int64_t cache_stride, int64_t num_slots, int max_pos, cudaStream_t s) {
  if (n == 0) return;
  const int warps = n * (nq + 2 * nkv), wpb = 8;
  const dim3 grid((warps + wpb - 1) / wpb);
  auto qo = reinterpret_cast<__nv_bfloat16*>(q_out);
  auto src = reinterpret_cast<const __nv_bfloat16*>(qkv);
  auto qn = reinterpret_cast<const __nv_bfloat16*>(q_norm);
  auto kn = reinterpret_cast<const __nv_bfloat16*>(k_norm);
  auto kc = reinterpret_cast<__nv_bfloat16*>(k_cache);
  auto vc = reinterpret_cast<__nv_bfloat16*>(v_cache);
  if (hd == 64)
    msgl_launch(qk_norm_rope_store_kernel<1>, grid, wpb * 32, 0, s, 1, qo, src, positions, cos_sin, qn, kn, eps, kc, vc, out_loc, n, nq, nkv, cache_stride, num_slots, max_pos);
  else if (hd == 128)
    msgl_launch(qk_norm_rope_store_kernel<2>, grid, wpb * 32, 0, s, 1, qo, src, positions, cos_sin, qn, kn, eps, kc, vc, out_loc, n, nq, nkv, cache_stride, num_slots, max_pos);
  else
    msgl_launch(qk_norm_rope_store_kernel<4>, grid, wpb * 32, 0, s, 1, qo, src, positions, cos_sin, qn, kn, eps, kc, vc, out_loc, n, nq, nkv, cache_stride, num_slots, max_pos);
}

extern "C" void msgl_argmax(int32_t* out, float* out_val, const void* logits, int rows, int vocab, int64_t stride,
                            int is_fp32, cudaStream_t s) {
  if (rows == 0) return;
  if (is_fp32)
    msgl_launch(argmax_kernel<float>, rows, 512, 0, s, 1, out, out_val, reinterpret_cast<const float*>(logits), vocab,
                stride);
  else
    msgl_launch(argmax_kernel<__nv_bfloat16>, rows, 512, 0, s, 1, out, out_val,
                reinterpret_cast<const __nv_bfloat16*>(logits), vocab, stride);
}

MSGL_ERROR_ACCESSOR(msgl_err_elementwise)
