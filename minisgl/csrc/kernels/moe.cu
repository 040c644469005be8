// Routed-expert (MoE) support kernels around the grouped tcgen05 GEMM:
//   route     - per token: softmax top-k (optionally renormalized) or top-k then softmax (gpt-oss)
//   align     - counting sort of the (token, slot) pairs by expert into padded segments of `bn`
//               rows, plus the device work list {expert, first row} of every token tile
//   gather    - permuted activations xs[row] = x[token(row)] (zero rows for padding)
//   act       - gate/up halves -> act(gate) * up, with the gpt-oss clamped SwiGLU variant
//   combine   - out[t] = sum_k w[t,k] * y[row(t,k)] in fp32
// Everything stays on the device (no host sync), so the MoE layer can be captured in CUDA graphs.
#include <cfloat>

#include "api.h"
#include "common.cuh"

using namespace msgl;

namespace {

constexpr int kMaxTopK = 16;

// one warp per token; E <= 32 * 16
__global__ void route_kernel(const float* __restrict__ logits, int T, int E, int topk, int renorm,
                             int softmax_after, float* __restrict__ weights, int32_t* __restrict__ ids) {
  pdl_wait();
  pdl_launch();
  const int t = blockIdx.x * (blockDim.x / 32) + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (t >= T) return;
  const float* row = logits + (size_t)t * E;
  constexpr int kPer = 16;
  float v[kPer];
#pragma unroll
  for (int i = 0; i < kPer; ++i) {
    const int e = lane + 32 * i;
    v[i] = e < E ? row[e] : -INFINITY;
  }
  float mx = -INFINITY;
#pragma unroll
  for (int i = 0; i < kPer; ++i) mx = fmaxf(mx, v[i]);
  mx = warp_max(mx);
  float denom = 0.f;
  if (!softmax_after) {
#pragma unroll
    for (int i = 0; i < kPer; ++i) denom += (lane + 32 * i < E) ? __expf(v[i] - mx) : 0.f;
    denom = warp_sum(denom);
  }
  float selw[kMaxTopK];
  int seli[kMaxTopK];
  float sum_sel = 0.f;
  for (int k = 0; k < topk; ++k) {
    // argmax over remaining (ties -> lowest expert id)
    float bv = -INFINITY;
    int bi = 0x7fffffff;
#pragma unroll
    for (int i = 0; i < kPer; ++i) {
      const int e = lane + 32 * i;
      if (e < E && (v[i] > bv || (v[i] == bv && e < bi))) { bv = v[i]; bi = e; }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
      const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
      if (ov > bv || (ov == bv && oi < bi)) { bv = ov; bi = oi; }
    }
    seli[k] = bi;
    selw[k] = softmax_after ? bv : __expf(bv - mx) / denom;
    sum_sel += selw[k];
#pragma unroll
    for (int i = 0; i < kPer; ++i)
      if (lane + 32 * i == bi) v[i] = -INFINITY;
  }
  if (lane == 0) {
    if (softmax_after) {  // softmax over the selected logits
      float m2 = selw[0], d = 0.f;
      for (int k = 0; k < topk; ++k) m2 = fmaxf(m2, selw[k]);
      for (int k = 0; k < topk; ++k) { selw[k] = __expf(selw[k] - m2); d += selw[k]; }
      for (int k = 0; k < topk; ++k) selw[k] /= d;
    } else if (renorm) {
      for (int k = 0; k < topk; ++k) selw[k] /= sum_sel;
    }
    for (int k = 0; k < topk; ++k) {
      weights[t * topk + k] = selw[k];
      ids[t * topk + k] = seli[k];
    }
  }
}

// single CTA: counts -> padded segment starts -> tile work list -> scatter of pair positions.
// perm[row] = pair index (token * topk + k) or -1 for padding; inv[pair] = row.
// Expert parallelism: only experts [e0, e0 + E) live on this rank; assignments to other experts
// are dropped (inv = -1, no rows) and contribute nothing to the combine.
__global__ void __launch_bounds__(1024) align_kernel(const int32_t* __restrict__ ids, int pairs, int E, int e0, int bn,
                                                     int max_tiles, int rows_cap, int32_t* __restrict__ perm,
                                                     int32_t* __restrict__ inv, int2* __restrict__ work,
                                                     int32_t* __restrict__ tile_count) {
  pdl_wait();
  pdl_launch();
  extern __shared__ int sm[];
  int* cnt = sm;            // [E]
  int* start = sm + E;      // [E]
  int* cursor = sm + 2 * E; // [E]
  int* tstart = sm + 3 * E; // [E]
  for (int e = threadIdx.x; e < E; e += blockDim.x) cnt[e] = 0;
  __syncthreads();
  for (int i = threadIdx.x; i < pairs; i += blockDim.x) {
    const int e = ids[i] - e0;
    if (e >= 0 && e < E) atomicAdd(&cnt[e], 1);
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    int row = 0, tile = 0;
    for (int e = 0; e < E; ++e) {
      start[e] = row;
      tstart[e] = tile;
      cursor[e] = 0;
      const int tiles = (cnt[e] + bn - 1) / bn;
      row += tiles * bn;
      tile += tiles;
    }
    *tile_count = min(tile, max_tiles);
  }
  __syncthreads();
  for (int r = threadIdx.x; r < rows_cap; r += blockDim.x) perm[r] = -1;
  for (int e = threadIdx.x; e < E; e += blockDim.x) {
    const int tiles = (cnt[e] + bn - 1) / bn;
    for (int j = 0; j < tiles && tstart[e] + j < max_tiles; ++j) work[tstart[e] + j] = make_int2(e, start[e] + j * bn);
  }
  __syncthreads();
  for (int i = threadIdx.x; i < pairs; i += blockDim.x) {
    const int e = ids[i] - e0;
    if (e < 0 || e >= E) {
      inv[i] = -1;
      continue;
    }
    const int pos = start[e] + atomicAdd(&cursor[e], 1);
    perm[pos] = i;
    inv[i] = pos;
  }
}

// xs[row] = x[perm[row] / topk] (16-byte vectors), zero for padding rows
__global__ void gather_rows_kernel(uint4* __restrict__ xs, const uint4* __restrict__ x, const int32_t* __restrict__ perm,
                                   int rows, int vec, int topk, int x_rows) {
  pdl_wait();
  pdl_launch();
  const int r = blockIdx.x * (blockDim.x / 32) + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (r >= rows) return;
  int p = perm[r];
  uint4* dst = xs + (size_t)r * vec;
  if (p >= 0 && !MSGL_IN_BOUNDS(p / topk < x_rows, kBcMoePerm)) p = -1;
  if (p < 0) {
    for (int i = lane; i < vec; i += 32) dst[i] = make_uint4(0, 0, 0, 0);
    return;
  }
  const uint4* src = x + (size_t)(p / topk) * vec;
  for (int i = lane; i < vec; i += 32) dst[i] = src[i];
}

// y = [gate | up] (halves of 2I) -> act(gate) * up ; act 0 silu, 1 gelu(tanh), 2 gpt-oss swiglu
__global__ void expert_act_kernel(__nv_bfloat16* __restrict__ out, const __nv_bfloat16* __restrict__ y, int rows,
                                  int inter, int act, const int32_t* __restrict__ perm) {
  pdl_wait();
  pdl_launch();
  const size_t total = (size_t)rows * inter;
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < total; i += (size_t)gridDim.x * blockDim.x) {
    const size_t r = i / inter, c = i % inter;
    if (perm[r] < 0) { out[i] = __float2bfloat16(0.f); continue; }
    float g = __bfloat162float(y[r * 2 * inter + c]);
    float u = __bfloat162float(y[r * 2 * inter + inter + c]);
    float a;
    if (act == 0) a = g / (1.f + __expf(-g)) * u;
    else if (act == 1) a = 0.5f * g * (1.f + tanhf(0.7978845608028654f * (g + 0.044715f * g * g * g))) * u;
    else {
      g = fminf(g, 7.f);
      u = fminf(fmaxf(u, -7.f), 7.f);
      a = g / (1.f + __expf(-1.702f * g)) * (u + 1.f);
    }
    out[i] = __float2bfloat16(a);
  }
}

// out[t, :] = sum_k w[t,k] * y[inv[t*topk+k], :]   (one CTA per token, fp32 accumulate)
__global__ void combine_kernel(__nv_bfloat16* __restrict__ out, const __nv_bfloat16* __restrict__ y,
                               const float* __restrict__ w, const int32_t* __restrict__ inv, int H, int topk,
                               int y_rows) {
  pdl_wait();
  pdl_launch();
  const int t = blockIdx.x;
  for (int c = threadIdx.x * 2; c < H; c += blockDim.x * 2) {
    float a0 = 0.f, a1 = 0.f;
    for (int k = 0; k < topk; ++k) {
      const int row = inv[t * topk + k];
      if (row < 0) continue;  // expert lives on another rank
      if (!MSGL_IN_BOUNDS(row < y_rows, kBcMoeInv)) continue;
      const float wk = w[t * topk + k];
      const __nv_bfloat162 v = *reinterpret_cast<const __nv_bfloat162*>(y + (size_t)row * H + c);
      a0 += wk * __bfloat162float(v.x);
      a1 += wk * __bfloat162float(v.y);
    }
    *reinterpret_cast<__nv_bfloat162*>(out + (size_t)t * H + c) = __floats2bfloat162_rn(a0, a1);
  }
}

}  // namespace

extern "C" {

void msgl_moe_route(const float* logits, int T, int E, int topk, int renorm, int softmax_after, float* weights,
                    int32_t* ids, cudaStream_t s) {
  if (T == 0) return;
  msgl_launch(route_kernel, dim3((T + 7) / 8), dim3(256), 0, s, 1, logits, T, E, topk, renorm, softmax_after,
              weights, ids);
}

void msgl_moe_align(const int32_t* ids, int pairs, int E, int e0, int bn, int max_tiles, int rows_cap, int32_t* perm,
                    int32_t* inv, void* work, int32_t* tile_count, cudaStream_t s) {
  msgl_launch(align_kernel, dim3(1), dim3(1024), (size_t)4 * E * sizeof(int), s, 1, ids, pairs, E, e0, bn, max_tiles,
              rows_cap, perm, inv, reinterpret_cast<int2*>(work), tile_count);
}

void msgl_moe_gather(void* xs, const void* x, const int32_t* perm, int rows, int H, int topk, int x_rows,
                     cudaStream_t s) {
  if (rows == 0) return;
  msgl_launch(gather_rows_kernel, dim3((rows + 7) / 8), dim3(256), 0, s, 1, reinterpret_cast<uint4*>(xs),
              reinterpret_cast<const uint4*>(x), perm, rows, H / 8, topk, x_rows);
}

void msgl_moe_act(void* out, const void* y, int rows, int inter, int act, const int32_t* perm, cudaStream_t s) {
  if (rows == 0) return;
  const size_t total = (size_t)rows * inter;
  const int grid = (int)std::min<size_t>((total + 255) / 256, 148 * 16);
  msgl_launch(expert_act_kernel, dim3(grid), dim3(256), 0, s, 1, reinterpret_cast<__nv_bfloat16*>(out),
              reinterpret_cast<const __nv_bfloat16*>(y), rows, inter, act, perm);
}

void msgl_moe_combine(void* out, const void* y, const float* w, const int32_t* inv, int T, int H, int topk,
                      int y_rows, cudaStream_t s) {
  if (T == 0) return;
  msgl_launch(combine_kernel, dim3(T), dim3(256), 0, s, 1, reinterpret_cast<__nv_bfloat16*>(out),
              reinterpret_cast<const __nv_bfloat16*>(y), w, inv, H, topk, y_rows);
}

}  // extern "C"

MSGL_ERROR_ACCESSOR(msgl_err_moe)
