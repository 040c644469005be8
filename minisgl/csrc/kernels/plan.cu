// Batch metadata on the device, from the one packed int32 upload per batch (the reference builds
// the same glue with PyTorch indexing: python/minisgl/scheduler/scheduler.py:204-267 and
// python/minisgl/scheduler/cache.py:127-146).
//
//   plan_apply:     page_table[pt_rows[i], pt_pos[i]] = pt_slots[i]   for every page-table write,
//                   then out_loc[t] = page_table[tok_rows[t], positions[t]] for every token
//                   (one CTA: the gather must see the writes, and a CTA barrier orders them);
//   gather_i32:     dst[i] = src[idx[i]]   (decode input ids from the per-row last sampled token);
//   scatter_i32:    dst[idx[i]] = src[i]   (sampled tokens back into their rows).
// Indices come from the host-built plan; the bounds-check build verifies them against the tables.
#include "api.h"
#include "common.cuh"

using namespace msgl;

namespace {

constexpr int kPlanThreads = 1024;

__global__ void __launch_bounds__(kPlanThreads) plan_apply_kernel(int32_t* __restrict__ page_table, int64_t pt_stride,
                                                                  int64_t pt_rows_total, const int32_t* __restrict__ pt_rows,
                                                                  const int32_t* __restrict__ pt_pos,
                                                                  const int32_t* __restrict__ pt_slots, int n_writes,
                                                                  const int32_t* __restrict__ tok_rows,
                                                                  const int32_t* __restrict__ positions, int n_tok,
                                                                  int32_t* __restrict__ out_loc) {
  pdl_wait();
  pdl_launch();
  for (int i = threadIdx.x; i < n_writes; i += kPlanThreads) {
    const int r = pt_rows[i], c = pt_pos[i];
    if (MSGL_IN_BOUNDS(r >= 0 && r < pt_rows_total && c >= 0 && c < pt_stride, kBcAttnRow))
      page_table[(int64_t)r * pt_stride + c] = pt_slots[i];
  }
  __syncthreads();  // the gather below reads entries written above (CTA-scope visibility)
  for (int t = threadIdx.x; t < n_tok; t += kPlanThreads) {
    const int r = tok_rows[t], c = positions[t];
    int32_t v = 0;
    if (MSGL_IN_BOUNDS(r >= 0 && r < pt_rows_total && c >= 0 && c < pt_stride, kBcAttnRow))
      v = page_table[(int64_t)r * pt_stride + c];
    out_loc[t] = v;
  }
}

__global__ void gather_i32_kernel(int32_t* __restrict__ dst, const int32_t* __restrict__ src, int64_t src_len,
                                  const int32_t* __restrict__ idx, int n) {
  pdl_wait();
  pdl_launch();
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n) return;
  const int j = idx[i];
  dst[i] = MSGL_IN_BOUNDS(j >= 0 && j < src_len, kBcAttnRow) ? src[j] : 0;
}

__global__ void scatter_i32_kernel(int32_t* __restrict__ dst, int64_t dst_len, const int32_t* __restrict__ idx,
                                   const int32_t* __restrict__ src, int n) {
  pdl_wait();
  pdl_launch();
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n) return;
  const int j = idx[i];
  if (MSGL_IN_BOUNDS(j >= 0 && j < dst_len, kBcAttnRow)) dst[j] = src[i];
}

}  // namespace

extern "C" void msgl_plan_apply(int32_t* page_table, int64_t pt_stride, int64_t pt_rows_total, const int32_t* pt_rows,
                                const int32_t* pt_pos, const int32_t* pt_slots, int n_writes, const int32_t* tok_rows,
                                const int32_t* positions, int n_tok, int32_t* out_loc, cudaStream_t s) {
  if (n_writes == 0 && n_tok == 0) return;
  msgl_launch(plan_apply_kernel, dim3(1), dim3(kPlanThreads), 0, s, 1, page_table, pt_stride, pt_rows_total, pt_rows,
              pt_pos, pt_slots, n_writes, tok_rows, positions, n_tok, out_loc);
}

extern "C" void msgl_gather_i32(int32_t* dst, const int32_t* src, int64_t src_len, const int32_t* idx, int n,
                                cudaStream_t s) {
  if (n == 0) return;
  msgl_launch(gather_i32_kernel, dim3((n + 255) / 256), dim3(256), 0, s, 1, dst, src, src_len, idx, n);
}

extern "C" void msgl_scatter_i32(int32_t* dst, int64_t dst_len, const int32_t* idx, const int32_t* src, int n,
                                 cudaStream_t s) {
  if (n == 0) return;
  msgl_launch(scatter_i32_kernel, dim3((n + 255) / 256), dim3(256), 0, s, 1, dst, dst_len, idx, src, n);
}

MSGL_ERROR_ACCESSOR(msgl_err_plan)
