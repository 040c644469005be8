// Persistent, warp-specialized bf16 GEMM on the 5th-generation tensor core (tcgen05 + TMEM + TMA).
//
//   out[M, N] = epilogue( x[M, K] @ w[N, K]^T + bias[N] )
//
// Orientation ("swap-AB"): the weight tile is the MMA's A operand (M = 128 weight rows) and the
// activations are the B operand (N = BN tokens, 16..256). A decode batch of any size therefore
// maps onto one MMA column tile, and every weight byte is streamed from HBM once per call.
//
// Warp roles (192 threads, one CTA per SM, persistent over work units):
//   warp 0      : TMA producer (one lane), fills a STAGES-deep ring of {A,B} tiles in smem.
//   warp 1      : TMEM allocator + MMA issuer (one lane); accumulates a 128 x BN fp32 tile in
//                 TMEM, double buffered so the epilogue of tile i overlaps the MMAs of tile i+1.
//   warps 2..5  : epilogue; warp w reads TMEM lanes 32*(w%4).. via tcgen05.ld, applies bias /
//                 activation, transposes through smem and writes 16-byte vectors.
// Split-K (small-M decode with few weight tiles): each split writes an fp32 partial to the
// workspace; the last split to arrive (atomic tile counter) reduces and runs the epilogue, then
// resets the counter so the next launch (or CUDA-graph replay) starts from zero.
#include <algorithm>
#include <cstdio>
#include <mutex>

#include "api.h"
#include "common.cuh"

namespace msgl {
namespace gemm {

constexpr int BM = 128;
constexpr int BK = 64;
constexpr int kThreads = 192;
constexpr int kEpiWarps = 4;

enum Epi : int { kBf16 = 0, kSilu = 1, kGelu = 2, kF32 = 3 };

template <int BN>
struct Cfg {
  static constexpr int kA = BM * BK * 2;
  static constexpr int kB = BN * BK * 2;
  static constexpr int kStage = kA + kB;
  static constexpr int kEpiBuf = 32 * 33 * 4;  // per epilogue warp: 32x32 fp32, padded
  static constexpr int kStages = std::min(8, (220 * 1024 - kEpiWarps * kEpiBuf) / kStage);
  static constexpr int kTmemCols = 2 * BN < 32 ? 32 : 2 * BN;
  static constexpr int kSmem = 1024 + kStages * kStage + kEpiWarps * kEpiBuf + 256;
};

struct Params {
  void* out;
  const __nv_bfloat16* bias;
  float* partials;  // [units_tiles * splits, BM, BN]
  int* counters;    // [tiles]
  int M, N, K, ldo;
  int n_tiles, m_tiles, splits, kblocks;
};

__device__ __forceinline__ float act_silu(float g) { return g / (1.f + __expf(-g)); }
__device__ __forceinline__ float act_gelu(float g) {
  const float k0 = 0.7978845608028654f, k1 = 0.044715f;
  return 0.5f * g * (1.f + tanhf(k0 * (g + k1 * g * g * g)));
}

// tile id -> (n_tile, m_tile); groups of 8 weight tiles sweep all token tiles so the weight
// tiles of one wave stay resident in L2 while activations stream.
__device__ __forceinline__ void tile_coords(int tile, int n_tiles, int m_tiles, int& nt, int& mt) {
  constexpr int G = 8;
  const int per_group = G * m_tiles;
  const int g = tile / per_group;
  const int r = tile - g * per_group;
  const int gsize = min(G, n_tiles - g * G);
  nt = g * G + r % gsize;
  mt = r / gsize;
}

template <int BN, int EPI>
__global__ void __launch_bounds__(kThreads, 1)
gemm_kernel(const __grid_constant__ CUtensorMap tmap_w, const __grid_constant__ CUtensorMap tmap_x,
            Params p) {
  using C = Cfg<BN>;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* stage_base = smem;
  float* epi_buf = reinterpret_cast<float*>(smem + C::kStages * C::kStage);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + C::kStages * C::kStage + kEpiWarps * C::kEpiBuf);
  uint64_t* full = bars;
  uint64_t* empty = bars + C::kStages;
  uint64_t* tfull = bars + 2 * C::kStages;
  uint64_t* tempty = tfull + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(tempty + 2);
  int* flag_slot = reinterpret_cast<int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int tiles = p.n_tiles * p.m_tiles;
  const int units = tiles * p.splits;

  if (threadIdx.x == 0) {
    for (int i = 0; i < C::kStages; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&tfull[i], 1);
      mbar_init(&tempty[i], kEpiWarps);
    }
    fence_barrier_init();
    prefetch_tmap(&tmap_w);
    prefetch_tmap(&tmap_x);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, C::kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 0) {
    // ------------------------------------------------------------------ TMA producer
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      for (int u = blockIdx.x; u < units && ok; u += gridDim.x) {
        const int split = u % p.splits, tile = u / p.splits;
        int nt, mt;
        tile_coords(tile, p.n_tiles, p.m_tiles, nt, mt);
        const int kb0 = (int)((long long)split * p.kblocks / p.splits);
        const int kb1 = (int)((long long)(split + 1) * p.kblocks / p.splits);
        for (int kb = kb0; kb < kb1; ++kb) {
          if (!mbar_wait(&empty[stage], phase ^ 1, 100)) { ok = false; break; }
          uint8_t* a = stage_base + stage * C::kStage;
          mbar_expect_tx(&full[stage], C::kStage);
          tma_load_2d(a, &tmap_w, &full[stage], kb * BK, nt * BM);
          tma_load_2d(a + C::kA, &tmap_x, &full[stage], kb * BK, mt * BN);
          if (++stage == C::kStages) { stage = 0; phase ^= 1; }
        }
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      constexpr uint32_t idesc = idesc_bf16_f32(BM, BN);
      int stage = 0;
      uint32_t phase = 0;
      int use = 0;
      bool ok = true;
      for (int u = blockIdx.x; u < units && ok; u += gridDim.x, ++use) {
        const int split = u % p.splits;
        const int kb0 = (int)((long long)split * p.kblocks / p.splits);
        const int kb1 = (int)((long long)(split + 1) * p.kblocks / p.splits);
        const int acc = use & 1;
        if (!mbar_wait(&tempty[acc], ((use >> 1) & 1) ^ 1, 200)) break;
        tc_fence_after();
        const uint32_t d = tmem_base + acc * BN;
        for (int kb = kb0; kb < kb1; ++kb) {
          if (!mbar_wait(&full[stage], phase, 201)) { ok = false; break; }
          tc_fence_after();
          const uint32_t a = smem_u32(stage_base + stage * C::kStage);
          const uint32_t b = a + C::kA;
#pragma unroll
          for (int k = 0; k < BK / 16; ++k) {
            tc_mma_f16(d, smem_desc_sw128(a + k * 32), smem_desc_sw128(b + k * 32), idesc,
                       (kb > kb0 || k > 0) ? 1u : 0u);
          }
          tc_commit(&empty[stage]);
          if (++stage == C::kStages) { stage = 0; phase ^= 1; }
        }
        tc_commit(&tfull[acc]);
      }
    }
  } else {
    // ------------------------------------------------------------------ epilogue
    const int q = warp & 3;  // TMEM lane quadrant this warp may access
    const int ep_tid = threadIdx.x - 64;
    float* buf = epi_buf + q * 32 * 33;
    int use = 0;
    for (int u = blockIdx.x; u < units; u += gridDim.x, ++use) {
      const int split = u % p.splits, tile = u / p.splits;
      int nt, mt;
      tile_coords(tile, p.n_tiles, p.m_tiles, nt, mt);
      const int acc = use & 1;
      if (!mbar_wait(&tfull[acc], (use >> 1) & 1, 300)) break;
      tc_fence_after();
      const uint32_t tbase = tmem_base + acc * BN + ((uint32_t)(q * 32) << 16);
      const int n_row = nt * BM + q * 32 + lane;  // weight row owned by this thread
      const int m0 = mt * BN;

      bool do_epilogue = true;
      if (p.splits > 1) {
        // write this split's partial (row-major [BM][BN] per unit), then count arrivals
        float* part = p.partials + ((size_t)tile * p.splits + split) * BM * BN + (size_t)(q * 32 + lane) * BN;
#pragma unroll 1
        for (int c = 0; c < BN; c += 32) {
          if constexpr (BN >= 32) {
            uint32_t r[32];
            tmem_ld_32x32b_x32(tbase + c, r);
            tc_wait_ld();
#pragma unroll
            for (int j = 0; j < 32; j += 4)
              *reinterpret_cast<float4*>(part + c + j) =
                  make_float4(__uint_as_float(r[j]), __uint_as_float(r[j + 1]),
                              __uint_as_float(r[j + 2]), __uint_as_float(r[j + 3]));
          } else {
            uint32_t r[16];
            tmem_ld_32x32b_x16(tbase + c, r);
            tc_wait_ld();
#pragma unroll
            for (int j = 0; j < 16; j += 4)
              *reinterpret_cast<float4*>(part + c + j) =
                  make_float4(__uint_as_float(r[j]), __uint_as_float(r[j + 1]),
                              __uint_as_float(r[j + 2]), __uint_as_float(r[j + 3]));
          }
        }
        __threadfence();
        named_bar_sync(1, kEpiWarps * 32);
        if (ep_tid == 0) {
          const int old = atomicAdd(&p.counters[tile], 1);
          const int last = old == p.splits - 1;
          if (last) p.counters[tile] = 0;  // re-arm for the next launch
          *flag_slot = last;
        }
        named_bar_sync(1, kEpiWarps * 32);
        do_epilogue = *flag_slot != 0;
        __threadfence();
      }

      if (do_epilogue) {
        float bias_v = 0.f;
        if (p.bias != nullptr && n_row < p.N) bias_v = __bfloat162float(p.bias[n_row]);
        const bool is_act = EPI == kSilu || EPI == kGelu;
#pragma unroll 1
        for (int c = 0; c < BN; c += 32) {
          constexpr int W = BN >= 32 ? 32 : 16;
          float v[32];
          if (p.splits > 1) {
            // reduce all partials of this tile for columns [c, c + W)
#pragma unroll
            for (int j = 0; j < W; ++j) v[j] = 0.f;
            for (int s = 0; s < p.splits; ++s) {
              const float* part = p.partials + ((size_t)tile * p.splits + s) * BM * BN +
                                  (size_t)(q * 32 + lane) * BN + c;
#pragma unroll
              for (int j = 0; j < W; j += 4) {
                const float4 t = __ldcg(reinterpret_cast<const float4*>(part + j));
                v[j] += t.x; v[j + 1] += t.y; v[j + 2] += t.z; v[j + 3] += t.w;
              }
            }
          } else if constexpr (W == 32) {
            uint32_t r[32];
            tmem_ld_32x32b_x32(tbase + c, r);
            tc_wait_ld();
#pragma unroll
            for (int j = 0; j < 32; ++j) v[j] = __uint_as_float(r[j]);
          } else {
            uint32_t r[16];
            tmem_ld_32x32b_x16(tbase + c, r);
            tc_wait_ld();
#pragma unroll
            for (int j = 0; j < 16; ++j) v[j] = __uint_as_float(r[j]);
          }
#pragma unroll
          for (int j = 0; j < W; ++j) v[j] += bias_v;

          if constexpr (is_act) {
            // quadrants 2,3 hold "up" rows, 0,1 hold the matching "gate" rows
            if (q >= 2) {
#pragma unroll
              for (int j = 0; j < W; ++j) buf[j * 33 + lane] = v[j];
            }
            named_bar_sync(1, kEpiWarps * 32);
            if (q < 2) {
              const float* up = epi_buf + (q + 2) * 32 * 33;
#pragma unroll
              for (int j = 0; j < W; ++j) {
                const float g = v[j];
                const float a = EPI == kSilu ? act_silu(g) : act_gelu(g);
                buf[j * 33 + lane] = a * up[j * 33 + lane];
              }
              __syncwarp();
              // 32 (or 16) token rows x 32 output cols bf16 = 4 x 16B per row
              const int ncol0 = nt * (BM / 2) + q * 32;
#pragma unroll
              for (int i = 0; i < W / 8; ++i) {
                const int idx = lane + 32 * i, row = idx >> 2, part = idx & 3;
                const int m = m0 + c + row, n = ncol0 + part * 8;
                if (m < p.M && n < p.N / 2) {
                  const float* s = buf + row * 33 + part * 8;
                  uint4 o;
                  o.x = pack_bf16(s[0], s[1]); o.y = pack_bf16(s[2], s[3]);
                  o.z = pack_bf16(s[4], s[5]); o.w = pack_bf16(s[6], s[7]);
                  *reinterpret_cast<uint4*>(reinterpret_cast<__nv_bfloat16*>(p.out) + (size_t)m * p.ldo + n) = o;
                }
              }
            }
            named_bar_sync(1, kEpiWarps * 32);
          } else {
#pragma unroll
            for (int j = 0; j < W; ++j) buf[j * 33 + lane] = v[j];
            __syncwarp();
            const int ncol0 = nt * BM + q * 32;
            if constexpr (EPI == kF32) {
#pragma unroll
              for (int i = 0; i < W / 4; ++i) {
                const int idx = lane + 32 * i, row = idx >> 3, part = idx & 7;
                const int m = m0 + c + row, n = ncol0 + part * 4;
                if (m < p.M && n < p.N) {
                  const float* s = buf + row * 33 + part * 4;
                  *reinterpret_cast<float4*>(reinterpret_cast<float*>(p.out) + (size_t)m * p.ldo + n) =
                      make_float4(s[0], s[1], s[2], s[3]);
                }
              }
            } else {
#pragma unroll
              for (int i = 0; i < W / 8; ++i) {
                const int idx = lane + 32 * i, row = idx >> 2, part = idx & 3;
                const int m = m0 + c + row, n = ncol0 + part * 8;
                if (m < p.M && n < p.N) {
                  const float* s = buf + row * 33 + part * 8;
                  uint4 o;
                  o.x = pack_bf16(s[0], s[1]); o.y = pack_bf16(s[2], s[3]);
                  o.z = pack_bf16(s[4], s[5]); o.w = pack_bf16(s[6], s[7]);
                  *reinterpret_cast<uint4*>(reinterpret_cast<__nv_bfloat16*>(p.out) + (size_t)m * p.ldo + n) = o;
                }
              }
            }
            __syncwarp();
          }
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&tempty[acc]);
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, C::kTmemCols);
  }
}

// ------------------------------------------------------------------------------------------ host
typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                  const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                  const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                  CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(ptr);
  });
  return fn;
}

// 2-D bf16 row-major [rows, cols] (cols contiguous), box [box_rows, 64], 128-byte swizzle.
static CUtensorMap make_map(const void* base, int rows, int cols, int ld, int box_rows) {
  CUtensorMap m;
  cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)ld * 2};
  cuuint32_t box[2] = {(cuuint32_t)BK, (cuuint32_t)box_rows};
  cuuint32_t estr[2] = {1, 1};
  EncodeTiledFn fn = encode_fn();
  if (fn == nullptr) {
    fprintf(stderr, "minisgl: cuTensorMapEncodeTiled unavailable\n");
    memset(&m, 0, sizeof(m));
    return m;
  }
  CUresult r = fn(&m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides,
                  box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) fprintf(stderr, "minisgl: cuTensorMapEncodeTiled failed (%d)\n", (int)r);
  return m;
}

static int num_sms_cached() {
  static int n = 0;
  if (n == 0) {
    int dev = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
    if (n <= 0) n = 148;
  }
  return n;
}

template <int BN, int EPI>
static void launch(const Params& p, const CUtensorMap& mw, const CUtensorMap& mx, cudaStream_t s) {
  using C = Cfg<BN>;
  static bool attr_set = false;
  if (!attr_set) {
    cudaFuncSetAttribute(gemm_kernel<BN, EPI>, cudaFuncAttributeMaxDynamicSharedMemorySize, C::kSmem);
    attr_set = true;
  }
  const int units = p.n_tiles * p.m_tiles * p.splits;
  const int grid = std::min(units, num_sms_cached());
  gemm_kernel<BN, EPI><<<grid, kThreads, C::kSmem, s>>>(mw, mx, p);
}

template <int BN>
static void dispatch_epi(int epi, const Params& p, const CUtensorMap& mw, const CUtensorMap& mx, cudaStream_t s) {
  switch (epi) {
    case kBf16: launch<BN, kBf16>(p, mw, mx, s); break;
    case kSilu: launch<BN, kSilu>(p, mw, mx, s); break;
    case kGelu: launch<BN, kGelu>(p, mw, mx, s); break;
    default: launch<BN, kF32>(p, mw, mx, s); break;
  }
}

static int pick_bn(int M) {
  if (M <= 16) return 16;
  if (M <= 32) return 32;
  if (M <= 64) return 64;
  if (M <= 128) return 128;
  return 256;
}

}  // namespace gemm
}  // namespace msgl

using namespace msgl;
using namespace msgl::gemm;

extern "C" int msgl_gemm_pick_splits(int M, int N, int K) {
  const int bn = pick_bn(M);
  const int tiles = ((N + BM - 1) / BM) * ((M + bn - 1) / bn);
  const int kblocks = (K + BK - 1) / BK;
  const int sms = num_sms_cached();
  if (tiles >= sms / 2 || kblocks < 8) return 1;
  int splits = std::min(sms / tiles, kblocks / 4);
  return std::max(1, std::min(splits, 16));
}

extern "C" int msgl_gemm_workspace_bytes(int M, int N, int K, int splits) {
  if (splits <= 1) return 0;
  const int bn = pick_bn(M);
  const int tiles = ((N + BM - 1) / BM) * ((M + bn - 1) / bn);
  return tiles * 4 + 256 + tiles * splits * BM * bn * 4;
}

extern "C" void msgl_gemm(void* out, const void* x, const void* w, const void* bias, int M, int N,
                          int K, int ldo, int epi, int splits, void* workspace, cudaStream_t s) {
  if (M <= 0 || N <= 0) return;
  const int bn = pick_bn(M);
  Params p;
  p.out = out;
  p.bias = reinterpret_cast<const __nv_bfloat16*>(bias);
  p.M = M; p.N = N; p.K = K; p.ldo = ldo;
  p.n_tiles = (N + BM - 1) / BM;
  p.m_tiles = (M + bn - 1) / bn;
  p.kblocks = (K + BK - 1) / BK;
  p.splits = std::max(1, std::min(splits, p.kblocks));
  const int tiles = p.n_tiles * p.m_tiles;
  if (p.splits > 1) {
    p.counters = reinterpret_cast<int*>(workspace);
    p.partials = reinterpret_cast<float*>(reinterpret_cast<uint8_t*>(workspace) + ((tiles * 4 + 255) & ~255));
  } else {
    p.counters = nullptr;
    p.partials = nullptr;
  }
  const CUtensorMap mw = make_map(w, N, K, K, BM);
  const CUtensorMap mx = make_map(x, M, K, K, bn);
  switch (bn) {
    case 16: dispatch_epi<16>(epi, p, mw, mx, s); break;
    case 32: dispatch_epi<32>(epi, p, mw, mx, s); break;
    case 64: dispatch_epi<64>(epi, p, mw, mx, s); break;
    case 128: dispatch_epi<128>(epi, p, mw, mx, s); break;
    default: dispatch_epi<256>(epi, p, mw, mx, s); break;
  }
}

MSGL_ERROR_ACCESSOR(msgl_err_gemm)

extern "C" int msgl_num_sms() { return num_sms_cached(); }
