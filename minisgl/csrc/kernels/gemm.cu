// Persistent, warp-specialized bf16 GEMM on the 5th-generation tensor core (tcgen05 + TMEM + TMA).
//
//   out[M, n] = epilogue( x[M, K] @ w[N, K]^T + bias )
//
// Orientation ("swap-AB"): weight rows are the MMA's M dimension (128 per instruction) and the
// tokens are its N dimension (BN = 16..256), so a decode batch of any size is one MMA column
// tile and every weight byte is streamed from HBM once per call.
//
// Warp roles (320 threads, one CTA per SM, persistent over work units):
//   warp 0      TMA producer (one lane): a kStages-deep ring of {weight tile, activation tile}.
//   warp 1      TMEM allocator + MMA issuer (one lane); fp32 accumulators live in TMEM, double
//               buffered so the epilogue of one tile overlaps the main loop of the next.
//   warps 2..9  epilogue: warp w reads TMEM lane quadrant (w % 4) (a hardware rule) and every
//               other 32-token chunk; values go through a per-warp smem tile to a TMA store.
//
// Gated activations (gate_up projection with SiLU/GELU): the weight is stored with gate and up
// rows interleaved in blocks of 128, so one 256-row weight tile holds 128 gate rows and their 128
// up rows. Two MMAs per k-step write two TMEM accumulators; each epilogue thread then owns the
// gate and up value of the same output element - no cross-warp exchange.
//
// Split-K (decode shapes with few weight tiles): the splits of one tile are launched as one
// thread-block cluster (co-scheduled by hardware). The fp32 tile is divided into items with one
// owner split each; every CTA stages the items it does not own in its drained operand ring and,
// after one cluster barrier, pushes them with bulk shared::cluster copies into the owners'
// receive slots. Owners add them to their TMEM accumulator and run the epilogue. No global
// atomics, no workspace.
#include <algorithm>
#include <atomic>
#include <cstdio>
#include <cstring>
#include <mutex>

#include "api.h"
#include "common.cuh"

namespace msgl {
namespace gemm {

constexpr int BK = 64;
constexpr int kEpiWarps = 8;
constexpr int kThreads = 64 + kEpiWarps * 32;

// kSwiglu: gpt-oss's clamped SwiGLU, min(g, 7) * sigmoid(1.702 min(g, 7)) * (clamp(u, -7, 7) + 1)
// kArgmax: no output tile; per (32 weight rows, token) the largest value and its row (the LM head's
// greedy pick, see argmax_item)
enum Epi : int { kBf16 = 0, kSilu = 1, kGelu = 2, kF32 = 3, kSwiglu = 4, kArgmax = 5 };

constexpr int pow2ceil(int x) {
  int p = 32;
  while (p < x) p <<= 1;
  return p;
}

template <int BN, int EPI, bool WIDE>
struct Cfg {
  static constexpr bool kAct = EPI == kSilu || EPI == kGelu || EPI == kSwiglu;
  static constexpr bool kTwo = kAct || WIDE;           // two 128-row MMA halves per tile
  static constexpr int kRowsA = kTwo ? 256 : 128;
  static constexpr int kOutPerTile = kAct ? 128 : kRowsA;
  static constexpr int kAccCols = (kTwo ? 2 : 1) * BN;
  static constexpr int kBufs = 2 * kAccCols <= 512 ? 2 : 1;  // TMEM double buffering if it fits
  static constexpr int kTmemCols = pow2ceil(kBufs * kAccCols);
  static constexpr int kA = kRowsA * BK * 2;
  static constexpr int kB = BN * BK * 2;
  static constexpr int kStage = kA + kB;
  static constexpr int kOutElem = (EPI == kF32 || EPI == kArgmax) ? 4 : 2;
  static constexpr int kChunk = BN >= 32 ? 32 : 16;
  static constexpr int kStageOut = kChunk * 32 * kOutElem;
  static constexpr int kEpiSmem = kEpiWarps * kStageOut;
  static constexpr int kStages = std::min(8, (220 * 1024 - kEpiSmem) / kStage);
  static constexpr int kSmem = 1024 + kStages * kStage + kEpiSmem + 256;
  // Split-K exchange: the fp32 tile is cut into items of 32 accumulator rows x kChunk tokens
  // (plus the matching up rows when gated); each item has one owner split.
  static constexpr int kItemParts = (kTwo && !kAct) ? 2 : 1;
  static constexpr int kItems = kItemParts * 4 * (BN / kChunk);
  static constexpr int kBlkBytes = 32 * kChunk * 4 * (kAct ? 2 : 1);
  // operand-ring bytes the exchange needs with S splits: this CTA's non-owned items (sent) plus
  // (S - 1) received copies of each owned item
  static constexpr int xchg_bytes(int S) {
    return (kItems - kItems / S + (S - 1) * ((kItems + S - 1) / S)) * kBlkBytes;
  }
  static constexpr bool kCanSplit = xchg_bytes(2) <= kStages * kStage;
  static_assert(kTmemCols <= 512, "accumulators exceed TMEM");
};

struct Params {
  const __nv_bfloat16* bias;
  int w_blocked;  // weight stored [K/64][N][64] (3-D map) instead of [N][K]
  // grouped (MoE) mode: weights [E][N][K] (3-D map), token tiles from a device work list
  const int* grp_count;   // number of valid token tiles (written by the routing kernels)
  const int2* grp_work;   // per token tile: {expert, first row in the permuted activations}
  int64_t bias_stride;    // per-expert bias stride (grouped)
  int M, n_out, kblocks;
  int n_tiles, m_tiles, splits;  // splits > 1: grid (splits, tiles), cluster (splits, 1, 1)
  // fused collective: when set, the output is this rank's staging region of the NVLS buffer and
  // the launch's last CTA to finish adds 1 to the multicast arrival counter (see comm.cu)
  uint32_t* arrive_ticket;
  void* arrive_mc;
  float2* argmax_out;  // kArgmax: [ceil(n_out / 32)][M] of {max, row as int bits}
};

// End of a GEMM CTA whose output feeds the NVLS reduce-scatter: every epilogue thread that issued
// TMA stores has waited for them (bulk_wait) and fenced the async proxy; after the CTA barrier that
// precedes this call, one thread takes the CTA's arrival ticket.
__device__ __forceinline__ void gemm_arrive(uint32_t* ticket, void* mc) {
  if (mc != nullptr && threadIdx.x == 0) rank_arrive(ticket, gridDim.x * gridDim.y * gridDim.z, mc);
}

__device__ __forceinline__ float act_silu(float g) { return g / (1.f + __expf(-g)); }
__device__ __forceinline__ float act_gelu(float g) {
  return 0.5f * g * (1.f + tanhf(0.7978845608028654f * (g + 0.044715f * g * g * g)));
}
template <int EPI>
__device__ __forceinline__ float gated_act(float g, float up) {
  if constexpr (EPI == kSwiglu) {
    g = fminf(g, 7.f);
    up = fminf(fmaxf(up, -7.f), 7.f);
    return g / (1.f + __expf(-1.702f * g)) * (up + 1.f);
  } else {
    return (EPI == kSilu ? act_silu(g) : act_gelu(g)) * up;
  }
}

// tile -> (weight tile, token tile): groups of 8 weight tiles sweep all token tiles so one wave's
// weight tiles stay in L2 while activations stream.
__device__ __forceinline__ void tile_coords(int tile, int n_tiles, int m_tiles, int& nt, int& mt) {
  constexpr int G = 8;
  const int g = tile / (G * m_tiles);
  const int r = tile - g * G * m_tiles;
  const int gs = min(G, n_tiles - g * G);
  nt = g * G + r % gs;
  mt = r / gs;
}

__device__ __forceinline__ void split_range(int split, int splits, int kblocks, int& kb0, int& kb1) {
  kb0 = (int)((long long)split * kblocks / splits);
  kb1 = (int)((long long)(split + 1) * kblocks / splits);
}

// Work unit -> (weight tile, first token row, expert); false if the unit has no work (grouped
// mode with fewer token tiles than the launch's capacity).
__device__ __forceinline__ bool unit_coords(const Params& p, int tile, int bn, int& nt, int& row0, int& expert) {
  if (p.grp_work != nullptr) {
    const int mt = tile / p.n_tiles;
    nt = tile - mt * p.n_tiles;
    if (mt >= *p.grp_count) return false;
    const int2 w = p.grp_work[mt];
    expert = w.x;
    row0 = w.y;
    return true;
  }
  int mt;
  tile_coords(tile, p.n_tiles, p.m_tiles, nt, mt);
  row0 = mt * bn;
  expert = 0;
  return true;
}

template <int W>
__device__ __forceinline__ void tmem_load_cols(uint32_t taddr, float (&v)[32]) {
  if constexpr (W == 32) {
    uint32_t r[32];
    tmem_ld_32x32b_x32(taddr, r);
    tc_wait_ld();
#pragma unroll
    for (int j = 0; j < 32; ++j) v[j] = __uint_as_float(r[j]);
  } else {
    uint32_t r[16];
    tmem_ld_32x32b_x16(taddr, r);
    tc_wait_ld();
#pragma unroll
    for (int j = 0; j < 16; ++j) v[j] = __uint_as_float(r[j]);
  }
}

// Split-K exchange blocks: 32 rows x W fp32, row = lane, 16-byte groups XOR-swizzled by row so a
// warp's vector accesses spread over all banks.
template <int W>
__device__ __forceinline__ void xchg_put(float* blk, int lane, const float (&v)[32]) {
  constexpr int G = W / 4;
#pragma unroll
  for (int j = 0; j < G; ++j)
    reinterpret_cast<float4*>(blk)[lane * G + (j ^ (lane & (G - 1)))] =
        make_float4(v[4 * j], v[4 * j + 1], v[4 * j + 2], v[4 * j + 3]);
}
template <int W>
__device__ __forceinline__ void xchg_add(const float* blk, int lane, float (&v)[32]) {
  constexpr int G = W / 4;
#pragma unroll
  for (int j = 0; j < G; ++j) {
    const float4 t = reinterpret_cast<const float4*>(blk)[lane * G + (j ^ (lane & (G - 1)))];
    v[4 * j] += t.x; v[4 * j + 1] += t.y; v[4 * j + 2] += t.z; v[4 * j + 3] += t.w;
  }
}

// kArgmax epilogue of one item: lane l holds o[j] = row (ocol0 + l) for tokens token0 + j, j < W.
// The 32 x W values go through the warp's staging smem transposed (XOR swizzle: both the row-wise
// writes and the token-wise reads touch 32 different banks); lane t then scans token t's 32 rows
// in order (strict > keeps the lowest row among equal values) and writes {max, row} to block
// ocol0 / 32 of argmax_out. Rows >= n_out do not take part.
template <int W>
__device__ __forceinline__ void argmax_item(const float (&o)[32], int ocol0, int n_out, int M, int token0, int lane,
                                            uint8_t* stage_out, float2* argmax_out) {
  float* s = reinterpret_cast<float*>(stage_out);
  __syncwarp();
  const bool row_ok = ocol0 + lane < n_out;
#pragma unroll
  for (int j = 0; j < W; ++j) s[j * 32 + (lane ^ j)] = row_ok ? o[j] : -INFINITY;
  __syncwarp();
  if (lane < W && token0 + lane < M) {
    float best = -INFINITY;
    int bi = 0;
#pragma unroll
    for (int c = 0; c < 32; ++c) {
      const float x = s[lane * 32 + (c ^ lane)];
      if (x > best) { best = x; bi = c; }
    }
    argmax_out[(int64_t)(ocol0 >> 5) * M + token0 + lane] = make_float2(best, __int_as_float(ocol0 + bi));
  }
  __syncwarp();
}

// bias + activation for one (part, 32-token chunk) item of a warp's 32 accumulator rows, staged
// in smem as [W tokens][32 cols] and written with a TMA store (rows >= M / cols >= n_out clipped)
template <int BN, int EPI, bool WIDE>
__device__ __forceinline__ void store_item(const float (&v)[32], const float (&g2)[32], const Params& p,
                                           const __nv_bfloat16* bias, int nt, int row0, int part, int c, int q,
                                           int lane, uint8_t* stage_out, const CUtensorMap* tmap_out) {
  using C = Cfg<BN, EPI, WIDE>;
  constexpr int W = C::kChunk;
  const int nrow = q * 32 + lane;
  const int wrow_idx = nt * C::kRowsA + part * 128 + nrow;
  const int ocol0 = nt * C::kOutPerTile + part * 128 + q * 32;
  float bias_a = 0.f, bias_b = 0.f;
  if (bias != nullptr && ocol0 + lane < p.n_out) {
    bias_a = __bfloat162float(bias[wrow_idx]);
    if constexpr (C::kAct) bias_b = __bfloat162float(bias[wrow_idx + 128]);
  }
  float o[32];
#pragma unroll
  for (int j = 0; j < W; ++j) {
    if constexpr (C::kAct) {
      const float g = v[j] + bias_a, up = g2[j] + bias_b;
      o[j] = gated_act<EPI>(g, up);
    } else {
      o[j] = v[j] + bias_a;
    }
  }
  if constexpr (EPI == kArgmax) {
    argmax_item<W>(o, ocol0, p.n_out, p.M, row0 + c * W, lane, stage_out, p.argmax_out);
    return;
  }
  if (lane == 0) bulk_wait_read<0>();
  __syncwarp();
  if constexpr (EPI == kF32) {
    float* s = reinterpret_cast<float*>(stage_out);
#pragma unroll
    for (int j = 0; j < W; ++j) s[j * 32 + lane] = o[j];
  } else {
    __nv_bfloat16* s = reinterpret_cast<__nv_bfloat16*>(stage_out);
#pragma unroll
    for (int j = 0; j < W; ++j) s[j * 32 + lane] = __float2bfloat16(o[j]);
  }
  fence_async_smem();
  __syncwarp();
  if (lane == 0) {
    tma_store_2d(tmap_out, stage_out, ocol0, row0 + c * W);
    bulk_commit();
  }
}

template <int BN, int EPI, bool WIDE>
__global__ void __launch_bounds__(kThreads, 1)
gemm_kernel(const __grid_constant__ CUtensorMap tmap_w, const __grid_constant__ CUtensorMap tmap_x,
            const __grid_constant__ CUtensorMap tmap_out, Params p) {
  using C = Cfg<BN, EPI, WIDE>;
  constexpr int W = C::kChunk;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* stages = smem;
  uint8_t* epi_smem = smem + C::kStages * C::kStage;
  uint64_t* bars = reinterpret_cast<uint64_t*>(epi_smem + C::kEpiSmem);
  uint64_t* full = bars;
  uint64_t* empty = bars + C::kStages;
  uint64_t* tfull = bars + 2 * C::kStages;
  uint64_t* tempty = tfull + 2;  // indexed by accumulator buffer (kBufs of them)
  uint64_t* xbar = tempty + 2;   // split-K: bytes of peers' partials received
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(xbar + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const bool split = p.splits > 1;
  // persistent over units, or exactly one unit per CTA when split (cluster rank = split index)
  const int units = p.n_tiles * p.m_tiles * p.splits;
  const int u_first = split ? blockIdx.y * p.splits + blockIdx.x : blockIdx.x;
  const int u_step = split ? units : gridDim.x;

  if (threadIdx.x == 0) {
    for (int i = 0; i < C::kStages; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&tfull[i], 1);
      mbar_init(&tempty[i], kEpiWarps);
    }
    mbar_init(xbar, 1);
    fence_barrier_init();
    if (split) {
      const int r = (int)cluster_ctarank();
      const int owned = r < C::kItems ? (C::kItems - 1 - r) / p.splits + 1 : 0;
      mbar_expect_tx(xbar, (uint32_t)(owned * (p.splits - 1) * C::kBlkBytes));
    }
    prefetch_tmap(&tmap_w);
    prefetch_tmap(&tmap_x);
    prefetch_tmap(&tmap_out);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, C::kTmemCols);
    tmem_relinquish();
  }
  pdl_launch();
  if (p.grp_work != nullptr) pdl_wait();  // every role reads the device work list
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 0) {
    // ------------------------------------------------------------------ TMA producer
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true, waited = false;
      const bool grouped = p.grp_work != nullptr;
      if (grouped) waited = true;
      for (int u = u_first; u < units && ok; u += u_step) {
        const int tile = u / p.splits;
        int nt, row0, expert, kb0, kb1;
        if (!unit_coords(p, tile, BN, nt, row0, expert)) continue;
        split_range(u % p.splits, p.splits, p.kblocks, kb0, kb1);
        int kb = kb0;
        if (!waited) {
          // Weights are static: fetch the first stages' weight tiles before waiting for the
          // previous kernel (programmatic dependent launch), then the activations.
          const int npre = min(C::kStages, kb1 - kb0);
          for (int i = 0; i < npre; ++i) {
            mbar_expect_tx(&full[i], C::kStage);
            uint8_t* a = stages + i * C::kStage;
            if (p.w_blocked) tma_load_3d(a, &tmap_w, &full[i], 0, nt * C::kRowsA, kb0 + i);
            else tma_load_2d(a, &tmap_w, &full[i], (kb0 + i) * BK, nt * C::kRowsA);
          }
          pdl_wait();
          waited = true;
          for (int i = 0; i < npre; ++i)
            tma_load_2d(stages + i * C::kStage + C::kA, &tmap_x, &full[i], (kb0 + i) * BK, row0);
          stage = npre % C::kStages;
          phase = npre == C::kStages ? 1u : 0u;
          kb = kb0 + npre;
        }
        for (; kb < kb1; ++kb) {
          if (!mbar_wait(&empty[stage], phase ^ 1, 100)) { ok = false; break; }
          uint8_t* a = stages + stage * C::kStage;
          mbar_expect_tx(&full[stage], C::kStage);
          if (grouped) tma_load_3d(a, &tmap_w, &full[stage], kb * BK, nt * C::kRowsA, expert);
          else if (p.w_blocked) tma_load_3d(a, &tmap_w, &full[stage], 0, nt * C::kRowsA, kb);
          else tma_load_2d(a, &tmap_w, &full[stage], kb * BK, nt * C::kRowsA);
          tma_load_2d(a + C::kA, &tmap_x, &full[stage], kb * BK, row0);
          if (++stage == C::kStages) { stage = 0; phase ^= 1; }
        }
      }
      if (!waited) pdl_wait();
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      constexpr uint32_t idesc = idesc_bf16_f32(128, BN);
      int stage = 0, use = 0;
      uint32_t phase = 0;
      bool ok = true;
      for (int u = u_first; u < units && ok; u += u_step) {
        int kb0, kb1, nt_, row0_, ex_;
        if (!unit_coords(p, u / p.splits, BN, nt_, row0_, ex_)) continue;
        split_range(u % p.splits, p.splits, p.kblocks, kb0, kb1);
        const int acc = C::kBufs == 2 ? (use & 1) : 0;
        const uint32_t par = C::kBufs == 2 ? ((use >> 1) & 1) : (use & 1);
        if (!mbar_wait(&tempty[acc], par ^ 1, 200)) break;
        tc_fence_after();
        const uint32_t d = tmem_base + acc * C::kAccCols;
        for (int kb = kb0; kb < kb1; ++kb) {
          if (!mbar_wait(&full[stage], phase, 201)) { ok = false; break; }
          tc_fence_after();
          const uint32_t a = smem_u32(stages + stage * C::kStage);
          const uint32_t b = a + C::kA;
#pragma unroll
          for (int k = 0; k < BK / 16; ++k) {
            const uint32_t accum = (kb > kb0 || k > 0) ? 1u : 0u;
            const uint64_t bd = smem_desc_sw128(b + k * 32);
            tc_mma_f16(d, smem_desc_sw128(a + k * 32), bd, idesc, accum);
            if constexpr (C::kTwo) tc_mma_f16(d + BN, smem_desc_sw128(a + 128 * 128 + k * 32), bd, idesc, accum);
          }
          tc_commit(&empty[stage]);
          if (++stage == C::kStages) { stage = 0; phase ^= 1; }
        }
        tc_commit(&tfull[acc]);
        ++use;
      }
    }
  } else {
    // ------------------------------------------------------------------ epilogue
    const int q = warp & 3;              // TMEM lane quadrant this warp may access
    const int half = (warp - 2) >> 2;    // which half of the work items it takes
    uint8_t* stage_out = epi_smem + (warp - 2) * C::kStageOut;
    constexpr int kChunks = BN / W;
    // work items: (part, chunk); a gated tile consumes both parts in one item
    constexpr int kParts = (C::kTwo && !C::kAct) ? 2 : 1;
    constexpr int kItems = kParts * kChunks;
    int use = 0;
    for (int u = u_first; u < units; u += u_step) {
      const int tile = u / p.splits;
      int nt, row0, expert;
      if (!unit_coords(p, tile, BN, nt, row0, expert)) continue;
      const __nv_bfloat16* bias = p.bias == nullptr ? nullptr : p.bias + (int64_t)expert * p.bias_stride;
      const int use_now = use++;
      const int acc = C::kBufs == 2 ? (use_now & 1) : 0;
      const uint32_t par = C::kBufs == 2 ? ((use_now >> 1) & 1) : (use_now & 1);
      if (!mbar_wait(&tfull[acc], par, 300)) break;
      tc_fence_after();
      const uint32_t tb = tmem_base + acc * C::kAccCols + ((uint32_t)(q * 32) << 16);
      const int nrow = q * 32 + lane;  // accumulator row inside a 128-row half
      if (split) {
        if constexpr (C::kCanSplit) {
          // stage the items other splits own, from TMEM into the drained operand ring
          const int S = p.splits, rank = (int)cluster_ctarank();
          constexpr int J = C::kItemParts * kChunks;
          for (int j = half; j < J; j += 2) {
            const int it = q * J + j;
            if (it % S == rank) continue;
            const int part = j / kChunks, c = j % kChunks;
            const int a_idx = it - (it > rank ? (it - rank - 1) / S + 1 : 0);
            float* blk = reinterpret_cast<float*>(stages + (size_t)a_idx * C::kBlkBytes);
            float v[32];
            tmem_load_cols<W>(tb + part * BN + c * W, v);
            xchg_put<W>(blk, lane, v);
            if constexpr (C::kAct) {
              tmem_load_cols<W>(tb + BN + c * W, v);
              xchg_put<W>(blk + 32 * W, lane, v);
            }
          }
          fence_async_smem();
        }
        break;  // the reduction + epilogue run after the cluster barrier below
      }
      for (int it = half; it < kItems; it += 2) {
        const int part = it / kChunks, c = it % kChunks;
        float v[32], g2[32];
        tmem_load_cols<W>(tb + part * BN + c * W, v);
        if constexpr (C::kAct) tmem_load_cols<W>(tb + BN + c * W, g2);
        store_item<BN, EPI, WIDE>(v, g2, p, bias, nt, row0, part, c, q, lane, stage_out, &tmap_out);
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&tempty[acc]);
    }
  }

  if (split) {
    if constexpr (C::kCanSplit) {
      // ---------------------------------------------------------------- cluster split-K exchange
      // Item it (32 accumulator rows of one quadrant x one token chunk) is owned by split
      // it % S. Every CTA has staged the items it does not own; after one cluster barrier (all
      // main loops done, so every receive area in the operand ring is free) each stager pushes
      // them with bulk shared::cluster copies into the owner's receive slots, completing on the
      // owner's mbarrier. Owners add the received partials to their own TMEM accumulator and run
      // the epilogue. Bulk copies move the data as a few large DMA transfers; per-lane DSMEM
      // loads of the same bytes cost several times longer.
      const int S = p.splits, rank = (int)cluster_ctarank();
      constexpr int kChunks = BN / W;
      constexpr int J = C::kItemParts * kChunks;
      const int b_off = (C::kItems - C::kItems / S) * C::kBlkBytes;  // receive slots start
      tc_fence_before();
      cluster_sync();
      tc_fence_after();
      if (warp >= 2) {
        const int q = warp & 3, half = (warp - 2) >> 2;
        if (lane == 0) {
          for (int j = half; j < J; j += 2) {
            const int it = q * J + j, o = it % S;
            if (o == rank) continue;
            const int a_idx = it - (it > rank ? (it - rank - 1) / S + 1 : 0);
            const int slot = (it / S) * (S - 1) + (rank - o - 1 + S) % S;
            const uint32_t dst = dsmem_addr(smem_u32(stages + b_off + (size_t)slot * C::kBlkBytes), o);
            bulk_push_dsmem(dst, stages + (size_t)a_idx * C::kBlkBytes, C::kBlkBytes, dsmem_addr(smem_u32(xbar), o));
          }
        }
        const int tile = blockIdx.y;
        int nt, mt;
        tile_coords(tile, p.n_tiles, p.m_tiles, nt, mt);
        const int row0 = mt * BN;
        uint8_t* stage_out = epi_smem + (warp - 2) * C::kStageOut;
        const uint32_t tb = tmem_base + ((uint32_t)(q * 32) << 16);
        bool have = false, ok = true;
        for (int j = half; j < J && ok; j += 2) {
          const int it = q * J + j;
          if (it % S != rank) continue;
          if (!have) {
            ok = mbar_wait(xbar, 0, 320);
            have = true;
            if (!ok) break;
          }
          const int part = j / kChunks, c = j % kChunks;
          float v[32], g2[32];
          tmem_load_cols<W>(tb + part * BN + c * W, v);
          if constexpr (C::kAct) tmem_load_cols<W>(tb + BN + c * W, g2);
          for (int src = 0; src < S - 1; ++src) {
            const float* blk =
                reinterpret_cast<const float*>(stages + b_off + (size_t)((it / S) * (S - 1) + src) * C::kBlkBytes);
            xchg_add<W>(blk, lane, v);
            if constexpr (C::kAct) xchg_add<W>(blk + 32 * W, lane, g2);
          }
          store_item<BN, EPI, WIDE>(v, g2, p, p.bias, nt, row0, part, c, q, lane, stage_out, &tmap_out);
        }
      }
      if (warp >= 2 && lane == 0) bulk_wait<0>();
      tc_fence_before();
      cluster_sync();  // every push into and out of this CTA's smem has landed
    }
  }
  if (warp >= 2 && lane == 0) {
    // Exiting only needs the staging smem read out (the writes complete before the grid does);
    // a GEMM that signals other ranks waits for its writes to land first.
    if (p.arrive_mc != nullptr) {
      bulk_wait<0>();
      fence_proxy_async_global();
    } else {
      bulk_wait_read<0>();
    }
  }

  tc_fence_before();
  __syncthreads();
  gemm_arrive(p.arrive_ticket, p.arrive_mc);
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, C::kTmemCols);
  }
}


// =================================================================================================
// MXFP4 weights (grouped / MoE mode): experts stay in HBM as e2m1 values (two per byte, low nibble
// first) with one e8m0 scale per 32 values along K, in a k-block-major layout
//   q [E][K/64][Np][32] bytes, s [E][K/64][Np][2] bytes   (Np = rows padded to whole weight tiles)
// so one (expert, 64-K block, weight tile) is a single contiguous bulk copy of each. Converter
// warps (8, or 4 for 128-token tiles whose epilogue needs the registers) turn every landed fp4
// tile into the bf16 operand tile (128B-swizzled, the layout the TMA writes for bf16 weights) and
// the rest of the pipeline is the bf16 kernel's: the MMA warp waits for the converted tile,
// epilogue warps 2..9 as in gemm_kernel. Conversion in registers (fp4_to_bf16x8): byte-permute
// lookups into 8-entry tables of the bf16 high and low bytes of |e2m1| at scale 1, the sign bits
// spread by the permute's sign-replicate mode, then one bf16x2 multiply by the block scale (a
// power of two, so the product is exact: the same bf16 values as dequantising at load).
// =================================================================================================
template <int BN>
constexpr int conv_warps() { return BN <= 64 ? 8 : 4; }
template <int BN>
constexpr int threads_f4() { return kThreads + conv_warps<BN>() * 32; }

// Eight e2m1 values (x: byte k = codes 2k (low nibble) and 2k + 1) -> four bf16x2 words at scale 1
__device__ __forceinline__ void fp4_to_bf16x8(uint32_t x, uint32_t (&o)[4]) {
  // bf16 of |e2m1| 0, 0.5, 1, 1.5, 2, 3, 4, 6: low bytes 00 00 80 C0 00 40 80 C0, high 00 3F 3F 3F 40 40 40 40
  constexpr uint32_t kLbLo = 0xC0800000u, kLbHi = 0xC0804000u, kHbLo = 0x3F3F3F00u, kHbHi = 0x40404040u;
  const uint32_t x4 = x << 4;  // each low nibble's sign bit becomes its byte's top bit
#pragma unroll
  for (int h = 0; h < 2; ++h) {  // values 4h .. 4h + 3 (bytes 2h, 2h + 1 of x)
    const uint32_t sel = (h == 0 ? x : __byte_perm(x, 0, 0x4432)) & 0x7777u;  // magnitude codes
    const uint32_t lo = __byte_perm(kLbLo, kLbHi, sel), hi = __byte_perm(kHbLo, kHbHi, sel);
    // signs: byte 1 <- top bit of byte (2h + j) of x4 (low nibble), byte 3 <- of x (high nibble)
    const uint32_t s0 = __byte_perm(x4, x, h == 0 ? 0xC080u : 0xE0A0u);
    const uint32_t s1 = __byte_perm(x4, x, h == 0 ? 0xD090u : 0xF0B0u);
    o[2 * h] = __byte_perm(lo, hi, 0x5140u) | (s0 & 0x80008000u);
    o[2 * h + 1] = __byte_perm(lo, hi, 0x7362u) | (s1 & 0x80008000u);
  }
}

template <int BN, int EPI, bool WIDE>
struct CfgF4 {
  using C = Cfg<BN, EPI, WIDE>;
  static constexpr int kQ = C::kRowsA * 32;                   // fp4 bytes of one k-block of a tile
  static constexpr int kS = C::kRowsA * 2;                    // its scale bytes
  static constexpr int kRaw = (kQ + kS + 1023) / 1024 * 1024;
  static constexpr int kStage = C::kA + C::kB + kRaw;         // {bf16 weight tile, activations, raw}
  static constexpr int kStages = std::min(8, (220 * 1024 - C::kEpiSmem) / kStage);
  static constexpr int kSmem = 1024 + kStages * kStage + C::kEpiSmem + 256;
  static_assert(kStages >= 2, "fp4 GEMM stages do not fit");
};

// bf16 of 2^(e - 127) for an e8m0 scale byte, in both halves
__device__ __forceinline__ uint32_t e8m0_bf16x2(uint32_t e) {
  const uint32_t b = e == 0 ? 0x0040u : (e << 7);  // 2^-127 is a bf16 subnormal
  return b | (b << 16);
}

// Pipeline: one ring of stages {bf16 weight tile, activation tile, raw fp4 + scales}; the producer
// lane loads the raw weights and the activations, converter threads write the bf16 tile from the
// raw bytes of the same stage, the MMA lane waits for the converted tile and releases the stage.
// A ring split into a deep raw ring and a short operand ring (converters loading the activations)
// measured slower: the activations' load latency then sits between conversion and MMA.
template <int BN, int EPI, bool WIDE>
__global__ void __launch_bounds__(threads_f4<BN>(), 1)
gemm_fp4_kernel(const __grid_constant__ CUtensorMap tmap_x, const __grid_constant__ CUtensorMap tmap_out,
                const uint8_t* __restrict__ wq, const uint8_t* __restrict__ wsc, int n_pad, Params p) {
  using C = Cfg<BN, EPI, WIDE>;
  using F = CfgF4<BN, EPI, WIDE>;
  constexpr int W = C::kChunk;
  constexpr int kConv = conv_warps<BN>();
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* stages = smem;
  uint8_t* epi_smem = smem + F::kStages * F::kStage;
  uint64_t* bars = reinterpret_cast<uint64_t*>(epi_smem + C::kEpiSmem);
  uint64_t* full = bars;                  // raw fp4 + scales + activations landed
  uint64_t* conv = bars + F::kStages;     // bf16 weight tile written (converter threads)
  uint64_t* empty = bars + 2 * F::kStages;
  uint64_t* tfull = bars + 3 * F::kStages;
  uint64_t* tempty = tfull + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(tempty + 2);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int units = p.n_tiles * p.m_tiles;

  if (threadIdx.x == 0) {
    for (int i = 0; i < F::kStages; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&conv[i], kConv * 32);
      mbar_init(&empty[i], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&tfull[i], 1);
      mbar_init(&tempty[i], kEpiWarps);
    }
    fence_barrier_init();
    prefetch_tmap(&tmap_x);
    prefetch_tmap(&tmap_out);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, C::kTmemCols);
    tmem_relinquish();
  }
  pdl_launch();
  pdl_wait();  // every role reads the device work list
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 0) {
    // ------------------------------------------------------------------ producer
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      for (int u = blockIdx.x; u < units && ok; u += gridDim.x) {
        int nt, row0, expert;
        if (!unit_coords(p, u, BN, nt, row0, expert)) continue;
        for (int kb = 0; kb < p.kblocks; ++kb) {
          if (!mbar_wait(&empty[stage], phase ^ 1, 150)) { ok = false; break; }
          uint8_t* st = stages + stage * F::kStage;
          uint8_t* raw = st + C::kA + C::kB;
          mbar_expect_tx(&full[stage], F::kQ + F::kS + C::kB);
          const size_t blk = ((size_t)expert * p.kblocks + kb) * n_pad + (size_t)nt * C::kRowsA;
          bulk_load(raw, wq + blk * 32, F::kQ, &full[stage]);
          bulk_load(raw + F::kQ, wsc + blk * 2, F::kS, &full[stage]);
          tma_load_2d(st + C::kA, &tmap_x, &full[stage], kb * BK, row0);
          if (++stage == F::kStages) { stage = 0; phase ^= 1; }
        }
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      constexpr uint32_t idesc = idesc_bf16_f32(128, BN);
      int stage = 0, use = 0;
      uint32_t phase = 0;
      bool ok = true;
      for (int u = blockIdx.x; u < units && ok; u += gridDim.x) {
        int nt_, row0_, ex_;
        if (!unit_coords(p, u, BN, nt_, row0_, ex_)) continue;
        const int acc = C::kBufs == 2 ? (use & 1) : 0;
        const uint32_t par = C::kBufs == 2 ? ((use >> 1) & 1) : (use & 1);
        if (!mbar_wait(&tempty[acc], par ^ 1, 250)) break;
        tc_fence_after();
        const uint32_t d = tmem_base + acc * C::kAccCols;
        for (int kb = 0; kb < p.kblocks; ++kb) {
          if (!mbar_wait(&conv[stage], phase, 251)) { ok = false; break; }
          tc_fence_after();
          const uint32_t a = smem_u32(stages + stage * F::kStage);
          const uint32_t b = a + C::kA;
#pragma unroll
          for (int k = 0; k < BK / 16; ++k) {
            const uint32_t accum = (kb > 0 || k > 0) ? 1u : 0u;
            const uint64_t bd = smem_desc_sw128(b + k * 32);
            tc_mma_f16(d, smem_desc_sw128(a + k * 32), bd, idesc, accum);
            if constexpr (C::kTwo) tc_mma_f16(d + BN, smem_desc_sw128(a + 128 * 128 + k * 32), bd, idesc, accum);
          }
          tc_commit(&empty[stage]);
          if (++stage == F::kStages) { stage = 0; phase ^= 1; }
        }
        tc_commit(&tfull[acc]);
        ++use;
      }
    }
  } else if (warp >= 2 + kEpiWarps) {
    // ------------------------------------------------------------------ fp4 -> bf16 converters
    // work item = (row, 32-value half): one e8m0 scale, four 16-byte output chunks
    constexpr int kHalves = C::kRowsA * 2;
    const int ct = threadIdx.x - kThreads;
    int stage = 0;
    uint32_t phase = 0;
    bool ok = true;
    for (int u = blockIdx.x; u < units && ok; u += gridDim.x) {
      int nt_, row0_, ex_;
      if (!unit_coords(p, u, BN, nt_, row0_, ex_)) continue;
      for (int kb = 0; kb < p.kblocks; ++kb) {
        if (!mbar_wait(&full[stage], phase, 350)) { ok = false; break; }
        uint8_t* op = stages + stage * F::kStage;
        const uint8_t* raw = op + C::kA + C::kB;
#pragma unroll
        for (int it = ct; it < kHalves; it += kConv * 32) {
          const int r = it >> 1, hv = it & 1;
          const uint4 qv = *reinterpret_cast<const uint4*>(raw + r * 32 + hv * 16);
          const uint32_t sb = e8m0_bf16x2(raw[F::kQ + r * 2 + hv]);
          const __nv_bfloat162 sc = *reinterpret_cast<const __nv_bfloat162*>(&sb);
          const uint32_t words[4] = {qv.x, qv.y, qv.z, qv.w};
          uint8_t* dst = op + (r >> 7) * 128 * 128 + (r & 127) * 128;
#pragma unroll
          for (int c = 0; c < 4; ++c) {  // 16-byte chunk 4 hv + c: values 8 (4 hv + c) .. + 7
            uint32_t o[4];
            fp4_to_bf16x8(words[c], o);
#pragma unroll
            for (int j = 0; j < 4; ++j) {
              __nv_bfloat162 v = *reinterpret_cast<const __nv_bfloat162*>(&o[j]);
              v = __hmul2(v, sc);
              o[j] = *reinterpret_cast<const uint32_t*>(&v);
            }
            *reinterpret_cast<uint4*>(dst + (((4 * hv + c) ^ (r & 7)) << 4)) = make_uint4(o[0], o[1], o[2], o[3]);
          }
        }
        fence_async_smem();  // generic-proxy writes -> the MMA's async-proxy reads
        mbar_arrive(&conv[stage]);
        if (++stage == F::kStages) { stage = 0; phase ^= 1; }
      }
    }
  } else {
    // ------------------------------------------------------------------ epilogue
    const int q = warp & 3;
    const int half = (warp - 2) >> 2;
    uint8_t* stage_out = epi_smem + (warp - 2) * C::kStageOut;
    constexpr int kChunks = BN / W;
    constexpr int kParts = (C::kTwo && !C::kAct) ? 2 : 1;
    constexpr int kItems = kParts * kChunks;
    int use = 0;
    for (int u = blockIdx.x; u < units; u += gridDim.x) {
      int nt, row0, expert;
      if (!unit_coords(p, u, BN, nt, row0, expert)) continue;
      const __nv_bfloat16* bias = p.bias == nullptr ? nullptr : p.bias + (int64_t)expert * p.bias_stride;
      const int use_now = use++;
      const int acc = C::kBufs == 2 ? (use_now & 1) : 0;
      const uint32_t par = C::kBufs == 2 ? ((use_now >> 1) & 1) : (use_now & 1);
      if (!mbar_wait(&tfull[acc], par, 352)) break;
      tc_fence_after();
      const uint32_t tb = tmem_base + acc * C::kAccCols + ((uint32_t)(q * 32) << 16);
      for (int it = half; it < kItems; it += 2) {
        const int part = it / kChunks, c = it % kChunks;
        float v[32], g2[32];
        tmem_load_cols<W>(tb + part * BN + c * W, v);
        if constexpr (C::kAct) tmem_load_cols<W>(tb + BN + c * W, g2);
        store_item<BN, EPI, WIDE>(v, g2, p, bias, nt, row0, part, c, q, lane, stage_out, &tmap_out);
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&tempty[acc]);
    }
    if (lane == 0) bulk_wait_read<0>();
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, C::kTmemCols);
  }
}

// =================================================================================================
// 2-SM variant (tcgen05.mma.cta_group::2): a CTA pair computes one 256-weight-row tile. Each CTA
// loads its own 128 weight rows (256 for gated outputs: 128 gate + 128 up) and HALF of the token
// tile into its own smem; the loads complete on the pair leader's barrier; the leader's single MMA
// thread issues M = 256 MMAs that read both CTAs' smem and write each CTA's TMEM (its 128 rows x
// BN tokens). Per SM this halves the activation traffic of the 1-SM kernel, which is what limits
// decode-sized GEMMs. Commits are multicast to both CTAs' barriers (tcgen05.commit multicast; no
// TMA multicast). Split-K uses clusters of 2 x S CTAs (pair member = rank & 1, split = rank >> 1)
// exchanging fp32 partials through an L2-resident buffer.
// =================================================================================================
template <int BN, int EPI>
struct Cfg2 {
  static constexpr bool kAct = EPI == kSilu || EPI == kGelu || EPI == kSwiglu;
  static constexpr int kRowsA = kAct ? 256 : 128;  // weight rows loaded per CTA
  static constexpr int kTok = BN / 2;               // token rows loaded per CTA
  static constexpr int kAccCols = (kAct ? 2 : 1) * BN;
  static constexpr int kBufs = 2 * kAccCols <= 512 ? 2 : 1;
  static constexpr int kTmemCols = pow2ceil(kBufs * kAccCols);
  static constexpr int kA = kRowsA * BK * 2;
  static constexpr int kB = kTok * BK * 2;
  static constexpr int kStage = kA + kB;
  static constexpr int kOutElem = (EPI == kF32 || EPI == kArgmax) ? 4 : 2;
  static constexpr int kStageOut = 32 * 32 * kOutElem;
  static constexpr int kEpiSmem = kEpiWarps * kStageOut;
  static constexpr int kStages = std::min(8, (220 * 1024 - kEpiSmem) / kStage);
  static constexpr int kSmem = 1024 + kStages * kStage + kEpiSmem + 256;
  static constexpr int kParts = kAct ? 2 : 1;
  // split-K exchange among the CTAs of one pair member: items of 32 accumulator rows x 32 tokens
  // (with the up rows when gated), staged and received in the drained operand ring
  static constexpr int kItems = 4 * (BN / 32);
  static constexpr int kBlkBytes = 32 * 32 * 4 * kParts;
  static constexpr int xchg_bytes(int S) {
    return (kItems - kItems / S + (S - 1) * ((kItems + S - 1) / S)) * kBlkBytes;
  }
  static_assert(BN >= 64 && BN <= 256, "2-SM tiles use 64..256 tokens");
  static_assert(kTmemCols <= 512, "accumulators exceed TMEM");
};

struct Params2 {
  const __nv_bfloat16* bias;
  int M, n_out, kblocks;
  int n_tiles, m_tiles, splits;  // n_tiles counts pair tiles (256 weight rows, 512 if gated)
  uint32_t* arrive_ticket;       // as in Params
  void* arrive_mc;
  float2* argmax_out;            // as in Params
};


template <int BN, int EPI>
__device__ __forceinline__ void store_item2(const float (&v)[32], const float (&g2)[32], const Params2& p, int nt,
                                            int row0, int x, int c, int q, int lane, uint8_t* stage_out,
                                            const CUtensorMap* tmap_out) {
  using C = Cfg2<BN, EPI>;
  const int nrow = q * 32 + lane;
  const int ocol0 = nt * 256 + x * 128 + q * 32;
  float bias_a = 0.f, bias_b = 0.f;
  if (p.bias != nullptr && ocol0 + lane < p.n_out) {
    if constexpr (C::kAct) {
      const int grow = nt * 512 + x * 256 + nrow;
      bias_a = __bfloat162float(p.bias[grow]);
      bias_b = __bfloat162float(p.bias[grow + 128]);
    } else {
      bias_a = __bfloat162float(p.bias[ocol0 + lane]);
    }
  }
  float o[32];
#pragma unroll
  for (int j = 0; j < 32; ++j) {
    if constexpr (C::kAct) {
      const float g = v[j] + bias_a, up = g2[j] + bias_b;
      o[j] = gated_act<EPI>(g, up);
    } else {
      o[j] = v[j] + bias_a;
    }
  }
  if constexpr (EPI == kArgmax) {
    argmax_item<32>(o, ocol0, p.n_out, p.M, row0 + c * 32, lane, stage_out, p.argmax_out);
    return;
  }
  if (lane == 0) bulk_wait_read<0>();
  __syncwarp();
  if constexpr (EPI == kF32) {
    float* sp = reinterpret_cast<float*>(stage_out);
#pragma unroll
    for (int j = 0; j < 32; ++j) sp[j * 32 + lane] = o[j];
  } else {
    __nv_bfloat16* sp = reinterpret_cast<__nv_bfloat16*>(stage_out);
#pragma unroll
    for (int j = 0; j < 32; ++j) sp[j * 32 + lane] = __float2bfloat16(o[j]);
  }
  fence_async_smem();
  __syncwarp();
  if (lane == 0) {
    tma_store_2d(tmap_out, stage_out, ocol0, row0 + c * 32);
    bulk_commit();
  }
}

template <int BN, int EPI>
__global__ void __launch_bounds__(kThreads, 1)
gemm2_kernel(const __grid_constant__ CUtensorMap tmap_w, const __grid_constant__ CUtensorMap tmap_x,
             const __grid_constant__ CUtensorMap tmap_out, Params2 p) {
  using C = Cfg2<BN, EPI>;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* stages = smem;
  uint8_t* epi_smem = smem + C::kStages * C::kStage;
  uint64_t* bars = reinterpret_cast<uint64_t*>(epi_smem + C::kEpiSmem);
  uint64_t* full = bars;
  uint64_t* empty = bars + C::kStages;
  uint64_t* tfull = bars + 2 * C::kStages;
  uint64_t* tempty = tfull + 2;
  uint64_t* xbar = tempty + 2;  // split-K: bytes of peers' partials received
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(xbar + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t rank = cluster_ctarank();
  const int x = rank & 1, ysplit = rank >> 1;
  const uint32_t leader = rank & ~1u;
  const uint16_t pair_mask = (uint16_t)(3u << leader);
  const bool split = p.splits > 1;
  const int tiles = p.n_tiles * p.m_tiles;

  if (threadIdx.x == 0) {
    for (int i = 0; i < C::kStages; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&tfull[i], 1);
      mbar_init(&tempty[i], 2 * kEpiWarps);
    }
    mbar_init(xbar, 1);
    if (split) {
      const int owned = ysplit < C::kItems ? (C::kItems - 1 - ysplit) / p.splits + 1 : 0;
      mbar_expect_tx(xbar, (uint32_t)(owned * (p.splits - 1) * C::kBlkBytes));
    }
    fence_barrier_init();
    prefetch_tmap(&tmap_w);
    prefetch_tmap(&tmap_x);
    prefetch_tmap(&tmap_out);
  }
  if (warp == 1) {
    tmem_alloc_2sm(tmem_slot, C::kTmemCols);
    tmem_relinquish_2sm();
  }
  pdl_launch();
  tc_fence_before();
  cluster_sync();  // barriers of both CTAs initialised before any remote use
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 0) {
    // ------------------------------------------------------------------ TMA producer (both CTAs)
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      bool waited = false;
      for (int t = blockIdx.y; t < tiles; t += gridDim.y) {
        int nt, mt, kb0, kb1;
        tile_coords(t, p.n_tiles, p.m_tiles, nt, mt);
        split_range(ysplit, p.splits, p.kblocks, kb0, kb1);
        const int wrow = nt * 2 * C::kRowsA + x * C::kRowsA;
        const int trow = mt * BN + x * C::kTok;
        int kb = kb0;
        if (!waited) {
          // Weights are static: fetch the first stages' weight tiles before waiting for the
          // previous kernel (programmatic dependent launch), then the activations.
          const int npre = min(C::kStages, kb1 - kb0);
          for (int i = 0; i < npre; ++i) {
            if (x == 0) mbar_expect_tx(&full[i], 2 * C::kStage);
            const uint32_t fbar = dsmem_addr(smem_u32(&full[i]), leader);
            tma_load_2d_2sm(stages + i * C::kStage, &tmap_w, fbar, (kb0 + i) * BK, wrow);
          }
          pdl_wait();
          waited = true;
          for (int i = 0; i < npre; ++i) {
            const uint32_t fbar = dsmem_addr(smem_u32(&full[i]), leader);
            tma_load_2d_2sm(stages + i * C::kStage + C::kA, &tmap_x, fbar, (kb0 + i) * BK, trow);
          }
          stage = npre % C::kStages;
          phase = npre == C::kStages ? 1u : 0u;
          kb = kb0 + npre;
        }
        bool ok = true;
        for (; kb < kb1; ++kb) {
          if (!mbar_wait(&empty[stage], phase ^ 1, 110)) { ok = false; break; }
          if (x == 0) mbar_expect_tx(&full[stage], 2 * C::kStage);
          uint8_t* a = stages + stage * C::kStage;
          const uint32_t fbar = dsmem_addr(smem_u32(&full[stage]), leader);
          tma_load_2d_2sm(a, &tmap_w, fbar, kb * BK, wrow);
          tma_load_2d_2sm(a + C::kA, &tmap_x, fbar, kb * BK, trow);
          if (++stage == C::kStages) { stage = 0; phase ^= 1; }
        }
        if (!ok) break;
      }
      if (!waited) pdl_wait();
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------------ MMA issuer (leader only)
    if (lane == 0 && x == 0) {
      constexpr uint32_t idesc = idesc_bf16_f32(256, BN);
      int stage = 0, use = 0;
      uint32_t phase = 0;
      for (int t = blockIdx.y; t < tiles; t += gridDim.y, ++use) {
        int kb0, kb1;
        split_range(ysplit, p.splits, p.kblocks, kb0, kb1);
        const int acc = C::kBufs == 2 ? (use & 1) : 0;
        const uint32_t par = C::kBufs == 2 ? ((use >> 1) & 1) : (use & 1);
        if (!mbar_wait(&tempty[acc], par ^ 1, 210)) break;
        tc_fence_after();
        const uint32_t d = tmem_base + acc * C::kAccCols;
        bool ok = true;
        for (int kb = kb0; kb < kb1; ++kb) {
          if (!mbar_wait(&full[stage], phase, 211)) { ok = false; break; }
          tc_fence_after();
          const uint32_t a = smem_u32(stages + stage * C::kStage);
          const uint32_t b = a + C::kA;
#pragma unroll
          for (int k = 0; k < BK / 16; ++k) {
            const uint32_t accum = (kb > kb0 || k > 0) ? 1u : 0u;
            const uint64_t bd = smem_desc_sw128(b + k * 32);
            tc_mma_f16_2sm(d, smem_desc_sw128(a + k * 32), bd, idesc, accum);
            if constexpr (C::kAct) tc_mma_f16_2sm(d + BN, smem_desc_sw128(a + 128 * 128 + k * 32), bd, idesc, accum);
          }
          tc_commit_2sm_mc(&empty[stage], pair_mask);
          if (++stage == C::kStages) { stage = 0; phase ^= 1; }
        }
        tc_commit_2sm_mc(&tfull[acc], pair_mask);
        if (!ok) break;
      }
    }
  } else {
    // ------------------------------------------------------------------ epilogue (both CTAs)
    const int q = warp & 3;
    const int half = (warp - 2) >> 2;
    uint8_t* stage_out = epi_smem + (warp - 2) * C::kStageOut;
    constexpr int kChunks = BN / 32;
    int use = 0;
    for (int t = blockIdx.y; t < tiles; t += gridDim.y, ++use) {
      int nt, mt;
      tile_coords(t, p.n_tiles, p.m_tiles, nt, mt);
      const int acc = C::kBufs == 2 ? (use & 1) : 0;
      const uint32_t par = C::kBufs == 2 ? ((use >> 1) & 1) : (use & 1);
      if (!mbar_wait(&tfull[acc], par, 310)) break;
      tc_fence_after();
      const uint32_t tb = tmem_base + acc * C::kAccCols + ((uint32_t)(q * 32) << 16);
      if (split) {
        // stage the items other splits own (same pair member), from TMEM into the drained ring
        const int S = p.splits;
        for (int c = half; c < kChunks; c += 2) {
          const int it = q * kChunks + c;
          if (it % S == ysplit) continue;
          const int a_idx = it - (it > ysplit ? (it - ysplit - 1) / S + 1 : 0);
          float* blk = reinterpret_cast<float*>(stages + (size_t)a_idx * C::kBlkBytes);
          float v[32];
          tmem_load_cols<32>(tb + c * 32, v);
          xchg_put<32>(blk, lane, v);
          if constexpr (C::kAct) {
            tmem_load_cols<32>(tb + BN + c * 32, v);
            xchg_put<32>(blk + 32 * 32, lane, v);
          }
        }
        fence_async_smem();
        break;  // pushed and reduced after the cluster barrier below
      }
      for (int c = half; c < kChunks; c += 2) {
        float v[32], g2[32];
        tmem_load_cols<32>(tb + c * 32, v);
        if constexpr (C::kAct) tmem_load_cols<32>(tb + BN + c * 32, g2);
        store_item2<BN, EPI>(v, g2, p, nt, mt * BN, x, c, q, lane, stage_out, &tmap_out);
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive_cluster(dsmem_addr(smem_u32(&tempty[acc]), leader));
    }
  }

  if (split) {
    // 2-SM split-K exchange among the S CTAs holding the same pair member's rows (cluster ranks
    // 2 * split + x). Item it (32 rows of one TMEM quadrant x 32 tokens) is owned by split
    // it % S; stagers push their copies with bulk shared::cluster transfers into the owner's
    // receive slots (completing on its mbarrier) once the cluster barrier shows every ring
    // drained; the owner adds them to its TMEM accumulator and runs the epilogue.
    const int S = p.splits;
    const int b_off = (C::kItems - C::kItems / S) * C::kBlkBytes;
    tc_fence_before();
    cluster_sync();
    tc_fence_after();
    if (warp >= 2) {
      const int q = warp & 3, half = (warp - 2) >> 2;
      constexpr int kChunks = BN / 32;
      if (lane == 0) {
        for (int c = half; c < kChunks; c += 2) {
          const int it = q * kChunks + c, o = it % S;
          if (o == ysplit) continue;
          const int a_idx = it - (it > ysplit ? (it - ysplit - 1) / S + 1 : 0);
          const int slot = (it / S) * (S - 1) + (ysplit - o - 1 + S) % S;
          const uint32_t dst_rank = (uint32_t)(2 * o + x);
          const uint32_t dst = dsmem_addr(smem_u32(stages + b_off + (size_t)slot * C::kBlkBytes), dst_rank);
          bulk_push_dsmem(dst, stages + (size_t)a_idx * C::kBlkBytes, C::kBlkBytes,
                          dsmem_addr(smem_u32(xbar), dst_rank));
        }
      }
      const int tile = blockIdx.y;
      int nt, mt;
      tile_coords(tile, p.n_tiles, p.m_tiles, nt, mt);
      uint8_t* stage_out = epi_smem + (warp - 2) * C::kStageOut;
      const uint32_t tb = tmem_base + ((uint32_t)(q * 32) << 16);
      bool have = false;
      for (int c = half; c < kChunks; c += 2) {
        const int it = q * kChunks + c;
        if (it % S != ysplit) continue;
        if (!have) {
          if (!mbar_wait(xbar, 0, 320)) break;
          have = true;
        }
        float v[32], g2[32];
        tmem_load_cols<32>(tb + c * 32, v);
        if constexpr (C::kAct) tmem_load_cols<32>(tb + BN + c * 32, g2);
        for (int src = 0; src < S - 1; ++src) {
          const float* blk =
              reinterpret_cast<const float*>(stages + b_off + (size_t)((it / S) * (S - 1) + src) * C::kBlkBytes);
          xchg_add<32>(blk, lane, v);
          if constexpr (C::kAct) xchg_add<32>(blk + 32 * 32, lane, g2);
        }
        store_item2<BN, EPI>(v, g2, p, nt, mt * BN, x, c, q, lane, stage_out, &tmap_out);
      }
    }
  }
  if (warp >= 2 && lane == 0) {
    // Exiting only needs the staging smem read out (the writes complete before the grid does);
    // a GEMM that signals other ranks waits for its writes to land first.
    if (p.arrive_mc != nullptr) {
      bulk_wait<0>();
      fence_proxy_async_global();
    } else {
      bulk_wait_read<0>();
    }
  }
  tc_fence_before();
  cluster_sync();  // no CTA leaves while its pair / cluster peers may still address its smem / TMEM
  gemm_arrive(p.arrive_ticket, p.arrive_mc);
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc_2sm(tmem_base, C::kTmemCols);
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

// 2-D row-major [rows, cols] tensor map with the given box; swizzle 128B for operand loads,
// none for epilogue stores.
static CUtensorMap make_map(const void* base, CUtensorMapDataType dt, int elem, int rows, int cols, int ld,
                            int box_cols, int box_rows, bool swizzle) {
  CUtensorMap m;
  memset(&m, 0, sizeof(m));
  EncodeTiledFn fn = encode_fn();
  if (fn == nullptr) {
    fprintf(stderr, "minisgl: cuTensorMapEncodeTiled unavailable\n");
    return m;
  }
  cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)ld * elem};
  cuuint32_t box[2] = {(cuuint32_t)box_cols, (cuuint32_t)box_rows};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = fn(&m, dt, 2, const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                  swizzle ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_NONE,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) fprintf(stderr, "minisgl: cuTensorMapEncodeTiled failed (%d)\n", (int)r);
  return m;
}

// [K/64][N][64] weight: 3-D map (k-in-block, row, k-block), box (64, rows, 1): each weight tile is
// one contiguous run of rows x 128 B in HBM.
static CUtensorMap make_map_blocked(const void* base, int N, int K, int box_rows) {
  CUtensorMap m;
  memset(&m, 0, sizeof(m));
  EncodeTiledFn fn = encode_fn();
  if (fn == nullptr) return m;
  cuuint64_t dims[3] = {(cuuint64_t)BK, (cuuint64_t)N, (cuuint64_t)(K / BK)};
  cuuint64_t strides[2] = {(cuuint64_t)BK * 2, (cuuint64_t)N * BK * 2};
  cuuint32_t box[3] = {(cuuint32_t)BK, (cuuint32_t)box_rows, 1};
  cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = fn(&m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void*>(base), dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) fprintf(stderr, "minisgl: cuTensorMapEncodeTiled (blocked) failed (%d)\n", (int)r);
  return m;
}

// [E][N][K] expert weights: 3-D map (k, row, expert), box (64, rows, 1)
static CUtensorMap make_map_experts(const void* base, int E, int N, int K, int box_rows) {
  CUtensorMap m;
  memset(&m, 0, sizeof(m));
  EncodeTiledFn fn = encode_fn();
  if (fn == nullptr) return m;
  cuuint64_t dims[3] = {(cuuint64_t)K, (cuuint64_t)N, (cuuint64_t)E};
  cuuint64_t strides[2] = {(cuuint64_t)K * 2, (cuuint64_t)N * K * 2};
  cuuint32_t box[3] = {(cuuint32_t)BK, (cuuint32_t)box_rows, 1};
  cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = fn(&m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void*>(base), dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) fprintf(stderr, "minisgl: cuTensorMapEncodeTiled (experts) failed (%d)\n", (int)r);
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

static bool is_act(int epi) { return epi == kSilu || epi == kGelu || epi == kSwiglu; }

struct Plan {
  int bn;
  bool wide;
  int rows_a;  // weight rows per tile
  int tiles;
  int splits;
};

// Tile shape (chosen from graph-replay measurements on B200): plain outputs use 128-row weight
// tiles with BN = round-up(M) <= 256 tokens; gated outputs use 256-row tiles (128 gate + 128 up)
// with BN <= 256 for decode and 128 for prefill. Split-K (a cluster of 2 or 4 CTAs per tile,
// reduced through DSMEM) only pays off for long K with few tiles.
// Plans for the decode GEMMs of tensor-parallel shards (few weight tiles), chosen from a sweep of
// every tiling at Qwen3-14B's TP2/4/8 shapes on B200 (`python -m minisgl.benchmark.kernels
// gemm-sweep`):
//  * gated outputs (gate_up) whose 256-row tiles x 128-token tiles fit in one wave: 128-token tiles
//    on one SM, with split-K while at most half the SMs would be busy (2.2x at TP8, 1.8x at TP4 and
//    1.6x at TP2 with 256 tokens, against one 256-token 2-SM tile per 512 rows);
//  * plain outputs of at most 16M weights with more than 64 tokens: 128-token tiles on one SM and
//    enough K-splits for about one wave (1.2-1.35x for the QKV / o_proj / down_proj shards at
//    TP4/TP8): several token tiles per weight tile keep each CTA's activation traffic near its
//    weight traffic instead of streaming all 256 tokens' activations per weight tile.
static bool small_gated(int M, int N, int epi) {
  const int tiles = (N / 256) * ((M + 127) / 128);
  return is_act(epi) && tiles <= (M <= 128 ? num_sms_cached() / 2 : num_sms_cached());
}
static bool small_plain(int M, int N, int K, int epi) {
  return !is_act(epi) && epi != kArgmax && M > 64 && (int64_t)N * K <= (16ll << 20);
}

// Token-tile override for tiling sweeps and tests (-1: automatic). 1-SM kernel: 16/32/64/128/256;
// 2-SM kernel: 64/128/160/192/224/256. Not for concurrent use.
static std::atomic<int> g_force_bn{-1};

static Plan make_plan(int M, int N, int K, int epi, int force_splits, int force_wide) {
  Plan pl;
  const bool act = is_act(epi);
  if (M <= 256) pl.bn = M <= 16 ? 16 : M <= 32 ? 32 : M <= 64 ? 64 : M <= 128 ? 128 : 256;
  else pl.bn = act ? 128 : 256;
  const bool gated_split = force_wide < 0 && small_gated(M, N, epi);
  const bool plain_split = force_wide < 0 && small_plain(M, N, K, epi);
  if (gated_split || plain_split) pl.bn = std::min(pl.bn, 128);
  if (const int fb = g_force_bn.load(); fb == 16 || fb == 32 || fb == 64 || fb == 128 || fb == 256) pl.bn = fb;
  pl.wide = act || force_wide == 1;
  pl.rows_a = pl.wide ? 256 : 128;
  pl.tiles = ((N + pl.rows_a - 1) / pl.rows_a) * ((M + pl.bn - 1) / pl.bn);
  const int kblocks = (K + BK - 1) / BK;
  const int sms = num_sms_cached();
  // split-K needs the partial ([rows][bn+4] fp32) to fit the operand ring: bn <= 128 if wide
  const bool can_split = !(pl.rows_a == 256 && pl.bn > 128);
  int splits = 1;
  if (force_splits > 0) splits = force_splits;
  else if (gated_split && kblocks >= 16 && pl.tiles <= sms / 2) {
    splits = std::max(1, std::min(std::min(sms / pl.tiles, kblocks / 8), 4));
  } else if (plain_split) {
    // short K (the TP8 o_proj shard: 10 k-blocks) with up to 128 tokens gains nothing from splits
    if (kblocks >= 16 || M > 128) splits = std::max(1, std::min(std::min((sms + pl.tiles - 1) / pl.tiles, kblocks / 2), 8));
  } else if (!act && M <= 128 && pl.tiles <= sms / 2 && kblocks >= 16) {
    // weight-streaming regime: use as many K-splits as keep every SM busy in one wave
    splits = std::max(1, std::min(sms / pl.tiles, kblocks / 8));
  } else if (!act && pl.tiles <= sms / 2 && kblocks >= 48) {
    splits = (kblocks >= 192 && pl.tiles * 4 <= sms) ? 4 : 2;
  }
  splits = std::min(std::min(splits, 8), std::max(1, kblocks / 4));
  pl.splits = can_split ? splits : 1;
  return pl;
}

template <int BN, int EPI>
static int max_clusters2(int size) {
  using C = Cfg2<BN, EPI>;
  static int cache[9] = {0};
  if (cache[size] == 0) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(size, 64, 1);
    cfg.blockDim = dim3(kThreads, 1, 1);
    cfg.dynamicSmemBytes = C::kSmem;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = size;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    int n = 0;
    if (cudaOccupancyMaxActiveClusters(&n, gemm2_kernel<BN, EPI>, &cfg) != cudaSuccess || n <= 0) {
      cudaGetLastError();
      n = num_sms_cached() / size;
    }
    cache[size] = n;
  }
  return cache[size];
}

template <int BN, int EPI>
static void launch2(Params2 p, const void* x, const void* w, void* out, int N, int K, int ldo, size_t ws_cap,
                    cudaStream_t s) {
  using C = Cfg2<BN, EPI>;
  msgl_set_smem<gemm2_kernel<BN, EPI>>(C::kSmem);
  const CUtensorMap mw = make_map(w, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, N, K, K, BK, C::kRowsA, true);
  const CUtensorMap mx = make_map(x, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, p.M, K, K, BK, C::kTok, true);
  const CUtensorMap mo = EPI == kF32
      ? make_map(out, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, p.M, p.n_out, ldo, 32, 32, false)
      : make_map(out, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, p.M, p.n_out, ldo, 32, 32, false);
  const int tiles = p.n_tiles * p.m_tiles;
  while (p.splits > 1 && (C::xchg_bytes(p.splits) > C::kStages * C::kStage ||
                          tiles > max_clusters2<BN, EPI>(2 * p.splits)))
    --p.splits;
  int groups = tiles;
  if (p.splits == 1) groups = std::min(tiles, std::max(1, max_clusters2<BN, EPI>(2)));
  msgl_launch(gemm2_kernel<BN, EPI>, dim3(2 * p.splits, groups, 1), dim3(kThreads), C::kSmem, s, 2 * p.splits, mw,
              mx, mo, p);
}

// Largest co-resident cluster count for a cluster size (GPCs do not divide evenly by every size).
template <int BN, int EPI, bool WIDE>
static int max_clusters(int size) {
  using C = Cfg<BN, EPI, WIDE>;
  static int cache[9] = {0};
  if (cache[size] == 0) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(size, 64, 1);
    cfg.blockDim = dim3(kThreads, 1, 1);
    cfg.dynamicSmemBytes = C::kSmem;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = size;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    int n = 0;
    if (cudaOccupancyMaxActiveClusters(&n, gemm_kernel<BN, EPI, WIDE>, &cfg) != cudaSuccess || n <= 0) {
      cudaGetLastError();
      n = num_sms_cached() / size;
    }
    cache[size] = n;
  }
  return cache[size];
}

// Choose the cluster (split) size minimizing waves x k-blocks per split + a reduction charge,
// never above `cap`.
template <int BN, int EPI, bool WIDE>
static int best_splits(int tiles, int kblocks, int cap) {
  int best = 1;
  double best_cost = 1e30;
  for (int sz = 1; sz <= std::min(cap, 8); ++sz) {
    const int mc = sz == 1 ? num_sms_cached() : max_clusters<BN, EPI, WIDE>(sz);
    if (mc <= 0) continue;
    const int waves = (tiles + mc - 1) / mc;
    const double cost = waves * ((double)(kblocks + sz - 1) / sz + 6.0) + (sz > 1 ? 2.0 : 0.0);
    if (cost < best_cost - 1e-9) { best_cost = cost; best = sz; }
  }
  return best;
}

template <int BN, int EPI, bool WIDE>
static void launch(const Params& p, const void* x, const void* w, void* out, int N, int K, int ldo, cudaStream_t s) {
  using C = Cfg<BN, EPI, WIDE>;
  msgl_set_smem<gemm_kernel<BN, EPI, WIDE>>(C::kSmem);
  const CUtensorMap mw = p.w_blocked ? make_map_blocked(w, N, K, C::kRowsA)
                                     : make_map(w, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, N, K, K, BK, C::kRowsA, true);
  const CUtensorMap mx = make_map(x, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, p.M, K, K, BK, BN, true);
  const CUtensorMap mo = EPI == kF32
      ? make_map(out, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, p.M, p.n_out, ldo, 32, C::kChunk, false)
      : make_map(out, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, p.M, p.n_out, ldo, 32, C::kChunk, false);
  Params q = p;
  if (q.splits > 1 && !C::kCanSplit) q.splits = 1;
  // shrink the cluster until every tile's cluster is co-resident (GPCs do not divide evenly) and
  // the split-K exchange fits the operand ring
  while (q.splits > 1 && (q.n_tiles * q.m_tiles > max_clusters<BN, EPI, WIDE>(q.splits) ||
                          C::xchg_bytes(q.splits) > C::kStages * C::kStage))
    --q.splits;
  const int tiles = q.n_tiles * q.m_tiles;
  if (q.splits > 1) {
    msgl_launch(gemm_kernel<BN, EPI, WIDE>, dim3(q.splits, tiles, 1), dim3(kThreads), C::kSmem, s, q.splits, mw, mx,
                mo, q);
  } else {
    const int grid = std::min(tiles, num_sms_cached());
    msgl_launch(gemm_kernel<BN, EPI, WIDE>, dim3(grid), dim3(kThreads), C::kSmem, s, 1, mw, mx, mo, q);
  }
}

template <int EPI, bool WIDE>
static void dispatch_bn(int bn, const Params& p, const void* x, const void* w, void* out, int N, int K, int ldo,
                        cudaStream_t s) {
  switch (bn) {
    case 16: launch<16, EPI, WIDE>(p, x, w, out, N, K, ldo, s); break;
    case 32: launch<32, EPI, WIDE>(p, x, w, out, N, K, ldo, s); break;
    case 64: launch<64, EPI, WIDE>(p, x, w, out, N, K, ldo, s); break;
    case 128: launch<128, EPI, WIDE>(p, x, w, out, N, K, ldo, s); break;
    default: launch<256, EPI, WIDE>(p, x, w, out, N, K, ldo, s); break;
  }
}

// 2-SM path: more than 64 tokens (larger decode batches and prefill), row-major weights.
// force_wide == 2 forces it, 0/1 forbid it (they select the 1-SM tile shapes).
static bool use_2sm(int M, int N, int K, int epi, int force_wide, int w_blocked) {
  if (w_blocked) return false;
  if (force_wide == 2) return true;
  if (force_wide >= 0) return false;
  if (const char* e = getenv("MINISGL_GEMM_2SM"))
    if (e[0] == '0') return false;
  if (small_gated(M, N, epi) || small_plain(M, N, K, epi)) return false;
  return M > 64 && K >= 4096;
}

template <int EPI>
static void launch_2sm_bn(int bn, Params2 p, const void* x, const void* w, void* out, int N, int K, int ldo,
                          size_t ws_cap, cudaStream_t s) {
  switch (bn) {
    case 64: launch2<64, EPI>(p, x, w, out, N, K, ldo, ws_cap, s); break;
    case 128: launch2<128, EPI>(p, x, w, out, N, K, ldo, ws_cap, s); break;
    case 160: launch2<160, EPI>(p, x, w, out, N, K, ldo, ws_cap, s); break;
    case 192: launch2<192, EPI>(p, x, w, out, N, K, ldo, ws_cap, s); break;
    case 224: launch2<224, EPI>(p, x, w, out, N, K, ldo, ws_cap, s); break;
    default: launch2<256, EPI>(p, x, w, out, N, K, ldo, ws_cap, s); break;
  }
}

static void launch_2sm(const void* x, const void* w, const void* bias, void* out, int M, int N, int K, int ldo,
                       int epi, int force_splits, void* ws, size_t ws_cap, uint32_t* arrive_ticket,
                       void* arrive_mc, float2* argmax_out, cudaStream_t s) {
  const bool act = is_act(epi);
  Params2 p;
  p.bias = reinterpret_cast<const __nv_bfloat16*>(bias);
  p.arrive_ticket = arrive_ticket;
  p.arrive_mc = arrive_mc;
  p.argmax_out = argmax_out;
  p.M = M;
  p.n_out = act ? N / 2 : N;
  p.kblocks = (K + BK - 1) / BK;
  // token tile = the batch rounded up to a multiple of 32 (MMA N up to 256), so little tensor
  // work is spent on padding; prefill-sized batches use 256-token tiles. Gated outputs then hold
  // gate + up in all 512 TMEM columns (no double buffering), which still beats 128-token tiles:
  // those re-read the weight tile from smem twice as often and saturate smem bandwidth.
  int bn = M <= 64 ? 64 : M <= 128 ? 128 : ((M + 31) / 32) * 32;
  if (M > 256) bn = 256;
  if (const int fb = g_force_bn.load(); fb >= 64 && fb <= 256 && (fb == 64 || fb % 32 == 0) && (fb <= 128 || fb >= 160))
    bn = fb;
  p.n_tiles = (N + (act ? 511 : 255)) / (act ? 512 : 256);
  p.m_tiles = (M + bn - 1) / bn;
  const int tiles = p.n_tiles * p.m_tiles;
  const int sms = num_sms_cached();
  int splits = 1;
  if (force_splits > 0) splits = force_splits;
  else if (2 * tiles <= sms / 2 && p.kblocks >= 32) splits = std::min(sms / (2 * tiles), p.kblocks / 16);
  p.splits = std::max(1, std::min(splits, 4));
  switch (epi) {
    case kBf16: launch_2sm_bn<kBf16>(bn, p, x, w, out, N, K, ldo, ws_cap, s); break;
    case kF32: launch_2sm_bn<kF32>(bn, p, x, w, out, N, K, ldo, ws_cap, s); break;
    case kSilu: launch_2sm_bn<kSilu>(bn, p, x, w, out, N, K, ldo, ws_cap, s); break;
    case kArgmax: launch_2sm_bn<kArgmax>(bn, p, x, w, out, N, K, ldo, ws_cap, s); break;
    default: launch_2sm_bn<kGelu>(bn, p, x, w, out, N, K, ldo, ws_cap, s); break;
  }
}

}  // namespace gemm
}  // namespace msgl

using namespace msgl;
using namespace msgl::gemm;

static void gemm_run(void* out, const void* x, const void* w, int w_blocked, const void* bias, int M, int N, int K,
                     int ldo, int epi, int force_splits, int force_wide, void* workspace, int64_t ws_cap,
                     uint32_t* arrive_ticket, void* arrive_mc, float2* argmax_out, cudaStream_t s);

extern "C" int msgl_gemm_pick_splits(int M, int N, int K) { return make_plan(M, N, K, kBf16, -1, -1).splits; }
extern "C" void msgl_gemm_force_bn(int bn) { g_force_bn.store(bn); }

// split-K exchange buffer of the 2-SM kernel: (pair tiles) x 2 x S(<=4) x 256 rows x 256 tokens fp32
extern "C" int msgl_gemm_workspace_bytes(int M, int N, int K, int splits) {
  const int64_t tiles = (int64_t)((N + 255) / 256) * ((M + 63) / 64);
  return (int)std::min<int64_t>(tiles * 2 * 4 * 256 * 256 * 4, 256ll << 20);
}

extern "C" void msgl_gemm_ex(void* out, const void* x, const void* w, const void* bias, int M, int N, int K,
                             int ldo, int epi, int force_splits, int force_wide, void* workspace, cudaStream_t s) {
  msgl_gemm_ex2(out, x, w, 0, bias, M, N, K, ldo, epi, force_splits, force_wide, workspace,
                workspace ? (int64_t)msgl_gemm_workspace_bytes(M, N, K, 0) : 0, s);
}

extern "C" void msgl_gemm_ex2(void* out, const void* x, const void* w, int w_blocked, const void* bias, int M,
                              int N, int K, int ldo, int epi, int force_splits, int force_wide, void* workspace,
                              int64_t ws_cap, cudaStream_t s) {
  msgl_gemm_ex3(out, x, w, w_blocked, bias, M, N, K, ldo, epi, force_splits, force_wide, workspace, ws_cap, nullptr,
                nullptr, s);
}

extern "C" void msgl_gemm_ex3(void* out, const void* x, const void* w, int w_blocked, const void* bias, int M,
                              int N, int K, int ldo, int epi, int force_splits, int force_wide, void* workspace,
                              int64_t ws_cap, uint32_t* arrive_ticket, void* arrive_mc, cudaStream_t s) {
  gemm_run(out, x, w, w_blocked, bias, M, N, K, ldo, epi, force_splits, force_wide, workspace, ws_cap, arrive_ticket,
           arrive_mc, nullptr, s);
}

// LM-head greedy pick fused into the GEMM: no logits are written; for every token and every block
// of 32 weight rows (vocab ids) the largest logit and its row go to part[block][token] (float2
// {value, row as int bits}); msgl_argmax_partials then reduces the blocks.
extern "C" void msgl_gemm_argmax(void* part, const void* x, const void* w, const void* bias, int M, int N, int K,
                                 void* workspace, int64_t ws_cap, cudaStream_t s) {
  gemm_run(part, x, w, 0, bias, M, N, K, N, kArgmax, -1, -1, workspace, ws_cap, nullptr, nullptr,
           reinterpret_cast<float2*>(part), s);
}

static void gemm_run(void* out, const void* x, const void* w, int w_blocked, const void* bias, int M, int N, int K,
                     int ldo, int epi, int force_splits, int force_wide, void* workspace, int64_t ws_cap,
                     uint32_t* arrive_ticket, void* arrive_mc, float2* argmax_out, cudaStream_t s) {
  if (M <= 0 || N <= 0) return;
  Plan pl = make_plan(M, N, K, epi, force_splits, force_wide);
  Params p;
  p.bias = reinterpret_cast<const __nv_bfloat16*>(bias);
  p.arrive_ticket = arrive_ticket;
  p.arrive_mc = arrive_mc;
  p.argmax_out = argmax_out;
  p.grp_count = nullptr;
  p.grp_work = nullptr;
  p.bias_stride = 0;
  p.w_blocked = w_blocked;
  p.M = M;
  p.n_out = is_act(epi) ? N / 2 : N;
  p.n_tiles = (N + pl.rows_a - 1) / pl.rows_a;
  p.m_tiles = (M + pl.bn - 1) / pl.bn;
  p.kblocks = (K + BK - 1) / BK;
  p.splits = pl.splits;
  if (use_2sm(M, N, K, epi, force_wide, w_blocked)) {
    launch_2sm(x, w, bias, out, M, N, K, ldo, epi, force_splits, workspace, (size_t)ws_cap, arrive_ticket, arrive_mc,
               argmax_out, s);
    return;
  }
  const bool wide = pl.wide;
  switch (epi) {
    case kBf16: wide ? dispatch_bn<kBf16, true>(pl.bn, p, x, w, out, N, K, ldo, s)
                     : dispatch_bn<kBf16, false>(pl.bn, p, x, w, out, N, K, ldo, s); break;
    case kArgmax: wide ? dispatch_bn<kArgmax, true>(pl.bn, p, x, w, out, N, K, ldo, s)
                       : dispatch_bn<kArgmax, false>(pl.bn, p, x, w, out, N, K, ldo, s); break;
    case kSilu: dispatch_bn<kSilu, true>(pl.bn, p, x, w, out, N, K, ldo, s); break;
    case kGelu: dispatch_bn<kGelu, true>(pl.bn, p, x, w, out, N, K, ldo, s); break;
    default: wide ? dispatch_bn<kF32, true>(pl.bn, p, x, w, out, N, K, ldo, s)
                  : dispatch_bn<kF32, false>(pl.bn, p, x, w, out, N, K, ldo, s); break;
  }
}

extern "C" void msgl_gemm(void* out, const void* x, const void* w, const void* bias, int M, int N, int K,
                          int ldo, int epi, int splits, void* workspace, cudaStream_t s) {
  msgl_gemm_ex(out, x, w, bias, M, N, K, ldo, epi, splits, -1, workspace, s);
}

template <int BN, int EPI>
static void launch_grouped(const Params& p, const void* x, const void* w, void* out, int E, int N, int K, int ldo,
                           cudaStream_t s) {
  constexpr bool kGated = EPI != kBf16;
  using C = Cfg<BN, EPI, kGated>;
  msgl_set_smem<gemm_kernel<BN, EPI, kGated>>(C::kSmem);
  const CUtensorMap mw = make_map_experts(w, E, N, K, C::kRowsA);
  const CUtensorMap mx = make_map(x, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, p.M, K, K, BK, BN, true);
  const CUtensorMap mo = make_map(out, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, p.M, p.n_out, ldo, 32, C::kChunk, false);
  const int units = p.n_tiles * p.m_tiles;
  msgl_launch(gemm_kernel<BN, EPI, kGated>, dim3(std::min(units, num_sms_cached())), dim3(kThreads), C::kSmem, s,
              1, mw, mx, mo, p);
}

template <int EPI>
static void launch_grouped_bn(int bn, const Params& p, const void* x, const void* w, void* out, int E, int N, int K,
                              int ldo, cudaStream_t s) {
  switch (bn) {
    case 16: launch_grouped<16, EPI>(p, x, w, out, E, N, K, ldo, s); break;
    case 32: launch_grouped<32, EPI>(p, x, w, out, E, N, K, ldo, s); break;
    case 64: launch_grouped<64, EPI>(p, x, w, out, E, N, K, ldo, s); break;
    default: launch_grouped<128, EPI>(p, x, w, out, E, N, K, ldo, s); break;
  }
}

// Grouped GEMM for routed experts: for every token tile t < *tile_count (device), rows
// [work[t].y, work[t].y + bn) of x (permuted activations, [rows_cap, K]) times expert work[t].x of
// w ([E, N, K]) -> the same rows of out ([rows_cap, N], row stride ldo), plus bias[e] if given.
// epi 1 / 2 / 4 (SiLU / GELU / gpt-oss SwiGLU): w's rows are gate / up interleaved in 128-row
// blocks (N % 256 == 0) and out is the activated [rows_cap, N / 2], computed in the epilogue.
extern "C" void msgl_gemm_grouped(void* out, const void* x, const void* w, const void* bias, int rows_cap, int N,
                                  int K, int ldo, int E, const int* tile_count, const void* work, int max_tiles,
                                  int bn, int epi, cudaStream_t s) {
  if (rows_cap <= 0 || N <= 0 || max_tiles <= 0) return;
  const bool gated = epi != kBf16;
  Params p;
  p.bias = reinterpret_cast<const __nv_bfloat16*>(bias);
  p.arrive_ticket = nullptr;
  p.arrive_mc = nullptr;
  p.argmax_out = nullptr;
  p.bias_stride = N;
  p.w_blocked = 0;
  p.grp_count = tile_count;
  p.grp_work = reinterpret_cast<const int2*>(work);
  p.M = rows_cap;
  p.n_out = gated ? N / 2 : N;
  p.n_tiles = gated ? N / 256 : (N + 127) / 128;
  p.m_tiles = max_tiles;
  p.kblocks = (K + BK - 1) / BK;
  p.splits = 1;
  switch (epi) {
    case kSilu: launch_grouped_bn<kSilu>(bn, p, x, w, out, E, N, K, ldo, s); break;
    case kGelu: launch_grouped_bn<kGelu>(bn, p, x, w, out, E, N, K, ldo, s); break;
    case kSwiglu: launch_grouped_bn<kSwiglu>(bn, p, x, w, out, E, N, K, ldo, s); break;
    default: launch_grouped_bn<kBf16>(bn, p, x, w, out, E, N, K, ldo, s); break;
  }
}

template <int BN, int EPI>
static void launch_grouped_fp4(const Params& p, const void* x, const uint8_t* q, const uint8_t* sc, int n_pad,
                               void* out, int K, int ldo, cudaStream_t s) {
  constexpr bool kGated = EPI != kBf16;
  using C = Cfg<BN, EPI, kGated>;
  using F = CfgF4<BN, EPI, kGated>;
  msgl_set_smem<gemm_fp4_kernel<BN, EPI, kGated>>(F::kSmem);
  const CUtensorMap mx = make_map(x, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, p.M, K, K, BK, BN, true);
  const CUtensorMap mo = make_map(out, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, p.M, p.n_out, ldo, 32, C::kChunk, false);
  const int units = p.n_tiles * p.m_tiles;
  msgl_launch(gemm_fp4_kernel<BN, EPI, kGated>, dim3(std::min(units, num_sms_cached())), dim3(threads_f4<BN>()), F::kSmem,
              s, 1, mx, mo, q, sc, n_pad, p);
}

template <int EPI>
static void launch_grouped_fp4_bn(int bn, const Params& p, const void* x, const uint8_t* q, const uint8_t* sc,
                                  int n_pad, void* out, int K, int ldo, cudaStream_t s) {
  switch (bn) {
    case 16: launch_grouped_fp4<16, EPI>(p, x, q, sc, n_pad, out, K, ldo, s); break;
    case 32: launch_grouped_fp4<32, EPI>(p, x, q, sc, n_pad, out, K, ldo, s); break;
    case 64: launch_grouped_fp4<64, EPI>(p, x, q, sc, n_pad, out, K, ldo, s); break;
    default: launch_grouped_fp4<128, EPI>(p, x, q, sc, n_pad, out, K, ldo, s); break;
  }
}

// msgl_gemm_grouped with MXFP4 expert weights in the k-block-major layout (see gemm_fp4_kernel):
// q [E][K/64][n_pad][32] e2m1 bytes, sc [E][K/64][n_pad][2] e8m0 scales; N logical rows (gated:
// gate / up interleaved in 128-row blocks, N % 256 == 0), n_pad >= N a multiple of the weight tile
// (256 gated, 128 otherwise), K % 64 == 0.
extern "C" int msgl_gemm_grouped_fp4(void* out, const void* x, const void* q, const void* sc, const void* bias,
                                     int rows_cap, int N, int n_pad, int K, int ldo, int E, const int* tile_count,
                                     const void* work, int max_tiles, int bn, int epi, cudaStream_t s) {
  if (rows_cap <= 0 || N <= 0 || max_tiles <= 0) return 0;
  const bool gated = epi != kBf16;
  if (K % BK != 0 || (gated && (N % 256 != 0 || n_pad != N)) || (!gated && (n_pad % 128 != 0 || n_pad < N)) ||
      E <= 0)
    return 3;
  Params p;
  p.bias = reinterpret_cast<const __nv_bfloat16*>(bias);
  p.arrive_ticket = nullptr;
  p.arrive_mc = nullptr;
  p.argmax_out = nullptr;
  p.bias_stride = N;
  p.w_blocked = 0;
  p.grp_count = tile_count;
  p.grp_work = reinterpret_cast<const int2*>(work);
  p.M = rows_cap;
  p.n_out = gated ? N / 2 : N;
  p.n_tiles = gated ? N / 256 : (N + 127) / 128;
  p.m_tiles = max_tiles;
  p.kblocks = K / BK;
  p.splits = 1;
  const uint8_t* q8 = reinterpret_cast<const uint8_t*>(q);
  const uint8_t* s8 = reinterpret_cast<const uint8_t*>(sc);
  switch (epi) {
    case kSilu: launch_grouped_fp4_bn<kSilu>(bn, p, x, q8, s8, n_pad, out, K, ldo, s); break;
    case kGelu: launch_grouped_fp4_bn<kGelu>(bn, p, x, q8, s8, n_pad, out, K, ldo, s); break;
    case kSwiglu: launch_grouped_fp4_bn<kSwiglu>(bn, p, x, q8, s8, n_pad, out, K, ldo, s); break;
    default: launch_grouped_fp4_bn<kBf16>(bn, p, x, q8, s8, n_pad, out, K, ldo, s); break;
  }
  return 0;
}

namespace {

// One CTA per token: the best of its blocks' {value, row} partials; equal values resolve to the
// lowest row, as torch.argmax does. Rows are offset by `id_offset` (a vocabulary shard's first id).
__global__ void argmax_partials_kernel(int32_t* __restrict__ out, float* __restrict__ out_val,
                                       const float2* __restrict__ part, int n_blk, int M, int id_offset) {
  pdl_wait();
  pdl_launch();
  const int t = blockIdx.x;
  float best = -INFINITY;
  int bi = 0x7fffffff;
  for (int b = threadIdx.x; b < n_blk; b += blockDim.x) {
    const float2 v = part[(int64_t)b * M + t];
    const int r = __float_as_int(v.y);
    if (v.x > best || (v.x == best && r < bi)) { best = v.x; bi = r; }
  }
  __shared__ float sv[32];
  __shared__ int si[32];
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float ov = __shfl_xor_sync(0xffffffffu, best, o);
    const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
    if (ov > best || (ov == best && oi < bi)) { best = ov; bi = oi; }
  }
  const int warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
  if ((threadIdx.x & 31) == 0) { sv[warp] = best; si[warp] = bi; }
  __syncthreads();
  if (threadIdx.x == 0) {
    for (int w = 1; w < nw; ++w)
      if (sv[w] > best || (sv[w] == best && si[w] < bi)) { best = sv[w]; bi = si[w]; }
    out[t] = bi + id_offset;
    if (out_val != nullptr) out_val[t] = best;
  }
}

}  // namespace

extern "C" void msgl_argmax_partials(int32_t* out, float* out_val, const void* part, int n_blk, int M, int id_offset,
                                     cudaStream_t s) {
  if (M <= 0) return;
  msgl_launch(argmax_partials_kernel, dim3(M), dim3(256), 0, s, 1, out, out_val, reinterpret_cast<const float2*>(part),
              n_blk, M, id_offset);
}

extern "C" int msgl_num_sms() { return num_sms_cached(); }

MSGL_ERROR_ACCESSOR(msgl_err_gemm)
