// C ABI between the torch bindings (bindings.cpp) and the CUDA translation units. Kernels take
// raw pointers, sizes and a stream; no torch headers are included on the device side.
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

extern "C" {

// ----- status
int msgl_get_error(int* info);  // returns and clears the device error word
int msgl_num_sms();

// ----- elementwise / normalization (bf16 activations)
void msgl_embedding(void* out, const void* weight, const int32_t* ids, int n, int dim,
                    int vocab_start, int vocab_len, int masked, cudaStream_t s);
void msgl_rmsnorm(void* out, const void* x, const void* w, int rows, int dim, float eps,
                  cudaStream_t s);
void msgl_fused_add_rmsnorm(void* x, void* residual, const void* w, int rows, int dim, float eps,
                            cudaStream_t s);
void msgl_act_and_mul(void* out, const void* x, int rows, int inter, int act, cudaStream_t s);
void msgl_store_kv(const void* k, const void* v, void* k_cache, void* v_cache,
                   const int32_t* out_loc, int n, int row_elems, int64_t k_stride, int64_t v_stride,
                   int64_t cache_stride, int64_t num_slots, cudaStream_t s);
void msgl_qk_norm_rope_store(void* q_out, const void* qkv, const int32_t* positions,
                             const float* cos_sin, const void* q_norm, const void* k_norm,
                             float eps, void* k_cache, void* v_cache, const int32_t* out_loc,
                             int n, int nq, int nkv, int hd, int64_t cache_stride, int64_t num_slots,
                             int max_pos, cudaStream_t s);
// row argmax over the first `vocab` columns; out_val (optional) receives the maximum
void msgl_argmax(int32_t* out, float* out_val, const void* logits, int rows, int vocab, int64_t stride,
                 int is_fp32, cudaStream_t s);
// col_ids (optional, [rows, vocab] int32): token id of each column (candidate lists); otherwise
// column i is token id_offset + i. out_val (optional): the winning Gumbel score per row (the max
// logit on greedy rows), for combining vocabulary shards.
void msgl_sample(int32_t* out, const float* logits, int rows, int vocab, int64_t stride,
                 const float* temperature, const int32_t* top_k, const float* top_p,
                 const int64_t* seed, const int64_t* step, const int32_t* col_ids, int id_offset,
                 float* out_val, cudaStream_t s);

// ----- GEMM: out[M,N] = epi(x[M,K] @ w[N,K]^T + bias)
//   epi 0: bf16 out; 1: silu(g)*u on 64-row interleaved gate/up (out has N/2 cols);
//   2: gelu(g)*u likewise; 3: fp32 out.
// workspace: L2-resident split-K exchange buffer of the 2-SM kernel (null disables its split-K).
int msgl_gemm_workspace_bytes(int M, int N, int K, int splits);
int msgl_gemm_pick_splits(int M, int N, int K);
void msgl_gemm(void* out, const void* x, const void* w, const void* bias, int M, int N, int K,
               int ldo, int epi, int splits, void* workspace, cudaStream_t s);
// same with explicit tiling overrides (splits > 0 forces split-K; wide 0/1 forces 128/256-row
// weight tiles for plain outputs; -1 = automatic)
void msgl_gemm_ex(void* out, const void* x, const void* w, const void* bias, int M, int N, int K,
                  int ldo, int epi, int splits, int wide, void* workspace, cudaStream_t s);
// w_blocked: weight stored K-block major as [K/64][N][64] (requires K % 64 == 0)
void msgl_gemm_ex2(void* out, const void* x, const void* w, int w_blocked, const void* bias, int M, int N,
                   int K, int ldo, int epi, int splits, int wide, void* workspace, int64_t ws_bytes,
                   cudaStream_t s);
// msgl_gemm_ex2 whose output is this rank's NVLS staging region: the launch's last CTA adds 1 to the
// multicast arrival counter `arrive_mc` (local ticket `arrive_ticket`), for the fused collective.
void msgl_gemm_ex3(void* out, const void* x, const void* w, int w_blocked, const void* bias, int M, int N,
                   int K, int ldo, int epi, int force_splits, int force_wide, void* workspace, int64_t ws_cap,
                   uint32_t* arrive_ticket, void* arrive_mc, cudaStream_t s);
// Token-tile override for tiling sweeps and tests (-1 restores the automatic choice).
void msgl_gemm_force_bn(int bn);
// LM-head greedy pick fused into the GEMM (out = x @ w^T is never written): part is
// [ceil(N / 32)][M] float2 {largest value, its row}; msgl_argmax_partials reduces it per token to the
// row (+ id_offset) and optionally its value. Ties resolve to the lowest row.
void msgl_gemm_argmax(void* part, const void* x, const void* w, const void* bias, int M, int N, int K,
                      void* workspace, int64_t ws_cap, cudaStream_t s);
void msgl_argmax_partials(int32_t* out, float* out_val, const void* part, int n_blk, int M, int id_offset,
                          cudaStream_t s);

// ----- routed experts (MoE)
// epi 0: plain bf16 output; 1 / 2 / 4 (SiLU / GELU / gpt-oss SwiGLU): w rows gate/up interleaved in
// 128-row blocks and the activated [rows, N / 2] written by the epilogue
void msgl_gemm_grouped(void* out, const void* x, const void* w, const void* bias, int rows_cap, int N, int K,
                       int ldo, int E, const int* tile_count, const void* work, int max_tiles, int bn, int epi,
                       cudaStream_t s);
// msgl_gemm_grouped with MXFP4 expert weights kept in HBM (k-block-major: q [E][K/64][n_pad][32]
// e2m1 bytes, sc [E][K/64][n_pad][2] e8m0 scales; N logical rows, K % 64 == 0). Returns 0, or 3 for
// an unsupported shape.
int msgl_gemm_grouped_fp4(void* out, const void* x, const void* q, const void* sc, const void* bias, int rows_cap,
                          int N, int n_pad, int K, int ldo, int E, const int* tile_count, const void* work,
                          int max_tiles, int bn, int epi, cudaStream_t s);
void msgl_moe_route(const float* logits, int T, int E, int topk, int renorm, int softmax_after, float* weights,
                    int32_t* ids, cudaStream_t s);
// experts [e0, e0 + E) are local (expert parallelism); other assignments get inv = -1
void msgl_moe_align(const int32_t* ids, int pairs, int E, int e0, int bn, int max_tiles, int rows_cap, int32_t* perm,
                    int32_t* inv, void* work, int32_t* tile_count, cudaStream_t s);
void msgl_moe_gather(void* xs, const void* x, const int32_t* perm, int rows, int H, int topk, int x_rows,
                     cudaStream_t s);
void msgl_moe_act(void* out, const void* y, int rows, int inter, int act, const int32_t* perm, cudaStream_t s);
void msgl_moe_combine(void* out, const void* y, const float* w, const int32_t* inv, int T, int H, int topk,
                      int y_rows, cudaStream_t s);

// ----- paged attention (bf16 q/kv, fp32 softmax)
void msgl_attention_prefill(void* o, const void* q, const void* k_cache, const void* v_cache,
                            const int32_t* page_table, int64_t pt_stride, const int32_t* rows,
                            const int32_t* cu_q, const int32_t* kv_lens, int num_reqs,
                            int total_q, int max_q_len, int nq, int nkv, int hd,
                            int64_t cache_stride, int64_t num_slots, float sm_scale, int window,
                            const float* sinks, cudaStream_t s);
void msgl_attention_decode(void* o, const void* q, const void* k_cache, const void* v_cache,
                           const int32_t* page_table, int64_t pt_stride, const int32_t* rows,
                           const int32_t* kv_lens, int bs, int nq, int nkv, int hd,
                           int64_t cache_stride, int64_t num_slots, float sm_scale, int window,
                           const float* sinks, int num_splits, void* workspace, cudaStream_t s);

// tcgen05 ragged causal prefill attention (head_dim 128, page size 16/32/64; see attention.cu).
// Returns 0 on success, 2 if a tensor map could not be encoded, 3 on unsupported arguments.
int msgl_attention_prefill_fmha(void* o, const void* q, int64_t total_q, const void* k_cache, const void* v_cache,
                                int64_t num_slots, int64_t cache_stride, const int32_t* page_table, int64_t pt_stride,
                                const int32_t* rows, const int32_t* cu_q, const int32_t* kv_lens, int num_reqs,
                                int max_q_len, int nq, int nkv, int hd, int page, float sm_scale, int window,
                                const float* sinks, cudaStream_t s);
// Profiling: record per-CTA phase stamps of later prefill launches into buf ([ctas][96] uint32, SM
// clock cycles since each CTA started; kv head 0 only); nullptr turns it off. Not for concurrent use.
void msgl_attention_prefill_trace(uint32_t* buf, int ctas);

// Persistent paged decode over a host-built work list (page size 16/32/64; see attention.cu).
// Returns 0 on success, 2 if a tensor map could not be encoded, 3 on unsupported arguments.
int msgl_attention_decode_paged(void* o, const void* q, int q_rows, const void* k_cache, const void* v_cache,
                                int64_t num_slots, int64_t cache_stride, const int32_t* page_table,
                                int64_t pt_stride, const int32_t* rows, const int32_t* kv_lens,
                                const int32_t* work, const int32_t* n_work, float* ws, int ws_slots,
                                int32_t* counters, int nq, int nkv, int hd, int page, float sm_scale,
                                int window, const float* sinks, cudaStream_t s);

// ----- allocation-free decode attention (no counterpart in the reference; see attention.cu):
// split-KV scratch comes from a fixed 8 MiB file-scope device array instead of a workspace
// argument. Returns 0 on success, 1 if the problem needs more scratch than that, 2 if the
// per-device set-up failed, 3 on bad arguments, 4 if a launch failed. `num_slots` bounds the
// page-table entries in the bounds-check build. Calls that overlap on the
// GPU race on the shared scratch; the first call on a device must precede any stream capture.
int msgl_attention_decode_noalloc(void* o, const void* q, const void* k_cache, const void* v_cache,
                                  const int32_t* page_table, int64_t pt_stride, const int32_t* rows,
                                  const int32_t* kv_lens, int bs, int nq, int nkv, int hd,
                                  int64_t cache_stride, int64_t num_slots, float sm_scale, int window,
                                  const float* sinks, int num_splits, cudaStream_t s);

// ----- NVLS (multicast) all-reduce fused with residual add + RMSNorm (see comm.cu)
// ----- batch metadata (plan.cu): page-table writes + out_loc gather in one launch; int32 gather /
// scatter through an index list
void msgl_plan_apply(int32_t* page_table, int64_t pt_stride, int64_t pt_rows_total, const int32_t* pt_rows,
                     const int32_t* pt_pos, const int32_t* pt_slots, int n_writes, const int32_t* tok_rows,
                     const int32_t* positions, int n_tok, int32_t* out_loc, cudaStream_t s);
void msgl_gather_i32(int32_t* dst, const int32_t* src, int64_t src_len, const int32_t* idx, int n, cudaStream_t s);
void msgl_scatter_i32(int32_t* dst, int64_t dst_len, const int32_t* idx, const int32_t* src, int n, cudaStream_t s);

// mode 0: LL (small messages; out written), 1: RS with x copied into staging, 2: RS with x already
// in staging, 3: RS with staging written and arrival signalled by msgl_gemm_ex3. RS writes the
// normalised rows into the buffer's gather region and only this rank's rows (i % world == rank) of
// the residual. `trace` (optional, [128][8] uint64) receives %globaltimer stamps of the RS phases per
// CTA. Returns 0, 3 on bad arguments, 4 if the launch failed.
int msgl_nvls_grid();
int msgl_nvls_flag_bytes();
int msgl_nvls_state_words();
int64_t msgl_nvls_ticket_offset();
int msgl_nvls_allreduce_rmsnorm(void* uc, void* mc, int rank, int world, const void* x, void* residual, const void* w,
                                void* out, int T, int H, float eps, int64_t cap_bytes, uint32_t* state,
                                int64_t timeout_ns, int first, int mode, uint64_t* trace, cudaStream_t s);

// ----- peer-memory collectives (CUDA IPC over NVLink)
int msgl_peer_flag_bytes();
void* msgl_peer_alloc(int64_t bytes);
void msgl_peer_free(void* p);
int msgl_ipc_handle(void* p, void* out64);
void* msgl_ipc_open(const void* in64);
void msgl_ipc_close(void* p);
int msgl_peer_grid();  // CTAs per collective; the state tensor holds 2 uint32 per CTA
// mode 0: one-shot all-reduce, 1: two-shot all-reduce, 2: all-gather (dim 0)
void msgl_peer_collective(void* const* bases, int rank, int world, int mode, void* out, const void* in,
                          int64_t bytes, int64_t cap_bytes, uint32_t* state, int64_t timeout_ns, cudaStream_t s);
}
