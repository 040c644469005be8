// Torch bindings for the sm_100a kernels: validate tensors (dtype / device / contiguity / shape),
// take the current CUDA stream, and call the C ABI in kernels/api.h.
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/extension.h>

#include <string>
#include <vector>

#include <mutex>
#include <unordered_map>

#include "kernels/api.h"

namespace {

#define CHECK(cond, ...) TORCH_CHECK(cond, "minisgl: ", __VA_ARGS__)

void check_cuda(const at::Tensor& t, const char* name) {
  CHECK(t.is_cuda(), name, " must be a CUDA tensor");
}
void check_dtype(const at::Tensor& t, at::ScalarType dt, const char* name) {
  CHECK(t.scalar_type() == dt, name, " must be ", c10::toString(dt), ", got ", t.scalar_type());
}
void check_contig(const at::Tensor& t, const char* name) { CHECK(t.is_contiguous(), name, " must be contiguous"); }
void check_bf16(const at::Tensor& t, const char* name) {
  check_cuda(t, name);
  check_dtype(t, at::kBFloat16, name);
}
void check_i32(const at::Tensor& t, const char* name) {
  check_cuda(t, name);
  check_dtype(t, at::kInt, name);
  check_contig(t, name);
}
const void* opt_ptr(const c10::optional<at::Tensor>& t) { return t.has_value() ? t->data_ptr() : nullptr; }

cudaStream_t stream() { return at::cuda::getCurrentCUDAStream().stream(); }

// Per-device scratch for split-K partials / counters (zero-initialised once; kernels leave the
// counters at zero). Sized generously on first use so CUDA-graph capture never reallocates it.
at::Tensor& gemm_workspace(const at::Device& dev, int64_t bytes) {
  static std::mutex mu;
  static std::unordered_map<int, at::Tensor> ws;
  std::lock_guard<std::mutex> g(mu);
  auto& t = ws[dev.index()];
  if (!t.defined() || t.numel() < bytes) {
    const int64_t sz = std::max<int64_t>(bytes, 64ll << 20);
    t = at::zeros({sz}, at::TensorOptions().dtype(at::kByte).device(dev));
  }
  return t;
}

void embedding(at::Tensor out, at::Tensor weight, at::Tensor ids, int64_t lo, int64_t n, bool masked) {
  check_bf16(out, "out"); check_bf16(weight, "weight"); check_i32(ids, "ids");
  check_contig(out, "out"); check_contig(weight, "weight");
  const int dim = weight.size(1);
  CHECK(dim % 8 == 0, "hidden size must be a multiple of 8");
  CHECK(out.size(0) == ids.size(0) && out.size(1) == dim, "embedding out shape");
  msgl_embedding(out.data_ptr(), weight.data_ptr(), ids.data_ptr<int32_t>(), ids.size(0), dim, lo, n,
                 masked, stream());
}

void rmsnorm(at::Tensor out, at::Tensor x, at::Tensor w, double eps) {
  check_bf16(out, "out"); check_bf16(x, "x"); check_bf16(w, "w");
  check_contig(out, "out"); check_contig(x, "x");
  const int dim = x.size(-1);
  CHECK(dim % 8 == 0 && w.numel() == dim, "rmsnorm dim");
  msgl_rmsnorm(out.data_ptr(), x.data_ptr(), w.data_ptr(), x.numel() / dim, dim, eps, stream());
}

void fused_add_rmsnorm(at::Tensor x, at::Tensor residual, at::Tensor w, double eps) {
  check_bf16(x, "x"); check_bf16(residual, "residual"); check_bf16(w, "w");
  check_contig(x, "x"); check_contig(residual, "residual");
  const int dim = x.size(-1);
  CHECK(dim % 8 == 0 && w.numel() == dim && residual.numel() == x.numel(), "fused_add_rmsnorm shapes");
  msgl_fused_add_rmsnorm(x.data_ptr(), residual.data_ptr(), w.data_ptr(), x.numel() / dim, dim, eps, stream());
}

// epi: 0 bf16, 1 silu-mul (interleaved gate/up), 2 gelu-mul, 3 fp32 out.
// w is [N, K] row-major, or K-block major [K/64, N, 64] (3-D tensor).
void gemm_ex(at::Tensor out, at::Tensor x, at::Tensor w, c10::optional<at::Tensor> bias, int64_t epi,
             int64_t splits, int64_t wide) {
  check_bf16(x, "x"); check_bf16(w, "w"); check_cuda(out, "out");
  check_contig(x, "x"); check_contig(w, "w");
  CHECK(out.stride(-1) == 1, "out must have unit inner stride");
  const bool blocked = w.dim() == 3;
  const int64_t M = x.size(0), K = x.size(1);
  const int64_t N = blocked ? w.size(1) : w.size(0);
  if (blocked) {
    CHECK(w.size(2) == 64 && w.size(0) * 64 == K, "blocked weight must be [K/64, N, 64], got ", w.sizes());
  } else {
    CHECK(w.size(1) == K, "gemm K mismatch: x ", x.sizes(), " w ", w.sizes());
  }
  CHECK(K % 8 == 0 && N % 8 == 0, "gemm needs K and N multiples of 8");
  if (epi == 3) {
    check_dtype(out, at::kFloat, "out");
  } else {
    check_dtype(out, at::kBFloat16, "out");
  }
  const int64_t n_out = (epi == 1 || epi == 2) ? N / 2 : N;
  CHECK(out.size(0) == M && out.size(1) == n_out, "gemm out shape");
  if (bias.has_value()) { check_bf16(*bias, "bias"); CHECK(bias->numel() == N, "bias size"); }
  if (M == 0) return;
  CHECK(out.stride(0) % (epi == 3 ? 4 : 8) == 0, "out row stride must be 16-byte aligned");
  if (epi == 1 || epi == 2) CHECK(N % 256 == 0, "gated GEMM needs N (gate+up rows) to be a multiple of 256");
  const int64_t wsb = msgl_gemm_workspace_bytes(M, N, K, 0);
  at::Tensor& ws = gemm_workspace(x.device(), wsb);
  msgl_gemm_ex2(out.data_ptr(), x.data_ptr(), w.data_ptr(), blocked ? 1 : 0, opt_ptr(bias), M, N, K,
                out.stride(0), epi, splits, wide, ws.data_ptr(), ws.numel(), stream());
}

void gemm(at::Tensor out, at::Tensor x, at::Tensor w, c10::optional<at::Tensor> bias, int64_t epi) {
  gemm_ex(out, x, w, bias, epi, -1, -1);
}

// Greedy pick fused into the LM-head GEMM: ids[t] = id_offset + argmax_r (x[t] . w[r]) over the first
// n_valid rows of w (and the max into vals when given), without writing the logits.
void lm_head_argmax(at::Tensor ids, c10::optional<at::Tensor> vals, at::Tensor x, at::Tensor w,
                    c10::optional<at::Tensor> bias, int64_t n_valid, int64_t id_offset) {
  check_bf16(x, "x"); check_bf16(w, "w"); check_contig(x, "x"); check_contig(w, "w");
  check_cuda(ids, "ids"); check_dtype(ids, at::kInt, "ids");
  CHECK(w.dim() == 2 && x.dim() == 2 && w.size(1) == x.size(1), "lm head shapes: x ", x.sizes(), " w ", w.sizes());
  const int64_t M = x.size(0), K = x.size(1);
  CHECK(n_valid > 0 && n_valid <= w.size(0), "n_valid out of range");
  CHECK(K % 8 == 0, "K must be a multiple of 8");
  CHECK(ids.numel() == M, "ids size");
  if (vals.has_value()) { check_cuda(*vals, "vals"); check_dtype(*vals, at::kFloat, "vals"); CHECK(vals->numel() == M, "vals size"); }
  if (bias.has_value()) { check_bf16(*bias, "bias"); CHECK(bias->numel() >= n_valid, "bias size"); }
  if (M == 0) return;
  const int64_t n_blk = (n_valid + 31) / 32;
  at::Tensor part = at::empty({n_blk, M, 2}, x.options().dtype(at::kFloat));
  const int64_t wsb = msgl_gemm_workspace_bytes(M, n_valid, K, 0);
  at::Tensor& ws = gemm_workspace(x.device(), wsb);
  msgl_gemm_argmax(part.data_ptr(), x.data_ptr(), w.data_ptr(), opt_ptr(bias), M, n_valid, K, ws.data_ptr(),
                   ws.numel(), stream());
  msgl_argmax_partials(ids.data_ptr<int32_t>(), vals.has_value() ? vals->data_ptr<float>() : nullptr,
                       part.data_ptr(), n_blk, M, id_offset, stream());
}

// bf16 GEMM into this rank's NVLS staging region (out), signalling arrival on the multicast counter
// at `arrive_mc` through the local ticket at `arrive_ticket` (fused row-parallel collective)
void gemm_signal(at::Tensor out, at::Tensor x, at::Tensor w, c10::optional<at::Tensor> bias, int64_t arrive_ticket,
                 int64_t arrive_mc) {
  check_bf16(x, "x"); check_bf16(w, "w"); check_bf16(out, "out");
  check_contig(x, "x"); check_contig(w, "w"); check_contig(out, "out");
  CHECK(w.dim() == 2, "gemm_signal takes a row-major [N, K] weight");
  const int64_t M = x.size(0), K = x.size(1), N = w.size(0);
  CHECK(w.size(1) == K, "gemm K mismatch: x ", x.sizes(), " w ", w.sizes());
  CHECK(K % 8 == 0 && N % 8 == 0, "gemm needs K and N multiples of 8");
  CHECK(out.size(0) == M && out.size(1) == N, "gemm out shape");
  CHECK(arrive_ticket != 0 && arrive_mc != 0, "gemm_signal needs the arrival ticket and counter");
  if (bias.has_value()) { check_bf16(*bias, "bias"); CHECK(bias->numel() == N, "bias size"); }
  CHECK(M > 0, "gemm_signal needs at least one row (every rank must arrive)");
  const int64_t wsb = msgl_gemm_workspace_bytes(M, N, K, 0);
  at::Tensor& ws = gemm_workspace(x.device(), wsb);
  msgl_gemm_ex3(out.data_ptr(), x.data_ptr(), w.data_ptr(), 0, opt_ptr(bias), M, N, K, out.stride(0), 0, -1, -1,
                ws.data_ptr(), ws.numel(), reinterpret_cast<uint32_t*>(arrive_ticket),
                reinterpret_cast<void*>(arrive_mc), stream());
}

void act_and_mul(at::Tensor out, at::Tensor x, int64_t act) {
  check_bf16(out, "out"); check_bf16(x, "x"); check_contig(out, "out"); check_contig(x, "x");
  const int inter = x.size(1) / 2;
  CHECK(inter % 8 == 0 && out.size(1) == inter, "act_and_mul shapes");
  msgl_act_and_mul(out.data_ptr(), x.data_ptr(), x.size(0), inter, act, stream());
}

void store_kv(at::Tensor k, at::Tensor v, at::Tensor k_cache, at::Tensor v_cache, at::Tensor out_loc) {
  check_bf16(k, "k"); check_bf16(v, "v"); check_bf16(k_cache, "k_cache"); check_bf16(v_cache, "v_cache");
  check_i32(out_loc, "out_loc");
  const int64_t row = k_cache.numel() / k_cache.size(0);
  CHECK(k.size(1) == row && v.size(1) == row && row % 8 == 0, "store_kv row size");
  CHECK(k.stride(1) == 1 && v.stride(1) == 1, "store_kv rows must be contiguous");
  CHECK(k.stride(0) % 8 == 0 && v.stride(0) % 8 == 0, "store_kv row stride alignment");
  msgl_store_kv(k.data_ptr(), v.data_ptr(), k_cache.data_ptr(), v_cache.data_ptr(), out_loc.data_ptr<int32_t>(),
                k.size(0), row, k.stride(0), v.stride(0), row, k_cache.size(0), stream());
}

void qk_norm_rope_store(at::Tensor q_out, at::Tensor qkv, at::Tensor positions, at::Tensor cos_sin,
                        c10::optional<at::Tensor> q_norm, c10::optional<at::Tensor> k_norm, double eps,
                        at::Tensor k_cache, at::Tensor v_cache, at::Tensor out_loc, int64_t nq, int64_t nkv,
                        int64_t hd) {
  check_bf16(q_out, "q_out"); check_bf16(qkv, "qkv"); check_i32(positions, "positions");
  check_cuda(cos_sin, "cos_sin"); check_dtype(cos_sin, at::kFloat, "cos_sin"); check_contig(cos_sin, "cos_sin");
  check_bf16(k_cache, "k_cache"); check_bf16(v_cache, "v_cache"); check_i32(out_loc, "out_loc");
  check_contig(qkv, "qkv"); check_contig(q_out, "q_out");
  CHECK(hd == 64 || hd == 128 || hd == 256, "head_dim must be 64, 128 or 256");
  CHECK(qkv.size(1) == (nq + 2 * nkv) * hd, "qkv width");
  CHECK(cos_sin.size(1) == hd, "cos_sin width");
  CHECK(q_norm.has_value() == k_norm.has_value(), "q_norm/k_norm must both be given or both absent");
  msgl_qk_norm_rope_store(q_out.data_ptr(), qkv.data_ptr(), positions.data_ptr<int32_t>(),
                          cos_sin.data_ptr<float>(), opt_ptr(q_norm), opt_ptr(k_norm), eps,
                          k_cache.data_ptr(), v_cache.data_ptr(), out_loc.data_ptr<int32_t>(),
                          qkv.size(0), nq, nkv, hd, nkv * hd, k_cache.size(0), cos_sin.size(0), stream());
}

// values (optional, fp32 [rows]) receives each row's maximum; vocab < 0 means all columns
void argmax(at::Tensor out, at::Tensor logits, c10::optional<at::Tensor> values, int64_t vocab) {
  check_i32(out, "out"); check_cuda(logits, "logits");
  CHECK(logits.stride(-1) == 1, "logits rows must be contiguous");
  const bool f32 = logits.scalar_type() == at::kFloat;
  CHECK(f32 || logits.scalar_type() == at::kBFloat16, "logits must be fp32 or bf16");
  const int64_t v = vocab < 0 ? logits.size(1) : std::min<int64_t>(vocab, logits.size(1));
  float* vp = nullptr;
  if (values.has_value()) {
    check_cuda(*values, "values"); check_dtype(*values, at::kFloat, "values");
    CHECK(values->numel() >= logits.size(0), "values too short");
    vp = values->data_ptr<float>();
  }
  msgl_argmax(out.data_ptr<int32_t>(), vp, logits.data_ptr(), logits.size(0), v, logits.stride(0), f32, stream());
}

// col_ids: optional [rows, vocab] int32 token id per column; id_offset: token id of column 0
// otherwise; values: optional fp32 [rows] winning score (see msgl_sample)
void sample(at::Tensor out, at::Tensor logits, at::Tensor temperature, at::Tensor top_k, at::Tensor top_p,
            at::Tensor seed, at::Tensor step, c10::optional<at::Tensor> col_ids, int64_t id_offset,
            c10::optional<at::Tensor> values) {
  check_i32(out, "out"); check_cuda(logits, "logits");
  at::Tensor lf = logits.scalar_type() == at::kFloat ? logits : logits.to(at::kFloat);
  CHECK(lf.stride(-1) == 1, "logits rows must be contiguous");
  check_dtype(temperature, at::kFloat, "temperature"); check_dtype(top_p, at::kFloat, "top_p");
  check_dtype(top_k, at::kInt, "top_k"); check_dtype(seed, at::kLong, "seed"); check_dtype(step, at::kLong, "step");
  const int64_t rows = lf.size(0), vocab = lf.size(1);
  CHECK(out.numel() >= rows && temperature.numel() >= rows && top_k.numel() >= rows && top_p.numel() >= rows &&
            seed.numel() >= rows && step.numel() >= rows, "sampling parameters shorter than the batch");
  const int32_t* ids = nullptr;
  if (col_ids.has_value()) {
    check_i32(*col_ids, "col_ids"); check_contig(*col_ids, "col_ids");
    CHECK(col_ids->size(0) == rows && col_ids->size(1) == vocab, "col_ids must be [rows, vocab]");
    ids = col_ids->data_ptr<int32_t>();
  }
  float* vals = nullptr;
  if (values.has_value()) {
    check_cuda(*values, "values"); check_dtype(*values, at::kFloat, "values");
    CHECK(values->numel() >= rows, "values too short");
    vals = values->data_ptr<float>();
  }
  msgl_sample(out.data_ptr<int32_t>(), lf.data_ptr<float>(), rows, vocab, lf.stride(0),
              temperature.data_ptr<float>(), top_k.data_ptr<int32_t>(), top_p.data_ptr<float>(),
              seed.data_ptr<int64_t>(), step.data_ptr<int64_t>(), ids, (int)id_offset, vals, stream());
}

void attention_prefill(at::Tensor o, at::Tensor q, at::Tensor k_cache, at::Tensor v_cache, at::Tensor page_table,
                       at::Tensor rows, at::Tensor cu_q, at::Tensor kv_lens, int64_t max_q_len, double scale,
                       int64_t window, c10::optional<at::Tensor> sinks) {
  check_bf16(o, "o"); check_bf16(q, "q"); check_bf16(k_cache, "k_cache"); check_bf16(v_cache, "v_cache");
  check_i32(rows, "rows"); check_i32(cu_q, "cu_q"); check_i32(kv_lens, "kv_lens");
  check_cuda(page_table, "page_table"); check_dtype(page_table, at::kInt, "page_table");
  check_contig(q, "q"); check_contig(o, "o");
  const int nq = q.size(1), hd = q.size(2), nkv = k_cache.size(1);
  CHECK(hd == 64 || hd == 128, "attention head_dim must be 64 or 128");
  CHECK(nq % nkv == 0, "nq must be a multiple of nkv");
  if (sinks.has_value()) { check_dtype(*sinks, at::kFloat, "sinks"); CHECK(sinks->numel() == nq, "sinks size"); }
  msgl_attention_prefill(o.data_ptr(), q.data_ptr(), k_cache.data_ptr(), v_cache.data_ptr(),
                         page_table.data_ptr<int32_t>(), page_table.stride(0), rows.data_ptr<int32_t>(),
                         cu_q.data_ptr<int32_t>(), kv_lens.data_ptr<int32_t>(), rows.size(0), q.size(0),
                         max_q_len, nq, nkv, hd, k_cache.stride(0), k_cache.size(0), scale, window,
                         sinks.has_value() ? sinks->data_ptr<float>() : nullptr, stream());
}

void attention_decode(at::Tensor o, at::Tensor q, at::Tensor k_cache, at::Tensor v_cache, at::Tensor page_table,
                      at::Tensor rows, at::Tensor kv_lens, double scale, int64_t window,
                      c10::optional<at::Tensor> sinks, int64_t num_splits, at::Tensor workspace) {
  check_bf16(o, "o"); check_bf16(q, "q"); check_bf16(k_cache, "k_cache"); check_bf16(v_cache, "v_cache");
  check_i32(rows, "rows"); check_i32(kv_lens, "kv_lens");
  check_cuda(page_table, "page_table"); check_dtype(page_table, at::kInt, "page_table");
  check_contig(q, "q"); check_contig(o, "o");
  const int bs = q.size(0), nq = q.size(1), hd = q.size(2), nkv = k_cache.size(1);
  CHECK(hd == 64 || hd == 128, "attention head_dim must be 64 or 128");
  CHECK(nq % nkv == 0 && nq / nkv <= 16, "decode supports up to 16 query heads per KV head");
  CHECK(rows.size(0) >= bs && kv_lens.size(0) >= bs, "metadata too short");
  if (num_splits > 1)
    CHECK(workspace.numel() >= (int64_t)bs * nq * num_splits * (hd + 2) * 4, "decode workspace too small");
  if (sinks.has_value()) { check_dtype(*sinks, at::kFloat, "sinks"); CHECK(sinks->numel() == nq, "sinks size"); }
  msgl_attention_decode(o.data_ptr(), q.data_ptr(), k_cache.data_ptr(), v_cache.data_ptr(),
                        page_table.data_ptr<int32_t>(), page_table.stride(0), rows.data_ptr<int32_t>(),
                        kv_lens.data_ptr<int32_t>(), bs, nq, nkv, hd, k_cache.stride(0), k_cache.size(0), scale,
                        window, sinks.has_value() ? sinks->data_ptr<float>() : nullptr, num_splits,
                        workspace.data_ptr(), stream());
}

// tcgen05 prefill attention for head_dim 128 and page sizes 16/32/64 (pages of `page` consecutive slots).
void attention_prefill_fmha(at::Tensor o, at::Tensor q, at::Tensor k_cache, at::Tensor v_cache, at::Tensor page_table,
                            at::Tensor rows, at::Tensor cu_q, at::Tensor kv_lens, int64_t max_q_len, double scale,
                            int64_t window, c10::optional<at::Tensor> sinks, int64_t page) {
  check_bf16(o, "o"); check_bf16(q, "q"); check_bf16(k_cache, "k_cache"); check_bf16(v_cache, "v_cache");
  check_i32(rows, "rows"); check_i32(cu_q, "cu_q"); check_i32(kv_lens, "kv_lens");
  check_cuda(page_table, "page_table"); check_dtype(page_table, at::kInt, "page_table");
  check_contig(q, "q"); check_contig(o, "o");
  const int64_t T = q.size(0), nq = q.size(1), hd = q.size(2), nkv = k_cache.size(1);
  CHECK(hd == 128, "tcgen05 prefill attention needs head_dim 128");
  CHECK(nq % nkv == 0, "query heads must be a multiple of kv heads");
  CHECK(page == 16 || page == 32 || page == 64, "tcgen05 prefill attention needs a page size of 16, 32 or 64");
  CHECK(k_cache.stride(2) == 1 && k_cache.stride(1) == hd && k_cache.stride(0) % 8 == 0, "k_cache layout");
  CHECK(v_cache.strides() == k_cache.strides() && v_cache.sizes() == k_cache.sizes(), "v_cache layout");
  CHECK(reinterpret_cast<uintptr_t>(q.data_ptr()) % 16 == 0 && reinterpret_cast<uintptr_t>(k_cache.data_ptr()) % 16 == 0 &&
            reinterpret_cast<uintptr_t>(v_cache.data_ptr()) % 16 == 0, "attention tensors must be 16-byte aligned");
  if (sinks.has_value()) { check_dtype(*sinks, at::kFloat, "sinks"); CHECK(sinks->numel() == nq, "sinks size"); }
  const int rc = msgl_attention_prefill_fmha(
      o.data_ptr(), q.data_ptr(), T, k_cache.data_ptr(), v_cache.data_ptr(), k_cache.size(0), k_cache.stride(0),
      page_table.data_ptr<int32_t>(), page_table.stride(0), rows.data_ptr<int32_t>(), cu_q.data_ptr<int32_t>(),
      kv_lens.data_ptr<int32_t>(), cu_q.size(0) - 1, max_q_len, nq, nkv, hd, page, scale, window,
      sinks.has_value() ? sinks->data_ptr<float>() : nullptr, stream());
  CHECK(rc == 0, "tcgen05 prefill attention failed to launch (code ", rc, ")");
}

// Profiling: phase stamps of later prefill launches into trace (int32 [ctas, 96], kv head 0); None: off.
void attention_prefill_trace(c10::optional<at::Tensor> trace) {
  if (!trace.has_value()) {
    msgl_attention_prefill_trace(nullptr, 0);
    return;
  }
  check_i32(*trace, "trace");
  check_contig(*trace, "trace");
  CHECK(trace->dim() == 2 && trace->size(1) == 96, "trace must be [ctas, 96]");
  msgl_attention_prefill_trace(reinterpret_cast<uint32_t*>(trace->data_ptr<int32_t>()), (int)trace->size(0));
}

// Paged decode attention over a host-built work list (page size 16/32/64). work: int32 [>= 8 * entries]
// (two int4 per entry), n_work: int32 [1] = entries, ws: fp32 partials for ws_slots chunk slots,
// counters: int32 [>= bs * nkv], zero on entry and left at zero.
void attention_decode_paged(at::Tensor o, at::Tensor q, at::Tensor k_cache, at::Tensor v_cache, at::Tensor page_table,
                            at::Tensor rows, at::Tensor kv_lens, at::Tensor work, at::Tensor n_work, at::Tensor ws,
                            int64_t ws_slots, at::Tensor counters, double scale, int64_t window,
                            c10::optional<at::Tensor> sinks, int64_t page) {
  check_bf16(o, "o"); check_bf16(q, "q"); check_bf16(k_cache, "k_cache"); check_bf16(v_cache, "v_cache");
  check_i32(rows, "rows"); check_i32(kv_lens, "kv_lens"); check_i32(work, "work"); check_i32(n_work, "n_work");
  check_i32(counters, "counters");
  check_cuda(ws, "ws"); check_dtype(ws, at::kFloat, "ws");
  check_cuda(page_table, "page_table"); check_dtype(page_table, at::kInt, "page_table");
  check_contig(q, "q"); check_contig(o, "o"); check_contig(work, "work");
  const int64_t T = q.size(0), nq = q.size(1), hd = q.size(2), nkv = k_cache.size(1);
  CHECK(hd == 64 || hd == 128, "attention head_dim must be 64 or 128");
  CHECK(nq % nkv == 0 && nq / nkv <= 16, "decode supports up to 16 query heads per KV head");
  CHECK(page == 16 || page == 32 || page == 64, "paged decode needs a page size of 16, 32 or 64");
  CHECK(k_cache.stride(2) == 1 && k_cache.stride(1) == hd && k_cache.stride(0) % 8 == 0, "k_cache layout");
  CHECK(v_cache.strides() == k_cache.strides() && v_cache.sizes() == k_cache.sizes(), "v_cache layout");
  CHECK(reinterpret_cast<uintptr_t>(q.data_ptr()) % 16 == 0 && reinterpret_cast<uintptr_t>(k_cache.data_ptr()) % 16 == 0 &&
            reinterpret_cast<uintptr_t>(v_cache.data_ptr()) % 16 == 0, "attention tensors must be 16-byte aligned");
  CHECK(ws.numel() >= ws_slots * nkv * (nq / nkv) * (hd + 2), "decode partial workspace too small");
  if (sinks.has_value()) { check_dtype(*sinks, at::kFloat, "sinks"); CHECK(sinks->numel() == nq, "sinks size"); }
  const int rc = msgl_attention_decode_paged(
      o.data_ptr(), q.data_ptr(), (int)(T * nq), k_cache.data_ptr(), v_cache.data_ptr(), k_cache.size(0),
      k_cache.stride(0), page_table.data_ptr<int32_t>(), page_table.stride(0), rows.data_ptr<int32_t>(),
      kv_lens.data_ptr<int32_t>(), work.data_ptr<int32_t>(), n_work.data_ptr<int32_t>(), ws.data_ptr<float>(),
      (int)ws_slots, counters.data_ptr<int32_t>(), nq, nkv, hd, page, scale, window,
      sinks.has_value() ? sinks->data_ptr<float>() : nullptr, stream());
  CHECK(rc == 0, "paged decode attention failed to launch (code ", rc, ")");
}

// ----- routed experts
// epi 0: out [rows, N]; 1 / 2 / 4 (SiLU / GELU / gpt-oss SwiGLU): w's rows gate/up interleaved in
// 128-row blocks, out the activated [rows, N / 2]
void gemm_grouped(at::Tensor out, at::Tensor xs, at::Tensor w, c10::optional<at::Tensor> bias, at::Tensor tile_count,
                  at::Tensor work, int64_t bn, int64_t epi) {
  check_bf16(out, "out"); check_bf16(xs, "xs"); check_bf16(w, "w");
  check_contig(xs, "xs"); check_contig(w, "w"); check_contig(out, "out");
  check_i32(tile_count, "tile_count"); check_i32(work, "work");
  CHECK(w.dim() == 3, "expert weights must be [E, N, K]");
  CHECK(epi == 0 || epi == 1 || epi == 2 || epi == 4, "grouped gemm epilogue must be 0, 1, 2 or 4");
  const int64_t E = w.size(0), N = w.size(1), K = w.size(2);
  const int64_t n_out = epi == 0 ? N : N / 2;
  if (epi != 0) CHECK(N % 256 == 0, "gated grouped gemm needs 2I to be a multiple of 256");
  CHECK(xs.size(1) == K && out.size(1) == n_out && out.size(0) == xs.size(0), "grouped gemm shapes");
  CHECK(K % 8 == 0 && N % 8 == 0, "grouped gemm needs K, N multiples of 8");
  CHECK(bn == 16 || bn == 32 || bn == 64 || bn == 128, "bn must be 16/32/64/128");
  CHECK(xs.size(0) % bn == 0, "row capacity must be a multiple of bn");
  if (bias.has_value()) { check_bf16(*bias, "bias"); CHECK(bias->numel() == E * N, "bias must be [E, N]"); }
  const int max_tiles = work.numel() / 2;
  msgl_gemm_grouped(out.data_ptr(), xs.data_ptr(), w.data_ptr(), opt_ptr(bias), xs.size(0), N, K, out.stride(0), E,
                    tile_count.data_ptr<int32_t>(), work.data_ptr(), max_tiles, bn, (int)epi, stream());
}

// Grouped GEMM over MXFP4 experts: q uint8 [E, K/64, n_pad, 32] (e2m1 pairs), s uint8
// [E, K/64, n_pad, 2] (e8m0 scales), n = logical rows (gated: gate / up interleaved in 128-row blocks).
void gemm_grouped_fp4(at::Tensor out, at::Tensor xs, at::Tensor q, at::Tensor s, int64_t n,
                      c10::optional<at::Tensor> bias, at::Tensor tile_count, at::Tensor work, int64_t bn, int64_t epi) {
  check_bf16(out, "out"); check_bf16(xs, "xs");
  check_contig(xs, "xs"); check_contig(out, "out"); check_contig(q, "q"); check_contig(s, "s");
  check_cuda(q, "q"); check_cuda(s, "s");
  check_dtype(q, at::kByte, "q"); check_dtype(s, at::kByte, "s");
  check_i32(tile_count, "tile_count"); check_i32(work, "work");
  CHECK(q.dim() == 4 && q.size(3) == 32 && s.dim() == 4 && s.size(3) == 2, "fp4 experts must be [E, K/64, Np, 32|2]");
  CHECK(q.size(0) == s.size(0) && q.size(1) == s.size(1) && q.size(2) == s.size(2), "fp4 blocks / scales mismatch");
  CHECK(epi == 0 || epi == 1 || epi == 2 || epi == 4, "grouped gemm epilogue must be 0, 1, 2 or 4");
  const int64_t E = q.size(0), K = q.size(1) * 64, n_pad = q.size(2);
  const int64_t n_out = epi == 0 ? n : n / 2;
  CHECK(n <= n_pad && n_pad % 128 == 0, "fp4 rows padded to whole tiles");
  if (epi != 0) CHECK(n % 256 == 0 && n_pad == n, "gated grouped gemm needs 2I to be a multiple of 256");
  CHECK(xs.size(1) == K && out.size(1) == n_out && out.size(0) == xs.size(0), "grouped gemm shapes");
  CHECK(bn == 16 || bn == 32 || bn == 64 || bn == 128, "bn must be 16/32/64/128");
  CHECK(xs.size(0) % bn == 0, "row capacity must be a multiple of bn");
  if (bias.has_value()) { check_bf16(*bias, "bias"); CHECK(bias->numel() == E * n, "bias must be [E, N]"); }
  CHECK(reinterpret_cast<uintptr_t>(q.data_ptr()) % 16 == 0 && reinterpret_cast<uintptr_t>(s.data_ptr()) % 16 == 0,
        "fp4 experts must be 16-byte aligned");
  const int max_tiles = work.numel() / 2;
  const int rc = msgl_gemm_grouped_fp4(out.data_ptr(), xs.data_ptr(), q.data_ptr(), s.data_ptr(), opt_ptr(bias),
                                       xs.size(0), n, n_pad, K, out.stride(0), E, tile_count.data_ptr<int32_t>(),
                                       work.data_ptr(), max_tiles, bn, (int)epi, stream());
  CHECK(rc == 0, "fp4 grouped gemm: unsupported shape (code ", rc, ")");
}

void moe_route(at::Tensor logits, int64_t topk, bool renorm, bool softmax_after, at::Tensor weights, at::Tensor ids) {
  check_cuda(logits, "logits"); check_dtype(logits, at::kFloat, "logits"); check_contig(logits, "logits");
  check_dtype(weights, at::kFloat, "weights"); check_i32(ids, "ids");
  CHECK(logits.size(1) <= 512 && topk <= 16 && topk <= logits.size(1), "route: E <= 512, topk <= 16");
  msgl_moe_route(logits.data_ptr<float>(), logits.size(0), logits.size(1), topk, renorm, softmax_after,
                 weights.data_ptr<float>(), ids.data_ptr<int32_t>(), stream());
}

void moe_align(at::Tensor ids, int64_t E, int64_t bn, at::Tensor perm, at::Tensor inv, at::Tensor work,
               at::Tensor tile_count, int64_t e0) {
  check_i32(ids, "ids"); check_i32(perm, "perm"); check_i32(inv, "inv"); check_i32(work, "work");
  check_i32(tile_count, "tile_count");
  CHECK(E <= 4096, "too many experts");
  msgl_moe_align(ids.data_ptr<int32_t>(), ids.numel(), E, e0, bn, work.numel() / 2, perm.numel(), perm.data_ptr<int32_t>(),
                 inv.data_ptr<int32_t>(), work.data_ptr(), tile_count.data_ptr<int32_t>(), stream());
}

void moe_gather(at::Tensor xs, at::Tensor x, at::Tensor perm, int64_t topk) {
  check_bf16(xs, "xs"); check_bf16(x, "x"); check_i32(perm, "perm"); check_contig(x, "x"); check_contig(xs, "xs");
  CHECK(x.size(1) % 8 == 0 && xs.size(1) == x.size(1), "gather shapes");
  msgl_moe_gather(xs.data_ptr(), x.data_ptr(), perm.data_ptr<int32_t>(), xs.size(0), x.size(1), topk, x.size(0),
                  stream());
}

void moe_act(at::Tensor out, at::Tensor y, int64_t act, at::Tensor perm) {
  check_bf16(out, "out"); check_bf16(y, "y"); check_i32(perm, "perm");
  CHECK(y.size(1) == 2 * out.size(1) && y.size(0) == out.size(0), "act shapes");
  msgl_moe_act(out.data_ptr(), y.data_ptr(), out.size(0), out.size(1), act, perm.data_ptr<int32_t>(), stream());
}

void moe_combine(at::Tensor out, at::Tensor y, at::Tensor w, at::Tensor inv, int64_t topk) {
  check_bf16(out, "out"); check_bf16(y, "y"); check_dtype(w, at::kFloat, "w"); check_i32(inv, "inv");
  CHECK(out.size(1) % 2 == 0 && y.size(1) == out.size(1), "combine shapes");
  msgl_moe_combine(out.data_ptr(), y.data_ptr(), w.data_ptr<float>(), inv.data_ptr<int32_t>(), out.size(0),
                   out.size(1), topk, y.size(0), stream());
}

// ----- peer-memory collectives
int64_t peer_alloc(int64_t bytes) {
  void* p = msgl_peer_alloc(bytes);
  CHECK(p != nullptr, "peer buffer allocation of ", bytes, " bytes failed");
  return reinterpret_cast<int64_t>(p);
}
void peer_free(int64_t p) { msgl_peer_free(reinterpret_cast<void*>(p)); }
py::bytes ipc_handle(int64_t p) {
  char buf[64];
  const int rc = msgl_ipc_handle(reinterpret_cast<void*>(p), buf);
  CHECK(rc == 0, "cudaIpcGetMemHandle failed (", rc, ")");
  return py::bytes(buf, 64);
}
int64_t ipc_open(py::bytes h) {
  std::string s = h;
  CHECK(s.size() == 64, "bad IPC handle");
  void* p = msgl_ipc_open(s.data());
  CHECK(p != nullptr, "cudaIpcOpenMemHandle failed");
  return reinterpret_cast<int64_t>(p);
}
void ipc_close(int64_t p) { msgl_ipc_close(reinterpret_cast<void*>(p)); }

void peer_collective(int64_t mode, at::Tensor out, at::Tensor in, std::vector<int64_t> bases, int64_t rank,
                     int64_t cap_bytes, at::Tensor state, int64_t timeout_ns) {
  check_cuda(out, "out"); check_cuda(in, "in"); check_contig(out, "out"); check_contig(in, "in");
  check_cuda(state, "state"); check_dtype(state, at::kInt, "state");
  CHECK(state.numel() >= 2 * msgl_peer_grid(), "peer state tensor too small");
  const int64_t bytes = in.numel() * in.element_size();
  CHECK(bytes % 16 == 0, "peer collectives need a multiple of 16 bytes");
  CHECK(bytes <= cap_bytes, "message of ", bytes, " bytes exceeds the peer buffer (", cap_bytes, ")");
  CHECK(bases.size() >= 1 && bases.size() <= 8, "1..8 ranks supported");
  std::vector<void*> b;
  for (auto v : bases) b.push_back(reinterpret_cast<void*>(v));
  if (mode == 2) {
    CHECK(out.numel() * out.element_size() == bytes * (int64_t)b.size(), "all-gather output size");
  } else {
    check_dtype(in, at::kBFloat16, "in");
    CHECK(out.numel() == in.numel(), "all-reduce output size");
  }
  msgl_peer_collective(b.data(), rank, b.size(), mode, out.data_ptr(), in.data_ptr(), bytes, cap_bytes,
                       reinterpret_cast<uint32_t*>(state.data_ptr()), timeout_ns, stream());
}

// NVLS all-reduce + residual add + RMSNorm over a multicast-bound symmetric buffer (uc/mc: this
// rank's and the multicast address of the same allocation).
void nvls_allreduce_rmsnorm(int64_t uc, int64_t mc, int64_t rank, int64_t world, at::Tensor x, at::Tensor residual, at::Tensor w,
                            at::Tensor out, double eps, int64_t cap_bytes, at::Tensor state, int64_t timeout_ns,
                            bool first, int64_t mode, c10::optional<at::Tensor> trace) {
  check_bf16(x, "x"); check_bf16(residual, "residual"); check_bf16(w, "w"); check_bf16(out, "out");
  check_contig(x, "x"); check_contig(residual, "residual"); check_contig(out, "out"); check_contig(w, "w");
  check_cuda(state, "state"); check_dtype(state, at::kInt, "state");
  CHECK(state.numel() >= msgl_nvls_state_words(), "nvls state tensor too small");
  if (trace.has_value()) {
    check_cuda(*trace, "trace"); check_dtype(*trace, at::kLong, "trace");
    CHECK(trace->numel() >= 8 * msgl_nvls_grid(), "nvls trace tensor too small");
  }
  const int64_t H = x.size(-1), T = x.numel() / H;
  CHECK(residual.numel() == x.numel() && out.numel() == x.numel() && w.numel() == H, "nvls norm shapes");
  const int rc = msgl_nvls_allreduce_rmsnorm(reinterpret_cast<void*>(uc), reinterpret_cast<void*>(mc), rank, world,
                                             x.data_ptr(), residual.data_ptr(), w.data_ptr(), out.data_ptr(), T, H,
                                             eps, cap_bytes, reinterpret_cast<uint32_t*>(state.data_ptr()),
                                             timeout_ns, first ? 1 : 0, (int)mode,
                                             trace.has_value() ? reinterpret_cast<uint64_t*>(trace->data_ptr()) : nullptr,
                                             stream());
  CHECK(rc == 0, "nvls all-reduce rejected its arguments (code ", rc, ")");
}

void plan_apply(at::Tensor page_table, at::Tensor pt_rows, at::Tensor pt_pos, at::Tensor pt_slots, at::Tensor tok_rows,
                at::Tensor positions, at::Tensor out_loc) {
  for (auto* t : {&page_table, &pt_rows, &pt_pos, &pt_slots, &tok_rows, &positions, &out_loc}) {
    check_cuda(*t, "plan tensor"); check_dtype(*t, at::kInt, "plan tensor"); check_contig(*t, "plan tensor");
  }
  CHECK(page_table.dim() == 2, "page table must be 2-D");
  CHECK(pt_rows.numel() == pt_pos.numel() && pt_rows.numel() == pt_slots.numel(), "page-table write lists");
  CHECK(tok_rows.numel() == positions.numel() && out_loc.numel() == positions.numel(), "token lists");
  msgl_plan_apply(page_table.data_ptr<int32_t>(), page_table.stride(0), page_table.size(0), pt_rows.data_ptr<int32_t>(),
                  pt_pos.data_ptr<int32_t>(), pt_slots.data_ptr<int32_t>(), (int)pt_rows.numel(),
                  tok_rows.data_ptr<int32_t>(), positions.data_ptr<int32_t>(), (int)positions.numel(),
                  out_loc.data_ptr<int32_t>(), stream());
}

void gather_i32(at::Tensor dst, at::Tensor src, at::Tensor idx) {
  for (auto* t : {&dst, &src, &idx}) {
    check_cuda(*t, "gather tensor"); check_dtype(*t, at::kInt, "gather tensor"); check_contig(*t, "gather tensor");
  }
  CHECK(dst.numel() == idx.numel(), "gather sizes");
  msgl_gather_i32(dst.data_ptr<int32_t>(), src.data_ptr<int32_t>(), src.numel(), idx.data_ptr<int32_t>(),
                  (int)idx.numel(), stream());
}

void scatter_i32(at::Tensor dst, at::Tensor idx, at::Tensor src) {
  for (auto* t : {&dst, &src, &idx}) {
    check_cuda(*t, "scatter tensor"); check_dtype(*t, at::kInt, "scatter tensor"); check_contig(*t, "scatter tensor");
  }
  CHECK(src.numel() == idx.numel(), "scatter sizes");
  msgl_scatter_i32(dst.data_ptr<int32_t>(), dst.numel(), idx.data_ptr<int32_t>(), src.data_ptr<int32_t>(),
                   (int)idx.numel(), stream());
}

std::tuple<int64_t, int64_t> get_error() {
  int info = 0;
  const int code = msgl_get_error(&info);
  return {code, info};
}

}  // namespace

PYBIND11_MODULE(TORCH_EXTENSION_NAME, m) {
  m.doc() = "minisgl sm_100a kernels";
  m.def("embedding", &embedding);
  m.def("rmsnorm", &rmsnorm);
  m.def("fused_add_rmsnorm", &fused_add_rmsnorm);
  m.def("gemm", &gemm);
  m.def("attention_decode_paged", &attention_decode_paged);
  m.def("attention_prefill_fmha", &attention_prefill_fmha);
  m.def("attention_prefill_trace", &attention_prefill_trace);
  m.def("gemm_grouped_fp4", &gemm_grouped_fp4);
  m.def("gemm_ex", &gemm_ex);
  m.def("act_and_mul", &act_and_mul);
  m.def("store_kv", &store_kv);
  m.def("qk_norm_rope_store", &qk_norm_rope_store);
  m.def("argmax", &argmax, py::arg("out"), py::arg("logits"), py::arg("values") = py::none(),
        py::arg("vocab") = -1);
  m.def("sample", &sample, py::arg("out"), py::arg("logits"), py::arg("temperature"), py::arg("top_k"),
        py::arg("top_p"), py::arg("seed"), py::arg("step"), py::arg("col_ids") = py::none(),
        py::arg("id_offset") = 0, py::arg("values") = py::none());
  m.def("attention_prefill", &attention_prefill);
  m.def("attention_decode", &attention_decode);
  m.def("get_error", &get_error);
  m.def("gemm_grouped", &gemm_grouped);

  m.def("moe_route", &moe_route);
  m.def("moe_align", &moe_align, py::arg("ids"), py::arg("E"), py::arg("bn"), py::arg("perm"), py::arg("inv"),
        py::arg("work"), py::arg("tile_count"), py::arg("e0") = 0);
  m.def("moe_gather", &moe_gather);
  m.def("moe_act", &moe_act);
  m.def("moe_combine", &moe_combine);
  m.def("peer_flag_bytes", []() { return msgl_peer_flag_bytes(); });
  m.def("peer_alloc", &peer_alloc);
  m.def("peer_free", &peer_free);
  m.def("ipc_handle", &ipc_handle);
  m.def("ipc_open", &ipc_open);
  m.def("ipc_close", &ipc_close);
  m.def("peer_grid", []() { return msgl_peer_grid(); });
  m.def("peer_collective", &peer_collective);
  m.def("nvls_grid", []() { return msgl_nvls_grid(); });
  m.def("nvls_flag_bytes", []() { return msgl_nvls_flag_bytes(); });
  m.def("nvls_state_words", []() { return msgl_nvls_state_words(); });
  m.def("nvls_ticket_offset", []() { return msgl_nvls_ticket_offset(); });
  m.def("gemm_signal", &gemm_signal);
  m.def("lm_head_argmax", &lm_head_argmax);
  m.def("plan_apply", &plan_apply);
  m.def("gather_i32", &gather_i32);
  m.def("scatter_i32", &scatter_i32);
  m.def("nvls_allreduce_rmsnorm", &nvls_allreduce_rmsnorm);
  m.def("num_sms", []() { return msgl_num_sms(); });
  m.def("gemm_splits", [](int64_t M, int64_t N, int64_t K) { return msgl_gemm_pick_splits(M, N, K); });
  m.def("gemm_force_bn", [](int64_t bn) { msgl_gemm_force_bn((int)bn); });
}
