// Python bindings of the sm_100a kernels: tensor validation, then a launch on
// the current CUDA stream (so every op is capturable in a CUDA graph).
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/extension.h>

#include "host/recall_dispatch.h"
#include "kernels/launchers.h"

namespace {

using torch::Tensor;

#define CHECK_CUDA(t) TORCH_CHECK((t).is_cuda(), #t " must be a CUDA tensor")
#define CHECK_DTYPE(t, d) TORCH_CHECK((t).scalar_type() == (d), #t " has dtype ", (t).scalar_type(), ", expected ", (d))
#define CHECK_LAST_CONTIG(t) TORCH_CHECK((t).stride(-1) == 1, #t " must be contiguous in its last dimension")

cudaStream_t stream() { return at::cuda::getCurrentCUDAStream().stream(); }

// One int32 error word per device, zero-initialised; kernels record the first
// failure (bounded-wait timeout, bad index) here instead of trapping.
Tensor& error_word_ref(int device) {
  static std::vector<Tensor> words(64);
  if (!words[device].defined()) {
    c10::cuda::CUDAGuard g(device);
    words[device] = torch::zeros({1}, torch::dtype(torch::kInt32).device(torch::kCUDA, device));
  }
  return words[device];
}
int* err_ptr(const Tensor& like) { return error_word_ref(like.get_device()).data_ptr<int>(); }

Tensor error_word(int64_t device) { return error_word_ref(int(device)); }

template <typename T>
T* ptr(const Tensor& t) { return reinterpret_cast<T*>(t.data_ptr()); }
template <typename T>
const T* cptr(const Tensor& t) { return reinterpret_cast<const T*>(t.data_ptr()); }

// ------------------------------------------------------------------ GEMMs
void fp8_gemm(const Tensor& a_q, const Tensor& a_s_t, const Tensor& w, const Tensor& w_s, Tensor& out,
              const c10::optional<Tensor>& residual, bool ue8m0) {
  CHECK_CUDA(a_q); CHECK_CUDA(w); CHECK_CUDA(out);
  CHECK_DTYPE(a_q, torch::kFloat8_e4m3fn); CHECK_DTYPE(w, torch::kFloat8_e4m3fn);
  CHECK_DTYPE(a_s_t, torch::kFloat32); CHECK_DTYPE(w_s, torch::kFloat32); CHECK_DTYPE(out, torch::kBFloat16);
  TORCH_CHECK(a_q.dim() == 2 && w.dim() == 2 && a_q.size(1) == w.size(1), "fp8_gemm: [M,K] x [N,K]");
  CHECK_LAST_CONTIG(a_q); CHECK_LAST_CONTIG(w); CHECK_LAST_CONTIG(out);
  TORCH_CHECK(w_s.is_contiguous() && a_s_t.stride(1) == 1, "fp8_gemm: scale layouts");
  const int M = a_q.size(0), N = w.size(0), K = a_q.size(1);
  TORCH_CHECK(out.size(0) == M && out.size(1) == N, "fp8_gemm: out shape");
  TORCH_CHECK(a_s_t.size(0) == (K + 127) / 128 && a_s_t.size(1) >= M, "fp8_gemm: activation scales [K/128, >=M]");
  TORCH_CHECK(w_s.size(0) == (N + 127) / 128 && w_s.size(1) == (K + 127) / 128, "fp8_gemm: weight scales");
  c10::cuda::CUDAGuard g(a_q.device());
  b200::FP8GemmArgs a{};
  a.A = cptr<uint8_t>(a_q); a.B = cptr<uint8_t>(w); a.sfa = cptr<float>(a_s_t); a.sfb = cptr<float>(w_s);
  a.out = ptr<__nv_bfloat16>(out);
  a.residual = nullptr; a.ldr = 0;
  if (residual && residual->defined()) {
    CHECK_DTYPE((*residual), torch::kBFloat16);
    TORCH_CHECK(residual->size(0) == M && residual->size(1) == N && residual->stride(1) == 1, "fp8_gemm: residual");
    a.residual = cptr<__nv_bfloat16>(*residual); a.ldr = residual->stride(0);
  }
  a.M = M; a.N = N; a.K = K; a.lda = a_q.stride(0); a.ldb = w.stride(0);
  a.lda_s = a_s_t.stride(0); a.ldo = out.stride(0); a.err = err_ptr(a_q);
  a.ue8m0 = ue8m0;
  // Split-K scratch for GEMMs whose tile count leaves SMs idle.
  constexpr int kMaxSplits = 8;
  const size_t scratch = b200::fp8_gemm_scratch_bytes(M, N, K, kMaxSplits);
  Tensor part;
  if (scratch) {
    part = torch::empty({int64_t(scratch / 4)}, torch::dtype(torch::kFloat32).device(a_q.device()));
    a.partial = part.data_ptr<float>();
    a.max_splits = kMaxSplits;
  }
  b200::launch_fp8_gemm(a, stream());
}

// out_g[m, n] = sum_k A_g[m, k] * B_g[n, k]; strides in elements.
void bf16_gemm(const Tensor& A, int64_t a_off, int64_t lda, int64_t a_batch, const Tensor& B, int64_t b_off,
               int64_t ldb, int64_t b_batch, Tensor& out, int64_t o_off, int64_t ldo, int64_t o_batch,
               int64_t M, int64_t N, int64_t K, int64_t batch) {
  CHECK_CUDA(A); CHECK_CUDA(B); CHECK_CUDA(out);
  CHECK_DTYPE(A, torch::kBFloat16); CHECK_DTYPE(B, torch::kBFloat16);
  TORCH_CHECK(out.scalar_type() == torch::kBFloat16 || out.scalar_type() == torch::kFloat32, "bf16_gemm: out dtype");
  auto span_ok = [](const Tensor& t, int64_t off, int64_t rows, int64_t ld, int64_t bs, int64_t nb, int64_t cols) {
    const int64_t last = off + (nb - 1) * bs + (rows - 1) * ld + cols;
    return off >= 0 && last <= t.numel() && t.is_contiguous();
  };
  TORCH_CHECK(span_ok(A, a_off, M, lda, a_batch, batch, K), "bf16_gemm: A view out of bounds");
  TORCH_CHECK(span_ok(B, b_off, N, ldb, b_batch, batch, K), "bf16_gemm: B view out of bounds");
  TORCH_CHECK(span_ok(out, o_off, M, ldo, o_batch, batch, N), "bf16_gemm: out view out of bounds");
  c10::cuda::CUDAGuard g(A.device());
  b200::BF16GemmArgs a{};
  a.A = cptr<__nv_bfloat16>(A) + a_off; a.B = cptr<__nv_bfloat16>(B) + b_off;
  const bool f32 = out.scalar_type() == torch::kFloat32;
  a.out = f32 ? static_cast<void*>(ptr<float>(out) + o_off) : static_cast<void*>(ptr<__nv_bfloat16>(out) + o_off);
  a.out_fp32 = f32; a.M = M; a.N = N; a.K = K; a.batch = batch;
  a.lda = lda; a.a_batch = a_batch; a.ldb = ldb; a.b_batch = b_batch; a.ldo = ldo; a.o_batch = o_batch;
  a.err = err_ptr(A);
  b200::launch_bf16_gemm(a, stream());
}

// ------------------------------------------------------------- elementwise
void rms_norm(const Tensor& x, const c10::optional<Tensor>& residual, const Tensor& weight, double eps,
              const c10::optional<Tensor>& out, const c10::optional<Tensor>& out_sum,
              const c10::optional<Tensor>& q, const c10::optional<Tensor>& sfa_t) {
  CHECK_CUDA(x); CHECK_DTYPE(x, torch::kBFloat16); CHECK_DTYPE(weight, torch::kFloat32);
  CHECK_LAST_CONTIG(x);
  TORCH_CHECK(x.dim() == 2 && weight.numel() == x.size(1) && weight.is_contiguous(), "rms_norm shapes");
  c10::cuda::CUDAGuard g(x.device());
  b200::NormArgs a{};
  a.x = cptr<__nv_bfloat16>(x); a.ldx = x.stride(0); a.weight = cptr<float>(weight);
  a.rows = x.size(0); a.D = x.size(1); a.eps = float(eps);
  if (residual && residual->defined()) {
    TORCH_CHECK(out_sum && out_sum->defined(), "rms_norm: residual needs out_sum");
    a.residual = cptr<__nv_bfloat16>(*residual); a.ldr = residual->stride(0);
    a.out_sum = ptr<__nv_bfloat16>(*out_sum); a.lds = out_sum->stride(0);
  }
  if (out && out->defined()) { a.out = ptr<__nv_bfloat16>(*out); a.ldo = out->stride(0); }
  if (q && q->defined()) {
    CHECK_DTYPE((*q), torch::kFloat8_e4m3fn);
    TORCH_CHECK(sfa_t && sfa_t->defined() && sfa_t->size(0) == x.size(1) / 128 && sfa_t->size(1) >= x.size(0), "rms_norm: sfa_t");
    a.q = ptr<uint8_t>(*q); a.ldq = q->stride(0); a.sfa_t = ptr<float>(*sfa_t); a.lda_s = sfa_t->stride(0);
  }
  b200::launch_rms_norm(a, stream());
}

void quant_act(const Tensor& x, Tensor& q, Tensor& sfa_t) {
  CHECK_CUDA(x); CHECK_DTYPE(x, torch::kBFloat16); CHECK_DTYPE(q, torch::kFloat8_e4m3fn); CHECK_DTYPE(sfa_t, torch::kFloat32);
  CHECK_LAST_CONTIG(x); CHECK_LAST_CONTIG(q);
  TORCH_CHECK(sfa_t.size(0) == x.size(1) / 128 && sfa_t.size(1) >= x.size(0) && sfa_t.stride(1) == 1, "quant_act: sfa_t");
  c10::cuda::CUDAGuard g(x.device());
  b200::launch_quant_act(cptr<__nv_bfloat16>(x), x.stride(0), x.size(0), x.size(1), ptr<uint8_t>(q), q.stride(0),
                         ptr<float>(sfa_t), sfa_t.stride(0), stream());
}

void silu_mul_quant(const Tensor& packed, const c10::optional<Tensor>& h, const c10::optional<Tensor>& q,
                    const c10::optional<Tensor>& sfa_t) {
  CHECK_CUDA(packed); CHECK_DTYPE(packed, torch::kBFloat16); CHECK_LAST_CONTIG(packed);
  const int rows = packed.size(0), I = packed.size(1) / 2;
  c10::cuda::CUDAGuard g(packed.device());
  __nv_bfloat16* hp = nullptr;
  if (h && h->defined()) { TORCH_CHECK(h->is_contiguous() && h->size(1) == I, "silu: h"); hp = ptr<__nv_bfloat16>(*h); }
  uint8_t* qp = nullptr; float* sp = nullptr; int lda_s = 0;
  if (q && q->defined()) {
    TORCH_CHECK(q->is_contiguous() && q->size(1) == I && sfa_t && sfa_t->defined(), "silu: q");
    qp = ptr<uint8_t>(*q); sp = ptr<float>(*sfa_t); lda_s = sfa_t->stride(0);
  }
  b200::launch_silu_mul_quant(cptr<__nv_bfloat16>(packed), packed.stride(0), rows, I, hp, qp, sp, lda_s, stream());
}

void mla_q_rope(const Tensor& q, int64_t ldq, int64_t T, int64_t H, int64_t nope, int64_t rope, const Tensor& freqs,
                const Tensor& positions, Tensor& out, int64_t ldo_tok, int64_t ldo_head, int64_t out_offset) {
  CHECK_CUDA(q); CHECK_DTYPE(q, torch::kBFloat16); CHECK_DTYPE(out, torch::kBFloat16);
  c10::cuda::CUDAGuard g(q.device());
  b200::launch_mla_q_rope(cptr<__nv_bfloat16>(q), ldq, T, H, nope, rope, cptr<float>(freqs), cptr<float>(positions),
                          ptr<__nv_bfloat16>(out), ldo_tok, ldo_head, out_offset, stream());
}

void kv_finish(const Tensor& kv, int64_t L, int64_t R, const Tensor& norm_w, double eps, const Tensor& freqs,
               const Tensor& positions, Tensor& out, const c10::optional<Tensor>& dst_row,
               const c10::optional<Tensor>& packed) {
  CHECK_CUDA(kv); CHECK_DTYPE(kv, torch::kBFloat16); CHECK_DTYPE(out, torch::kBFloat16); CHECK_LAST_CONTIG(kv);
  c10::cuda::CUDAGuard g(kv.device());
  const int64_t* dr = nullptr;
  if (dst_row && dst_row->defined()) { CHECK_DTYPE((*dst_row), torch::kInt64); dr = cptr<int64_t>(*dst_row); }
  uint8_t* pk = nullptr;
  if (packed && packed->defined()) {
    CHECK_DTYPE((*packed), torch::kUInt8);
    TORCH_CHECK(packed->is_contiguous() && packed->dim() == 2 && packed->size(1) == 656 && packed->size(0) >= kv.size(0),
                "kv_finish: packed records [>= T, 656] uint8");
    pk = ptr<uint8_t>(*packed);
  }
  b200::launch_kv_finish(cptr<__nv_bfloat16>(kv), kv.stride(0), kv.size(0), L, R, cptr<float>(norm_w), float(eps),
                         cptr<float>(freqs), cptr<float>(positions), ptr<__nv_bfloat16>(out), out.stride(0), dr,
                         out.size(0), err_ptr(kv), stream(), pk);
}

// records[slots[i]] = dequant(packed[i]) for i < min(n, device_count).
void dequant_kv_rows(const Tensor& packed, Tensor& records, const c10::optional<Tensor>& slots, int64_t n,
                     const c10::optional<Tensor>& device_count) {
  CHECK_CUDA(packed); CHECK_DTYPE(packed, torch::kUInt8); CHECK_DTYPE(records, torch::kBFloat16);
  TORCH_CHECK(packed.is_contiguous() && packed.size(1) == 656 && packed.size(0) >= n, "dequant_kv_rows: packed [n, 656]");
  TORCH_CHECK(records.is_contiguous() && records.size(1) == 576, "dequant_kv_rows: records [*, 576]");
  c10::cuda::CUDAGuard g(packed.device());
  const int64_t* sl = nullptr;
  if (slots && slots->defined()) { CHECK_DTYPE((*slots), torch::kInt64); sl = cptr<int64_t>(*slots); }
  b200::launch_dequant_kv_rows(cptr<uint8_t>(packed), ptr<__nv_bfloat16>(records), sl, int(n),
                               (device_count && device_count->defined()) ? cptr<int>(*device_count) : nullptr,
                               records.size(0), err_ptr(records), stream());
}

void index_k(const Tensor& k, int64_t R, const Tensor& ln_w, const Tensor& ln_b, double eps, const Tensor& freqs,
             const Tensor& positions, Tensor& k_q, Tensor& k_scale) {
  CHECK_CUDA(k); CHECK_DTYPE(k, torch::kBFloat16); CHECK_DTYPE(k_q, torch::kFloat8_e4m3fn); CHECK_LAST_CONTIG(k);
  c10::cuda::CUDAGuard g(k.device());
  b200::launch_index_k(cptr<__nv_bfloat16>(k), k.stride(0), k.size(0), k.size(1), R, cptr<float>(ln_w), cptr<float>(ln_b),
                       float(eps), cptr<float>(freqs), cptr<float>(positions), ptr<uint8_t>(k_q), ptr<float>(k_scale), stream());
}

// kv_finish(kv, ...) and index_k(k, ...) of one chunk in one launch.
void kv_finish_index_k(const Tensor& kv, int64_t L, int64_t R, const Tensor& norm_w, double eps, Tensor& out,
                       const Tensor& dst_row, const c10::optional<Tensor>& packed, const Tensor& k, int64_t RK,
                       const Tensor& ln_w, const Tensor& ln_b, double ln_eps, Tensor& k_q, Tensor& k_scale,
                       const Tensor& freqs, const Tensor& positions) {
  CHECK_CUDA(kv); CHECK_DTYPE(kv, torch::kBFloat16); CHECK_DTYPE(out, torch::kBFloat16); CHECK_LAST_CONTIG(kv);
  CHECK_DTYPE(k, torch::kBFloat16); CHECK_DTYPE(k_q, torch::kFloat8_e4m3fn); CHECK_LAST_CONTIG(k);
  CHECK_DTYPE(dst_row, torch::kInt64);
  TORCH_CHECK(k.size(0) == kv.size(0), "kv_finish_index_k: kv and k rows differ");
  c10::cuda::CUDAGuard g(kv.device());
  uint8_t* pk = nullptr;
  if (packed && packed->defined()) {
    CHECK_DTYPE((*packed), torch::kUInt8);
    TORCH_CHECK(packed->is_contiguous() && packed->dim() == 2 && packed->size(1) == 656 && packed->size(0) >= kv.size(0),
                "kv_finish: packed records [>= T, 656] uint8");
    pk = ptr<uint8_t>(*packed);
  }
  b200::launch_kv_finish_index_k(cptr<__nv_bfloat16>(kv), kv.stride(0), kv.size(0), L, R, cptr<float>(norm_w),
                                 float(eps), ptr<__nv_bfloat16>(out), out.stride(0), cptr<int64_t>(dst_row),
                                 out.size(0), err_ptr(kv), pk, cptr<__nv_bfloat16>(k), k.stride(0), k.size(1), RK,
                                 cptr<float>(ln_w), cptr<float>(ln_b), float(ln_eps), ptr<uint8_t>(k_q),
                                 ptr<float>(k_scale), cptr<float>(freqs), cptr<float>(positions), stream());
}

void index_q(const Tensor& q, int64_t ldq, int64_t T, int64_t H, int64_t D, int64_t R, const Tensor& freqs,
             const Tensor& positions, Tensor& q_q, Tensor& q_scale, const Tensor& w_raw, double head_scale,
             Tensor& weights) {
  CHECK_CUDA(q); CHECK_DTYPE(q, torch::kBFloat16); CHECK_DTYPE(q_q, torch::kFloat8_e4m3fn);
  c10::cuda::CUDAGuard g(q.device());
  TORCH_CHECK(w_raw.is_contiguous() && (w_raw.size(-1) == H || w_raw.size(-1) == 2 * H), "index_q: w_raw");
  b200::launch_index_q(cptr<__nv_bfloat16>(q), ldq, T, H, D, R, cptr<float>(freqs), cptr<float>(positions),
                       ptr<uint8_t>(q_q), ptr<float>(q_scale), cptr<float>(w_raw), w_raw.size(-1) == 2 * H ? 1 : 0,
                       float(head_scale), ptr<float>(weights), stream());
}

// mla_q_rope(q, ...) and index_q(iq, ...) of one chunk in one launch.
void q_rope_index_q(const Tensor& q, int64_t ldq, int64_t T, int64_t H, int64_t nope, int64_t rope, Tensor& out,
                    int64_t ldo_tok, int64_t ldo_head, int64_t out_offset, const Tensor& iq, int64_t ldiq,
                    int64_t IH, int64_t D, int64_t R, Tensor& q_q, Tensor& q_scale, const Tensor& w_raw,
                    double head_scale, Tensor& weights, const Tensor& freqs, const Tensor& positions) {
  CHECK_CUDA(q); CHECK_DTYPE(q, torch::kBFloat16); CHECK_DTYPE(out, torch::kBFloat16);
  CHECK_DTYPE(iq, torch::kBFloat16); CHECK_DTYPE(q_q, torch::kFloat8_e4m3fn);
  c10::cuda::CUDAGuard g(q.device());
  TORCH_CHECK(w_raw.is_contiguous() && (w_raw.size(-1) == IH || w_raw.size(-1) == 2 * IH), "q_rope_index_q: w_raw");
  b200::launch_q_rope_index_q(cptr<__nv_bfloat16>(q), ldq, T, H, nope, rope, ptr<__nv_bfloat16>(out), ldo_tok,
                              ldo_head, out_offset, cptr<__nv_bfloat16>(iq), ldiq, IH, D, R, ptr<uint8_t>(q_q),
                              ptr<float>(q_scale), cptr<float>(w_raw), w_raw.size(-1) == 2 * IH ? 1 : 0,
                              float(head_scale), ptr<float>(weights), cptr<float>(freqs), cptr<float>(positions),
                              stream());
}

void linear_f32(const Tensor& x, const Tensor& W, Tensor& out) {
  CHECK_CUDA(x); CHECK_DTYPE(x, torch::kBFloat16); CHECK_DTYPE(W, torch::kFloat32); CHECK_DTYPE(out, torch::kFloat32);
  CHECK_LAST_CONTIG(x); TORCH_CHECK(W.is_contiguous() && out.is_contiguous(), "linear_f32 layout");
  c10::cuda::CUDAGuard g(x.device());
  b200::launch_linear_f32(cptr<__nv_bfloat16>(x), x.stride(0), cptr<float>(W), x.size(0), W.size(0), W.size(1),
                          ptr<float>(out), stream());
}

void l2_prefetch(const Tensor& t, int64_t bytes) {
  CHECK_CUDA(t);
  TORCH_CHECK(t.is_contiguous(), "l2_prefetch: contiguous tensor");
  const int64_t total = t.numel() * t.element_size();
  const int64_t n = bytes < 0 ? total : std::min(bytes, total);
  c10::cuda::CUDAGuard g(t.device());
  b200::launch_l2_prefetch(t.data_ptr(), n / 16 * 16, stream());
}

void embed(const Tensor& ids, const Tensor& table, Tensor& out, int64_t row0, int64_t vocab_total) {
  CHECK_CUDA(ids); CHECK_DTYPE(ids, torch::kInt64); CHECK_DTYPE(table, torch::kBFloat16); CHECK_DTYPE(out, torch::kBFloat16);
  TORCH_CHECK(table.is_contiguous() && out.is_contiguous() && ids.is_contiguous(), "embed layout");
  c10::cuda::CUDAGuard g(ids.device());
  const int64_t total = vocab_total > 0 ? vocab_total : table.size(0);
  b200::launch_embed(cptr<int64_t>(ids), ids.numel(), cptr<__nv_bfloat16>(table), table.size(0), row0, total,
                     table.size(1), ptr<__nv_bfloat16>(out), err_ptr(ids), stream());
}

// ------------------------------------------------------------- indexer
void indexer_logits(const Tensor& q, const Tensor& k, const Tensor& w, const Tensor& kscale, Tensor& logits,
                    int64_t query_start) {
  CHECK_CUDA(q); CHECK_DTYPE(q, torch::kFloat8_e4m3fn); CHECK_DTYPE(k, torch::kFloat8_e4m3fn);
  CHECK_DTYPE(w, torch::kFloat32); CHECK_DTYPE(kscale, torch::kFloat32); CHECK_DTYPE(logits, torch::kFloat32);
  TORCH_CHECK(q.dim() == 3 && q.size(1) == 64 && q.size(2) == 128 && q.is_contiguous(), "indexer: q [Q,64,128]");
  TORCH_CHECK(k.dim() == 2 && k.size(1) == 128 && k.is_contiguous(), "indexer: k [N,128]");
  TORCH_CHECK(w.is_contiguous() && w.size(0) == q.size(0) && w.size(1) == 64, "indexer: w [Q,64]");
  TORCH_CHECK(reinterpret_cast<uintptr_t>(w.data_ptr()) % 16 == 0, "indexer: w must be 16-byte aligned");
  TORCH_CHECK(kscale.numel() >= k.size(0), "indexer: kscale");
  TORCH_CHECK(logits.size(0) >= q.size(0) && logits.size(1) >= k.size(0) && logits.stride(1) == 1, "indexer: logits");
  // Rows past the last key see every key (a key shard before the queries).
  TORCH_CHECK(query_start >= 0, "indexer: query_start");
  c10::cuda::CUDAGuard g(q.device());
  b200::IndexerArgs a{};
  a.q = cptr<uint8_t>(q); a.k = cptr<uint8_t>(k); a.w = cptr<float>(w); a.kscale = cptr<float>(kscale);
  a.logits = ptr<float>(logits); a.ldl = logits.stride(0); a.Q = q.size(0); a.N = k.size(0);
  a.query_start = query_start; a.n_cols = logits.size(1); a.err = err_ptr(q);
  b200::launch_indexer_logits(a, stream());
}

// Fused exact selection: ids/values [Q, width] equal to topk(indexer_logits(...))
// with the causal rule, without full logits in HBM (logits = the fallback
// buffer, written only for rows the candidate lists cannot finish).
void indexer_select(const Tensor& q, const Tensor& k, const Tensor& w, const Tensor& kscale, Tensor& logits,
                    int64_t query_start, int64_t topk, Tensor& values, Tensor& ids, bool index_order,
                    int64_t sample_stride, int64_t cand_cap, const c10::optional<Tensor>& diag) {
  CHECK_CUDA(q); CHECK_DTYPE(q, torch::kFloat8_e4m3fn); CHECK_DTYPE(k, torch::kFloat8_e4m3fn);
  CHECK_DTYPE(w, torch::kFloat32); CHECK_DTYPE(kscale, torch::kFloat32); CHECK_DTYPE(logits, torch::kFloat32);
  CHECK_DTYPE(values, torch::kFloat32); CHECK_DTYPE(ids, torch::kInt32);
  TORCH_CHECK(q.dim() == 3 && q.size(1) == 64 && q.size(2) == 128 && q.is_contiguous(), "indexer_select: q [Q,64,128]");
  TORCH_CHECK(k.dim() == 2 && k.size(1) == 128 && k.is_contiguous(), "indexer_select: k [N,128]");
  TORCH_CHECK(w.is_contiguous() && w.size(0) == q.size(0) && w.size(1) == 64, "indexer_select: w [Q,64]");
  TORCH_CHECK(reinterpret_cast<uintptr_t>(w.data_ptr()) % 16 == 0, "indexer_select: w must be 16-byte aligned");
  TORCH_CHECK(kscale.numel() >= k.size(0), "indexer_select: kscale");
  TORCH_CHECK(logits.size(0) >= q.size(0) && logits.size(1) >= k.size(0) && logits.stride(1) == 1,
              "indexer_select: fallback logits [>=Q, >=N]");
  TORCH_CHECK(values.is_contiguous() && ids.is_contiguous() && values.size(0) == q.size(0) &&
                  ids.size(0) == q.size(0) && values.size(1) == ids.size(1),
              "indexer_select: outputs [Q, width]");
  TORCH_CHECK(query_start >= 0, "indexer_select: query_start");
  c10::cuda::CUDAGuard g(q.device());
  const int64_t Q = q.size(0), N = k.size(0);
  auto f32 = torch::dtype(torch::kFloat32).device(q.device());
  auto i32 = torch::dtype(torch::kInt32).device(q.device());
  const int64_t ns = (N + sample_stride - 1) / sample_stride;
  Tensor slog = torch::empty({Q, std::max<int64_t>(4, (ns + 3) / 4 * 4)}, f32);
  Tensor thresh = torch::empty({Q}, f32);
  Tensor cand = torch::empty({Q, cand_cap}, torch::dtype(torch::kInt64).device(q.device()));
  Tensor counts = torch::empty({Q + 1}, i32);  // per-row counts, then the any-row-flagged word
  Tensor small = torch::empty({2, Q}, i32);    // flags, overflow
  b200::IndexerSelectArgs a{};
  a.idx.q = cptr<uint8_t>(q); a.idx.k = cptr<uint8_t>(k); a.idx.w = cptr<float>(w);
  a.idx.kscale = cptr<float>(kscale); a.idx.logits = ptr<float>(logits); a.idx.ldl = logits.stride(0);
  a.idx.Q = int(Q); a.idx.N = int(N); a.idx.query_start = int(query_start); a.idx.n_cols = int(logits.size(1));
  a.idx.err = err_ptr(q);
  a.k = int(topk); a.width = int(ids.size(1)); a.sample_stride = int(sample_stride); a.cand_cap = int(cand_cap);
  a.sample_logits = slog.data_ptr<float>(); a.ld_sample = slog.stride(0); a.thresh = thresh.data_ptr<float>();
  a.cand = reinterpret_cast<uint64_t*>(cand.data_ptr<int64_t>());
  a.cand_count = counts.data_ptr<int>(); a.any_flag = a.cand_count + Q;
  a.flags = small[0].data_ptr<int>(); a.overflow = small[1].data_ptr<int>();
  a.values = ptr<float>(values); a.ids = ptr<int>(ids); a.index_order = index_order;
  b200::launch_indexer_select(a, stream());
  if (diag) {  // [rows redone from full logits, candidates kept, most candidates of a row]
    TORCH_CHECK(diag->dtype() == torch::kInt64 && diag->numel() >= 3, "indexer_select: diag int64 [3]");
    Tensor d = *diag;
    Tensor c = counts.narrow(0, 0, Q);
    d.select(0, 0).copy_(small[0].sum());
    d.select(0, 1).copy_(c.to(torch::kInt64).sum());
    d.select(0, 2).copy_(c.max());
  }
}

void topk(const Tensor& scores, int64_t N, int64_t k, int64_t causal_start, Tensor& values, Tensor& ids,
          int64_t algo) {
  CHECK_CUDA(scores); CHECK_DTYPE(scores, torch::kFloat32); CHECK_DTYPE(values, torch::kFloat32);
  CHECK_DTYPE(ids, torch::kInt32); CHECK_LAST_CONTIG(scores);
  TORCH_CHECK(values.is_contiguous() && ids.is_contiguous() && values.size(1) == k && ids.size(1) == k, "topk outputs");
  TORCH_CHECK(N <= scores.size(1), "topk: N exceeds scores width");
  c10::cuda::CUDAGuard g(scores.device());
  // algo 0: histogram select, descending; 2: histogram select, ascending index order
  // (rows finished by the multi-pass fallback stay descending); 1: multi-pass only.
  const bool select = algo == 0 || algo == 2;
  Tensor overflow;
  if (select) overflow = torch::zeros({scores.size(0)}, torch::dtype(torch::kInt32).device(scores.device()));
  b200::launch_topk_causal(cptr<float>(scores), scores.stride(0), scores.size(0), N, k, causal_start,
                           ptr<float>(values), ptr<int>(ids), err_ptr(scores), stream(),
                           select ? overflow.data_ptr<int>() : nullptr, algo == 2);
}

// ------------------------------------------------------------- attention
void sparse_mla(const Tensor& q, const Tensor& kv, const Tensor& ids, double scale, Tensor& out,
                const c10::optional<Tensor>& lse, int64_t splits, const c10::optional<Tensor>& scratch,
                int64_t impl) {
  CHECK_CUDA(q); CHECK_DTYPE(q, torch::kBFloat16); CHECK_DTYPE(kv, torch::kBFloat16); CHECK_DTYPE(ids, torch::kInt32);
  CHECK_DTYPE(out, torch::kBFloat16);
  TORCH_CHECK(q.dim() == 3 && q.size(2) == 576 && q.is_contiguous(), "sparse_mla: q [T,H,576]");
  TORCH_CHECK(kv.dim() == 2 && kv.size(1) == 576 && kv.is_contiguous(), "sparse_mla: kv [P,576]");
  TORCH_CHECK(ids.dim() == 2 && ids.size(0) == q.size(0) && ids.is_contiguous(), "sparse_mla: ids [T,K]");
  TORCH_CHECK(out.is_contiguous() && out.size(0) == q.size(0) && out.size(1) == q.size(1) && out.size(2) == 512, "sparse_mla: out");
  c10::cuda::CUDAGuard g(q.device());
  b200::MLAArgs a{};
  a.q = cptr<__nv_bfloat16>(q); a.kv = cptr<__nv_bfloat16>(kv); a.ids = cptr<int>(ids);
  a.out = ptr<__nv_bfloat16>(out); a.lse = (lse && lse->defined()) ? ptr<float>(*lse) : nullptr;
  a.T = q.size(0); a.H = q.size(1); a.K = ids.size(1); a.P = kv.size(0); a.scale = float(scale); a.err = err_ptr(q);
  float* sp = nullptr;
  if (splits > 1) {
    TORCH_CHECK(scratch && scratch->defined() && scratch->scalar_type() == torch::kFloat32, "sparse_mla: scratch");
    TORCH_CHECK(size_t(scratch->numel()) * 4 >= b200::sparse_mla_scratch_bytes(a.T, a.H, splits), "sparse_mla: scratch too small");
    sp = ptr<float>(*scratch);
  }
  // impl 0 / 2: the cta_group::2 kernel (default); 1: the mma.sync baseline;
  // 3: probe; 4 / 16-31: the DSMEM-exchange tcgen05 kernel; 32-63 and 128-255:
  // pair kernel with debug bits impl - 32 / impl - 128 (bit 64: cp.async gathers).
  if (impl == 0 || impl == 2 || (impl >= 32 && impl < 64) || (impl >= 128 && impl < 256)) {
    const int dbg = impl >= 128 ? int(impl - 128) : impl >= 32 ? int(impl - 32) : 0;
    b200::launch_sparse_mla_2sm(a, int(splits), sp, stream(), nullptr, dbg);
  } else if (impl == 3) {  // debug: raw first-tile scores of cluster 0 into `scratch` (splits must be 1)
    TORCH_CHECK(splits == 1 && scratch && scratch->defined() && scratch->numel() >= 2 * 128 * 32, "sparse_mla: probe buffer");
    b200::launch_sparse_mla_2sm(a, 1, nullptr, stream(), ptr<float>(*scratch));
  } else if (impl == 4 || (impl >= 16 && impl < 32)) {
    b200::launch_sparse_mla_tc(a, int(splits), sp, stream(), impl >= 16 ? int(impl - 16) : 0);
  } else {
    b200::launch_sparse_mla_split(a, int(splits), sp, stream());
  }
}

Tensor topk_trace(int64_t row) {
  Tensor t = torch::empty({16}, torch::kInt64);
  if (row >= -1) b200::set_topk_trace_row(int(row));
  b200::copy_topk_trace(reinterpret_cast<unsigned long long*>(t.data_ptr<int64_t>()));
  return t;
}

Tensor sparse_mla_2sm_trace() {
  Tensor t = torch::empty({4, 65, 16}, torch::kInt64);
  b200::copy_sparse_mla_2sm_trace(reinterpret_cast<unsigned long long*>(t.data_ptr<int64_t>()));
  return t;
}

Tensor sparse_mla_trace() {
  Tensor t = torch::empty({4, 65, 16}, torch::kInt64);
  b200::copy_sparse_mla_trace(reinterpret_cast<unsigned long long*>(t.data_ptr<int64_t>()));
  return t;
}

int64_t fp8_gemm_splits(int64_t M, int64_t N, int64_t K, bool ue8m0) {
  return b200::fp8_gemm_launch_splits(int(M), int(N), int(K), 8, ue8m0);
}

int64_t sparse_mla_scratch_bytes(int64_t T, int64_t H, int64_t splits) {
  return int64_t(b200::sparse_mla_scratch_bytes(T, H, splits));
}

// ------------------------------------------------------------ transfer
void gather_rows(const Tensor& host, Tensor& records, const Tensor& host_ids, const c10::optional<Tensor>& slots,
                 int64_t n, const c10::optional<Tensor>& device_count) {
  TORCH_CHECK(host.is_pinned(), "gather_rows: host must be pinned");
  CHECK_CUDA(records); CHECK_DTYPE(host_ids, torch::kInt64);
  const bool have_slots = slots && slots->defined();
  if (have_slots) CHECK_DTYPE((*slots), torch::kInt64);
  TORCH_CHECK(host.is_contiguous() && records.is_contiguous() && host.stride(0) * host.element_size() == records.stride(0) * records.element_size(),
              "gather_rows: matching contiguous rows");
  c10::cuda::CUDAGuard g(records.device());
  const int row_bytes = records.stride(0) * records.element_size();
  b200::launch_gather_rows(cptr<uint8_t>(host), ptr<uint8_t>(records), cptr<int64_t>(host_ids),
                           have_slots ? cptr<int64_t>(*slots) : nullptr, int(n), (device_count && device_count->defined()) ? cptr<int>(*device_count) : nullptr,
                           row_bytes, host.size(0), records.size(0), err_ptr(records), stream());
}

b200::PoolRecallArgs pool_args(const c10::optional<Tensor>& ids, int64_t hist_end, const c10::optional<Tensor>& page_table,
                               Tensor& h2d, Tensor& d2h, Tensor& priority, Tensor& meta, Tensor& mark,
                               Tensor& miss_list, Tensor& victims, Tensor& stats) {
  CHECK_DTYPE(h2d, torch::kInt32); CHECK_DTYPE(d2h, torch::kInt64); CHECK_DTYPE(priority, torch::kInt64);
  CHECK_DTYPE(meta, torch::kInt64); CHECK_DTYPE(mark, torch::kInt32); CHECK_DTYPE(miss_list, torch::kInt64);
  CHECK_DTYPE(victims, torch::kInt64); CHECK_DTYPE(stats, torch::kInt64);
  TORCH_CHECK(d2h.numel() == priority.numel() && miss_list.numel() >= d2h.numel() && victims.numel() >= d2h.numel() &&
              mark.numel() == h2d.numel() && meta.numel() >= 4 && stats.numel() >= 5, "pool metadata shapes");
  b200::PoolRecallArgs a;
  if (ids && ids->defined()) {
    CHECK_DTYPE((*ids), torch::kInt32);
    TORCH_CHECK(ids->is_contiguous(), "pool: contiguous ids");
    a.ids = ids->data_ptr<int>();
    a.n = int(ids->numel());
  }
  if (page_table && page_table->defined()) {
    CHECK_DTYPE((*page_table), torch::kInt32);
    a.page_table = page_table->data_ptr<int>();
    a.npages = int(page_table->numel());
  }
  a.hist_end = int(hist_end);
  a.h2d = h2d.data_ptr<int>();
  a.d2h = d2h.data_ptr<int64_t>();
  a.priority = priority.data_ptr<int64_t>();
  a.P = int(d2h.numel() - 1);
  a.meta = meta.data_ptr<int64_t>();
  a.meta_words = int(meta.numel());
  a.mark = mark.data_ptr<int>();
  a.host_rows = h2d.numel();
  a.miss_list = miss_list.data_ptr<int64_t>();
  a.victims = victims.data_ptr<int64_t>();
  a.max_miss = int(d2h.numel());
  a.stats = stats.data_ptr<int64_t>();
  a.err = err_ptr(h2d);
  return a;
}

// begin + classify: dedupe the selection, stamp resident rows, collect misses (all on the device).
void pool_recall(const Tensor& ids, int64_t hist_end, const Tensor& page_table, Tensor& h2d, Tensor& d2h,
                 Tensor& priority, Tensor& meta, Tensor& mark, Tensor& miss_list, Tensor& victims, Tensor& stats) {
  c10::cuda::CUDAGuard g(h2d.device());
  auto a = pool_args(ids, hist_end, page_table, h2d, d2h, priority, meta, mark, miss_list, victims, stats);
  b200::launch_pool_recall(a, stream());
}

// Choose k slots (k_host >= 0, else the device miss count; k_limit caps it), map new_rows (or the misses).
void pool_select(Tensor& h2d, Tensor& d2h, Tensor& priority, Tensor& meta, Tensor& mark, Tensor& miss_list,
                 Tensor& victims, Tensor& stats, int64_t k_host, int64_t k_limit, const c10::optional<Tensor>& new_rows,
                 int64_t count_slot) {
  c10::cuda::CUDAGuard g(h2d.device());
  auto a = pool_args(c10::nullopt, 0, c10::nullopt, h2d, d2h, priority, meta, mark, miss_list, victims, stats);
  const int64_t* rows = nullptr;
  if (new_rows && new_rows->defined()) {
    CHECK_DTYPE((*new_rows), torch::kInt64);
    TORCH_CHECK(new_rows->numel() >= k_host, "pool_select: new_rows shorter than k");
    rows = new_rows->data_ptr<int64_t>();
  }
  TORCH_CHECK(k_host <= a.P, "pool_select: more rows than slots");
  b200::launch_pool_begin(a.meta, stream());  // a select without classify is its own event
  b200::launch_pool_select(a, int(k_host), int(k_limit), rows, int(count_slot), stream());
}

// Continue a pool_recall event: select victims for the device-side misses (no begin).
void pool_recall_select(Tensor& h2d, Tensor& d2h, Tensor& priority, Tensor& meta, Tensor& mark, Tensor& miss_list,
                        Tensor& victims, Tensor& stats, int64_t k_limit, int64_t count_slot) {
  c10::cuda::CUDAGuard g(h2d.device());
  auto a = pool_args(c10::nullopt, 0, c10::nullopt, h2d, d2h, priority, meta, mark, miss_list, victims, stats);
  b200::launch_pool_select(a, -1, int(k_limit), nullptr, int(count_slot), stream());
}

b200::TensorDesc desc_of(const Tensor& t) {
  b200::TensorDesc d;
  d.defined = t.defined();
  if (!d.defined) return d;
  switch (t.scalar_type()) {
    case torch::kInt32: d.dtype = b200::DType::I32; break;
    case torch::kInt64: d.dtype = b200::DType::I64; break;
    case torch::kUInt8: d.dtype = b200::DType::U8; break;
    case torch::kBFloat16: d.dtype = b200::DType::BF16; break;
    case torch::kFloat32: d.dtype = b200::DType::F32; break;
    default: d.dtype = b200::DType::Other;
  }
  d.numel = t.numel();
  d.ndim = int(t.dim());
  d.rows = t.dim() ? t.size(0) : 0;
  d.row_bytes = t.dim() == 2 ? t.stride(0) * int64_t(t.element_size()) : 0;
  d.contiguous = t.is_contiguous();
  d.device = t.is_cuda() ? int(t.get_device()) : -1;
  d.pinned = !t.is_cuda() && t.is_pinned();
  return d;
}

// One exact recall event (classify -> select -> gather), each stage validated
// right before it is enqueued; see host/recall_dispatch.h.
void pool_recall_dispatch(const Tensor& ids, int64_t hist_end, const Tensor& page_table, Tensor& h2d, Tensor& d2h,
                          Tensor& priority, Tensor& meta, Tensor& mark, Tensor& miss_list, Tensor& victims,
                          Tensor& stats, Tensor& select_stats, int64_t k_limit, int64_t count_slot, const Tensor& host,
                          Tensor& records, const c10::optional<Tensor>& fp8_scratch) {
  b200::RecallDesc d;
  d.ids = desc_of(ids); d.page_table = desc_of(page_table); d.h2d = desc_of(h2d); d.d2h = desc_of(d2h);
  d.priority = desc_of(priority); d.meta = desc_of(meta); d.mark = desc_of(mark); d.miss_list = desc_of(miss_list);
  d.victims = desc_of(victims); d.stats = desc_of(stats); d.select_stats = desc_of(select_stats);
  d.host = desc_of(host); d.records = desc_of(records);
  d.hist_end = hist_end; d.k_limit = k_limit; d.count_slot = count_slot;
  d.fp8_host = fp8_scratch && fp8_scratch->defined();
  c10::cuda::CUDAGuard g(h2d.device());
  Tensor scratch = (fp8_scratch && fp8_scratch->defined()) ? *fp8_scratch : Tensor();
  if (scratch.defined())
    TORCH_CHECK(scratch.scalar_type() == torch::kUInt8 && scratch.size(1) == 656 && scratch.size(0) >= miss_list.numel() &&
                host.size(1) * host.element_size() == 656, "pool_recall_dispatch: FP8 scratch [>= P+1, 656]");
  struct Stages {
    const Tensor &ids, &page_table, &host;
    Tensor &h2d, &d2h, &priority, &meta, &mark, &miss_list, &victims, &stats, &select_stats, &records, &scratch;
    int64_t hist_end, k_limit, count_slot;
    void classify() {
      auto a = pool_args(ids, hist_end, page_table, h2d, d2h, priority, meta, mark, miss_list, victims, stats);
      b200::launch_pool_recall(a, stream());
    }
    void select() {
      auto a = pool_args(c10::nullopt, 0, c10::nullopt, h2d, d2h, priority, meta, mark, miss_list, victims,
                         select_stats);
      b200::launch_pool_select(a, -1, int(k_limit), nullptr, int(count_slot), stream());
    }
    void gather() {
      // meta word 2 holds the rows placed; its low 32 bits are the gather's device-side count.
      const int* count = reinterpret_cast<const int*>(meta.data_ptr<int64_t>()) + 4;
      if (scratch.defined()) {
        // FP8 host records: the 656-byte rows cross PCIe into a dense scratch,
        // then are dequantized into their pool slots.
        b200::launch_gather_rows(cptr<uint8_t>(host), ptr<uint8_t>(scratch), cptr<int64_t>(miss_list), nullptr,
                                 int(miss_list.numel()), count, 656, host.size(0), scratch.size(0), err_ptr(records),
                                 stream());
        b200::launch_dequant_kv_rows(cptr<uint8_t>(scratch), ptr<__nv_bfloat16>(records), cptr<int64_t>(victims),
                                     int(miss_list.numel()), count, records.size(0), err_ptr(records), stream());
        return;
      }
      const int row_bytes = int(records.stride(0) * records.element_size());
      b200::launch_gather_rows(cptr<uint8_t>(host), ptr<uint8_t>(records), cptr<int64_t>(miss_list),
                               cptr<int64_t>(victims), int(miss_list.numel()), count, row_bytes, host.size(0),
                               records.size(0), err_ptr(records), stream());
    }
  } stages{ids, page_table, host, h2d, d2h, priority, meta, mark, miss_list, victims, stats, select_stats, records,
           scratch, hist_end, k_limit, count_slot};
  b200::run_recall(d, stages);
}

// offset[0] = mean of the finite logits of the last min(4, rows) rows over columns [0, cols).
void echo_hint(const Tensor& logits, int64_t rows, int64_t cols, Tensor& offset) {
  c10::cuda::CUDAGuard g(logits.device());
  CHECK_DTYPE(logits, torch::kFloat32); CHECK_DTYPE(offset, torch::kFloat32);
  TORCH_CHECK(logits.stride(1) == 1 && rows <= logits.size(0) && cols <= logits.size(1), "echo_hint shapes");
  const int64_t tail = rows < 4 ? rows : 4;
  if (tail <= 0) return;
  b200::launch_echo_hint(logits.data_ptr<float>(), logits.stride(0), int(rows - tail), int(tail), int(cols),
                         offset.data_ptr<float>(), stream());
}

// pred_ids[c] = c for history rows certainly in some row's top-k (caller pre-fills -1).
void echo_predict(const Tensor& logits, int64_t rows, int64_t hist_end, const Tensor& offset, int64_t k, Tensor& pred_ids) {
  c10::cuda::CUDAGuard g(logits.device());
  CHECK_DTYPE(logits, torch::kFloat32); CHECK_DTYPE(offset, torch::kFloat32); CHECK_DTYPE(pred_ids, torch::kInt32);
  TORCH_CHECK(logits.stride(1) == 1 && pred_ids.numel() >= hist_end && logits.size(1) >= hist_end, "echo_predict shapes");
  b200::launch_echo_predict(logits.data_ptr<float>(), logits.stride(0), int(rows), int(hist_end), offset.data_ptr<float>(),
                            int(k), pred_ids.data_ptr<int>(), stream());
}

void pool_map(const Tensor& ids, int64_t hist_end, int64_t tail, int64_t committed_end, const Tensor& page_table,
              const Tensor& h2d, Tensor& out) {
  c10::cuda::CUDAGuard g(h2d.device());
  CHECK_DTYPE(ids, torch::kInt32); CHECK_DTYPE(out, torch::kInt32); CHECK_DTYPE(page_table, torch::kInt32);
  CHECK_DTYPE(h2d, torch::kInt32);
  b200::PoolRecallArgs a;
  a.ids = ids.data_ptr<int>();
  a.n = int(ids.numel());
  a.hist_end = int(hist_end);
  a.page_table = page_table.data_ptr<int>();
  a.npages = int(page_table.numel());
  a.h2d = const_cast<int*>(h2d.data_ptr<int>());
  b200::launch_pool_map(a, int(tail), int(committed_end), out.data_ptr<int>(), stream());
}

// `call` numbers this op's calls from 1 (parity = call & 1); targets are the cumulative flag counts.
void moe_route(const Tensor& logits, bool split, const Tensor& bias, int64_t E, int64_t n_group, int64_t topk_group,
               int64_t K, bool normalize, double scaling, Tensor& ids, Tensor& weights) {
  c10::cuda::CUDAGuard guard(logits.device());
  TORCH_CHECK(logits.dtype() == torch::kFloat32 && logits.stride(1) == 1, "moe_route: fp32 row-major logits");
  b200::launch_moe_route(logits.data_ptr<float>(), int(logits.stride(0)), split, bias.data_ptr<float>(),
                         int(logits.size(0)), int(E), int(n_group), int(topk_group), int(K), normalize, float(scaling),
                         ids.data_ptr<int>(), weights.data_ptr<float>(), at::cuda::getCurrentCUDAStream());
}

void moe_layout(const Tensor& ids, int64_t e0, int64_t E_loc, int64_t max_blocks, Tensor& row_pos,
                Tensor& block_expert, Tensor& cursor, Tensor& total_rows) {
  c10::cuda::CUDAGuard guard(ids.device());
  b200::launch_moe_layout(ids.data_ptr<int>(), int(ids.numel()), int(e0), int(E_loc), int(max_blocks),
                          row_pos.data_ptr<int>(), block_expert.data_ptr<int>(), cursor.data_ptr<int>(),
                          total_rows.data_ptr<int>(), err_ptr(ids), at::cuda::getCurrentCUDAStream());
}

void moe_gather(const Tensor& q, const Tensor& s_t, int64_t topk, const Tensor& row_pos, Tensor& a, Tensor& a_s) {
  c10::cuda::CUDAGuard guard(q.device());
  TORCH_CHECK(q.is_contiguous() && a.is_contiguous() && a_s.is_contiguous(), "moe_gather: contiguous buffers");
  b200::launch_moe_gather(reinterpret_cast<const uint8_t*>(q.data_ptr()), s_t.data_ptr<float>(), int(s_t.stride(0)),
                          int(row_pos.numel()), int(topk), int(q.size(1)), row_pos.data_ptr<int>(),
                          reinterpret_cast<uint8_t*>(a.data_ptr()), a_s.data_ptr<float>(), int(a_s.stride(0)),
                          at::cuda::getCurrentCUDAStream());
}

void moe_combine(const Tensor& y, const Tensor& row_pos, const Tensor& w, int64_t topk, Tensor& out) {
  c10::cuda::CUDAGuard guard(y.device());
  b200::launch_moe_combine(reinterpret_cast<const __nv_bfloat16*>(y.data_ptr()), int(y.size(1)), row_pos.data_ptr<int>(),
                           w.data_ptr<float>(), int(out.size(0)), int(topk),
                           reinterpret_cast<__nv_bfloat16*>(out.data_ptr()), at::cuda::getCurrentCUDAStream());
}

// a [M_pad, K] fp8, a_s [K/128, M_pad], w [E, N, K] fp8, w_s [E, N/128, K/128] -> out [M_pad, N] bf16.
void fp8_gemm_grouped(const Tensor& a, const Tensor& a_s, const Tensor& w, const Tensor& w_s,
                      const Tensor& block_expert, Tensor& out) {
  c10::cuda::CUDAGuard guard(a.device());
  TORCH_CHECK(w.dim() == 3 && w.is_contiguous() && w_s.is_contiguous(), "grouped: stacked expert weights");
  b200::launch_fp8_gemm_grouped(reinterpret_cast<const uint8_t*>(a.data_ptr()), a_s.data_ptr<float>(),
                                int(a_s.stride(0)), reinterpret_cast<const uint8_t*>(w.data_ptr()),
                                w_s.data_ptr<float>(), block_expert.data_ptr<int>(), int(a.size(0)), int(w.size(1)),
                                int(a.size(1)), int(w.size(0)), reinterpret_cast<__nv_bfloat16*>(out.data_ptr()),
                                int(out.stride(0)), err_ptr(a), at::cuda::getCurrentCUDAStream());
}

b200::EpArgs make_ep(int64_t rank, int64_t world, int64_t E, int64_t D, int64_t topk, int64_t T, int64_t M_pad,
                     int64_t call, const std::vector<int64_t>& flags, const std::vector<int64_t>& cnt,
                     const std::vector<int64_t>& a, const std::vector<int64_t>& as, const std::vector<int64_t>& y,
                     const std::vector<int64_t>& rsrc) {
  if (world < 1 || world > b200::kMaxRanks || int64_t(flags.size()) != world) throw std::invalid_argument("ep: bad world");
  b200::EpArgs p;
  p.rank = int(rank);
  p.world = int(world);
  p.E = int(E);
  p.E_loc = int(E / world);
  p.D = int(D);
  p.topk = int(topk);
  p.T = int(T);
  p.M_pad = int(M_pad);
  p.call = uint64_t(call);
  p.parity = int(call & 1);
  for (int q = 0; q < world; ++q) {
    p.flags[q] = reinterpret_cast<uint64_t*>(flags[q]);
    p.cnt[q] = reinterpret_cast<int*>(cnt[q]);
    p.a[q] = reinterpret_cast<uint8_t*>(a[q]);
    p.as[q] = reinterpret_cast<float*>(as[q]);
    p.y[q] = reinterpret_cast<__nv_bfloat16*>(y[q]);
    if (!rsrc.empty()) p.rsrc[q] = reinterpret_cast<int*>(rsrc[q]);
  }
  return p;
}

void ep_dispatch(const Tensor& ids, const Tensor& q, const Tensor& s_t, Tensor& cursor, Tensor& pos_out,
                 Tensor& block_expert, int64_t rank, int64_t world, int64_t E, int64_t M_pad, int64_t call,
                 const std::vector<int64_t>& flags, const std::vector<int64_t>& cnt, const std::vector<int64_t>& a,
                 const std::vector<int64_t>& as, const std::vector<int64_t>& y, const std::vector<int64_t>& rsrc,
                 const c10::optional<Tensor>& block_valid) {
  c10::cuda::CUDAGuard guard(q.device());
  TORCH_CHECK(ids.dtype() == torch::kInt32 && ids.is_contiguous() && q.is_contiguous(), "ep_dispatch: layouts");
  if (block_valid) TORCH_CHECK(block_valid->numel() == block_expert.numel(), "ep_dispatch: block_valid size");
  auto p = make_ep(rank, world, E, q.size(1), ids.size(1), ids.size(0), M_pad, call, flags, cnt, a, as, y, rsrc);
  b200::launch_ep_dispatch(p, ids.data_ptr<int>(), reinterpret_cast<const uint8_t*>(q.data_ptr()), s_t.data_ptr<float>(),
                           int(s_t.stride(0)), cursor.data_ptr<int>(), pos_out.data_ptr<int>(),
                           block_expert.data_ptr<int>(), int(block_expert.numel()), err_ptr(q),
                           at::cuda::getCurrentCUDAStream(), block_valid ? block_valid->data_ptr<int>() : nullptr);
}

void ep_combine(const Tensor& ids, const Tensor& pos, const Tensor& w, Tensor& out, int64_t rank, int64_t world,
                int64_t E, int64_t M_pad, int64_t call, const std::vector<int64_t>& flags,
                const std::vector<int64_t>& cnt, const std::vector<int64_t>& a, const std::vector<int64_t>& as,
                const std::vector<int64_t>& y, const std::vector<int64_t>& rsrc, bool push) {
  c10::cuda::CUDAGuard guard(out.device());
  auto p = make_ep(rank, world, E, out.size(1), ids.size(1), ids.size(0), M_pad, call, flags, cnt, a, as, y, rsrc);
  b200::launch_ep_combine(p, ids.data_ptr<int>(), pos.data_ptr<int>(), w.data_ptr<float>(),
                          reinterpret_cast<__nv_bfloat16*>(out.data_ptr()), err_ptr(out),
                          at::cuda::getCurrentCUDAStream(), push);
}

// Down projection of the expert-parallel MoE that pushes every row to its
// source rank's receive slot (call parity half) and raises the ready flags.
void fp8_gemm_grouped_push(const Tensor& a, const Tensor& a_s, const Tensor& w, const Tensor& w_s,
                           const Tensor& block_expert, const Tensor& block_valid, int64_t row_src,
                           const std::vector<int64_t>& dst, const std::vector<int64_t>& flags, Tensor& finish,
                           int64_t rank, int64_t world) {
  c10::cuda::CUDAGuard guard(a.device());
  TORCH_CHECK(w.dim() == 3 && w.is_contiguous() && w_s.is_contiguous(), "grouped push: stacked expert weights");
  TORCH_CHECK(int64_t(dst.size()) == world && int64_t(flags.size()) == world, "grouped push: peer lists");
  TORCH_CHECK(block_valid.numel() * 128 >= a.size(0) && finish.dtype() == torch::kInt32, "grouped push: tables");
  b200::EpPushArgs push;
  push.row_src = reinterpret_cast<const int*>(row_src);
  push.block_valid = block_valid.data_ptr<int>();
  push.finish = reinterpret_cast<unsigned int*>(finish.data_ptr<int>());
  push.ld = int(w.size(1));
  push.rank = int(rank);
  push.world = int(world);
  for (int q = 0; q < world; ++q) {
    push.dst[q] = reinterpret_cast<__nv_bfloat16*>(dst[q]);
    push.flags[q] = reinterpret_cast<uint64_t*>(flags[q]);
  }
  b200::launch_fp8_gemm_grouped(reinterpret_cast<const uint8_t*>(a.data_ptr()), a_s.data_ptr<float>(),
                                int(a_s.stride(0)), reinterpret_cast<const uint8_t*>(w.data_ptr()),
                                w_s.data_ptr<float>(), block_expert.data_ptr<int>(), int(a.size(0)), int(w.size(1)),
                                int(a.size(1)), int(w.size(0)), nullptr, int(w.size(1)), err_ptr(a),
                                at::cuda::getCurrentCUDAStream(), &push);
}

b200::P2PArgs make_p2p(int64_t rank, int64_t world, int64_t S, int64_t call, int64_t arrive_target,
                      int64_t reuse_target, const std::vector<int64_t>& flags, const std::vector<int64_t>& g,
                      const std::vector<int64_t>& gs, const std::vector<int64_t>& rb) {
  if (world < 1 || world > b200::kMaxRanks || int64_t(flags.size()) != world) throw std::invalid_argument("p2p: bad world");
  b200::P2PArgs p;
  p.rank = int(rank);
  p.world = int(world);
  p.S = int(S);
  p.parity = int(call & 1);
  p.arrive_target = uint64_t(arrive_target);
  p.reuse_target = uint64_t(reuse_target);
  for (int q = 0; q < world; ++q) {
    p.flags[q] = reinterpret_cast<uint64_t*>(flags[q]);
    if (!g.empty()) p.g[q] = reinterpret_cast<uint8_t*>(g[q]);
    if (!gs.empty()) p.gs[q] = reinterpret_cast<float*>(gs[q]);
    if (!rb.empty()) p.rb[q] = reinterpret_cast<__nv_bfloat16*>(rb[q]);
  }
  return p;
}

// Device-resident op state (epoch != 0): the call's number, parity and flag
// targets come from the op-state block; the host passes only its increments.
void set_epoch(b200::P2PArgs& p, int64_t epoch, int64_t arrive_inc, int64_t done_inc) {
  if (epoch == 0) return;
  TORCH_CHECK(epoch % 8 == 0, "p2p: op-state block must be 8-byte aligned");
  TORCH_CHECK(arrive_inc > 0 && done_inc >= 0, "p2p: op-state increments");
  p.epoch = reinterpret_cast<uint64_t*>(epoch);
  p.arrive_inc = uint32_t(arrive_inc);
  p.done_inc = uint32_t(done_inc);
}

// AG-GEMM: q_local [S, K] fp8, s_local_t [K/128, S] fp32 -> out [world*S, N] bf16.
void fp8_gemm_ag(const Tensor& q_local, const Tensor& s_local_t, const Tensor& w, const Tensor& w_s, Tensor& out,
                 int64_t rank, int64_t world, int64_t call, int64_t arrive_target, int64_t reuse_target,
                 const std::vector<int64_t>& flags, const std::vector<int64_t>& g, const std::vector<int64_t>& gs,
                 int64_t epoch, int64_t arrive_inc, int64_t done_inc) {
  const int64_t S = q_local.size(0), K = q_local.size(1), N = w.size(0);
  TORCH_CHECK(q_local.is_contiguous() && s_local_t.is_contiguous() && s_local_t.size(1) == S, "ag: layout");
  TORCH_CHECK(out.size(0) == world * S && out.size(1) == N && out.is_contiguous(), "ag: out shape");
  c10::cuda::CUDAGuard guard(q_local.device());
  auto p = make_p2p(rank, world, S, call, arrive_target, reuse_target, flags, g, gs, {});
  set_epoch(p, epoch, arrive_inc, done_inc);
  p.grid = b200::fp8_gemm_ag_grid(int(world * S), int(N), int(K));
  p.a_local = reinterpret_cast<const uint8_t*>(q_local.data_ptr());
  p.sfa_local = s_local_t.data_ptr<float>();
  b200::launch_fp8_gemm_ag(p, reinterpret_cast<const uint8_t*>(w.data_ptr()), int(w.stride(0)), w_s.data_ptr<float>(),
                           reinterpret_cast<__nv_bfloat16*>(out.data_ptr()), int(out.stride(0)), int(world * S), int(N),
                           int(K), err_ptr(q_local), at::cuda::getCurrentCUDAStream());
}

// GEMM-RS: a_q [world*S, K] fp8 (+ a_s_t [K/128, world*S]) -> out [S, N] bf16 (+ residual).
void fp8_gemm_rs(const Tensor& a_q, const Tensor& a_s_t, const Tensor& w, const Tensor& w_s,
                 const c10::optional<Tensor>& residual, Tensor& out, int64_t rank, int64_t world, int64_t call,
                 int64_t arrive_target, int64_t reuse_target, const std::vector<int64_t>& flags,
                 const std::vector<int64_t>& rb, int64_t epoch, int64_t arrive_inc, int64_t done_inc) {
  const int64_t M = a_q.size(0), K = a_q.size(1), N = w.size(0);
  TORCH_CHECK(M % world == 0, "rs: rows must split evenly");
  const int64_t S = M / world;
  TORCH_CHECK(out.size(0) == S && out.size(1) == N && out.is_contiguous(), "rs: out shape");
  c10::cuda::CUDAGuard guard(a_q.device());
  auto p = make_p2p(rank, world, S, call, arrive_target, reuse_target, flags, {}, {}, rb);
  set_epoch(p, epoch, arrive_inc, done_inc);
  p.reduce_grid = b200::rs_reduce_grid(int(S), int(N));
  const __nv_bfloat16* res = residual ? reinterpret_cast<const __nv_bfloat16*>(residual->data_ptr()) : nullptr;
  b200::launch_fp8_gemm_rs(p, reinterpret_cast<const uint8_t*>(a_q.data_ptr()), int(a_q.stride(0)),
                           a_s_t.data_ptr<float>(), int(a_s_t.stride(0)), reinterpret_cast<const uint8_t*>(w.data_ptr()),
                           int(w.stride(0)), w_s.data_ptr<float>(), int(M), int(N), int(K), res,
                           residual ? int(residual->stride(0)) : 0, reinterpret_cast<__nv_bfloat16*>(out.data_ptr()),
                           int(out.stride(0)), err_ptr(a_q), at::cuda::getCurrentCUDAStream());
}

void p2p_barrier(int64_t device, int64_t rank, int64_t world, int64_t call, const std::vector<int64_t>& flags,
                 int64_t wait_ns, int64_t epoch) {
  c10::cuda::CUDAGuard guard(static_cast<c10::DeviceIndex>(device));
  auto p = make_p2p(rank, world, 1, call, std::max<int64_t>(call, 1), 0, flags, {}, {}, {});
  set_epoch(p, epoch, 1, 0);
  TORCH_CHECK(wait_ns > 0, "p2p_barrier: wait budget must be positive");
  p.wait_ns = uint64_t(wait_ns);
  b200::launch_p2p_barrier(p, error_word_ref(int(device)).data_ptr<int>(), at::cuda::getCurrentCUDAStream());
}

int64_t symm_alloc(int64_t device, int64_t bytes) {
  c10::cuda::CUDAGuard guard(static_cast<c10::DeviceIndex>(device));
  return int64_t(b200::symm_alloc(size_t(bytes)));
}
void symm_free(int64_t device, int64_t ptr) {
  c10::cuda::CUDAGuard guard(static_cast<c10::DeviceIndex>(device));
  b200::symm_free(uintptr_t(ptr));
}
py::bytes symm_handle(int64_t device, int64_t ptr) {
  c10::cuda::CUDAGuard guard(static_cast<c10::DeviceIndex>(device));
  auto h = b200::symm_handle(uintptr_t(ptr));
  return py::bytes(reinterpret_cast<const char*>(h.data()), h.size());
}
int64_t symm_open(int64_t device, const std::string& handle) {
  c10::cuda::CUDAGuard guard(static_cast<c10::DeviceIndex>(device));
  return int64_t(b200::symm_open(std::vector<uint8_t>(handle.begin(), handle.end())));
}
void symm_close(int64_t device, int64_t ptr) {
  c10::cuda::CUDAGuard guard(static_cast<c10::DeviceIndex>(device));
  b200::symm_close(uintptr_t(ptr));
}
// A tensor view of device memory at `ptr` (no ownership; the heap owns it).
Tensor symm_view(int64_t device, int64_t ptr, int64_t bytes) {
  auto opts = torch::TensorOptions().dtype(torch::kUInt8).device(torch::kCUDA, device);
  return torch::from_blob(reinterpret_cast<void*>(ptr), {bytes}, [](void*) {}, opts);
}

}  // namespace

PYBIND11_MODULE(TORCH_EXTENSION_NAME, m) {
  m.doc() = "sm_100a kernels of the B200 DeepSeek-V3.2 DSA framework";
  m.def("error_word", &error_word);
  m.def("fp8_gemm", &fp8_gemm);
  m.def("bf16_gemm", &bf16_gemm);
  m.def("rms_norm", &rms_norm);
  m.def("quant_act", &quant_act);
  m.def("silu_mul_quant", &silu_mul_quant);
  m.def("mla_q_rope", &mla_q_rope);
  m.def("kv_finish", &kv_finish, py::arg("kv"), py::arg("L"), py::arg("R"), py::arg("norm_w"), py::arg("eps"),
        py::arg("freqs"), py::arg("positions"), py::arg("out"), py::arg("dst_row"), py::arg("packed") = py::none());
  m.def("index_k", &index_k);
  m.def("index_q", &index_q);
  m.def("q_rope_index_q", &q_rope_index_q);
  m.def("kv_finish_index_k", &kv_finish_index_k);
  m.def("linear_f32", &linear_f32);
  m.def("l2_prefetch", &l2_prefetch, py::arg("t"), py::arg("bytes") = int64_t(-1));
  m.def("set_pdl", [](bool on) { b200::pdl_flag() = on; },
        "programmatic dependent launch of the decode-path kernels (default on)");
  m.def("pdl_enabled", []() { return b200::pdl_flag(); });
  m.def("embed", &embed, py::arg("ids"), py::arg("table"), py::arg("out"), py::arg("row0") = int64_t(0),
        py::arg("vocab_total") = int64_t(0));
  m.def("indexer_logits", &indexer_logits);
  m.def("indexer_select", &indexer_select, py::arg("q"), py::arg("k"), py::arg("w"), py::arg("kscale"),
        py::arg("logits"), py::arg("query_start"), py::arg("topk"), py::arg("values"), py::arg("ids"),
        py::arg("index_order") = true, py::arg("sample_stride") = 32, py::arg("cand_cap") = 8192,
        py::arg("diag") = py::none());
  m.def("topk", &topk);
  m.def("sparse_mla", &sparse_mla);
  m.def("sparse_mla_scratch_bytes", &sparse_mla_scratch_bytes);
  m.def("sparse_mla_trace", &sparse_mla_trace);
  m.def("topk_trace", &topk_trace);
  m.def("fp8_gemm_splits", &fp8_gemm_splits, py::arg("M"), py::arg("N"), py::arg("K"), py::arg("ue8m0") = false);
  m.def("gather_rows", &gather_rows);
  m.def("pool_recall", &pool_recall);
  m.def("pool_select", &pool_select);
  m.def("pool_recall_select", &pool_recall_select);
  m.def("pool_recall_dispatch", &pool_recall_dispatch, py::arg("ids"), py::arg("hist_end"), py::arg("page_table"),
        py::arg("h2d"), py::arg("d2h"), py::arg("priority"), py::arg("meta"), py::arg("mark"), py::arg("miss_list"),
        py::arg("victims"), py::arg("stats"), py::arg("select_stats"), py::arg("k_limit"), py::arg("count_slot"),
        py::arg("host"), py::arg("records"), py::arg("fp8_scratch") = py::none());
  m.def("dequant_kv_rows", &dequant_kv_rows);
  m.def("pool_map", &pool_map);
  m.def("echo_predict", &echo_predict);
  m.def("echo_hint", &echo_hint);
  m.def("fp8_gemm_ag", &fp8_gemm_ag, py::arg("q_local"), py::arg("s_local_t"), py::arg("w"), py::arg("w_s"),
        py::arg("out"), py::arg("rank"), py::arg("world"), py::arg("call"), py::arg("arrive_target"),
        py::arg("reuse_target"), py::arg("flags"), py::arg("g"), py::arg("gs"), py::arg("epoch") = int64_t(0),
        py::arg("arrive_inc") = int64_t(0), py::arg("done_inc") = int64_t(0));
  m.def("fp8_gemm_rs", &fp8_gemm_rs, py::arg("a_q"), py::arg("a_s_t"), py::arg("w"), py::arg("w_s"),
        py::arg("residual"), py::arg("out"), py::arg("rank"), py::arg("world"), py::arg("call"),
        py::arg("arrive_target"), py::arg("reuse_target"), py::arg("flags"), py::arg("rb"),
        py::arg("epoch") = int64_t(0), py::arg("arrive_inc") = int64_t(0), py::arg("done_inc") = int64_t(0));
  m.def("set_fp8_gemm_pair_tiles", &b200::set_fp8_gemm_pair_tiles);
  m.def("set_decode_gemv", &b200::set_decode_gemv);
  m.def("set_gemv_k_split", &b200::set_gemv_k_split);
  m.def("p2p_barrier", &p2p_barrier, py::arg("device"), py::arg("rank"), py::arg("world"), py::arg("call"),
        py::arg("flags"), py::arg("wait_ns") = int64_t(2000000000), py::arg("epoch") = int64_t(0));
  m.def("sparse_mla_2sm_trace", &sparse_mla_2sm_trace);
  m.def("moe_route", &moe_route);
  m.def("ep_dispatch", &ep_dispatch);
  m.def("ep_combine", &ep_combine);
  m.def("moe_layout", &moe_layout);
  m.def("moe_gather", &moe_gather);
  m.def("moe_combine", &moe_combine);
  m.def("fp8_gemm_grouped", &fp8_gemm_grouped);
  m.def("fp8_gemm_grouped_push", &fp8_gemm_grouped_push);
  m.def("fp8_gemm_ag_grid", [](int64_t M, int64_t N, int64_t K) {
    return int64_t(b200::fp8_gemm_ag_grid(int(M), int(N), int(K)));
  });
  m.def("fp8_gemm_p2p_bn", [](int64_t M, int64_t N, int64_t K) {
    return int64_t(b200::fp8_gemm_p2p_bn(int(M), int(N), int(K)));
  });
  m.def("rs_reduce_grid", [](int64_t S, int64_t N) { return int64_t(b200::rs_reduce_grid(int(S), int(N))); });
  m.def("symm_alloc", &symm_alloc);
  m.def("symm_free", &symm_free);
  m.def("symm_handle", &symm_handle);
  m.def("symm_open", &symm_open);
  m.def("symm_close", &symm_close);
  m.def("symm_view", &symm_view);
}
