// Python bindings of the sm_100a kernels.  Only this file includes torch headers; the .cu
// files export plain C++ launchers so that they compile quickly and stay independent of torch.
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/extension.h>

#include <atomic>

#include "attention_sm100.h"
#include "comm.h"
#include "linear_attn.h"
#include "delta_prep.h"
#include "delta_scan.h"
#include "moe.h"
#include "moe_route.h"
#include "sparse_attn.h"
#include "sparse_teacher.h"
#include "nsa_compress.h"
#include "msar.h"
#include "plugin_ops.h"
#include "probe_sm100.h"
#include "residual.h"
#include "elementwise.h"
#include "gemm_sm100.h"
#include "optim.h"

namespace {

using torch::Tensor;
using OptT = c10::optional<Tensor>;

cudaStream_t stream() { return at::cuda::getCurrentCUDAStream().stream(); }

void check_cuda(const Tensor& t, const char* name) {
  TORCH_CHECK(t.is_cuda(), name, " must be a CUDA tensor");
}
void check_rows(const Tensor& t, const char* name) {
  check_cuda(t, name);
  TORCH_CHECK(t.is_contiguous(), name, " must be contiguous");
  TORCH_CHECK(reinterpret_cast<uintptr_t>(t.data_ptr()) % 16 == 0, name, " must be 16-byte aligned");
}
const void* ptr_or_null(const OptT& t) { return t.has_value() && t->defined() ? t->data_ptr() : nullptr; }
void* mptr_or_null(const OptT& t) { return t.has_value() && t->defined() ? t->data_ptr() : nullptr; }
void ok(int rc, const char* what) { TORCH_CHECK(rc == 0, what, ": unsupported shape"); }

int num_sms(const Tensor& t) {
  // cached per device for ids 0..63 (relaxed atomics: concurrent callers store the same value)
  static std::atomic<int> cached[64] = {};
  const int dev = t.get_device();
  if (dev < 0 || dev >= 64) return at::cuda::getDeviceProperties(dev)->multiProcessorCount;
  int v = cached[dev].load(std::memory_order_relaxed);
  if (!v) {
    v = at::cuda::getDeviceProperties(dev)->multiProcessorCount;
    cached[dev].store(v, std::memory_order_relaxed);
  }
  return v;
}

// ------------------------------------------------------------------ GEMM
// A logical [M,K] (stored [M,K] or, with a_mn, [K,M]); B logical [N,K] (stored [N,K] or, with
// b_mn, [K,N]); C [M,N].  2-D or 3-D (batched) tensors; the last dimension must be contiguous.
void gemm(const Tensor& A, bool a_mn, const Tensor& B, bool b_mn, const Tensor& C, int64_t epi, const OptT& R,
          const OptT& P, double s_acc, double s_res, const OptT& s_dev) {
  check_cuda(A, "A");
  check_cuda(B, "B");
  check_cuda(C, "C");
  TORCH_CHECK(A.scalar_type() == at::kBFloat16 && B.scalar_type() == at::kBFloat16, "gemm operands must be bf16");
  TORCH_CHECK(A.dim() == B.dim() && A.dim() == C.dim() && (A.dim() == 2 || A.dim() == 3), "gemm rank mismatch");
  TORCH_CHECK(A.stride(-1) == 1 && B.stride(-1) == 1 && C.stride(-1) == 1, "gemm needs unit inner stride");
  const bool batched = A.dim() == 3;
  GemmArgs g;
  g.batch = batched ? static_cast<int>(A.size(0)) : 1;
  g.M = static_cast<int>(C.size(-2));
  g.N = static_cast<int>(C.size(-1));
  g.K = static_cast<int>(a_mn ? A.size(-2) : A.size(-1));
  TORCH_CHECK((a_mn ? A.size(-1) : A.size(-2)) == g.M, "A rows != C rows");
  TORCH_CHECK((b_mn ? B.size(-1) : B.size(-2)) == g.N, "B rows != C cols");
  TORCH_CHECK((b_mn ? B.size(-2) : B.size(-1)) == g.K, "A/B reduction mismatch");
  g.A = A.data_ptr();
  g.lda = A.stride(-2);
  g.strideA = batched ? A.stride(0) : 0;
  g.a_mn = a_mn;
  g.B = B.data_ptr();
  g.ldb = B.stride(-2);
  g.strideB = batched ? B.stride(0) : 0;
  g.b_mn = b_mn;
  g.C = C.data_ptr();
  g.ldc = C.stride(-2);
  g.strideC = batched ? C.stride(0) : 0;
  const bool f32_out = epi == EPI_F32 || epi == EPI_F32_ACC;
  TORCH_CHECK(C.scalar_type() == (f32_out ? at::kFloat : at::kBFloat16), "gemm output dtype does not match epilogue");
  if (epi == EPI_BF16_AXPBY || epi == EPI_RELU2_BWD) {
    TORCH_CHECK(R.has_value() && R->defined(), "epilogue needs R");
    TORCH_CHECK(R->scalar_type() == at::kBFloat16 && R->stride(-1) == 1 && R->size(-1) == g.N && R->size(-2) == g.M,
                "R must be bf16 [.., M, N]");
    g.R = R->data_ptr();
    g.ldr = R->stride(-2);
    g.strideR = batched ? R->stride(0) : 0;
  }
  if (epi == EPI_RELU2) {
    TORCH_CHECK(P.has_value() && P->defined(), "relu2 epilogue needs P");
    TORCH_CHECK(P->scalar_type() == at::kBFloat16 && P->stride(-1) == 1 && P->size(-1) == g.N && P->size(-2) == g.M,
                "P must be bf16 [.., M, N]");
    g.P = P->data_ptr();
    g.ldp = P->stride(-2);
    g.strideP = batched ? P->stride(0) : 0;
  }
  g.s_acc = static_cast<float>(s_acc);
  g.s_res = static_cast<float>(s_res);
  if (s_dev.has_value() && s_dev->defined()) {
    TORCH_CHECK(s_dev->is_cuda() && s_dev->scalar_type() == at::kFloat && s_dev->numel() == 1, "s_dev: one fp32 value");
    g.s_ptr = s_dev->data_ptr<float>();
  }
  g.epi = static_cast<int>(epi);
  g.num_sms = num_sms(C);
  const c10::cuda::CUDAGuard guard(C.device());
  Tensor ws;
  const size_t ws_bytes = nt_gemm_splitk_bytes(g);
  if (ws_bytes) {
    // split-K partials live in a caching-allocator buffer for the duration of this call
    ws = at::empty({static_cast<int64_t>(ws_bytes / sizeof(float))}, C.options().dtype(at::kFloat));
    g.workspace = ws.data_ptr();
    g.workspace_bytes = ws_bytes;
  }
  nt_gemm_launch(g, stream());
}

// ------------------------------------------------------------------ norms
void mix_norm_fwd(const Tensor& x, const OptT& x0, const OptT& ab, const OptT& xm, const Tensor& h,
                  const OptT& rstd, double out_scale) {
  check_rows(x, "x");
  check_rows(h, "h");
  const int d = static_cast<int>(x.size(-1));
  const int M = static_cast<int>(x.numel() / d);
  if (x0.has_value() && x0->defined()) {
    check_rows(*x0, "x0");
    TORCH_CHECK(ab.has_value() && xm.has_value(), "mix needs ab and xm");
    check_rows(*xm, "xm");
  }
  ok(nt_mix_norm_fwd(x.data_ptr(), ptr_or_null(x0), ab.has_value() ? ab->data_ptr<float>() : nullptr, mptr_or_null(xm),
                     h.data_ptr(), rstd.has_value() ? rstd->data_ptr<float>() : nullptr, M, d,
                     static_cast<float>(out_scale), stream()),
     "mix_norm_fwd");
}

void norm_bwd(const Tensor& x, const Tensor& dy, const OptT& dres, const Tensor& dx) {
  check_rows(x, "x");
  check_rows(dy, "dy");
  check_rows(dx, "dx");
  if (dres.has_value() && dres->defined()) check_rows(*dres, "dres");
  const int d = static_cast<int>(x.size(-1));
  ok(nt_norm_bwd(x.data_ptr(), dy.data_ptr(), ptr_or_null(dres), dx.data_ptr(), static_cast<int>(x.numel() / d), d,
                 stream()),
     "norm_bwd");
}

void mix_norm_bwd(const Tensor& x, const Tensor& x0, const Tensor& xm, const Tensor& dh, const Tensor& dres,
                  const Tensor& ab, const Tensor& dx, const Tensor& dx0_acc, const Tensor& part) {
  for (auto* t : {&x, &x0, &xm, &dh, &dres, &dx, &dx0_acc}) check_rows(*t, "mix_norm_bwd operand");
  const int d = static_cast<int>(x.size(-1));
  ok(nt_mix_norm_bwd(x.data_ptr(), x0.data_ptr(), xm.data_ptr(), dh.data_ptr(), dres.data_ptr(), ab.data_ptr<float>(),
                     dx.data_ptr(), dx0_acc.data_ptr<float>(), part.data_ptr<float>(),
                     static_cast<int>(x.numel() / d), d, stream()),
     "mix_norm_bwd");
}

void rope_norm_fwd(const Tensor& qkv, const Tensor& cosb, const Tensor& sinb, const Tensor& rstd, int64_t T, int64_t H,
                   int64_t Hk, int64_t D, double scale, const OptT& ve_table, const OptT& idx, const OptT& hrow,
                   const OptT& wg, const OptT& gate_out) {
  check_rows(qkv, "qkv");
  const int M = static_cast<int>(qkv.numel() / ((H + 2 * Hk) * D));
  const bool ve = ve_table.has_value() && ve_table->defined();
  ok(nt_rope_norm_fwd(qkv.data_ptr(), cosb.data_ptr(), sinb.data_ptr(), rstd.data_ptr<float>(), M,
                      static_cast<int>(T), static_cast<int>(H), static_cast<int>(Hk), static_cast<int>(D),
                      static_cast<float>(scale), ve ? ve_table->data_ptr() : nullptr,
                      ve ? idx->data_ptr<int64_t>() : nullptr, ve ? hrow->data_ptr() : nullptr,
                      ve ? static_cast<int>(hrow->stride(-2)) : 0, ve ? wg->data_ptr() : nullptr,
                      ve ? static_cast<int>(wg->size(-1)) : 0, ve ? gate_out->data_ptr<float>() : nullptr, stream()),
     "rope_norm_fwd");
}

void rope_norm_bwd(const Tensor& dqkv, const Tensor& qkv, const Tensor& cosb, const Tensor& sinb, const Tensor& rstd,
                   int64_t T, int64_t H, int64_t Hk, int64_t D, double scale, const OptT& ve_table, const OptT& idx,
                   const OptT& gate, const OptT& dz, const OptT& ve_grad) {
  check_rows(dqkv, "dqkv");
  const int M = static_cast<int>(qkv.numel() / ((H + 2 * Hk) * D));
  const bool ve = ve_table.has_value() && ve_table->defined();
  ok(nt_rope_norm_bwd(dqkv.data_ptr(), qkv.data_ptr(), cosb.data_ptr(), sinb.data_ptr(), rstd.data_ptr<float>(), M,
                      static_cast<int>(T), static_cast<int>(H), static_cast<int>(Hk), static_cast<int>(D),
                      static_cast<float>(scale), ve ? ve_table->data_ptr() : nullptr,
                      ve ? idx->data_ptr<int64_t>() : nullptr, ve ? gate->data_ptr<float>() : nullptr,
                      ve ? dz->data_ptr<float>() : nullptr, ve ? ve_grad->data_ptr<float>() : nullptr, stream()),
     "rope_norm_bwd");
}

void softcap_ce(const Tensor& logits, const Tensor& tgt, const Tensor& loss, const OptT& lse, int64_t V, double cap,
                int64_t variant) {
  check_cuda(logits, "logits");
  TORCH_CHECK(logits.stride(-1) == 1 && reinterpret_cast<uintptr_t>(logits.data_ptr()) % 16 == 0, "logits layout");
  ok(nt_softcap_ce(logits.data_ptr(), logits.stride(-2), tgt.data_ptr<int64_t>(), loss.data_ptr<float>(),
                   lse.has_value() ? lse->data_ptr<float>() : nullptr, static_cast<int>(logits.size(-2)),
                   static_cast<int>(V), static_cast<int>(logits.size(-1)), static_cast<float>(cap),
                   static_cast<int>(variant), stream()),
     "softcap_ce");
}

void embed_smear(const Tensor& wte, const Tensor& idx, const Tensor& wsm, const Tensor& lam, const Tensor& n_out,
                 const Tensor& x_out, const Tensor& gate_out, int64_t T) {
  check_rows(wte, "wte");
  check_rows(n_out, "n_out");
  check_rows(x_out, "x_out");
  const int d = static_cast<int>(wte.size(-1));
  ok(nt_embed_smear(wte.data_ptr(), idx.data_ptr<int64_t>(), wsm.data_ptr(), lam.data_ptr<float>(), n_out.data_ptr(),
                    x_out.data_ptr(), gate_out.data_ptr<float>(), static_cast<int>(idx.numel()), static_cast<int>(T), d,
                    static_cast<int>(wsm.numel()), stream()),
     "embed_smear");
}

void embed_scatter(const Tensor& dy, const Tensor& idx, const Tensor& grad) {
  check_cuda(dy, "dy");
  TORCH_CHECK(dy.is_contiguous() && grad.is_contiguous(), "embed_scatter layout");
  ok(nt_embed_scatter(dy.data_ptr(), dy.scalar_type() == at::kFloat, idx.data_ptr<int64_t>(), grad.data_ptr<float>(),
                      static_cast<int>(idx.numel()), static_cast<int>(grad.size(-1)), stream()),
     "embed_scatter");
}

void cast_bf16(const Tensor& src, const Tensor& dst) {
  TORCH_CHECK(src.is_contiguous() && dst.is_contiguous() && src.numel() == dst.numel(), "cast layout");
  ok(nt_cast_bf16(src.data_ptr<float>(), dst.data_ptr(), src.numel(), stream()), "cast_bf16");
}

// ------------------------------------------------------------------ optimizer
void adamw(const Tensor& p, const Tensor& g, const Tensor& m, const Tensor& v, const OptT& shadow, double lr,
           double b1, double b2, double eps, double wd, int64_t step) {
  TORCH_CHECK(p.is_contiguous() && g.is_contiguous() && m.is_contiguous() && v.is_contiguous(), "adamw layout");
  TORCH_CHECK(g.scalar_type() == at::kFloat && m.scalar_type() == at::kFloat, "adamw grad/state must be fp32");
  AdamWHyper h;
  h.lr = static_cast<float>(lr);
  h.beta1 = static_cast<float>(b1);
  h.beta2 = static_cast<float>(b2);
  h.eps = static_cast<float>(eps);
  h.wd = static_cast<float>(wd);
  h.bias1 = static_cast<float>(1.0 - std::pow(b1, static_cast<double>(step)));
  h.bias2 = static_cast<float>(1.0 - std::pow(b2, static_cast<double>(step)));
  ok(nt_adamw(p.data_ptr(), p.scalar_type() == at::kBFloat16, g.data_ptr<float>(), m.data_ptr<float>(),
              v.data_ptr<float>(), mptr_or_null(shadow), p.numel(), h, stream()),
     "adamw");
}

void muon_prep(const Tensor& grad_ptrs, const Tensor& mom_ptrs, const Tensor& X, const Tensor& rowss, double mu) {
  const int K = static_cast<int>(X.size(0)), m = static_cast<int>(X.size(1)), n = static_cast<int>(X.size(2));
  ok(nt_muon_prep(reinterpret_cast<float* const*>(grad_ptrs.data_ptr<int64_t>()),
                  reinterpret_cast<float* const*>(mom_ptrs.data_ptr<int64_t>()), X.data_ptr(), rowss.data_ptr<float>(), K,
                  m, n, static_cast<float>(mu), stream()),
     "muon_prep");
}

void muon_normalize(const Tensor& X, const Tensor& rowss, const Tensor& tot) {
  const int K = static_cast<int>(X.size(0)), m = static_cast<int>(X.size(1)), n = static_cast<int>(X.size(2));
  ok(nt_muon_normalize(X.data_ptr(), rowss.data_ptr<float>(), tot.data_ptr<float>(), K, m, n, stream()),
     "muon_normalize");
}

void muon_finish(const Tensor& X, const Tensor& red, const Tensor& tot, const Tensor& smb_ptrs, const Tensor& fscale,
                 const Tensor& param_ptrs, const OptT& shadow_ptrs, double beta2, double lr, double wd) {
  const int K = static_cast<int>(X.size(0)), m = static_cast<int>(X.size(1)), n = static_cast<int>(X.size(2));
  ok(nt_muon_finish(X.data_ptr(), red.data_ptr<float>(), tot.data_ptr<float>(),
                    reinterpret_cast<float* const*>(smb_ptrs.data_ptr<int64_t>()), fscale.data_ptr<float>(),
                    reinterpret_cast<float* const*>(param_ptrs.data_ptr<int64_t>()),
                    shadow_ptrs.has_value() ? reinterpret_cast<void* const*>(shadow_ptrs->data_ptr<int64_t>()) : nullptr,
                    K, m, n, static_cast<float>(beta2), static_cast<float>(lr), static_cast<float>(wd), stream()),
     "muon_finish");
}

// ------------------------------------------------------------------ attention
AttnArgs attn_args(const Tensor& q, const Tensor& k, const Tensor& v, const Tensor& o, const Tensor& lse, int64_t B,
                   int64_t T, int64_t H, int64_t Hk, int64_t D, int64_t window, double scale) {
  for (auto* t : {&q, &k, &v, &o}) {
    check_cuda(*t, "attention operand");
    TORCH_CHECK(t->scalar_type() == at::kBFloat16 && t->stride(-1) == 1, "attention operands: bf16, unit stride");
  }
  AttnArgs a;
  a.q = q.data_ptr(); a.k = k.data_ptr(); a.v = v.data_ptr(); a.o = o.data_ptr();
  a.lse = lse.data_ptr<float>();
  a.ldq = q.stride(-2); a.ldk = k.stride(-2); a.ldv = v.stride(-2); a.ldo = o.stride(-2);
  a.B = static_cast<int>(B); a.T = static_cast<int>(T); a.H = static_cast<int>(H); a.Hk = static_cast<int>(Hk);
  a.D = static_cast<int>(D);
  a.window = static_cast<int>(window);
  a.scale = static_cast<float>(scale);
  a.num_sms = num_sms(q);
  return a;
}

// q [B*T, >=H*D] (row stride ldq), k/v [B*T, >=Hk*D], o [B*T, H*D], lse [B, H, T]
void attn_fwd(const Tensor& q, const Tensor& k, const Tensor& v, const Tensor& o, const Tensor& lse, int64_t B,
              int64_t T, int64_t H, int64_t Hk, int64_t D, int64_t window, double scale) {
  AttnArgs a = attn_args(q, k, v, o, lse, B, T, H, Hk, D, window, scale);
  const c10::cuda::CUDAGuard guard(q.device());
  ok(nt_attention_fwd(a, stream()), "attention_fwd");
}

// the forward with the pipeline stamps of its first CTA in `trace` (int64 [4][64][8], zero-filled)
void attn_fwd_trace(const Tensor& q, const Tensor& k, const Tensor& v, const Tensor& o, const Tensor& lse, int64_t B,
                    int64_t T, int64_t H, int64_t Hk, int64_t D, int64_t window, double scale, const Tensor& trace) {
  AttnArgs a = attn_args(q, k, v, o, lse, B, T, H, Hk, D, window, scale);
  TORCH_CHECK(trace.scalar_type() == at::kLong && trace.numel() >= 4 * 64 * 8, "trace: int64 [4, 64, 8]");
  a.trace = reinterpret_cast<long long*>(trace.data_ptr<int64_t>());
  const c10::cuda::CUDAGuard guard(q.device());
  ok(nt_attention_fwd(a, stream()), "attention_fwd");
}

void attn_bwd(const Tensor& q, const Tensor& k, const Tensor& v, const Tensor& o, const Tensor& lse,
              const Tensor& dout, const Tensor& dq, const Tensor& dk, const Tensor& dv, const Tensor& dq_acc,
              const Tensor& delta, int64_t B, int64_t T, int64_t H, int64_t Hk, int64_t D, int64_t window,
              double scale, const OptT& trace, int64_t dq_slices) {
  AttnArgs a = attn_args(q, k, v, o, lse, B, T, H, Hk, D, window, scale);
  a.dq_slices = static_cast<int>(dq_slices);
  TORCH_CHECK(dq_acc.numel() >= (dq_slices ? dq_slices : 1) * B * T * H * D, "dq_acc too small");
  a.dout = dout.data_ptr(); a.lddo = dout.stride(-2);
  a.dq = dq.data_ptr(); a.dk = dk.data_ptr(); a.dv = dv.data_ptr();
  a.lddq = dq.stride(-2); a.lddk = dk.stride(-2); a.lddv = dv.stride(-2);
  a.dq_acc = dq_acc.data_ptr<float>();
  a.delta = delta.data_ptr<float>();
  a.trace = trace.has_value() && trace->defined() ? reinterpret_cast<long long*>(trace->data_ptr<int64_t>()) : nullptr;
  const c10::cuda::CUDAGuard guard(q.device());
  ok(nt_attention_bwd(a, stream()), "attention_bwd");
}

// Block-sparse attention (lists of 64-key blocks per query tile, see sparse_attn.h).
SparseAttnArgs sparse_args(const Tensor& q, const Tensor& k, const Tensor& v, const Tensor& lists, const Tensor& masks,
                           int64_t B, int64_t T, int64_t H, int64_t Hk, double scale) {
  for (auto* t : {&q, &k, &v}) {
    check_cuda(*t, "sparse attention operand");
    TORCH_CHECK(t->scalar_type() == at::kBFloat16 && t->stride(-1) == 1, "q / k / v: bf16 rows with unit inner stride");
  }
  TORCH_CHECK(lists.is_cuda() && lists.scalar_type() == at::kInt && lists.is_contiguous() && lists.dim() == 4,
              "lists: int32 [B, G, n_qt, Lmax]");
  TORCH_CHECK(masks.is_cuda() && masks.scalar_type() == at::kInt && masks.is_contiguous() && masks.dim() == 5 &&
                  masks.size(-1) == 4,
              "masks: int32 [B, G, n_qt, Lmax, 4]");
  TORCH_CHECK(lists.size(0) == B && lists.size(2) == (T + 127) / 128 && masks.size(3) == lists.size(3),
              "list shapes");
  SparseAttnArgs a;
  a.B = static_cast<int>(B); a.T = static_cast<int>(T); a.H = static_cast<int>(H); a.Hk = static_cast<int>(Hk);
  a.G = static_cast<int>(lists.size(1)); a.Lmax = static_cast<int>(lists.size(3));
  a.scale = static_cast<float>(scale);
  a.q = q.data_ptr(); a.ldq = q.stride(-2);
  a.k = k.data_ptr(); a.ldk = k.stride(-2);
  a.v = v.data_ptr(); a.ldv = v.stride(-2);
  a.lists = lists.data_ptr<int>();
  a.masks = reinterpret_cast<const uint32_t*>(masks.data_ptr<int>());
  return a;
}

void set_rel(SparseAttnArgs& a, const OptT& rel, const OptT& drel) {
  if (!(rel.has_value() && rel->defined())) return;
  TORCH_CHECK(rel->is_cuda() && rel->scalar_type() == at::kFloat && rel->is_contiguous() && rel->dim() == 4 &&
                  rel->size(0) == a.B && rel->size(1) == a.H && rel->size(2) == a.T && rel->size(3) >= a.T,
              "rel: contiguous fp32 [B, H, T, extent >= T]");
  a.rel = rel->data_ptr<float>();
  a.rel_extent = static_cast<int>(rel->size(3));
  if (drel.has_value() && drel->defined()) {
    TORCH_CHECK(drel->sizes() == rel->sizes() && drel->is_contiguous() && drel->scalar_type() == at::kFloat,
                "drel: like rel");
    a.drel = drel->data_ptr<float>();
  }
}

void sparse_attn_fwd(const Tensor& q, const Tensor& k, const Tensor& v, const Tensor& lists, const Tensor& masks,
                     const Tensor& o, const Tensor& lse, int64_t B, int64_t T, int64_t H, int64_t Hk, double scale,
                     const OptT& rel) {
  SparseAttnArgs a = sparse_args(q, k, v, lists, masks, B, T, H, Hk, scale);
  set_rel(a, rel, c10::nullopt);
  TORCH_CHECK(o.scalar_type() == at::kBFloat16 && o.stride(-1) == 1 && lse.scalar_type() == at::kFloat, "o / lse");
  a.o = reinterpret_cast<__nv_bfloat16*>(o.data_ptr()); a.ldo = o.stride(-2);
  a.lse = lse.data_ptr<float>();
  const c10::cuda::CUDAGuard guard(q.device());
  ok(nt_sparse_attn_fwd(a, stream()), "sparse_attn_fwd");
}

void sparse_attn_bwd(const Tensor& q, const Tensor& k, const Tensor& v, const Tensor& lists, const Tensor& masks,
                     const Tensor& lse, const Tensor& dout, const Tensor& delta, const Tensor& dq, const Tensor& dk_acc,
                     const Tensor& dv_acc, int64_t B, int64_t T, int64_t H, int64_t Hk, double scale,
                     const OptT& rel, const OptT& drel) {
  SparseAttnArgs a = sparse_args(q, k, v, lists, masks, B, T, H, Hk, scale);
  set_rel(a, rel, drel);
  TORCH_CHECK(!a.rel || a.drel, "the backward with a relative bias needs drel");
  TORCH_CHECK(dout.scalar_type() == at::kBFloat16 && dout.stride(-1) == 1 && dq.scalar_type() == at::kBFloat16 &&
                  dq.stride(-1) == 1,
              "dout / dq: bf16 rows");
  TORCH_CHECK(dk_acc.scalar_type() == at::kFloat && dv_acc.scalar_type() == at::kFloat && dk_acc.is_contiguous() &&
                  dv_acc.is_contiguous(),
              "dk / dv accumulators: contiguous fp32");
  a.lse = lse.data_ptr<float>();
  a.dout = dout.data_ptr(); a.lddo = dout.stride(-2);
  a.delta = delta.data_ptr<float>();
  a.dq = reinterpret_cast<__nv_bfloat16*>(dq.data_ptr()); a.lddq = dq.stride(-2);
  a.dk_acc = dk_acc.data_ptr<float>();
  a.dv_acc = dv_acc.data_ptr<float>();
  const c10::cuda::CUDAGuard guard(q.device());
  ok(nt_sparse_attn_bwd(a, stream()), "sparse_attn_bwd");
}

// LM head + soft-capped cross-entropy, forward: G = e (1 - t^2) for x = hf W^T (see EPI_CE_FWD),
// per-row partial sums and target logits, then the row statistics.
void gemm_ce_fwd(const Tensor& hf, const Tensor& w, const Tensor& G, const Tensor& tgt, const Tensor& part,
                 const Tensor& ztgt, const Tensor& loss, const Tensor& rscale, const Tensor& rcorr, int64_t vocab,
                 double cap) {
  for (auto* t : {&hf, &w, &G}) check_rows(*t, "ce operand");
  for (auto* t : {&tgt, &part, &ztgt, &loss, &rscale, &rcorr}) check_rows(*t, "ce row vector");
  TORCH_CHECK(hf.scalar_type() == at::kBFloat16 && w.scalar_type() == at::kBFloat16 && G.scalar_type() == at::kBFloat16,
              "ce operands must be bf16");
  TORCH_CHECK(tgt.scalar_type() == at::kLong, "targets must be int64");
  GemmArgs g;
  g.M = static_cast<int>(hf.size(0));
  g.N = static_cast<int>(w.size(0));
  g.K = static_cast<int>(hf.size(1));
  TORCH_CHECK(w.size(1) == g.K && G.size(0) == g.M && G.size(1) == g.N, "ce shapes");
  const int nparts = (g.N + 127) / 128;
  TORCH_CHECK(part.numel() == static_cast<int64_t>(g.M) * nparts, "ce part must be [rows, ceil(N/128)]");
  g.A = hf.data_ptr(); g.lda = hf.stride(0);
  g.B = w.data_ptr(); g.ldb = w.stride(0);
  g.C = G.data_ptr(); g.ldc = G.stride(0);
  g.epi = EPI_CE_FWD;
  g.num_sms = num_sms(hf);
  g.ce.tgt = tgt.data_ptr<int64_t>();
  g.ce.part = part.data_ptr<float>();
  g.ce.ztgt = ztgt.data_ptr<float>();
  g.ce.vocab = static_cast<int>(vocab);
  g.ce.cap = static_cast<float>(cap);
  const c10::cuda::CUDAGuard guard(hf.device());
  nt_gemm_launch(g, stream());
  ok(nt_ce_finish(g.ce.part, nparts, g.ce.tgt, g.ce.ztgt, loss.data_ptr<float>(), rscale.data_ptr<float>(),
                  rcorr.data_ptr<float>(), g.M, g.ce.cap, stream()),
     "ce_finish");
}

// Input gradient of the head: dh = s (rscale G W - rcorr W[target]) (see EPI_CE_DGRAD).
void gemm_ce_dgrad(const Tensor& G, const Tensor& w, const Tensor& dh, const Tensor& tgt, const Tensor& rscale,
                   const Tensor& rcorr, const Tensor& s_dev) {
  for (auto* t : {&G, &w, &dh}) check_rows(*t, "ce operand");
  GemmArgs g;
  g.M = static_cast<int>(G.size(0));
  g.K = static_cast<int>(G.size(1));
  g.N = static_cast<int>(w.size(1));
  TORCH_CHECK(w.size(0) == g.K && dh.size(0) == g.M && dh.size(1) == g.N, "ce dgrad shapes");
  g.A = G.data_ptr(); g.lda = G.stride(0);
  g.B = w.data_ptr(); g.ldb = w.stride(0); g.b_mn = 1;
  g.C = dh.data_ptr(); g.ldc = dh.stride(0);
  g.epi = EPI_CE_DGRAD;
  g.s_ptr = s_dev.data_ptr<float>();
  g.num_sms = num_sms(G);
  g.ce.tgt = tgt.data_ptr<int64_t>();
  g.ce.rscale = rscale.data_ptr<float>();
  g.ce.rcorr = rcorr.data_ptr<float>();
  g.ce.w = w.data_ptr();
  g.ce.ldw = w.stride(0);
  const c10::cuda::CUDAGuard guard(G.device());
  nt_gemm_launch(g, stream());
}

// Reduce-scatter over symmetric memory (see comm.h); pointer tables are int64 CUDA tensors.
void p2p_reduce_scatter(const Tensor& peers, const Tensor& pads, const Tensor& seg_off, const Tensor& seg_len,
                        int64_t rank, int64_t world, double scale, int64_t epoch, int64_t blocks, double timeout_s) {
  for (auto* t : {&peers, &pads, &seg_off, &seg_len}) {
    check_cuda(*t, "p2p table");
    TORCH_CHECK(t->scalar_type() == at::kLong && t->is_contiguous(), "p2p tables must be contiguous int64");
  }
  TORCH_CHECK(peers.numel() == world && pads.numel() == world && seg_off.numel() == seg_len.numel(), "p2p table sizes");
  const c10::cuda::CUDAGuard guard(peers.device());
  ok(nt_p2p_reduce_scatter(reinterpret_cast<const uint64_t*>(peers.data_ptr<int64_t>()),
                           reinterpret_cast<const uint64_t*>(pads.data_ptr<int64_t>()), seg_off.data_ptr<int64_t>(),
                           seg_len.data_ptr<int64_t>(), static_cast<int>(seg_off.numel()), static_cast<int>(rank),
                           static_cast<int>(world), static_cast<float>(scale), static_cast<uint32_t>(epoch),
                           static_cast<int>(blocks), static_cast<uint64_t>(timeout_s * 1e9), stream()),
     "p2p_reduce_scatter");
}

// ------------------------------------------------------------------ grouped (expert) GEMM
// k_mode false: A [M, K] (or [K, M] with a_mn), B a stack [E, N, K] (or [E, K, N] with b_mn),
//   C [M, N]; grp int32 [ceil(M / 128)] names the expert of every 128-row tile (-1: empty).
// k_mode true: A [K, M] / [M, K], B [K, N] / [N, K] (single matrices), C fp32 [E, M, N] accumulated
//   (EPI_F32_ACC); grp int32 [E + 1] row offsets of each expert along K (multiples of 64).
void gemm_grouped(const Tensor& A, bool a_mn, const Tensor& B, bool b_mn, const Tensor& C, int64_t epi,
                  const Tensor& grp, bool k_mode, const OptT& R, const OptT& P, double s_acc) {
  check_cuda(A, "A");
  check_cuda(B, "B");
  check_cuda(C, "C");
  TORCH_CHECK(grp.is_cuda() && grp.scalar_type() == at::kInt && grp.is_contiguous(), "grp must be int32 CUDA");
  TORCH_CHECK(A.scalar_type() == at::kBFloat16 && B.scalar_type() == at::kBFloat16, "gemm operands must be bf16");
  TORCH_CHECK(A.stride(-1) == 1 && B.stride(-1) == 1 && C.stride(-1) == 1, "gemm needs unit inner stride");
  GemmArgs g;
  if (!k_mode) {
    TORCH_CHECK(A.dim() == 2 && B.dim() == 3 && C.dim() == 2, "grouped-M: A 2-D, B 3-D, C 2-D");
    g.groups = static_cast<int>(B.size(0));
    g.M = static_cast<int>(C.size(0));
    g.N = static_cast<int>(C.size(1));
    TORCH_CHECK(grp.numel() >= (g.M + 127) / 128, "grp too short");
    g.grp_m = grp.data_ptr<int>();
    g.strideB = B.stride(0);
  } else {
    TORCH_CHECK(A.dim() == 2 && B.dim() == 2 && C.dim() == 3, "grouped-K: A 2-D, B 2-D, C 3-D");
    TORCH_CHECK(epi == EPI_F32_ACC, "grouped-K accumulates (EPI_F32_ACC)");
    g.groups = static_cast<int>(C.size(0));
    g.M = static_cast<int>(C.size(1));
    g.N = static_cast<int>(C.size(2));
    TORCH_CHECK(grp.numel() == g.groups + 1, "grp must hold E + 1 offsets");
    g.grp_k = grp.data_ptr<int>();
    g.strideC = C.stride(0);
  }
  g.K = static_cast<int>(a_mn ? A.size(-2) : A.size(-1));
  TORCH_CHECK((a_mn ? A.size(-1) : A.size(-2)) == g.M, "A rows != C rows");
  TORCH_CHECK((b_mn ? B.size(-1) : B.size(-2)) == g.N, "B rows != C cols");
  TORCH_CHECK((b_mn ? B.size(-2) : B.size(-1)) == g.K, "A/B reduction mismatch");
  g.A = A.data_ptr();
  g.lda = A.stride(-2);
  g.a_mn = a_mn;
  g.B = B.data_ptr();
  g.ldb = B.stride(-2);
  g.b_mn = b_mn;
  g.C = C.data_ptr();
  g.ldc = C.stride(-2);
  const bool f32_out = epi == EPI_F32 || epi == EPI_F32_ACC;
  TORCH_CHECK(C.scalar_type() == (f32_out ? at::kFloat : at::kBFloat16), "gemm output dtype does not match epilogue");
  if (epi == EPI_RELU2_BWD) {
    TORCH_CHECK(R.has_value() && R->defined() && R->scalar_type() == at::kBFloat16 && R->stride(-1) == 1 &&
                    R->dim() == 2 && R->size(0) == g.M && R->size(1) == g.N,
                "R must be bf16 [M, N]");
    g.R = R->data_ptr();
    g.ldr = R->stride(0);
  }
  if (epi == EPI_RELU2) {
    TORCH_CHECK(P.has_value() && P->defined() && P->scalar_type() == at::kBFloat16 && P->stride(-1) == 1 &&
                    P->dim() == 2 && P->size(0) == g.M && P->size(1) == g.N,
                "P must be bf16 [M, N]");
    g.P = P->data_ptr();
    g.ldp = P->stride(0);
  }
  TORCH_CHECK(epi == EPI_BF16 || epi == EPI_RELU2 || epi == EPI_RELU2_BWD || epi == EPI_F32 || epi == EPI_F32_ACC,
              "grouped GEMM epilogue");
  g.s_acc = static_cast<float>(s_acc);
  g.epi = static_cast<int>(epi);
  g.num_sms = num_sms(C);
  const c10::cuda::CUDAGuard guard(C.device());
  nt_gemm_launch(g, stream());
}

// ------------------------------------------------------------------ peer barrier / put
void p2p_barrier(const Tensor& pads, int64_t rank, int64_t world, int64_t epoch, double timeout_s) {
  TORCH_CHECK(pads.is_cuda() && pads.scalar_type() == at::kLong, "pads: int64 CUDA pointer table");
  const c10::cuda::CUDAGuard guard(pads.device());
  ok(nt_p2p_barrier(reinterpret_cast<const uint64_t*>(pads.data_ptr<int64_t>()), static_cast<int>(rank),
                    static_cast<int>(world), static_cast<uint32_t>(epoch), static_cast<uint64_t>(timeout_s * 1e9),
                    stream()),
     "p2p_barrier");
}

void p2p_gather(const Tensor& peers, const Tensor& pads, const Tensor& seg_off, const Tensor& seg_len,
                const Tensor& seg_owner, const Tensor& seg_shadow, int64_t rank, int64_t world, int64_t epoch,
                int64_t blocks, double timeout_s) {
  for (auto* t : {&peers, &pads, &seg_off, &seg_len, &seg_shadow})
    TORCH_CHECK(t->is_cuda() && t->scalar_type() == at::kLong && t->is_contiguous(), "p2p_gather tables: int64 CUDA");
  TORCH_CHECK(seg_owner.is_cuda() && seg_owner.scalar_type() == at::kInt, "seg_owner: int32 CUDA");
  const c10::cuda::CUDAGuard guard(peers.device());
  ok(nt_p2p_gather(reinterpret_cast<const uint64_t*>(peers.data_ptr<int64_t>()),
                   reinterpret_cast<const uint64_t*>(pads.data_ptr<int64_t>()), seg_off.data_ptr<int64_t>(),
                   seg_len.data_ptr<int64_t>(), seg_owner.data_ptr<int>(),
                   reinterpret_cast<const uint64_t*>(seg_shadow.data_ptr<int64_t>()), static_cast<int>(seg_off.numel()),
                   static_cast<int>(rank), static_cast<int>(world), static_cast<uint32_t>(epoch), static_cast<int>(blocks),
                   static_cast<uint64_t>(timeout_s * 1e9), stream()),
     "p2p_gather");
}

void p2p_put(const Tensor& peers, int64_t world, int64_t dst_off, const Tensor& src) {
  TORCH_CHECK(peers.is_cuda() && peers.scalar_type() == at::kLong, "peers: int64 CUDA pointer table");
  TORCH_CHECK(src.is_cuda() && src.is_contiguous(), "src must be contiguous CUDA");
  const c10::cuda::CUDAGuard guard(src.device());
  ok(nt_p2p_put(reinterpret_cast<const uint64_t*>(peers.data_ptr<int64_t>()), static_cast<int>(world), dst_off,
                src.data_ptr(), src.numel() * src.element_size(), stream()),
     "p2p_put");
}

// ------------------------------------------------------------------ mHC Sinkhorn-Knopp
void sinkhorn_fwd(const Tensor& logits, const Tensor& out, int64_t iterations) {
  TORCH_CHECK(logits.is_cuda() && logits.scalar_type() == at::kFloat && logits.is_contiguous() && out.is_contiguous(),
              "sinkhorn: contiguous fp32 [.., n, n]");
  const int n = static_cast<int>(logits.size(-1));
  const c10::cuda::CUDAGuard guard(logits.device());
  ok(nt_sinkhorn_fwd(logits.data_ptr<float>(), out.data_ptr<float>(), logits.numel() / (n * n), n,
                     static_cast<int>(iterations), stream()),
     "sinkhorn_fwd");
}

void sinkhorn_bwd(const Tensor& logits, const Tensor& dout, const Tensor& dlogits, int64_t iterations) {
  TORCH_CHECK(logits.is_contiguous() && dout.is_contiguous() && dlogits.is_contiguous() &&
                  dout.scalar_type() == at::kFloat,
              "sinkhorn: contiguous fp32");
  const int n = static_cast<int>(logits.size(-1));
  const c10::cuda::CUDAGuard guard(logits.device());
  ok(nt_sinkhorn_bwd(logits.data_ptr<float>(), dout.data_ptr<float>(), dlogits.data_ptr<float>(),
                     logits.numel() / (n * n), n, static_cast<int>(iterations), stream()),
     "sinkhorn_bwd");
}

// ------------------------------------------------------------------ MoE row movement
void check_i32(const Tensor& t, const char* name) {
  TORCH_CHECK(t.is_cuda() && t.scalar_type() == at::kInt && t.is_contiguous(), name, " must be contiguous int32 CUDA");
}

void moe_gather_rows(const Tensor& src, const Tensor& src_of, const Tensor& out) {
  check_rows(src, "src");
  check_rows(out, "out");
  check_i32(src_of, "src_of");
  TORCH_CHECK(src_of.numel() == out.size(0) && src.size(-1) == out.size(-1), "gather shapes");
  const c10::cuda::CUDAGuard guard(out.device());
  ok(nt_moe_gather_rows(src.data_ptr(), src_of.data_ptr<int>(), out.data_ptr(), out.size(0), out.size(-1), stream()),
     "moe_gather_rows");
}

void moe_combine(const Tensor& rows, const Tensor& row_of, const OptT& w, const OptT& add, const Tensor& out) {
  check_rows(rows, "rows");
  check_rows(out, "out");
  check_i32(row_of, "row_of");
  const int T = static_cast<int>(out.size(0)), k = static_cast<int>(row_of.numel() / std::max<int64_t>(1, out.size(0)));
  const float* wp = nullptr;
  if (w.has_value() && w->defined()) {
    TORCH_CHECK(w->scalar_type() == at::kFloat && w->is_contiguous() && w->numel() == row_of.numel(), "w: fp32 [T, k]");
    wp = w->data_ptr<float>();
  }
  const void* ap = nullptr;
  if (add.has_value() && add->defined()) {
    check_rows(*add, "add");
    ap = add->data_ptr();
  }
  const c10::cuda::CUDAGuard guard(out.device());
  ok(nt_moe_combine(rows.data_ptr(), row_of.data_ptr<int>(), wp, ap, out.data_ptr(), T, k,
                    static_cast<int>(out.size(-1)), stream()),
     "moe_combine");
}

void moe_combine_bwd(const Tensor& dy, const Tensor& rows, const Tensor& row_of, const Tensor& w, const Tensor& d_rows,
                     const Tensor& dw) {
  check_rows(dy, "dy");
  check_rows(rows, "rows");
  check_rows(d_rows, "d_rows");
  check_i32(row_of, "row_of");
  TORCH_CHECK(w.scalar_type() == at::kFloat && dw.scalar_type() == at::kFloat && w.is_contiguous() && dw.is_contiguous(),
              "w / dw fp32");
  const int T = static_cast<int>(dy.size(0)), k = static_cast<int>(row_of.numel() / std::max<int64_t>(1, dy.size(0)));
  const c10::cuda::CUDAGuard guard(dy.device());
  ok(nt_moe_combine_bwd(dy.data_ptr(), rows.data_ptr(), row_of.data_ptr<int>(), w.data_ptr<float>(), d_rows.data_ptr(),
                        dw.data_ptr<float>(), T, k, static_cast<int>(dy.size(-1)), stream()),
     "moe_combine_bwd");
}

// Fused routing: (choice, w, lse, row_of, src_of, grp_m, grp_k, counts, aux_grad, aux[2]) of fp32
// logits [N, E]; P rows of padded layout.
std::vector<Tensor> moe_route(const Tensor& logits, const OptT& bias, int64_t k, double aux_coeff, double z_coeff,
                              const OptT& load) {
  check_rows(logits, "logits");
  TORCH_CHECK(logits.scalar_type() == at::kFloat && logits.dim() == 2, "router logits must be fp32 [N, E]");
  const int N = static_cast<int>(logits.size(0)), E = static_cast<int>(logits.size(1)), K = static_cast<int>(k);
  const int nblk = (N + NT_ROUTE_TOKENS - 1) / NT_ROUTE_TOKENS;
  const int64_t P = (static_cast<int64_t>(N) * K + NT_ROUTE_PAD - 1) / NT_ROUTE_PAD * NT_ROUTE_PAD +
                    static_cast<int64_t>(NT_ROUTE_PAD) * E;
  auto i32 = logits.options().dtype(at::kInt);
  auto f32 = logits.options();
  Tensor choice = torch::empty({N, K}, i32), w = torch::empty({N, K}, f32), lse = torch::empty({N}, f32);
  Tensor blk_counts = torch::empty({nblk, E}, i32), blk_offset = torch::empty({nblk, E}, i32);
  Tensor blk_probs = torch::empty({nblk, E}, f32), blk_z = torch::empty({nblk}, f32);
  Tensor counts = torch::empty({E}, i32), seg = torch::empty({E}, i32), grp_k = torch::empty({E + 1}, i32);
  Tensor grp_m = torch::empty({P / NT_ROUTE_PAD}, i32), row_of = torch::empty({static_cast<int64_t>(N) * K}, i32);
  Tensor src_of = torch::empty({P}, i32), aux_grad = torch::empty({E}, f32), aux = torch::empty({2}, f32);
  if (bias.has_value() && bias->defined())
    TORCH_CHECK(bias->scalar_type() == at::kFloat && bias->numel() == E && bias->is_contiguous(), "bias: fp32 [E]");
  if (load.has_value() && load->defined())
    TORCH_CHECK(load->scalar_type() == at::kFloat && load->numel() == E && load->is_contiguous(), "load: fp32 [E]");
  MoeRouteArgs a;
  a.N = N;
  a.E = E;
  a.k = K;
  a.P = static_cast<int>(P);
  a.logits = logits.data_ptr<float>();
  a.bias = static_cast<const float*>(ptr_or_null(bias));
  a.aux_coeff = static_cast<float>(aux_coeff);
  a.z_coeff = static_cast<float>(z_coeff);
  a.choice = choice.data_ptr<int>();
  a.w = w.data_ptr<float>();
  a.lse = lse.data_ptr<float>();
  a.blk_counts = blk_counts.data_ptr<int>();
  a.blk_probs = blk_probs.data_ptr<float>();
  a.blk_z = blk_z.data_ptr<float>();
  a.counts = counts.data_ptr<int>();
  a.seg_start = seg.data_ptr<int>();
  a.blk_offset = blk_offset.data_ptr<int>();
  a.grp_m = grp_m.data_ptr<int>();
  a.grp_k = grp_k.data_ptr<int>();
  a.row_of = row_of.data_ptr<int>();
  a.src_of = src_of.data_ptr<int>();
  a.load = static_cast<float*>(mptr_or_null(load));
  a.aux_grad = aux_grad.data_ptr<float>();
  a.aux = aux.data_ptr<float>();
  ok(nt_moe_route(a, stream()), "moe_route");
  return {choice, w, lse, row_of, src_of, grp_m, grp_k, counts, aux_grad, aux};
}

Tensor moe_route_bwd(const Tensor& logits, const Tensor& lse, const Tensor& choice, const Tensor& w, const OptT& dw,
                     const Tensor& aux_grad, const OptT& daux, double z_coeff) {
  check_rows(logits, "logits");
  if (dw.has_value() && dw->defined())
    TORCH_CHECK(dw->scalar_type() == at::kFloat && dw->is_contiguous() && dw->sizes() == w.sizes(), "dw: fp32 like w");
  if (daux.has_value() && daux->defined())
    TORCH_CHECK(daux->scalar_type() == at::kFloat && daux->numel() == 1 && daux->is_cuda(), "daux: fp32 device scalar");
  Tensor d = torch::empty_like(logits);
  ok(nt_moe_route_bwd(logits.data_ptr<float>(), lse.data_ptr<float>(), choice.data_ptr<int>(), w.data_ptr<float>(),
                      static_cast<const float*>(ptr_or_null(dw)), aux_grad.data_ptr<float>(),
                      static_cast<const float*>(ptr_or_null(daux)),
                      static_cast<float>(z_coeff), d.data_ptr<float>(), static_cast<int>(logits.size(0)),
                      static_cast<int>(logits.size(1)), static_cast<int>(choice.size(1)), stream()),
     "moe_route_bwd");
  return d;
}

// Head-mean teacher [B, Q, T] fp32 of q [B, H, Q, 128] and k [B, Hk, T, 128] (bf16, any strides with a
// unit feature stride); mask [B, Q, T] bool / uint8 or None (causal only).
Tensor sparse_teacher(const Tensor& q, const Tensor& k, const OptT& mask, int64_t q_start, double scale) {
  check_cuda(q, "q");
  check_cuda(k, "k");
  TORCH_CHECK(q.scalar_type() == at::kBFloat16 && k.scalar_type() == at::kBFloat16, "teacher: bf16 q and k");
  TORCH_CHECK(q.dim() == 4 && k.dim() == 4 && q.stride(3) == 1 && k.stride(3) == 1, "teacher: [B, H, L, D] views");
  TeacherArgs a;
  a.B = static_cast<int>(q.size(0));
  a.H = static_cast<int>(q.size(1));
  a.Q = static_cast<int>(q.size(2));
  a.D = static_cast<int>(q.size(3));
  a.Hk = static_cast<int>(k.size(1));
  a.T = static_cast<int>(k.size(2));
  a.q_start = static_cast<int>(q_start);
  a.scale = static_cast<float>(scale);
  a.q = reinterpret_cast<const __nv_bfloat16*>(q.data_ptr());
  a.sqb = q.stride(0);
  a.sqh = q.stride(1);
  a.sqt = q.stride(2);
  a.k = reinterpret_cast<const __nv_bfloat16*>(k.data_ptr());
  a.skb = k.stride(0);
  a.skh = k.stride(1);
  a.skt = k.stride(2);
  Tensor m;
  if (mask.has_value() && mask->defined()) {
    TORCH_CHECK(mask->dim() == 3 && mask->size(0) == a.B && mask->size(1) == a.Q && mask->size(2) == a.T,
                "teacher: mask [B, Q, T]");
    m = mask->to(at::kByte).contiguous();
    a.mask = m.data_ptr<uint8_t>();
  }
  Tensor lse = torch::empty({a.B, a.H, a.Q}, q.options().dtype(at::kFloat));
  Tensor out = torch::zeros({a.B, a.Q, a.T}, q.options().dtype(at::kFloat));
  a.lse = lse.data_ptr<float>();
  a.out = out.data_ptr<float>();
  ok(nt_sparse_teacher(a, stream()), "sparse_teacher");
  return out;
}

// NSA compressed branch: q [B, T, H, 128], ck / cv [B, Nc, Hk, 128] bf16 contiguous.
static NsaArgs nsa_args(const Tensor& q, const Tensor& ck, const Tensor& cv, int64_t cstride, int64_t csize,
                        int64_t ssize, int64_t topk, double scale) {
  for (const Tensor* t : {&q, &ck, &cv}) {
    check_rows(*t, "nsa operand");
    TORCH_CHECK(t->scalar_type() == at::kBFloat16 && t->dim() == 4, "nsa operands: bf16 [B, L, heads, 128]");
  }
  NsaArgs a;
  a.B = static_cast<int>(q.size(0));
  a.T = static_cast<int>(q.size(1));
  a.H = static_cast<int>(q.size(2));
  a.D = static_cast<int>(q.size(3));
  a.Nc = static_cast<int>(ck.size(1));
  a.Hk = static_cast<int>(ck.size(2));
  a.cstride = static_cast<int>(cstride);
  a.csize = static_cast<int>(csize);
  a.ssize = static_cast<int>(ssize);
  a.topk = static_cast<int>(topk);
  a.scale = static_cast<float>(scale);
  a.q = reinterpret_cast<const __nv_bfloat16*>(q.data_ptr());
  a.k = reinterpret_cast<const __nv_bfloat16*>(ck.data_ptr());
  a.v = reinterpret_cast<const __nv_bfloat16*>(cv.data_ptr());
  return a;
}

std::vector<Tensor> nsa_compressed_fwd(const Tensor& q, const Tensor& ck, const Tensor& cv, int64_t cstride,
                                       int64_t csize, int64_t ssize, int64_t topk, double scale) {
  NsaArgs a = nsa_args(q, ck, cv, cstride, csize, ssize, topk, scale);
  const int64_t nsel = (a.T + a.ssize - 1) / a.ssize;
  Tensor o = torch::empty_like(q);
  Tensor lse = torch::empty({a.B, a.H, a.T}, q.options().dtype(at::kFloat));
  Tensor sel = torch::empty({a.B, a.H, a.T, nsel}, q.options().dtype(at::kByte));
  a.o = reinterpret_cast<__nv_bfloat16*>(o.data_ptr());
  a.lse = lse.data_ptr<float>();
  a.sel = sel.data_ptr<uint8_t>();
  ok(nt_nsa_compressed_fwd(a, stream()), "nsa_compressed_fwd");
  return {o, lse, sel};
}

std::vector<Tensor> nsa_compressed_bwd(const Tensor& q, const Tensor& ck, const Tensor& cv, const Tensor& lse,
                                       const Tensor& dout, const Tensor& delta, int64_t cstride, int64_t csize,
                                       double scale) {
  NsaArgs a = nsa_args(q, ck, cv, cstride, csize, 64, 0, scale);
  check_rows(dout, "dout");
  TORCH_CHECK(dout.sizes() == q.sizes() && dout.scalar_type() == at::kBFloat16, "dout like q");
  TORCH_CHECK(lse.is_contiguous() && delta.is_contiguous() && lse.scalar_type() == at::kFloat &&
              delta.scalar_type() == at::kFloat, "lse / delta: fp32 [B, H, T]");
  Tensor dq = torch::zeros(q.sizes(), q.options().dtype(at::kFloat));
  Tensor dk = torch::zeros(ck.sizes(), ck.options().dtype(at::kFloat));
  Tensor dv = torch::zeros(cv.sizes(), cv.options().dtype(at::kFloat));
  a.lse = const_cast<float*>(lse.data_ptr<float>());
  a.dout = reinterpret_cast<const __nv_bfloat16*>(dout.data_ptr());
  a.delta = delta.data_ptr<float>();
  a.dq_acc = dq.data_ptr<float>();
  a.dk_acc = dk.data_ptr<float>();
  a.dv_acc = dv.data_ptr<float>();
  ok(nt_nsa_compressed_bwd(a, stream()), "nsa_compressed_bwd");
  return {dq, dk, dv};
}

// MSAR temporal augmentation: x [B, T, C] (bf16 / fp32), taps fp32 [C, 24] -> y [B, T, 4, C]
Tensor msar_temporal_fwd(const Tensor& x, const Tensor& taps) {
  check_rows(x, "x");
  TORCH_CHECK(x.dim() == 3 && (x.scalar_type() == at::kBFloat16 || x.scalar_type() == at::kFloat), "x: [B, T, C]");
  TORCH_CHECK(taps.scalar_type() == at::kFloat && taps.is_contiguous() && taps.size(0) == x.size(2) &&
              taps.size(1) == 24, "taps: fp32 [C, 24]");
  MsarTemporalArgs a;
  a.B = static_cast<int>(x.size(0));
  a.T = static_cast<int>(x.size(1));
  a.C = static_cast<int>(x.size(2));
  a.bf16 = x.scalar_type() == at::kBFloat16;
  Tensor y = torch::empty({a.B, a.T, 4, a.C}, x.options());
  a.x = x.data_ptr();
  a.taps = taps.data_ptr<float>();
  a.y = y.data_ptr();
  ok(nt_msar_temporal_fwd(a, stream()), "msar_temporal_fwd");
  return y;
}

std::vector<Tensor> msar_temporal_bwd(const Tensor& x, const Tensor& taps, const Tensor& dy) {
  check_rows(x, "x");
  check_rows(dy, "dy");
  TORCH_CHECK(dy.scalar_type() == x.scalar_type() && dy.dim() == 4 && dy.size(2) == 4, "dy like y");
  MsarTemporalArgs a;
  a.B = static_cast<int>(x.size(0));
  a.T = static_cast<int>(x.size(1));
  a.C = static_cast<int>(x.size(2));
  a.bf16 = x.scalar_type() == at::kBFloat16;
  Tensor dx = torch::empty_like(x);
  Tensor part = torch::empty({nt_msar_temporal_part_floats(a.B, a.T, a.C)}, x.options().dtype(at::kFloat));
  Tensor dtaps = torch::empty({a.C, 24}, x.options().dtype(at::kFloat));
  a.x = x.data_ptr();
  a.taps = taps.data_ptr<float>();
  a.dy = dy.data_ptr();
  a.dx = dx.data_ptr();
  a.part = part.data_ptr<float>();
  a.dtaps = dtaps.data_ptr<float>();
  ok(nt_msar_temporal_bwd(a, stream()), "msar_temporal_bwd");
  return {dx, dtaps};
}

// MSAR depth-read gate: s [N, 4, C], P fp32 [4C, 4], alpha fp32 [1], bias fp32 [4] -> (out [N, C], zr [N, 5])
std::vector<Tensor> msar_gate_fwd(const Tensor& s, const Tensor& P, const Tensor& alpha, const Tensor& bias) {
  check_rows(s, "s");
  TORCH_CHECK(s.dim() == 3 && s.size(1) == 4, "s: [N, 4, C]");
  TORCH_CHECK(P.scalar_type() == at::kFloat && P.is_contiguous() && P.size(0) == 4 * s.size(2) && P.size(1) == 4,
              "P: fp32 [4C, 4]");
  MsarGateArgs a;
  a.N = static_cast<int>(s.size(0));
  a.C = static_cast<int>(s.size(2));
  a.bf16 = s.scalar_type() == at::kBFloat16;
  Tensor out = torch::empty({a.N, a.C}, s.options());
  Tensor zr = torch::empty({a.N, 5}, s.options().dtype(at::kFloat));
  a.s = s.data_ptr();
  a.P = P.data_ptr<float>();
  a.alpha = alpha.data_ptr<float>();
  a.bias = bias.data_ptr<float>();
  a.out = out.data_ptr();
  a.zr = zr.data_ptr<float>();
  ok(nt_msar_gate_fwd(a, stream()), "msar_gate_fwd");
  return {out, zr};
}

// -> (ds [N, 4, C], dP [4C, 4], dalpha [1], dbias [4]); the token reductions are fixed-order sums
std::vector<Tensor> msar_gate_bwd(const Tensor& s, const Tensor& P, const Tensor& alpha, const Tensor& bias,
                                  const Tensor& zr, const Tensor& dout) {
  check_rows(s, "s");
  check_rows(dout, "dout");
  MsarGateArgs a;
  a.N = static_cast<int>(s.size(0));
  a.C = static_cast<int>(s.size(2));
  a.bf16 = s.scalar_type() == at::kBFloat16;
  auto f32 = s.options().dtype(at::kFloat);
  Tensor ds = torch::empty_like(s), y = torch::empty({a.N, 4}, f32), ab = torch::empty({a.N, 5}, f32);
  Tensor pp = torch::empty({nt_msar_gate_proj_slices(a.N), 4 * a.C, 4}, f32);
  a.s = s.data_ptr();
  a.P = P.data_ptr<float>();
  a.alpha = alpha.data_ptr<float>();
  a.bias = bias.data_ptr<float>();
  a.zr = const_cast<float*>(zr.data_ptr<float>());
  a.dout = dout.data_ptr();
  a.ds = ds.data_ptr();
  a.y = y.data_ptr<float>();
  a.ab_part = ab.data_ptr<float>();
  a.p_part = pp.data_ptr<float>();
  ok(nt_msar_gate_bwd(a, stream()), "msar_gate_bwd");
  Tensor sums = ab.sum(0);
  return {ds, pp.sum(0), sums.narrow(0, 0, 1), sums.narrow(0, 1, 4)};
}

void moe_pull_rows(const Tensor& peers, const Tensor& src_rank, const Tensor& src_row, const Tensor& out) {
  TORCH_CHECK(peers.is_cuda() && peers.scalar_type() == at::kLong, "peers: int64 CUDA pointer table");
  check_i32(src_rank, "src_rank");
  check_i32(src_row, "src_row");
  check_rows(out, "out");
  const c10::cuda::CUDAGuard guard(out.device());
  ok(nt_moe_pull_rows(reinterpret_cast<const uint64_t*>(peers.data_ptr<int64_t>()), src_rank.data_ptr<int>(),
                      src_row.data_ptr<int>(), out.data_ptr(), out.size(0), static_cast<int>(out.size(-1)), stream()),
     "moe_pull_rows");
}

void moe_push_rows(const Tensor& rows, const Tensor& peers, const Tensor& dst_rank, const Tensor& dst_row) {
  TORCH_CHECK(peers.is_cuda() && peers.scalar_type() == at::kLong, "peers: int64 CUDA pointer table");
  check_i32(dst_rank, "dst_rank");
  check_i32(dst_row, "dst_row");
  check_rows(rows, "rows");
  const c10::cuda::CUDAGuard guard(rows.device());
  ok(nt_moe_push_rows(rows.data_ptr(), reinterpret_cast<const uint64_t*>(peers.data_ptr<int64_t>()),
                      dst_rank.data_ptr<int>(), dst_row.data_ptr<int>(), rows.size(0), static_cast<int>(rows.size(-1)),
                      stream()),
     "moe_push_rows");
}

// ------------------------------------------------------------------ linear-attention elementwise
void conv_silu_fwd(const Tensor& x, const Tensor& w, const Tensor& y, const OptT& pre) {
  check_rows(x, "x");
  check_rows(y, "y");
  TORCH_CHECK(w.scalar_type() == at::kFloat && w.is_contiguous(), "conv weight must be contiguous fp32 [C, K]");
  const int B = static_cast<int>(x.size(0)), T = static_cast<int>(x.size(1)), C = static_cast<int>(x.size(2));
  const c10::cuda::CUDAGuard guard(x.device());
  ok(nt_causal_conv_silu_fwd(x.data_ptr(), w.data_ptr<float>(), y.data_ptr(), mptr_or_null(pre), B, T, C,
                             static_cast<int>(w.size(-1)), stream()),
     "conv_silu_fwd");
}

void conv_silu_bwd(const Tensor& x, const Tensor& pre, const Tensor& dy, const Tensor& w, const Tensor& dx,
                   const Tensor& dw) {
  for (auto* t : {&x, &pre, &dy, &dx}) check_rows(*t, "conv operand");
  TORCH_CHECK(w.scalar_type() == at::kFloat && dw.scalar_type() == at::kFloat, "conv weights are fp32");
  const int B = static_cast<int>(x.size(0)), T = static_cast<int>(x.size(1)), C = static_cast<int>(x.size(2));
  const c10::cuda::CUDAGuard guard(x.device());
  ok(nt_causal_conv_silu_bwd(x.data_ptr(), pre.data_ptr(), dy.data_ptr(), w.data_ptr<float>(), dx.data_ptr(),
                             dw.data_ptr<float>(), B, T, C, static_cast<int>(w.size(-1)), stream()),
     "conv_silu_bwd");
}

void canon_conv_fwd(const Tensor& x, const Tensor& w, const Tensor& y) {
  check_rows(x, "x");
  check_rows(y, "y");
  TORCH_CHECK(w.scalar_type() == at::kFloat && w.is_contiguous(), "canon weight must be contiguous fp32 [C, K]");
  const int B = static_cast<int>(x.size(0)), T = static_cast<int>(x.size(1)), C = static_cast<int>(x.size(2));
  const c10::cuda::CUDAGuard guard(x.device());
  ok(nt_canon_conv_fwd(x.data_ptr(), w.data_ptr<float>(), y.data_ptr(), B, T, C, static_cast<int>(w.size(-1)),
                       stream()),
     "canon_conv_fwd");
}

void canon_conv_bwd(const Tensor& x, const Tensor& dy, const Tensor& w, const Tensor& dx, const Tensor& dw) {
  for (auto* t : {&x, &dy, &dx}) check_rows(*t, "canon operand");
  TORCH_CHECK(w.scalar_type() == at::kFloat && dw.scalar_type() == at::kFloat, "canon weights are fp32");
  const int B = static_cast<int>(x.size(0)), T = static_cast<int>(x.size(1)), C = static_cast<int>(x.size(2));
  const c10::cuda::CUDAGuard guard(x.device());
  ok(nt_canon_conv_bwd(x.data_ptr(), dy.data_ptr(), w.data_ptr<float>(), dx.data_ptr(), dw.data_ptr<float>(), B, T, C,
                       static_cast<int>(w.size(-1)), stream()),
     "canon_conv_bwd");
}

// gated attention / XSA heads: y [rows, H, 128] bf16; g [rows, H, G]; v [rows, Hk, 128]
void gate_mul_fwd(const Tensor& y, const Tensor& g, const Tensor& z) {
  for (auto* t : {&y, &g, &z}) check_rows(*t, "gate operand");
  TORCH_CHECK(y.scalar_type() == at::kBFloat16 && g.scalar_type() == at::kBFloat16 && y.dim() == 3 && y.size(2) == 128,
              "gate_mul: bf16 y [rows, H, 128]");
  const c10::cuda::CUDAGuard guard(y.device());
  ok(nt_gate_mul_fwd(y.data_ptr(), g.data_ptr(), z.data_ptr(), y.size(0), static_cast<int>(y.size(1)),
                     static_cast<int>(g.size(-1)), stream()),
     "gate_mul_fwd");
}

void gate_mul_bwd(const Tensor& y, const Tensor& g, const Tensor& dz, const Tensor& dy, const Tensor& dg) {
  for (auto* t : {&y, &g, &dz, &dy, &dg}) check_rows(*t, "gate operand");
  const c10::cuda::CUDAGuard guard(y.device());
  ok(nt_gate_mul_bwd(y.data_ptr(), g.data_ptr(), dz.data_ptr(), dy.data_ptr(), dg.data_ptr(), y.size(0),
                     static_cast<int>(y.size(1)), static_cast<int>(g.size(-1)), stream()),
     "gate_mul_bwd");
}

void xsa_fwd(const Tensor& y, const Tensor& v, const Tensor& z) {
  for (auto* t : {&y, &v, &z}) check_rows(*t, "xsa operand");
  TORCH_CHECK(y.scalar_type() == at::kBFloat16 && v.scalar_type() == at::kBFloat16 && y.dim() == 3 && v.dim() == 3 &&
                  y.size(2) == 128 && v.size(2) == 128 && y.size(0) == v.size(0),
              "xsa: bf16 y [rows, H, 128], v [rows, Hk, 128]");
  const c10::cuda::CUDAGuard guard(y.device());
  ok(nt_xsa_fwd(y.data_ptr(), v.data_ptr(), z.data_ptr(), y.size(0), static_cast<int>(y.size(1)),
                static_cast<int>(v.size(1)), stream()),
     "xsa_fwd");
}

void xsa_bwd(const Tensor& y, const Tensor& v, const Tensor& dz, const Tensor& dy, const Tensor& dv) {
  for (auto* t : {&y, &v, &dz, &dy, &dv}) check_rows(*t, "xsa operand");
  const c10::cuda::CUDAGuard guard(y.device());
  ok(nt_xsa_bwd(y.data_ptr(), v.data_ptr(), dz.data_ptr(), dy.data_ptr(), dv.data_ptr(), y.size(0),
                static_cast<int>(y.size(1)), static_cast<int>(v.size(1)), stream()),
     "xsa_bwd");
}

void gated_rmsnorm_fwd(const Tensor& x, const Tensor& g, const Tensor& gain, const Tensor& y, const Tensor& rstd) {
  for (auto* t : {&x, &g, &y}) check_rows(*t, "gated norm operand");
  const int D = static_cast<int>(gain.numel());
  const c10::cuda::CUDAGuard guard(x.device());
  ok(nt_gated_rmsnorm_fwd(x.data_ptr(), g.data_ptr(), gain.data_ptr<float>(), y.data_ptr(), rstd.data_ptr<float>(),
                          x.numel() / D, D, stream()),
     "gated_rmsnorm_fwd");
}

void gated_rmsnorm_bwd(const Tensor& x, const Tensor& g, const Tensor& gain, const Tensor& rstd, const Tensor& dy,
                       const Tensor& dx, const Tensor& dg, const Tensor& dgain) {
  for (auto* t : {&x, &g, &dy, &dx, &dg}) check_rows(*t, "gated norm operand");
  const int D = static_cast<int>(gain.numel());
  const c10::cuda::CUDAGuard guard(x.device());
  auto work = at::empty({NT_GATED_NORM_PARTS, D}, x.options().dtype(at::kFloat));
  ok(nt_gated_rmsnorm_bwd(x.data_ptr(), g.data_ptr(), gain.data_ptr<float>(), rstd.data_ptr<float>(), dy.data_ptr(),
                          dx.data_ptr(), dg.data_ptr(), dgain.data_ptr<float>(), work.data_ptr<float>(), x.numel() / D,
                          D, stream()),
     "gated_rmsnorm_bwd");
}

// ------------------------------------------------------------------ delta-rule chunk scan
void check_chunks(const Tensor& t, int64_t cols, const char* name) {
  TORCH_CHECK(t.is_cuda() && t.scalar_type() == at::kBFloat16 && t.is_contiguous() && t.dim() == 4 &&
                  t.size(-1) == cols,
              name, " must be a contiguous bf16 CUDA tensor [BH, N, rows, ", cols, "]");
}

// Per-chunk delta-rule terms (delta_prep.cu): q, k, v bf16 [B, T, H, 128] contiguous, g fp32 [B, T, H]
// (gate 1) or [B, T, H, 128] (gate 2), beta fp32 [B, T, H]; chunk-major outputs [B*H, N, 64, ..].
static DeltaPrepArgs prep_args(const Tensor& q, const Tensor& k, const Tensor& v, const OptT& g, const Tensor& beta,
                               int64_t gate, double qk_scale) {
  for (auto* t : {&q, &k, &v}) {
    check_cuda(*t, "delta operand");
    TORCH_CHECK(t->scalar_type() == at::kBFloat16 && t->is_contiguous() && t->dim() == 4 && t->size(-1) == 128,
                "q / k / v: contiguous bf16 [B, T, H, 128]");
    TORCH_CHECK(t->sizes() == q.sizes(), "q / k / v shapes differ");
  }
  TORCH_CHECK(beta.is_cuda() && beta.scalar_type() == at::kFloat && beta.is_contiguous() && beta.numel() == q.numel() / 128,
              "beta: contiguous fp32 [B, T, H]");
  DeltaPrepArgs a;
  a.B = static_cast<int>(q.size(0)); a.T = static_cast<int>(q.size(1)); a.H = static_cast<int>(q.size(2));
  a.gate = static_cast<int>(gate);
  a.qk_scale = static_cast<float>(qk_scale);
  a.q = q.data_ptr(); a.k = k.data_ptr(); a.v = v.data_ptr();
  a.beta = beta.data_ptr<float>();
  if (gate != DELTA_NONE) {
    TORCH_CHECK(g.has_value() && g->defined() && g->is_cuda() && g->scalar_type() == at::kFloat && g->is_contiguous(),
                "g: contiguous fp32");
    TORCH_CHECK(g->numel() == (gate == DELTA_FEATURE ? q.numel() : q.numel() / 128), "g shape");
    a.g = g->data_ptr<float>();
  }
  return a;
}

void delta_prep_fwd(const Tensor& q, const Tensor& k, const Tensor& v, const OptT& g, const Tensor& beta, int64_t gate,
                    double qk_scale, const Tensor& w, const Tensor& u0, const Tensor& qt, const Tensor& kc,
                    const Tensor& aqk, const Tensor& carry) {
  DeltaPrepArgs a = prep_args(q, k, v, g, beta, gate, qk_scale);
  const int64_t rows = static_cast<int64_t>(a.B) * a.H * ((a.T + 63) / 64) * 64;
  for (auto* t : {&w, &u0, &qt, &kc})
    TORCH_CHECK(t->scalar_type() == at::kBFloat16 && t->is_contiguous() && t->numel() == rows * 128, "chunk outputs");
  TORCH_CHECK(aqk.scalar_type() == at::kBFloat16 && aqk.is_contiguous() && aqk.numel() == rows * 64, "aqk");
  TORCH_CHECK(carry.scalar_type() == at::kFloat && carry.is_contiguous() && carry.numel() == rows * 2, "carry");
  a.w = w.data_ptr(); a.u0 = u0.data_ptr(); a.qt = qt.data_ptr(); a.kc = kc.data_ptr(); a.aqk = aqk.data_ptr();
  a.carry = carry.data_ptr<float>();
  const c10::cuda::CUDAGuard guard(q.device());
  ok(nt_delta_prep_fwd(a, stream()), "delta_prep_fwd");
}

// KDA with the gate from its pre-activation and (qk_norm) the q / k L2 normalisation in the kernel:
// g_raw bf16 [B, T, H, 128], g_log / g_bias fp32 [H, 128].
static DeltaPrepArgs kda_args(const Tensor& q, const Tensor& k, const Tensor& v, const Tensor& g_raw,
                              const Tensor& g_log, const Tensor& g_bias, const Tensor& beta, double qk_scale,
                              bool qk_norm) {
  DeltaPrepArgs a = prep_args(q, k, v, c10::nullopt, beta, DELTA_NONE, qk_scale);
  check_cuda(g_raw, "g_raw");
  TORCH_CHECK(g_raw.scalar_type() == at::kBFloat16 && g_raw.is_contiguous() && g_raw.sizes() == q.sizes(),
              "g_raw: contiguous bf16 [B, T, H, 128]");
  for (auto* t : {&g_log, &g_bias})
    TORCH_CHECK(t->is_cuda() && t->scalar_type() == at::kFloat && t->is_contiguous() && t->numel() == q.size(2) * 128,
                "g_log / g_bias: contiguous fp32 [H, 128]");
  a.gate = DELTA_FEATURE;
  a.qk_norm = qk_norm ? 1 : 0;
  a.g_raw = reinterpret_cast<const __nv_bfloat16*>(g_raw.data_ptr());
  a.g_log = g_log.data_ptr<float>();
  a.g_bias = g_bias.data_ptr<float>();
  return a;
}

void delta_prep_kda_fwd(const Tensor& q, const Tensor& k, const Tensor& v, const Tensor& g_raw, const Tensor& g_log,
                        const Tensor& g_bias, const Tensor& beta, double qk_scale, bool qk_norm, const Tensor& w,
                        const Tensor& u0, const Tensor& qt, const Tensor& kc, const Tensor& aqk, const Tensor& carry) {
  DeltaPrepArgs a = kda_args(q, k, v, g_raw, g_log, g_bias, beta, qk_scale, qk_norm);
  const int64_t rows = static_cast<int64_t>(a.B) * a.H * ((a.T + 63) / 64) * 64;
  for (auto* t : {&w, &u0, &qt, &kc})
    TORCH_CHECK(t->scalar_type() == at::kBFloat16 && t->is_contiguous() && t->numel() == rows * 128, "chunk outputs");
  TORCH_CHECK(aqk.scalar_type() == at::kBFloat16 && aqk.is_contiguous() && aqk.numel() == rows * 64, "aqk");
  TORCH_CHECK(carry.scalar_type() == at::kFloat && carry.is_contiguous() && carry.numel() == rows * 2, "carry");
  a.w = w.data_ptr(); a.u0 = u0.data_ptr(); a.qt = qt.data_ptr(); a.kc = kc.data_ptr(); a.aqk = aqk.data_ptr();
  a.carry = carry.data_ptr<float>();
  const c10::cuda::CUDAGuard guard(q.device());
  ok(nt_delta_prep_fwd(a, stream()), "delta_prep_kda_fwd");
}

void delta_prep_kda_bwd(const Tensor& q, const Tensor& k, const Tensor& v, const Tensor& g_raw, const Tensor& g_log,
                        const Tensor& g_bias, const Tensor& beta, double qk_scale, bool qk_norm, const Tensor& w,
                        const Tensor& u0, const Tensor& dw, const Tensor& du0, const Tensor& dqt, const Tensor& dkc,
                        const Tensor& daqk, const Tensor& dcarry, const Tensor& dq, const Tensor& dk, const Tensor& dv,
                        const Tensor& dg_raw, const Tensor& dg_log_part, const Tensor& dg_bias_part,
                        const Tensor& dbeta) {
  DeltaPrepArgs a = kda_args(q, k, v, g_raw, g_log, g_bias, beta, qk_scale, qk_norm);
  const int64_t N = (a.T + 63) / 64, rows = static_cast<int64_t>(a.B) * a.H * N * 64;
  for (auto* t : {&w, &u0})
    TORCH_CHECK(t->scalar_type() == at::kBFloat16 && t->is_contiguous() && t->numel() == rows * 128, "w / u0");
  for (auto* t : {&dw, &du0, &dqt, &dkc})
    TORCH_CHECK(t->scalar_type() == at::kFloat && t->is_contiguous() && t->numel() == rows * 128, "chunk gradients");
  TORCH_CHECK(daqk.scalar_type() == at::kFloat && daqk.is_contiguous() && daqk.numel() == rows * 64, "daqk");
  TORCH_CHECK(dcarry.scalar_type() == at::kFloat && dcarry.is_contiguous() && dcarry.numel() == rows * 2, "dcarry");
  for (auto* t : {&dq, &dk, &dv})
    TORCH_CHECK(t->scalar_type() == at::kFloat && t->is_contiguous() && t->numel() == q.numel(), "dq / dk / dv");
  TORCH_CHECK(dbeta.scalar_type() == at::kFloat && dbeta.is_contiguous() && dbeta.numel() == q.numel() / 128, "dbeta");
  TORCH_CHECK(dg_raw.scalar_type() == at::kBFloat16 && dg_raw.is_contiguous() && dg_raw.sizes() == q.sizes(), "dg_raw");
  for (auto* t : {&dg_log_part, &dg_bias_part})
    TORCH_CHECK(t->scalar_type() == at::kFloat && t->is_contiguous() && t->numel() == a.B * N * a.H * 128,
                "g_log / g_bias partials: fp32 [B, N, H, 128]");
  a.w = w.data_ptr(); a.u0 = u0.data_ptr();
  a.dw = dw.data_ptr<float>(); a.du0 = du0.data_ptr<float>(); a.dqt = dqt.data_ptr<float>();
  a.dkc = dkc.data_ptr<float>(); a.daqk = daqk.data_ptr<float>(); a.dcarry = dcarry.data_ptr<float>();
  a.dq = dq.data_ptr<float>(); a.dk = dk.data_ptr<float>(); a.dv = dv.data_ptr<float>();
  a.dbeta = dbeta.data_ptr<float>();
  a.dg_raw = reinterpret_cast<__nv_bfloat16*>(dg_raw.data_ptr());
  a.dg_log_part = dg_log_part.data_ptr<float>();
  a.dg_bias_part = dg_bias_part.data_ptr<float>();
  const c10::cuda::CUDAGuard guard(q.device());
  ok(nt_delta_prep_bwd(a, stream()), "delta_prep_kda_bwd");
}

void delta_prep_bwd(const Tensor& q, const Tensor& k, const Tensor& v, const OptT& g, const Tensor& beta, int64_t gate,
                    double qk_scale, const Tensor& w, const Tensor& u0, const Tensor& dw, const Tensor& du0,
                    const Tensor& dqt, const Tensor& dkc, const Tensor& daqk, const Tensor& dcarry, const Tensor& dq,
                    const Tensor& dk, const Tensor& dv, const OptT& dg, const Tensor& dbeta) {
  DeltaPrepArgs a = prep_args(q, k, v, g, beta, gate, qk_scale);
  const int64_t rows = static_cast<int64_t>(a.B) * a.H * ((a.T + 63) / 64) * 64;
  for (auto* t : {&w, &u0})
    TORCH_CHECK(t->scalar_type() == at::kBFloat16 && t->is_contiguous() && t->numel() == rows * 128, "w / u0");
  for (auto* t : {&dw, &du0, &dqt, &dkc})
    TORCH_CHECK(t->scalar_type() == at::kFloat && t->is_contiguous() && t->numel() == rows * 128, "chunk gradients");
  TORCH_CHECK(daqk.scalar_type() == at::kFloat && daqk.is_contiguous() && daqk.numel() == rows * 64, "daqk");
  TORCH_CHECK(dcarry.scalar_type() == at::kFloat && dcarry.is_contiguous() && dcarry.numel() == rows * 2, "dcarry");
  for (auto* t : {&dq, &dk, &dv})
    TORCH_CHECK(t->scalar_type() == at::kFloat && t->is_contiguous() && t->numel() == q.numel(), "dq / dk / dv");
  TORCH_CHECK(dbeta.scalar_type() == at::kFloat && dbeta.is_contiguous() && dbeta.numel() == q.numel() / 128, "dbeta");
  a.w = w.data_ptr(); a.u0 = u0.data_ptr();
  a.dw = dw.data_ptr<float>(); a.du0 = du0.data_ptr<float>(); a.dqt = dqt.data_ptr<float>();
  a.dkc = dkc.data_ptr<float>(); a.daqk = daqk.data_ptr<float>(); a.dcarry = dcarry.data_ptr<float>();
  a.dq = dq.data_ptr<float>(); a.dk = dk.data_ptr<float>(); a.dv = dv.data_ptr<float>();
  a.dbeta = dbeta.data_ptr<float>();
  if (gate != DELTA_NONE) {
    TORCH_CHECK(dg.has_value() && dg->defined() && dg->scalar_type() == at::kFloat && dg->is_contiguous() &&
                    dg->numel() == g->numel(), "dg");
    a.dg = dg->data_ptr<float>();
  }
  const c10::cuda::CUDAGuard guard(q.device());
  ok(nt_delta_prep_bwd(a, stream()), "delta_prep_bwd");
}

void delta_scan_fwd(const Tensor& w, const Tensor& qt, const Tensor& kc, const Tensor& aqk, const Tensor& u0,
                    const Tensor& carry, const Tensor& o, const Tensor& states, const Tensor& u) {
  for (auto* t : {&w, &qt, &kc, &u0, &o, &u}) check_chunks(*t, 128, "delta scan operand");
  check_chunks(aqk, 64, "aqk");
  check_chunks(states, 128, "states");
  TORCH_CHECK(w.size(2) == 64 && states.size(2) == 128, "chunk length 64, state 128 x 128");
  TORCH_CHECK(carry.scalar_type() == at::kFloat && carry.is_contiguous() && carry.numel() == w.size(0) * w.size(1) * 128,
              "carry must be contiguous fp32 [BH, N, 128]");
  DeltaScanFwdArgs a;
  a.BH = static_cast<int>(w.size(0));
  a.N = static_cast<int>(w.size(1));
  a.w = w.data_ptr(); a.qt = qt.data_ptr(); a.kc = kc.data_ptr(); a.aqk = aqk.data_ptr(); a.u0 = u0.data_ptr();
  a.carry = carry.data_ptr<float>();
  a.o = reinterpret_cast<__nv_bfloat16*>(o.data_ptr());
  a.states = reinterpret_cast<__nv_bfloat16*>(states.data_ptr());
  a.u = reinterpret_cast<__nv_bfloat16*>(u.data_ptr());
  const c10::cuda::CUDAGuard guard(w.device());
  ok(nt_delta_scan_fwd(a, stream()), "delta_scan_fwd");
}

void delta_scan_bwd(const Tensor& dout, const Tensor& w, const Tensor& qt, const Tensor& kc, const Tensor& aqk,
                    const Tensor& carry, const Tensor& states, const Tensor& ds, const Tensor& dut,
                    const Tensor& dcarry) {
  for (auto* t : {&dout, &w, &qt, &kc}) check_chunks(*t, 128, "delta scan operand");
  check_chunks(aqk, 64, "aqk");
  check_chunks(dut, 64, "du^T");
  check_chunks(states, 128, "states");
  check_chunks(ds, 128, "dS");
  TORCH_CHECK(carry.scalar_type() == at::kFloat && dcarry.scalar_type() == at::kFloat && dcarry.is_contiguous(),
              "carry / dcarry are fp32");
  DeltaScanBwdArgs a;
  a.BH = static_cast<int>(w.size(0));
  a.N = static_cast<int>(w.size(1));
  a.dout = dout.data_ptr(); a.w = w.data_ptr(); a.qt = qt.data_ptr(); a.kc = kc.data_ptr(); a.aqk = aqk.data_ptr();
  a.carry = carry.data_ptr<float>();
  a.states = reinterpret_cast<const __nv_bfloat16*>(states.data_ptr());
  a.ds = reinterpret_cast<__nv_bfloat16*>(ds.data_ptr());
  a.dut = reinterpret_cast<__nv_bfloat16*>(dut.data_ptr());
  a.dcarry = dcarry.data_ptr<float>();
  const c10::cuda::CUDAGuard guard(w.device());
  ok(nt_delta_scan_bwd(a, stream()), "delta_scan_bwd");
}

std::vector<int64_t> read_comm_errors() {
  unsigned w = 0;
  const int c = nt_comm_read_error(&w);
  return {c, static_cast<int64_t>(w)};
}

void clear_comm_errors() { ok(nt_comm_clear_error(), "clear_comm_errors"); }

std::vector<int64_t> read_errors() {
  unsigned w = 0;
  const int g = nt_gemm_read_error(&w);
  unsigned wa = 0;
  const int a = nt_attention_read_error(&wa);
  unsigned wd = 0;
  const int d = nt_delta_scan_read_error(&wd);
  unsigned ws = 0;
  const int sp = nt_sparse_attn_read_error(&ws);
  return {g, static_cast<int64_t>(w), a, static_cast<int64_t>(wa), d, static_cast<int64_t>(wd), sp,
          static_cast<int64_t>(ws)};
}

}  // namespace

// tcgen05 issue-rate probe (microbenchmark): out int64 [ctas, 3]
void mma_rate(int64_t variant, int64_t groups, const Tensor& out) {
  check_cuda(out, "out");
  TORCH_CHECK(out.scalar_type() == at::kLong && out.is_contiguous() && out.dim() == 2 && out.size(1) == 3, "out: int64 [ctas, 3]");
  const c10::cuda::CUDAGuard guard(out.device());
  ok(nt_mma_rate(static_cast<int>(variant), static_cast<int>(groups), static_cast<int>(out.size(0)),
                 reinterpret_cast<long long*>(out.data_ptr<int64_t>()), stream()),
     "mma_rate");
}

PYBIND11_MODULE(TORCH_EXTENSION_NAME, m) {
  m.doc() = "nexttransformer_b200 sm_100a kernels";
  m.def("gemm", &gemm, "bf16 tcgen05 GEMM with fused epilogue");
  m.def("mix_norm_fwd", &mix_norm_fwd);
  m.def("norm_bwd", &norm_bwd);
  m.def("mix_norm_bwd", &mix_norm_bwd);
  m.def("rope_norm_fwd", &rope_norm_fwd);
  m.def("rope_norm_bwd", &rope_norm_bwd);
  m.def("softcap_ce", &softcap_ce, py::arg("logits"), py::arg("tgt"), py::arg("loss"), py::arg("lse"), py::arg("V"),
        py::arg("cap"), py::arg("variant") = 0);
  m.def("embed_smear", &embed_smear);
  m.def("embed_scatter", &embed_scatter);
  m.def("cast_bf16", &cast_bf16);
  m.def("adamw", &adamw);
  m.def("muon_prep", &muon_prep);
  m.def("muon_normalize", &muon_normalize);
  m.def("muon_finish", &muon_finish);
  m.def("attn_fwd", &attn_fwd);
  m.def("attn_fwd_trace", &attn_fwd_trace);
  m.def("attn_bwd", &attn_bwd, py::arg("q"), py::arg("k"), py::arg("v"), py::arg("o"), py::arg("lse"),
        py::arg("dout"), py::arg("dq"), py::arg("dk"), py::arg("dv"), py::arg("dq_acc"), py::arg("delta"), py::arg("B"),
        py::arg("T"), py::arg("H"), py::arg("Hk"), py::arg("D"), py::arg("window"), py::arg("scale"),
        py::arg("trace") = py::none(), py::arg("dq_slices") = 0);
  m.def("read_errors", &read_errors);
  m.def("gemm_ce_fwd", &gemm_ce_fwd);
  m.def("p2p_reduce_scatter", &p2p_reduce_scatter);
  m.def("conv_silu_fwd", &conv_silu_fwd);
  m.def("gemm_grouped", &gemm_grouped);
  m.def("sinkhorn_fwd", &sinkhorn_fwd);
  m.def("sinkhorn_bwd", &sinkhorn_bwd);
  m.def("sparse_attn_fwd", &sparse_attn_fwd);
  m.def("sparse_attn_bwd", &sparse_attn_bwd);
  m.def("moe_gather_rows", &moe_gather_rows);
  m.def("p2p_barrier", &p2p_barrier);
  m.def("clear_comm_errors", &clear_comm_errors, "reset the peer-collective error word");
  m.def("p2p_put", &p2p_put);
  m.def("p2p_gather", &p2p_gather);
  m.def("moe_combine", &moe_combine);
  m.def("moe_combine_bwd", &moe_combine_bwd);
  m.def("moe_pull_rows", &moe_pull_rows);
  m.def("moe_route", &moe_route);
  m.def("sparse_teacher", &sparse_teacher);
  m.def("nsa_compressed_fwd", &nsa_compressed_fwd);
  m.def("nsa_compressed_bwd", &nsa_compressed_bwd);
  m.def("msar_temporal_fwd", &msar_temporal_fwd);
  m.def("msar_temporal_bwd", &msar_temporal_bwd);
  m.def("msar_gate_fwd", &msar_gate_fwd);
  m.def("msar_gate_bwd", &msar_gate_bwd);
  m.def("moe_route_bwd", &moe_route_bwd);
  m.def("moe_push_rows", &moe_push_rows);
  m.def("delta_scan_fwd", &delta_scan_fwd);
  m.def("delta_prep_fwd", &delta_prep_fwd, "per-chunk delta-rule terms (WY solve, gates, q/k norm)");
  m.def("delta_prep_bwd", &delta_prep_bwd, "backward of the per-chunk delta-rule terms");
  m.def("delta_prep_kda_fwd", &delta_prep_kda_fwd, "KDA chunk terms with the gate from its pre-activation");
  m.def("delta_prep_kda_bwd", &delta_prep_kda_bwd, "backward of delta_prep_kda_fwd");
  m.def("mma_rate", &mma_rate, "tcgen05.mma issue-rate probe");
  m.def("delta_scan_bwd", &delta_scan_bwd);
  m.def("conv_silu_bwd", &conv_silu_bwd);
  m.def("canon_conv_fwd", &canon_conv_fwd);
  m.def("canon_conv_bwd", &canon_conv_bwd);
  m.def("gate_mul_fwd", &gate_mul_fwd);
  m.def("gate_mul_bwd", &gate_mul_bwd);
  m.def("xsa_fwd", &xsa_fwd);
  m.def("xsa_bwd", &xsa_bwd);
  m.def("gated_rmsnorm_fwd", &gated_rmsnorm_fwd);
  m.def("gated_rmsnorm_bwd", &gated_rmsnorm_bwd);
  m.def("read_comm_errors", &read_comm_errors);
  m.def("gemm_ce_dgrad", &gemm_ce_dgrad);
  m.attr("EPI_BF16") = static_cast<int>(EPI_BF16);
  m.attr("EPI_F32") = static_cast<int>(EPI_F32);
  m.attr("EPI_F32_ACC") = static_cast<int>(EPI_F32_ACC);
  m.attr("EPI_BF16_AXPBY") = static_cast<int>(EPI_BF16_AXPBY);
  m.attr("EPI_RELU2") = static_cast<int>(EPI_RELU2);
  m.attr("EPI_RELU2_BWD") = static_cast<int>(EPI_RELU2_BWD);
}
