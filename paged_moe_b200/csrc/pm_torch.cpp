// pm_torch.cpp -- the thin PyTorch extension over the C ABI of
// libpm_sample.so (include/pm_sample.h).
//
// The Python layer resolves the sampler / processor settings once (a cached
// device array of pm_row_params) and hands tensors to these functions; they
// pack the C structs, allocate the outputs on the logits' device, call the C
// ABI on the current CUDA stream and raise on a bad status.  No arithmetic
// happens here: every kernel is in libpm_sample.so.
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/extension.h>

#include <optional>
#include <string>
#include <vector>

#include "../../include/pm_sample.h"

namespace {

using OptT = std::optional<torch::Tensor>;

const void* ptr(const OptT& t) { return t.has_value() ? t->data_ptr() : nullptr; }

void check(int rc, const char* what) {
  if (rc == PM_OK) return;
  std::string msg = std::string(what) + ": ";
  switch (rc) {
    case PM_ERR_ARG: msg += "invalid argument"; break;
    case PM_ERR_CUDA: msg += "CUDA error " + std::to_string(pm_last_cuda_error()); break;
    case PM_ERR_UNSUPPORTED: msg += "outside this build's limits"; break;
    case PM_ERR_WORKSPACE: msg += "workspace too small"; break;
    default: msg += "status " + std::to_string(rc);
  }
  if (rc == PM_ERR_ARG) throw std::invalid_argument(msg);
  throw std::runtime_error(msg);
}

int dtype_code(const torch::Tensor& t) {
  if (t.scalar_type() == torch::kFloat32) return PM_DTYPE_F32;
  if (t.scalar_type() == torch::kBFloat16) return PM_DTYPE_BF16;
  throw std::invalid_argument("logits must be float32 or bfloat16");
}

// The rows struct over prepared tensors (contiguous, on the device, except
// logits / mask, which may be pinned host memory for the masked pass).
pm_rows make_rows(const torch::Tensor& logits, const torch::Tensor& params, bool per_row, int64_t flags_any,
                  int64_t top_k_max, const OptT& hist, const OptT& hist_len, const OptT& feed, int64_t feed_group,
                  const OptT& bias_tok, const OptT& bias_val, const OptT& mask, const OptT& forced) {
  if (logits.dim() != 2 || logits.stride(1) != 1) throw std::invalid_argument("logits must be [rows, vocab], unit stride");
  pm_rows r;
  std::memset(&r, 0, sizeof(r));
  r.logits = logits.data_ptr();
  r.dtype = dtype_code(logits);
  r.rows = logits.size(0);
  r.vocab = logits.size(1);
  r.row_stride = logits.stride(0);
  r.params = reinterpret_cast<const pm_row_params*>(params.data_ptr());
  r.params_per_row = per_row ? 1 : 0;
  r.flags_any = (uint32_t)flags_any;
  r.top_k_max = (int32_t)top_k_max;
  if (hist.has_value()) {
    r.hist = reinterpret_cast<const int32_t*>(hist->data_ptr());
    r.hist_stride = hist->size(1);
    r.hist_len = reinterpret_cast<const int32_t*>(ptr(hist_len));
  }
  if (feed.has_value()) {
    r.feed = reinterpret_cast<const int32_t*>(feed->data_ptr());
    r.feed_group = (int32_t)feed_group;
  }
  if (bias_tok.has_value()) {
    r.bias_tokens = reinterpret_cast<const int32_t*>(bias_tok->data_ptr());
    r.bias_values = reinterpret_cast<const float*>(ptr(bias_val));
    r.n_bias = (int32_t)bias_tok->numel();
  }
  if (mask.has_value()) {
    r.mask = reinterpret_cast<const uint32_t*>(mask->data_ptr());
    r.mask_stride = mask->size(1);
  }
  r.forced = reinterpret_cast<const int32_t*>(ptr(forced));
  return r;
}

pm_noise make_noise(int64_t seed, int64_t offset, int64_t row_base, const OptT& gumbel, const OptT& uniform) {
  pm_noise n;
  std::memset(&n, 0, sizeof(n));
  n.mode = (gumbel.has_value() || uniform.has_value()) ? PM_NOISE_INJECTED : PM_NOISE_PHILOX;
  n.seed = (uint64_t)seed;
  n.offset = (uint64_t)offset;
  n.row_base = (uint32_t)row_base;
  if (gumbel.has_value()) {
    n.gumbel = reinterpret_cast<const float*>(gumbel->data_ptr());
    n.gumbel_stride = gumbel->size(1);
  }
  n.uniform = reinterpret_cast<const double*>(ptr(uniform));
  return n;
}

void* stream_of(const torch::Device& dev) {
  return reinterpret_cast<void*>(at::cuda::getCurrentCUDAStream(dev.index()).stream());
}

// pm_sample_rows: [tokens, lse?, logprob?, surv_ids?, surv_probs?, n_surv?]
// (absent outputs are empty tensors; all are views of one allocation).
std::vector<torch::Tensor> sample_rows(torch::Tensor logits, torch::Tensor params, bool per_row, int64_t flags_any,
                                       int64_t top_k_max, OptT hist, OptT hist_len, OptT bias_tok, OptT bias_val,
                                       OptT mask, OptT forced, int64_t seed, int64_t offset, int64_t row_base,
                                       OptT gumbel, OptT uniform, bool want_lse, bool want_logprob,
                                       int64_t survivors, torch::Tensor workspace) {
  const torch::Device dev = params.device();
  const c10::cuda::CUDAGuard guard(dev);
  pm_rows r = make_rows(logits, params, per_row, flags_any, top_k_max, hist, hist_len, std::nullopt, 0, bias_tok,
                        bias_val, mask, forced);
  pm_noise nz = make_noise(seed, offset, row_base, gumbel, uniform);
  const int64_t B = r.rows;
  const int64_t S = survivors > 0 ? survivors : 0;
  // every output in one device allocation (32-bit words), handed out as views
  const int64_t words = B + (want_lse ? B : 0) + (want_logprob ? B : 0) + (S ? 2 * B * S + B : 0);
  torch::Tensor buf = torch::empty({words}, torch::TensorOptions().dtype(torch::kInt32).device(dev));
  torch::Tensor none = buf.narrow(0, 0, 0);
  int64_t at = 0;
  auto take = [&](int64_t n) {
    torch::Tensor t = buf.narrow(0, at, n);
    at += n;
    return t;
  };
  std::vector<torch::Tensor> res(6, none);
  pm_sample_out out;
  std::memset(&out, 0, sizeof(out));
  res[0] = take(B);
  out.tokens = res[0].data_ptr<int32_t>();
  if (want_lse) {
    res[1] = take(B).view(torch::kFloat32);
    out.lse = res[1].data_ptr<float>();
  }
  if (want_logprob) {
    res[2] = take(B).view(torch::kFloat32);
    out.token_logprob = res[2].data_ptr<float>();
  }
  if (S) {
    res[3] = take(B * S).view({B, S});
    res[4] = take(B * S).view(torch::kFloat32).view({B, S});
    res[5] = take(B);
    out.surv_ids = res[3].data_ptr<int32_t>();
    out.surv_probs = res[4].data_ptr<float>();
    out.n_surv = res[5].data_ptr<int32_t>();
    out.surv_cap = (int32_t)S;
  }
  check(pm_sample_rows(&r, &nz, &out, workspace.data_ptr(), (size_t)workspace.numel(), stream_of(dev)),
        "pm_sample_rows");
  return res;
}

// Workspace bytes pm_sample_rows needs for these rows (0: unsupported).
int64_t sample_workspace_bytes(torch::Tensor logits, torch::Tensor params, bool per_row, int64_t flags_any,
                               int64_t top_k_max, OptT hist, OptT mask) {
  pm_rows r = make_rows(logits, params, per_row, flags_any, top_k_max, hist, std::nullopt, std::nullopt, 0,
                        std::nullopt, std::nullopt, mask, std::nullopt);
  return (int64_t)pm_sample_workspace_bytes(&r);
}

// pm_verify: [tokens [B, k+1], n_accepted [B], row_tokens [B, k+1] or empty]
std::vector<torch::Tensor> verify(torch::Tensor logits, torch::Tensor params, bool per_row, int64_t flags_any,
                                  int64_t top_k_max, OptT hist, OptT hist_len, OptT feed, int64_t feed_group,
                                  OptT bias_tok, OptT bias_val, OptT mask, int64_t seed, int64_t offset,
                                  int64_t row_base, OptT gumbel, OptT uniform, int64_t mode, torch::Tensor drafts,
                                  OptT draft_logits, OptT u_accept, OptT u_residual, bool want_row_tokens,
                                  torch::Tensor workspace_cache) {
  const torch::Device dev = params.device();
  const c10::cuda::CUDAGuard guard(dev);
  pm_rows r = make_rows(logits, params, per_row, flags_any, top_k_max, hist, hist_len, feed, feed_group, bias_tok,
                        bias_val, mask, std::nullopt);
  pm_noise nz = make_noise(seed, offset, row_base, gumbel, uniform);
  const int64_t B = drafts.size(0), k = drafts.size(1);
  // every output in one device allocation, handed out as views
  const int64_t K1 = k + 1;
  torch::Tensor buf = torch::empty({B * K1 + B + (want_row_tokens ? B * K1 : 0)},
                                   torch::TensorOptions().dtype(torch::kInt32).device(dev));
  std::vector<torch::Tensor> res(3);
  res[0] = buf.narrow(0, 0, B * K1).view({B, K1});
  res[1] = buf.narrow(0, B * K1, B);
  res[2] = want_row_tokens ? buf.narrow(0, B * K1 + B, B * K1).view({B, K1}) : buf.narrow(0, 0, 0);
  pm_verify_args va;
  std::memset(&va, 0, sizeof(va));
  va.mode = (int32_t)mode;
  va.drafts = reinterpret_cast<const int32_t*>(drafts.data_ptr());
  va.n_draft = (int32_t)k;
  if (draft_logits.has_value()) {
    va.draft_logits = draft_logits->data_ptr();
    va.draft_dtype = dtype_code(*draft_logits);
    va.draft_row_stride = draft_logits->stride(0);
  }
  va.u_accept = reinterpret_cast<const double*>(ptr(u_accept));
  va.u_residual = reinterpret_cast<const double*>(ptr(u_residual));
  va.tokens = res[0].data_ptr<int32_t>();
  va.n_accepted = res[1].data_ptr<int32_t>();
  if (want_row_tokens) va.row_tokens = res[2].data_ptr<int32_t>();
  const size_t need = pm_verify_workspace_bytes(&r, &va);
  if (need == 0) check(PM_ERR_UNSUPPORTED, "pm_verify_workspace_bytes");
  if ((size_t)workspace_cache.numel() < need) check(PM_ERR_WORKSPACE, "pm_verify");
  check(pm_verify(&r, &nz, &va, workspace_cache.data_ptr(), (size_t)workspace_cache.numel(), stream_of(dev)),
        "pm_verify");
  return res;
}

int64_t verify_workspace_bytes(torch::Tensor logits, torch::Tensor params, bool per_row, int64_t flags_any,
                               int64_t top_k_max, OptT hist, OptT feed, int64_t feed_group, OptT mask, int64_t mode,
                               torch::Tensor drafts) {
  pm_rows r = make_rows(logits, params, per_row, flags_any, top_k_max, hist, std::nullopt, feed, feed_group,
                        std::nullopt, std::nullopt, mask, std::nullopt);
  pm_verify_args va;
  std::memset(&va, 0, sizeof(va));
  va.mode = (int32_t)mode;
  va.n_draft = (int32_t)drafts.size(1);
  return (int64_t)pm_verify_workspace_bytes(&r, &va);
}

}  // namespace

PYBIND11_MODULE(TORCH_EXTENSION_NAME, m) {
  m.doc() = "PyTorch binding of libpm_sample.so (C ABI: include/pm_sample.h)";
  m.def("sample_rows", &sample_rows);
  m.def("sample_workspace_bytes", &sample_workspace_bytes);
  m.def("verify", &verify);
  m.def("verify_workspace_bytes", &verify_workspace_bytes);
  m.def("version", [] { return std::string(pm_version()); });
}
