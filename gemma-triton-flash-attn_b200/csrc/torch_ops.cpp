// torch operators over the C ABI (include/gqa_fa_b200.h): torch.ops.gqafa.fwd
// and torch.ops.gqafa.bwd.
//
// These are the launch sites of the reference's autograd function
// (flash_attn/attention.py:1435-1473 forward, :1476-1622 backward) as
// dispatcher operators: they allocate the outputs the reference allocates
// (O, LSE; dQ, dK, dV and the delta scratch), pass the current CUDA stream of
// the input's device and turn a non-zero status into the Python exception the
// reference's callers expect (ValueError / NotImplementedError /
// RuntimeError). Compared with calling the C ABI through ctypes this removes
// the per-call Python marshalling of ~30 arguments and stride arrays. No CUDA
// code is compiled here: every kernel lives in libgqa_fa_b200.so.
#include <ATen/ATen.h>
#include <c10/cuda/CUDAGuard.h>
#include <c10/cuda/CUDAStream.h>
#include <torch/library.h>

#include <tuple>

#include "../../include/gqa_fa_b200.h"

namespace {

int dtype_code(const at::Tensor& t) {
  if (t.scalar_type() == at::kHalf) return GQAFA_DTYPE_FP16;
  if (t.scalar_type() == at::kBFloat16) return GQAFA_DTYPE_BF16;
  TORCH_CHECK_NOT_IMPLEMENTED(false, "gqafa: dtype ", t.scalar_type(), " is not supported (fp16, bf16)");
  return -1;
}

void check(int rc) {
  if (rc == GQAFA_OK) return;
  const char* msg = gqafa_last_error();
  TORCH_CHECK_NOT_IMPLEMENTED(rc != GQAFA_ERR_UNSUPPORTED, msg);
  TORCH_CHECK_VALUE(rc != GQAFA_ERR_INVALID, msg);
  TORCH_CHECK(false, "gqafa: ", msg);
}

void check_4d(const at::Tensor& t, const char* name) {
  TORCH_CHECK_VALUE(t.dim() == 4, "gqafa: ", name, " must be 4-D (B, H, N, D)");
  TORCH_CHECK(t.is_cuda(), "gqafa: ", name, " must be a CUDA tensor (there is no CPU path)");
}

// A layout the tensor maps accept: last stride 1, other strides multiples of 8
// elements (size-1 dimensions excepted), 16-byte aligned data. Otherwise a
// contiguous copy, as the Python layer does.
at::Tensor abi_ready(const at::Tensor& t) {
  bool ok = t.stride(3) == 1 && reinterpret_cast<uintptr_t>(t.data_ptr()) % 16 == 0;
  for (int i = 0; i < 3 && ok; ++i) ok = (t.stride(i) % 8 == 0) || t.size(i) == 1;
  return ok ? t : t.contiguous();
}

struct Strides {
  long long s[4];
  explicit Strides(const at::Tensor& t) {
    for (int i = 0; i < 4; ++i) s[i] = t.stride(i);
  }
};

std::tuple<at::Tensor, at::Tensor> fwd(const at::Tensor& q_in, const at::Tensor& k_in, const at::Tensor& v_in,
                                       bool causal, int64_t window, double scale, bool want_lse) {
  check_4d(q_in, "q");
  check_4d(k_in, "k");
  check_4d(v_in, "v");
  c10::cuda::CUDAGuard guard(q_in.device());
  const at::Tensor q = abi_ready(q_in), k = abi_ready(k_in), v = abi_ready(v_in);
  const int64_t B = q.size(0), Hq = q.size(1), N = q.size(2), D = q.size(3), Hkv = k.size(1), Nk = k.size(2);
  at::Tensor o = abi_ready(at::empty_like(q));  // keeps q's layout (HF's (B, N, H, D) storage)
  at::Tensor lse = want_lse ? at::empty({B, Hq, N}, q.options().dtype(at::kFloat)) : at::Tensor();
  const Strides sq(q), sk(k), sv(v), so(o);
  void* stream = c10::cuda::getCurrentCUDAStream(q.get_device()).stream();
  float* lp = want_lse ? lse.data_ptr<float>() : nullptr;
  int rc;
  if (Nk == N) {
    rc = gqafa_fwd(q.data_ptr(), sq.s, k.data_ptr(), sk.s, v.data_ptr(), sv.s, o.data_ptr(), so.s, lp, (int)B,
                   (int)Hq, (int)Hkv, (int)N, (int)D, (float)scale, causal ? 1 : 0, (int)window, dtype_code(q),
                   stream);
  } else {
    rc = gqafa_fwd_kv(q.data_ptr(), sq.s, k.data_ptr(), sk.s, v.data_ptr(), sv.s, o.data_ptr(), so.s, lp, (int)B,
                      (int)Hq, (int)Hkv, (int)N, (int)Nk, (int)D, (float)scale, causal ? 1 : 0, (int)window,
                      dtype_code(q), stream);
  }
  check(rc);
  return {o, want_lse ? lse : at::empty({0}, q.options().dtype(at::kFloat))};
}

std::tuple<at::Tensor, at::Tensor, at::Tensor> bwd(const at::Tensor& q_in, const at::Tensor& k_in,
                                                   const at::Tensor& v_in, const at::Tensor& o_in,
                                                   const at::Tensor& lse_in, const at::Tensor& do_in, bool causal,
                                                   int64_t window, double scale,
                                                   const c10::optional<at::Tensor>& workspace) {
  for (auto* t : {&q_in, &k_in, &v_in, &o_in, &do_in}) check_4d(*t, "tensor");
  c10::cuda::CUDAGuard guard(q_in.device());
  const at::Tensor q = abi_ready(q_in), k = abi_ready(k_in), v = abi_ready(v_in), o = abi_ready(o_in),
                   dout = abi_ready(do_in), lse = lse_in.contiguous();
  const int64_t B = q.size(0), Hq = q.size(1), N = q.size(2), D = q.size(3), Hkv = k.size(1);
  TORCH_CHECK_VALUE(lse.scalar_type() == at::kFloat && lse.numel() == B * Hq * N,
                    "gqafa: lse must be float32 (B, H_Q, N)");
  at::Tensor dq = abi_ready(at::empty_like(q)), dk = abi_ready(at::empty_like(k)),
             dv = abi_ready(at::empty_like(v));
  at::Tensor delta = at::empty({B, Hq, N}, q.options().dtype(at::kFloat));
  const Strides sq(q), sk(k), sv(v), so(o), sd(dout), sdq(dq), sdk(dk), sdv(dv);
  void* stream = c10::cuda::getCurrentCUDAStream(q.get_device()).stream();
  int rc;
  if (workspace.has_value() && workspace->defined() && workspace->numel() > 0) {
    const at::Tensor& ws = *workspace;
    TORCH_CHECK_VALUE(ws.is_cuda() && ws.is_contiguous(), "gqafa: workspace must be a contiguous CUDA tensor");
    rc = gqafa_bwd_ws(q.data_ptr(), sq.s, k.data_ptr(), sk.s, v.data_ptr(), sv.s, o.data_ptr(), so.s,
                      dout.data_ptr(), sd.s, lse.data_ptr<float>(), dq.data_ptr(), sdq.s, dk.data_ptr(), sdk.s,
                      dv.data_ptr(), sdv.s, delta.data_ptr<float>(), (int)B, (int)Hq, (int)Hkv, (int)N, (int)D,
                      (float)scale, causal ? 1 : 0, (int)window, dtype_code(q), stream, ws.data_ptr(),
                      (long long)(ws.numel() * ws.element_size()));
  } else {
    rc = gqafa_bwd(q.data_ptr(), sq.s, k.data_ptr(), sk.s, v.data_ptr(), sv.s, o.data_ptr(), so.s, dout.data_ptr(),
                   sd.s, lse.data_ptr<float>(), dq.data_ptr(), sdq.s, dk.data_ptr(), sdk.s, dv.data_ptr(), sdv.s,
                   delta.data_ptr<float>(), (int)B, (int)Hq, (int)Hkv, (int)N, (int)D, (float)scale,
                   causal ? 1 : 0, (int)window, dtype_code(q), stream);
  }
  check(rc);
  return {dq, dk, dv};
}

// Shapes only (no launch), for tracing and fake-tensor propagation.
std::tuple<at::Tensor, at::Tensor> fwd_meta(const at::Tensor& q, const at::Tensor& k, const at::Tensor& v, bool,
                                            int64_t, double, bool want_lse) {
  return {at::empty_like(q),
          at::empty(want_lse ? std::vector<int64_t>{q.size(0), q.size(1), q.size(2)} : std::vector<int64_t>{0},
                    q.options().dtype(at::kFloat))};
}

std::tuple<at::Tensor, at::Tensor, at::Tensor> bwd_meta(const at::Tensor& q, const at::Tensor& k,
                                                        const at::Tensor& v, const at::Tensor&, const at::Tensor&,
                                                        const at::Tensor&, bool, int64_t, double,
                                                        const c10::optional<at::Tensor>&) {
  return {at::empty_like(q), at::empty_like(k), at::empty_like(v)};
}

}  // namespace

TORCH_LIBRARY(gqafa, m) {
  m.def("fwd(Tensor q, Tensor k, Tensor v, bool causal, int window, float scale, bool want_lse) -> (Tensor, Tensor)");
  m.def(
      "bwd(Tensor q, Tensor k, Tensor v, Tensor o, Tensor lse, Tensor dout, bool causal, int window, float scale, "
      "Tensor? workspace) -> (Tensor, Tensor, Tensor)");
}

TORCH_LIBRARY_IMPL(gqafa, CUDA, m) {
  m.impl("fwd", &fwd);
  m.impl("bwd", &bwd);
}

TORCH_LIBRARY_IMPL(gqafa, Meta, m) {
  m.impl("fwd", &fwd_meta);
  m.impl("bwd", &bwd_meta);
}
