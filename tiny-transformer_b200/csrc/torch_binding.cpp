// PyTorch extension `tt_attention_C`: the reference's native operator surface
// (`attention_forward(q, k, v, past_len=0, segment_ids=None) -> (O, LSE)`, Tiny-transformer
// csrc/attention/bindings.cpp:4-8, attention.cu:32-159) on top of the C ABI in
// include/tt_attention.h. This file owns validation (same checks and message fragments as
// csrc/attention/attention_common.h:9-87 and attention.cu:36-73), output / workspace
// allocation through the caching allocator, and the layout decision; all device work goes
// through tt_attn_forward_bf16 on the current stream.
#include <torch/extension.h>

#include <ATen/cuda/CUDAContext.h>
#include <c10/core/GradMode.h>
#include <c10/cuda/CUDAGuard.h>
#include <c10/cuda/CUDAStream.h>

#include <cstdint>
#include <limits>
#include <optional>
#include <tuple>

#include "tt_attention.h"

namespace {

void check_tensors(const torch::Tensor& q, const torch::Tensor& k, const torch::Tensor& v) {
  for (const auto* t : {&q, &k, &v}) {
    TORCH_CHECK(t->defined(), "attention inputs must be defined");
    TORCH_CHECK(t->is_cuda(), "All inputs must be CUDA tensors");
  }
  for (const auto* t : {&q, &k, &v}) {
    TORCH_CHECK(t->device() == q.device(), "All inputs must be on the same device");
    TORCH_CHECK(t->scalar_type() == at::kFloat || t->scalar_type() == at::kBFloat16,
                "attention supports only float32 and bf16 inputs");
    TORCH_CHECK(t->scalar_type() == q.scalar_type(), "q, k, v must have the same dtype");
    TORCH_CHECK(t->layout() == at::kStrided, "All inputs must be strided tensors");
  }
  TORCH_CHECK(q.dim() == 4 && k.dim() == 4 && v.dim() == 4, "q, k, v must be a 4D tensor");
  TORCH_CHECK(k.size(0) == q.size(0) && v.size(0) == q.size(0),
              "q, k, v must have the same first dimension");
  TORCH_CHECK(k.size(1) == q.size(1) && v.size(1) == q.size(1),
              "q, k, v must have the same second dimension");
  TORCH_CHECK(k.size(3) == q.size(3) && v.size(3) == q.size(3),
              "q, k, v must have the same last dimension");
  TORCH_CHECK(q.size(3) == TT_ATTN_HEAD_DIM, "attention currently supports only head_dim=64");
  TORCH_CHECK(q.size(0) > 0 && q.size(1) > 0 && q.size(2) > 0 && k.size(2) > 0,
              "attention batch, heads and sequence lengths must be positive");
}

void check_mask(const torch::Tensor& q, const torch::Tensor& k, const torch::Tensor& v,
                int64_t past_len) {
  TORCH_CHECK(past_len >= 0, "past_len must be non-negative");
  TORCH_CHECK(v.size(2) == k.size(2), "k and v must have the same sequence length");
  // Subtract instead of adding: past_len + Tq may overflow.
  TORCH_CHECK(k.size(2) >= q.size(2) && past_len == k.size(2) - q.size(2),
              "expected Tk == past_len + Tq");
}

bool readable_in_place(const torch::Tensor& x) {
  const int64_t st[4] = {x.stride(0), x.stride(1), x.stride(2), x.stride(3)};
  int64_t canon[4] = {st[0], st[1], st[2], st[3]};
  // Size-1 dimensions are never stepped over; their stride does not matter.
  const int64_t contiguous[3] = {x.size(1) * x.size(2) * x.size(3), x.size(2) * x.size(3),
                                 x.size(3)};
  for (int d = 0; d < 3; ++d)
    if (x.size(d) == 1) canon[d] = contiguous[d];
  return tt_attn_layout_supported(x.data_ptr(), canon) != 0;
}

// Same fallback as the reference's aligned_contiguous (attention.cu:20-29), taken only
// when the TMA / bulk-copy path cannot read the view in place.
torch::Tensor aligned_contiguous(torch::Tensor x) {
  if (readable_in_place(x)) return x;
  x = x.contiguous();
  if (reinterpret_cast<uintptr_t>(x.data_ptr()) % 16 != 0) x = x.clone();
  return x;
}

}  // namespace

std::tuple<torch::Tensor, torch::Tensor> attention_forward(
    torch::Tensor q, torch::Tensor k, torch::Tensor v, int64_t past_len,
    std::optional<torch::Tensor> segment_ids, std::optional<torch::Tensor> kv_lens) {
  check_tensors(q, k, v);
  check_mask(q, k, v, past_len);
  TORCH_CHECK(!(at::GradMode::is_enabled() &&
                (q.requires_grad() || k.requires_grad() || v.requires_grad())),
              "student attention backward requires the Python autograd binding; "
              "use student.attention or no_grad for inference");
  TORCH_CHECK(q.scalar_type() == at::kBFloat16,
              "float32 attention is not provided by the sm_100a path; pass bf16 q, k, v");
  TORCH_CHECK(!segment_ids.has_value(), "segment_ids is not supported for bf16 kernel");
  const int64_t B = q.size(0), H = q.size(1), Tq = q.size(2), Tk = k.size(2);
  const int64_t max_grid = std::numeric_limits<int32_t>::max();
  const int64_t q_tiles = (Tq + 127) / 128;
  // Divide before multiplying: B * H * tiles must fit grid.x.
  TORCH_CHECK(q_tiles <= max_grid && B <= max_grid / q_tiles / H,
              "attention shape exceeds the supported CUDA grid limits");
  TORCH_CHECK(Tk <= std::numeric_limits<int32_t>::max(),
              "bf16 attention sequence lengths must fit int32 (Tk <= INT32_MAX)");
  if (kv_lens.has_value()) {
    const auto& lens = *kv_lens;
    TORCH_CHECK(lens.defined() && lens.is_cuda() && lens.device() == q.device(),
                "kv_lens must be a CUDA tensor on the same device as q");
    TORCH_CHECK(lens.scalar_type() == at::kInt || lens.scalar_type() == at::kLong,
                "kv_lens must be int32 or int64");
    TORCH_CHECK(lens.dim() == 1 && lens.size(0) == B, "kv_lens must have shape [B]");
    TORCH_CHECK(Tq == 1, "kv_lens requires single-token decode (Tq == 1)");
  }

  const c10::cuda::CUDAGuard device_guard(q.device());
  const auto* props = at::cuda::getDeviceProperties(q.get_device());
  TORCH_CHECK(props->major == 10,
              "the bf16 attention kernels require an sm_100 GPU (compute capability 10.x); "
              "found SM", props->major, props->minor);
  auto stream = c10::cuda::getCurrentCUDAStream(q.get_device());

  q = aligned_contiguous(q);
  k = aligned_contiguous(k);
  v = aligned_contiguous(v);
  torch::Tensor lens32;
  if (kv_lens.has_value()) lens32 = kv_lens->to(at::kInt).contiguous();

  auto o = torch::empty({B, H, Tq, TT_ATTN_HEAD_DIM}, q.options());
  auto lse = torch::empty({B, H, Tq}, q.options().dtype(at::kFloat));
  const size_t ws_bytes = tt_attn_forward_workspace_size(B, H, Tq, Tk);
  torch::Tensor ws;
  if (ws_bytes > 0)
    ws = torch::empty({static_cast<int64_t>(ws_bytes)}, q.options().dtype(at::kByte));

  const int64_t qs[4] = {q.stride(0), q.stride(1), q.stride(2), q.stride(3)};
  const int64_t ks[4] = {k.stride(0), k.stride(1), k.stride(2), k.stride(3)};
  const int64_t vs[4] = {v.stride(0), v.stride(1), v.stride(2), v.stride(3)};
  const tt_attn_status st = tt_attn_forward_bf16(
      q.data_ptr(), qs, k.data_ptr(), ks, v.data_ptr(), vs, B, H, Tq, Tk, TT_ATTN_HEAD_DIM,
      past_len, lens32.defined() ? lens32.data_ptr<int32_t>() : nullptr, o.data_ptr(),
      lse.data_ptr<float>(), ws_bytes > 0 ? ws.data_ptr() : nullptr, ws_bytes,
      static_cast<void*>(stream.stream()));
  TORCH_CHECK(st == TT_ATTN_OK, "tt_attn_forward_bf16 failed: ", tt_attn_status_string(st),
              ": ", tt_attn_last_error());
  return {o, lse};
}

void check_upstream(const torch::Tensor& q, const torch::Tensor& dO, const torch::Tensor& o,
                    const torch::Tensor& lse) {
  for (const torch::Tensor* x : {&dO, &o, &lse}) {
    TORCH_CHECK(x->defined(), "dO, O and LSE must be defined");
    TORCH_CHECK(x->is_cuda() && x->device() == q.device(),
                "dO, O and LSE must be CUDA tensors on the same device as q");
    TORCH_CHECK(x->layout() == at::kStrided, "dO, O and LSE must have strided layout");
  }
  TORCH_CHECK(dO.scalar_type() == q.scalar_type() && o.scalar_type() == q.scalar_type(),
              "dO and O must have the same dtype as q");
  TORCH_CHECK(dO.sizes() == q.sizes() && o.sizes() == q.sizes(),
              "dO and O must have the same shape as q");
  TORCH_CHECK(lse.scalar_type() == at::kFloat, "LSE must be float32");
  TORCH_CHECK(lse.dim() == 3 && lse.size(0) == q.size(0) && lse.size(1) == q.size(1) &&
                  lse.size(2) == q.size(2),
              "LSE must have shape [B, Nh, Tq]");
}

// Contiguous, 16-byte aligned copy of x unless it already is one.
torch::Tensor contiguous_aligned(torch::Tensor x) {
  x = x.contiguous();
  if (reinterpret_cast<uintptr_t>(x.data_ptr()) % 16 != 0) x = x.clone();
  return x;
}

// The reference's native backward (attention.cu:161-234): same argument order, validation
// order and message fragments; all device work through tt_attn_backward_bf16.
std::tuple<torch::Tensor, torch::Tensor, torch::Tensor> attention_backward(
    torch::Tensor q, torch::Tensor k, torch::Tensor v, torch::Tensor dO, torch::Tensor O,
    torch::Tensor lse, int64_t past_len, std::optional<torch::Tensor> segment_ids) {
  check_tensors(q, k, v);
  check_mask(q, k, v, past_len);
  TORCH_CHECK(q.scalar_type() == at::kBFloat16, "student attention backward supports only bf16");
  TORCH_CHECK(!segment_ids.has_value(),
              "segment_ids is not supported for bf16 attention backward");
  check_upstream(q, dO, O, lse);
  const int64_t B = q.size(0), H = q.size(1), Tq = q.size(2), Tk = k.size(2);
  TORCH_CHECK(Tk <= std::numeric_limits<int32_t>::max(),
              "bf16 attention sequence lengths must fit int32 (Tk <= INT32_MAX)");
  const int64_t max_grid = std::numeric_limits<int32_t>::max();
  const int64_t k_tiles = (Tk + 127) / 128;  // >= query tiles
  TORCH_CHECK(B <= max_grid / H && k_tiles <= max_grid / (B * H),
              "attention backward shape exceeds the supported CUDA grid limits");
  const c10::cuda::CUDAGuard device_guard(q.device());
  const auto* props = at::cuda::getDeviceProperties(q.get_device());
  TORCH_CHECK(props->major == 10,
              "the bf16 attention kernels require an sm_100 GPU (compute capability 10.x); "
              "found SM", props->major, props->minor);
  auto stream = c10::cuda::getCurrentCUDAStream(q.get_device());
  // Validated; now materialise the layouts the kernels read (on the current stream).
  q = aligned_contiguous(q);
  k = aligned_contiguous(k);
  v = aligned_contiguous(v);
  dO = contiguous_aligned(dO);
  O = contiguous_aligned(O);
  lse = lse.contiguous();
  auto dq = torch::empty({B, H, Tq, TT_ATTN_HEAD_DIM}, q.options());
  auto dk = torch::empty({B, H, Tk, TT_ATTN_HEAD_DIM}, q.options());
  auto dv = torch::empty({B, H, Tk, TT_ATTN_HEAD_DIM}, q.options());
  const size_t ws_bytes = tt_attn_backward_workspace_size(B, H, Tq);
  auto ws = torch::empty({static_cast<int64_t>(ws_bytes)}, q.options().dtype(at::kByte));
  const int64_t qs[4] = {q.stride(0), q.stride(1), q.stride(2), q.stride(3)};
  const int64_t ks[4] = {k.stride(0), k.stride(1), k.stride(2), k.stride(3)};
  const int64_t vs[4] = {v.stride(0), v.stride(1), v.stride(2), v.stride(3)};
  // Under torch.use_deterministic_algorithms(True) take the fixed-order path (the fused kernel
  // adds dQ contributions with reduce-adds in timing-dependent order).
  const auto backward_fn = at::globalContext().deterministicAlgorithms()
                               ? tt_attn_backward_bf16_deterministic
                               : tt_attn_backward_bf16;
  const tt_attn_status st = backward_fn(
      q.data_ptr(), qs, k.data_ptr(), ks, v.data_ptr(), vs, dO.data_ptr(), O.data_ptr(),
      lse.data_ptr<float>(), B, H, Tq, Tk, TT_ATTN_HEAD_DIM, past_len, dq.data_ptr(),
      dk.data_ptr(), dv.data_ptr(), ws.data_ptr(), ws_bytes, static_cast<void*>(stream.stream()));
  TORCH_CHECK(st == TT_ATTN_OK, "tt_attn_backward_bf16 failed: ", tt_attn_status_string(st),
              ": ", tt_attn_last_error());
  return {dq, dk, dv};
}

// Fused RoPE + KV-cache append (tt_rope_append_bf16). `position` is either a Python int or an
// int64 CUDA tensor with one element (read on the device, for captured decode steps).
torch::Tensor rope_append(const torch::Tensor& qkv, const torch::Tensor& cos,
                          const torch::Tensor& sin, const pybind11::object& position,
                          torch::Tensor cache_k, torch::Tensor cache_v) {
  TORCH_CHECK(qkv.is_cuda() && cos.is_cuda() && sin.is_cuda() && cache_k.is_cuda() &&
                  cache_v.is_cuda(), "rope_append: all tensors must be CUDA tensors");
  for (const torch::Tensor* t : {&cos, &sin, static_cast<const torch::Tensor*>(&cache_k),
                                 static_cast<const torch::Tensor*>(&cache_v)})
    TORCH_CHECK(t->device() == qkv.device(), "rope_append: all tensors must be on the same device");
  TORCH_CHECK(qkv.scalar_type() == at::kBFloat16 && cache_k.scalar_type() == at::kBFloat16 &&
                  cache_v.scalar_type() == at::kBFloat16, "rope_append: qkv and caches must be bf16");
  TORCH_CHECK(cos.scalar_type() == at::kFloat && sin.scalar_type() == at::kFloat,
              "rope_append: cos/sin tables must be float32");
  TORCH_CHECK(qkv.dim() == 5 && qkv.size(2) == 3 && qkv.size(4) == TT_ATTN_HEAD_DIM &&
                  qkv.is_contiguous(), "rope_append: qkv must be a contiguous [B, T, 3, H, 64] tensor");
  TORCH_CHECK(cos.dim() == 2 && cos.size(1) == TT_ATTN_HEAD_DIM / 2 && cos.is_contiguous() &&
                  sin.sizes() == cos.sizes() && sin.is_contiguous(),
              "rope_append: cos/sin must be contiguous [L, 32] tables");
  const int64_t B = qkv.size(0), T = qkv.size(1), H = qkv.size(3);
  for (const torch::Tensor* c : {&cache_k, &cache_v})
    TORCH_CHECK(c->dim() == 4 && c->size(0) == B && c->size(1) == H &&
                    c->size(3) == TT_ATTN_HEAD_DIM && c->stride(3) == 1,
                "rope_append: caches must be [B, H, capacity, 64] with contiguous rows");
  TORCH_CHECK(cache_v.size(2) == cache_k.size(2), "rope_append: caches must have equal capacity");
  int64_t pos = 0;
  const int64_t* pos_dev = nullptr;
  torch::Tensor pos_t;
  if (pybind11::isinstance<pybind11::int_>(position)) {
    pos = position.cast<int64_t>();
  } else {
    pos_t = position.cast<torch::Tensor>();
    TORCH_CHECK(pos_t.is_cuda() && pos_t.device() == qkv.device() &&
                    pos_t.scalar_type() == at::kLong && pos_t.numel() == 1,
                "rope_append: a tensor position must be a one-element int64 CUDA tensor");
    pos_dev = pos_t.data_ptr<int64_t>();
  }
  const c10::cuda::CUDAGuard device_guard(qkv.device());
  auto q_out = torch::empty({B, H, T, TT_ATTN_HEAD_DIM}, qkv.options());
  const int64_t ks[4] = {cache_k.stride(0), cache_k.stride(1), cache_k.stride(2), 1};
  const int64_t vs[4] = {cache_v.stride(0), cache_v.stride(1), cache_v.stride(2), 1};
  auto stream = c10::cuda::getCurrentCUDAStream(qkv.get_device());
  const tt_attn_status st = tt_rope_append_bf16(
      qkv.data_ptr(), B, T, H, cos.data_ptr<float>(), sin.data_ptr<float>(), cos.size(0), pos,
      pos_dev, q_out.data_ptr(), cache_k.data_ptr(), ks, cache_v.data_ptr(), vs, cache_k.size(2),
      static_cast<void*>(stream.stream()));
  TORCH_CHECK(st == TT_ATTN_OK, "tt_rope_append_bf16 failed: ", tt_attn_status_string(st), ": ",
              tt_attn_last_error());
  return q_out;
}

// QKV projection + RoPE + KV-cache append in one kernel (tt_qkv_rope_append_bf16). `hidden`
// is the normalised hidden state [B, T, dim]; `w_qkv` the layer's [3 * H * 64, dim] weight;
// `position` as for rope_append.
torch::Tensor qkv_rope_append(const torch::Tensor& hidden, const torch::Tensor& w_qkv,
                              const torch::Tensor& cos, const torch::Tensor& sin,
                              const pybind11::object& position, torch::Tensor cache_k,
                              torch::Tensor cache_v) {
  for (const torch::Tensor* t : {&hidden, &w_qkv, &cos, &sin,
                                 static_cast<const torch::Tensor*>(&cache_k),
                                 static_cast<const torch::Tensor*>(&cache_v)}) {
    TORCH_CHECK(t->is_cuda(), "qkv_rope_append: all tensors must be CUDA tensors");
    TORCH_CHECK(t->device() == hidden.device(),
                "qkv_rope_append: all tensors must be on the same device");
  }
  TORCH_CHECK(hidden.scalar_type() == at::kBFloat16 && w_qkv.scalar_type() == at::kBFloat16 &&
                  cache_k.scalar_type() == at::kBFloat16 && cache_v.scalar_type() == at::kBFloat16,
              "qkv_rope_append: hidden, w_qkv and the caches must be bf16");
  TORCH_CHECK(cos.scalar_type() == at::kFloat && sin.scalar_type() == at::kFloat,
              "qkv_rope_append: cos/sin tables must be float32");
  TORCH_CHECK(hidden.dim() == 3 && hidden.is_contiguous(),
              "qkv_rope_append: hidden must be a contiguous [B, T, dim] tensor");
  const int64_t B = hidden.size(0), T = hidden.size(1), dim = hidden.size(2);
  TORCH_CHECK(w_qkv.dim() == 2 && w_qkv.is_contiguous() && w_qkv.size(1) == dim &&
                  w_qkv.size(0) % (3 * TT_ATTN_HEAD_DIM) == 0,
              "qkv_rope_append: w_qkv must be a contiguous [3 * H * 64, dim] weight");
  const int64_t H = w_qkv.size(0) / (3 * TT_ATTN_HEAD_DIM);
  TORCH_CHECK(cos.dim() == 2 && cos.size(1) == TT_ATTN_HEAD_DIM / 2 && cos.is_contiguous() &&
                  sin.sizes() == cos.sizes() && sin.is_contiguous(),
              "qkv_rope_append: cos/sin must be contiguous [L, 32] tables");
  for (const torch::Tensor* c : {&cache_k, &cache_v})
    TORCH_CHECK(c->dim() == 4 && c->size(0) == B && c->size(1) == H &&
                    c->size(3) == TT_ATTN_HEAD_DIM && c->stride(3) == 1,
                "qkv_rope_append: caches must be [B, H, capacity, 64] with contiguous rows");
  TORCH_CHECK(cache_v.size(2) == cache_k.size(2),
              "qkv_rope_append: caches must have equal capacity");
  int64_t pos = 0;
  const int64_t* pos_dev = nullptr;
  torch::Tensor pos_t;
  if (pybind11::isinstance<pybind11::int_>(position)) {
    pos = position.cast<int64_t>();
  } else {
    pos_t = position.cast<torch::Tensor>();
    TORCH_CHECK(pos_t.is_cuda() && pos_t.device() == hidden.device() &&
                    pos_t.scalar_type() == at::kLong && pos_t.numel() == 1,
                "qkv_rope_append: a tensor position must be a one-element int64 CUDA tensor");
    pos_dev = pos_t.data_ptr<int64_t>();
  }
  const c10::cuda::CUDAGuard device_guard(hidden.device());
  auto q_out = torch::empty({B, H, T, TT_ATTN_HEAD_DIM}, hidden.options());
  const int64_t ks[4] = {cache_k.stride(0), cache_k.stride(1), cache_k.stride(2), 1};
  const int64_t vs[4] = {cache_v.stride(0), cache_v.stride(1), cache_v.stride(2), 1};
  auto stream = c10::cuda::getCurrentCUDAStream(hidden.get_device());
  const tt_attn_status st = tt_qkv_rope_append_bf16(
      hidden.data_ptr(), B, T, dim, w_qkv.data_ptr(), H, cos.data_ptr<float>(),
      sin.data_ptr<float>(), cos.size(0), pos, pos_dev, q_out.data_ptr(), cache_k.data_ptr(), ks,
      cache_v.data_ptr(), vs, cache_k.size(2), static_cast<void*>(stream.stream()));
  TORCH_CHECK(st == TT_ATTN_OK, "tt_qkv_rope_append_bf16 failed: ", tt_attn_status_string(st),
              ": ", tt_attn_last_error());
  return q_out;
}

PYBIND11_MODULE(TORCH_EXTENSION_NAME, m) {
  m.def("attention_forward", &attention_forward,
        "BF16 causal attention forward on sm_100a (returns O and natural-log FP32 LSE)",
        pybind11::arg("q"), pybind11::arg("k"), pybind11::arg("v"),
        pybind11::arg("past_len") = 0, pybind11::arg("segment_ids") = pybind11::none(),
        pybind11::arg("kv_lens") = pybind11::none());
  m.def("attention_backward", &attention_backward,
        "BF16 causal attention backward on sm_100a (preprocess, dQ, dK/dV); returns dq, dk, dv",
        pybind11::arg("q"), pybind11::arg("k"), pybind11::arg("v"), pybind11::arg("dO"),
        pybind11::arg("O"), pybind11::arg("lse"), pybind11::arg("past_len") = 0,
        pybind11::arg("segment_ids") = pybind11::none());
  m.def("rope_append", &rope_append,
        "Fused RoPE on q/k of a [B, T, 3, H, 64] QKV projection + KV-cache append; returns rope(q)",
        pybind11::arg("qkv"), pybind11::arg("cos"), pybind11::arg("sin"),
        pybind11::arg("position"), pybind11::arg("cache_k"), pybind11::arg("cache_v"));
  m.def("qkv_rope_append", &qkv_rope_append,
        "QKV projection + RoPE on q/k + KV-cache append in one kernel; returns rope(q)",
        pybind11::arg("hidden"), pybind11::arg("w_qkv"), pybind11::arg("cos"),
        pybind11::arg("sin"), pybind11::arg("position"), pybind11::arg("cache_k"),
        pybind11::arg("cache_v"));
  m.attr("HEAD_DIM") = TT_ATTN_HEAD_DIM;
  m.attr("ABI_VERSION") = TT_ATTN_ABI_VERSION;
}
