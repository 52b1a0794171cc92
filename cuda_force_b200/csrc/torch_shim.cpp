// PyTorch dispatcher shim over the C ABI, loadable as the reference's
// `cudaforge._C` extension module.
//
// Registers all ten of the reference's operator schemas in the `cudaforge`
// namespace, byte-identical (reference cpp/src/bindings.cpp:342-355), plus
// additive ops. For the five on the accelerated path (quantize_int8,
// dequantize_int8, lora_linear, rmsnorm, fused_residual_rmsnorm) the CUDA key
// runs this build's sm_100a kernels through the C ABI; the other five keep the
// reference's semantics as ATen compositions (see below). The Autograd key raises
// (autogradNotImplementedFallback), as the reference does (bindings.cpp:369-377).
//
// CPU tensors: the reference's extension registers ATen CPU kernels for its
// schemas (bindings.cpp:379-390), and its Python wrapper sends CPU tensors to
// them (python/cudaforge/ops.py:150-152). The five reference schemas keep that
// contract here with ATen compositions of the reference semantics, so callers
// of the reference that pass host tensors still work. The dispatcher selects
// the kernel by the tensors' device: a CUDA tensor never reaches these, and
// this package's own Python API refuses host tensors before dispatching.
//
// Each CUDA impl validates like the reference's CUDA impl (TORCH_CHECK
// messages that name the operand), allocates its outputs on the input's
// device, and launches on PyTorch's current stream.
#include <Python.h>

#include <ATen/ATen.h>
#include <c10/cuda/CUDAGuard.h>
#include <c10/cuda/CUDAStream.h>
#include <torch/csrc/autograd/autograd_not_implemented_fallback.h>
#include <torch/library.h>

#include <vector>

#include "cudaforge_b200.h"

namespace {

cf_stream_t current_stream() {
  return reinterpret_cast<cf_stream_t>(at::cuda::getCurrentCUDAStream().stream());
}

void check_status(int status, const char *op) {
  if (status == CF_OK) return;
  if (status == CF_ERR_CUDA) {
    TORCH_CHECK(false, op, ": ", cf_status_string(status), " (cudaError ", cf_last_cuda_error(),
                ")");
  }
  TORCH_CHECK(false, op, ": ", cf_status_string(status));
}

int dtype_code(const at::Tensor &t, const char *name) {
  switch (t.scalar_type()) {
    case at::kFloat: return CF_DTYPE_F32;
    case at::kHalf: return CF_DTYPE_F16;
    case at::kBFloat16: return CF_DTYPE_BF16;
    default:
      TORCH_CHECK(false, name, " must be float32, float16 or bfloat16, got ", t.scalar_type());
  }
  return -1;
}

void check_contiguous(const at::Tensor &t, const char *name) {
  TORCH_CHECK(t.is_contiguous(), name, " must be contiguous; call .contiguous() first");
}

void check_cuda(const at::Tensor &t, const char *name) {
  TORCH_CHECK(t.is_cuda(), name, " must be a CUDA tensor (this build has no CPU path)");
}

// Storage order of a 2-D operand that is either contiguous (REF) or the
// transpose of a contiguous tensor (T). Anything else is rejected.
int layout_of(const at::Tensor &t, const char *name) {
  TORCH_CHECK(t.dim() == 2, name, " must be 2-D, got ", t.dim(), " dimensions");
  if (t.is_contiguous()) return CF_LAYOUT_REF;
  if (t.t().is_contiguous()) return CF_LAYOUT_T;
  TORCH_CHECK(false, name, " must be contiguous (or the transpose of a contiguous tensor)");
  return -1;
}

// The kernels take ranks 16, 32 and 64 (the MMA's K granularity). A smaller
// rank is zero-padded to the next of those, which leaves the product unchanged.
int64_t padded_rank(int64_t r) {
  TORCH_CHECK(r >= 1 && r <= 64, "rank must be between 1 and 64, got ", r);
  return r <= 16 ? 16 : r <= 32 ? 32 : 64;
}

void pad_adapter(at::Tensor &a, at::Tensor &b, int &al, int &bl, int64_t r, int64_t rp) {
  if (rp == r) return;
  at::Tensor ap = at::zeros({a.size(0), rp}, a.options());
  ap.narrow(1, 0, r).copy_(a);
  at::Tensor bp = at::zeros({rp, b.size(1)}, b.options());
  bp.narrow(0, 0, r).copy_(b);
  a = ap;
  b = bp;
  al = CF_LAYOUT_REF;
  bl = CF_LAYOUT_REF;
}

std::vector<at::Tensor> quantize_int8_cuda(const at::Tensor &input) {
  check_cuda(input, "input");
  check_contiguous(input, "input");
  const int dtype = dtype_code(input, "input");
  const c10::cuda::CUDAGuard guard(input.device());
  const int64_t count = input.numel();
  at::Tensor codes = at::empty(input.sizes(), input.options().dtype(at::kChar));
  at::Tensor scales = at::empty({cf_quant_scale_count(count)}, input.options().dtype(at::kFloat));
  check_status(cf_quantize_int8(input.data_ptr(), dtype, codes.data_ptr<int8_t>(),
                                scales.data_ptr<float>(), count, current_stream()),
               "quantize_int8");
  return {codes, scales};
}

at::Tensor dequantize_int8_cuda(const at::Tensor &quantised, const at::Tensor &scales) {
  check_cuda(quantised, "quantised");
  check_cuda(scales, "scales");
  TORCH_CHECK(quantised.scalar_type() == at::kChar, "quantised must be int8");
  TORCH_CHECK(scales.scalar_type() == at::kFloat, "scales must be float32, got ",
              scales.scalar_type());
  check_contiguous(quantised, "quantised");
  check_contiguous(scales, "scales");
  const int64_t count = quantised.numel();
  TORCH_CHECK(scales.numel() == cf_quant_scale_count(count), "expected ",
              cf_quant_scale_count(count), " block scales, got ", scales.numel());
  const c10::cuda::CUDAGuard guard(quantised.device());
  at::Tensor out = at::empty(quantised.sizes(), scales.options());
  check_status(cf_dequantize_int8(quantised.data_ptr<int8_t>(), scales.data_ptr<float>(),
                                  out.data_ptr<float>(), count, current_stream()),
               "dequantize_int8");
  return out;
}

at::Tensor quantize_dequantize_cuda(const at::Tensor &input) {
  check_cuda(input, "input");
  check_contiguous(input, "input");
  const int dtype = dtype_code(input, "input");
  const c10::cuda::CUDAGuard guard(input.device());
  at::Tensor out = at::empty(input.sizes(), input.options().dtype(at::kFloat));
  check_status(cf_quantize_dequantize(input.data_ptr(), dtype, out.data_ptr<float>(),
                                      input.numel(), current_stream()),
               "quantize_dequantize");
  return out;
}

std::vector<at::Tensor> quantize_int8_many_cuda(at::TensorList inputs) {
  std::vector<at::Tensor> result;
  if (inputs.empty()) return result;
  const int dtype = dtype_code(inputs[0], "inputs[0]");
  const c10::cuda::CUDAGuard guard(inputs[0].device());
  std::vector<cf_quant_segment> segs;
  segs.reserve(inputs.size());
  result.reserve(2 * inputs.size());
  for (const at::Tensor &t : inputs) {
    check_cuda(t, "inputs[i]");
    check_contiguous(t, "inputs[i]");
    TORCH_CHECK(t.scalar_type() == inputs[0].scalar_type(), "all inputs must share one dtype");
    TORCH_CHECK(t.device() == inputs[0].device(), "all inputs must be on one device");
    at::Tensor codes = at::empty(t.sizes(), t.options().dtype(at::kChar));
    at::Tensor scales = at::empty({cf_quant_scale_count(t.numel())}, t.options().dtype(at::kFloat));
    segs.push_back({t.data_ptr(), codes.data_ptr<int8_t>(), scales.data_ptr<float>(), t.numel()});
    result.push_back(codes);
    result.push_back(scales);
  }
  check_status(cf_quantize_int8_many(segs.data(), static_cast<int>(segs.size()), dtype,
                                     current_stream()),
               "quantize_int8_many");
  return result;
}

// Shapes are those of the reference op: x [M, K], w [K, N], a [K, r], b [r, N]
// (reference cpp/src/bindings.cpp:94-127). w, a and b may also be transposed
// views of contiguous tensors, which is how nn.Linear-layout weights arrive.
at::Tensor lora_linear_cuda(const at::Tensor &x, const at::Tensor &w, const at::Tensor &a,
                            const at::Tensor &b, double scale) {
  for (const auto &[t, name] : std::vector<std::pair<at::Tensor, const char *>>{
           {x, "x"}, {w, "w"}, {a, "a"}, {b, "b"}}) {
    check_cuda(t, name);
  }
  TORCH_CHECK(x.dim() == 2, "x must be 2-D, got ", x.dim(), " dimensions");
  check_contiguous(x, "x");
  const int dtype = dtype_code(x, "x");
  for (const at::Tensor *t : {&w, &a, &b}) {
    TORCH_CHECK(t->scalar_type() == x.scalar_type(), "x, w, a and b must share one dtype");
  }
  const int wl = layout_of(w, "w");
  const int al = layout_of(a, "a");
  const int bl = layout_of(b, "b");
  const int64_t m = x.size(0), k = x.size(1), n = w.size(1), r = a.size(1);
  TORCH_CHECK(w.size(0) == k, "w must be [in_features, out_features]; got [", w.size(0), ", ",
              w.size(1), "] for in_features=", k);
  TORCH_CHECK(a.size(0) == k, "a must be [in_features, rank]; got [", a.size(0), ", ", a.size(1),
              "] for in_features=", k);
  TORCH_CHECK(b.size(0) == r && b.size(1) == n, "b must be [rank, out_features] = [", r, ", ", n,
              "]; got [", b.size(0), ", ", b.size(1), "]");
  const c10::cuda::CUDAGuard guard(x.device());
  at::Tensor ap = a, bp = b;
  int alp = al, blp = bl;
  const int64_t rp = padded_rank(r);
  pad_adapter(ap, bp, alp, blp, r, rp);
  // The kernels read rows with TMA, whose row strides are whole 16-byte units
  // (8 16-bit or 4 fp32 elements). Other feature counts are zero-padded here,
  // which leaves the product unchanged, and the output is cut back.
  const int64_t unit = dtype == CF_DTYPE_F32 ? 4 : 8;
  const int64_t kp = (k + unit - 1) / unit * unit;
  const int64_t np = (n + unit - 1) / unit * unit;
  at::Tensor xp = x, wp = w;
  int wlp = wl;
  if (kp != k || np != n) {
    if (kp != k) {
      xp = at::zeros({m, kp}, x.options());
      xp.narrow(1, 0, k).copy_(x);
      at::Tensor a2 = at::zeros({kp, rp}, ap.options());
      a2.narrow(0, 0, k).copy_(ap);
      ap = a2;
      alp = CF_LAYOUT_REF;
    }
    wp = at::zeros({kp, np}, w.options());
    wp.narrow(0, 0, k).narrow(1, 0, n).copy_(w);
    wlp = CF_LAYOUT_REF;
    if (np != n) {
      at::Tensor b2 = at::zeros({rp, np}, bp.options());
      b2.narrow(1, 0, n).copy_(bp);
      bp = b2;
      blp = CF_LAYOUT_REF;
    }
  }
  at::Tensor y = at::empty({m, np}, x.options());
  const size_t ws_bytes = cf_lora_linear_workspace_bytes(m, rp);
  at::Tensor ws = at::empty({static_cast<int64_t>(ws_bytes)}, x.options().dtype(at::kByte));
  check_status(cf_lora_linear(xp.data_ptr(), wp.data_ptr(), wlp, ap.data_ptr(), alp,
                              bp.data_ptr(), blp, y.data_ptr(), m, kp, np, rp,
                              static_cast<float>(scale), dtype, ws.data_ptr(), ws_bytes,
                              current_stream()),
               "lora_linear");
  return np == n ? y : y.narrow(1, 0, n).contiguous();
}

// x [M, K]; w_codes int8 [N, K] (nn.Linear layout, blocks of 64 along K);
// w_scales float32 [N*K/64]; a [K, r]; b [r, N].
at::Tensor lora_linear_int8_cuda(const at::Tensor &x, const at::Tensor &w_codes,
                                 const at::Tensor &w_scales, const at::Tensor &a,
                                 const at::Tensor &b, double scale) {
  for (const auto &[t, name] : std::vector<std::pair<at::Tensor, const char *>>{
           {x, "x"}, {w_codes, "w_codes"}, {w_scales, "w_scales"}, {a, "a"}, {b, "b"}}) {
    check_cuda(t, name);
  }
  TORCH_CHECK(x.dim() == 2, "x must be 2-D, got ", x.dim(), " dimensions");
  check_contiguous(x, "x");
  const int dtype = dtype_code(x, "x");
  TORCH_CHECK(dtype != CF_DTYPE_F32, "lora_linear_int8: x must be bfloat16 or float16");
  TORCH_CHECK(a.scalar_type() == x.scalar_type() && b.scalar_type() == x.scalar_type(),
              "x, a and b must share one dtype");
  TORCH_CHECK(w_codes.scalar_type() == at::kChar, "w_codes must be int8");
  TORCH_CHECK(w_scales.scalar_type() == at::kFloat, "w_scales must be float32");
  TORCH_CHECK(w_codes.dim() == 2, "w_codes must be 2-D [out_features, in_features]");
  check_contiguous(w_codes, "w_codes");
  check_contiguous(w_scales, "w_scales");
  const int al = layout_of(a, "a");
  const int bl = layout_of(b, "b");
  const int64_t m = x.size(0), k = x.size(1), n = w_codes.size(0), r = a.size(1);
  TORCH_CHECK(w_codes.size(1) == k, "w_codes must be [out_features, in_features]; got [",
              w_codes.size(0), ", ", w_codes.size(1), "] for in_features=", k);
  TORCH_CHECK(w_scales.numel() == cf_quant_scale_count(n * k), "expected ",
              cf_quant_scale_count(n * k), " block scales, got ", w_scales.numel());
  TORCH_CHECK(a.size(0) == k, "a must be [in_features, rank]; got [", a.size(0), ", ", a.size(1),
              "] for in_features=", k);
  TORCH_CHECK(b.size(0) == r && b.size(1) == n, "b must be [rank, out_features] = [", r, ", ", n,
              "]; got [", b.size(0), ", ", b.size(1), "]");
  const c10::cuda::CUDAGuard guard(x.device());
  at::Tensor ap = a, bp = b;
  int alp = al, blp = bl;
  const int64_t rp = padded_rank(r);
  pad_adapter(ap, bp, alp, blp, r, rp);
  at::Tensor y = at::empty({m, n}, x.options());
  const size_t ws_bytes = cf_lora_linear_workspace_bytes(m, rp);
  at::Tensor ws = at::empty({static_cast<int64_t>(ws_bytes)}, x.options().dtype(at::kByte));
  check_status(cf_lora_linear_int8(x.data_ptr(), w_codes.data_ptr<int8_t>(),
                                   w_scales.data_ptr<float>(), ap.data_ptr(), alp, bp.data_ptr(),
                                   blp, y.data_ptr(), m, k, n, rp, static_cast<float>(scale), dtype,
                                   ws.data_ptr(), ws_bytes, current_stream()),
               "lora_linear_int8");
  return y;
}

// Reference shapes (cpp/src/bindings.cpp:65-80, 129-151): 2-D rows x cols,
// weight [cols]. Any float dtype here (the reference kernels are fp32 only).
// The kernels read the weight in x's dtype or in float32; a weight of another
// float dtype is widened to float32 first, which is exactly the reference
// composition's weight.float(). Outputs: normalised (and the rounded sum).
void check_norm_args(const at::Tensor &x, const at::Tensor &weight, const char *xname) {
  check_cuda(x, xname);
  check_cuda(weight, "weight");
  TORCH_CHECK(x.dim() == 2, xname, " must be 2-D, got ", x.dim(), " dimensions");
  check_contiguous(x, xname);
  check_contiguous(weight, "weight");
  TORCH_CHECK(weight.dim() == 1 && weight.size(0) == x.size(1), "weight must be 1-D of length ",
              x.size(1), ", got ", weight.sizes());
  dtype_code(weight, "weight");
  TORCH_CHECK(weight.device() == x.device(), "weight must be on ", xname, "'s device");
}

at::Tensor kernel_weight(const at::Tensor &weight, const at::Tensor &x) {
  if (weight.scalar_type() == x.scalar_type() || weight.scalar_type() == at::kFloat) return weight;
  return weight.to(at::kFloat);
}

at::Tensor rmsnorm_cuda(const at::Tensor &input, const at::Tensor &weight, double eps) {
  check_norm_args(input, weight, "input");
  const int dtype = dtype_code(input, "input");
  const c10::cuda::CUDAGuard guard(input.device());
  const at::Tensor w = kernel_weight(weight, input);
  at::Tensor out = at::empty_like(input);
  check_status(cf_fused_residual_rmsnorm(input.data_ptr(), nullptr, w.data_ptr(),
                                         dtype_code(w, "weight"), out.data_ptr(), nullptr,
                                         input.size(0), input.size(1), static_cast<float>(eps),
                                         dtype, current_stream()),
               "rmsnorm");
  return out;
}

std::vector<at::Tensor> fused_residual_rmsnorm_cuda(const at::Tensor &x, const at::Tensor &residual,
                                                    const at::Tensor &weight, double eps) {
  check_norm_args(x, weight, "x");
  check_cuda(residual, "residual");
  check_contiguous(residual, "residual");
  TORCH_CHECK(x.sizes() == residual.sizes(), "x and residual must have the same shape, got ",
              x.sizes(), " and ", residual.sizes());
  TORCH_CHECK(residual.scalar_type() == x.scalar_type(), "x and residual must share one dtype");
  TORCH_CHECK(residual.device() == x.device(), "residual must be on x's device");
  const int dtype = dtype_code(x, "x");
  const c10::cuda::CUDAGuard guard(x.device());
  const at::Tensor w = kernel_weight(weight, x);
  at::Tensor out = at::empty_like(x);
  at::Tensor summed = at::empty_like(x);
  check_status(cf_fused_residual_rmsnorm(x.data_ptr(), residual.data_ptr(), w.data_ptr(),
                                         dtype_code(w, "weight"), out.data_ptr(),
                                         summed.data_ptr(), x.size(0), x.size(1),
                                         static_cast<float>(eps), dtype, current_stream()),
               "fused_residual_rmsnorm");
  return {out, summed};
}

// ---- host tensors: the reference semantics (python/cudaforge/ops.py:164-240)

std::vector<at::Tensor> quantize_int8_host(const at::Tensor &input) {
  at::Tensor flat = input.reshape({-1}).to(at::kFloat);
  const int64_t count = flat.numel();
  const int64_t pad = cf_quant_scale_count(count) * CF_QUANT_BLOCK_SIZE - count;
  if (pad > 0) flat = at::constant_pad_nd(flat, {0, pad});
  const at::Tensor blocks = flat.view({-1, CF_QUANT_BLOCK_SIZE});
  at::Tensor scales = blocks.abs().amax(1) / 127.0;
  scales = at::where(scales > 0, scales, at::ones_like(scales));
  const at::Tensor codes = at::clamp(at::round(blocks / scales.unsqueeze(1)), -127, 127);
  return {codes.reshape({-1}).narrow(0, 0, count).to(at::kChar).view(input.sizes()), scales};
}

at::Tensor dequantize_int8_host(const at::Tensor &quantised, const at::Tensor &scales) {
  const int64_t count = quantised.numel();
  TORCH_CHECK(scales.numel() == cf_quant_scale_count(count), "expected ",
              cf_quant_scale_count(count), " block scales, got ", scales.numel());
  const int64_t pad = scales.numel() * CF_QUANT_BLOCK_SIZE - count;
  at::Tensor flat = quantised.reshape({-1}).to(at::kFloat);
  if (pad > 0) flat = at::constant_pad_nd(flat, {0, pad});
  const at::Tensor values = flat.view({-1, CF_QUANT_BLOCK_SIZE}) * scales.to(at::kFloat).unsqueeze(1);
  return values.reshape({-1}).narrow(0, 0, count).view(quantised.sizes());
}

at::Tensor lora_linear_host(const at::Tensor &x, const at::Tensor &w, const at::Tensor &a,
                            const at::Tensor &b, double scale) {
  return at::matmul(x, w) + scale * at::matmul(at::matmul(x, a), b);
}

at::Tensor rmsnorm_host(const at::Tensor &input, const at::Tensor &weight, double eps) {
  TORCH_CHECK(input.dim() == 2, "input must be 2-D, got ", input.dim(), " dimensions");
  TORCH_CHECK(weight.size(0) == input.size(1), "weight length ", weight.size(0),
              " does not match the input's last dimension ", input.size(1));
  const at::Tensor f = input.to(at::kFloat);
  const at::Tensor norm = f * at::rsqrt(f.pow(2).mean({-1}, /*keepdim=*/true) + eps);
  return (norm * weight.to(at::kFloat)).to(input.scalar_type());
}

std::vector<at::Tensor> fused_residual_rmsnorm_host(const at::Tensor &x,
                                                    const at::Tensor &residual,
                                                    const at::Tensor &weight, double eps) {
  TORCH_CHECK(x.sizes() == residual.sizes(), "x and residual must have the same shape, got ",
              x.sizes(), " and ", residual.sizes());
  const at::Tensor summed = x + residual;
  return {rmsnorm_host(summed, weight, eps), summed};
}

// ---- the reference's other operators (not on the accelerated path)
//
// softmax, sum, silu, gelu and swiglu keep their schemas registered so the
// reference package behaves the same with this extension installed
// (python/cudaforge/ops.py probes each op by name and calls it for host and
// device tensors alike). They are ATen compositions of the reference semantics
// (cpp/src/bindings.cpp:250-295) on whichever device the tensors live.

at::Tensor softmax_any(const at::Tensor &input) {
  TORCH_CHECK(input.dim() == 2, "input must be 2-D, got ", input.dim(), " dimensions");
  return at::softmax(input, -1);
}

at::Tensor sum_any(const at::Tensor &input) { return input.sum(); }

at::Tensor silu_any(const at::Tensor &input) { return at::silu(input); }

at::Tensor gelu_any(const at::Tensor &input) { return at::gelu(input, "tanh"); }

at::Tensor swiglu_any(const at::Tensor &gate, const at::Tensor &up) {
  TORCH_CHECK(gate.sizes() == up.sizes(), "gate and up must have the same shape, got ",
              gate.sizes(), " and ", up.sizes());
  const auto t = gate.scalar_type();
  if (t != at::kHalf && t != at::kBFloat16) return at::silu(gate) * up;
  // 16-bit inputs are computed in fp32 and rounded once.
  return (at::silu(gate.to(at::kFloat)) * up.to(at::kFloat)).to(t);
}

}  // namespace

TORCH_LIBRARY(cudaforge, m) {
  // Byte-identical to the reference (cpp/src/bindings.cpp:345, 353-354).
  m.def("lora_linear(Tensor x, Tensor w, Tensor a, Tensor b, float scale) -> Tensor");
  m.def("quantize_int8(Tensor input) -> Tensor[]");
  m.def("dequantize_int8(Tensor quantised, Tensor scales) -> Tensor");
  // Byte-identical to the reference (cpp/src/bindings.cpp:343, 350-352).
  m.def("rmsnorm(Tensor input, Tensor weight, float eps) -> Tensor");
  m.def(
      "fused_residual_rmsnorm(Tensor x, Tensor residual, Tensor weight, float eps) "
      "-> Tensor[]");
  // The reference's remaining schemas (cpp/src/bindings.cpp:344, 346-349), byte-identical.
  m.def("softmax(Tensor input) -> Tensor");
  m.def("sum(Tensor input) -> Tensor");
  m.def("silu(Tensor input) -> Tensor");
  m.def("gelu(Tensor input) -> Tensor");
  m.def("swiglu(Tensor gate, Tensor up) -> Tensor");
  // Additive.
  m.def(
      "lora_linear_int8(Tensor x, Tensor w_codes, Tensor w_scales, Tensor a, Tensor b, "
      "float scale) -> Tensor");
  m.def("quantize_dequantize(Tensor input) -> Tensor");
  m.def("quantize_int8_many(Tensor[] inputs) -> Tensor[]");
}

TORCH_LIBRARY_IMPL(cudaforge, Autograd, m) {
  for (const char *name : {"lora_linear", "quantize_int8", "dequantize_int8", "lora_linear_int8",
                           "quantize_dequantize", "quantize_int8_many", "rmsnorm",
                           "fused_residual_rmsnorm", "softmax", "sum", "silu", "gelu",
                           "swiglu"}) {
    m.impl(name, torch::autograd::autogradNotImplementedFallback());
  }
}

TORCH_LIBRARY_IMPL(cudaforge, CUDA, m) {
  m.impl("lora_linear", &lora_linear_cuda);
  m.impl("quantize_int8", &quantize_int8_cuda);
  m.impl("dequantize_int8", &dequantize_int8_cuda);
  m.impl("lora_linear_int8", &lora_linear_int8_cuda);
  m.impl("quantize_dequantize", &quantize_dequantize_cuda);
  m.impl("quantize_int8_many", &quantize_int8_many_cuda);
  m.impl("rmsnorm", &rmsnorm_cuda);
  m.impl("fused_residual_rmsnorm", &fused_residual_rmsnorm_cuda);
}

TORCH_LIBRARY_IMPL(cudaforge, CompositeExplicitAutograd, m) {
  m.impl("softmax", &softmax_any);
  m.impl("sum", &sum_any);
  m.impl("silu", &silu_any);
  m.impl("gelu", &gelu_any);
  m.impl("swiglu", &swiglu_any);
}

TORCH_LIBRARY_IMPL(cudaforge, CPU, m) {
  m.impl("quantize_int8", &quantize_int8_host);
  m.impl("dequantize_int8", &dequantize_int8_host);
  m.impl("lora_linear", &lora_linear_host);
  m.impl("rmsnorm", &rmsnorm_host);
  m.impl("fused_residual_rmsnorm", &fused_residual_rmsnorm_host);
}

// `from cudaforge import _C` (python/cudaforge/ops.py:44-58) imports this file
// as a Python extension module; loading it runs the registrations above.
// cuda_kernels_available() answers as the reference's does (bindings.cpp:
// 331-337): this build always has its CUDA kernels.
namespace {

PyObject *cuda_kernels_available(PyObject *, PyObject *) { Py_RETURN_TRUE; }

PyMethodDef kModuleMethods[] = {
    {"cuda_kernels_available", cuda_kernels_available, METH_NOARGS,
     "True: the operators have sm_100a CUDA kernels."},
    {nullptr, nullptr, 0, nullptr}};

PyModuleDef kModuleDef = {PyModuleDef_HEAD_INIT, "_C",
                          "cudaforge operators on sm_100a kernels (C-ABI shim)", -1,
                          kModuleMethods};

}  // namespace

PyMODINIT_FUNC PyInit__C(void) { return PyModule_Create(&kModuleDef); }
