// crumpet_b200: torch dispatcher registration of the crumpet_ops namespace.
//
// Same op names, schemas and tags as the reference registration
// (torch-ext/torch_binding.cpp:9-39), CUDA implementations only, plus
// fused_swin_attention, which the reference exposes only as a Python/Triton
// function (torch-ext/crumpet/fused_attention.py:149-226).  Every impl checks
// the tensors, takes the current stream and calls the C ABI in
// libcrumpet_b200.so; ops never allocate (outputs are preallocated `Tensor!`).
#include <ATen/ATen.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/library.h>

#include "crumpet_b200.h"

namespace {

const std::vector<at::Tag> kTags = {at::Tag::pt2_compliant_tag,
                                    at::Tag::needs_fixed_stride_order};

int dtype_code(const at::Tensor& t) {
  switch (t.scalar_type()) {
    case at::kFloat:
      return CRUMPET_DTYPE_F32;
    case at::kHalf:
      return CRUMPET_DTYPE_F16;
    case at::kBFloat16:
      return CRUMPET_DTYPE_BF16;
    default:
      TORCH_CHECK_TYPE(false, "CRUMPET supports torch.float32, torch.float16 and torch.bfloat16");
  }
  return -1;
}

void check_rc(int rc) { TORCH_CHECK(rc == CRUMPET_OK, "crumpet_b200: ", crumpet_last_error()); }

void* cur_stream(const at::Tensor& t) {
  return static_cast<void*>(at::cuda::getCurrentCUDAStream(t.device().index()).stream());
}

void check_cuda_contig(const at::Tensor& t, const char* name) {
  TORCH_CHECK(t.is_cuda(), name, " must be a CUDA tensor");
  TORCH_CHECK(t.is_contiguous(), name, " must be contiguous");
}

// Every operand of a launch must live on the device the launch is guarded to: a
// pointer into another GPU's memory would be dereferenced by the kernel as if local.
void same_device(const at::Tensor& ref, const at::Tensor& t, const char* name) {
  TORCH_CHECK(t.device() == ref.device(), name, " must be on ", ref.device(), " (got ",
              t.device(), ")");
}

int64_t num_windows(int64_t D, int64_t H, int64_t W, int64_t wd, int64_t wh, int64_t ww) {
  TORCH_CHECK(wd > 0 && wh > 0 && ww > 0, "window_size values must be positive");
  return (D / wd) * (H / wh) * (W / ww);
}

void compute_attn_mask_3d(at::Tensor& output, int64_t D, int64_t H, int64_t W, int64_t ws_d,
                          int64_t ws_h, int64_t ws_w, int64_t ss_d, int64_t ss_h, int64_t ss_w) {
  check_cuda_contig(output, "output");
  const c10::cuda::CUDAGuard guard(output.device());
  if (output.numel() == 0) return;
  const int64_t vol = ws_d * ws_h * ws_w;
  const int64_t nw = num_windows(D, H, W, ws_d, ws_h, ws_w);
  TORCH_CHECK(output.dim() == 3 && output.size(0) == nw && output.size(1) == vol &&
                  output.size(2) == vol,
              "output must have shape [num_windows, volume, volume]");
  check_rc(crumpet_compute_attn_mask_3d(output.data_ptr(), dtype_code(output), D, H, W, ws_d, ws_h,
                                        ws_w, ss_d, ss_h, ss_w, cur_stream(output)));
}

void fused_shift_partition_3d(at::Tensor& output, const at::Tensor& x, int64_t ws_d, int64_t ws_h,
                              int64_t ws_w, int64_t ss_d, int64_t ss_h, int64_t ss_w) {
  check_cuda_contig(x, "x");
  check_cuda_contig(output, "output");
  TORCH_CHECK(x.dim() == 5, "x must have shape [B, D, H, W, C]");
  TORCH_CHECK(output.scalar_type() == x.scalar_type(), "output and x dtypes differ");
  same_device(x, output, "output");
  const c10::cuda::CUDAGuard guard(x.device());
  if (output.numel() == 0) return;
  const int64_t B = x.size(0), D = x.size(1), H = x.size(2), W = x.size(3), C = x.size(4);
  const int64_t nw = num_windows(D, H, W, ws_d, ws_h, ws_w);
  TORCH_CHECK(output.dim() == 3 && output.size(0) == B * nw &&
                  output.size(1) == ws_d * ws_h * ws_w && output.size(2) == C,
              "output must have shape [B * num_windows, volume, C]");
  check_rc(crumpet_fused_shift_partition_3d(output.data_ptr(), x.data_ptr(), dtype_code(x), B, D,
                                            H, W, C, ws_d, ws_h, ws_w, ss_d, ss_h, ss_w,
                                            cur_stream(x)));
}

void fused_unshift_unpartition_3d(at::Tensor& output, const at::Tensor& windows, int64_t B,
                                  int64_t D, int64_t H, int64_t W, int64_t C, int64_t ws_d,
                                  int64_t ws_h, int64_t ws_w, int64_t ss_d, int64_t ss_h,
                                  int64_t ss_w) {
  check_cuda_contig(windows, "windows");
  check_cuda_contig(output, "output");
  TORCH_CHECK(output.scalar_type() == windows.scalar_type(), "output and windows dtypes differ");
  same_device(windows, output, "output");
  const c10::cuda::CUDAGuard guard(windows.device());
  if (output.numel() == 0) return;
  const int64_t nw = num_windows(D, H, W, ws_d, ws_h, ws_w);
  TORCH_CHECK(windows.dim() == 3 && windows.size(0) == B * nw &&
                  windows.size(1) == ws_d * ws_h * ws_w && windows.size(2) == C,
              "windows must have shape [B * num_windows, volume, C]");
  TORCH_CHECK(output.numel() == B * D * H * W * C, "output must have B*D*H*W*C elements");
  check_rc(crumpet_fused_unshift_unpartition_3d(output.data_ptr(), windows.data_ptr(),
                                                dtype_code(windows), B, D, H, W, C, ws_d, ws_h,
                                                ws_w, ss_d, ss_h, ss_w, cur_stream(windows)));
}

// Gradient of the partition is the unpartition (reference:
// cuda/unshift_unpartition_3d.cu:320-348).
void fused_shift_partition_3d_backward(at::Tensor& grad_x, const at::Tensor& grad_windows,
                                       int64_t B, int64_t D, int64_t H, int64_t W, int64_t C,
                                       int64_t ws_d, int64_t ws_h, int64_t ws_w, int64_t ss_d,
                                       int64_t ss_h, int64_t ss_w) {
  fused_unshift_unpartition_3d(grad_x, grad_windows, B, D, H, W, C, ws_d, ws_h, ws_w, ss_d, ss_h,
                               ss_w);
}

// Gradient of the unpartition is the partition (reference:
// cuda/shift_partition_3d.cu:349-367).
void fused_unshift_unpartition_3d_backward(at::Tensor& grad_windows, const at::Tensor& grad_x,
                                           int64_t ws_d, int64_t ws_h, int64_t ws_w, int64_t ss_d,
                                           int64_t ss_h, int64_t ss_w) {
  fused_shift_partition_3d(grad_windows, grad_x, ws_d, ws_h, ws_w, ss_d, ss_h, ss_w);
}

void fused_swin_attention(at::Tensor& out, const at::Tensor& q, const at::Tensor& k,
                          const at::Tensor& v, const at::Tensor& rel_bias,
                          const c10::optional<at::Tensor>& mask,
                          const c10::optional<at::Tensor>& boundary, double scale) {
  check_cuda_contig(out, "out");
  check_cuda_contig(q, "q");
  check_cuda_contig(k, "k");
  check_cuda_contig(v, "v");
  check_cuda_contig(rel_bias, "relative_position_bias");
  TORCH_CHECK(q.dim() == 4 && q.sizes() == k.sizes() && q.sizes() == v.sizes() &&
                  q.sizes() == out.sizes(),
              "q, k, v and out must share the shape [B, H, N, head_dim]");
  const int64_t B = q.size(0), H = q.size(1), N = q.size(2), Dh = q.size(3);
  TORCH_CHECK(rel_bias.dim() == 3 && rel_bias.size(0) == H && rel_bias.size(1) == N &&
                  rel_bias.size(2) == N,
              "relative_position_bias must have shape [H, N, N]");
  const auto st = q.scalar_type();
  TORCH_CHECK(k.scalar_type() == st && v.scalar_type() == st && out.scalar_type() == st &&
                  rel_bias.scalar_type() == st,
              "q, k, v, out and relative_position_bias must share one dtype");
  same_device(q, k, "k");
  same_device(q, v, "v");
  same_device(q, out, "out");
  same_device(q, rel_bias, "relative_position_bias");
  const c10::cuda::CUDAGuard guard(q.device());
  const void* mask_ptr = nullptr;
  int64_t mask_windows = 0;
  if (mask.has_value() && mask->defined()) {
    check_cuda_contig(*mask, "mask");
    same_device(q, *mask, "mask");
    TORCH_CHECK(mask->dim() == 3 && mask->size(1) == N && mask->size(2) == N,
                "mask must have shape [num_windows, N, N]");
    TORCH_CHECK(mask->scalar_type() == st, "mask must have the dtype of q");
    mask_windows = mask->size(0);
    TORCH_CHECK(mask_windows >= 1 && B % mask_windows == 0,
                "mask windows must divide the batch of windows");
    mask_ptr = mask->data_ptr();
  }
  const uint8_t* bnd = nullptr;
  if (boundary.has_value() && boundary->defined()) {
    check_cuda_contig(*boundary, "boundary");
    same_device(q, *boundary, "boundary");
    TORCH_CHECK(boundary->scalar_type() == at::kByte && boundary->numel() == B,
                "boundary must be a uint8 tensor of B elements");
    bnd = boundary->data_ptr<uint8_t>();
  }
  check_rc(crumpet_fused_swin_attention(out.data_ptr(), q.data_ptr(), k.data_ptr(), v.data_ptr(),
                                        rel_bias.data_ptr(), mask_ptr, mask_windows, bnd,
                                        dtype_code(q), B, H, N, Dh, static_cast<float>(scale),
                                        cur_stream(q)));
}

void swin_window_attention_qkv(at::Tensor& out, const at::Tensor& qkv, const at::Tensor& table,
                               const at::Tensor& index, at::IntArrayRef num_windows,
                               at::IntArrayRef window_size, at::IntArrayRef shift_size,
                               double scale) {
  check_cuda_contig(out, "out");
  check_cuda_contig(qkv, "qkv");
  check_cuda_contig(table, "relative_position_bias_table");
  check_cuda_contig(index, "relative_position_index");
  TORCH_CHECK(qkv.dim() == 5 && qkv.size(2) == 3, "qkv must have shape [B, N, 3, H, head_dim]");
  const int64_t B = qkv.size(0), N = qkv.size(1), H = qkv.size(3), Dh = qkv.size(4);
  TORCH_CHECK(out.dim() == 3 && out.size(0) == B && out.size(1) == N && out.size(2) == H * Dh,
              "out must have shape [B, N, H * head_dim]");
  TORCH_CHECK(out.scalar_type() == qkv.scalar_type(), "out and qkv dtypes differ");
  TORCH_CHECK(table.dim() == 2 && table.size(1) == H, "relative_position_bias_table must be [T, H]");
  TORCH_CHECK(table.scalar_type() == at::kFloat || table.scalar_type() == qkv.scalar_type(),
              "relative_position_bias_table must be float32 or the dtype of qkv");
  TORCH_CHECK(index.scalar_type() == at::kLong && index.dim() == 2 && index.size(0) >= N &&
                  index.size(1) >= N,
              "relative_position_index must be int64 [>=N, >=N]");
  TORCH_CHECK(num_windows.size() == 3 && window_size.size() == 3 && shift_size.size() == 3,
              "num_windows, window_size and shift_size take three values");
  same_device(qkv, out, "out");
  same_device(qkv, table, "relative_position_bias_table");
  same_device(qkv, index, "relative_position_index");
  const c10::cuda::CUDAGuard guard(qkv.device());
  check_rc(crumpet_swin_window_attention_qkv(
      out.data_ptr(), qkv.data_ptr(), table.data_ptr(), table.scalar_type() == at::kFloat ? 1 : 0,
      table.size(0), index.data_ptr<int64_t>(), index.size(1), num_windows[0], num_windows[1], num_windows[2],
      window_size[0], window_size[1], window_size[2], shift_size[0], shift_size[1],
      shift_size[2], dtype_code(qkv), B, H, N, Dh, static_cast<float>(scale), cur_stream(qkv)));
}

void attention_bias_tiles(at::Tensor& tiles, const at::Tensor& table, const at::Tensor& index,
                          int64_t N, double scale, at::ScalarType dtype) {
  check_cuda_contig(tiles, "tiles");
  check_cuda_contig(table, "relative_position_bias_table");
  check_cuda_contig(index, "relative_position_index");
  same_device(tiles, table, "relative_position_bias_table");
  same_device(tiles, index, "relative_position_index");
  TORCH_CHECK(tiles.scalar_type() == at::kByte, "tiles must be a uint8 tensor");
  TORCH_CHECK(table.dim() == 2, "relative_position_bias_table must be [T, H]");
  TORCH_CHECK(dtype == at::kHalf || dtype == at::kBFloat16, "bias tiles are float16 or bfloat16");
  TORCH_CHECK(table.scalar_type() == at::kFloat || table.scalar_type() == dtype,
              "relative_position_bias_table must be float32 or the tiles' dtype");
  TORCH_CHECK(index.scalar_type() == at::kLong && index.dim() == 2 && index.size(0) >= N &&
                  index.size(1) >= N,
              "relative_position_index must be int64 [>=N, >=N]");
  const int64_t H = table.size(1);
  TORCH_CHECK(tiles.numel() == crumpet_attention_bias_tiles_bytes(H, N),
              "tiles must hold crumpet_attention_bias_tiles_bytes(H, N) bytes");
  const c10::cuda::CUDAGuard guard(tiles.device());
  const int code = dtype == at::kHalf ? CRUMPET_DTYPE_F16 : CRUMPET_DTYPE_BF16;
  check_rc(crumpet_attention_bias_tiles(tiles.data_ptr(), table.data_ptr(),
                                        table.scalar_type() == at::kFloat ? 1 : 0, table.size(0),
                                        index.data_ptr<int64_t>(), index.size(1), code, H, N,
                                        static_cast<float>(scale), cur_stream(tiles)));
}

// fused_swin_attention with the shifted-window mask of a window grid computed on chip
// (crumpet_fused_swin_attention_shifted) in place of a dense mask tensor.
void fused_swin_attention_shifted(at::Tensor& out, const at::Tensor& q, const at::Tensor& k,
                                  const at::Tensor& v, const at::Tensor& rel_bias,
                                  const c10::optional<at::Tensor>& boundary,
                                  at::IntArrayRef num_windows, at::IntArrayRef window_size,
                                  at::IntArrayRef shift_size, double scale) {
  check_cuda_contig(out, "out");
  check_cuda_contig(q, "q");
  check_cuda_contig(k, "k");
  check_cuda_contig(v, "v");
  check_cuda_contig(rel_bias, "relative_position_bias");
  TORCH_CHECK(q.dim() == 4 && q.sizes() == k.sizes() && q.sizes() == v.sizes() &&
                  q.sizes() == out.sizes(),
              "q, k, v and out must share the shape [B, H, N, head_dim]");
  const int64_t B = q.size(0), H = q.size(1), N = q.size(2), Dh = q.size(3);
  TORCH_CHECK(rel_bias.dim() == 3 && rel_bias.size(0) == H && rel_bias.size(1) == N &&
                  rel_bias.size(2) == N,
              "relative_position_bias must have shape [H, N, N]");
  const auto st = q.scalar_type();
  TORCH_CHECK(k.scalar_type() == st && v.scalar_type() == st && out.scalar_type() == st &&
                  rel_bias.scalar_type() == st,
              "q, k, v, out and relative_position_bias must share one dtype");
  TORCH_CHECK(num_windows.size() == 3 && window_size.size() == 3 && shift_size.size() == 3,
              "num_windows, window_size and shift_size take three values");
  same_device(q, k, "k");
  same_device(q, v, "v");
  same_device(q, out, "out");
  same_device(q, rel_bias, "relative_position_bias");
  const c10::cuda::CUDAGuard guard(q.device());
  const uint8_t* bnd = nullptr;
  if (boundary.has_value() && boundary->defined()) {
    check_cuda_contig(*boundary, "boundary");
    same_device(q, *boundary, "boundary");
    TORCH_CHECK(boundary->scalar_type() == at::kByte && boundary->numel() == B,
                "boundary must be a uint8 tensor of B elements");
    bnd = boundary->data_ptr<uint8_t>();
  }
  check_rc(crumpet_fused_swin_attention_shifted(
      out.data_ptr(), q.data_ptr(), k.data_ptr(), v.data_ptr(), rel_bias.data_ptr(), bnd,
      dtype_code(q), B, H, N, Dh, num_windows[0], num_windows[1], num_windows[2],
      window_size[0], window_size[1], window_size[2], shift_size[0], shift_size[1],
      shift_size[2], static_cast<float>(scale), cur_stream(q)));
}

void swin_window_attention_qkv_tiles(at::Tensor& out, const at::Tensor& qkv,
                                     const at::Tensor& tiles, at::IntArrayRef num_windows,
                                     at::IntArrayRef window_size, at::IntArrayRef shift_size,
                                     double scale) {
  check_cuda_contig(out, "out");
  check_cuda_contig(qkv, "qkv");
  check_cuda_contig(tiles, "bias_tiles");
  TORCH_CHECK(qkv.dim() == 5 && qkv.size(2) == 3, "qkv must have shape [B, N, 3, H, head_dim]");
  const int64_t B = qkv.size(0), N = qkv.size(1), H = qkv.size(3), Dh = qkv.size(4);
  TORCH_CHECK(out.dim() == 3 && out.size(0) == B && out.size(1) == N && out.size(2) == H * Dh,
              "out must have shape [B, N, H * head_dim]");
  TORCH_CHECK(out.scalar_type() == qkv.scalar_type(), "out and qkv dtypes differ");
  TORCH_CHECK(tiles.scalar_type() == at::kByte &&
                  tiles.numel() == crumpet_attention_bias_tiles_bytes(H, N),
              "bias_tiles must be the uint8 tiles built for these H and N");
  TORCH_CHECK(num_windows.size() == 3 && window_size.size() == 3 && shift_size.size() == 3,
              "num_windows, window_size and shift_size take three values");
  same_device(qkv, out, "out");
  same_device(qkv, tiles, "bias_tiles");
  const c10::cuda::CUDAGuard guard(qkv.device());
  check_rc(crumpet_swin_window_attention_qkv_tiles(
      out.data_ptr(), qkv.data_ptr(), tiles.data_ptr(), num_windows[0], num_windows[1],
      num_windows[2], window_size[0], window_size[1], window_size[2], shift_size[0],
      shift_size[1], shift_size[2], dtype_code(qkv), B, H, N, Dh, static_cast<float>(scale),
      cur_stream(qkv)));
}

int64_t ceil_to(int64_t v, int64_t m) { return (v + m - 1) / m * m; }

void norm_shift_partition_3d(at::Tensor& output, const at::Tensor& x, const at::Tensor& weight,
                             const at::Tensor& bias, double eps, int64_t ws_d, int64_t ws_h,
                             int64_t ws_w, int64_t ss_d, int64_t ss_h, int64_t ss_w) {
  check_cuda_contig(x, "x");
  check_cuda_contig(output, "output");
  check_cuda_contig(weight, "weight");
  check_cuda_contig(bias, "bias");
  TORCH_CHECK(x.dim() == 5, "x must have shape [B, D, H, W, C]");
  const int64_t B = x.size(0), D = x.size(1), H = x.size(2), W = x.size(3), C = x.size(4);
  TORCH_CHECK(weight.scalar_type() == at::kFloat && bias.scalar_type() == at::kFloat &&
                  weight.numel() == C && bias.numel() == C,
              "weight and bias must be float32 tensors of C elements");
  same_device(x, output, "output");
  same_device(x, weight, "weight");
  same_device(x, bias, "bias");
  const c10::cuda::CUDAGuard guard(x.device());
  const int64_t nw = num_windows(ceil_to(D, ws_d), ceil_to(H, ws_h), ceil_to(W, ws_w), ws_d, ws_h,
                                 ws_w);
  TORCH_CHECK(output.dim() == 3 && output.size(0) == B * nw &&
                  output.size(1) == ws_d * ws_h * ws_w && output.size(2) == C,
              "output must have shape [B * num_windows(padded), volume, C]");
  if (output.numel() == 0) return;
  check_rc(crumpet_norm_shift_partition_3d(
      output.data_ptr(), dtype_code(output), x.data_ptr(), dtype_code(x), weight.data_ptr<float>(),
      bias.data_ptr<float>(), static_cast<float>(eps), B, D, H, W, C, ws_d, ws_h, ws_w, ss_d, ss_h,
      ss_w, cur_stream(x)));
}

void unshift_unpartition_crop_3d(at::Tensor& output, const at::Tensor& windows,
                                 const c10::optional<at::Tensor>& residual, int64_t B, int64_t D,
                                 int64_t H, int64_t W, int64_t C, int64_t ws_d, int64_t ws_h,
                                 int64_t ws_w, int64_t ss_d, int64_t ss_h, int64_t ss_w) {
  check_cuda_contig(windows, "windows");
  check_cuda_contig(output, "output");
  TORCH_CHECK(output.scalar_type() == windows.scalar_type(), "output and windows dtypes differ");
  same_device(windows, output, "output");
  const c10::cuda::CUDAGuard guard(windows.device());
  const int64_t nw = num_windows(ceil_to(D, ws_d), ceil_to(H, ws_h), ceil_to(W, ws_w), ws_d, ws_h,
                                 ws_w);
  TORCH_CHECK(windows.dim() == 3 && windows.size(0) == B * nw &&
                  windows.size(1) == ws_d * ws_h * ws_w && windows.size(2) == C,
              "windows must have shape [B * num_windows(padded), volume, C]");
  TORCH_CHECK(output.numel() == B * D * H * W * C, "output must have B*D*H*W*C elements");
  const void* res = nullptr;
  if (residual.has_value() && residual->defined()) {
    check_cuda_contig(*residual, "residual");
    same_device(windows, *residual, "residual");
    TORCH_CHECK(residual->scalar_type() == windows.scalar_type(),
                "residual must have the dtype of windows");
    TORCH_CHECK(residual->numel() == B * D * H * W * C, "residual must have B*D*H*W*C elements");
    res = residual->data_ptr();
  }
  if (output.numel() == 0) return;
  check_rc(crumpet_unshift_unpartition_crop_3d(output.data_ptr(), windows.data_ptr(), res,
                                               dtype_code(windows), B, D, H, W, C, ws_d, ws_h,
                                               ws_w, ss_d, ss_h, ss_w, cur_stream(windows)));
}

void unshift_unpartition_crop_norm_3d(at::Tensor& output, at::Tensor& normed,
                                      const at::Tensor& windows,
                                      const c10::optional<at::Tensor>& residual,
                                      const at::Tensor& weight, const at::Tensor& bias, double eps,
                                      int64_t B, int64_t D, int64_t H, int64_t W, int64_t C,
                                      int64_t ws_d, int64_t ws_h, int64_t ws_w, int64_t ss_d,
                                      int64_t ss_h, int64_t ss_w) {
  check_cuda_contig(windows, "windows");
  check_cuda_contig(output, "output");
  check_cuda_contig(normed, "normed");
  check_cuda_contig(weight, "weight");
  check_cuda_contig(bias, "bias");
  TORCH_CHECK(output.scalar_type() == windows.scalar_type(), "output and windows dtypes differ");
  TORCH_CHECK(weight.scalar_type() == at::kFloat && bias.scalar_type() == at::kFloat &&
                  weight.numel() == C && bias.numel() == C,
              "weight and bias must be float32 tensors of C elements");
  same_device(windows, output, "output");
  same_device(windows, normed, "normed");
  same_device(windows, weight, "weight");
  same_device(windows, bias, "bias");
  const c10::cuda::CUDAGuard guard(windows.device());
  const int64_t nw = num_windows(ceil_to(D, ws_d), ceil_to(H, ws_h), ceil_to(W, ws_w), ws_d, ws_h,
                                 ws_w);
  TORCH_CHECK(windows.dim() == 3 && windows.size(0) == B * nw &&
                  windows.size(1) == ws_d * ws_h * ws_w && windows.size(2) == C,
              "windows must have shape [B * num_windows(padded), volume, C]");
  TORCH_CHECK(output.numel() == B * D * H * W * C && normed.numel() == B * D * H * W * C,
              "output and normed must have B*D*H*W*C elements");
  const void* res = nullptr;
  if (residual.has_value() && residual->defined()) {
    check_cuda_contig(*residual, "residual");
    same_device(windows, *residual, "residual");
    TORCH_CHECK(residual->scalar_type() == windows.scalar_type(),
                "residual must have the dtype of windows");
    TORCH_CHECK(residual->numel() == B * D * H * W * C, "residual must have B*D*H*W*C elements");
    res = residual->data_ptr();
  }
  if (output.numel() == 0) return;
  check_rc(crumpet_unshift_unpartition_crop_norm_3d(
      output.data_ptr(), normed.data_ptr(), dtype_code(normed), windows.data_ptr(), res,
      dtype_code(windows), weight.data_ptr<float>(), bias.data_ptr<float>(), static_cast<float>(eps),
      B, D, H, W, C, ws_d, ws_h, ws_w, ss_d, ss_h, ss_w, cur_stream(windows)));
}

void patch_merge_norm_3d(at::Tensor& output, const at::Tensor& x, const at::Tensor& weight,
                         const at::Tensor& bias, double eps, at::IntArrayRef parts) {
  check_cuda_contig(x, "x");
  check_cuda_contig(output, "output");
  check_cuda_contig(weight, "weight");
  check_cuda_contig(bias, "bias");
  TORCH_CHECK(x.dim() == 5, "x must have shape [B, D, H, W, C]");
  TORCH_CHECK(parts.size() == 8, "parts takes eight neighbour codes");
  const int64_t B = x.size(0), D = x.size(1), H = x.size(2), W = x.size(3), C = x.size(4);
  TORCH_CHECK(weight.scalar_type() == at::kFloat && bias.scalar_type() == at::kFloat &&
                  weight.numel() == 8 * C && bias.numel() == 8 * C,
              "weight and bias must be float32 tensors of 8C elements");
  TORCH_CHECK(output.dim() == 5 && output.size(0) == B && output.size(1) == (D + 1) / 2 &&
                  output.size(2) == (H + 1) / 2 && output.size(3) == (W + 1) / 2 &&
                  output.size(4) == 8 * C,
              "output must have shape [B, ceil(D/2), ceil(H/2), ceil(W/2), 8C]");
  same_device(x, output, "output");
  same_device(x, weight, "weight");
  same_device(x, bias, "bias");
  const c10::cuda::CUDAGuard guard(x.device());
  if (output.numel() == 0) return;
  int codes[8];
  for (int p = 0; p < 8; ++p) codes[p] = static_cast<int>(parts[p]);
  check_rc(crumpet_patch_merge_norm_3d(output.data_ptr(), dtype_code(output), x.data_ptr(),
                                       dtype_code(x), weight.data_ptr<float>(),
                                       bias.data_ptr<float>(), static_cast<float>(eps), B, D, H, W,
                                       C, codes, cur_stream(x)));
}

void proj_out_norm_3d(at::Tensor& output, const at::Tensor& x,
                      const c10::optional<at::Tensor>& weight,
                      const c10::optional<at::Tensor>& bias, double eps) {
  check_cuda_contig(x, "x");
  check_cuda_contig(output, "output");
  TORCH_CHECK(x.dim() == 5, "x must have shape [B, C, D, H, W]");
  const int64_t B = x.size(0), C = x.size(1), D = x.size(2), H = x.size(3), W = x.size(4);
  TORCH_CHECK(weight.has_value() == bias.has_value(),
              "weight and bias must both be given or both be None");
  const float* w = nullptr;
  const float* b = nullptr;
  if (weight.has_value()) {
    check_cuda_contig(*weight, "weight");
    check_cuda_contig(*bias, "bias");
    same_device(x, *weight, "weight");
    same_device(x, *bias, "bias");
    TORCH_CHECK(weight->scalar_type() == at::kFloat && bias->scalar_type() == at::kFloat &&
                    weight->numel() == C && bias->numel() == C,
                "weight and bias must be float32 tensors of C elements");
    w = weight->data_ptr<float>();
    b = bias->data_ptr<float>();
  }
  TORCH_CHECK(output.dim() == 5 && output.size(0) == B && output.size(1) == D &&
                  output.size(2) == H && output.size(3) == W && output.size(4) == C,
              "output must have shape [B, D, H, W, C]");
  same_device(x, output, "output");
  const c10::cuda::CUDAGuard guard(x.device());
  if (output.numel() == 0) return;
  check_rc(crumpet_proj_out_norm_3d(output.data_ptr(), dtype_code(output), x.data_ptr(),
                                    dtype_code(x), w, b, static_cast<float>(eps), B, C, D, H, W,
                                    cur_stream(x)));
}

void window_linear(at::Tensor& out, const at::Tensor& x, const at::Tensor& weight,
                   const c10::optional<at::Tensor>& bias) {
  check_cuda_contig(x, "x");
  check_cuda_contig(out, "out");
  check_cuda_contig(weight, "weight");
  TORCH_CHECK(x.dim() == 2 && weight.dim() == 2, "x must be [M, K] and weight [N, K]");
  const int64_t M = x.size(0), K = x.size(1), N = weight.size(0);
  TORCH_CHECK(weight.size(1) == K, "weight must be [N, K]");
  TORCH_CHECK(weight.scalar_type() == x.scalar_type() && out.scalar_type() == x.scalar_type(),
              "x, weight and out must share one dtype");
  TORCH_CHECK(out.dim() == 2 && out.size(0) == M && out.size(1) == N, "out must be [M, N]");
  same_device(x, out, "out");
  same_device(x, weight, "weight");
  const float* b = nullptr;
  if (bias.has_value()) {
    check_cuda_contig(*bias, "bias");
    same_device(x, *bias, "bias");
    TORCH_CHECK(bias->scalar_type() == at::kFloat && bias->numel() == N,
                "bias must be a float32 tensor of N elements");
    b = bias->data_ptr<float>();
  }
  const c10::cuda::CUDAGuard guard(x.device());
  if (out.numel() == 0) return;
  check_rc(crumpet_window_linear(out.data_ptr(), x.data_ptr(), weight.data_ptr(), b,
                                 dtype_code(x), M, K, N, cur_stream(x)));
}

std::vector<int64_t> roi_list(at::IntArrayRef starts, at::IntArrayRef roi) {
  TORCH_CHECK(roi.size() == 3, "roi takes three values");
  TORCH_CHECK(starts.size() % 3 == 0, "starts must hold (z, y, x) triples");
  return std::vector<int64_t>(starts.begin(), starts.end());
}

void roi_gather(at::Tensor& out, const at::Tensor& volume, at::IntArrayRef starts,
                at::IntArrayRef roi) {
  check_cuda_contig(out, "out");
  check_cuda_contig(volume, "volume");
  TORCH_CHECK(volume.dim() == 4, "volume must have shape [C, D, H, W]");
  const auto s = roi_list(starts, roi);
  const int64_t n = int64_t(s.size() / 3);
  TORCH_CHECK(out.dim() == 5 && out.size(0) == n && out.size(1) == volume.size(0) &&
                  out.size(2) == roi[0] && out.size(3) == roi[1] && out.size(4) == roi[2],
              "out must have shape [n, C, rd, rh, rw]");
  same_device(volume, out, "out");
  const c10::cuda::CUDAGuard guard(volume.device());
  check_rc(crumpet_roi_gather(out.data_ptr(), dtype_code(out), volume.data_ptr(),
                              dtype_code(volume), volume.size(0), volume.size(1), volume.size(2),
                              volume.size(3), s.data(), n, roi[0], roi[1], roi[2],
                              cur_stream(volume)));
}

void roi_accumulate(at::Tensor& acc, const at::Tensor& pred, at::IntArrayRef starts,
                    at::IntArrayRef roi) {
  check_cuda_contig(acc, "acc");
  check_cuda_contig(pred, "pred");
  TORCH_CHECK(acc.scalar_type() == at::kFloat && acc.dim() == 4,
              "acc must be a float32 [classes, D, H, W] tensor");
  const auto s = roi_list(starts, roi);
  const int64_t n = int64_t(s.size() / 3);
  TORCH_CHECK(pred.dim() == 5 && pred.size(0) == n && pred.size(1) == acc.size(0) &&
                  pred.size(2) == roi[0] && pred.size(3) == roi[1] && pred.size(4) == roi[2],
              "pred must have shape [n, classes, rd, rh, rw]");
  same_device(acc, pred, "pred");
  const c10::cuda::CUDAGuard guard(acc.device());
  check_rc(crumpet_roi_accumulate(acc.data_ptr<float>(), pred.data_ptr(), dtype_code(pred),
                                  acc.size(0), acc.size(1), acc.size(2), acc.size(3), s.data(), n,
                                  roi[0], roi[1], roi[2], cur_stream(acc)));
}

void roi_argmax_impl(uint8_t* labels, float* logits, const at::Tensor& acc,
                     const at::Tensor& count_d, const at::Tensor& count_h,
                     const at::Tensor& count_w) {
  check_cuda_contig(acc, "acc");
  TORCH_CHECK(acc.scalar_type() == at::kFloat && acc.dim() == 4,
              "acc must be a float32 [classes, D, H, W] tensor");
  const at::Tensor* counts[3] = {&count_d, &count_h, &count_w};
  for (int a = 0; a < 3; ++a) {
    check_cuda_contig(*counts[a], "count");
    same_device(acc, *counts[a], "count");
    TORCH_CHECK(counts[a]->scalar_type() == at::kFloat && counts[a]->numel() == acc.size(1 + a),
                "counts must be float32 vectors of D, H and W elements");
  }
  const c10::cuda::CUDAGuard guard(acc.device());
  check_rc(crumpet_roi_argmax(labels, logits, acc.data_ptr<float>(), count_d.data_ptr<float>(),
                              count_h.data_ptr<float>(), count_w.data_ptr<float>(), acc.size(0),
                              acc.size(1), acc.size(2), acc.size(3), cur_stream(acc)));
}

void roi_argmax(at::Tensor& labels, const at::Tensor& acc, const at::Tensor& count_d,
                const at::Tensor& count_h, const at::Tensor& count_w) {
  check_cuda_contig(labels, "labels");
  check_cuda_contig(acc, "acc");
  same_device(acc, labels, "labels");
  TORCH_CHECK(labels.scalar_type() == at::kByte && labels.numel() == acc.numel() / acc.size(0),
              "labels must be a uint8 [D, H, W] tensor");
  roi_argmax_impl(labels.data_ptr<uint8_t>(), nullptr, acc, count_d, count_h, count_w);
}

void roi_normalize(at::Tensor& logits, const at::Tensor& acc, const at::Tensor& count_d,
                   const at::Tensor& count_h, const at::Tensor& count_w) {
  check_cuda_contig(logits, "logits");
  check_cuda_contig(acc, "acc");
  same_device(acc, logits, "logits");
  TORCH_CHECK(logits.scalar_type() == at::kFloat && logits.sizes() == acc.sizes(),
              "logits must be a float32 tensor shaped like acc");
  roi_argmax_impl(nullptr, logits.data_ptr<float>(), acc, count_d, count_h, count_w);
}

}  // namespace

TORCH_LIBRARY(crumpet_ops, ops) {
  ops.def(
      "compute_attn_mask_3d(Tensor! output, int D, int H, int W, int ws_d, int ws_h, int ws_w, "
      "int ss_d, int ss_h, int ss_w) -> ()",
      kTags);
  ops.def(
      "fused_shift_partition_3d(Tensor! output, Tensor x, int ws_d, int ws_h, int ws_w, int ss_d, "
      "int ss_h, int ss_w) -> ()",
      kTags);
  ops.def(
      "fused_shift_partition_3d_backward(Tensor! grad_x, Tensor grad_windows, int B, int D, int H, "
      "int W, int C, int ws_d, int ws_h, int ws_w, int ss_d, int ss_h, int ss_w) -> ()",
      kTags);
  ops.def(
      "fused_unshift_unpartition_3d(Tensor! output, Tensor windows, int B, int D, int H, int W, "
      "int C, int ws_d, int ws_h, int ws_w, int ss_d, int ss_h, int ss_w) -> ()",
      kTags);
  ops.def(
      "fused_unshift_unpartition_3d_backward(Tensor! grad_windows, Tensor grad_x, int ws_d, "
      "int ws_h, int ws_w, int ss_d, int ss_h, int ss_w) -> ()",
      kTags);
  ops.def(
      "fused_swin_attention(Tensor! out, Tensor q, Tensor k, Tensor v, Tensor rel_bias, "
      "Tensor? mask, Tensor? boundary, float scale) -> ()",
      kTags);
  ops.def(
      "fused_swin_attention_shifted(Tensor! out, Tensor q, Tensor k, Tensor v, Tensor rel_bias, "
      "Tensor? boundary, int[] num_windows, int[] window_size, int[] shift_size, float scale) "
      "-> ()",
      kTags);
  ops.def(
      "attention_bias_tiles(Tensor! tiles, Tensor table, Tensor index, int N, float scale, "
      "ScalarType dtype) -> ()",
      kTags);
  ops.def(
      "swin_window_attention_qkv_tiles(Tensor! out, Tensor qkv, Tensor bias_tiles, "
      "int[] num_windows, int[] window_size, int[] shift_size, float scale) -> ()",
      kTags);
  ops.def(
      "swin_window_attention_qkv(Tensor! out, Tensor qkv, Tensor table, Tensor index, "
      "int[] num_windows, int[] window_size, int[] shift_size, float scale) -> ()",
      kTags);
  ops.def(
      "norm_shift_partition_3d(Tensor! output, Tensor x, Tensor weight, Tensor bias, float eps, "
      "int ws_d, int ws_h, int ws_w, int ss_d, int ss_h, int ss_w) -> ()",
      kTags);
  ops.def(
      "unshift_unpartition_crop_3d(Tensor! output, Tensor windows, Tensor? residual, int B, int D, "
      "int H, int W, int C, int ws_d, int ws_h, int ws_w, int ss_d, int ss_h, int ss_w) -> ()",
      kTags);
  ops.def(
      "unshift_unpartition_crop_norm_3d(Tensor(a!) output, Tensor(b!) normed, Tensor windows, "
      "Tensor? residual, Tensor weight, Tensor bias, float eps, int B, int D, int H, int W, int C, "
      "int ws_d, int ws_h, int ws_w, int ss_d, int ss_h, int ss_w) -> ()",
      kTags);
  ops.def(
      "patch_merge_norm_3d(Tensor! output, Tensor x, Tensor weight, Tensor bias, float eps, "
      "int[] parts) -> ()",
      kTags);
  ops.def(
      "proj_out_norm_3d(Tensor! output, Tensor x, Tensor? weight, Tensor? bias, float eps) -> ()",
      kTags);
  ops.def("window_linear(Tensor! out, Tensor x, Tensor weight, Tensor? bias) -> ()", kTags);
  ops.def("roi_gather(Tensor! out, Tensor volume, int[] starts, int[] roi) -> ()", kTags);
  ops.def("roi_accumulate(Tensor! acc, Tensor pred, int[] starts, int[] roi) -> ()", kTags);
  ops.def(
      "roi_argmax(Tensor! labels, Tensor acc, Tensor count_d, Tensor count_h, Tensor count_w) -> ()",
      kTags);
  ops.def(
      "roi_normalize(Tensor! logits, Tensor acc, Tensor count_d, Tensor count_h, "
      "Tensor count_w) -> ()",
      kTags);
}

TORCH_LIBRARY_IMPL(crumpet_ops, CUDA, ops) {
  ops.impl("compute_attn_mask_3d", &compute_attn_mask_3d);
  ops.impl("fused_shift_partition_3d", &fused_shift_partition_3d);
  ops.impl("fused_shift_partition_3d_backward", &fused_shift_partition_3d_backward);
  ops.impl("fused_unshift_unpartition_3d", &fused_unshift_unpartition_3d);
  ops.impl("fused_unshift_unpartition_3d_backward", &fused_unshift_unpartition_3d_backward);
  ops.impl("fused_swin_attention", &fused_swin_attention);
  ops.impl("swin_window_attention_qkv", &swin_window_attention_qkv);
  ops.impl("attention_bias_tiles", &attention_bias_tiles);
  ops.impl("swin_window_attention_qkv_tiles", &swin_window_attention_qkv_tiles);
  ops.impl("fused_swin_attention_shifted", &fused_swin_attention_shifted);
  ops.impl("norm_shift_partition_3d", &norm_shift_partition_3d);
  ops.impl("unshift_unpartition_crop_3d", &unshift_unpartition_crop_3d);
  ops.impl("unshift_unpartition_crop_norm_3d", &unshift_unpartition_crop_norm_3d);
  ops.impl("patch_merge_norm_3d", &patch_merge_norm_3d);
  ops.impl("proj_out_norm_3d", &proj_out_norm_3d);
  ops.impl("window_linear", &window_linear);
  ops.impl("roi_gather", &roi_gather);
  ops.impl("roi_accumulate", &roi_accumulate);
  ops.impl("roi_argmax", &roi_argmax);
  ops.impl("roi_normalize", &roi_normalize);
}
