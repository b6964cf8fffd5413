// crumpet_b200: the C ABI (declared in include/crumpet_b200.h).
//
// Every entry point validates its arguments the way the reference's Python
// wrappers and C++ ops do (torch-ext/crumpet/__init__.py:89-123,
// cuda/attn_mask_3d.cu:143), launches on the caller's stream, never allocates
// and never synchronises.  Failures return a non-zero status and leave a
// message for crumpet_last_error().
#include <cstdio>
#include <cstring>

#include "../../include/crumpet_b200.h"
#include "common.cuh"
#include "kernels.h"

namespace crumpet {

namespace {
thread_local char g_last_error[512] = {0};
}

int set_error(int code, const char* msg) {
  std::snprintf(g_last_error, sizeof(g_last_error), "%s", msg);
  return code;
}

int set_cuda_error(cudaError_t err, const char* where) {
  std::snprintf(g_last_error, sizeof(g_last_error), "%s: %s", where, cudaGetErrorString(err));
  return kErrCuda;
}

namespace {

int check_dtype(int dtype) {
  if (dtype != kF32 && dtype != kF16 && dtype != kBF16)
    return set_error(kErrInvalid, "CRUMPET supports float32, float16 and bfloat16");
  return kOk;
}

// Mirrors _validate_shape (torch-ext/crumpet/__init__.py:98-117).
int check_window_shape(int64_t D, int64_t H, int64_t W, int64_t ws_d, int64_t ws_h, int64_t ws_w,
                       int64_t ss_d, int64_t ss_h, int64_t ss_w) {
  if (D <= 0 || H <= 0 || W <= 0) return set_error(kErrInvalid, "D, H and W must be positive");
  if (ws_d <= 0 || ws_h <= 0 || ws_w <= 0)
    return set_error(kErrInvalid, "window_size values must be positive");
  if (D % ws_d || H % ws_h || W % ws_w)
    return set_error(kErrInvalid,
                     "standalone CRUMPET kernels require D, H and W to be divisible by window_size");
  const int64_t ss[3] = {ss_d, ss_h, ss_w};
  const int64_t ws[3] = {ws_d, ws_h, ws_w};
  for (int a = 0; a < 3; ++a) {
    if (ss[a] < 0 || ss[a] >= ws[a]) {
      char buf[96];
      std::snprintf(buf, sizeof(buf), "shift_size[%d] must satisfy 0 <= shift < window_size[%d]", a,
                    a);
      return set_error(kErrInvalid, buf);
    }
  }
  // 32-bit index arithmetic inside one window and one volume slice.
  if (D * H * W >= (int64_t(1) << 31)) return set_error(kErrInvalid, "D*H*W must be below 2^31");
  return kOk;
}

int window_copy(bool forward, void* out, const void* in, int dtype, int64_t B, int64_t D, int64_t H,
                int64_t W, int64_t C, int64_t ws_d, int64_t ws_h, int64_t ws_w, int64_t ss_d,
                int64_t ss_h, int64_t ss_w, void* stream) {
  if (int e = check_dtype(dtype)) return e;
  if (int e = check_window_shape(D, H, W, ws_d, ws_h, ws_w, ss_d, ss_h, ss_w)) return e;
  if (B < 0 || C < 0) return set_error(kErrInvalid, "B and C must be non-negative");
  if (B == 0 || C == 0) return kOk;  // empty output: nothing to do
  if (out == nullptr || in == nullptr) return set_error(kErrInvalid, "null tensor pointer");
  const ShapeArgs s{B, D, H, W, C, ws_d, ws_h, ws_w, ss_d, ss_h, ss_w};
  return launch_window_copy(forward, out, in, s, dtype, static_cast<cudaStream_t>(stream));
}

}  // namespace
}  // namespace crumpet

using namespace crumpet;

extern "C" {

const char* crumpet_last_error(void) { return g_last_error; }

int crumpet_abi_version(void) { return CRUMPET_ABI_VERSION; }

int crumpet_fused_shift_partition_3d(void* output, const void* x, int dtype, int64_t B, int64_t D,
                                     int64_t H, int64_t W, int64_t C, int64_t ws_d, int64_t ws_h,
                                     int64_t ws_w, int64_t ss_d, int64_t ss_h, int64_t ss_w,
                                     void* stream) {
  return window_copy(true, output, x, dtype, B, D, H, W, C, ws_d, ws_h, ws_w, ss_d, ss_h, ss_w,
                     stream);
}

int crumpet_fused_unshift_unpartition_3d(void* output, const void* windows, int dtype, int64_t B,
                                         int64_t D, int64_t H, int64_t W, int64_t C, int64_t ws_d,
                                         int64_t ws_h, int64_t ws_w, int64_t ss_d, int64_t ss_h,
                                         int64_t ss_w, void* stream) {
  return window_copy(false, output, windows, dtype, B, D, H, W, C, ws_d, ws_h, ws_w, ss_d, ss_h,
                     ss_w, stream);
}

int crumpet_fused_shift_partition_3d_backward(void* grad_x, const void* grad_windows, int dtype,
                                              int64_t B, int64_t D, int64_t H, int64_t W,
                                              int64_t C, int64_t ws_d, int64_t ws_h, int64_t ws_w,
                                              int64_t ss_d, int64_t ss_h, int64_t ss_w,
                                              void* stream) {
  return window_copy(false, grad_x, grad_windows, dtype, B, D, H, W, C, ws_d, ws_h, ws_w, ss_d,
                     ss_h, ss_w, stream);
}

int crumpet_fused_unshift_unpartition_3d_backward(void* grad_windows, const void* grad_x,
                                                  int dtype, int64_t B, int64_t D, int64_t H,
                                                  int64_t W, int64_t C, int64_t ws_d, int64_t ws_h,
                                                  int64_t ws_w, int64_t ss_d, int64_t ss_h,
                                                  int64_t ss_w, void* stream) {
  return window_copy(true, grad_windows, grad_x, dtype, B, D, H, W, C, ws_d, ws_h, ws_w, ss_d, ss_h,
                     ss_w, stream);
}

int crumpet_compute_attn_mask_3d(void* output, int dtype, int64_t D, int64_t H, int64_t W,
                                 int64_t ws_d, int64_t ws_h, int64_t ws_w, int64_t ss_d,
                                 int64_t ss_h, int64_t ss_w, void* stream) {
  if (int e = check_dtype(dtype)) return e;
  if (int e = check_window_shape(D, H, W, ws_d, ws_h, ws_w, ss_d, ss_h, ss_w)) return e;
  if (output == nullptr) return set_error(kErrInvalid, "null tensor pointer");
  return launch_attn_mask(output, D, H, W, ws_d, ws_h, ws_w, ss_d, ss_h, ss_w, dtype,
                          static_cast<cudaStream_t>(stream));
}

int crumpet_fused_swin_attention(void* out, const void* q, const void* k, const void* v,
                                 const void* rel_bias, const void* mask, int64_t mask_windows,
                                 const uint8_t* boundary, int dtype, int64_t B, int64_t H,
                                 int64_t N, int64_t head_dim, float scale, void* stream) {
  AttnArgs a{};
  a.q = q;
  a.k = k;
  a.v = v;
  a.qkv_stride_n = head_dim;
  a.qkv_stride_h = N * head_dim;
  a.qkv_stride_b = H * N * head_dim;
  a.out = out;
  a.out_stride_n = head_dim;
  a.out_stride_h = N * head_dim;
  a.out_stride_b = H * N * head_dim;
  a.bias = rel_bias;
  a.mask = mask;
  a.mask_windows = mask_windows;
  a.boundary = boundary;
  a.B = B;
  a.H = H;
  a.N = N;
  a.head_dim = head_dim;
  a.scale = scale;
  a.dtype = dtype;
  return launch_window_attention(a, static_cast<cudaStream_t>(stream));
}

int crumpet_fused_swin_attention_shifted(void* out, const void* q, const void* k,
                                         const void* v, const void* rel_bias,
                                         const uint8_t* boundary, int dtype, int64_t B,
                                         int64_t H, int64_t N, int64_t head_dim, int64_t nw_d,
                                         int64_t nw_h, int64_t nw_w, int64_t ws_d, int64_t ws_h,
                                         int64_t ws_w, int64_t ss_d, int64_t ss_h, int64_t ss_w,
                                         float scale, void* stream) {
  AttnArgs a{};
  a.q = q;
  a.k = k;
  a.v = v;
  a.qkv_stride_n = head_dim;
  a.qkv_stride_h = N * head_dim;
  a.qkv_stride_b = H * N * head_dim;
  a.out = out;
  a.out_stride_n = head_dim;
  a.out_stride_h = N * head_dim;
  a.out_stride_b = H * N * head_dim;
  a.bias = rel_bias;
  a.boundary = boundary;
  a.analytic = (ss_d | ss_h | ss_w) != 0;
  a.nwin[0] = nw_d;
  a.nwin[1] = nw_h;
  a.nwin[2] = nw_w;
  a.win[0] = ws_d;
  a.win[1] = ws_h;
  a.win[2] = ws_w;
  a.shift[0] = ss_d;
  a.shift[1] = ss_h;
  a.shift[2] = ss_w;
  a.B = B;
  a.H = H;
  a.N = N;
  a.head_dim = head_dim;
  a.scale = scale;
  a.dtype = dtype;
  return launch_window_attention(a, static_cast<cudaStream_t>(stream));
}

int crumpet_swin_window_attention_qkv(void* out, const void* qkv, const void* bias_table,
                                      int table_f32, int64_t table_rows, const int64_t* rel_index,
                                      int64_t index_stride, int64_t nw_d, int64_t nw_h,
                                      int64_t nw_w, int64_t ws_d, int64_t ws_h, int64_t ws_w,
                                      int64_t ss_d, int64_t ss_h, int64_t ss_w, int dtype,
                                      int64_t B, int64_t H, int64_t N, int64_t head_dim,
                                      float scale, void* stream) {
  AttnArgs a{};
  const int64_t hd = H * head_dim;
  const int64_t esize = dtype == kF32 ? 4 : 2;
  a.q = qkv;
  a.k = static_cast<const char*>(qkv) + hd * esize;
  a.v = static_cast<const char*>(qkv) + 2 * hd * esize;
  a.qkv_stride_n = 3 * hd;
  a.qkv_stride_h = head_dim;
  a.qkv_stride_b = N * 3 * hd;
  a.out = out;
  a.out_stride_n = hd;
  a.out_stride_h = head_dim;
  a.out_stride_b = N * hd;
  a.bias_from_table = true;
  a.table = bias_table;
  a.table_f32 = table_f32 != 0;
  a.table_rows = table_rows;
  a.index = rel_index;
  a.index_stride = index_stride;
  a.analytic = (ss_d | ss_h | ss_w) != 0;
  a.nwin[0] = nw_d;
  a.nwin[1] = nw_h;
  a.nwin[2] = nw_w;
  a.win[0] = ws_d;
  a.win[1] = ws_h;
  a.win[2] = ws_w;
  a.shift[0] = ss_d;
  a.shift[1] = ss_h;
  a.shift[2] = ss_w;
  a.B = B;
  a.H = H;
  a.N = N;
  a.head_dim = head_dim;
  a.scale = scale;
  a.dtype = dtype;
  return launch_window_attention(a, static_cast<cudaStream_t>(stream));
}

int crumpet_swin_window_attention_qkv_static_tiles(
    void* out, const void* qkv, const void* bias_table, int table_f32, int64_t table_rows,
    const int64_t* rel_index, int64_t index_stride, int64_t nw_d, int64_t nw_h, int64_t nw_w,
    int64_t ws_d, int64_t ws_h, int64_t ws_w, int64_t ss_d, int64_t ss_h, int64_t ss_w,
    int dtype, int64_t B, int64_t H, int64_t N, int64_t head_dim, float scale, void* stream) {
  AttnArgs a{};
  const int64_t hd = H * head_dim;
  const int64_t esize = dtype == kF32 ? 4 : 2;
  a.q = qkv;
  a.k = static_cast<const char*>(qkv) + hd * esize;
  a.v = static_cast<const char*>(qkv) + 2 * hd * esize;
  a.qkv_stride_n = 3 * hd;
  a.qkv_stride_h = head_dim;
  a.qkv_stride_b = N * 3 * hd;
  a.out = out;
  a.out_stride_n = hd;
  a.out_stride_h = head_dim;
  a.out_stride_b = N * hd;
  a.bias_from_table = true;
  a.table = bias_table;
  a.table_f32 = table_f32 != 0;
  a.table_rows = table_rows;
  a.index = rel_index;
  a.index_stride = index_stride;
  a.analytic = (ss_d | ss_h | ss_w) != 0;
  a.nwin[0] = nw_d;
  a.nwin[1] = nw_h;
  a.nwin[2] = nw_w;
  a.win[0] = ws_d;
  a.win[1] = ws_h;
  a.win[2] = ws_w;
  a.shift[0] = ss_d;
  a.shift[1] = ss_h;
  a.shift[2] = ss_w;
  a.B = B;
  a.H = H;
  a.N = N;
  a.head_dim = head_dim;
  a.scale = scale;
  a.dtype = dtype;
  return launch_window_attention_static_tiles(a, static_cast<cudaStream_t>(stream));
}

int64_t crumpet_attention_bias_tiles_bytes(int64_t H, int64_t N) {
  return attention_bias_tiles_bytes(H, N);
}

int crumpet_attention_bias_tiles(void* tiles, const void* bias_table, int table_f32,
                                 int64_t table_rows, const int64_t* rel_index,
                                 int64_t index_stride, int dtype, int64_t H, int64_t N, float scale,
                                 void* stream) {
  AttnArgs a{};
  a.table = bias_table;
  a.table_f32 = table_f32 != 0;
  a.table_rows = table_rows;
  a.index = rel_index;
  a.index_stride = index_stride;
  a.bias_from_table = true;
  a.H = H;
  a.N = N;
  a.scale = scale;
  a.dtype = dtype;
  return launch_attention_bias_tiles(tiles, a, static_cast<cudaStream_t>(stream));
}

int crumpet_swin_window_attention_qkv_tiles(void* out, const void* qkv, const void* bias_tiles,
                                            int64_t nw_d, int64_t nw_h, int64_t nw_w,
                                            int64_t ws_d, int64_t ws_h, int64_t ws_w,
                                            int64_t ss_d, int64_t ss_h, int64_t ss_w, int dtype,
                                            int64_t B, int64_t H, int64_t N, int64_t head_dim,
                                            float scale, void* stream) {
  if (bias_tiles == nullptr) return set_error(kErrInvalid, "null bias tiles");
  AttnArgs a{};
  const int64_t hd = H * head_dim;
  const int64_t esize = dtype == kF32 ? 4 : 2;
  a.q = qkv;
  a.k = static_cast<const char*>(qkv) + hd * esize;
  a.v = static_cast<const char*>(qkv) + 2 * hd * esize;
  a.qkv_stride_n = 3 * hd;
  a.qkv_stride_h = head_dim;
  a.qkv_stride_b = N * 3 * hd;
  a.out = out;
  a.out_stride_n = hd;
  a.out_stride_h = head_dim;
  a.out_stride_b = N * hd;
  a.bias_from_table = true;
  a.bias_tiles = bias_tiles;
  a.analytic = (ss_d | ss_h | ss_w) != 0;
  a.nwin[0] = nw_d;
  a.nwin[1] = nw_h;
  a.nwin[2] = nw_w;
  a.win[0] = ws_d;
  a.win[1] = ws_h;
  a.win[2] = ws_w;
  a.shift[0] = ss_d;
  a.shift[1] = ss_h;
  a.shift[2] = ss_w;
  a.B = B;
  a.H = H;
  a.N = N;
  a.head_dim = head_dim;
  a.scale = scale;
  a.dtype = dtype;
  return launch_window_attention(a, static_cast<cudaStream_t>(stream));
}

int crumpet_norm_shift_partition_3d(void* output, int out_dtype, const void* x, int in_dtype,
                                    const float* weight, const float* bias, float eps, int64_t B,
                                    int64_t D, int64_t H, int64_t W, int64_t C, int64_t ws_d,
                                    int64_t ws_h, int64_t ws_w, int64_t ss_d, int64_t ss_h,
                                    int64_t ss_w, void* stream) {
  if (int e = check_dtype(out_dtype)) return e;
  if (int e = check_dtype(in_dtype)) return e;
  const int64_t ws[3] = {ws_d, ws_h, ws_w}, ss[3] = {ss_d, ss_h, ss_w};
  return launch_norm_shift_partition(output, out_dtype, x, in_dtype, weight, bias, eps, B, D, H, W,
                                     C, ws, ss, static_cast<cudaStream_t>(stream));
}

int crumpet_unshift_unpartition_crop_3d(void* output, const void* windows, const void* residual,
                                        int dtype, int64_t B, int64_t D, int64_t H, int64_t W,
                                        int64_t C, int64_t ws_d, int64_t ws_h, int64_t ws_w,
                                        int64_t ss_d, int64_t ss_h, int64_t ss_w, void* stream) {
  if (int e = check_dtype(dtype)) return e;
  const int64_t ws[3] = {ws_d, ws_h, ws_w}, ss[3] = {ss_d, ss_h, ss_w};
  return launch_unshift_unpartition_crop(output, windows, residual, dtype, B, D, H, W, C, ws, ss,
                                         static_cast<cudaStream_t>(stream));
}

int crumpet_unshift_unpartition_crop_norm_3d(void* output, void* normed, int norm_dtype,
                                             const void* windows, const void* residual, int dtype,
                                             const float* weight, const float* bias, float eps,
                                             int64_t B, int64_t D, int64_t H, int64_t W, int64_t C,
                                             int64_t ws_d, int64_t ws_h, int64_t ws_w,
                                             int64_t ss_d, int64_t ss_h, int64_t ss_w,
                                             void* stream) {
  if (int e = check_dtype(dtype)) return e;
  if (int e = check_dtype(norm_dtype)) return e;
  const int64_t ws[3] = {ws_d, ws_h, ws_w}, ss[3] = {ss_d, ss_h, ss_w};
  return launch_unshift_unpartition_crop_norm(output, normed, norm_dtype, windows, residual, dtype,
                                              weight, bias, eps, B, D, H, W, C, ws, ss,
                                              static_cast<cudaStream_t>(stream));
}

int crumpet_patch_merge_norm_3d(void* output, int out_dtype, const void* x, int in_dtype,
                                const float* weight, const float* bias, float eps, int64_t B,
                                int64_t D, int64_t H, int64_t W, int64_t C, const int* parts,
                                void* stream) {
  if (int e = check_dtype(out_dtype)) return e;
  if (int e = check_dtype(in_dtype)) return e;
  return launch_patch_merge_norm(output, out_dtype, x, in_dtype, weight, bias, eps, B, D, H, W, C,
                                 parts, static_cast<cudaStream_t>(stream));
}

int crumpet_window_linear(void* out, const void* x, const void* weight, const float* bias,
                          int dtype, int64_t M, int64_t K, int64_t N, void* stream) {
  if (int e = check_dtype(dtype)) return e;
  return launch_window_linear(out, x, weight, bias, dtype, M, K, N,
                              static_cast<cudaStream_t>(stream));
}

int crumpet_proj_out_norm_3d(void* output, int out_dtype, const void* x, int in_dtype,
                             const float* weight, const float* bias, float eps, int64_t B,
                             int64_t C, int64_t D, int64_t H, int64_t W, void* stream) {
  if (int e = check_dtype(out_dtype)) return e;
  if (int e = check_dtype(in_dtype)) return e;
  return launch_proj_out_norm(output, out_dtype, x, in_dtype, weight, bias, eps, B, C, D, H, W,
                              static_cast<cudaStream_t>(stream));
}

int crumpet_roi_gather(void* out, int out_dtype, const void* volume, int in_dtype, int64_t C,
                       int64_t D, int64_t H, int64_t W, const int64_t* roi_starts, int64_t n,
                       int64_t rd, int64_t rh, int64_t rw, void* stream) {
  if (int e = check_dtype(out_dtype)) return e;
  if (int e = check_dtype(in_dtype)) return e;
  return launch_roi_gather(out, out_dtype, volume, in_dtype, C, D, H, W, roi_starts, n, rd, rh,
                           rw, static_cast<cudaStream_t>(stream));
}

int crumpet_roi_accumulate(float* acc, const void* pred, int pred_dtype, int64_t classes,
                           int64_t D, int64_t H, int64_t W, const int64_t* roi_starts, int64_t n,
                           int64_t rd, int64_t rh, int64_t rw, void* stream) {
  if (int e = check_dtype(pred_dtype)) return e;
  return launch_roi_accumulate(acc, pred, pred_dtype, classes, D, H, W, roi_starts, n, rd, rh, rw,
                               static_cast<cudaStream_t>(stream));
}

int crumpet_roi_argmax(uint8_t* labels, float* logits, const float* acc, const float* count_d,
                       const float* count_h, const float* count_w, int64_t classes, int64_t D,
                       int64_t H, int64_t W, void* stream) {
  return launch_roi_argmax(labels, logits, acc, count_d, count_h, count_w, classes, D, H, W,
                           static_cast<cudaStream_t>(stream));
}

int crumpet_test_stall_attention(int enable) { return set_attention_test_stall(enable); }

int crumpet_device_status(int clear) {
  const int v = read_device_error(clear != 0);
  if (v < 0) return set_error(kErrCuda, "could not read the device error word");
  return v;
}

}  // extern "C"
