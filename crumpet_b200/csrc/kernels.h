// crumpet_b200: internal launcher interface between the C ABI (capi.cu) and
// the kernel translation units.  Nothing here is exported.
#pragma once

#include <cstdint>
#include <cuda_runtime.h>

namespace crumpet {

enum Status : int {
  kOk = 0,
  kErrInvalid = 1,
  kErrCuda = 2,
  kErrUnsupported = 3,
  kErrDevice = 4,
};

// Records a message for crumpet_last_error() and returns `code`.
int set_error(int code, const char* msg);
int set_cuda_error(cudaError_t err, const char* where);

struct ShapeArgs {
  int64_t B, D, H, W, C;
  int64_t ws_d, ws_h, ws_w;
  int64_t ss_d, ss_h, ss_w;
};

int launch_window_copy(bool forward, void* out, const void* in, const ShapeArgs& s, int dtype,
                       cudaStream_t stream);

int launch_attn_mask(void* out, int64_t D, int64_t H, int64_t W, int64_t ws_d, int64_t ws_h,
                     int64_t ws_w, int64_t ss_d, int64_t ss_h, int64_t ss_w, int dtype,
                     cudaStream_t stream);

// LayerNorm + zero pad to a window multiple + roll(-ss) + partition.  D/H/W are the
// unpadded dims; ws/ss point at 3 values.  gamma/beta are fp32 [C].
int launch_norm_shift_partition(void* out, int out_dtype, const void* x, int in_dtype,
                                const float* gamma, const float* beta, float eps, int64_t B,
                                int64_t D, int64_t H, int64_t W, int64_t C, const int64_t* ws,
                                const int64_t* ss, cudaStream_t stream);

// Unpartition on the padded grid + roll(+ss) + crop to D/H/W (+ residual, same dtype).
int launch_unshift_unpartition_crop(void* out, const void* windows, const void* residual,
                                    int dtype, int64_t B, int64_t D, int64_t H, int64_t W,
                                    int64_t C, const int64_t* ws, const int64_t* ss,
                                    cudaStream_t stream);

// Unpartition + roll back + crop (+ residual) as above, plus normed = LayerNorm(out)
// (fp32 gamma/beta, written in norm_dtype) in the same pass.
int launch_unshift_unpartition_crop_norm(void* out, void* normed, int norm_dtype,
                                         const void* windows, const void* residual, int dtype,
                                         const float* gamma, const float* beta, float eps,
                                         int64_t B, int64_t D, int64_t H, int64_t W, int64_t C,
                                         const int64_t* ws, const int64_t* ss, cudaStream_t stream);

// Patch merging: out [B, ceil(D/2), ceil(H/2), ceil(W/2), 8C] = LayerNorm over the 8
// neighbours' channels concatenated in the order parts[0..7] (code i | j<<1 | k<<2 for
// the offset (i, j, k)), zero rows past odd dims.  fp32 gamma/beta of 8C.
int launch_patch_merge_norm(void* out, int out_dtype, const void* x, int in_dtype,
                            const float* gamma, const float* beta, float eps, int64_t B, int64_t D,
                            int64_t H, int64_t W, int64_t C, const int* parts, cudaStream_t stream);

// LayerNorm over the channels of a channels-first volume x [B, C, D, H, W], written
// channels-last out [B, D, H, W, C]; fp32 gamma/beta of C, or both null (no affine).
// proj_out_norm_lanes(C) is the lanes per voxel (0: C unsupported).
int proj_out_norm_lanes(int64_t C);

// out[M, N] = x[M, K] * w[N, K]^T + bias[N] on the tensor cores (fp16 / bf16 operands,
// fp32 accumulation, fp32 bias or null); K = 48 (N <= 256) or 96 (N <= 160), N % 16 == 0.
bool window_linear_supported(int64_t K, int64_t N);
int launch_window_linear(void* out, const void* x, const void* w, const float* bias, int dtype,
                         int64_t M, int64_t K, int64_t N, cudaStream_t stream);
int read_linear_error(bool clear);
int launch_proj_out_norm(void* out, int out_dtype, const void* x, int in_dtype,
                         const float* gamma, const float* beta, float eps, int64_t B, int64_t C,
                         int64_t D, int64_t H, int64_t W, cudaStream_t stream);

// Sliding-window ROI inference: crop a batch of ROIs, accumulate their predictions,
// normalise by the ROI count and take the arg-max.  `starts` is a HOST array of
// n (z, y, x) triples (n <= 64), passed to the kernels by value.
int launch_roi_gather(void* out, int out_dtype, const void* vol, int in_dtype, int64_t C,
                      int64_t D, int64_t H, int64_t W, const int64_t* starts, int64_t n,
                      int64_t rd, int64_t rh, int64_t rw, cudaStream_t stream);
int launch_roi_accumulate(float* acc, const void* pred, int pred_dtype, int64_t classes,
                          int64_t D, int64_t H, int64_t W, const int64_t* starts, int64_t n,
                          int64_t rd, int64_t rh, int64_t rw, cudaStream_t stream);
int launch_roi_argmax(uint8_t* labels, float* logits, const float* acc, const float* count_d,
                      const float* count_h, const float* count_w, int64_t classes, int64_t D,
                      int64_t H, int64_t W, cudaStream_t stream);

// Window attention: out = softmax(q k^T * scale + bias[h] + mask[b mod nmask]) v.
struct AttnArgs {
  // q/k/v addressing: element (b, h, n, d) lives at
  //   base + b*stride_b + h*stride_h + n*stride_n + d     (elements)
  const void* q;
  const void* k;
  const void* v;
  int64_t qkv_stride_b, qkv_stride_h, qkv_stride_n;
  void* out;
  int64_t out_stride_b, out_stride_h, out_stride_n;
  const void* bias;        // [H, N, N] contiguous, same dtype as q (when !bias_from_table)
  bool bias_from_table;    // gather bias[h,i,j] = table[index[i*index_stride + j], h]
  const void* table;       // [T, H] fp32 (table_f32) or the element type
  bool table_f32;
  int64_t table_rows;      // T: index values outside [0, T) are flagged, not read
  const void* bias_tiles;  // prebuilt bias tiles (attention_bias_tiles) or nullptr
  const int64_t* index;    // [>=N, index_stride] relative position index, sliced [:N, :N]
  int64_t index_stride;
  const void* mask;        // [mask_windows, N, N] contiguous or nullptr
  int64_t mask_windows;    // window b uses mask[b % mask_windows]
  const uint8_t* boundary; // [B] or nullptr (nullptr + mask => every window masked)
  bool analytic;           // shifted-window mask computed on chip from the geometry below
  int64_t nwin[3];         // windows per axis of one batch entry (window b is b % prod)
  int64_t win[3];          // window size (win[0]*win[1]*win[2] == N)
  int64_t shift[3];        // cyclic shift; all zero means no mask
  int64_t B, H, N, head_dim;
  float scale;
  int dtype;               // kF32, kF16 or kBF16
};

int launch_window_attention(const AttnArgs& a, cudaStream_t stream);

// Prebuilt bias tiles for the tensor-core attention kernel: the per-(head, query tile)
// bias operand images it would otherwise gather from table + index in every CTA
// (reads table, table_f32, table_rows, index, index_stride, H, N, scale, dtype).
int64_t attention_bias_tiles_bytes(int64_t H, int64_t N);
int launch_attention_bias_tiles(void* tiles, const AttnArgs& a, cudaStream_t stream);
// launch_attention_bias_tiles into a fixed 4 MiB device buffer of the library, then the
// attention with those tiles: no device allocation by anyone.
int launch_window_attention_static_tiles(const AttnArgs& a, cudaStream_t stream);

// The fp32 SIMT attention kernel (attention_simt.cu) for what the tensor-core kernel does
// not take: float32 q/k/v, head_dim 64..256, N > 384, unaligned operands.  Arguments are
// validated by launch_window_attention, which dispatches here.
bool simt_attention_head_dim(int64_t head_dim);
int launch_window_attention_simt(const AttnArgs& a, cudaStream_t stream);

// Test hook: while enabled, attention launches issue no TMA loads (every wait in
// the kernel expires after its time limit).  Returns the previous setting.
int set_attention_test_stall(int enable);

// Device-side error word written by kernels whose bounded waits expired.
// Reads it (synchronously); clears it when `clear`.  Returns -1 on failure.
int read_device_error(bool clear);

}  // namespace crumpet
