/*
 * crumpet_b200 — C ABI of the B200 (sm_100a) shifted-window kernels.
 *
 * Plain pointers, sizes and a CUDA stream (passed as void*, i.e. cudaStream_t;
 * NULL = legacy default stream).  No entry point allocates device memory or
 * synchronises the device; all of them launch asynchronously on `stream` and
 * return CRUMPET_OK or an error status, with a message in crumpet_last_error().
 * Tensors are dense and C-contiguous unless a stride argument says otherwise.
 *
 * Each entry point names the reference interface it replaces
 * (chrisvoncsefalvay/crumpet, path:line).  The torch dispatcher ops in
 * crumpet_b200/csrc/torch_binding.cpp are thin adapters over these functions.
 */
#ifndef CRUMPET_B200_H_
#define CRUMPET_B200_H_

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define CRUMPET_ABI_VERSION 2

#if defined(__GNUC__)
#define CRUMPET_API __attribute__((visibility("default")))
#else
#define CRUMPET_API
#endif

/* Element types. */
#define CRUMPET_DTYPE_F32 0
#define CRUMPET_DTYPE_F16 1
#define CRUMPET_DTYPE_BF16 2

/* Status codes. */
#define CRUMPET_OK 0
#define CRUMPET_ERR_INVALID 1     /* bad shape, size, dtype or pointer */
#define CRUMPET_ERR_CUDA 2        /* a CUDA runtime call or launch failed */
#define CRUMPET_ERR_UNSUPPORTED 3 /* valid request this build does not handle */
#define CRUMPET_ERR_DEVICE 4      /* a kernel reported a device-side error */

/* Message of the last failing call on this host thread ("" if none). */
CRUMPET_API const char* crumpet_last_error(void);

/* Returns CRUMPET_ABI_VERSION. */
CRUMPET_API int crumpet_abi_version(void);

/*
 * Cyclic roll by -ss over (D,H,W) followed by the 3D window partition.
 *   x      [B, D, H, W, C]                 (dtype)
 *   output [B * nW, ws_d*ws_h*ws_w, C]     nW = (D/ws_d)(H/ws_h)(W/ws_w)
 * Requires D, H, W divisible by the window and 0 <= ss < ws per axis.
 * Replaces op crumpet_ops::fused_shift_partition_3d
 *   (torch-ext/torch_binding.cpp:20-22, torch-ext/torch_binding.h:19-27,
 *    cuda/shift_partition_3d.cu:318-347).  Shapes are explicit here because
 *    the C ABI carries no tensor metadata.
 */
CRUMPET_API int crumpet_fused_shift_partition_3d(void* output, const void* x, int dtype, int64_t B, int64_t D,
                                     int64_t H, int64_t W, int64_t C, int64_t ws_d, int64_t ws_h,
                                     int64_t ws_w, int64_t ss_d, int64_t ss_h, int64_t ss_w,
                                     void* stream);

/*
 * Window reverse followed by a cyclic roll by +ss: the exact inverse of
 * crumpet_fused_shift_partition_3d.
 *   windows [B * nW, ws_d*ws_h*ws_w, C]  ->  output [B, D, H, W, C]
 * Replaces op crumpet_ops::fused_unshift_unpartition_3d
 *   (torch-ext/torch_binding.cpp:26-28, torch-ext/torch_binding.h:43-56,
 *    cuda/unshift_unpartition_3d.cu:284-318).
 */
CRUMPET_API int crumpet_fused_unshift_unpartition_3d(void* output, const void* windows, int dtype, int64_t B,
                                         int64_t D, int64_t H, int64_t W, int64_t C, int64_t ws_d,
                                         int64_t ws_h, int64_t ws_w, int64_t ss_d, int64_t ss_h,
                                         int64_t ss_w, void* stream);

/*
 * Gradient of the partition: grad_x = unshift_unpartition(grad_windows).
 * Replaces op crumpet_ops::fused_shift_partition_3d_backward
 *   (torch-ext/torch_binding.cpp:23-25, cuda/unshift_unpartition_3d.cu:320-348).
 */
CRUMPET_API int crumpet_fused_shift_partition_3d_backward(void* grad_x, const void* grad_windows, int dtype,
                                              int64_t B, int64_t D, int64_t H, int64_t W,
                                              int64_t C, int64_t ws_d, int64_t ws_h, int64_t ws_w,
                                              int64_t ss_d, int64_t ss_h, int64_t ss_w,
                                              void* stream);

/*
 * Gradient of the unpartition: grad_windows = shift_partition(grad_x).
 * Replaces op crumpet_ops::fused_unshift_unpartition_3d_backward
 *   (torch-ext/torch_binding.cpp:29-31, cuda/shift_partition_3d.cu:349-367).
 */
CRUMPET_API int crumpet_fused_unshift_unpartition_3d_backward(void* grad_windows, const void* grad_x,
                                                  int dtype, int64_t B, int64_t D, int64_t H,
                                                  int64_t W, int64_t C, int64_t ws_d, int64_t ws_h,
                                                  int64_t ws_w, int64_t ss_d, int64_t ss_h,
                                                  int64_t ss_w, void* stream);

/*
 * Shifted-window attention mask, output [nW, N, N] with N = ws_d*ws_h*ws_w <= 1024:
 * -100 where two tokens of a window come from different roll regions, else 0
 * (all zeros when every shift is zero).
 * Replaces op crumpet_ops::compute_attn_mask_3d
 *   (torch-ext/torch_binding.cpp:17-19, torch-ext/torch_binding.h:8-17,
 *    cuda/attn_mask_3d.cu:127-168).
 */
CRUMPET_API int crumpet_compute_attn_mask_3d(void* output, int dtype, int64_t D, int64_t H, int64_t W,
                                 int64_t ws_d, int64_t ws_h, int64_t ws_w, int64_t ss_d,
                                 int64_t ss_h, int64_t ss_w, void* stream);

/*
 * Fused window attention, per window b and head h:
 *   out[b,h] = softmax(q[b,h] k[b,h]^T * scale + rel_bias[h] + mask[b % mask_windows]) v[b,h]
 * with fp32 accumulation and softmax.  q, k, v, out: [B, H, N, head_dim];
 * rel_bias: [H, N, N]; mask: [mask_windows, N, N] or NULL; boundary: uint8 [B]
 * or NULL.  When boundary is given, mask rows are read only for windows with
 * boundary[b] != 0 (the others are treated as unmasked); when it is NULL and a
 * mask is given, every window reads its mask.  dtype: F32, F16 or BF16 (all
 * tensors share it); head_dim 16, 32, 64, 128 or 256; any N >= 1.  F16 / BF16
 * with head_dim 16 or 32, N <= 352 and 16-byte aligned tensors run the tcgen05
 * tensor-core kernel; every other call runs an fp32 SIMT kernel.
 * Replaces crumpet.fused_attention.fused_swin_attention
 *   (torch-ext/crumpet/fused_attention.py:149-226; kernel :48-146), which the
 *   reference exposes only as a Python/Triton function.
 */
CRUMPET_API int crumpet_fused_swin_attention(void* out, const void* q, const void* k, const void* v,
                                 const void* rel_bias, const void* mask, int64_t mask_windows,
                                 const uint8_t* boundary, int dtype, int64_t B, int64_t H,
                                 int64_t N, int64_t head_dim, float scale, void* stream);

/*
 * crumpet_fused_swin_attention with, in place of a dense mask tensor, the shifted-window
 * mask that crumpet_compute_attn_mask_3d builds for the window grid
 *   nw_* windows per axis of one batch entry (window b is b % (nw_d*nw_h*nw_w)),
 *   ws_* window size (ws_d*ws_h*ws_w == N), ss_* cyclic shift (all 0: no mask),
 * computed on chip instead of read from memory (-100 where two tokens of a window come
 * from different roll regions).  boundary: uint8 [B] or NULL, as for
 * crumpet_fused_swin_attention: windows with boundary[b] == 0 are treated as unmasked.
 * The same function as crumpet_fused_swin_attention given that mask tensor, up to fp32
 * rounding, without the mask's HBM reads (645 MB at a 98^3 grid of 7^3 windows).  No
 * reference counterpart: the reference reads the mask tensor
 * (torch-ext/crumpet/fused_attention.py:123-129); crumpet_b200.fused_swin_attention
 * routes here when the mask it is given is one that compute_attn_mask_3d returned and
 * that has not been modified since.
 */
CRUMPET_API int crumpet_fused_swin_attention_shifted(
    void* out, const void* q, const void* k, const void* v, const void* rel_bias,
    const uint8_t* boundary, int dtype, int64_t B, int64_t H, int64_t N, int64_t head_dim,
    int64_t nw_d, int64_t nw_h, int64_t nw_w, int64_t ws_d, int64_t ws_h, int64_t ws_w,
    int64_t ss_d, int64_t ss_h, int64_t ss_w, float scale, void* stream);

/*
 * Fused window attention straight from the packed qkv Linear output, with the
 * relative-position bias gathered in-kernel and the shifted-window mask
 * computed on chip -- the whole body of MONAI's WindowAttention.forward
 * between its qkv and proj Linears.
 *   qkv   [B, N, 3, H, head_dim]   (q | k | v along dim 2; B = batch * nW)
 *   out   [B, N, H * head_dim]     (heads interleaved per token: ready for proj)
 *   bias_table [T, H]              fp32 when table_f32 != 0, else dtype; T = table_rows
 *   rel_index  [>=N, index_stride] int64; bias[h,i,j] = table[rel_index[i,j], h]
 *              for i, j < N (MONAI slices the configured window's index [:N, :N]).
 *              An index value outside [0, T) is not read: its bias is taken as 0 and
 *              the device error word (crumpet_device_status) gets bit 2 (value 2),
 *              where the eager table[index] would raise an indexing error.
 *   nw_*  windows per axis of one batch entry (window b is b % (nw_d*nw_h*nw_w))
 *   ws_*  window size (ws_d*ws_h*ws_w == N); ss_* cyclic shift (all 0: no mask)
 * The mask equals crumpet_compute_attn_mask_3d's on the padded grid; masked
 * scores are dropped exactly (e^-100 and e^-inf are both 0 in fp32).
 * dtype F32, F16 or BF16, head_dim 16 to 256 (powers of two), any N >= 1, with
 * the same split between the tensor-core and SIMT kernels as above.
 * Replaces the eager glue of torch-ext/crumpet/monai_patch.py:152-196 (q/k/v
 * split and .contiguous() copies, bias gather and permute, mask repeat, the
 * per-call mask abs().amax() scan, the output transpose) plus
 * fused_swin_attention.
 */
CRUMPET_API int crumpet_swin_window_attention_qkv(
    void* out, const void* qkv, const void* bias_table, int table_f32, int64_t table_rows,
    const int64_t* rel_index,
    int64_t index_stride, int64_t nw_d, int64_t nw_h, int64_t nw_w, int64_t ws_d, int64_t ws_h,
    int64_t ws_w, int64_t ss_d, int64_t ss_h, int64_t ss_w, int dtype, int64_t B, int64_t H,
    int64_t N, int64_t head_dim, float scale, void* stream);

/*
 * Prebuilt relative-position bias operands for the attention kernel.  The tensor-core
 * kernel adds the bias through the tensor cores from a per-(head, query tile) operand
 * image in shared memory, which crumpet_swin_window_attention_qkv gathers from the
 * table and index in every CTA.  With eval weights fixed, a caller can build the
 * images once (they depend on table, index, N, H, dtype and scale only) and pass them
 * to crumpet_swin_window_attention_qkv_tiles, whose CTAs then copy them in.
 *   crumpet_attention_bias_tiles_bytes: the buffer size for H heads and windows of N
 *     tokens, 0 when 1 <= N <= 352 does not hold (the tensor-core kernel's domain).
 *   crumpet_attention_bias_tiles: builds them into `tiles` (16-byte aligned, that many
 *     bytes); table, index and their checks as for crumpet_swin_window_attention_qkv
 *     (index values outside [0, table_rows) set bit 2 of crumpet_device_status).
 *   crumpet_swin_window_attention_qkv_tiles: crumpet_swin_window_attention_qkv with the
 *     bias from tiles built for the same H, N, dtype and scale (not checked: tiles of
 *     other parameters give wrong outputs).  dtype F16 or BF16, head_dim 16 or 32,
 *     N <= 352, 16-byte aligned tensors; other calls return CRUMPET_ERR_UNSUPPORTED.
 * No reference counterpart: the reference re-gathers the bias with torch on every
 * call (torch-ext/crumpet/monai_patch.py:160-162).
 */
CRUMPET_API int64_t crumpet_attention_bias_tiles_bytes(int64_t H, int64_t N);
CRUMPET_API int crumpet_attention_bias_tiles(void* tiles, const void* bias_table, int table_f32,
                                             int64_t table_rows, const int64_t* rel_index,
                                             int64_t index_stride, int dtype, int64_t H,
                                             int64_t N, float scale, void* stream);
CRUMPET_API int crumpet_swin_window_attention_qkv_tiles(
    void* out, const void* qkv, const void* bias_tiles, int64_t nw_d, int64_t nw_h, int64_t nw_w,
    int64_t ws_d, int64_t ws_h, int64_t ws_w, int64_t ss_d, int64_t ss_h, int64_t ss_w, int dtype,
    int64_t B, int64_t H, int64_t N, int64_t head_dim, float scale, void* stream);

/*
 * crumpet_swin_window_attention_qkv_static_tiles: the packed-qkv window attention
 * (arguments as crumpet_swin_window_attention_qkv; domain and results as
 * crumpet_swin_window_attention_qkv_tiles, with the tiles built from table and index
 * as crumpet_attention_bias_tiles builds them) for a
 * caller that cannot allocate device memory: one that runs where cudaMalloc is not
 * allowed or not wanted (an allocator-less runtime, a host that hands over only the
 * buffers it owns, a path that must not touch the device heap).  It still passes its
 * own qkv, table, index and output.  The bias tiles go into a buffer that is part of
 * the library image, 4 MiB on every GPU that loads the library, held until exit:
 * crumpet_attention_bias_tiles_bytes(H, N) must not exceed 4 MiB (at most 46 (head,
 * query tile) tiles at N = 343, 73 at N = 216), else CRUMPET_ERR_UNSUPPORTED.
 * Each call rebuilds every tile it reads, so nothing depends on an earlier call.
 * All calls on a GPU share that one buffer: calls that can overlap on the GPU (other
 * streams, other host threads) race on it; calls on one stream are ordered.
 * The first call on a device looks up the buffer's device address (with that device
 * current) and keeps it; make that first call before capturing a stream.
 * It allocates nothing itself, and nothing it calls does.  No counterpart in the
 * reference, which allocates its outputs and intermediates through torch.
 */
CRUMPET_API int crumpet_swin_window_attention_qkv_static_tiles(
    void* out, const void* qkv, const void* bias_table, int table_f32, int64_t table_rows,
    const int64_t* rel_index, int64_t index_stride, int64_t nw_d, int64_t nw_h, int64_t nw_w,
    int64_t ws_d, int64_t ws_h, int64_t ws_w, int64_t ss_d, int64_t ss_h, int64_t ss_w,
    int dtype, int64_t B, int64_t H, int64_t N, int64_t head_dim, float scale, void* stream);

/*
 * LayerNorm, zero padding, cyclic roll by -ss and window partition in one pass:
 * the first half of a Swin block's attention branch.
 *   x      [B, D, H, W, C]  (in_dtype), any D/H/W (not window multiples)
 *   output [B * nW, ws_d*ws_h*ws_w, C]  (out_dtype)
 *          nW = ceil(D/ws_d) * ceil(H/ws_h) * ceil(W/ws_w)
 * Token (b, win, loc) is LN(x[b, s]) with s = (win_coord*ws + loc_coord + ss)
 * mod padded dim when s lies inside the volume, and exactly 0 in the padding.
 * LN = (v - mean) / sqrt(var + eps) * weight + bias over C, fp32 arithmetic,
 * biased variance, one rounding to out_dtype.  weight, bias: fp32 [C].
 * C a multiple of 8, at most 768; all pointers 16-byte aligned.
 * Replaces norm1 -> F.pad -> crumpet_ops::fused_shift_partition_3d, and the fp16
 * cast autocast inserts before the qkv Linear, in
 *   torch-ext/crumpet/monai_patch.py:79-97 (the reference runs them as separate
 *   torch passes around its partition op).
 */
CRUMPET_API int crumpet_norm_shift_partition_3d(void* output, int out_dtype, const void* x,
                                                int in_dtype, const float* weight,
                                                const float* bias, float eps, int64_t B, int64_t D,
                                                int64_t H, int64_t W, int64_t C, int64_t ws_d,
                                                int64_t ws_h, int64_t ws_w, int64_t ss_d,
                                                int64_t ss_h, int64_t ss_w, void* stream);

/*
 * Window reverse on the padded grid, cyclic roll by +ss and crop to D/H/W in one
 * pass, optionally adding a residual:
 *   windows  [B * nW, ws_d*ws_h*ws_w, C]  (nW on the padded grid, as above)
 *   residual [B, D, H, W, C] or NULL
 *   output   [B, D, H, W, C] = unpartition(windows)[:, :D, :H, :W] (+ residual)
 * All three share dtype; the add is done in fp32 and rounded once (torch's
 * elementwise add).  Rows of C elements and the pointers must be 4-byte aligned.
 * Replaces crumpet_ops::fused_unshift_unpartition_3d -> crop .contiguous() in
 *   torch-ext/crumpet/monai_patch.py:108-111, and the residual add of the Swin
 *   block that calls it.
 */
CRUMPET_API int crumpet_unshift_unpartition_crop_3d(void* output, const void* windows,
                                                    const void* residual, int dtype, int64_t B,
                                                    int64_t D, int64_t H, int64_t W, int64_t C,
                                                    int64_t ws_d, int64_t ws_h, int64_t ws_w,
                                                    int64_t ss_d, int64_t ss_h, int64_t ss_w,
                                                    void* stream);

/*
 * crumpet_unshift_unpartition_crop_3d followed by the LayerNorm of its result, in
 * one pass: output = unpartition(windows)[:, :D, :H, :W] (+ residual), rounded to
 * dtype, and normed = LN(output) over C with fp32 weight/bias and eps, written in
 * norm_dtype (the LN reads the rounded output values).  In a Swin block this is
 * the residual add of the attention half and the norm2 that opens the MLP half.
 * All pointers 16-byte aligned, C a multiple of 8 and at most 768; residual may be
 * NULL.  No reference counterpart: the reference leaves the crop, the residual add
 * and norm2 to eager torch (torch-ext/crumpet/monai_patch.py:108-111 and the MONAI
 * block around it).
 */
CRUMPET_API int crumpet_unshift_unpartition_crop_norm_3d(
    void* output, void* normed, int norm_dtype, const void* windows, const void* residual,
    int dtype, const float* weight, const float* bias, float eps, int64_t B, int64_t D,
    int64_t H, int64_t W, int64_t C, int64_t ws_d, int64_t ws_h, int64_t ws_w, int64_t ss_d,
    int64_t ss_h, int64_t ss_w, void* stream);

/*
 * Patch merging (the downsample of a Swin stage) up to its LayerNorm: for every
 * output voxel (d2, h2, w2) of the half-resolution grid (odd dims round up), the
 * eight neighbours x[b, 2 d2 + i, 2 h2 + j, 2 w2 + k, :] are concatenated in the
 * order parts[0..7] (code i | j << 1 | k << 2; neighbours past an odd dim are zero
 * rows) and normalised over the 8C channels with fp32 weight/bias of 8C elements:
 *   x [B, D, H, W, C] (in_dtype) -> output [B, ceil(D/2), ceil(H/2), ceil(W/2), 8C] (out_dtype)
 * C a multiple of 8 with 8C <= 3072; pointers 16-byte aligned.  No reference
 * counterpart: the reference's patched BasicLayer calls the MONAI downsample
 * module eagerly (torch-ext/crumpet/monai_patch.py:228-230).
 */
CRUMPET_API int crumpet_patch_merge_norm_3d(void* output, int out_dtype, const void* x,
                                            int in_dtype, const float* weight, const float* bias,
                                            float eps, int64_t B, int64_t D, int64_t H, int64_t W,
                                            int64_t C, const int* parts, void* stream);

/*
 * Hidden-state normalisation of the Swin trunk: LayerNorm over the channels of a
 * channels-first volume, written channels-last,
 *   x [B, C, D, H, W] (in_dtype)  ->  output [B, D, H, W, C] (out_dtype),
 *   output[b, d, h, w, :] = LN(x[b, :, d, h, w]) over C in fp32 arithmetic,
 * with fp32 weight/bias of C elements, or both NULL for no affine (MONAI's
 * SwinTransformer.proj_out calls F.layer_norm without one).  The channels-last
 * result viewed as [B, C, D, H, W] is what proj_out returns.  C a multiple of 8,
 * at most 768, divisible by the lanes per voxel (C / 24 rounded up to a power of
 * two: every C = 24 * 2^k, 48 * 2^k, ...); pointers 16-byte aligned.  No
 * reference counterpart: the reference's end-to-end runs (benchmarks/bench_e2e.py,
 * torch-ext/crumpet/demo_btcv.py:98-129) execute MONAI's proj_out eagerly
 * (permute, fp32 cast under autocast, contiguous copy, LayerNorm).
 */
/*
 * Linear projection of window tokens on the tensor cores:
 *   out[m, n] = sum_k x[m, k] * weight[n, k] + bias[n]
 *   x [M, K], weight [N, K] (nn.Linear layout), out [M, N]: float16 or bfloat16
 *   (dtype), fp32 accumulation, one rounding; bias fp32 [N] or NULL.
 * K = 48 with N <= 256, or K = 96 with N <= 160; N a multiple of 16; pointers 16-byte
 * aligned.  Replaces
 * the qkv and proj nn.Linear calls of MONAI's WindowAttention around the
 * attention kernel (torch-ext/crumpet/monai_patch.py:154-197 runs them through
 * cuBLAS); a tcgen05 GEMM with TMA loads/stores and the bias add in its epilogue.
 */
CRUMPET_API int crumpet_window_linear(void* out, const void* x, const void* weight,
                                      const float* bias, int dtype, int64_t M, int64_t K,
                                      int64_t N, void* stream);

CRUMPET_API int crumpet_proj_out_norm_3d(void* output, int out_dtype, const void* x, int in_dtype,
                                         const float* weight, const float* bias, float eps,
                                         int64_t B, int64_t C, int64_t D, int64_t H, int64_t W,
                                         void* stream);

/*
 * Sliding-window ROI inference around the network forward.  The reference drives
 * its patched network with MONAI's sliding_window_inference (a third-party
 * Python function, called at torch-ext/crumpet/demo_btcv.py:98-129 with
 * mode="constant"); these three entry points replace its crop, accumulate and
 * normalise/arg-max passes.  `roi_starts` is a HOST array of n (z, y, x)
 * triples, n <= 64 (one ROI batch), copied into the kernel parameters; every
 * ROI must lie inside the D x H x W volume.
 *
 * crumpet_roi_gather: out[i] = volume[:, z_i:z_i+rd, y_i:y_i+rh, x_i:x_i+rw]
 *   volume [C, D, H, W] (in_dtype)  ->  out [n, C, rd, rh, rw] (out_dtype, one
 *   rounding).  Replaces the per-ROI slicing + torch.cat of the inferer.
 */
CRUMPET_API int crumpet_roi_gather(void* out, int out_dtype, const void* volume, int in_dtype,
                                   int64_t C, int64_t D, int64_t H, int64_t W,
                                   const int64_t* roi_starts, int64_t n, int64_t rd, int64_t rh,
                                   int64_t rw, void* stream);

/*
 * crumpet_roi_accumulate: acc[:, ROI i] += float(pred[i]) for i = 0 .. n-1 in
 * order (the same fp32 additions, in the same order, as a per-ROI loop).
 *   acc [classes, D, H, W] fp32, pred [n, classes, rd, rh, rw] (pred_dtype).
 */
CRUMPET_API int crumpet_roi_accumulate(float* acc, const void* pred, int pred_dtype,
                                       int64_t classes, int64_t D, int64_t H, int64_t W,
                                       const int64_t* roi_starts, int64_t n, int64_t rd,
                                       int64_t rh, int64_t rw, void* stream);

/*
 * crumpet_roi_argmax: per voxel v, logits[c, v] = acc[c, v] / count(v) with
 * count(d, h, w) = count_d[d] * count_h[h] * count_w[w] (ROIs covering the voxel
 * along each axis), labels[v] = first c maximising logits[c, v] (NaN is the
 * maximum, as torch.argmax).  labels (uint8 [D, H, W]) and logits (fp32
 * [classes, D, H, W]) may each be NULL.  classes <= 256.
 */
CRUMPET_API int crumpet_roi_argmax(uint8_t* labels, float* logits, const float* acc,
                                   const float* count_d, const float* count_h,
                                   const float* count_w, int64_t classes, int64_t D, int64_t H,
                                   int64_t W, void* stream);

/*
 * Device error word: non-zero once a kernel of this library gave up on a
 * bounded wait (bit 1: it then drained its work, freed its tensor memory and
 * returned without completing its output) or met a relative-position index
 * outside its table (bit 2).  Reading it synchronises with the
 * device; `clear` != 0 resets it.  Returns the word (0 = healthy) or a negative
 * value / CRUMPET_ERR_CUDA when it cannot be read.  No reference counterpart:
 * the reference kernels contain no waits.
 */
CRUMPET_API int crumpet_device_status(int clear);

/*
 * Test hook for the bounded-wait error path (no reference counterpart: the
 * reference kernels contain no waits).  While enabled (enable != 0), attention
 * launches issue no TMA loads, so every wait of the kernel runs into its 2 s
 * limit; the kernel then drains, frees its tensor memory, returns and sets the
 * device error word read by crumpet_device_status.  Returns the previous
 * setting.  Process-wide; for tests only.
 */
CRUMPET_API int crumpet_test_stall_attention(int enable);

#ifdef __cplusplus
}
#endif

#endif /* CRUMPET_B200_H_ */
