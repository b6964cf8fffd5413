// crumpet_b200: sliding-window ROI inference around the Swin UNETR forward.
//
// The reference's end-to-end runs drive the patched network with MONAI's
// sliding_window_inference (torch-ext/crumpet/demo_btcv.py:98-129; mode
// "constant", sw_batch_size ROIs per forward): crop the ROIs of a batch out of the
// volume, run the model, add every ROI's prediction into a float32 accumulator,
// divide by the per-voxel ROI count and take the arg-max.  Eager, that is one
// copy per ROI for the crop, a cast and an add per ROI for the accumulation, and
// three full-volume passes (count division, arg-max, cast) at the end.  Three
// kernels replace them:
//
// roi_gather:     out[i, c, z, y, x] = vol[c, sz_i + z, sy_i + y, sx_i + x], cast to
//                 the output type (the model's input type: fp16 under autocast).
// roi_accumulate: for every voxel of the batch's bounding box and every class,
//                 acc += float(pred[i, c, voxel - start_i]) over the ROIs i of the
//                 batch that cover it, in batch order -- the same fp32 additions in
//                 the same order as the eager per-ROI loop, so the sums are
//                 bit-identical.
// roi_argmax:     label = argmax_c acc[c, voxel] / count(voxel), count = cd[d]*ch[h]*cw[w]
//                 (the ROI grid is a product of per-axis start lists, so the count
//                 map factorises), first maximal index on ties, NaN counts as the
//                 maximum (torch.argmax); optionally writes the normalised logits.
// ROI starts travel in the kernel parameters: no device buffers, no copies.
#include "common.cuh"
#include "kernels.h"

namespace crumpet {

namespace {

constexpr int kThreads = 256;
constexpr int kMaxRois = 64;  // ROIs per call (an ROI batch of sliding-window inference)

struct RoiList {
  int n;
  int rd, rh, rw;
  int z[kMaxRois], y[kMaxRois], x[kMaxRois];
};

template <typename TOut>
__device__ __forceinline__ TOut cast_out(float v);
template <>
__device__ __forceinline__ float cast_out<float>(float v) { return v; }
template <>
__device__ __forceinline__ __half cast_out<__half>(float v) { return __float2half_rn(v); }
template <>
__device__ __forceinline__ __nv_bfloat16 cast_out<__nv_bfloat16>(float v) {
  return __float2bfloat16_rn(v);
}

template <typename TIn>
__device__ __forceinline__ float load_f32(const TIn* p);
template <>
__device__ __forceinline__ float load_f32<float>(const float* p) { return __ldg(p); }
template <>
__device__ __forceinline__ float load_f32<__half>(const __half* p) { return __half2float(__ldg(p)); }
template <>
__device__ __forceinline__ float load_f32<__nv_bfloat16>(const __nv_bfloat16* p) {
  return __bfloat162float(__ldg(p));
}

// One thread per output element; x fastest, so a warp reads one contiguous row.
template <typename TIn, typename TOut>
__global__ void __launch_bounds__(kThreads)
roi_gather_kernel(TOut* __restrict__ out, const TIn* __restrict__ vol, const RoiList rois,
                  uint32_t D, uint32_t H, uint32_t W, uint64_t total, DivMod64 f_roi,
                  DivMod32 f_rw, DivMod32 f_rh, DivMod32 f_rd) {
  for (uint64_t o = uint64_t(blockIdx.x) * kThreads + threadIdx.x; o < total;
       o += uint64_t(gridDim.x) * kThreads) {
    const uint32_t i = uint32_t(f_roi.div(o));  // ROI index
    const uint32_t r = uint32_t(o - uint64_t(i) * f_roi.d);
    uint32_t t, x, t2, y, c, z;
    f_rw.divmod(r, t, x);
    f_rh.divmod(t, t2, y);
    f_rd.divmod(t2, c, z);
    const uint64_t src = ((uint64_t(c) * D + (rois.z[i] + z)) * H + (rois.y[i] + y)) * W +
                         (rois.x[i] + x);
    out[o] = cast_out<TOut>(load_f32<TIn>(vol + src));
  }
}

// Four consecutive predictions as fp32 (the pointer is aligned to 4 elements).
template <typename TP>
__device__ __forceinline__ float4 load4_f32(const TP* p);
template <>
__device__ __forceinline__ float4 load4_f32<float>(const float* p) {
  return __ldg(reinterpret_cast<const float4*>(p));
}
template <>
__device__ __forceinline__ float4 load4_f32<__half>(const __half* p) {
  const uint2 w = __ldg(reinterpret_cast<const uint2*>(p));
  const float2 a = __half22float2(*reinterpret_cast<const __half2*>(&w.x));
  const float2 b = __half22float2(*reinterpret_cast<const __half2*>(&w.y));
  return make_float4(a.x, a.y, b.x, b.y);
}
template <>
__device__ __forceinline__ float4 load4_f32<__nv_bfloat16>(const __nv_bfloat16* p) {
  const uint2 w = __ldg(reinterpret_cast<const uint2*>(p));
  return make_float4(__uint_as_float(w.x << 16), __uint_as_float(w.x & 0xFFFF0000u),
                     __uint_as_float(w.y << 16), __uint_as_float(w.y & 0xFFFF0000u));
}

// Eight consecutive elements as fp32 (the pointer is aligned to 8 elements).
template <typename TP>
__device__ __forceinline__ void load8_f32(const TP* p, float (&v)[8]) {
  if constexpr (sizeof(TP) == 4) {
    const float4 a = __ldg(reinterpret_cast<const float4*>(p));
    const float4 b = __ldg(reinterpret_cast<const float4*>(p) + 1);
    v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w;
    v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
  } else {
    const float4 a = load4_f32<TP>(p), b = load4_f32<TP>(p + 4);
    v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w;
    v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
  }
}

// Eight consecutive outputs, one rounding each (16-byte aligned destination).
template <typename TOut>
__device__ __forceinline__ void store8_out(TOut* p, const float (&v)[8]) {
  if constexpr (sizeof(TOut) == 4) {
    reinterpret_cast<float4*>(p)[0] = make_float4(v[0], v[1], v[2], v[3]);
    reinterpret_cast<float4*>(p)[1] = make_float4(v[4], v[5], v[6], v[7]);
  } else {
    uint32_t w[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const TOut lo = cast_out<TOut>(v[2 * i]), hi = cast_out<TOut>(v[2 * i + 1]);
      w[i] = uint32_t(*reinterpret_cast<const uint16_t*>(&lo)) |
             (uint32_t(*reinterpret_cast<const uint16_t*>(&hi)) << 16);
    }
    *reinterpret_cast<uint4*>(p) = make_uint4(w[0], w[1], w[2], w[3]);
  }
}

// Eight consecutive x voxels of one ROI row per thread: two 16-byte volume loads
// (fp32) and one 16-byte output store (16-bit types).  Every ROI x start, the ROI
// width and the volume width are multiples of 8.
template <typename TIn, typename TOut>
__global__ void __launch_bounds__(kThreads)
roi_gather8_kernel(TOut* __restrict__ out, const TIn* __restrict__ vol, const RoiList rois,
                   uint32_t D, uint32_t H, uint32_t W, uint64_t total8, DivMod64 f_roi8,
                   DivMod32 f_rw8, DivMod32 f_rh, DivMod32 f_rd) {
  for (uint64_t o8 = uint64_t(blockIdx.x) * kThreads + threadIdx.x; o8 < total8;
       o8 += uint64_t(gridDim.x) * kThreads) {
    const uint32_t i = uint32_t(f_roi8.div(o8));  // ROI index
    const uint32_t r = uint32_t(o8 - uint64_t(i) * f_roi8.d);
    uint32_t t, x8, t2, y, c, z;
    f_rw8.divmod(r, t, x8);
    f_rh.divmod(t, t2, y);
    f_rd.divmod(t2, c, z);
    const uint64_t src = ((uint64_t(c) * D + (rois.z[i] + z)) * H + (rois.y[i] + y)) * W +
                         (rois.x[i] + 8 * x8);
    float v[8];
    load8_f32<TIn>(vol + src, v);
    store8_out<TOut>(out + 8 * o8, v);
  }
}

// One thread per (class, VX consecutive x voxels) of the batch's bounding box.  With
// VX = 4 or 8 every ROI x start, the ROI width and the box are multiples of VX, so
// the voxels share their ROI membership and move as 16-byte accumulator vectors.
template <typename TP, int VX>
__global__ void __launch_bounds__(kThreads)
roi_accumulate_kernel(float* __restrict__ acc, const TP* __restrict__ pred, const RoiList rois,
                      uint32_t classes, uint32_t H, uint32_t W, uint64_t plane, int bz0,
                      int by0, int bx0, uint32_t total, DivMod32 f_bw, DivMod32 f_bh,
                      DivMod32 f_bd) {
  const uint32_t o = blockIdx.x * kThreads + threadIdx.x;
  if (o >= total) return;
  uint32_t t, bx, t2, by, c, bz;
  f_bw.divmod(o, t, bx);
  f_bh.divmod(t, t2, by);
  f_bd.divmod(t2, c, bz);
  const int z = bz0 + int(bz), y = by0 + int(by), x = bx0 + int(bx) * VX;
  const uint32_t roi_vol = uint32_t(rois.rd) * rois.rh * rois.rw;
  float* a = acc + uint64_t(c) * plane + (uint64_t(z) * H + y) * W + x;
  float sum[VX];
  bool touched = false;
  for (int i = 0; i < rois.n; ++i) {
    const int lz = z - rois.z[i], ly = y - rois.y[i], lx = x - rois.x[i];
    if (unsigned(lz) < unsigned(rois.rd) && unsigned(ly) < unsigned(rois.rh) &&
        unsigned(lx) < unsigned(rois.rw)) {
      if (!touched) {
        if constexpr (VX >= 4) {
#pragma unroll
          for (int h = 0; h < VX; h += 4) {
            const float4 v = *reinterpret_cast<const float4*>(a + h);
            sum[h] = v.x; sum[h + 1] = v.y; sum[h + 2] = v.z; sum[h + 3] = v.w;
          }
        } else {
          sum[0] = *a;
        }
        touched = true;
      }
      const uint64_t p = (uint64_t(i) * classes + c) * roi_vol +
                         (uint32_t(lz) * rois.rh + uint32_t(ly)) * uint32_t(rois.rw) + uint32_t(lx);
      if constexpr (VX == 8) {
        float q[8];
        load8_f32<TP>(pred + p, q);
#pragma unroll
        for (int e = 0; e < 8; ++e) sum[e] += q[e];
      } else if constexpr (VX == 4) {
        const float4 q = load4_f32<TP>(pred + p);
        sum[0] += q.x; sum[1] += q.y; sum[2] += q.z; sum[3] += q.w;
      } else {
        sum[0] += load_f32<TP>(pred + p);
      }
    }
  }
  if (touched) {
    if constexpr (VX >= 4) {
#pragma unroll
      for (int h = 0; h < VX; h += 4)
        *reinterpret_cast<float4*>(a + h) = make_float4(sum[h], sum[h + 1], sum[h + 2], sum[h + 3]);
    } else {
      *a = sum[0];
    }
  }
}

// One thread per voxel: arg-max over classes of acc / count.
__global__ void __launch_bounds__(kThreads)
roi_argmax_kernel(uint8_t* __restrict__ labels, float* __restrict__ logits,
                  const float* __restrict__ acc, const float* __restrict__ cd,
                  const float* __restrict__ ch, const float* __restrict__ cw, uint32_t classes,
                  uint32_t H, uint32_t W, uint64_t plane, DivMod64 f_w, DivMod64 f_h) {
  for (uint64_t v = uint64_t(blockIdx.x) * kThreads + threadIdx.x; v < plane;
       v += uint64_t(gridDim.x) * kThreads) {
    const uint64_t t = f_w.div(v);
    const uint32_t w = uint32_t(v - t * W);
    const uint64_t d = f_h.div(t);
    const uint32_t h = uint32_t(t - d * H);
    const float cnt = __ldg(cd + d) * __ldg(ch + h) * __ldg(cw + w);
    float best = 0.f;
    uint32_t arg = 0;
    for (uint32_t c = 0; c < classes; ++c) {
      const float val = __fdiv_rn(acc[uint64_t(c) * plane + v], cnt);
      if (logits) logits[uint64_t(c) * plane + v] = val;
      // first maximum wins; a NaN is the maximum (as torch.argmax)
      if (c == 0 || (!(best != best) && (val > best || val != val))) {
        best = val;
        arg = c;
      }
    }
    if (labels) labels[v] = uint8_t(arg);
  }
}

// Four consecutive voxels per thread (W a multiple of 4): 16-byte loads of each class
// plane, four class planes in flight at a time, one 4-byte label store.  Same
// division, comparison order and tie / NaN rules as roi_argmax_kernel.
__global__ void __launch_bounds__(kThreads)
roi_argmax4_kernel(uint8_t* __restrict__ labels, float* __restrict__ logits,
                   const float* __restrict__ acc, const float* __restrict__ cd,
                   const float* __restrict__ ch, const float* __restrict__ cw, uint32_t classes,
                   uint32_t H, uint32_t W, uint64_t plane, DivMod64 f_w, DivMod64 f_h) {
  for (uint64_t q = uint64_t(blockIdx.x) * kThreads + threadIdx.x; q < plane / 4;
       q += uint64_t(gridDim.x) * kThreads) {
    const uint64_t v = 4 * q;
    const uint64_t t = f_w.div(v);
    const uint32_t w = uint32_t(v - t * W);
    const uint64_t d = f_h.div(t);
    const uint32_t h = uint32_t(t - d * H);
    const float cdh = __ldg(cd + d) * __ldg(ch + h);
    float cnt[4], best[4];
    uint32_t arg[4] = {0, 0, 0, 0};
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      cnt[e] = cdh * __ldg(cw + w + e);
      best[e] = 0.f;
    }
    for (uint32_t c0 = 0; c0 < classes; c0 += 4) {
      float4 a[4];
#pragma unroll
      for (int k = 0; k < 4; ++k)
        if (c0 + k < classes)
          a[k] = __ldg(reinterpret_cast<const float4*>(acc + uint64_t(c0 + k) * plane + v));
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        const uint32_t c = c0 + k;
        if (c >= classes) break;
        const float val[4] = {__fdiv_rn(a[k].x, cnt[0]), __fdiv_rn(a[k].y, cnt[1]),
                              __fdiv_rn(a[k].z, cnt[2]), __fdiv_rn(a[k].w, cnt[3])};
        if (logits)
          *reinterpret_cast<float4*>(logits + uint64_t(c) * plane + v) =
              make_float4(val[0], val[1], val[2], val[3]);
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          // first maximum wins; a NaN is the maximum (as torch.argmax)
          if (c == 0 || (!(best[e] != best[e]) && (val[e] > best[e] || val[e] != val[e]))) {
            best[e] = val[e];
            arg[e] = c;
          }
        }
      }
    }
    if (labels)
      *reinterpret_cast<uint32_t*>(labels + v) = arg[0] | (arg[1] << 8) | (arg[2] << 16) |
                                                  (arg[3] << 24);
  }
}

int fill_rois(RoiList& r, const int64_t* starts, int64_t n, int64_t rd, int64_t rh, int64_t rw,
              int64_t D, int64_t H, int64_t W) {
  if (n < 0 || n > kMaxRois) return set_error(kErrInvalid, "between 0 and 64 ROIs per call");
  if (rd <= 0 || rh <= 0 || rw <= 0) return set_error(kErrInvalid, "roi sizes must be positive");
  if (n > 0 && !starts) return set_error(kErrInvalid, "null ROI start list");
  r.n = int(n);
  r.rd = int(rd);
  r.rh = int(rh);
  r.rw = int(rw);
  for (int64_t i = 0; i < n; ++i) {
    const int64_t z = starts[3 * i], y = starts[3 * i + 1], x = starts[3 * i + 2];
    if (z < 0 || y < 0 || x < 0 || z + rd > D || y + rh > H || x + rw > W)
      return set_error(kErrInvalid, "ROI outside the volume");
    r.z[i] = int(z);
    r.y[i] = int(y);
    r.x[i] = int(x);
  }
  return kOk;
}

int grid_for(uint64_t total) {
  int dev = 0, sms = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const uint64_t blocks = (total + kThreads - 1) / kThreads;
  const uint64_t cap = uint64_t(sms) * 64;
  return int(blocks < cap ? blocks : cap);
}

}  // namespace

int launch_roi_gather(void* out, int out_dtype, const void* vol, int in_dtype, int64_t C,
                      int64_t D, int64_t H, int64_t W, const int64_t* starts, int64_t n,
                      int64_t rd, int64_t rh, int64_t rw, cudaStream_t stream) {
  if (C <= 0 || D <= 0 || H <= 0 || W <= 0) return set_error(kErrInvalid, "volume dims must be positive");
  if (D * H * W >= (int64_t(1) << 31)) return set_error(kErrInvalid, "volume must be below 2^31 voxels");
  RoiList r{};
  if (int e = fill_rois(r, starts, n, rd, rh, rw, D, H, W)) return e;
  if (n == 0) return kOk;
  if (!out || !vol) return set_error(kErrInvalid, "null tensor pointer");
  if (C * rd * rh * rw >= (int64_t(1) << 31)) return set_error(kErrInvalid, "ROI too large");
  const uint64_t total = uint64_t(n) * C * rd * rh * rw;
  const DivMod32 f_rw = DivMod32::make(uint32_t(rw)), f_rh = DivMod32::make(uint32_t(rh)),
                 f_rd = DivMod32::make(uint32_t(rd));
  const DivMod64 f_roi = DivMod64::make(uint64_t(C) * rd * rh * rw);
  // eight x voxels per thread when every ROI x start, the ROI width and the volume
  // width are multiples of 8 and both tensors are 16-byte aligned
  bool vec8 = (W % 8 == 0) && (rw % 8 == 0) &&
              ((reinterpret_cast<uintptr_t>(out) | reinterpret_cast<uintptr_t>(vol)) % 16 == 0);
  for (int i = 0; i < r.n && vec8; ++i) vec8 = (r.x[i] % 8 == 0);
  const int grid = grid_for(vec8 ? total / 8 : total);
  const DivMod32 f_rw8 = DivMod32::make(uint32_t(rw / 8 > 0 ? rw / 8 : 1));
  const DivMod64 f_roi8 = DivMod64::make(uint64_t(C) * rd * rh * (rw / 8 > 0 ? rw / 8 : 1));
#define CRUMPET_GATHER(TI, TO)                                                                   \
  if (vec8)                                                                                      \
    roi_gather8_kernel<TI, TO><<<grid, kThreads, 0, stream>>>(                                  \
        static_cast<TO*>(out), static_cast<const TI*>(vol), r, uint32_t(D), uint32_t(H),        \
        uint32_t(W), total / 8, f_roi8, f_rw8, f_rh, f_rd);                                      \
  else                                                                                           \
    roi_gather_kernel<TI, TO><<<grid, kThreads, 0, stream>>>(                                   \
        static_cast<TO*>(out), static_cast<const TI*>(vol), r, uint32_t(D), uint32_t(H),        \
        uint32_t(W), total, f_roi, f_rw, f_rh, f_rd)
  auto by_out = [&](auto tin) {
    using TI = decltype(tin);
    if (out_dtype == kF32) CRUMPET_GATHER(TI, float);
    else if (out_dtype == kF16) CRUMPET_GATHER(TI, __half);
    else CRUMPET_GATHER(TI, __nv_bfloat16);
  };
#undef CRUMPET_GATHER
  if (in_dtype == kF32) by_out(float{});
  else if (in_dtype == kF16) by_out(__half{});
  else by_out(__nv_bfloat16{});
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return set_cuda_error(e, "roi_gather launch");
  return kOk;
}

int launch_roi_accumulate(float* acc, const void* pred, int pred_dtype, int64_t classes,
                          int64_t D, int64_t H, int64_t W, const int64_t* starts, int64_t n,
                          int64_t rd, int64_t rh, int64_t rw, cudaStream_t stream) {
  if (classes <= 0 || D <= 0 || H <= 0 || W <= 0)
    return set_error(kErrInvalid, "classes and volume dims must be positive");
  RoiList r{};
  if (int e = fill_rois(r, starts, n, rd, rh, rw, D, H, W)) return e;
  if (n == 0) return kOk;
  if (!acc || !pred) return set_error(kErrInvalid, "null tensor pointer");
  int z0 = r.z[0], y0 = r.y[0], x0 = r.x[0], z1 = z0, y1 = y0, x1 = x0;
  for (int i = 1; i < r.n; ++i) {
    z0 = r.z[i] < z0 ? r.z[i] : z0;
    y0 = r.y[i] < y0 ? r.y[i] : y0;
    x0 = r.x[i] < x0 ? r.x[i] : x0;
    z1 = r.z[i] > z1 ? r.z[i] : z1;
    y1 = r.y[i] > y1 ? r.y[i] : y1;
    x1 = r.x[i] > x1 ? r.x[i] : x1;
  }
  const int64_t bd = z1 + rd - z0, bh = y1 + rh - y0, bw = x1 + rw - x0;
  // eight (four) voxels per thread when every x offset and width is a multiple of 8 (4)
  bool vec4 = (W % 4 == 0) && (rw % 4 == 0) && (reinterpret_cast<uintptr_t>(acc) % 16 == 0) &&
              (reinterpret_cast<uintptr_t>(pred) % (pred_dtype == kF32 ? 16 : 8) == 0);
  for (int i = 0; i < r.n && vec4; ++i) vec4 = (r.x[i] % 4 == 0);
  bool vec8 = vec4 && (W % 8 == 0) && (rw % 8 == 0) &&
              (reinterpret_cast<uintptr_t>(pred) % 16 == 0);
  for (int i = 0; i < r.n && vec8; ++i) vec8 = (r.x[i] % 8 == 0);
  const int vx = vec8 ? 8 : (vec4 ? 4 : 1);
  const uint64_t total = uint64_t(classes) * bd * bh * (bw / vx);
  if (total >= (uint64_t(1) << 31) || uint64_t(n) * classes * rd * rh * rw >= (uint64_t(1) << 40))
    return set_error(kErrInvalid, "ROI batch too large for one launch");
  const uint64_t plane = uint64_t(D) * H * W;
  const uint32_t blocks = uint32_t((total + kThreads - 1) / kThreads);
  const DivMod32 f_bw = DivMod32::make(uint32_t(bw / vx)), f_bh = DivMod32::make(uint32_t(bh)),
                 f_bd = DivMod32::make(uint32_t(bd));
  auto launch = [&](auto tp) {
    using TP = decltype(tp);
    if (vec8)
      roi_accumulate_kernel<TP, 8><<<blocks, kThreads, 0, stream>>>(
          acc, static_cast<const TP*>(pred), r, uint32_t(classes), uint32_t(H), uint32_t(W),
          plane, z0, y0, x0, uint32_t(total), f_bw, f_bh, f_bd);
    else if (vec4)
      roi_accumulate_kernel<TP, 4><<<blocks, kThreads, 0, stream>>>(
          acc, static_cast<const TP*>(pred), r, uint32_t(classes), uint32_t(H), uint32_t(W),
          plane, z0, y0, x0, uint32_t(total), f_bw, f_bh, f_bd);
    else
      roi_accumulate_kernel<TP, 1><<<blocks, kThreads, 0, stream>>>(
          acc, static_cast<const TP*>(pred), r, uint32_t(classes), uint32_t(H), uint32_t(W),
          plane, z0, y0, x0, uint32_t(total), f_bw, f_bh, f_bd);
  };
  if (pred_dtype == kF32) launch(float{});
  else if (pred_dtype == kF16) launch(__half{});
  else launch(__nv_bfloat16{});
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return set_cuda_error(e, "roi_accumulate launch");
  return kOk;
}

int launch_roi_argmax(uint8_t* labels, float* logits, const float* acc, const float* count_d,
                      const float* count_h, const float* count_w, int64_t classes, int64_t D,
                      int64_t H, int64_t W, cudaStream_t stream) {
  if (classes <= 0 || classes > 256 || D <= 0 || H <= 0 || W <= 0)
    return set_error(kErrInvalid, "1 <= classes <= 256 and positive volume dims required");
  if (!acc || !count_d || !count_h || !count_w) return set_error(kErrInvalid, "null tensor pointer");
  if (!labels && !logits) return kOk;
  const uint64_t plane = uint64_t(D) * H * W;
  // four voxels per thread when W is a multiple of 4 and the tensors are aligned for it
  const bool vec4 = (W % 4 == 0) && (reinterpret_cast<uintptr_t>(acc) % 16 == 0) &&
                    (reinterpret_cast<uintptr_t>(logits) % 16 == 0) &&
                    (reinterpret_cast<uintptr_t>(labels) % 4 == 0);
  if (vec4)
    roi_argmax4_kernel<<<grid_for(plane / 4), kThreads, 0, stream>>>(
        labels, logits, acc, count_d, count_h, count_w, uint32_t(classes), uint32_t(H),
        uint32_t(W), plane, DivMod64::make(uint64_t(W)), DivMod64::make(uint64_t(H)));
  else
    roi_argmax_kernel<<<grid_for(plane), kThreads, 0, stream>>>(
        labels, logits, acc, count_d, count_h, count_w, uint32_t(classes), uint32_t(H),
        uint32_t(W), plane, DivMod64::make(uint64_t(W)), DivMod64::make(uint64_t(H)));
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return set_cuda_error(e, "roi_argmax launch");
  return kOk;
}

}  // namespace crumpet
