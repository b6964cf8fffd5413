// crumpet_b200: cyclic roll + 3D window partition, and its inverse.
//
// Forward  (fused_shift_partition_3d):
//   out[b*nW + win, loc, :] = x[b, (wd*ws_d + ld + ss_d) % D, (wh*ws_h + lh + ss_h) % H,
//                               (ww*ws_w + lw + ss_w) % W, :]
//   with win = (wd*nWh + wh)*nWw + ww and loc = (ld*ws_h + lh)*ws_w + lw.  This is
//   torch.roll(x, -ss, dims=(1,2,3)) followed by the Swin window partition
//   (reference: torch-ext/crumpet/reference.py:101-118 and :141-160).
// Inverse  (fused_unshift_unpartition_3d):
//   out[b, d, h, w, :] = windows[b*nW + win(p), loc(p), :] with
//   p = ((d - ss_d) mod D, (h - ss_h) mod H, (w - ss_w) mod W)
//   (reference: torch-ext/crumpet/reference.py:121-138 and :163-184).
//
// Both are pure permutation copies.  One thread moves U vectors of VB bytes;
// the vector index runs linearly over the OUTPUT, so every warp writes 32
// consecutive vectors and reads consecutive vectors of the same token row
// (a token row is C*sizeof(T) contiguous bytes on both sides).  All window
// index arithmetic is done in registers with multiply-high division.
#include "common.cuh"
#include "kernels.h"

namespace crumpet {

namespace {

constexpr int kThreads = 256;

struct PartGeom {
  uint32_t D, H, W;
  uint32_t wd, wh, ww;
  uint32_t sd, sh, sw;
  uint32_t nwd, nwh, nww, nw, N, cv;
  DivMod32 f_cv, f_N, f_nw, f_nww, f_nwh, f_ww, f_wh;  // output = windows
  DivMod32 f_W, f_H, f_D, f_wd;                         // output = volume
};

template <int VB, int U>
__global__ void __launch_bounds__(kThreads)
shift_partition_kernel(typename VecT<VB>::type* __restrict__ out,
                       const typename VecT<VB>::type* __restrict__ x,
                       const PartGeom g, const uint32_t total) {
  using V = typename VecT<VB>::type;
  const uint32_t base = blockIdx.x * (uint32_t(kThreads) * U) + threadIdx.x;
  V vals[U];
#pragma unroll
  for (int u = 0; u < U; ++u) {
    const uint32_t o = base + uint32_t(u) * kThreads;
    if (o < total) {
      uint32_t p, v, bw, loc, b, win, t, iw, id, ih, t2, lw, ld, lh;
      g.f_cv.divmod(o, p, v);
      g.f_N.divmod(p, bw, loc);
      g.f_nw.divmod(bw, b, win);
      g.f_nww.divmod(win, t, iw);
      g.f_nwh.divmod(t, id, ih);
      g.f_ww.divmod(loc, t2, lw);
      g.f_wh.divmod(t2, ld, lh);
      uint32_t sd = id * g.wd + ld + g.sd;
      uint32_t sh = ih * g.wh + lh + g.sh;
      uint32_t sw = iw * g.ww + lw + g.sw;
      sd -= (sd >= g.D) ? g.D : 0u;
      sh -= (sh >= g.H) ? g.H : 0u;
      sw -= (sw >= g.W) ? g.W : 0u;
      const uint32_t src = (((b * g.D + sd) * g.H + sh) * g.W + sw) * g.cv + v;
      vals[u] = ldg_stream(x + src);
    }
  }
#pragma unroll
  for (int u = 0; u < U; ++u) {
    const uint32_t o = base + uint32_t(u) * kThreads;
    if (o < total) stg(out + o, vals[u]);
  }
}

template <int VB, int U>
__global__ void __launch_bounds__(kThreads)
unshift_unpartition_kernel(typename VecT<VB>::type* __restrict__ out,
                           const typename VecT<VB>::type* __restrict__ windows,
                           const PartGeom g, const uint32_t total) {
  using V = typename VecT<VB>::type;
  const uint32_t base = blockIdx.x * (uint32_t(kThreads) * U) + threadIdx.x;
  V vals[U];
#pragma unroll
  for (int u = 0; u < U; ++u) {
    const uint32_t o = base + uint32_t(u) * kThreads;
    if (o < total) {
      uint32_t p, v, t, w, t2, h, b, d, id, ld, ih, lh, iw, lw;
      g.f_cv.divmod(o, p, v);
      g.f_W.divmod(p, t, w);
      g.f_H.divmod(t, t2, h);
      g.f_D.divmod(t2, b, d);
      // position in the rolled frame: roll(+ss) reads index (i - ss) mod dim
      d = (d >= g.sd) ? d - g.sd : d + g.D - g.sd;
      h = (h >= g.sh) ? h - g.sh : h + g.H - g.sh;
      w = (w >= g.sw) ? w - g.sw : w + g.W - g.sw;
      g.f_wd.divmod(d, id, ld);
      g.f_wh.divmod(h, ih, lh);
      g.f_ww.divmod(w, iw, lw);
      const uint32_t win = (id * g.nwh + ih) * g.nww + iw;
      const uint32_t loc = (ld * g.wh + lh) * g.ww + lw;
      const uint32_t src = ((b * g.nw + win) * g.N + loc) * g.cv + v;
      vals[u] = ldg_stream(windows + src);
    }
  }
#pragma unroll
  for (int u = 0; u < U; ++u) {
    const uint32_t o = base + uint32_t(u) * kThreads;
    if (o < total) stg(out + o, vals[u]);
  }
}

// Widest vector (16/8/4/2 bytes) that divides a token row and both pointers.
int pick_vector_bytes(int64_t row_bytes, const void* a, const void* b) {
  const uintptr_t mis = reinterpret_cast<uintptr_t>(a) | reinterpret_cast<uintptr_t>(b);
  for (int vb = 16; vb >= 2; vb /= 2) {
    if (row_bytes % vb == 0 && (mis % vb) == 0) return vb;
  }
  return 0;
}

PartGeom make_geom(const ShapeArgs& s, int vb, int64_t row_bytes) {
  PartGeom g{};
  g.D = uint32_t(s.D);
  g.H = uint32_t(s.H);
  g.W = uint32_t(s.W);
  g.wd = uint32_t(s.ws_d);
  g.wh = uint32_t(s.ws_h);
  g.ww = uint32_t(s.ws_w);
  g.sd = uint32_t(s.ss_d);
  g.sh = uint32_t(s.ss_h);
  g.sw = uint32_t(s.ss_w);
  g.nwd = g.D / g.wd;
  g.nwh = g.H / g.wh;
  g.nww = g.W / g.ww;
  g.nw = g.nwd * g.nwh * g.nww;
  g.N = g.wd * g.wh * g.ww;
  g.cv = uint32_t(row_bytes / vb);
  g.f_cv = DivMod32::make(g.cv);
  g.f_N = DivMod32::make(g.N);
  g.f_nw = DivMod32::make(g.nw);
  g.f_nww = DivMod32::make(g.nww);
  g.f_nwh = DivMod32::make(g.nwh);
  g.f_ww = DivMod32::make(g.ww);
  g.f_wh = DivMod32::make(g.wh);
  g.f_W = DivMod32::make(g.W);
  g.f_H = DivMod32::make(g.H);
  g.f_D = DivMod32::make(g.D);
  g.f_wd = DivMod32::make(g.wd);
  return g;
}

template <int VB>
cudaError_t launch_vb(bool forward, void* out, const void* in, const PartGeom& g,
                      uint32_t total, cudaStream_t stream) {
  constexpr int U = VB == 16 ? 4 : 8;
  using V = typename VecT<VB>::type;
  const uint32_t per_block = uint32_t(kThreads) * U;
  const uint32_t blocks = (total + per_block - 1) / per_block;
  if (forward) {
    shift_partition_kernel<VB, U><<<blocks, kThreads, 0, stream>>>(
        static_cast<V*>(out), static_cast<const V*>(in), g, total);
  } else {
    unshift_unpartition_kernel<VB, U><<<blocks, kThreads, 0, stream>>>(
        static_cast<V*>(out), static_cast<const V*>(in), g, total);
  }
  return cudaGetLastError();
}

}  // namespace

// forward == true : x [B,D,H,W,C] -> windows [B*nW, N, C]
// forward == false: windows [B*nW, N, C] -> x [B,D,H,W,C]
int launch_window_copy(bool forward, void* out, const void* in, const ShapeArgs& s,
                       int dtype, cudaStream_t stream) {
  const int64_t esize = dtype_size(dtype);
  const int64_t row_bytes = s.C * esize;
  const int vb = pick_vector_bytes(row_bytes, out, in);
  if (vb == 0) return set_error(kErrInvalid, "pointers must be aligned to the element size");
  const PartGeom g = make_geom(s, vb, row_bytes);
  const int64_t vec_per_batch = s.D * s.H * s.W * (row_bytes / vb);
  // Each launch indexes at most 2^31 - 1 vectors with 32-bit arithmetic;
  // larger tensors are processed in slices of whole batch entries.
  const int64_t kMaxVec = (int64_t(1) << 31) - 1 - int64_t(kThreads) * 8;
  if (vec_per_batch > kMaxVec) return set_error(kErrInvalid, "a single batch entry exceeds 2^31 vectors");
  const int64_t batch_step = kMaxVec / vec_per_batch;
  const int64_t bytes_per_batch = vec_per_batch * vb;
  for (int64_t b0 = 0; b0 < s.B; b0 += batch_step) {
    const int64_t nb = (s.B - b0) < batch_step ? (s.B - b0) : batch_step;
    const uint32_t total = uint32_t(nb * vec_per_batch);
    char* o = static_cast<char*>(out) + b0 * bytes_per_batch;
    const char* i = static_cast<const char*>(in) + b0 * bytes_per_batch;
    cudaError_t err;
    switch (vb) {
      case 16: err = launch_vb<16>(forward, o, i, g, total, stream); break;
      case 8: err = launch_vb<8>(forward, o, i, g, total, stream); break;
      case 4: err = launch_vb<4>(forward, o, i, g, total, stream); break;
      default: err = launch_vb<2>(forward, o, i, g, total, stream); break;
    }
    if (err != cudaSuccess) return set_cuda_error(err, "window copy launch");
  }
  return kOk;
}

}  // namespace crumpet
