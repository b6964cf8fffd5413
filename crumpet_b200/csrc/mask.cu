// crumpet_b200: shifted-window attention mask [nW, N, N].
//
// Reference semantics (torch-ext/crumpet/reference.py:50-98, cuda/attn_mask_3d.cu:42-50):
// every voxel gets a region label 9*r(d) + 3*r(h) + r(w) with
//   r(x) = 0 if x < dim - ws, 1 if x < dim - ss, else 2,
// and mask[win, i, j] = -100 when tokens i and j of window `win` carry different
// labels, else 0.  All zeros when every shift is zero.
//
// Closed form used here.  Because dim is a multiple of ws, region 0 covers every
// window but the last along an axis, and the last window only holds regions 1 and
// 2, split at local coordinate ws - ss.  So labels differ exactly when, on some
// axis where the window is the last one (and ss > 0), the two tokens sit on
// different sides of ws - ss.  With a 3-bit side code per token
//   code(t) = [ld >= ws_d-ss_d] | [lh >= ws_h-ss_h] << 1 | [lw >= ws_w-ss_w] << 2
// and a 3-bit "last window on this axis" flag am(win), the entry is
//   ((code(i) ^ code(j)) & am(win)) ? -100 : 0.
// The kernel is a pure store stream: 16-byte stores over the flat output
// (windows are only element-aligned because N*N is odd), codes in shared memory,
// and interior windows (am == 0) written as zero vectors without per-element work.
#include "common.cuh"
#include "kernels.h"

namespace crumpet {

namespace {

constexpr int kThreads = 256;
constexpr int kMaxTokens = 1024;

struct MaskGeom {
  uint32_t N;
  uint32_t wd, wh, ww, sd, sh, sw;
  uint32_t nwd, nwh, nww;
  uint64_t NN;
  uint64_t total;  // nW * N * N elements
  DivMod64 f_NN;
  DivMod32 f_N, f_ww, f_wh, f_nww, f_nwh;
  uint32_t neg;    // bit pattern of -100 in the element type
};

__device__ __forceinline__ uint32_t axis_flags(const MaskGeom& g, uint32_t win) {
  uint32_t t, iw, id, ih;
  g.f_nww.divmod(win, t, iw);
  g.f_nwh.divmod(t, id, ih);
  return uint32_t(g.sd != 0 && id == g.nwd - 1) | (uint32_t(g.sh != 0 && ih == g.nwh - 1) << 1) |
         (uint32_t(g.sw != 0 && iw == g.nww - 1) << 2);
}

// E: element bytes (2 or 4); V: elements per store (16/E, or 1 for unaligned output).
template <int E, int V>
__global__ void __launch_bounds__(kThreads)
attn_mask_kernel(uint8_t* __restrict__ out, const MaskGeom g) {
  __shared__ uint8_t codes[kMaxTokens];
  for (uint32_t t = threadIdx.x; t < g.N; t += kThreads) {
    uint32_t t2, lw, ld, lh;
    g.f_ww.divmod(t, t2, lw);
    g.f_wh.divmod(t2, ld, lh);
    codes[t] = uint8_t(uint32_t(ld >= g.wd - g.sd) | (uint32_t(lh >= g.wh - g.sh) << 1) |
                       (uint32_t(lw >= g.ww - g.sw) << 2));
  }
  __syncthreads();

  const uint64_t nchunks = g.total / V;
  const uint64_t stride = uint64_t(gridDim.x) * kThreads;
  for (uint64_t c = uint64_t(blockIdx.x) * kThreads + threadIdx.x; c < nchunks; c += stride) {
    const uint64_t e0 = c * V;
    uint32_t win = uint32_t(g.f_NN.div(e0));
    uint32_t rem = uint32_t(e0 - uint64_t(win) * g.NN);
    uint32_t am = axis_flags(g, win);
    const bool spans = uint64_t(rem) + V > g.NN;
    const uint32_t am_all = spans ? (am | axis_flags(g, win + 1)) : am;
    uint32_t packed[V * E / 4 > 0 ? V * E / 4 : 1];
#pragma unroll
    for (int k = 0; k < (V * E / 4 > 0 ? V * E / 4 : 1); ++k) packed[k] = 0u;
    if (am_all != 0) {
      uint32_t i, j;
      g.f_N.divmod(rem, i, j);
      uint32_t ci = codes[i];
#pragma unroll
      for (int k = 0; k < V; ++k) {
        const bool neg = ((ci ^ codes[j]) & am) != 0;
        if (neg) {
          if constexpr (E == 4) {
            packed[k] = g.neg;
          } else if constexpr (V > 1) {
            packed[k >> 1] |= g.neg << (16 * (k & 1));
          } else {
            packed[0] = g.neg;
          }
        }
        if (++j == g.N) {
          j = 0;
          if (++i == g.N) {
            i = 0;
            ++win;
            am = axis_flags(g, win);
          }
          ci = codes[i];
        }
      }
    }
    uint8_t* dst = out + e0 * E;
    if constexpr (V * E == 16) {
      stg(reinterpret_cast<uint4*>(dst), make_uint4(packed[0], packed[1], packed[2], packed[3]));
    } else if constexpr (E == 4) {
      stg(reinterpret_cast<uint32_t*>(dst), packed[0]);
    } else {
      stg(reinterpret_cast<uint16_t*>(dst), uint16_t(packed[0]));
    }
  }

  // Ragged tail (total not a multiple of V): one element per thread of block 0.
  if constexpr (V > 1) {
    const uint64_t tail0 = nchunks * V;
    if (blockIdx.x == 0 && tail0 + threadIdx.x < g.total) {
      const uint64_t e = tail0 + threadIdx.x;
      const uint32_t win = uint32_t(g.f_NN.div(e));
      const uint32_t rem = uint32_t(e - uint64_t(win) * g.NN);
      uint32_t i, j;
      g.f_N.divmod(rem, i, j);
      const bool neg = ((codes[i] ^ codes[j]) & axis_flags(g, win)) != 0;
      uint8_t* dst = out + e * E;
      if constexpr (E == 4) {
        stg(reinterpret_cast<uint32_t*>(dst), neg ? g.neg : 0u);
      } else {
        stg(reinterpret_cast<uint16_t*>(dst), uint16_t(neg ? g.neg : 0u));
      }
    }
  }
}

template <int E, int V>
cudaError_t launch_ev(void* out, const MaskGeom& g, cudaStream_t stream) {
  int dev = 0, sms = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const uint64_t nchunks = g.total / V;
  uint64_t blocks = (nchunks + kThreads - 1) / kThreads;
  const uint64_t cap = uint64_t(sms) * 16;
  if (blocks > cap) blocks = cap;
  if (blocks == 0) blocks = 1;
  attn_mask_kernel<E, V><<<unsigned(blocks), kThreads, 0, stream>>>(static_cast<uint8_t*>(out), g);
  return cudaGetLastError();
}

}  // namespace

int launch_attn_mask(void* out, int64_t D, int64_t H, int64_t W, int64_t ws_d, int64_t ws_h,
                     int64_t ws_w, int64_t ss_d, int64_t ss_h, int64_t ss_w, int dtype,
                     cudaStream_t stream) {
  MaskGeom g{};
  g.wd = uint32_t(ws_d);
  g.wh = uint32_t(ws_h);
  g.ww = uint32_t(ws_w);
  g.sd = uint32_t(ss_d);
  g.sh = uint32_t(ss_h);
  g.sw = uint32_t(ss_w);
  g.N = g.wd * g.wh * g.ww;
  if (g.N > uint32_t(kMaxTokens))
    return set_error(kErrInvalid, "compute_attn_mask_3d supports window volumes up to 1024");
  g.nwd = uint32_t(D / ws_d);
  g.nwh = uint32_t(H / ws_h);
  g.nww = uint32_t(W / ws_w);
  g.NN = uint64_t(g.N) * g.N;
  g.total = uint64_t(g.nwd) * g.nwh * g.nww * g.NN;
  if (g.total == 0) return kOk;
  g.f_NN = DivMod64::make(g.NN);
  g.f_N = DivMod32::make(g.N);
  g.f_ww = DivMod32::make(g.ww);
  g.f_wh = DivMod32::make(g.wh);
  g.f_nww = DivMod32::make(g.nww);
  g.f_nwh = DivMod32::make(g.nwh);
  g.neg = neg100_bits(dtype);
  const bool aligned = (reinterpret_cast<uintptr_t>(out) % 16) == 0;
  cudaError_t err;
  if (dtype == kF32) {
    err = aligned ? launch_ev<4, 4>(out, g, stream) : launch_ev<4, 1>(out, g, stream);
  } else {
    err = aligned ? launch_ev<2, 8>(out, g, stream) : launch_ev<2, 1>(out, g, stream);
  }
  if (err != cudaSuccess) return set_cuda_error(err, "attention mask launch");
  return kOk;
}

}  // namespace crumpet
