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
// The kernel is a pure store stream: 16-byte stores (windows are only
// element-aligned because N*N is odd), codes in shared memory, and interior windows
// (am == 0) written as zero vectors without per-element work.
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
  DivMod32 f_N, f_ww, f_wh, f_nww, f_nwh;
  uint32_t neg;         // bit pattern of -100 in the element type
  uint32_t win_offset;  // global index of the launch's first window
};

__device__ __forceinline__ uint32_t axis_flags(const MaskGeom& g, uint32_t win) {
  uint32_t t, iw, id, ih;
  win += g.win_offset;
  g.f_nww.divmod(win, t, iw);
  g.f_nwh.divmod(t, id, ih);
  return uint32_t(g.sd != 0 && id == g.nwd - 1) | (uint32_t(g.sh != 0 && ih == g.nwh - 1) << 1) |
         (uint32_t(g.sw != 0 && iw == g.nww - 1) << 2);
}

// Grid (blocks per window, windows): block (x, w) writes part of window w's
// N*N contiguous elements.  The window's 16-byte-aligned interior is written
// with 16-byte stores, its unaligned head and tail (at most 15 bytes each, since
// N*N is odd the windows are only element-aligned) with element stores.  A window
// that is not the last one on any shifted axis is all zeros: its blocks store
// zero vectors with no per-element work.  Otherwise the token codes go to shared
// memory and every element is ((code_i ^ code_j) & flags) ? -100 : 0.
constexpr int kVecPerThread = 4;

template <int E>
__device__ __forceinline__ uint32_t mask_value(const uint8_t* codes, uint32_t am, uint32_t i,
                                               uint32_t j, uint32_t neg) {
  return ((codes[i] ^ codes[j]) & am) ? neg : 0u;
}

template <int E>
__global__ void __launch_bounds__(kThreads)
attn_mask_kernel(uint8_t* __restrict__ out, const MaskGeom g) {
  __shared__ uint8_t codes[kMaxTokens];
  const uint32_t win = blockIdx.y;
  const uint32_t am = axis_flags(g, win);  // uniform for the block
  const uint64_t wbytes = g.NN * E;
  uint8_t* wbase = out + uint64_t(win) * wbytes;
  const uintptr_t a0 = reinterpret_cast<uintptr_t>(wbase);
  uintptr_t v_begin = (a0 + 15) & ~uintptr_t(15);
  uintptr_t v_end = (a0 + wbytes) & ~uintptr_t(15);
  if (v_end <= v_begin) v_begin = v_end = a0;  // window shorter than two vectors: all scalar
  const uint32_t nvec = uint32_t((v_end - v_begin) / 16);
  const uint32_t head = uint32_t(v_begin - a0) / E;        // elements before the vectors
  const uint32_t tail_first = uint32_t((v_end - a0) / E);  // first element after them

  if (am != 0) {
    for (uint32_t t = threadIdx.x; t < g.N; t += kThreads) {
      uint32_t t2, lw, ld, lh;
      g.f_ww.divmod(t, t2, lw);
      g.f_wh.divmod(t2, ld, lh);
      codes[t] = uint8_t(uint32_t(ld >= g.wd - g.sd) | (uint32_t(lh >= g.wh - g.sh) << 1) |
                         (uint32_t(lw >= g.ww - g.sw) << 2));
    }
    __syncthreads();
  }

  // 16-byte interior
  constexpr uint32_t kElems = 16 / E;
  const uint32_t v0 = blockIdx.x * (kThreads * kVecPerThread) + threadIdx.x;
#pragma unroll
  for (int u = 0; u < kVecPerThread; ++u) {
    const uint32_t v = v0 + uint32_t(u) * kThreads;
    if (v >= nvec) break;
    uint4 val = make_uint4(0u, 0u, 0u, 0u);
    if (am != 0) {
      const uint32_t e0 = head + v * kElems;  // element index inside the window
      uint32_t i, j;
      g.f_N.divmod(e0, i, j);
      uint32_t w[4] = {0u, 0u, 0u, 0u};
#pragma unroll
      for (uint32_t k = 0; k < kElems; ++k) {
        const uint32_t bits = mask_value<E>(codes, am, i, j, g.neg);
        if constexpr (E == 4) {
          w[k] = bits;
        } else {
          w[k >> 1] |= bits << (16 * (k & 1));
        }
        if (++j == g.N) {
          j = 0;
          ++i;
        }
      }
      val = make_uint4(w[0], w[1], w[2], w[3]);
    }
    stg(reinterpret_cast<uint4*>(v_begin) + v, val);
  }

  // unaligned head and tail elements of the window (block x == 0 only)
  if (blockIdx.x == 0) {
    const uint32_t ntail = uint32_t(g.NN) - tail_first;
    const uint32_t t = threadIdx.x;
    uint32_t e = 0xffffffffu;
    if (t < head) e = t;
    else if (t - head < ntail) e = tail_first + (t - head);
    if (e != 0xffffffffu && e < uint32_t(g.NN)) {
      uint32_t bits = 0u;
      if (am != 0) {
        uint32_t i, j;
        g.f_N.divmod(e, i, j);
        bits = mask_value<E>(codes, am, i, j, g.neg);
      }
      if constexpr (E == 4) {
        stg(reinterpret_cast<uint32_t*>(wbase) + e, bits);
      } else {
        stg(reinterpret_cast<uint16_t*>(wbase) + e, uint16_t(bits));
      }
    }
  }
}

template <int E>
cudaError_t launch_e(void* out, const MaskGeom& g, uint32_t nwin, cudaStream_t stream) {
  const uint64_t nvec_max = g.NN * E / 16 + 1;
  const uint64_t per_block = uint64_t(kThreads) * kVecPerThread;
  const uint64_t bx = (nvec_max + per_block - 1) / per_block;
  // window volume <= 1024 tokens keeps bx small; windows go on grid y (<= 65535 per launch)
  for (uint32_t w0 = 0; w0 < nwin; w0 += 65535u) {
    const uint32_t nw = (nwin - w0) < 65535u ? (nwin - w0) : 65535u;
    MaskGeom gg = g;
    // launch-local window numbering: shift the base pointer and keep axis flags global
    uint8_t* base = static_cast<uint8_t*>(out) + uint64_t(w0) * g.NN * E;
    gg.win_offset = w0;
    attn_mask_kernel<E><<<dim3(unsigned(bx), nw), kThreads, 0, stream>>>(base, gg);
    const cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return e;
  }
  return cudaSuccess;
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
  g.f_N = DivMod32::make(g.N);
  g.f_ww = DivMod32::make(g.ww);
  g.f_wh = DivMod32::make(g.wh);
  g.f_nww = DivMod32::make(g.nww);
  g.f_nwh = DivMod32::make(g.nwh);
  g.neg = neg100_bits(dtype);
  if (reinterpret_cast<uintptr_t>(out) % (dtype == kF32 ? 4 : 2) != 0)
    return set_error(kErrInvalid, "mask output must be aligned to its element size");
  const uint32_t nwin = g.nwd * g.nwh * g.nww;
  const cudaError_t err = dtype == kF32 ? launch_e<4>(out, g, nwin, stream)
                                        : launch_e<2>(out, g, nwin, stream);
  if (err != cudaSuccess) return set_cuda_error(err, "attention mask launch");
  return kOk;
}

}  // namespace crumpet
