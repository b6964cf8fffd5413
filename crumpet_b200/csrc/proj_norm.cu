// crumpet_b200: LayerNorm over the channels of a channels-first volume, written
// channels-last -- the hidden-state normalisation of the Swin trunk.
//
// MONAI's SwinTransformer.proj_out(x, normalize=True) turns every stage output
// x [B, C, D, H, W] (channels-first, contiguous) into
//   rearrange(F.layer_norm(rearrange(x, "n c d h w -> n d h w c"), [C]), back)
// i.e. out[b, d, h, w, :] = LN(x[b, :, d, h, w]) stored channels-last and
// returned as the [B, C, D, H, W] view of that storage.  Under fp16 autocast the
// norm runs in fp32 (input cast, contiguous copy, fp32 LayerNorm): three passes
// over the volume, and torch's LayerNorm kernel is latency-bound at C = 48.
//
// One kernel here: a CTA takes T consecutive voxels of one batch entry, reads
// the C channel planes of those voxels with coalesced loads (the voxels are
// contiguous inside each plane) into a token-major shared tile [T][C + 1] (odd
// row stride: the plane-wise writes and the token-wise reads hit distinct
// banks), normalises each token with P threads of one warp (24 channels per
// thread, two passes in registers, shuffle reductions), and writes the tile's
// T x C output elements -- contiguous in the channels-last result -- with
// coalesced stores.  T * P = 256, P the smallest power of two with 24 P >= C,
// so the tile is ~25 KB for every C up to 768.
#include "common.cuh"
#include "kernels.h"

namespace crumpet {

namespace {

constexpr int kPnThreads = 256;
constexpr int kPnVals = 24;                    // channels per thread in the norm phase
constexpr int kPnMaxC = 32 * kPnVals;          // P <= 32: C <= 768

struct ProjNormGeom {
  uint32_t C;       // channels
  uint32_t S;       // voxels per batch entry (D*H*W)
  uint32_t nv;      // C / P
  uint32_t tiles;   // batch entries of this launch x tiles per entry
  DivMod32 f_tpb;   // tiles per batch entry
  DivMod32 f_C;
  float inv_c;
  float eps;
  int affine;
};

template <typename T>
__device__ __forceinline__ float load_scalar(const T* p);
template <>
__device__ __forceinline__ float load_scalar<float>(const float* p) {
  return __uint_as_float(ldg_stream(reinterpret_cast<const uint32_t*>(p)));
}
template <>
__device__ __forceinline__ float load_scalar<__half>(const __half* p) {
  const uint16_t h = ldg_stream(reinterpret_cast<const uint16_t*>(p));
  return __half2float(__ushort_as_half(h));
}
template <>
__device__ __forceinline__ float load_scalar<__nv_bfloat16>(const __nv_bfloat16* p) {
  const uint16_t h = ldg_stream(reinterpret_cast<const uint16_t*>(p));
  return __uint_as_float(uint32_t(h) << 16);
}

template <typename T>
__device__ __forceinline__ uint32_t pack_pair(float a, float b);
template <>
__device__ __forceinline__ uint32_t pack_pair<__half>(float a, float b) {
  const __half2 h = __floats2half2_rn(a, b);
  return *reinterpret_cast<const uint32_t*>(&h);
}
template <>
__device__ __forceinline__ uint32_t pack_pair<__nv_bfloat16>(float a, float b) {
  const __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
  return *reinterpret_cast<const uint32_t*>(&h);
}

template <int P>
__device__ __forceinline__ float lane_group_sum(float v) {
#pragma unroll
  for (int off = P / 2; off > 0; off >>= 1) v += __shfl_xor_sync(0xffffffffu, v, off);
  return v;
}

template <typename TIn, typename TOut, int P>
__global__ void __launch_bounds__(kPnThreads)
    proj_out_norm_kernel(TOut* __restrict__ out, const TIn* __restrict__ x,
                         const float* __restrict__ gamma, const float* __restrict__ beta,
                         ProjNormGeom g) {
  constexpr uint32_t T = kPnThreads / P;
  extern __shared__ float tile[];  // [T][C + 1]
  const uint32_t stride = g.C + 1;
  const uint32_t tid = threadIdx.x;

  for (uint32_t t = blockIdx.x; t < g.tiles; t += gridDim.x) {
    uint32_t b, tb;
    g.f_tpb.divmod(t, b, tb);
    const uint32_t t0 = tb * T;
    const uint32_t n = min(T, g.S - t0);

    // 1. channel planes -> registers: thread (voxel tid % T, channel group tid / T)
    //    loads channels cg, cg + P, ... of its voxel; a warp reads consecutive voxels
    //    of one plane.
    float v[kPnVals];
    {
      const uint32_t tok = tid % T, cg = tid / T;
      const TIn* src = x + uint64_t(b) * g.C * g.S + uint64_t(cg) * g.S + t0 + tok;
#pragma unroll
      for (int k = 0; k < kPnVals; ++k)
        v[k] = (uint32_t(k) < g.nv && tok < n) ? load_scalar(src + uint64_t(k) * P * g.S) : 0.f;
      __syncthreads();  // the previous tile's output pass has finished reading
#pragma unroll
      for (int k = 0; k < kPnVals; ++k)
        if (uint32_t(k) < g.nv) tile[tok * stride + cg + uint32_t(k) * P] = v[k];
    }
    __syncthreads();

    // 2. per-token LayerNorm: P lanes of one warp per token, channels part + P j.
    {
      const uint32_t tok = tid / P, part = tid % P;
      float* row = tile + tok * stride + part;
      float s = 0.f;
#pragma unroll
      for (int j = 0; j < kPnVals; ++j) {
        v[j] = uint32_t(j) < g.nv ? row[j * P] : 0.f;
        s += v[j];
      }
      const float mean = lane_group_sum<P>(s) * g.inv_c;
      float sq = 0.f;
#pragma unroll
      for (int j = 0; j < kPnVals; ++j) {
        if (uint32_t(j) < g.nv) {
          const float d = v[j] - mean;
          sq = fmaf(d, d, sq);
        }
      }
      const float rstd = rsqrtf(lane_group_sum<P>(sq) * g.inv_c + g.eps);
#pragma unroll
      for (int j = 0; j < kPnVals; ++j) {
        if (uint32_t(j) < g.nv) {
          float y = (v[j] - mean) * rstd;
          if (g.affine) {
            const uint32_t c = part + uint32_t(j) * P;
            y = fmaf(y, __ldg(gamma + c), __ldg(beta + c));
          }
          row[j * P] = y;
        }
      }
    }
    __syncthreads();

    // 3. the tile's n x C output elements are contiguous channels-last: linear
    //    coalesced stores, one element (fp32) or one pair (16-bit types) per thread.
    TOut* dst = out + (uint64_t(b) * g.S + t0) * g.C;
    if constexpr (sizeof(TOut) == 4) {
      const uint32_t total = n * g.C;
      for (uint32_t i = tid; i < total; i += kPnThreads) {
        uint32_t tok, c;
        g.f_C.divmod(i, tok, c);
        stg(reinterpret_cast<uint32_t*>(dst) + i, __float_as_uint(tile[tok * stride + c]));
      }
    } else {
      const uint32_t pairs = n * g.C / 2;
      for (uint32_t i = tid; i < pairs; i += kPnThreads) {
        uint32_t tok, c;
        g.f_C.divmod(2 * i, tok, c);
        const float* r = tile + tok * stride + c;
        stg(reinterpret_cast<uint32_t*>(dst) + i, pack_pair<TOut>(r[0], r[1]));
      }
    }
  }
}

template <typename TIn, typename TOut>
cudaError_t launch_pn_t(int P, void* out, const void* x, const float* gamma, const float* beta,
                        const ProjNormGeom& g, cudaStream_t stream) {
  const uint32_t T = kPnThreads / P;
  const size_t smem = size_t(T) * (g.C + 1) * sizeof(float);
  auto o = static_cast<TOut*>(out);
  auto xi = static_cast<const TIn*>(x);
  const uint32_t blocks = g.tiles;
  switch (P) {
    case 1: proj_out_norm_kernel<TIn, TOut, 1><<<blocks, kPnThreads, smem, stream>>>(o, xi, gamma, beta, g); break;
    case 2: proj_out_norm_kernel<TIn, TOut, 2><<<blocks, kPnThreads, smem, stream>>>(o, xi, gamma, beta, g); break;
    case 4: proj_out_norm_kernel<TIn, TOut, 4><<<blocks, kPnThreads, smem, stream>>>(o, xi, gamma, beta, g); break;
    case 8: proj_out_norm_kernel<TIn, TOut, 8><<<blocks, kPnThreads, smem, stream>>>(o, xi, gamma, beta, g); break;
    case 16: proj_out_norm_kernel<TIn, TOut, 16><<<blocks, kPnThreads, smem, stream>>>(o, xi, gamma, beta, g); break;
    default: proj_out_norm_kernel<TIn, TOut, 32><<<blocks, kPnThreads, smem, stream>>>(o, xi, gamma, beta, g); break;
  }
  return cudaGetLastError();
}

template <typename TIn>
cudaError_t launch_pn_out(int out_dtype, int P, void* out, const void* x, const float* gamma,
                          const float* beta, const ProjNormGeom& g, cudaStream_t stream) {
  if (out_dtype == kF32) return launch_pn_t<TIn, float>(P, out, x, gamma, beta, g, stream);
  if (out_dtype == kF16) return launch_pn_t<TIn, __half>(P, out, x, gamma, beta, g, stream);
  return launch_pn_t<TIn, __nv_bfloat16>(P, out, x, gamma, beta, g, stream);
}

}  // namespace

int proj_out_norm_lanes(int64_t C) {
  if (C <= 0 || C > kPnMaxC || C % 8 != 0) return 0;
  int P = 1;
  while (int64_t(P) * kPnVals < C) P *= 2;
  return C % P == 0 ? P : 0;
}

int launch_proj_out_norm(void* out, int out_dtype, const void* x, int in_dtype,
                         const float* gamma, const float* beta, float eps, int64_t B, int64_t C,
                         int64_t D, int64_t H, int64_t W, cudaStream_t stream) {
  if (B < 0 || D <= 0 || H <= 0 || W <= 0) return set_error(kErrInvalid, "bad volume dims");
  const int P = proj_out_norm_lanes(C);
  if (P == 0)
    return set_error(kErrUnsupported,
                     "proj_out_norm_3d needs C a multiple of 8, at most 768, and divisible by "
                     "the lanes per voxel (C / 24 rounded up to a power of two)");
  const int64_t S = D * H * W;
  if (S >= (int64_t(1) << 31)) return set_error(kErrInvalid, "D*H*W must be below 2^31");
  if ((gamma == nullptr) != (beta == nullptr))
    return set_error(kErrInvalid, "weight and bias must both be given or both be null");
  if (B == 0) return kOk;
  if (!out || !x) return set_error(kErrInvalid, "null tensor pointer");
  if ((reinterpret_cast<uintptr_t>(out) | reinterpret_cast<uintptr_t>(x) |
       reinterpret_cast<uintptr_t>(gamma) | reinterpret_cast<uintptr_t>(beta)) & 15u)
    return set_error(kErrInvalid, "tensors must be 16-byte aligned");
  ProjNormGeom g{};
  g.C = uint32_t(C);
  g.S = uint32_t(S);
  g.nv = uint32_t(C / P);
  const uint32_t T = kPnThreads / P;
  const uint32_t tpb = uint32_t((S + T - 1) / T);
  g.f_tpb = DivMod32::make(tpb);
  g.f_C = DivMod32::make(g.C);
  g.inv_c = 1.0f / float(C);
  g.eps = eps;
  g.affine = gamma != nullptr;
  // one tile per CTA; split the batch so the tile count stays a 32-bit grid size
  const int64_t bmax = ((int64_t(1) << 31) - 1) / tpb;
  const int64_t in_sz = dtype_size(in_dtype), out_sz = dtype_size(out_dtype);
  for (int64_t b0 = 0; b0 < B; b0 += bmax) {
    const int64_t nb = B - b0 < bmax ? B - b0 : bmax;
    g.tiles = uint32_t(nb * tpb);
    const void* xs = static_cast<const uint8_t*>(x) + uint64_t(b0) * C * S * in_sz;
    void* os = static_cast<uint8_t*>(out) + uint64_t(b0) * C * S * out_sz;
    cudaError_t err;
    if (in_dtype == kF32)
      err = launch_pn_out<float>(out_dtype, P, os, xs, gamma, beta, g, stream);
    else if (in_dtype == kF16)
      err = launch_pn_out<__half>(out_dtype, P, os, xs, gamma, beta, g, stream);
    else
      err = launch_pn_out<__nv_bfloat16>(out_dtype, P, os, xs, gamma, beta, g, stream);
    if (err != cudaSuccess) return set_cuda_error(err, "proj_out_norm launch");
  }
  return kOk;
}

}  // namespace crumpet
