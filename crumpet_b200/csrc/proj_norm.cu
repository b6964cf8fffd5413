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
//
// Two variants of that scheme:
// * proj_out_norm_pipelined_kernel (the common case: every channel plane row of a
//   tile starts on a 16-byte boundary, i.e. D*H*W*sizeof(in) % 16 == 0): a
//   persistent CTA streams its tiles through a 3-stage shared ring with
//   cp.async 16-byte copies, so the next two tiles' channel rows are in flight
//   while the current tile is normalised and stored;
// * proj_out_norm_kernel (any shape): one tile per CTA, the planes read with
//   scalar loads into registers.
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
  DivMod32 f_CE;    // C / outputs per 16-byte store (pipelined variant)
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

template <typename T>
__device__ __forceinline__ float smem_to_float(const uint8_t* p);
template <>
__device__ __forceinline__ float smem_to_float<float>(const uint8_t* p) {
  return *reinterpret_cast<const float*>(p);
}
template <>
__device__ __forceinline__ float smem_to_float<__half>(const uint8_t* p) {
  return __half2float(*reinterpret_cast<const __half*>(p));
}
template <>
__device__ __forceinline__ float smem_to_float<__nv_bfloat16>(const uint8_t* p) {
  return __uint_as_float(uint32_t(*reinterpret_cast<const uint16_t*>(p)) << 16);
}

// 16-byte global -> shared copy (cp.async.cg: bypasses L1); bytes past
// `src_bytes` (0 or 16 here) are zero-filled and not read.
__device__ __forceinline__ void cp_async16(void* smem, const void* gmem, uint32_t src_bytes) {
  const uint32_t s = static_cast<uint32_t>(__cvta_generic_to_shared(smem));
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(s), "l"(gmem), "r"(src_bytes)
               : "memory");
}
__device__ __forceinline__ void cp_async_commit() {
  asm volatile("cp.async.commit_group;" ::: "memory");
}
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

template <int P>
__device__ __forceinline__ float lane_group_sum(float v) {
#pragma unroll
  for (int off = P / 2; off > 0; off >>= 1) v += __shfl_xor_sync(0xffffffffu, v, off);
  return v;
}

// Per-token LayerNorm of one tile: thread (token tid / P, part tid % P) takes
// channels part + P j from `value(c, token)`, writes the normalised values to
// the token-major fp32 tile [T][C + 1].
template <int P, typename ValueFn>
__device__ __forceinline__ void norm_tile(const ProjNormGeom& g, const float* __restrict__ gamma,
                                          const float* __restrict__ beta, float* tile,
                                          uint32_t stride, ValueFn value) {
  const uint32_t tok = threadIdx.x / P, part = threadIdx.x % P;
  float v[kPnVals];
  float s = 0.f;
#pragma unroll
  for (int j = 0; j < kPnVals; ++j) {
    v[j] = uint32_t(j) < g.nv ? value(part + uint32_t(j) * P, tok) : 0.f;
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
  float* row = tile + tok * stride + part;
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

// The tile's n x C outputs are contiguous channels-last: linear coalesced
// stores, one element (fp32) or one pair (16-bit types) per thread.
template <typename TOut>
__device__ __forceinline__ void store_tile(const ProjNormGeom& g, TOut* dst, const float* tile,
                                           uint32_t stride, uint32_t n) {
  if constexpr (sizeof(TOut) == 4) {
    const uint32_t total = n * g.C;
    for (uint32_t i = threadIdx.x; i < total; i += kPnThreads) {
      uint32_t tok, c;
      g.f_C.divmod(i, tok, c);
      stg(reinterpret_cast<uint32_t*>(dst) + i, __float_as_uint(tile[tok * stride + c]));
    }
  } else {
    const uint32_t pairs = n * g.C / 2;
    for (uint32_t i = threadIdx.x; i < pairs; i += kPnThreads) {
      uint32_t tok, c;
      g.f_C.divmod(2 * i, tok, c);
      const float* r = tile + tok * stride + c;
      stg(reinterpret_cast<uint32_t*>(dst) + i, pack_pair<TOut>(r[0], r[1]));
    }
  }
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

    // channel planes -> registers -> token-major tile: thread (voxel tid % T,
    // channel group tid / T) loads channels cg, cg + P, ... of its voxel; a warp
    // reads consecutive voxels of one plane.
    {
      float v[kPnVals];
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
    norm_tile<P>(g, gamma, beta, tile, stride,
                 [&](uint32_t c, uint32_t tok) { return tile[tok * stride + c]; });
    __syncthreads();
    store_tile<TOut>(g, out + (uint64_t(b) * g.S + t0) * g.C, tile, stride, n);
  }
}

// Pipelined variant: 128-thread CTAs, one voxel per thread up to C = 48 (P lanes
// per voxel above, 48 channels each), the tile's channel rows streamed into a
// 3-stage shared ring with 16-byte cp.async copies (the next two tiles are in
// flight while this one is normalised and stored), normalised values staged
// token-major with 16-byte shared stores, and the tile's contiguous T x C outputs
// written with 16-byte global stores.  ~66 KB of shared memory per CTA (fp16 in,
// fp32 out): three CTAs per SM, six tiles in flight.
constexpr int kPipeThreads = 128;
constexpr int kPipeVals = 48;
constexpr int kPipeStages = 3;

template <typename TIn, typename TOut, int P>
struct PipeCfg {
  static constexpr uint32_t T = kPipeThreads / P;            // voxels per tile
  static constexpr uint32_t kRowBytes = T * sizeof(TIn);     // one channel's voxels of a tile
  static constexpr uint32_t kPitch = kRowBytes + 16;         // padded row pitch in a stage
  static constexpr uint32_t kChunksPerRow = kRowBytes / 16;
  static constexpr uint32_t E = 16 / sizeof(TOut);           // outputs per 16-byte store
  static_assert(kRowBytes % 16 == 0, "tile rows are whole 16-byte chunks");
  static size_t stage_bytes(uint32_t C) { return size_t(C) * kPitch; }
  static size_t smem_bytes(uint32_t C) {
    return kPipeStages * stage_bytes(C) + size_t(T) * (C + 4) * sizeof(float);
  }
};

template <typename T>
__device__ __forceinline__ uint4 pack16(const float* v);
template <>
__device__ __forceinline__ uint4 pack16<float>(const float* v) {
  return make_uint4(__float_as_uint(v[0]), __float_as_uint(v[1]), __float_as_uint(v[2]),
                    __float_as_uint(v[3]));
}
template <>
__device__ __forceinline__ uint4 pack16<__half>(const float* v) {
  return make_uint4(pack_pair<__half>(v[0], v[1]), pack_pair<__half>(v[2], v[3]),
                    pack_pair<__half>(v[4], v[5]), pack_pair<__half>(v[6], v[7]));
}
template <>
__device__ __forceinline__ uint4 pack16<__nv_bfloat16>(const float* v) {
  return make_uint4(pack_pair<__nv_bfloat16>(v[0], v[1]), pack_pair<__nv_bfloat16>(v[2], v[3]),
                    pack_pair<__nv_bfloat16>(v[4], v[5]), pack_pair<__nv_bfloat16>(v[6], v[7]));
}

// NV: channels per lane when it is the full kPipeVals (every C = 48 * 2^k), else 0
// (a runtime count g.nv, with predicated channel slots).
template <typename TIn, typename TOut, int P, int NV, bool AFFINE>
__global__ void __launch_bounds__(kPipeThreads)
    proj_out_norm_pipelined_kernel(TOut* __restrict__ out, const TIn* __restrict__ x,
                                   const float* __restrict__ gamma,
                                   const float* __restrict__ beta, ProjNormGeom g) {
  using Cfg = PipeCfg<TIn, TOut, P>;
  const uint32_t nv = NV > 0 ? uint32_t(NV) : g.nv;
  constexpr uint32_t T = Cfg::T;
  extern __shared__ __align__(16) uint8_t smem[];
  const uint32_t stage_bytes = g.C * Cfg::kPitch;
  float* tile = reinterpret_cast<float*>(smem + kPipeStages * stage_bytes);  // [T][C + 4]
  const uint32_t stride = g.C + 4;
  const uint32_t chunks = g.C * Cfg::kChunksPerRow;

  // cp.async group per tile (empty past the last tile, so the group count per
  // thread stays uniform): the tile's C rows of T voxels into stage `s`; chunks
  // past the volume's end are zero-filled and not read.
  auto issue = [&](uint32_t t, uint32_t s) {
    if (t < g.tiles) {
      uint32_t b, tb;
      g.f_tpb.divmod(t, b, tb);
      const uint32_t t0 = tb * T;
      const uint32_t valid = min(T, g.S - t0) * uint32_t(sizeof(TIn));
      const uint8_t* base =
          reinterpret_cast<const uint8_t*>(x) + (uint64_t(b) * g.C * g.S + t0) * sizeof(TIn);
      uint8_t* dst = smem + s * stage_bytes;
      for (uint32_t q = threadIdx.x; q < chunks; q += kPipeThreads) {
        const uint32_t c = q / Cfg::kChunksPerRow, off = (q % Cfg::kChunksPerRow) * 16;
        const bool in = off < valid;
        const uint8_t* src = base + uint64_t(c) * g.S * sizeof(TIn) + (in ? off : 0);
        cp_async16(dst + c * Cfg::kPitch + off, src, in ? 16u : 0u);
      }
    }
    cp_async_commit();
  };

  const uint32_t tok = threadIdx.x / P, part = threadIdx.x % P;
  const uint32_t c0 = part * nv;  // this lane's channels: c0 .. c0 + nv - 1
  uint32_t t = blockIdx.x;
#pragma unroll
  for (int s = 0; s < kPipeStages - 1; ++s) issue(t + s * gridDim.x, s);
  for (uint32_t i = 0; t < g.tiles; ++i, t += gridDim.x) {
    const uint32_t s = i % kPipeStages;
    cp_async_wait<kPipeStages - 2>();  // this thread's copies of tile i have landed
    __syncthreads();                   // everyone's have; iteration i-1 is finished
    issue(t + (kPipeStages - 1) * gridDim.x, (i + kPipeStages - 1) % kPipeStages);

    // LayerNorm of voxel `tok` over the lane's channels (+ the other P-1 lanes)
    const uint8_t* col = smem + s * stage_bytes + tok * sizeof(TIn) + c0 * Cfg::kPitch;
    float v[kPipeVals];
    float sum = 0.f;
#pragma unroll
    for (int j = 0; j < kPipeVals; ++j) {
      v[j] = uint32_t(j) < nv ? smem_to_float<TIn>(col + j * Cfg::kPitch) : 0.f;
      sum += v[j];
    }
    const float mean = lane_group_sum<P>(sum) * g.inv_c;
    float sq = 0.f;
#pragma unroll
    for (int j = 0; j < kPipeVals; ++j) {
      if (uint32_t(j) < nv) {
        const float d = v[j] - mean;
        sq = fmaf(d, d, sq);
      }
    }
    const float rstd = rsqrtf(lane_group_sum<P>(sq) * g.inv_c + g.eps);
    float* row = tile + tok * stride + c0;
#pragma unroll
    for (int j = 0; j < kPipeVals; j += 4) {
      if (uint32_t(j) < nv) {
        float y[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          y[e] = (v[j + e] - mean) * rstd;
          if constexpr (AFFINE)
            y[e] = fmaf(y[e], __ldg(gamma + c0 + j + e), __ldg(beta + c0 + j + e));
        }
        *reinterpret_cast<float4*>(row + j) = make_float4(y[0], y[1], y[2], y[3]);
      }
    }
    __syncthreads();

    // the tile's n x C outputs are one contiguous run of the channels-last result
    uint32_t b, tb;
    g.f_tpb.divmod(t, b, tb);
    const uint32_t t0 = tb * T;
    const uint32_t n = min(T, g.S - t0);
    uint4* dst = reinterpret_cast<uint4*>(out + (uint64_t(b) * g.S + t0) * g.C);
    const uint32_t vecs = n * g.C / Cfg::E;
    for (uint32_t q = threadIdx.x; q < vecs; q += kPipeThreads) {
      uint32_t vt, ce;
      g.f_CE.divmod(q, vt, ce);
      const float* r = tile + vt * stride + ce * Cfg::E;
      float y[Cfg::E];
#pragma unroll
      for (uint32_t e = 0; e < Cfg::E; e += 4) {
        const float4 f = *reinterpret_cast<const float4*>(r + e);
        y[e] = f.x;
        y[e + 1] = f.y;
        y[e + 2] = f.z;
        y[e + 3] = f.w;
      }
      stg(dst + q, pack16<TOut>(y));
    }
  }
  cp_async_wait<0>();
}

int pn_num_sms() {
  int dev = 0, sms = 0;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  return sms > 0 ? sms : 148;
}

template <typename TIn, typename TOut, int P, int NV, bool AFFINE>
cudaError_t launch_pipelined_k(void* out, const void* x, const float* gamma, const float* beta,
                               const ProjNormGeom& g, cudaStream_t stream) {
  auto kern = proj_out_norm_pipelined_kernel<TIn, TOut, P, NV, AFFINE>;
  const size_t smem = PipeCfg<TIn, TOut, P>::smem_bytes(g.C);
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       int(smem));
  if (e != cudaSuccess) return e;
  int per_sm = 0;
  e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, kPipeThreads, smem);
  if (e != cudaSuccess) return e;
  const uint64_t cap = uint64_t(pn_num_sms()) * uint64_t(per_sm > 0 ? per_sm : 1);
  const uint32_t blocks = uint32_t(g.tiles < cap ? g.tiles : cap);
  kern<<<blocks, kPipeThreads, smem, stream>>>(static_cast<TOut*>(out), static_cast<const TIn*>(x),
                                             gamma, beta, g);
  return cudaGetLastError();
}

template <typename TIn, typename TOut, int P>
cudaError_t launch_pipelined(void* out, const void* x, const float* gamma, const float* beta,
                             const ProjNormGeom& g, cudaStream_t stream) {
  if (g.nv == uint32_t(kPipeVals)) {
    if (g.affine) return launch_pipelined_k<TIn, TOut, P, kPipeVals, true>(out, x, gamma, beta, g, stream);
    return launch_pipelined_k<TIn, TOut, P, kPipeVals, false>(out, x, gamma, beta, g, stream);
  }
  if (g.affine) return launch_pipelined_k<TIn, TOut, P, 0, true>(out, x, gamma, beta, g, stream);
  return launch_pipelined_k<TIn, TOut, P, 0, false>(out, x, gamma, beta, g, stream);
}

template <typename TIn, typename TOut>
cudaError_t launch_pipelined_p(int P, void* out, const void* x, const float* gamma,
                               const float* beta, const ProjNormGeom& g, cudaStream_t stream) {
  switch (P) {
    case 1: return launch_pipelined<TIn, TOut, 1>(out, x, gamma, beta, g, stream);
    case 2: return launch_pipelined<TIn, TOut, 2>(out, x, gamma, beta, g, stream);
    case 4: return launch_pipelined<TIn, TOut, 4>(out, x, gamma, beta, g, stream);
    case 8: return launch_pipelined<TIn, TOut, 8>(out, x, gamma, beta, g, stream);
    default: return launch_pipelined<TIn, TOut, 16>(out, x, gamma, beta, g, stream);
  }
}

template <typename TIn, typename TOut>
cudaError_t launch_pn_t(bool pipelined, int P, void* out, const void* x, const float* gamma,
                        const float* beta, const ProjNormGeom& g, cudaStream_t stream) {
  if (pipelined) return launch_pipelined_p<TIn, TOut>(P, out, x, gamma, beta, g, stream);
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
cudaError_t launch_pn_out(int out_dtype, bool pipelined, int P, void* out, const void* x,
                          const float* gamma, const float* beta, const ProjNormGeom& g,
                          cudaStream_t stream) {
  if (out_dtype == kF32)
    return launch_pn_t<TIn, float>(pipelined, P, out, x, gamma, beta, g, stream);
  if (out_dtype == kF16)
    return launch_pn_t<TIn, __half>(pipelined, P, out, x, gamma, beta, g, stream);
  return launch_pn_t<TIn, __nv_bfloat16>(pipelined, P, out, x, gamma, beta, g, stream);
}

}  // namespace

// Lanes per voxel of the pipelined variant (48 channels per lane, each lane's
// range a whole number of 16-byte float4 groups), 0 if it does not apply.
int pipelined_lanes(int64_t C) {
  if (C <= 0 || C > kPnMaxC || C % 8 != 0) return 0;
  int P = 1;
  while (int64_t(P) * kPipeVals < C) P *= 2;
  return C % (4 * P) == 0 ? P : 0;
}

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
  const int64_t in_sz = dtype_size(in_dtype), out_sz = dtype_size(out_dtype);
  // cp.async variant when every tile's plane rows start on a 16-byte boundary
  const int P3 = pipelined_lanes(C);
  const bool pipelined = P3 > 0 && (S * in_sz) % 16 == 0;
  const int lanes = pipelined ? P3 : P;
  ProjNormGeom g{};
  g.C = uint32_t(C);
  g.S = uint32_t(S);
  g.nv = uint32_t(C / lanes);
  const uint32_t T = (pipelined ? kPipeThreads : kPnThreads) / lanes;
  const uint32_t tpb = uint32_t((S + T - 1) / T);
  g.f_tpb = DivMod32::make(tpb);
  g.f_C = DivMod32::make(g.C);
  g.f_CE = DivMod32::make(uint32_t(C / (16 / out_sz)));
  g.inv_c = 1.0f / float(C);
  g.eps = eps;
  g.affine = gamma != nullptr;
  // split the batch so the tile index (plus a grid's lookahead) stays below 2^31
  const int64_t bmax = ((int64_t(1) << 30) - 1) / tpb;
  for (int64_t b0 = 0; b0 < B; b0 += bmax) {
    const int64_t nb = B - b0 < bmax ? B - b0 : bmax;
    g.tiles = uint32_t(nb * tpb);
    const void* xs = static_cast<const uint8_t*>(x) + uint64_t(b0) * C * S * in_sz;
    void* os = static_cast<uint8_t*>(out) + uint64_t(b0) * C * S * out_sz;
    cudaError_t err;
    if (in_dtype == kF32)
      err = launch_pn_out<float>(out_dtype, pipelined, lanes, os, xs, gamma, beta, g, stream);
    else if (in_dtype == kF16)
      err = launch_pn_out<__half>(out_dtype, pipelined, lanes, os, xs, gamma, beta, g, stream);
    else
      err = launch_pn_out<__nv_bfloat16>(out_dtype, pipelined, lanes, os, xs, gamma, beta, g, stream);
    if (err != cudaSuccess) return set_cuda_error(err, "proj_out_norm launch");
  }
  return kOk;
}

}  // namespace crumpet
